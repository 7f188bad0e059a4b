"""Benchmark of the causal depthwise conv1d path (forward + backward) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|triton]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1)
    python bench.py --sweep     (every BASELINE config, ours vs the reference's Triton kernels)

Workload (the sweep the headline metric is quoted on, at its largest
sequence length): per GPU x bf16 (B=8, T=32768, D=1024) ~ N(0,1), weight fp32 (1024, 4) ~ N(0, 1/4),
bias fp32 ~ N(0, 0.1), activation SiLU, dout bf16 ~ N(0,1); seed 0, generated on the host and copied
to the device. One step = forward + backward (dx, dweight, dbias). With N GPUs each rank runs its own
batch shard of 8 rows (weak scaling) and the fp32 dweight||dbias vector is all-reduced over NCCL
every step. Every tensor (537 MB) is larger than the 126 MB L2, so no flush is needed between steps.

`value` is the aggregate algorithmic HBM throughput (GB/s, bytes as below) over all GPUs with inputs
resident in HBM, from CUDA events around exactly K steps, max over ranks. `e2e` is the same metric
measured through the public API (`causal_conv1d_fn` + autograd) with the step's inputs copied from
pinned host memory and its results (out, dx, dweight, dbias) copied back inside the timed region.

Algorithmic bytes per call (bf16 x/out/dout/dx = 2 B, fp32 weight/bias):
  forward  = B*T*D*(2 + 2) + D*W*4 + D*4
  backward = B*T*D*(2 + 2 + 2) + 2*(D*W*4 + D*4)

--impl reference times the reference algorithm on the host CPU: the oracle (oracle/, a C
restatement of the reference's per-element algorithm; the reference itself is Python/Triton and has
no CPU implementation), with all host threads; each step is one whole batch row (T x D) forward +
backward, the same sample the `cpu_baseline` leg of the default arm times.
--impl triton times the reference's own Triton kernels (baseline/_ref) on the same B200; at N=1 the
default arm runs it in a subprocess on the same workload and embeds it as `triton_reference`.

At every N the default arm also runs BASELINE config 5 strong-scaled (`cfg5_sharded`: B=64 T=8192
D=8192 W=8 bias+SiLU split over the N ranks, NCCL all-reduce of dweight||dbias included) and checks
the sharded weight/bias gradient against the single-GPU full-batch gradient computed on rank 0.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "causal-conv1d-triton_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "fwd/bwd HBM GB/s (% of ~8 TB/s) and µs/call, bf16 D=1024 W=4"
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0

# Per-launch DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of the backward kernel at
# this workload (B=8, T=32768, D=1024, W=4, bias+SiLU), read from an ncu launch list of this
# command on a B200; it scales with the B*T rows processed. Re-captured after each change of the
# backward kernel.
BWD_DRAM_BYTES_PER_LAUNCH = 1089.6e6 + 509.0e6
BWD_DRAM_ROWS = 8 * 32768


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "triton"])
    ap.add_argument("--batch", type=int, default=8, help="batch rows per GPU")
    ap.add_argument("--seqlen", type=int, default=32768)
    ap.add_argument("--dim", type=int, default=1024)
    ap.add_argument("--width", type=int, default=4)
    ap.add_argument("--no-bias-silu", action="store_true", help="the no-bias/no-activation mode")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="CPU baseline budget (0 skips the CPU baselines)")
    ap.add_argument("--cfg5-steps", type=int, default=10,
                    help="timed steps of the strong-scaled config-5 sub-record (0 skips it)")
    ap.add_argument("--no-triton-arm", action="store_true",
                    help="skip the embedded reference-Triton run at N=1")
    ap.add_argument("--sweep", action="store_true",
                    help="time every BASELINE config through both implementations' public APIs "
                         "(ours and the reference's Triton kernels) and print one JSON line each")
    ap.add_argument("--fusion", action="store_true",
                    help="time split_conv1d (the conv fused with a Mamba-2 block's splits) against "
                         "torch.split around causal_conv1d_fn, forward + backward, at cfg4's shape")
    ap.add_argument("--decode", action="store_true",
                    help="time the decode-time companions (causal_conv1d_update, "
                         "seq_idx_from_cu_seqlens) and print one JSON line each")
    return ap.parse_args()


def algo_bytes(B, T, D, W, es=2):
    fwd = B * T * D * (es + es) + D * W * 4 + D * 4
    bwd = B * T * D * (3 * es) + 2 * (D * W * 4 + D * 4)
    return fwd, bwd


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def make_inputs(B, T, D, W, bias_silu, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, D, generator=g).to(torch.bfloat16)
    w = torch.randn(D, W, generator=g) * 0.5
    b = torch.randn(D, generator=g) * (0.1**0.5) if bias_silu else None
    dy = torch.randn(B, T, D, generator=g).to(torch.bfloat16)
    return x, w, b, dy


class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons every 100 ms in the background."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.rows = []
        self.proc = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.time(), line.strip()))

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def stop(self):
        if self.proc is None:
            return {"unavailable": "nvidia-smi not runnable"}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sel = [r for t, r in self.rows if self.t0 - 0.15 <= t <= self.t1 + 0.15] or [r for _, r in self.rows]
        sms, maxs, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in sel:
            f = [c.strip() for c in r.split(",")]
            if len(f) < 10:
                continue
            try:
                sms.append(float(f[2]))
                maxs.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[6:10]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sms:
            return {"unavailable": "no samples"}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxs), "samples": len(sms),
                "reasons": sorted(reasons)}


def same_size_copy_gbs(x, stream, reps=20):
    """Read+write throughput of torch's device copy of a tensor the size of x: the copy rate this
    workload's tensors can reach, a tighter ceiling than the 2 GiB copy of MEASURED_PEAKS.json."""
    out = torch.empty_like(x)
    for _ in range(3):
        out.copy_(x)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(reps):
        out.copy_(x)
    e.record(stream)
    torch.cuda.synchronize()
    return 2 * x.numel() * x.element_size() * reps / (s.elapsed_time(e) * 1e-3) / 1e9


class CpuSample:
    """The CPU sample both CPU timings use: batch row 0 of the workload (all T rows, all D
    channels), forward + backward through the oracle, fp32 copies prepared once."""

    def __init__(self, x, w, b, dy, silu, nthreads):
        from oracle import oracle

        self.oracle = oracle
        self.xs, self.dys = x[:1].float().numpy(), dy[:1].float().numpy()
        self.w, self.b, self.silu, self.nthreads = w, b, silu, nthreads
        _, self.T, self.D = self.xs.shape
        self.W = w.shape[1]
        fb, bb = algo_bytes(1, self.T, self.D, self.W)
        self.bytes = fb + bb
        self.desc = f"batch row 0 (T={self.T}, D={self.D}, W={self.W}), fwd+bwd per rep"

    def step(self):
        o = self.oracle
        o.fwd(self.xs, self.w, self.b, None, None, silu=self.silu, nthreads=self.nthreads)
        o.bwd(self.xs, self.w, self.b, None, None, self.dys, None, False, silu=self.silu,
              nthreads=self.nthreads)


def cpu_sample_gbs(w, b, x, dy, silu, seconds, nthreads=0):
    """Times the oracle (fwd + bwd) on the CPU sample until `seconds` have passed (after one
    untimed rep); returns (GB/s of algorithmic bytes, sample description, reps)."""
    cs = CpuSample(x, w, b, dy, silu, nthreads)
    cs.step()
    reps, t0 = 0, time.perf_counter()
    while True:
        cs.step()
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return cs.bytes * reps / el / 1e9, f"{cs.desc}: x{reps} in {el:.1f} s", reps


def torch_conv1d_cpu_gbs(w, b, x, dy, silu, seconds):
    """The reference semantics as PyTorch F.conv1d(groups=D) with left padding on the host cores
    (forward + autograd backward, bf16 as the workload), on batch row 0: the CPU baseline the
    task names beside the port. Returns (GB/s of algorithmic bytes, threads, sample)."""
    import torch.nn.functional as F

    T, D = x.shape[1], x.shape[2]
    W = w.shape[1]
    xl = x[:1].clone().requires_grad_(True)
    wl = w.to(torch.bfloat16).clone().requires_grad_(True)
    bl = b.to(torch.bfloat16).clone().requires_grad_(True) if b is not None else None
    dyl = dy[:1]

    def step():
        y = F.conv1d(F.pad(xl.transpose(1, 2), (W - 1, 0)), wl[:, None, :], bl, groups=D)
        if silu:
            y = F.silu(y)
        y.transpose(1, 2).backward(dyl)
        xl.grad = wl.grad = None
        if bl is not None:
            bl.grad = None

    step()
    reps, t0 = 0, time.perf_counter()
    while True:
        step()
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    fb, bb = algo_bytes(1, T, D, W)
    sample = (f"batch row 0 (T={T}, D={D}, W={W}), bf16 F.conv1d(F.pad(x.transpose(1, 2), (W-1, 0)), "
              f"weight[:, None], bias, groups=D){' + SiLU' if silu else ''} + autograd backward: "
              f"x{reps} in {el:.1f} s")
    return (fb + bb) * reps / el / 1e9, torch.get_num_threads(), sample


def run_reference_cpu(args):
    """--impl reference: the reference algorithm on the host cores (the oracle port), each step
    the same CPU sample the default arm's cpu_baseline times (one whole batch row)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    B, T, D, W = args.batch, args.seqlen, args.dim, args.width
    bias_silu = not args.no_bias_silu
    x, w, b, dy = make_inputs(B, T, D, W, bias_silu)
    threads = os.cpu_count()
    cs = CpuSample(x, w, b, dy, bias_silu, threads)
    for _ in range(args.warmup):
        cs.step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cs.step()
    el = time.perf_counter() - t0
    gbs = cs.bytes * args.steps / el / 1e9
    print(json.dumps({
        "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "impl": "reference",
        "data": "synthetic, seed 0",
        "config": workload_config(args),
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"per step: {cs.desc}"},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def workload_config(args):
    n = args.gpus
    if args.dim == 1024 and args.width == 4 and args.batch == 8:
        name = "BASELINE config 2 (sweep)"
    elif args.dim == 8192 and args.width == 8:
        name = "BASELINE config 5 shape"
    else:
        name = "custom shape"
    l2 = ("no flush: every tensor is larger than L2 (126 MB)" if args.batch * args.seqlen * args.dim * 2 > 126e6
          else "tensors smaller than L2, no flush: not a headline configuration")
    return {
        "workload": f"{name}, B={args.batch}/GPU T={args.seqlen} D={args.dim} "
                    f"W={args.width} {'none' if args.no_bias_silu else 'bias+silu'}, fwd+bwd step",
        "global_batch": args.batch * n, "seq_len": args.seqlen, "dim": args.dim,
        "width": args.width,
        "parallelism": f"dp{n}: batch shards, NCCL all-reduce of fp32 dweight||dbias" if n > 1 else "single GPU",
        "l2": l2,
    }


def run_triton_reference(args, dev):
    """--impl triton: the reference's Triton kernels (baseline/_ref) on this GPU."""
    sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
    import causal_conv1d_triton.causal_conv1d as ref

    return ref._fwd, ref._bwd


# ---------------------------------------------------------------------------------------------
# --sweep: every BASELINE.json config through the public API of both implementations.
# ---------------------------------------------------------------------------------------------
def _sweep_cases():
    """(name, builder) for each BASELINE config; a builder returns the call's tensors on the host."""
    def dense(B, T, D, W, wstd, bstd, silu, seed=0):
        def build():
            g = torch.Generator().manual_seed(seed)
            x = torch.randn(B, T, D, generator=g).to(torch.bfloat16)
            w = torch.randn(D, W, generator=g) * wstd
            b = torch.randn(D, generator=g) * bstd if bstd else None
            dy = torch.randn(B, T, D, generator=g).to(torch.bfloat16)
            return dict(x=x, w=w, b=b, dy=dy, silu=silu)
        return build

    def varlen():
        g = torch.Generator().manual_seed(4)
        B, T, D, W = 4, 16384, 4352, 4
        x = torch.randn(B, T, D, generator=g).to(torch.bfloat16)
        w = torch.randn(D, W, generator=g) * 0.5
        b = torch.randn(D, generator=g) * 0.1 ** 0.5
        seq = torch.empty(B, T, dtype=torch.int32)
        for r in range(B):
            pad = int(torch.randint(0, 256, (1,), generator=g))
            t, sid = 0, 0
            while t < T - pad:
                n = int(torch.randint(64, 4097, (1,), generator=g))
                seq[r, t:min(t + n, T - pad)] = sid
                t, sid = t + n, sid + 1
            seq[r, T - pad:] = -1
        init = torch.randn(B, W - 1, D, generator=g).to(torch.bfloat16)
        dy = torch.randn(B, T, D, generator=g).to(torch.bfloat16)
        return dict(x=x, w=w, b=b, dy=dy, silu=True, seq=seq, init=init)

    def chain():
        d = dense(16, 8192, 2048, 4, 0.5, 0.1 ** 0.5, True, seed=3)()
        g = torch.Generator().manual_seed(33)
        d["init"] = torch.randn(16, 3, 2048, generator=g).to(torch.bfloat16)
        # Each chunk is its own leaf (a streaming caller gets the chunks one at a time); slicing one
        # leaf would time torch's slice-backward (a full-size zero tensor per chunk), not the conv.
        L = 8192 // 4
        d["xs"] = [d["x"][:, i * L:(i + 1) * L].contiguous() for i in range(4)]
        d["dys"] = [d["dy"][:, i * L:(i + 1) * L].contiguous() for i in range(4)]
        return d

    cases = [("cfg1 B=2 T=1024 D=512 W=4 bias+silu", dense(2, 1024, 512, 4, 1.0, 1.0, True))]
    for T in (512, 2048, 8192, 32768):
        cases.append((f"cfg2 B=8 T={T} D=1024 W=4 none", dense(8, T, 1024, 4, 0.5, 0, False)))
        cases.append((f"cfg2 B=8 T={T} D=1024 W=4 bias+silu", dense(8, T, 1024, 4, 0.5, 0.1 ** 0.5, True)))
    cases.append(("cfg3 B=16 T=8192 D=2048 W=4 bias+silu, 4 chained chunks", chain))
    cases.append(("cfg4 B=4 T=16384 D=4352 W=4 varlen seq_idx+init bias+silu", varlen))
    cases.append(("cfg5 B=64 T=8192 D=8192 W=8 bias+silu, 1 GPU", dense(64, 8192, 8192, 8, 8 ** -0.5, 0.1 ** 0.5, True)))
    return cases


def _sweep_step(fn, t, grad):
    """One call of the workload through `fn` (a causal_conv1d_fn): forward, and backward if grad."""
    act = "silu" if t["silu"] else None
    if "xs" in t:
        state, outs = t["init"], []
        for xc in t["xs"]:
            o, state = fn(xc, t["w"], t["b"], initial_states=state, return_final_states=True,
                          activation=act)
            outs.append(o)
        if grad:
            torch.autograd.backward(outs, t["dys"])
        return outs
    out = fn(t["x"], t["w"], t["b"], seq_idx=t.get("seq"), initial_states=t.get("init"), activation=act)
    if grad:
        out.backward(t["dy"])
    return out


def run_sweep(args):
    import statistics as st

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    from causal_conv1d_b200 import causal_conv1d_fn as ours

    sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
    try:
        from causal_conv1d_triton import causal_conv1d_fn as ref
    except Exception as e:  # the reference install is optional for the sweep
        ref, ref_err = None, str(e)
    peak, _ = measured_peak()
    for name, build in _sweep_cases():
        h = build()
        t = {k: (v.to(dev) if torch.is_tensor(v) else [u.to(dev) for u in v] if isinstance(v, list) else v)
             for k, v in h.items()}
        for k in ("x", "w", "b", "init"):
            if t.get(k) is not None:
                t[k].requires_grad_(True)
        for xc in t.get("xs", []):
            xc.requires_grad_(True)
        B, T, D = h["x"].shape
        W = h["w"].shape[1]
        fb, bb = algo_bytes(B, T, D, W)
        impls = [("ours", ours)] + ([("reference-triton", ref)] if ref is not None else [])
        res = {n: {"fwd": [], "fwdbwd": []} for n, _ in impls}
        outs = {}
        for n, fn in impls:  # warm-up and results for the agreement check
            with torch.no_grad():
                outs[n] = _sweep_step(fn, t, False)
            _sweep_step(fn, t, True)
        torch.cuda.synchronize()
        reps = max(2, min(50, int(4e9 / (fb + bb))))
        for _ in range(5):
            for n, fn in impls:
                e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
                e[0].record()
                with torch.no_grad():
                    for _ in range(reps):
                        _sweep_step(fn, t, False)
                e[1].record()
                for _ in range(reps):
                    for v in [t.get(k) for k in ("x", "w", "b", "init")] + t.get("xs", []):
                        if v is not None:
                            v.grad = None
                    _sweep_step(fn, t, True)
                e[2].record()
                torch.cuda.synchronize()
                res[n]["fwd"].append(e[0].elapsed_time(e[1]) / reps * 1e3)
                res[n]["fwdbwd"].append(e[1].elapsed_time(e[2]) / reps * 1e3)
        agree = None
        if ref is not None:
            a = torch.cat([o.flatten() for o in (outs["ours"] if isinstance(outs["ours"], list) else [outs["ours"]])]).float()
            r = torch.cat([o.flatten() for o in (outs["reference-triton"] if isinstance(outs["reference-triton"], list) else [outs["reference-triton"]])]).float()
            agree = bool(((a - r).abs() <= 1e-2 + 1e-2 * r.abs()).all().item())
        line = {"sweep": name, "reps": reps, "outputs_agree_within_bf16_tol": agree}
        for n in res:
            f, fbw = st.median(res[n]["fwd"]), st.median(res[n]["fwdbwd"])
            line[n] = {"fwd_us": f, "fwd_bwd_us": fbw, "fwd_gbs": fb / f / 1e3,
                       "fwd_bwd_gbs": (fb + bb) / fbw / 1e3,
                       "fwd_frac_of_measured": fb / f / 1e3 / peak,
                       "fwd_bwd_frac_of_measured": (fb + bb) / fbw / 1e3 / peak}
        if ref is not None:
            line["speedup_fwd"] = line["reference-triton"]["fwd_us"] / line["ours"]["fwd_us"]
            line["speedup_fwd_bwd"] = line["reference-triton"]["fwd_bwd_us"] / line["ours"]["fwd_bwd_us"]
        else:
            line["reference-triton"] = {"unavailable": ref_err}
        print(json.dumps(line), flush=True)
        del t, h, outs
        torch.cuda.empty_cache()


def _graph_us_per_call(fn, calls=100, reps=5):
    """Device time per call of `fn` (no host sync inside), from replays of a CUDA graph holding
    `calls` calls, so host launch overhead does not hide the kernel time; plus the eager host time
    per call (launch-bound when the kernel is short)."""
    import statistics as st

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(calls):
            fn()
    g.replay()
    torch.cuda.synchronize()
    dev_us = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        dev_us.append(e0.elapsed_time(e1) * 1e3 / calls)
    # Eager host time: warm-up calls first (the first eager allocation after a capture can go to
    # cudaMalloc), then the median of `reps` timed loops.
    for _ in range(10):
        fn()
    torch.cuda.synchronize()
    host = []
    for _ in range(reps):
        t0 = time.perf_counter()
        for _ in range(calls):
            fn()
        torch.cuda.synchronize()
        host.append((time.perf_counter() - t0) * 1e6 / calls)
    del g
    return st.median(dev_us), st.median(host)


def run_decode(args):
    """Decode-time companions of the conv: the state update and the cu_seqlens front end.

    causal_conv1d_update: one new row per sequence through the conv, the (slots, W-1, D) state read
    and rewritten in place through a slot index, bias + SiLU, bf16 data and state, fp32 weights.
    Algorithmic bytes per call: x and out rows (2 B each), the W-1 state rows read and written,
    weight, bias and indices. seq_idx_from_cu_seqlens: cfg4's packed rows (B=4, T=16384, lengths
    U[64, 4096]); bytes = the int32 seq_idx written + cu_seqlens read."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    from causal_conv1d_b200 import causal_conv1d_update, seq_idx_from_cu_seqlens

    peak, kind = measured_peak()
    g = torch.Generator().manual_seed(0)
    for name, B, D, W, slots in [("decode Mamba-2 conv dim (cfg4 D=4352, W=4), 256 sequences", 256, 4352, 4, 512),
                                 ("decode cfg5 D=8192 W=8, 64 sequences", 64, 8192, 8, 128),
                                 ("decode cfg2 D=1024 W=4, 8 sequences", 8, 1024, 4, 8)]:
        x = torch.randn(B, D, generator=g).to(torch.bfloat16).to(dev)
        state = torch.randn(slots, W - 1, D, generator=g).to(torch.bfloat16).to(dev)
        idx = torch.randperm(slots, generator=g)[:B].to(torch.int32).to(dev)
        w = (torch.randn(D, W, generator=g) * W ** -0.5).to(dev)
        b = (torch.randn(D, generator=g) * 0.1 ** 0.5).to(dev)
        dev_us, host_us = _graph_us_per_call(
            lambda: causal_conv1d_update(x, state, w, b, activation="silu", conv_state_indices=idx))
        nbytes = B * D * 2 * 2 + 2 * B * (W - 1) * D * 2 + D * W * 4 + D * 4 + B * 4
        gbs = nbytes / (dev_us * 1e-6) / 1e9
        print(json.dumps({"decode": name, "kernel": "cc1d_update_kernel", "batch": B, "dim": D, "width": W,
                          "us_per_call": dev_us, "host_us_per_eager_call": host_us,
                          "bytes_per_call": nbytes, "gbs": gbs, "frac_of_measured": gbs / peak,
                          "peak": f"{kind} hbm_gbs {peak}", "timing": "CUDA graph of 100 calls, median of 5 replays"}),
              flush=True)

    B, T = 4, 16384
    rows = []
    for _ in range(B):
        lens, tot = [], 0
        while True:
            n = int(torch.randint(64, 4097, (1,), generator=g))
            if tot + n > T - int(torch.randint(0, 256, (1,), generator=g)):
                break
            lens.append(n)
            tot += n
        rows.append(lens)
    n = max(len(r) for r in rows)
    cu = torch.zeros(B, n + 1, dtype=torch.int32)
    for i, r in enumerate(rows):  # rows with fewer sequences repeat their last boundary (empty seqs)
        c = torch.tensor([0] + r).cumsum(0)
        cu[i, :len(c)] = c
        cu[i, len(c):] = c[-1]
    cu = cu.to(dev)
    dev_us, host_us = _graph_us_per_call(lambda: seq_idx_from_cu_seqlens(cu, T))
    nbytes = B * T * 4 + cu.numel() * 4
    gbs = nbytes / (dev_us * 1e-6) / 1e9
    print(json.dumps({"decode": "seq_idx_from_cu_seqlens, cfg4 rows (B=4, T=16384)", "kernel": "cc1d_seq_idx_kernel",
                      "n_seqs_per_row": n, "us_per_call": dev_us, "host_us_per_eager_call": host_us,
                      "bytes_per_call": nbytes, "gbs": gbs, "frac_of_measured": gbs / peak,
                      "timing": "CUDA graph of 100 calls, median of 5 replays"}), flush=True)


def run_fusion(args):
    """split_conv1d against the unfused Mamba-2 composition at BASELINE config 4's shape.

    zxbcdt (B=4, T=16384, 4096 + 4352 + 64 channels) bf16: z (d_inner 4096), xBC (x 4096, B 128,
    C 128: cfg4's D=4352 conv dim) and dt (64 heads). Bias + SiLU, cfg4's packed seq_idx and
    initial states. One step = forward and backward through autograd with fixed upstream gradients
    for z, x, B, C and dt (separate tensors, as the SSM produces them). The unfused step
    concatenates the x/B/C gradients into dout and then dz, dxBC and ddt into d(zxbcdt); the fused
    step does neither (bytes avoided: 4 x B*T*D_xbc*2)."""
    import statistics as st

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    from causal_conv1d_b200 import causal_conv1d_fn, split_conv1d

    B, T, d_z, split, d_dt, W = 4, 16384, 4096, (4096, 128, 128), 64, 4
    d_xbc = sum(split)
    g = torch.Generator().manual_seed(0)
    zx = torch.randn(B, T, d_z + d_xbc + d_dt, generator=g).to(torch.bfloat16).to(dev).requires_grad_(True)
    w = (torch.randn(d_xbc, W, generator=g) * 0.5).to(dev).requires_grad_(True)
    b = (torch.randn(d_xbc, generator=g) * 0.1 ** 0.5).to(dev).requires_grad_(True)
    init = torch.randn(B, W - 1, d_xbc, generator=g).to(torch.bfloat16).to(dev).requires_grad_(True)
    seq = torch.empty(B, T, dtype=torch.int32)
    for r in range(B):
        t, i = 0, 0
        pad = int(torch.randint(0, 256, (1,), generator=g))
        while t < T - pad:
            n = min(int(torch.randint(64, 4097, (1,), generator=g)), T - pad - t)
            seq[r, t:t + n] = i
            t, i = t + n, i + 1
        seq[r, T - pad:] = -1
    seq = seq.to(dev)
    widths = [d_z, *split, d_dt]
    ups = [torch.randn(B, T, c, generator=g).to(torch.bfloat16).to(dev) for c in widths]

    def fused():
        outs = split_conv1d(zx, w, b, d_z=d_z, xbc_split=split, seq_idx=seq, initial_states=init,
                            activation="silu")
        torch.autograd.backward(outs, ups)

    def unfused():
        z, xbc, dtp = zx.split([d_z, d_xbc, d_dt], dim=-1)
        y = causal_conv1d_fn(xbc, w, b, seq_idx=seq, initial_states=init, activation="silu")
        torch.autograd.backward((z, *y.split(list(split), dim=-1), dtp), ups)

    res = {"fused": [], "unfused": []}
    for _ in range(3):
        fused(), unfused()
    for _ in range(7):
        for name, fn in (("fused", fused), ("unfused", unfused)):
            for t in (zx, w, b, init):
                t.grad = None
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(5):
                fn()
            e1.record()
            torch.cuda.synchronize()
            res[name].append(e0.elapsed_time(e1) / 5 * 1e3)
    f, u = st.median(res["fused"]), st.median(res["unfused"])
    print(json.dumps({"fusion": "split_conv1d vs torch.split + causal_conv1d_fn + split, fwd + bwd",
                      "shape": {"batch": B, "seqlen": T, "d_z": d_z, "xbc_split": list(split), "d_dt": d_dt,
                                "width": W, "seq_idx": "cfg4 packed", "initial_states": True},
                      "fused_us": f, "unfused_us": u, "speedup": u / f,
                      "bytes_avoided_per_step": 4 * B * T * d_xbc * 2,
                      "timing": "CUDA events, 5 steps per sample, median of 7 interleaved samples"}),
          flush=True)


def main():
    args = parse()
    if args.sweep:
        run_sweep(args)
        return
    if args.fusion:
        run_fusion(args)
        return
    if args.decode:
        run_decode(args)
        return
    if args.impl == "reference":
        run_reference_cpu(args)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    B, T, D, W = args.batch, args.seqlen, args.dim, args.width
    bias_silu = not args.no_bias_silu
    x_h, w_h, b_h, dy_h = make_inputs(B, T, D, W, bias_silu, seed=rank)
    x, w = x_h.to(dev), w_h.to(dev)
    b = b_h.to(dev) if b_h is not None else None
    dy = dy_h.to(dev)
    fbytes, bbytes = algo_bytes(B, T, D, W)

    if args.impl == "triton":
        fwd_fn, bwd_fn = run_triton_reference(args, dev)

        def fwd():
            return fwd_fn(x, w, b, None, None, None, bias_silu)

        def bwd():
            return bwd_fn(x, w, b, None, None, dy, None, False, bias_silu)
        grad_buf = None
    else:
        from causal_conv1d_b200.causal_conv1d import _bwd, _fwd

        # Two fp32 dweight||dbias buffers: step i's all-reduce runs on NCCL's stream while step
        # i+1's forward runs; step i+2's backward, which rewrites the buffer, waits for it first.
        grad_buf = [torch.zeros(D * (W + 1), device=dev, dtype=torch.float32) for _ in range(2)] if world > 1 else None
        pending = [None, None]
        n_bwd = [0]

        def fwd():
            return _fwd(x, w, b, None, None, None, bias_silu)

        def bwd():
            if world == 1:
                return _bwd(x, w, b, None, None, dy, None, False, bias_silu)
            k = n_bwd[0] % 2
            n_bwd[0] += 1
            if pending[k] is not None:
                pending[k].wait()  # the compute stream waits for the all-reduce that last read buf k
            r = _bwd(x, w, b, None, None, dy, None, False, bias_silu, grad_f32=grad_buf[k])
            pending[k] = dist.all_reduce(grad_buf[k], async_op=True)
            return r

    stream = torch.cuda.current_stream(dev)
    def join():
        if args.impl != "triton" and world > 1:
            for k in range(2):
                if pending[k] is not None:
                    pending[k].wait()
                    pending[k] = None

    for _ in range(args.warmup):
        fwd()
        bwd()
    join()
    torch.cuda.synchronize(dev)

    n_ev = args.steps
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(n_ev)]
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler.mark_start()
    start.record(stream)
    for i in range(args.steps):
        ev[i][0].record(stream)
        fwd()
        ev[i][1].record(stream)
        bwd()
        ev[i][2].record(stream)
    join()
    end.record(stream)
    torch.cuda.synchronize(dev)
    sampler.mark_end()
    if dist is not None:
        dist.barrier()
    clocks = sampler.stop()
    total_ms = start.elapsed_time(end)
    fwd_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / n_ev
    bwd_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / n_ev
    if dist is not None:
        t = torch.tensor([total_ms, fwd_ms, bwd_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, fwd_ms, bwd_ms = t.tolist()

    copy_gbs = same_size_copy_gbs(x, stream)
    ms_step = total_ms / args.steps
    value = (fbytes + bbytes) * world / (ms_step * 1e-3) / 1e9
    peak, peak_kind = measured_peak()
    fwd_gbs = fbytes / (fwd_ms * 1e-3) / 1e9
    bwd_gbs = bbytes / (bwd_ms * 1e-3) / 1e9

    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: x, dout ~ N(0,1) bf16; weight ~ N(0,1/4), bias ~ N(0,0.1) fp32; seed = rank",
        "config": workload_config(args),
        "fwd": {"us_per_call": fwd_ms * 1e3, "gbs": fwd_gbs, "frac_of_8tbs": fwd_gbs / NOMINAL_HBM_GBS,
                "frac_of_measured": fwd_gbs / peak},
        "bwd": {"us_per_call": bwd_ms * 1e3, "gbs": bwd_gbs, "frac_of_8tbs": bwd_gbs / NOMINAL_HBM_GBS,
                "frac_of_measured": bwd_gbs / peak,
                "note": "backward kernel + fixed-order partial reduce" + (" + NCCL all-reduce" if world > 1 else "")},
        "clocks": clocks,
    }
    if args.impl == "triton":
        line["impl"] = "reference-triton"
        line["gpu_launches"] = 0
        if rank == 0:
            print(json.dumps(line), flush=True)
        if dist is not None:
            dist.destroy_process_group()
        return

    line["impl"] = "ours"
    line["gpu_launches"] = 3 * args.steps
    line["roofline"] = {
        "bound": "hbm", "kernel": "cc1d_bwd_walk_kernel (+ reduce)", "achieved": bwd_gbs,
        "peak": peak, "unit": "GB/s", "frac": bwd_gbs / peak, "peak_source": f"{peak_kind} hbm_gbs",
        "traffic": BWD_DRAM_BYTES_PER_LAUNCH * (B * T) / BWD_DRAM_ROWS,
        "algorithmic_bytes": bbytes,
        "copy_same_size_gbs": copy_gbs,
        "frac_of_copy_same_size": bwd_gbs / copy_gbs,
    }

    if world > 1:
        line["allreduce_us"] = allreduce_us(dist, grad_buf[0].clone(), stream)
    else:
        line["host_overhead_cfg1"] = host_overhead(dev)

    # End to end through the public API, host buffers in and out.
    line["e2e"] = e2e(args, dev, x_h, w_h, b_h, dy_h, bias_silu, world, dist)

    if args.cfg5_steps > 0:
        del x, dy
        torch.cuda.empty_cache()
        line["cfg5_sharded"] = cfg5_sharded(args, dev, world, rank, dist)

    if rank == 0:
        if world == 1 and args.cpu_seconds > 0:  # the CPU baselines are measured at N = 1 only
            threads = os.cpu_count()
            gbs, sample, _ = cpu_sample_gbs(w_h, b_h, x_h, dy_h, bias_silu, args.cpu_seconds,
                                            nthreads=threads)
            line["cpu_baseline"] = {"value": gbs, "unit": "GB/s", "cores": threads,
                                    "kind": "port", "sample": sample}
            tg, tthreads, tsample = torch_conv1d_cpu_gbs(w_h, b_h, x_h, dy_h, bias_silu,
                                                         args.cpu_seconds / 2)
            line["cpu_baseline_torch_conv1d"] = {"value": tg, "unit": "GB/s", "cores": os.cpu_count(),
                                                 "threads": tthreads, "sample": tsample}
        if world == 1 and not args.no_triton_arm:
            line["triton_reference"] = triton_arm(args, line)
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def allreduce_us(dist, buf, stream, reps=50):
    """Device time of one blocking NCCL all-reduce (sum) of `buf` on its own, max over ranks."""
    for _ in range(5):
        dist.all_reduce(buf)
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(reps):
        dist.all_reduce(buf)
    e.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([s.elapsed_time(e) / reps * 1e3], device=buf.device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def cfg5_sharded(args, dev, world, rank, dist):
    """BASELINE config 5 strong-scaled over the ranks: B=64 T=8192 D=8192 W=8 bf16, bias + SiLU,
    rows 64/N per GPU (shard_rows), forward + backward per step with the fp32 dweight||dbias vector
    all-reduced over NCCL (asynchronously, double-buffered as in the headline loop). Batch row r's
    x and dout come from generators seeded by r, so every N sees the same global batch.

    After the timed steps rank 0 runs the whole batch on its one GPU and compares: the all-reduced
    weight/bias gradient against the single-GPU one (within the bf16 sum tolerance,
    1e-2 * max(1, max|g|)), and its own shard's out and dx against the same rows of the
    single-GPU run (bit for bit: a row's results do not depend on the other rows)."""
    from causal_conv1d_b200.causal_conv1d import _bwd, _fwd
    from causal_conv1d_b200.distributed import shard_rows

    B, T, D, W = 64, 8192, 8192, 8
    rows = shard_rows(B, rank, world)
    nb = rows.stop - rows.start
    g = torch.Generator(device=dev)

    def rows_of(r0, r1, seed):
        t = torch.empty(r1 - r0, T, D, dtype=torch.bfloat16, device=dev)
        for r in range(r0, r1):
            g.manual_seed(seed + r)
            t[r - r0].normal_(generator=g)
        return t

    g.manual_seed(5)
    w = torch.randn(D, W, generator=g, device=dev) * W ** -0.5
    b = torch.randn(D, generator=g, device=dev) * 0.1 ** 0.5
    x = rows_of(rows.start, rows.stop, 1 << 20)
    dy = rows_of(rows.start, rows.stop, 2 << 20)
    flat = [torch.zeros(D * (W + 1), device=dev) for _ in range(2)]
    pending = [None, None]
    stream = torch.cuda.current_stream(dev)
    last = {}

    def step(i, ev_mid=None):
        last["out"] = _fwd(x, w, b, None, None, None, True)
        if ev_mid is not None:
            ev_mid.record(stream)
        k = i % 2
        if pending[k] is not None:
            pending[k].wait()
            pending[k] = None
        last["dx"] = _bwd(x, w, b, None, None, dy, None, False, True, grad_f32=flat[k])[0]
        last["k"] = k
        if world > 1:
            pending[k] = dist.all_reduce(flat[k], async_op=True)

    def join():
        for k in range(2):
            if pending[k] is not None:
                pending[k].wait()
                pending[k] = None

    warm, K = 3, args.cfg5_steps
    for i in range(warm):
        step(i)
    join()
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K)]
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for i in range(K):
        ev[i][0].record(stream)
        last["out"] = None  # the previous step's output is released before the next is made
        step(warm + i, ev[i][1])
        ev[i][2].record(stream)
    join()
    e.record(stream)
    torch.cuda.synchronize(dev)
    total = s.elapsed_time(e)
    t = torch.tensor([total], device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = t.item() / K
    ft = torch.tensor([sum(a[0].elapsed_time(a[1]) for a in ev) / K * 1e3,
                       sum(a[1].elapsed_time(a[2]) for a in ev) / K * 1e3], device=dev)
    if dist is not None:
        dist.all_reduce(ft, op=dist.ReduceOp.MAX)
    fwd_us, bwd_us = ft.tolist()
    ar_us = allreduce_us(dist, flat[0].clone(), stream) if world > 1 else 0.0

    # Single-GPU full-batch reference on rank 0.
    res = {}
    if rank == 0:
        grad = flat[last["k"]]
        if world == 1:
            xf, dyf = x, dy
        else:
            xf, dyf = rows_of(0, B, 1 << 20), rows_of(0, B, 2 << 20)
        ref = torch.zeros_like(grad)
        outf = _fwd(xf, w, b, None, None, None, True)
        dxf = _bwd(xf, w, b, None, None, dyf, None, False, True, grad_f32=ref)[0]
        torch.cuda.synchronize(dev)
        scale = max(1.0, float(ref.abs().max()))
        diff = float((grad - ref).abs().max())
        res = {"dweight_dbias_maxdiff_vs_1gpu": diff, "dweight_dbias_scale": scale,
               "within_bf16_sum_tol": diff <= 1e-2 * scale,
               "rank0_out_dx_bitexact_vs_1gpu": bool(torch.equal(outf[:nb], last["out"]) and
                                                      torch.equal(dxf[:nb], last["dx"]))}
        del xf, dyf, outf, dxf, ref
    del x, dy, last
    torch.cuda.empty_cache()
    if dist is not None:
        dist.barrier()
    fb, bb = algo_bytes(B, T, D, W)
    peak, kind = measured_peak()
    agg = (fb + bb) / (ms * 1e-3) / 1e9
    return {
        "workload": "BASELINE config 5: B=64 T=8192 D=8192 W=8 bf16 bias+silu fwd+bwd, strong-scaled "
                    "(64/N rows per GPU), NCCL all-reduce of fp32 dweight||dbias (295 KB)",
        "rows_per_gpu": nb, "steps": K, "ms_per_step": ms, "fwd_us": fwd_us,
        "bwd_us": bwd_us, "bwd_note": "backward kernel + reduce; the all-reduce runs on NCCL's stream",
        "allreduce_us": ar_us, "agg_gbs": agg, "frac_of_measured_per_gpu": agg / (world * peak),
        "peak": f"{kind} hbm_gbs {peak}", **res,
    }


def host_overhead(dev, calls=300):
    """Host time per eager call at BASELINE config 1 (B=2 T=1024 D=512 W=4 bf16, bias + SiLU),
    where each kernel runs for a few microseconds and the host decides the step time: the raw
    launchers (_fwd, _bwd: argument checks, output allocation, the C ABI call) and the whole
    public-API step (causal_conv1d_fn + autograd backward). CPU wall time over `calls` calls,
    median of 5 repeats, device synchronised around each repeat."""
    from causal_conv1d_b200 import causal_conv1d_fn
    from causal_conv1d_b200.causal_conv1d import _bwd, _fwd

    g = torch.Generator(device=dev).manual_seed(0)
    B, T, D, W = 2, 1024, 512, 4
    x = torch.randn(B, T, D, generator=g, device=dev, dtype=torch.bfloat16)
    w = torch.randn(D, W, generator=g, device=dev)
    b = torch.randn(D, generator=g, device=dev)
    dy = torch.randn(B, T, D, generator=g, device=dev, dtype=torch.bfloat16)
    xl, wl, bl = x.clone().requires_grad_(True), w.clone().requires_grad_(True), b.clone().requires_grad_(True)

    def step():
        xl.grad = wl.grad = bl.grad = None
        causal_conv1d_fn(xl, wl, bl, activation="silu").backward(dy)

    fns = {"fwd_launcher_us": lambda: _fwd(x, w, b, None, None, None, True),
           "bwd_launcher_us": lambda: _bwd(x, w, b, None, None, dy, None, False, True),
           "autograd_step_us": step}
    out = {}
    for name, fn in fns.items():
        for _ in range(20):
            fn()
        reps = []
        for _ in range(5):
            torch.cuda.synchronize(dev)
            t0 = time.perf_counter()
            for _ in range(calls):
                fn()
            reps.append((time.perf_counter() - t0) / calls * 1e6)
            torch.cuda.synchronize(dev)
        out[name] = statistics.median(reps)
    out["workload"] = "BASELINE config 1: B=2 T=1024 D=512 W=4 bf16 bias+silu, eager, CPU wall time per call"
    return out


def triton_arm(args, ours_line):
    """The reference's Triton kernels on this GPU and workload (`--impl triton` in a subprocess,
    same steps and warm-up), with the speed-ups of this repository's kernels over them."""
    cmd = [sys.executable, os.path.abspath(__file__), "--impl", "triton", "--gpus", "1",
           "--steps", str(args.steps), "--warmup", str(args.warmup), "--batch", str(args.batch),
           "--seqlen", str(args.seqlen), "--dim", str(args.dim), "--width", str(args.width)]
    if args.no_bias_silu:
        cmd.append("--no-bias-silu")
    drop = {"RANK", "WORLD_SIZE", "LOCAL_RANK", "LOCAL_WORLD_SIZE", "GROUP_RANK", "ROLE_RANK",
            "MASTER_ADDR", "MASTER_PORT", "TORCHELASTIC_RUN_ID"}
    env = {k: v for k, v in os.environ.items() if k not in drop}
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env)
    except Exception as e:  # noqa: BLE001 - reported in the line
        return {"unavailable": f"{type(e).__name__}: {e}"}
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    if r.returncode != 0 or not lines:
        return {"unavailable": f"rc {r.returncode}: {r.stderr.strip()[-400:]}"}
    t = json.loads(lines[-1])
    f_us, b_us = t["fwd"]["us_per_call"], t["bwd"]["us_per_call"]
    return {
        "source": "reference causal_conv1d_triton._fwd/_bwd from baseline/_ref (unmodified), same "
                  "workload and step count, run after this arm in a subprocess",
        "fwd_us": f_us, "bwd_us": b_us, "ms_per_step": t["ms_per_step"], "gbs": t["value"],
        "fwd_gbs": t["fwd"]["gbs"], "bwd_gbs": t["bwd"]["gbs"], "clocks": t.get("clocks"),
        "speedup_fwd": f_us / ours_line["fwd"]["us_per_call"],
        "speedup_bwd": b_us / ours_line["bwd"]["us_per_call"],
        "speedup_step": t["ms_per_step"] / ours_line["ms_per_step"],
    }


def e2e(args, dev, x_h, w_h, b_h, dy_h, bias_silu, world, dist):
    """Forward + backward through the public API with host buffers, as a data-loading training
    loop runs it: each step copies its x and dout from pinned host memory into one of two device
    slots on an input stream, runs causal_conv1d_fn and backward on the compute stream, and copies
    out, dx, dweight and dbias back to pinned host memory on an output stream. Step i+1's inputs
    cross the host link while step i's results come back (the link is full duplex); events order
    each slot's reuse after the compute that read it."""
    from causal_conv1d_b200 import causal_conv1d_fn
    from causal_conv1d_b200.distributed import sharded_causal_conv1d_fn

    fn = sharded_causal_conv1d_fn if world > 1 else causal_conv1d_fn

    xp, dyp = x_h.pin_memory(), dy_h.pin_memory()
    out_h = torch.empty_like(x_h).pin_memory()
    dx_h = torch.empty_like(x_h).pin_memory()
    dw_h = torch.empty_like(w_h).pin_memory()
    db_h = torch.empty_like(b_h).pin_memory() if b_h is not None else None
    w = w_h.to(dev).requires_grad_(True)
    b = b_h.to(dev).requires_grad_(True) if b_h is not None else None
    main = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    x_slot = [torch.empty(x_h.shape, dtype=x_h.dtype, device=dev) for _ in range(2)]
    dy_slot = [torch.empty(dy_h.shape, dtype=dy_h.dtype, device=dev) for _ in range(2)]
    slot_free = [None, None]  # event after the compute that last read each slot

    def h2d(i):
        k = i % 2
        if slot_free[k] is not None:
            s_in.wait_event(slot_free[k])
        with torch.cuda.stream(s_in):
            x_slot[k].copy_(xp, non_blocking=True)
            dy_slot[k].copy_(dyp, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(s_in)
        return ev

    def compute_and_d2h(i, ev_in):
        k = i % 2
        main.wait_event(ev_in)
        x = x_slot[k].detach().requires_grad_(True)
        w.grad = None
        if b is not None:
            b.grad = None
        out = fn(x, w, b, activation="silu" if bias_silu else None)
        out.backward(dy_slot[k])
        done = torch.cuda.Event()
        done.record(main)
        slot_free[k] = done
        res = [(out_h, out), (dx_h, x.grad), (dw_h, w.grad)] + ([(db_h, b.grad)] if b is not None else [])
        s_out.wait_event(done)
        with torch.cuda.stream(s_out):
            for h, d in res:
                h.copy_(d, non_blocking=True)
        for _, d in res:
            d.record_stream(s_out)

    def run(n):
        ev_next = h2d(0)
        for i in range(n):
            ev_in = ev_next
            if i + 1 < n:
                ev_next = h2d(i + 1)
            compute_and_d2h(i, ev_in)
        main.wait_stream(s_out)

    s_in.wait_stream(main)
    run(2)
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(main)
    s_in.wait_stream(main)
    run(args.e2e_steps)
    e.record(main)
    torch.cuda.synchronize(dev)
    ms = s.elapsed_time(e) / args.e2e_steps
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    B, T, D = x_h.shape
    W = w_h.shape[1]
    fb, bb = algo_bytes(B, T, D, W)
    h2d_bytes = xp.numel() * xp.element_size() + dyp.numel() * dyp.element_size()
    d2h_bytes = sum(t.numel() * t.element_size() for t in (out_h, dx_h, dw_h, db_h) if t is not None)
    return {"value": (fb + bb) * world / (ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms,
            "steps": args.e2e_steps, "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": d2h_bytes,
            "copies": "pinned host buffers; step i+1's inputs copied in while step i's results are "
                      "copied out (separate streams)"}


if __name__ == "__main__":
    main()
