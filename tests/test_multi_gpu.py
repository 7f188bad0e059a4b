"""Data-parallel path on 2 GPUs over NCCL: each rank runs its batch shard through
sharded_causal_conv1d_fn, and the all-reduced weight/bias gradients must equal the single-GPU
gradients of the whole batch (within the bf16 tolerance; the sum is grouped differently) and be
identical on both ranks, while out, dx, dinit and the final states of each shard equal the
single-GPU results for those rows bit for bit. Three cases: plain bias + SiLU; packed
variable-length rows (seq_idx with padding, initial states) with the all-reduce deferred to the
end of the backward pass; chunked streaming state (initial and final states, final_states_out).
The first two again with the rank-order (deterministic) gradient sum, immediate and deferred.
Skipped with fewer than two GPUs."""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

TESTS = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(TESTS)
PATHS = [TESTS, ROOT, os.path.join(ROOT, "causal-conv1d-triton_b200")]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(case):
    g = torch.Generator().manual_seed(4)
    B, T, D, W = 6, 2048, 512, 4
    x = torch.randn(B, T, D, generator=g).to(torch.bfloat16)
    w = torch.randn(D, W, generator=g) * 0.5
    b = torch.randn(D, generator=g) * 0.3
    dy = torch.randn(B, T, D, generator=g).to(torch.bfloat16)
    init = torch.randn(B, W - 1, D, generator=g).to(torch.bfloat16) if case != "plain" else None
    seq = None
    if case == "varlen":
        seq = torch.zeros(B, T, dtype=torch.int32)
        for r in range(B):
            cuts = sorted(torch.randint(64, T - 300, (3,), generator=g).tolist())
            for i, c in enumerate(cuts):
                seq[r, c:] = i + 1
            seq[r, T - 17 * (r + 1):] = -1
    dfin = torch.randn(B, W - 1, D, generator=g).to(torch.bfloat16) if case == "stream" else None
    return dict(x=x, w=w, b=b, dy=dy, init=init, seq=seq, dfin=dfin)


def _run(fn, t, dev, sl, **kw):
    """Forward + backward of one case on rows `sl`; returns the results on the host."""
    x = t["x"][sl].to(dev).requires_grad_(True)
    w = t["w"].to(dev).requires_grad_(True)
    b = t["b"].to(dev).requires_grad_(True)
    init = t["init"][sl].to(dev).requires_grad_(True) if t["init"] is not None else None
    seq = t["seq"][sl].to(dev) if t["seq"] is not None else None
    r = {}
    if t["dfin"] is not None:
        fso = torch.empty(x.shape[0], w.shape[1] - 1, x.shape[2], device=dev, dtype=x.dtype)
        out, fin = fn(x, w, b, initial_states=init, return_final_states=True, final_states_out=fso,
                      activation="silu", **kw)
        assert fin is fso
        torch.autograd.backward([out, fin], [t["dy"][sl].to(dev), t["dfin"][sl].to(dev)])
        r["final"] = fin.detach().cpu()
    else:
        out = fn(x, w, b, seq_idx=seq, initial_states=init, activation="silu", **kw)
        out.backward(t["dy"][sl].to(dev))
    torch.cuda.synchronize()
    r.update(out=out.detach().cpu(), dx=x.grad.cpu(), dw=w.grad.cpu(), db=b.grad.cpu())
    if init is not None:
        r["dinit"] = init.grad.cpu()
    return r


# (result name, input case, deferred all-reduce, rank-order sum)
CASES = [("plain", "plain", False, False), ("varlen", "varlen", True, False), ("stream", "stream", False, False),
         ("plain_det", "plain", False, True), ("varlen_det", "varlen", True, True)]


def _worker(rank, world, port, out_dir):
    import sys

    sys.path[:0] = PATHS
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    from causal_conv1d_b200.distributed import shard_rows, sharded_causal_conv1d_fn

    res = {}
    for name, case, overlap, det in CASES:
        t = _inputs(case)
        sl = shard_rows(t["x"].shape[0], rank, world)
        res[name] = _run(sharded_causal_conv1d_fn, t, dev, sl, overlap_grad_reduce=overlap,
                         deterministic_grad_reduce=det)
    torch.save(res, os.path.join(out_dir, f"r{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_batch_shards_match_single_gpu(tmp_path):
    from _tol import assert_close_sum
    from causal_conv1d_b200 import causal_conv1d_fn

    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    r = [torch.load(tmp_path / f"r{i}.pt") for i in range(2)]
    dev = torch.device("cuda", 0)
    for name, case, _, _ in CASES:
        a, c = r[0][name], r[1][name]
        assert torch.equal(a["dw"], c["dw"]) and torch.equal(a["db"], c["db"]), name
        full = _run(causal_conv1d_fn, _inputs(case), dev, slice(None))
        for k in ("out", "dx", "dinit", "final"):
            if k in full:
                assert torch.equal(torch.cat([a[k], c[k]]), full[k]), f"{name}: {k}"
        assert_close_sum(a["dw"], full["dw"], "bf16", f"{name}: dweight")
        assert_close_sum(a["db"], full["db"], "bf16", f"{name}: dbias")
    # Two ranks: the rank-order sum v_0 + v_1 and NCCL's sum of the same two vectors are one
    # floating-point addition, so both modes give the same bits.
    for name in ("plain", "varlen"):
        assert torch.equal(r[0][name]["dw"], r[0][name + "_det"]["dw"]), name
