"""Parity at the full shapes of the five BASELINE configurations.

Each configuration is built as specified (shapes, dtypes, input distributions, seq_idx packing,
state chaining) and run through the public `causal_conv1d_fn` with autograd, then checked three
ways:

- every element of out, dx, dinit and the dweight / dbias sums against the torch fp32
  restatement of the reference (tests/_torch_ref.py, itself checked against the C oracle and the
  reference's golden vectors on the CPU), computed on the GPU over chunks of batch rows;
- two sampled batch rows of out, dx and dinit against the pinned C oracle;
- the same call through the unmodified reference, jxiong21029/causal-conv1d-triton's
  `causal_conv1d_fn` (causal_conv1d_triton/causal_conv1d.py:579-639, installed under
  baseline/_ref), on the same B200 with the same inputs: outputs and gradients within the
  tolerance, final states and padding zeros bit-exact.

Tolerances (tests/_tol.py): bf16 |a - e| <= 1e-2 + 1e-2 |e|, fp32 1e-5 in both terms;
dweight / dbias (sums over B*T rows) within tol * max(1, max |e|). Bit-exact: the final states
after every chunk of the config-3 chain, and out / dx at every config-4 padding row (exact zeros).

Two further cases (not BASELINE configurations) give the backward walks of more than 2048 rows
per CTA, where it switches to 24-row stages, with states, seq_idx packing and partial channel
groups.

Config 5 (B=64, T=8192, D=8192, W=8: 4.3e9 elements per tensor) is the only one whose element
offsets pass 2^31; it exercises the kernels' 64-bit indexing. It holds about 52 GB on the device
at its peak.
"""

from __future__ import annotations

import gc
import os
import sys

import numpy as np
import pytest
import torch

from _tol import TOL, assert_close
from _torch_ref import backward_chunk, forward_chunk

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _reference_fn():
    """The unmodified reference's causal_conv1d_fn from baseline/_ref, or None with the reason."""
    path = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(path, "causal_conv1d_triton")):
        return None, "baseline/_ref is not installed"
    if path not in sys.path:
        sys.path.insert(0, path)
    try:
        from causal_conv1d_triton import causal_conv1d_fn
    except Exception as e:  # pragma: no cover - depends on the box
        return None, f"reference import failed: {e}"
    return causal_conv1d_fn, None


# name -> spec. w_std / b_std are the standard deviations of the fp32 weight and bias.
CONFIGS = {
    "cfg1_B2_T1024_D512": dict(B=2, T=1024, D=512, W=4, w_std=1.0, b_std=1.0, silu=True),
    **{f"cfg2_B8_T{T}_D1024_{m}": dict(B=8, T=T, D=1024, W=4, w_std=0.5,
                                        b_std=(0.1 ** 0.5 if m == "bias_silu" else None),
                                        silu=m == "bias_silu")
       for T in (512, 2048, 8192, 32768) for m in ("none", "bias_silu")},
    "cfg3_B16_T8192_D2048_chain4": dict(B=16, T=8192, D=2048, W=4, w_std=0.5, b_std=0.1 ** 0.5,
                                        silu=True, init=True, chunks=4),
    "cfg4_B4_T16384_D4352_varlen": dict(B=4, T=16384, D=4352, W=4, w_std=0.5, b_std=0.1 ** 0.5,
                                        silu=True, init=True, varlen=True),
    "cfg5_B64_T8192_D8192_W8": dict(B=64, T=8192, D=8192, W=8, w_std=8 ** -0.5, b_std=0.1 ** 0.5,
                                    silu=True),
    # Not a BASELINE config: cfg2's shape in fp32, held to the fp32 tolerance.
    "cfg2_B8_T8192_D1024_bias_silu_fp32": dict(B=8, T=8192, D=1024, W=4, w_std=0.5,
                                               b_std=0.1 ** 0.5, silu=True, dtype=torch.float32),
    # Not BASELINE configs: walks long enough (more than 2048 rows per CTA) for the backward's
    # 24-row-stage kernel, at widths 8 and 7 (chained chunks: initial and final states) and 5 and 6
    # (packed seq_idx with padding and initial states), in bf16, fp16 and fp32, with a partial last
    # channel group (D = 7936) and stages that cross batch rows and end partial (T not a multiple
    # of 24).
    "long_walk_W8_B2_T40000_D7936_chain2": dict(B=2, T=40000, D=7936, W=8, w_std=8 ** -0.5,
                                                b_std=0.1 ** 0.5, silu=True, init=True, chunks=2),
    "long_walk_W5_B2_T40000_D7936_varlen": dict(B=2, T=40000, D=7936, W=5, w_std=5 ** -0.5,
                                                b_std=0.1 ** 0.5, silu=True, init=True, varlen=True),
    "long_walk_W6_B2_T40000_D7936_varlen_fp16": dict(B=2, T=40000, D=7936, W=6, w_std=6 ** -0.5,
                                                     b_std=0.1 ** 0.5, silu=True, init=True, varlen=True,
                                                     dtype=torch.float16),
    "long_walk_W7_B2_T40000_D7936_chain2_fp32": dict(B=2, T=40000, D=7936, W=7, w_std=7 ** -0.5,
                                                     b_std=0.1 ** 0.5, silu=True, init=True, chunks=2,
                                                     dtype=torch.float32),
}


def _varlen_seq(B, T, seed):
    """Rows filled with consecutive sequences of lengths U[64, 4096] (ids 0, 1, ...), the trailing
    U[0, 255] positions of each row set to -1 (padding)."""
    g = torch.Generator().manual_seed(seed)
    seq = torch.empty(B, T, dtype=torch.int32)
    for r in range(B):
        pad = int(torch.randint(0, 256, (1,), generator=g))
        t, sid = 0, 0
        while t < T - pad:
            n = int(torch.randint(64, 4097, (1,), generator=g))
            seq[r, t:min(t + n, T - pad)] = sid
            t, sid = t + n, sid + 1
        seq[r, T - pad:] = -1
    return seq


def make_case(name, seed=0):
    s = CONFIGS[name]
    B, T, D, W = s["B"], s["T"], s["D"], s["W"]
    dt = s.get("dtype", torch.bfloat16)
    g = torch.Generator(device=DEV).manual_seed(seed)
    c = dict(spec=s, dtype=dt)
    c["x"] = torch.randn(B, T, D, generator=g, device=DEV, dtype=dt)
    c["w"] = torch.randn(D, W, generator=g, device=DEV) * s["w_std"]
    c["b"] = torch.randn(D, generator=g, device=DEV) * s["b_std"] if s["b_std"] else None
    c["init"] = torch.randn(B, W - 1, D, generator=g, device=DEV, dtype=dt) if s.get("init") else None
    c["seq"] = _varlen_seq(B, T, seed + 4).to(DEV) if s.get("varlen") else None
    c["dy"] = torch.randn(B, T, D, generator=g, device=DEV, dtype=dt)
    return c


def run(fn, c):
    """Forward + backward through `fn` (a causal_conv1d_fn). Returns a dict of detached results."""
    s = c["spec"]
    act = "silu" if s["silu"] else None
    w = c["w"].detach().clone().requires_grad_(True)
    b = c["b"].detach().clone().requires_grad_(True) if c["b"] is not None else None
    init = c["init"].detach().clone().requires_grad_(True) if c["init"] is not None else None
    r = {}
    if s.get("chunks"):
        L = s["T"] // s["chunks"]
        xs = [c["x"][:, i * L:(i + 1) * L].detach().clone().requires_grad_(True)
              for i in range(s["chunks"])]
        state, outs, finals = init, [], []
        for xc in xs:
            o, state = fn(xc, w, b, initial_states=state, return_final_states=True, activation=act)
            outs.append(o)
            finals.append(state.detach().clone())
        torch.autograd.backward(outs, [c["dy"][:, i * L:(i + 1) * L] for i in range(s["chunks"])])
        r["out"] = torch.cat([o.detach() for o in outs], 1)
        r["dx"] = torch.cat([xc.grad for xc in xs], 1)
        r["finals"] = finals
        del outs, xs
    else:
        x = c["x"].detach().requires_grad_(True)
        out = fn(x, w, b, seq_idx=c["seq"], initial_states=init, activation=act)
        out.backward(c["dy"])
        r["out"] = out.detach()
        r["dx"] = x.grad
        x.grad = None
        del out
    r["dw"] = w.grad
    r["db"] = b.grad if b is not None else None
    r["dinit"] = init.grad if init is not None else None
    torch.cuda.synchronize()
    return r


def _rows_per_chunk(c):
    T, D = c["x"].shape[1:]
    return max(1, int(2 ** 28 // (T * D)))  # ~1 GB of fp32 per temporary


def _close_gpu(a, e, tol, what):
    """|a - e| <= tol + tol |e| elementwise, on the GPU (a, e any float dtype, same shape)."""
    err = (a.float() - e.float()).abs()
    bad = ~(err <= tol + tol * e.float().abs())
    if bool(bad.any()):
        i = int(torch.argmax((err - tol * e.float().abs()).flatten()))
        idx = np.unravel_index(i, a.shape)
        raise AssertionError(f"{what}: {int(bad.sum())} of {a.numel()} outside tol {tol}; worst at {idx}: "
                             f"actual {float(a[idx])!r} expected {float(e[idx])!r}")


def _close_sum(a, e, tol, what):
    a, e = a.double(), e.double()
    scale = max(1.0, float(e.abs().max()))
    err = (a - e).abs()
    if not bool((err <= tol * scale).all()):
        i = int(torch.argmax(err.flatten()))
        raise AssertionError(f"{what}: max err {float(err.max()):.4g} > {tol}*{scale:.4g} at flat index {i}")


def _free():
    gc.collect()
    torch.cuda.empty_cache()


def check_against_torch(c, r):
    s = c["spec"]
    tol = TOL["f32" if c["dtype"] == torch.float32 else "bf16"]
    B, T, D = c["x"].shape
    W = s["W"]
    dw = torch.zeros(D, W, dtype=torch.float64, device=DEV)
    db = torch.zeros(D, dtype=torch.float64, device=DEV) if c["b"] is not None else None
    step = _rows_per_chunk(c)
    for i in range(0, B, step):
        j = min(B, i + step)
        sl = slice(i, j)
        init = c["init"][sl] if c["init"] is not None else None
        seq = c["seq"][sl] if c["seq"] is not None else None
        _, out = forward_chunk(c["x"][sl], c["w"], c["b"], init, seq, s["silu"])
        _close_gpu(r["out"][sl], out, tol, f"out rows {i}:{j}")
        del out
        dx, dinit, dwc, dbc = backward_chunk(c["x"][sl], c["w"], c["b"], init, seq, c["dy"][sl], None, s["silu"])
        _close_gpu(r["dx"][sl], dx, tol, f"dx rows {i}:{j}")
        if dinit is not None:
            _close_gpu(r["dinit"][sl], dinit, tol, f"dinit rows {i}:{j}")
        dw += dwc
        if db is not None:
            db += dbc
        del dx, dinit
        _free()
    _close_sum(r["dw"], dw, tol, "dweight")
    if db is not None:
        _close_sum(r["db"], db, tol, "dbias")


def check_against_oracle(c, r):
    """Batch rows 0 and B-1 of out, dx and dinit against the C oracle (one long call per row: the
    config-3 chain equals one call over the whole sequence)."""
    from oracle import oracle

    s = c["spec"]
    key = "f32" if c["dtype"] == torch.float32 else "bf16"
    B = c["x"].shape[0]
    for row in sorted({0, B - 1}):
        sl = slice(row, row + 1)
        x = c["x"][sl].float().cpu()
        init = c["init"][sl].float().cpu() if c["init"] is not None else None
        seq = c["seq"][sl].cpu() if c["seq"] is not None else None
        dy = c["dy"][sl].float().cpu()
        w = c["w"].cpu()
        b = c["b"].cpu() if c["b"] is not None else None
        eo = oracle.fwd(x, w, b, init, seq, silu=s["silu"])
        assert_close(r["out"][sl].float().cpu(), eo, key, f"out row {row} vs oracle")
        del eo
        edx, _, _, edi = oracle.bwd(x, w, b, init, seq, dy, None, need_dinit=init is not None, silu=s["silu"])
        assert_close(r["dx"][sl].float().cpu(), edx, key, f"dx row {row} vs oracle")
        if init is not None:
            assert_close(r["dinit"][sl].float().cpu(), edi, key, f"dinit row {row} vs oracle")


def check_bitexact_contracts(c, r):
    s = c["spec"]
    if s.get("chunks"):  # final states after chunk i = x rows [(i+1)L - (W-1), (i+1)L)
        L, pad = s["T"] // s["chunks"], s["W"] - 1
        for i, f in enumerate(r["finals"]):
            e = c["x"][:, (i + 1) * L - pad:(i + 1) * L]
            assert torch.equal(f, e), f"final states after chunk {i} are not bit-exact"
    if c["seq"] is not None:
        padrows = (c["seq"] < 0).unsqueeze(-1).expand_as(r["out"])
        assert int(padrows.sum()) > 0
        assert bool((r["out"][padrows] == 0).all()), "out at padding rows is not exactly zero"
        assert bool((r["dx"][padrows] == 0).all()), "dx at padding rows is not exactly zero"


@pytest.mark.parametrize("name", list(CONFIGS))
def test_config_matches_torch_reference_and_oracle(name):
    from causal_conv1d_b200 import causal_conv1d_fn

    c = make_case(name)
    r = run(causal_conv1d_fn, c)
    check_bitexact_contracts(c, r)
    check_against_oracle(c, r)
    check_against_torch(c, r)
    del r, c
    _free()


@pytest.mark.parametrize("name", [n for n in CONFIGS if not n.endswith("fp32")])
def test_config_matches_reference_triton_on_b200(name):
    ref, why = _reference_fn()
    if ref is None:
        pytest.skip(why)
    from causal_conv1d_b200 import causal_conv1d_fn

    c = make_case(name)
    ours = run(causal_conv1d_fn, c)
    check_bitexact_contracts(c, ours)
    theirs = run(ref, c)
    tol = TOL["bf16"]
    for k in ("out", "dx", "dinit"):
        if ours[k] is not None:
            B = ours[k].shape[0]
            step = _rows_per_chunk(c)
            for i in range(0, B, step):
                _close_gpu(ours[k][i:i + step], theirs[k][i:i + step], tol, f"{k} rows {i}: ours vs reference")
    _close_sum(ours["dw"], theirs["dw"], tol, "dweight: ours vs reference")
    if ours["db"] is not None:
        _close_sum(ours["db"], theirs["db"], tol, "dbias: ours vs reference")
    for i, (a, e) in enumerate(zip(ours.get("finals", []), theirs.get("finals", []))):
        assert torch.equal(a, e), f"final states after chunk {i}: ours and the reference's differ"
    if c["seq"] is not None:
        padrows = (c["seq"] < 0).unsqueeze(-1).expand_as(ours["out"])
        assert torch.equal(ours["out"][padrows], theirs["out"][padrows])
        assert torch.equal(ours["dx"][padrows], theirs["dx"][padrows])
    del ours, theirs, c
    _free()
