"""Parity of the CUDA path (through the C ABI, via causal_conv1d_fn) with the reference.

- Every golden vector of the reference implementation (tests/golden/, produced by the reference's
  own `_fwd`/`_bwd`) is replayed through the public API, forward and backward.
- A sweep over dtypes, widths (TMA path 2..8, generic path above), flags, ragged sizes and
  strided/misaligned layouts is compared with the CPU oracle (oracle/, pinned to the same golden
  vectors) on identical inputs.
- Bit-exact items: final_states, zero outputs (and dx) at seq_idx padding rows.

Tolerances are those of tests/_tol.py (bf16/fp16 1e-2 rel + 1e-2 abs, fp32 1e-5).
"""

import itertools

import numpy as np
import pytest
import torch

from _golden import CASE_IDS, CASES
from _tol import assert_bitexact, assert_close, assert_close_sum
from oracle import oracle

pytestmark = pytest.mark.gpu

DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
DEV = "cuda:0"


@pytest.fixture(scope="module")
def cc():
    import causal_conv1d_b200

    return causal_conv1d_b200


def run_api(cc, x, weight, bias, seq_idx, init, return_final, silu, dout, dfinal, need_dinit):
    """Forward + backward through causal_conv1d_fn; returns numpy fp32 copies of every result."""
    x = x.detach().clone().requires_grad_(True)
    weight = weight.detach().clone().requires_grad_(True)
    bias = bias.detach().clone().requires_grad_(True) if bias is not None else None
    if init is not None:
        init = init.detach().clone().requires_grad_(need_dinit)
    res = cc.causal_conv1d_fn(x, weight, bias, seq_idx=seq_idx, initial_states=init,
                              return_final_states=return_final,
                              activation="silu" if silu else None)
    out, final = res if return_final else (res, None)
    outs, grads = [out], [dout]
    if final is not None and dfinal is not None:
        outs.append(final)
        grads.append(dfinal)
    torch.autograd.backward(outs, grads)
    torch.cuda.synchronize()
    f = lambda t: None if t is None else t.detach().float().cpu().numpy()  # noqa: E731
    return {
        "out": f(out), "final": f(final), "dx": f(x.grad), "dweight": f(weight.grad),
        "dbias": f(bias.grad) if bias is not None else None,
        "dinit": f(init.grad) if (init is not None and need_dinit) else None,
    }


@pytest.mark.parametrize("case", CASES, ids=CASE_IDS)
def test_golden_vectors(cc, case):
    m, g = case
    xdt, wdt = DT[m["x_dtype"]], DT[m["w_dtype"]]
    t = lambda k, dt: torch.from_numpy(g[k]).to(dt).to(DEV) if k in g else None  # noqa: E731
    seq = torch.from_numpy(g["seq_idx"]).to(DEV) if "seq_idx" in g else None
    r = run_api(cc, t("x", xdt), t("weight", wdt), t("bias", wdt), seq,
                t("initial_states", xdt), m["return_final_states"], m["silu"], t("dout", xdt),
                t("dfinal_states", xdt), m["need_dinit"])
    key = m["x_dtype"]
    assert_close(r["out"], g["out"], key, "out")
    if m["return_final_states"]:
        assert_bitexact(r["final"], g["final_states"], "final_states")
    assert_close(r["dx"], g["dx"], key, "dx")
    assert_close_sum(r["dweight"], g["dweight"], key, "dweight")
    if m["bias"]:
        assert_close_sum(r["dbias"], g["dbias"], key, "dbias")
    if m["need_dinit"]:
        assert_close(r["dinit"], g["dinit"], key, "dinit")
    if m["seq"] and m["T"] > 0:
        pad = g["seq_idx"] < 0
        assert (r["out"][pad] == 0).all() and (r["dx"][pad] == 0).all()


def make_seq(B, T, gen, max_len=None):
    seq = torch.empty(B, T, dtype=torch.int32)
    max_len = max_len or max(2, T // 3)
    for b in range(B):
        pad = int(torch.randint(0, max(1, T // 8), (1,), generator=gen))
        t, sid = 0, 0
        while t < T - pad:
            n = int(torch.randint(1, max_len + 1, (1,), generator=gen))
            seq[b, t:min(t + n, T - pad)] = sid
            t += n
            sid += 1
        seq[b, T - pad:] = -1
    return seq


def layout(x, mode):
    """Re-lays x (B, T, D) out in device memory: contiguous, time-strided (padded rows), batch
    strided, or with a base address that is not 16-byte aligned."""
    B, T, D = x.shape
    if mode == "contig":
        return x.contiguous()
    if mode == "row_pad8":  # row stride D + 8: 16-byte aligned for 16-bit types
        buf = torch.zeros(B, T, D + 8, dtype=x.dtype, device=x.device)
        buf[..., :D] = x
        return buf[..., :D]
    if mode == "row_pad1":  # row stride D + 1: not 16-byte aligned
        buf = torch.zeros(B, T, D + 1, dtype=x.dtype, device=x.device)
        buf[..., :D] = x
        return buf[..., :D]
    if mode == "batch_gap":  # batch stride (T + 3) * D
        buf = torch.zeros(B, T + 3, D, dtype=x.dtype, device=x.device)
        buf[:, 1:T + 1] = x
        return buf[:, 1:T + 1]
    if mode == "offset1":  # base address shifted by one element
        flat = torch.zeros(B * T * D + 1, dtype=x.dtype, device=x.device)
        v = flat[1:].view(B, T, D)
        v.copy_(x)
        return v
    raise ValueError(mode)


def check_vs_oracle(cc, B, T, D, W, dt, has_bias, silu, has_init, has_seq, ret_final, dfinal,
                    need_dinit, seed, x_layout="contig", dy_layout="contig", wdt=torch.float32):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, D, generator=gen).to(dt)
    weight = (torch.randn(D, W, generator=gen) / W**0.5).to(wdt)
    bias = (torch.randn(D, generator=gen) * 0.3).to(wdt) if has_bias else None
    init = torch.randn(B, W - 1, D, generator=gen).to(dt) if has_init else None
    seq = make_seq(B, T, gen) if has_seq else None
    dy = torch.randn(B, T, D, generator=gen).to(dt)
    dfin = torch.randn(B, W - 1, D, generator=gen).to(dt) if (dfinal and ret_final) else None

    gx = layout(x.to(DEV), x_layout)
    gdy = layout(dy.to(DEV), dy_layout)
    r = run_api(cc, gx, weight.to(DEV), bias.to(DEV) if bias is not None else None,
                seq.to(DEV) if seq is not None else None,
                init.to(DEV) if init is not None else None, ret_final, silu, gdy,
                dfin.to(DEV) if dfin is not None else None, need_dinit and has_init)

    o = oracle.fwd(x, weight, bias, init, seq, silu=silu, return_final_states=ret_final)
    out, final = o if ret_final else (o, None)
    dx, dw, db, dinit = oracle.bwd(x, weight, bias, init, seq, dy, dfin,
                                   need_dinit=need_dinit and has_init, silu=silu)
    rnd = lambda a, d: torch.from_numpy(a).to(d).float().numpy()  # noqa: E731
    key = str(dt)
    assert_close(r["out"], rnd(out, dt), key, "out")
    if ret_final:
        assert_bitexact(r["final"], rnd(final, dt), "final_states")
    assert_close(r["dx"], rnd(dx, dt), key, "dx")
    assert_close_sum(r["dweight"], rnd(dw, wdt), key, "dweight")
    if has_bias:
        assert_close_sum(r["dbias"], rnd(db, wdt), key, "dbias")
    if need_dinit and has_init:
        assert_close(r["dinit"], rnd(dinit, dt), key, "dinit")
    if has_seq:
        pad = (seq < 0).numpy()
        assert (r["out"][pad] == 0).all(), "padding outputs must be exactly 0"
        assert (r["dx"][pad] == 0).all(), "padding dx must be exactly 0"


SWEEP = []
# 9..16 run on the width-12/16 kernels with leading zero taps.
for dt, W in itertools.product([torch.bfloat16, torch.float16, torch.float32], [2, 3, 4, 5, 6, 7, 8, 9, 12, 13, 16]):
    SWEEP.append((dt, W))


@pytest.mark.parametrize("dt,W", SWEEP, ids=[f"{str(d)[6:]}-W{w}" for d, w in SWEEP])
@pytest.mark.parametrize("flags", ["plain", "bias_silu", "state_chain", "seq_init", "seq"])
def test_sweep_tma_path(cc, dt, W, flags):
    f = dict(has_bias=False, silu=False, has_init=False, has_seq=False, ret_final=False,
             dfinal=False, need_dinit=False)
    if flags == "bias_silu":
        f.update(has_bias=True, silu=True)
    elif flags == "state_chain":
        f.update(has_bias=True, silu=True, has_init=True, ret_final=True, dfinal=True, need_dinit=True)
    elif flags == "seq_init":
        f.update(has_bias=True, silu=True, has_init=True, has_seq=True, need_dinit=True)
    elif flags == "seq":
        f.update(silu=True, has_seq=True)
    # D = 200: a partial channel block; T = 150: a partial time tile.
    check_vs_oracle(cc, 3, 150, 200, W, dt, seed=W * 7 + len(flags), **f)


@pytest.mark.parametrize("W", [17, 33, 64])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_generic_width(cc, W, dt):
    check_vs_oracle(cc, 2, 130, 72, W, dt, has_bias=True, silu=True, has_init=True,
                    has_seq=False, ret_final=True, dfinal=True, need_dinit=True, seed=W)


@pytest.mark.parametrize("W", [4, 12])
def test_generic_width_seq(cc, W):
    # D = 36: rows of 72 bytes keep these on the generic kernels (no aligned copy helps).
    check_vs_oracle(cc, 2, 140, 36, W, torch.bfloat16, has_bias=True, silu=True, has_init=True,
                    has_seq=True, ret_final=False, dfinal=False, need_dinit=True, seed=3 + W,
                    x_layout="row_pad1")


@pytest.mark.parametrize("x_layout,dy_layout", [
    ("row_pad8", "contig"), ("row_pad1", "contig"), ("batch_gap", "row_pad8"),
    ("offset1", "contig"), ("contig", "row_pad1"), ("contig", "offset1"),
])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_strided_layouts(cc, x_layout, dy_layout, dt):
    check_vs_oracle(cc, 2, 100, 136, 4, dt, has_bias=True, silu=True, has_init=True,
                    has_seq=False, ret_final=True, dfinal=True, need_dinit=True, seed=11,
                    x_layout=x_layout, dy_layout=dy_layout)


@pytest.mark.parametrize("B,T,D,W", [
    (1, 1, 8, 4), (2, 2, 16, 4), (3, 5, 24, 8), (1, 64, 128, 4), (1, 65, 128, 4),
    (2, 63, 8, 2), (1, 300, 13, 4), (4, 17, 1000, 3), (1, 7, 2048, 5),
])
def test_ragged_sizes(cc, B, T, D, W):
    check_vs_oracle(cc, B, T, D, W, torch.bfloat16, has_bias=True, silu=True, has_init=True,
                    has_seq=False, ret_final=True, dfinal=True, need_dinit=True, seed=B * T + D)


@pytest.mark.parametrize("seq", [False, True])
def test_more_batch_rows_than_a_grid_dimension(cc, seq):
    """More than 65535 batch rows: the forward's grid cannot be 3-D (channel block, time tile, batch
    row) and falls back to a flat grid whose index the kernel decomposes."""
    check_vs_oracle(cc, 70000, 3, 64, 4, torch.bfloat16, has_bias=True, silu=True, has_init=True,
                    has_seq=seq, ret_final=not seq, dfinal=not seq, need_dinit=True, seed=70000)


def test_bf16_weights(cc):
    check_vs_oracle(cc, 2, 90, 64, 4, torch.bfloat16, has_bias=True, silu=True, has_init=True,
                    has_seq=False, ret_final=True, dfinal=True, need_dinit=True, seed=5,
                    wdt=torch.bfloat16)


def test_empty_seqlen(cc):
    """T == 0: final = initial_states, dinit = dfinal, zero weight/bias grads (causal_conv1d.py:
    437-444, 480-489)."""
    check_vs_oracle(cc, 2, 0, 16, 4, torch.float32, has_bias=True, silu=True, has_init=True,
                    has_seq=False, ret_final=True, dfinal=True, need_dinit=True, seed=1)


def test_streaming_chain_matches_single_call(cc):
    """Chunked streaming (the BASELINE chunk-chain config, scaled down): four calls chained through
    initial/final states equal one call; every final state is bit-exact."""
    gen = torch.Generator().manual_seed(7)
    B, T, D, W, n = 2, 512, 256, 4, 4
    x = torch.randn(B, T, D, generator=gen).to(torch.bfloat16).to(DEV)
    w = (torch.randn(D, W, generator=gen) * 0.5).to(DEV)
    b = torch.randn(D, generator=gen).to(DEV)
    init = torch.randn(B, W - 1, D, generator=gen).to(torch.bfloat16).to(DEV)
    full = cc.causal_conv1d_fn(x, w, b, initial_states=init, activation="silu")
    state, outs = init, []
    cat = torch.cat([init, x], 1)
    for i in range(n):
        xi = x[:, i * T // n:(i + 1) * T // n]
        o, state = cc.causal_conv1d_fn(xi, w, b, initial_states=state, return_final_states=True,
                                       activation="silu")
        outs.append(o)
        end = W - 1 + (i + 1) * T // n
        assert torch.equal(state, cat[:, end - (W - 1):end]), "final state not bit-exact"
    assert torch.equal(torch.cat(outs, 1), full)


def test_final_states_out_and_swish(cc):
    x = torch.randn(2, 33, 64, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(64, 4, device=DEV)
    buf = torch.empty(2, 3, 64, device=DEV, dtype=torch.bfloat16)
    o1, f1 = cc.causal_conv1d_fn(x, w, return_final_states=True, final_states_out=buf,
                                 activation="swish")
    o2 = cc.causal_conv1d_fn(x, w, activation="silu")
    assert f1.data_ptr() == buf.data_ptr()
    assert torch.equal(buf, x[:, -3:])
    assert torch.equal(o1, o2)


def test_deterministic_weight_grads(cc):
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(4, 4096, 512, generator=gen).to(torch.bfloat16).to(DEV)
    w = torch.randn(512, 4, generator=gen).to(DEV)
    b = torch.randn(512, generator=gen).to(DEV)
    dy = torch.randn(4, 4096, 512, generator=gen).to(torch.bfloat16).to(DEV)
    from causal_conv1d_b200.causal_conv1d import _bwd

    r1 = _bwd(x, w, b, None, None, dy, None, False, True)
    r2 = _bwd(x, w, b, None, None, dy, None, False, True)
    for a, c in zip(r1[:3], r2[:3]):
        assert torch.equal(a, c)


@pytest.mark.parametrize("bias", [True, False])
def test_fp32_gradient_vector_output(cc, bias):
    """The backward's fp32 [dweight (D, W), dbias (D)] output (`grad_f32`, what the data-parallel
    path all-reduces) holds the same bits as the ordinary dweight/dbias outputs; dx is unchanged
    and dweight/dbias are not returned."""
    gen = torch.Generator().manual_seed(5)
    D, W = 512, 8
    x = torch.randn(2, 3000, D, generator=gen).to(torch.bfloat16).to(DEV)
    w = torch.randn(D, W, generator=gen).to(DEV)
    b = torch.randn(D, generator=gen).to(DEV) if bias else None
    dy = torch.randn(2, 3000, D, generator=gen).to(torch.bfloat16).to(DEV)
    from causal_conv1d_b200.causal_conv1d import _bwd

    dx, dw, db, _ = _bwd(x, w, b, None, None, dy, None, False, True)
    flat = torch.full((D * (W + 1),), float("nan"), device=DEV)
    dx2, dw2, db2, _ = _bwd(x, w, b, None, None, dy, None, False, True, grad_f32=flat)
    assert dw2 is None and db2 is None
    assert torch.equal(dx2, dx)
    assert torch.equal(flat[: D * W].view(D, W), dw)
    if bias:
        assert torch.equal(flat[D * W:], db)
    else:
        assert bool((flat[D * W:] == 0).all()), "dbias part of the vector is zero without bias"


def test_status_word_clear(cc):
    from causal_conv1d_b200 import _native

    x = torch.randn(2, 300, 256, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    w = torch.randn(256, 4, device=DEV, requires_grad=True)
    cc.causal_conv1d_fn(x, w, activation="silu").sum().backward()
    assert _native.status(clear=True) == 0


def test_no_grad_path_and_other_device_stream(cc):
    """Inference path (no autograd) on a non-default stream gives the same output."""
    x = torch.randn(2, 200, 128, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(128, 4, device=DEV)
    ref = cc.causal_conv1d_fn(x, w, activation="silu")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.no_grad(), torch.cuda.stream(s):
        out = cc.causal_conv1d_fn(x, w, activation="silu")
    s.synchronize()
    assert torch.equal(out, ref)


def test_sharded_fn_single_rank_matches_api(cc):
    """Without a process group the data-parallel wrapper equals causal_conv1d_fn exactly."""
    from causal_conv1d_b200.distributed import sharded_causal_conv1d_fn

    g = torch.Generator().manual_seed(9)
    x0 = torch.randn(2, 300, 256, generator=g).to(torch.bfloat16).to(DEV)
    w0 = (torch.randn(256, 4, generator=g) * 0.5).to(DEV)
    b0 = torch.randn(256, generator=g).to(DEV)
    i0 = torch.randn(2, 3, 256, generator=g).to(torch.bfloat16).to(DEV)
    dy = torch.randn(2, 300, 256, generator=g).to(torch.bfloat16).to(DEV)
    res = []
    for fn in (cc.causal_conv1d_fn, sharded_causal_conv1d_fn):
        x, w, b, i = (t.clone().requires_grad_(True) for t in (x0, w0, b0, i0))
        out = fn(x, w, b, initial_states=i, activation="silu")
        out.backward(dy)
        res.append([out, x.grad, w.grad, b.grad, i.grad])
    for a, c in zip(*res):
        assert torch.equal(a, c)


@pytest.mark.parametrize("x_layout", ["offset1", "row_pad1", "batch_gap"])
@pytest.mark.parametrize("dt,W", [(torch.bfloat16, 4), (torch.bfloat16, 8), (torch.float16, 12), (torch.float32, 4)])
def test_plain_load_forward_equals_tma(cc, x_layout, dt, W):
    """The forward on a layout a tensor map cannot describe (its tile filled with plain loads)
    gives the same bits as on a contiguous copy (tile filled by TMA): with initial and final
    states, and with seq_idx."""
    g = torch.Generator().manual_seed(W)
    B, T, D = 3, 200, 136
    x = torch.randn(B, T, D, generator=g).to(dt).to(DEV)
    w = (torch.randn(D, W, generator=g) / W**0.5).to(DEV)
    b = (torch.randn(D, generator=g) * 0.3).to(DEV)
    init = torch.randn(B, W - 1, D, generator=g).to(dt).to(DEV)
    seq = torch.cat([torch.zeros(B, 70), torch.ones(B, 100), torch.full((B, 30), -1.0)], 1).to(torch.int32).to(DEV)
    xv = layout(x, x_layout)
    with torch.no_grad():
        got = cc.causal_conv1d_fn(xv, w, b, initial_states=init, return_final_states=True, activation="silu")
        want = cc.causal_conv1d_fn(x, w, b, initial_states=init, return_final_states=True, activation="silu")
        assert torch.equal(got[0], want[0]) and torch.equal(got[1], want[1])
        got = cc.causal_conv1d_fn(xv, w, b, seq_idx=seq, initial_states=init, activation="silu")
        want = cc.causal_conv1d_fn(x, w, b, seq_idx=seq, initial_states=init, activation="silu")
        assert torch.equal(got, want)


def test_plain_load_forward_rows_of_8_bytes(cc):
    """D = 36 bf16 (72-byte rows: no tensor map, plain-load tile) against the oracle."""
    g = torch.Generator().manual_seed(36)
    B, T, D, W = 2, 150, 36, 4
    x = torch.randn(B, T, D, generator=g).to(torch.bfloat16)
    w = torch.randn(D, W, generator=g) * 0.5
    b = torch.randn(D, generator=g) * 0.3
    init = torch.randn(B, W - 1, D, generator=g).to(torch.bfloat16)
    with torch.no_grad():
        out, fin = cc.causal_conv1d_fn(x.to(DEV), w.to(DEV), b.to(DEV), initial_states=init.to(DEV),
                                       return_final_states=True, activation="silu")
    ro, rf = oracle.fwd(x, w, b, init, None, silu=True, return_final_states=True)
    assert_close(out.cpu(), torch.from_numpy(ro).to(torch.bfloat16).float(), torch.bfloat16, "out")
    assert_bitexact(fin.cpu().float(), torch.from_numpy(rf).to(torch.bfloat16).float(), "final_states")


CHUNK = [(torch.bfloat16, 36, 4), (torch.bfloat16, 100, 2), (torch.bfloat16, 100, 8), (torch.float16, 36, 12),
         (torch.float32, 34, 4)]


@pytest.mark.parametrize("dt,D,W", CHUNK, ids=[f"{str(d)[6:]}-D{D}-W{W}" for d, D, W in CHUNK])
@pytest.mark.parametrize("flags", ["bias_silu", "state_chain", "seq_init", "plain"])
def test_backward_8_byte_rows(cc, dt, D, W, flags):
    """Rows of 8-byte but not 16-byte multiples: no tensor map, the backward walk copies its stages
    in 8-byte cp.async chunks (and the forward fills its tile with plain loads)."""
    f = dict(has_bias=False, silu=False, has_init=False, has_seq=False, ret_final=False, dfinal=False,
             need_dinit=False)
    if flags == "bias_silu":
        f.update(has_bias=True, silu=True)
    elif flags == "state_chain":
        f.update(has_bias=True, silu=True, has_init=True, ret_final=True, dfinal=True, need_dinit=True)
    elif flags == "seq_init":
        f.update(has_bias=True, silu=True, has_init=True, has_seq=True, need_dinit=True)
    check_vs_oracle(cc, 3, 150, D, W, dt, seed=D + W + len(flags), **f)
