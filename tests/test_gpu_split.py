"""The conv fused with a Mamba-2 block's splits (split_conv1d; C entry cc1d_bwd_split).

split_conv1d(zxbcdt, ...) must equal the unfused composition
    z, xBC, dt = zxbcdt.split(...); parts = causal_conv1d_fn(xBC, ...).split(...)
in every output and every gradient, bit for bit: the same kernels compute the same elements; the
fused backward only reads the parts' gradients where they lie and writes dxBC into d(zxbcdt). The
fused results are also checked against the CPU oracle: the conv outputs and the xBC slice of
d(zxbcdt), dweight, dbias and dinit within the parity tolerance, the z and dt slices of d(zxbcdt)
equal to their upstream gradients.
Cases cover the TMA split path (piece boundaries on 128- or 64-channel blocks), seq_idx with
initial states, W = 8, fp32, and layouts outside the fast path (misaligned pieces, a row stride
that is not a 16-byte multiple), which fall back to concatenating. A direct C-ABI call checks that
aligned pieces really take the split path (return code 0, not CC1D_ERR_LAYOUT).
"""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"

CASES = {
    # name: (dtype, W, d_z, xbc_split, d_dt, silu, seq+init)
    "mamba2_bf16_silu": (torch.bfloat16, 4, 256, (256, 128, 128), 8, True, False),
    "bf16_no_activation": (torch.bfloat16, 4, 128, (192, 64, 64), 16, False, False),
    "seq_idx_and_init": (torch.bfloat16, 4, 64, (256, 128, 128), 8, True, True),
    "width8": (torch.bfloat16, 8, 128, (256, 128), 8, True, False),
    "fp32": (torch.float32, 4, 64, (128, 64, 64), 4, True, False),
    "misaligned_pieces": (torch.bfloat16, 4, 64, (200, 28, 28), 8, True, False),
    "odd_row_stride": (torch.bfloat16, 4, 64, (256, 128, 128), 7, True, False),
    "five_pieces": (torch.bfloat16, 4, 0, (128, 128, 128, 128, 128), 8, True, False),
}


def _inputs(dt, W, d_z, split, d_dt, seq, seed=0):
    g = torch.Generator().manual_seed(seed)
    B, T = 2, 300
    d_xbc = sum(split)
    zx = torch.randn(B, T, d_z + d_xbc + d_dt, generator=g).to(dt).to(DEV)
    w = (torch.randn(d_xbc, W, generator=g) * W**-0.5).to(DEV)
    b = (torch.randn(d_xbc, generator=g) * 0.3).to(DEV)
    seq_idx = init = None
    if seq:
        seq_idx = torch.cat([torch.zeros(B, 100), torch.ones(B, 150), torch.full((B, 50), -1.0)], 1)
        seq_idx = seq_idx.to(torch.int32).to(DEV)
        init = torch.randn(B, W - 1, d_xbc, generator=g).to(dt).to(DEV)
    return zx, w, b, seq_idx, init, g


@pytest.mark.parametrize("case", list(CASES))
def test_split_conv1d_equals_unfused(case):
    from causal_conv1d_b200 import causal_conv1d_fn
    from causal_conv1d_b200.split_conv1d import split_conv1d

    dt, W, d_z, split, d_dt, silu, seq = CASES[case]
    zx, w, b, seq_idx, init, g = _inputs(dt, W, d_z, split, d_dt, seq)
    d_xbc = sum(split)
    act = "silu" if silu else None

    def fused(zx, w, b, init):
        return split_conv1d(zx, w, b, d_z=d_z, xbc_split=split, seq_idx=seq_idx, initial_states=init,
                            activation=act)

    def unfused(zx, w, b, init):
        z, xbc, dtp = zx.split([d_z, d_xbc, d_dt], dim=-1)
        y = causal_conv1d_fn(xbc, w, b, seq_idx=seq_idx, initial_states=init, activation=act)
        return (z, *y.split(list(split), dim=-1), dtp)

    results = []
    upstream = None
    for fn in (fused, unfused):
        leaves = [t.detach().clone().requires_grad_(True) if t is not None else None for t in (zx, w, b, init)]
        outs = fn(*leaves)
        if upstream is None:
            upstream = [torch.randn(o.shape, generator=g).to(o.dtype).to(DEV) for o in outs]
        torch.autograd.backward(outs, upstream)
        results.append(([o.detach() for o in outs], [t.grad for t in leaves if t is not None]))
    (of, gf), (ou, gu) = results
    for i, (a, c) in enumerate(zip(of, ou)):
        assert torch.equal(a, c), f"output {i} differs"
    for i, (a, c) in enumerate(zip(gf, gu)):
        assert torch.equal(a, c), f"gradient {i} differs"

    # Against the oracle, on the conv's own input slice.
    from _tol import assert_close, assert_close_sum
    from oracle import oracle

    key = "f32" if dt == torch.float32 else "bf16"
    xbc = zx[..., d_z:d_z + d_xbc]
    ups = upstream[1:1 + len(split)]
    eo = oracle.fwd(xbc, w, b, init, seq_idx, silu=silu)
    assert_close(torch.cat(of[1:1 + len(split)], -1), eo, key, "conv output vs oracle")
    edx, edw, edb, edi = oracle.bwd(xbc, w, b, init, seq_idx, torch.cat(ups, -1), None,
                                    need_dinit=init is not None, silu=silu)
    dzx = gf[0]
    assert_close(dzx[..., d_z:d_z + d_xbc], edx, key, "dxBC vs oracle")
    assert torch.equal(dzx[..., :d_z], upstream[0]) and torch.equal(dzx[..., d_z + d_xbc:], upstream[-1])
    assert_close_sum(gf[1], edw, key, "dweight vs oracle")
    assert_close_sum(gf[2], edb, key, "dbias vs oracle")
    if init is not None:
        assert_close(gf[3], edi, key, "dinit vs oracle")
    from causal_conv1d_b200 import _native

    assert _native.status(clear=True) == 0


def test_aligned_pieces_take_the_split_path():
    """cc1d_bwd_split on aligned pieces returns 0 and matches cc1d_bwd on the concatenated dout."""
    from causal_conv1d_b200 import _native
    from causal_conv1d_b200.causal_conv1d import _bwd, _stream

    g = torch.Generator().manual_seed(9)
    B, T, D, W = 2, 500, 512, 4
    x = torch.randn(B, T, D, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(D, W, generator=g) * 0.5).to(DEV)
    b = (torch.randn(D, generator=g) * 0.3).to(DEV)
    pieces = [torch.randn(B, T, c, generator=g).to(torch.bfloat16).to(DEV) for c in (256, 128, 128)]
    dx_ref, dw_ref, db_ref, _ = _bwd(x, w, b, None, None, torch.cat(pieces, -1), None, False, True)

    wide = torch.zeros(B, T, D + 64, dtype=torch.bfloat16, device=DEV)  # dx written into a slice
    dx = wide[..., 32:32 + D]
    dw, db = torch.empty_like(w), torch.empty_like(b)
    lib = _native.lib
    ws = lib.cc1d_bwd_workspace_bytes(x.data_ptr(), x.stride(0), x.stride(1), pieces[0].data_ptr(),
                                      pieces[0].stride(0), pieces[0].stride(1), B, T, D, W, 2)
    work = torch.empty(max(1, ws // 4), device=DEV)
    arr = (_native.DoutPiece * 3)(*[_native.DoutPiece(p.data_ptr(), p.stride(0), p.stride(1), p.shape[2])
                                    for p in pieces])
    rc = lib.cc1d_bwd_split(x.data_ptr(), x.stride(0), x.stride(1), w.data_ptr(), b.data_ptr(), None, None,
                            arr, 3, None, dx.data_ptr(), dx.stride(0), dx.stride(1), dw.data_ptr(),
                            db.data_ptr(), None, None, work.data_ptr(), ws, B, T, D, W, 2, 0, 0, 0, 1,
                            _stream(x.device))
    assert rc == 0, lib.cc1d_error_string(rc)
    torch.cuda.synchronize()
    assert torch.equal(dx, dx_ref) and torch.equal(dw, dw_ref) and torch.equal(db, db_ref)
    assert (wide[..., :32] == 0).all() and (wide[..., 32 + D:] == 0).all(), "wrote outside the dx slice"


@pytest.mark.parametrize("dt,C,shift", [(torch.bfloat16, 4096, 0), (torch.bfloat16, 100, 3), (torch.float32, 64, 1),
                                        (torch.float16, 7, 1)])
def test_copy_channels(dt, C, shift):
    """cc1d_copy_channels equals an indexed copy, at 16-byte vectors and at narrower ones."""
    from causal_conv1d_b200.causal_conv1d import _copy_channels

    g = torch.Generator().manual_seed(C)
    B, T = 3, 37
    src = torch.randn(B, T, C + 5, generator=g).to(dt).to(DEV)[..., shift:shift + C]
    wide = torch.zeros(B, T, C + 9, dtype=dt, device=DEV)
    dst = wide[..., 2 + shift:2 + shift + C]
    _copy_channels(dst, src)
    torch.cuda.synchronize()
    assert torch.equal(dst, src)
    outside = torch.ones_like(wide, dtype=torch.bool)
    outside[..., 2 + shift:2 + shift + C] = False
    assert (wide[outside] == 0).all()
