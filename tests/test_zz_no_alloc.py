"""cc1d_bwd_noalloc: the backward for callers that cannot allocate device memory.

Such callers (a runtime that owns all of device memory in its own arena and must not call
cudaMalloc after start-up, a path where cudaMalloc/cudaFree could synchronise the device, or host
code that reaches the library only through its C ABI with no device allocator) cannot hand
cc1d_bwd a workspace. cc1d_bwd_noalloc keeps the partial sums in a fixed 8 MiB array inside the
library instead. This test calls it through the C ABI and checks it against cc1d_bwd (given a
workspace) on the same inputs, twice in a row, since every call reuses the same array. Both run
the same kernels with the same partial count and a fixed-order reduction, so the results must be
identical bit for bit. It also checks that the device's free memory does not change across a
call, that a problem too large for the array is refused before any device work, and that other
errors come back with cc1d_bwd's own codes.

The file name makes pytest collect it last, so a failure here comes after every other test ran.
It passes on its own in a fresh process as well as after the other tests.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
BF16 = 2
F32 = 0


def _p(t):
    return None if t is None else t.data_ptr()


def _inputs(seed, B=3, T=1000, D=384, W=4):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, D, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(D, W, generator=g) * 0.5).to(DEV)
    b = (torch.randn(D, generator=g) * 0.3).to(DEV)
    init = torch.randn(B, W - 1, D, generator=g).to(torch.bfloat16).to(DEV)
    dy = torch.randn(B, T, D, generator=g).to(torch.bfloat16).to(DEV)
    dfin = torch.randn(B, W - 1, D, generator=g).to(torch.bfloat16).to(DEV)
    return x, w, b, init, dy, dfin


def _outputs(x, w, b, init):
    return (torch.empty_like(x), torch.empty_like(w), torch.empty_like(b), torch.empty_like(init))


# A short walk (W = 4, 16-row stages) and one long enough for the warp-specialized W = 8 backward's
# 24-row stages (18 CTAs per channel group, each walking about 4460 rows; 5.1 MB of partials).
SHAPES = [(3, 1000, 384, 4), (2, 40000, 7936, 8)]


@pytest.mark.parametrize("shape", SHAPES, ids=["W4_short", "W8_long_walk"])
def test_noalloc_matches_workspace_backward_twice(shape):
    from causal_conv1d_b200 import _native

    lib = _native.lib
    stream = torch.cuda.current_stream().cuda_stream
    for seed in (1, 2):  # two calls in a row reuse the library's scratch array
        x, w, b, init, dy, dfin = _inputs(seed, *shape)
        B, T, D = x.shape
        W = w.shape[1]
        args_in = (x.data_ptr(), x.stride(0), x.stride(1), w.data_ptr(), b.data_ptr(),
                   init.data_ptr(), None, dy.data_ptr(), dy.stride(0), dy.stride(1),
                   dfin.data_ptr())

        ref = _outputs(x, w, b, init)
        n = lib.cc1d_bwd_workspace_bytes(x.data_ptr(), x.stride(0), x.stride(1), dy.data_ptr(),
                                         dy.stride(0), dy.stride(1), B, T, D, W, BF16)
        assert 0 < n <= 8 << 20
        ws = torch.empty(n // 4, device=DEV, dtype=torch.float32)
        rc = lib.cc1d_bwd(*args_in, *[_p(t) for t in ref], None, ws.data_ptr(), n,
                          B, T, D, W, BF16, F32, F32, BF16, 1, stream)
        assert rc == 0, lib.cc1d_error_string(rc)

        got = _outputs(x, w, b, init)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        rc = lib.cc1d_bwd_noalloc(*args_in, *[_p(t) for t in got], None,
                                  B, T, D, W, BF16, F32, F32, BF16, 1, stream)
        assert rc == 0, lib.cc1d_error_string(rc)
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free_before, "the call changed the device's free memory"

        for name, a, e in zip(("dx", "dweight", "dbias", "dinit"), got, ref):
            assert torch.equal(a, e), f"{name}: cc1d_bwd_noalloc differs from cc1d_bwd"


def test_noalloc_rejects_problems_above_its_scratch():
    from causal_conv1d_b200 import _native

    lib = _native.lib
    # Width 256 runs the generic backward, whose partials (P x 257 x 16384 fp32) exceed 8 MiB.
    B, T, D, W = 1, 64, 16384, 256
    x = torch.zeros(B, T, D, device=DEV, dtype=torch.bfloat16)
    dy = torch.zeros_like(x)
    w = torch.zeros(D, W, device=DEV)
    dx = torch.empty_like(x)
    dw = torch.empty_like(w)
    need = lib.cc1d_bwd_workspace_bytes(x.data_ptr(), x.stride(0), x.stride(1), dy.data_ptr(),
                                        dy.stride(0), dy.stride(1), B, T, D, W, BF16)
    assert need > 8 << 20
    rc = lib.cc1d_bwd_noalloc(x.data_ptr(), x.stride(0), x.stride(1), w.data_ptr(), None, None,
                              None, dy.data_ptr(), dy.stride(0), dy.stride(1), None, dx.data_ptr(),
                              dw.data_ptr(), None, None, None, B, T, D, W, BF16, F32, F32, F32, 0,
                              torch.cuda.current_stream().cuda_stream)
    assert rc == _native.CC1D_ERR_SCRATCH_LIMIT
    assert b"8 MiB" in lib.cc1d_error_string(rc)


def test_noalloc_returns_cc1d_bwd_error_codes():
    from causal_conv1d_b200 import _native

    lib = _native.lib
    B, T, D = 1, 16, 64
    x = torch.zeros(B, T, D, device=DEV, dtype=torch.bfloat16)
    dy = torch.zeros_like(x)
    dx = torch.empty_like(x)
    stream = torch.cuda.current_stream().cuda_stream
    for W, want in ((257, _native.CC1D_ERR_UNSUPPORTED), (1, _native.CC1D_ERR_INVALID)):
        w = torch.zeros(D, max(W, 1), device=DEV)
        dw = torch.empty_like(w)
        rc = lib.cc1d_bwd_noalloc(x.data_ptr(), x.stride(0), x.stride(1), w.data_ptr(), None, None,
                                  None, dy.data_ptr(), dy.stride(0), dy.stride(1), None,
                                  dx.data_ptr(), dw.data_ptr(), None, None, None, B, T, D, W,
                                  BF16, F32, F32, F32, 0, stream)
        ws = torch.empty(1024, device=DEV)
        rc_ws = lib.cc1d_bwd(x.data_ptr(), x.stride(0), x.stride(1), w.data_ptr(), None, None,
                             None, dy.data_ptr(), dy.stride(0), dy.stride(1), None, dx.data_ptr(),
                             dw.data_ptr(), None, None, None, ws.data_ptr(), 4096, B, T, D, W,
                             BF16, F32, F32, F32, 0, stream)
        assert rc == want == rc_ws, (W, rc, rc_ws)
