"""CUDA-graph capture of the forward and backward launches (the boundary's contract: no allocation
outside torch's graph pool, no host synchronisation inside a call).

1. The host launchers `_fwd` / `_bwd` are captured once on static buffers and replayed on new
   inputs copied into them; every output must equal an eager call on the same inputs bit for bit
   (the kernels are deterministic).
2. The public autograd path through `torch.cuda.make_graphed_callables`: the graphed forward and
   backward must equal the eager `causal_conv1d_fn` forward and backward bit for bit.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture
def status():
    from causal_conv1d_b200 import _native

    return lambda: _native.status(clear=True)


def _data(seed, B, T, D, W, init):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, D, generator=g).to(torch.bfloat16).cuda()
    dy = torch.randn(B, T, D, generator=g).to(torch.bfloat16).cuda()
    s = torch.randn(B, W - 1, D, generator=g).to(torch.bfloat16).cuda() if init else None
    return x, dy, s


@pytest.mark.parametrize("W,silu,init", [(4, True, True), (4, False, False), (8, True, False)])
def test_launchers_replay_equal_eager(status, W, silu, init):
    from causal_conv1d_b200.causal_conv1d import _bwd, _fwd

    B, T, D = 3, 1000, 384
    g = torch.Generator().manual_seed(1)
    w = (torch.randn(D, W, generator=g) * 0.5).cuda()
    b = (torch.randn(D, generator=g) * 0.3).cuda()
    sx, sdy, sinit = _data(2, B, T, D, W, init)
    sfinal = torch.empty(B, W - 1, D, device="cuda", dtype=torch.bfloat16)

    def step():
        out = _fwd(sx, w, b, None, sinit, sfinal, silu)
        return (out,) + _bwd(sx, w, b, None, sinit, sdy, None, init, silu)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static = step()

    for seed in (3, 4):
        x, dy, init_t = _data(seed, B, T, D, W, init)
        sx.copy_(x)
        sdy.copy_(dy)
        if init:
            sinit.copy_(init_t)
        graph.replay()
        torch.cuda.synchronize()
        final = torch.empty_like(sfinal)
        eager = (_fwd(x, w, b, None, init_t, final, silu),) + _bwd(x, w, b, None, init_t, dy, None, init, silu)
        torch.cuda.synchronize()
        for name, got, want in zip(("out", "dx", "dweight", "dbias", "dinit"), static, eager):
            if want is None:
                assert got is None, name
                continue
            assert torch.equal(got, want), f"{name} differs after graph replay (seed {seed})"
        assert torch.equal(sfinal, final), "final_states differ after graph replay"
    assert status() == 0


def test_make_graphed_callables_equal_eager(status):
    from causal_conv1d_b200 import causal_conv1d_fn

    B, T, D, W = 2, 777, 256, 4
    g = torch.Generator().manual_seed(5)
    w = (torch.randn(D, W, generator=g) * 0.5).cuda().requires_grad_(True)
    b = (torch.randn(D, generator=g) * 0.3).cuda().requires_grad_(True)

    def fn(x, w, b):
        return causal_conv1d_fn(x, w, b, activation="silu")

    x0, _, _ = _data(6, B, T, D, W, False)
    graphed = torch.cuda.make_graphed_callables(fn, (x0.requires_grad_(True), w, b))

    x, dy, _ = _data(7, B, T, D, W, False)
    xg = x.clone().requires_grad_(True)
    out_g = graphed(xg, w, b)
    out_g.backward(dy)
    grads_g = (xg.grad.clone(), w.grad.clone(), b.grad.clone())
    w.grad = b.grad = None

    xe = x.clone().requires_grad_(True)
    out_e = fn(xe, w, b)
    out_e.backward(dy)
    torch.cuda.synchronize()
    assert torch.equal(out_g, out_e)
    for name, got, want in zip(("dx", "dweight", "dbias"), grads_g, (xe.grad, w.grad, b.grad)):
        assert torch.equal(got, want), f"{name} differs between the graphed and eager calls"
    assert status() == 0
