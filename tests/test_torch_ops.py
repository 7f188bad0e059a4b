"""torch.library registration (causal_conv1d_b200.torch_ops).

CPU: the fake (meta) implementations give the shapes and dtypes the real kernels produce, so graph
tracers can propagate shapes without a GPU. GPU: torch.library.opcheck on the registered ops, and a
torch.compile'd (aot_eager) forward + backward through the op equals the eager causal_conv1d_fn.
"""

import pytest
import torch


def test_fake_shapes_on_meta():
    import causal_conv1d_b200.torch_ops  # noqa: F401  (registers the ops)

    B, T, D, W = 2, 17, 24, 4
    x = torch.empty(B, T, D, device="meta", dtype=torch.bfloat16)
    w = torch.empty(D, W, device="meta")
    b = torch.empty(D, device="meta")
    init = torch.empty(B, W - 1, D, device="meta", dtype=torch.bfloat16)
    out, final = torch.ops.causal_conv1d_b200.fwd(x, w, b, None, init, True, True)
    assert out.shape == (B, T, D) and out.dtype == torch.bfloat16
    assert final.shape == (B, W - 1, D) and final.dtype == torch.bfloat16
    out, final = torch.ops.causal_conv1d_b200.fwd(x, w, None, None, None, False, False)
    assert final.numel() == 0
    dx, dw, db, di = torch.ops.causal_conv1d_b200.bwd(x, w, b, None, init, x, None, True, True)
    assert dx.shape == x.shape and dw.shape == w.shape and db.shape == b.shape
    assert di.shape == init.shape and di.dtype == init.dtype


@pytest.mark.gpu
def test_opcheck_and_compile():
    from causal_conv1d_b200 import causal_conv1d_fn
    from causal_conv1d_b200.torch_ops import bwd_op, causal_conv1d_fn_op, fwd_op

    dev = "cuda:0"
    g = torch.Generator().manual_seed(5)
    B, T, D, W = 2, 200, 128, 4
    x = torch.randn(B, T, D, generator=g).to(torch.bfloat16).to(dev)
    w = (torch.randn(D, W, generator=g) * 0.5).to(dev)
    b = torch.randn(D, generator=g).to(dev)
    init = torch.randn(B, W - 1, D, generator=g).to(torch.bfloat16).to(dev)
    dy = torch.randn(B, T, D, generator=g).to(torch.bfloat16).to(dev)

    torch.library.opcheck(fwd_op, (x, w, b, None, init, True, True),
                          test_utils=("test_schema", "test_faketensor", "test_aot_dispatch_static"))
    torch.library.opcheck(bwd_op, (x, w, b, None, init, dy, None, True, True),
                          test_utils=("test_schema", "test_faketensor"))

    def run(fn):
        xs, ws, bs, i_s = (t.clone().requires_grad_(True) for t in (x, w, b, init))
        out, final = fn(xs, ws, bs, initial_states=i_s, return_final_states=True, activation="silu")
        (out.float() * dy.float()).sum().backward()
        return out, final, xs.grad, ws.grad, bs.grad, i_s.grad

    eager = run(causal_conv1d_fn)
    compiled = run(torch.compile(causal_conv1d_fn_op, backend="aot_eager", fullgraph=True))
    for a, c in zip(eager, compiled):
        assert torch.equal(a, c)
