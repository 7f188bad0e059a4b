"""The data-parallel wrapper on a single GPU: two ranks over gloo share cuda:0, each running its batch
shard through sharded_causal_conv1d_fn (plain, with the all-reduce deferred to the end of the
backward pass, and with the rank-order sum). Each shard's out, dx and dinit must equal the
single-process full-batch results bit for bit, and the weight/bias gradients must be identical on
both ranks and within the bf16 sum tolerance of the full-batch ones.

This covers the sharded path's host logic and its CUDA kernels where only one GPU is available
(tests/test_multi_gpu.py runs the same over NCCL on two GPUs). The ranks exchange only host-side
gloo messages; no kernel waits on another process.
"""

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
MODES = (("plain", {}), ("deferred", {"overlap_grad_reduce": True}),
         ("rank_order", {"deterministic_grad_reduce": True}))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    g = torch.Generator().manual_seed(4)
    B, T, D, W = 4, 2048, 512, 4
    x = torch.randn(B, T, D, generator=g).to(torch.bfloat16)
    w = torch.randn(D, W, generator=g) * 0.5
    b = torch.randn(D, generator=g) * 0.3
    dy = torch.randn(B, T, D, generator=g).to(torch.bfloat16)
    init = torch.randn(B, W - 1, D, generator=g).to(torch.bfloat16)
    return x, w, b, dy, init


def _run(fn, sl, **kw):
    x, w, b, dy, init = _inputs()
    dev = torch.device("cuda", 0)
    xs = x[sl].to(dev).requires_grad_(True)
    wd = w.to(dev).requires_grad_(True)
    bd = b.to(dev).requires_grad_(True)
    ini = init[sl].to(dev).requires_grad_(True)
    out = fn(xs, wd, bd, initial_states=ini, activation="silu", **kw)
    out.backward(dy[sl].to(dev))
    torch.cuda.synchronize()
    return dict(out=out.detach().cpu(), dx=xs.grad.cpu(), dw=wd.grad.cpu(), db=bd.grad.cpu(),
                dinit=ini.grad.cpu())


def _worker(rank, world, port, out_dir):
    import sys

    sys.path[:0] = PATHS
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(0)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from causal_conv1d_b200.distributed import shard_rows, sharded_causal_conv1d_fn

    res = {name: _run(sharded_causal_conv1d_fn, shard_rows(4, rank, world), **kw) for name, kw in MODES}
    torch.save(res, os.path.join(out_dir, f"r{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_on_one_gpu_match_single_process(tmp_path):
    from _tol import assert_close_sum
    from causal_conv1d_b200 import causal_conv1d_fn

    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    full = _run(causal_conv1d_fn, slice(None))
    r = [torch.load(tmp_path / f"r{i}.pt") for i in range(2)]
    for name, _ in MODES:
        a, c = r[0][name], r[1][name]
        assert torch.equal(a["dw"], c["dw"]) and torch.equal(a["db"], c["db"]), name
        for k in ("out", "dx", "dinit"):
            assert torch.equal(torch.cat([a[k], c[k]]), full[k]), f"{name}: {k}"
        assert_close_sum(a["dw"], full["dw"], "bf16", f"{name}: dweight")
        assert_close_sum(a["db"], full["db"], "bf16", f"{name}: dbias")
