"""Data-parallel path on 2 GPUs over NCCL: each rank runs its batch shard, and the all-reduced
weight/bias gradients must equal the single-GPU gradients of the whole batch (within the bf16
tolerance; the sum is grouped differently) and be identical on both ranks. Skipped with fewer than
two GPUs."""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    g = torch.Generator().manual_seed(4)
    B, T, D, W = 6, 2048, 512, 4
    return (torch.randn(B, T, D, generator=g).to(torch.bfloat16),
            (torch.randn(D, W, generator=g) * 0.5), torch.randn(D, generator=g) * 0.3,
            torch.randn(B, T, D, generator=g).to(torch.bfloat16))


def _worker(rank, world, port, out_dir, paths):
    import sys

    sys.path[:0] = paths
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    from causal_conv1d_b200.distributed import shard_rows, sharded_causal_conv1d_fn

    x, w, b, dy = _inputs()
    sl = shard_rows(x.shape[0], rank, world)
    xs = x[sl].to(dev).requires_grad_(True)
    wd, bd = w.to(dev).requires_grad_(True), b.to(dev).requires_grad_(True)
    out = sharded_causal_conv1d_fn(xs, wd, bd, activation="silu")
    out.backward(dy[sl].to(dev))
    torch.cuda.synchronize()
    torch.save({"dw": wd.grad.cpu(), "db": bd.grad.cpu(), "dx": xs.grad.cpu(), "out": out.detach().cpu()},
               os.path.join(out_dir, f"r{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_batch_shards_match_single_gpu(tmp_path):
    import sys

    from _tol import assert_close, assert_close_sum
    from causal_conv1d_b200 import causal_conv1d_fn

    paths = [p for p in sys.path if "repo" in p]
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path), paths), nprocs=2, join=True)
    r = [torch.load(tmp_path / f"r{i}.pt") for i in range(2)]
    assert torch.equal(r[0]["dw"], r[1]["dw"]) and torch.equal(r[0]["db"], r[1]["db"])

    x, w, b, dy = _inputs()
    dev = torch.device("cuda", 0)
    xd, wd, bd = x.to(dev).requires_grad_(True), w.to(dev).requires_grad_(True), b.to(dev).requires_grad_(True)
    out = causal_conv1d_fn(xd, wd, bd, activation="silu")
    out.backward(dy.to(dev))
    assert torch.equal(torch.cat([r[0]["out"], r[1]["out"]]), out.detach().cpu())
    assert torch.equal(torch.cat([r[0]["dx"], r[1]["dx"]]), xd.grad.cpu())
    assert_close_sum(r[0]["dw"], wd.grad, "bf16", "dweight")
    assert_close_sum(r[0]["db"], bd.grad, "bf16", "dbias")
