"""Host logic of the batch-sharded data-parallel path, with gloo ranks on the CPU (no GPU).

Each of 2 ranks takes its shard of the batch (shard_rows), computes its weight/bias gradient with
the CPU oracle as the flat fp32 vector [dweight (D, W), dbias (D)] the backward kernel writes,
all-reduces it (allreduce_flat_grad_) and splits it (split_flat_grad); the result must equal the
oracle's gradient over the whole batch on every rank. A rank that raises leaves the others with an
error from the process group instead of a hang.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_rows_cover_batch_exactly():
    from causal_conv1d_b200.distributed import shard_rows

    for batch in (1, 2, 7, 8, 64, 65):
        for world in (1, 2, 3, 4, 8):
            got = [shard_rows(batch, r, world) for r in range(world)]
            rows = [i for s in got for i in range(s.start, s.stop)]
            assert rows == list(range(batch))
            sizes = [s.stop - s.start for s in got]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_rows(8, 2, 2)


def test_split_flat_grad_layout():
    from causal_conv1d_b200.distributed import flat_grad_size, split_flat_grad

    D, W = 5, 3
    flat = torch.arange(flat_grad_size(D, W), dtype=torch.float32)
    dw, db = split_flat_grad(flat, D, W, torch.float32, torch.bfloat16)
    assert dw.shape == (D, W) and dw[1, 2].item() == 5.0
    assert db.dtype == torch.bfloat16 and db[0].item() == 15.0
    dw2, db2 = split_flat_grad(flat, D, W, torch.float16, None)
    assert dw2.dtype == torch.float16 and db2 is None


def _worker(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import sys

    sys.path[:0] = [p for p in os.environ["CC1D_TEST_PATHS"].split(os.pathsep)]
    from causal_conv1d_b200.distributed import (allreduce_flat_grad_, flat_grad_size, shard_rows,
                                                split_flat_grad)
    from oracle import oracle

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    g = torch.Generator().manual_seed(0)
    B, T, D, W = 5, 40, 24, 4
    x = torch.randn(B, T, D, generator=g)
    w = torch.randn(D, W, generator=g) * 0.5
    b = torch.randn(D, generator=g) * 0.3
    dy = torch.randn(B, T, D, generator=g)
    sl = shard_rows(B, rank, world)
    _, dw, db, _ = oracle.bwd(x[sl], w, b, None, None, dy[sl], None, False, silu=True)
    flat = torch.from_numpy(np.concatenate([dw.reshape(-1), db]))
    assert flat.numel() == flat_grad_size(D, W)
    allreduce_flat_grad_(flat)
    dweight, dbias = split_flat_grad(flat, D, W, torch.float32, torch.float32)
    _, rdw, rdb, _ = oracle.bwd(x, w, b, None, None, dy, None, False, silu=True)
    np.testing.assert_allclose(dweight.numpy(), rdw, rtol=1e-5, atol=1e-5 * np.abs(rdw).max())
    np.testing.assert_allclose(dbias.numpy(), rdb, rtol=1e-5, atol=1e-5 * np.abs(rdb).max())
    torch.save({"dw": dweight, "db": dbias}, os.path.join(result_dir, f"r{rank}.pt"))
    dist.destroy_process_group()


def _paths():
    tests = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(tests)
    return os.pathsep.join([tests, root, os.path.join(root, "causal-conv1d-triton_b200")])


def test_gloo_two_ranks_match_full_batch(tmp_path):
    os.environ["CC1D_TEST_PATHS"] = _paths()
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    r0, r1 = torch.load(tmp_path / "r0.pt"), torch.load(tmp_path / "r1.pt")
    assert torch.equal(r0["dw"], r1["dw"]) and torch.equal(r0["db"], r1["db"])


def _failing_worker(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        raise RuntimeError("rank 1 fails before its all-reduce")
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
    except Exception:
        return  # the surviving rank sees an error, not a hang
    raise AssertionError("all_reduce with a dead peer should have failed")


def test_gloo_dead_rank_raises_instead_of_hanging():
    with pytest.raises(Exception):
        mp.spawn(_failing_worker, args=(2, _free_port()), nprocs=2, join=True)


def _oracle_fn_class():
    """An autograd Function that stands in for the sharded conv on the CPU: its backward computes
    this rank's flat [dweight, dbias] with the oracle and hands it to reduce_weight_grads, the
    same call the CUDA path makes."""
    from causal_conv1d_b200.distributed import reduce_weight_grads
    from oracle import oracle

    class OracleShardFn(torch.autograd.Function):
        @staticmethod
        def forward(ctx, x, weight, bias, seq, init, deferred, deterministic=False):
            ctx.save_for_backward(x, weight, bias, seq, init)
            ctx.deferred, ctx.deterministic = deferred, deterministic
            ctx.leaves = (weight, bias)
            return torch.from_numpy(oracle.fwd(x, weight, bias, init, seq, silu=True))

        @staticmethod
        def backward(ctx, dout):
            x, weight, bias, seq, init = ctx.saved_tensors
            dx, dw, db, dinit = oracle.bwd(x, weight, bias, init, seq, dout, None,
                                           need_dinit=init is not None, silu=True)
            flat = torch.from_numpy(np.concatenate([dw.reshape(-1), db]))
            w_leaf, b_leaf = ctx.leaves
            if ctx.deterministic:
                torch.save(flat.clone(), os.path.join(os.environ["CC1D_TEST_OUT"],
                                                      f"flat{dist.get_rank()}_{int(ctx.deferred)}.pt"))
            gw, gb = reduce_weight_grads(flat, w_leaf, b_leaf, deferred=ctx.deferred,
                                         deterministic=ctx.deterministic)
            gi = torch.from_numpy(dinit) if dinit is not None else None
            return torch.from_numpy(dx), gw, gb, None, gi, None, None

    return OracleShardFn


def _varlen_inputs():
    g = torch.Generator().manual_seed(7)
    B, T, D, W = 5, 64, 16, 4
    x = torch.randn(B, T, D, generator=g)
    w = torch.randn(D, W, generator=g) * 0.5
    b = torch.randn(D, generator=g) * 0.3
    init = torch.randn(B, W - 1, D, generator=g)
    seq = torch.zeros(B, T, dtype=torch.int32)
    for r in range(B):
        cut = int(torch.randint(8, 40, (1,), generator=g))
        seq[r, cut:] = 1
        seq[r, T - 3 - r:] = -1  # padding tail
    dy = torch.randn(B, T, D, generator=g)
    return x, w, b, init, seq, dy


def _deferred_worker(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import sys

    sys.path[:0] = [p for p in os.environ["CC1D_TEST_PATHS"].split(os.pathsep)]
    from causal_conv1d_b200.distributed import shard_rows

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    Fn = _oracle_fn_class()
    x, w, b, init, seq, dy = _varlen_inputs()
    sl = shard_rows(x.shape[0], rank, world)
    res = {}
    for deferred in (False, True):
        wl, bl = w.clone().requires_grad_(True), b.clone().requires_grad_(True)
        il = init[sl].clone().requires_grad_(True)
        out = Fn.apply(x[sl], wl, bl, seq[sl], il, deferred)
        # A second use of the weight after the conv: its gradient must add to the reduced one.
        loss = (out * dy[sl]).sum() + (wl * 2.0).sum()
        loss.backward()
        res[deferred] = (wl.grad.clone(), bl.grad.clone(), il.grad.clone())
    torch.save(res, os.path.join(result_dir, f"d{rank}.pt"))
    dist.destroy_process_group()


def test_gloo_deferred_reduce_equals_immediate_on_packed_shards(tmp_path):
    """Packed variable-length rows (seq_idx with padding, initial states) sharded over 2 gloo
    ranks: the all-reduced weight/bias gradient equals the oracle's over the whole batch, both
    when reduced inside the backward and when deferred to the end of the backward pass."""
    from oracle import oracle

    os.environ["CC1D_TEST_PATHS"] = _paths()
    mp.spawn(_deferred_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    r = [torch.load(tmp_path / f"d{i}.pt") for i in range(2)]
    x, w, b, init, seq, dy = _varlen_inputs()
    _, rdw, rdb, rdi = oracle.bwd(x, w, b, init, seq, dy, None, need_dinit=True, silu=True)
    for rank in range(2):
        for deferred in (False, True):
            gw, gb, gi = r[rank][deferred]
            np.testing.assert_allclose(gw.numpy(), rdw + 2.0, rtol=1e-5, atol=1e-5 * np.abs(rdw).max())
            np.testing.assert_allclose(gb.numpy(), rdb, rtol=1e-5, atol=1e-5 * np.abs(rdb).max())
        assert torch.equal(r[rank][False][0], r[rank][True][0])
    # Each rank's dinit is its own rows' (no exchange).
    np.testing.assert_allclose(torch.cat([r[0][True][2], r[1][True][2]]).numpy(), rdi, rtol=1e-5, atol=1e-5)


def _deterministic_worker(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), CC1D_TEST_OUT=result_dir)
    import datetime
    import sys

    sys.path[:0] = [p for p in os.environ["CC1D_TEST_PATHS"].split(os.pathsep)]
    from causal_conv1d_b200.distributed import shard_rows

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    Fn = _oracle_fn_class()
    x, w, b, init, seq, dy = _varlen_inputs()
    sl = shard_rows(x.shape[0], rank, world)
    res = {}
    for deferred in (False, True):
        wl, bl = w.clone().requires_grad_(True), b.clone().requires_grad_(True)
        il = init[sl].clone().requires_grad_(True)
        out = Fn.apply(x[sl], wl, bl, seq[sl], il, deferred, True)
        (out * dy[sl]).sum().backward()
        res[deferred] = (wl.grad.clone(), bl.grad.clone())
    torch.save(res, os.path.join(result_dir, f"det{rank}.pt"))
    dist.destroy_process_group()


def test_gloo_deterministic_reduce_sums_in_rank_order(tmp_path):
    """deterministic=True: every rank's weight/bias gradient is exactly v_0 + v_1 + v_2 (the ranks'
    own flat vectors added in rank order), the same bits on every rank, immediate and deferred,
    and within tolerance of the oracle's full-batch gradient; 3 ranks, uneven shards."""
    from oracle import oracle

    world = 3
    os.environ["CC1D_TEST_PATHS"] = _paths()
    mp.spawn(_deterministic_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    x, w, b, init, seq, dy = _varlen_inputs()
    _, rdw, rdb, _ = oracle.bwd(x, w, b, init, seq, dy, None, need_dinit=True, silu=True)
    D, W = w.shape
    for deferred in (False, True):
        v = [torch.load(tmp_path / f"flat{r}_{int(deferred)}.pt") for r in range(world)]
        want = v[0].clone()
        for p in v[1:]:
            want += p
        for r in range(world):
            gw, gb = torch.load(tmp_path / f"det{r}.pt")[deferred]
            assert torch.equal(gw.reshape(-1), want[: D * W]) and torch.equal(gb, want[D * W:])
        np.testing.assert_allclose(gw.numpy(), rdw, rtol=1e-5, atol=1e-5 * np.abs(rdw).max())
        np.testing.assert_allclose(gb.numpy(), rdb, rtol=1e-5, atol=1e-5 * np.abs(rdb).max())
