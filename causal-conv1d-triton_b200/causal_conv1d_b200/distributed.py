"""Batch-sharded data parallelism for the causal conv1d (one process per GPU).

Rows of the batch are independent, so each rank runs the forward and backward on its own slice of
the batch with no exchange of activations. The only exchange is the weight/bias gradient: each
rank's backward writes its gradient as one fp32 vector [dweight (D, W) row-major, dbias (D)]
(`cc1d_bwd`'s `grad_f32` output), and one all-reduce (sum) over the process group combines it; over
NCCL on NVLink that is D * (W + 1) * 4 bytes per step (20 KB at D = 1024, W = 4).

The all-reduce either runs inside the conv's backward (the default: weight.grad / bias.grad are
complete when backward returns to the caller, and torch.autograd.grad works), or, with
`overlap_grad_reduce=True`, asynchronously on NCCL's stream while the rest of the backward pass
runs: the summed gradient is added to the leaf weight / bias .grad by a callback at the end of the
backward pass, as DistributedDataParallel does. The latter needs leaf parameters and
Tensor.backward / torch.autograd.backward (not torch.autograd.grad).

With `deterministic_grad_reduce=True` the sum is formed in a fixed order instead: the ranks'
vectors are all-gathered and every rank adds them in rank order, so the gradient has the same bits
on every rank and from run to run at a given world size, whichever algorithm the collective library
picks (world x the vector's bytes cross the links instead of about 2x).

The reference implementation has no distributed code; this is the data-parallel layer above its
`causal_conv1d_fn` (causal_conv1d_triton/causal_conv1d.py:579-639), with the same arguments.
"""

from __future__ import annotations

import contextlib

import torch
import torch.distributed as dist
from torch import Tensor


def shard_rows(batch: int, rank: int, world: int) -> slice:
    """Contiguous, balanced slice of `batch` rows owned by `rank` (the first batch % world ranks
    get one extra row)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return slice(start, start + base + (1 if rank < extra else 0))


def flat_grad_size(dim: int, width: int) -> int:
    """Length of the fp32 gradient vector [dweight (dim, width), dbias (dim)]."""
    return dim * (width + 1)


def _world(group) -> int:
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(group)
    return 1


def allreduce_flat_grad_(flat: Tensor, group=None) -> Tensor:
    """Sums the flat fp32 gradient vector over the ranks of `group`, in place."""
    if _world(group) > 1:
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    return flat


def gather_sum_flat_grad_(flat: Tensor, group=None, async_op: bool = False):
    """Sums the flat fp32 gradient vector over the ranks of `group` in rank order, in place:
    all-gathers the ranks' vectors, then flat = v_0 + v_1 + ... + v_{n-1} on every rank. Returns a
    function that completes the sum (after waiting for the gather when `async_op`); nothing may
    write `flat` before it is called."""
    world = _world(group)
    if world == 1:
        return lambda: flat
    parts = [torch.empty_like(flat) for _ in range(world)]
    work = dist.all_gather(parts, flat, group=group, async_op=async_op)

    def finish():
        if async_op:
            work.wait()
        flat.copy_(parts[0])
        for p in parts[1:]:
            flat.add_(p)
        return flat

    return finish


def split_flat_grad(flat: Tensor, dim: int, width: int, weight_dtype, bias_dtype=None):
    """(dweight (dim, width), dbias (dim) or None) from the flat vector, in the parameters' dtypes."""
    dweight = flat[: dim * width].view(dim, width)
    dweight = dweight if weight_dtype == torch.float32 else dweight.to(weight_dtype)
    dbias = None
    if bias_dtype is not None:
        dbias = flat[dim * width: dim * (width + 1)]
        dbias = dbias if bias_dtype == torch.float32 else dbias.to(bias_dtype)
    return dweight, dbias


def _accumulate(param: Tensor, grad: Tensor) -> None:
    if param.grad is None:
        param.grad = grad.detach().clone()
    else:
        param.grad.add_(grad)


def reduce_weight_grads(flat: Tensor, weight: Tensor, bias: Tensor | None, group=None,
                        deferred: bool = False, deterministic: bool = False):
    """The cross-rank sum of one conv's flat fp32 weight/bias gradient.

    deferred=False: all-reduces in place now and returns (dweight, dbias) for autograd to
    accumulate. deferred=True: starts the all-reduce asynchronously (on NCCL's stream for CUDA
    tensors, after the work already queued on the current stream) and returns (None, None); a
    callback queued on the running backward pass waits for it and adds the result to weight.grad
    / bias.grad (which must be leaves) once every other node of the pass has run. Must be called
    from inside a backward pass in that case. deterministic=True sums in rank order
    (gather_sum_flat_grad_) instead of all-reducing."""
    D, W = weight.shape
    bias_dtype = bias.dtype if bias is not None else None
    if not deferred:
        if deterministic:
            gather_sum_flat_grad_(flat, group)()
        else:
            allreduce_flat_grad_(flat, group)
        return split_flat_grad(flat, D, W, weight.dtype, bias_dtype)
    gather_fin, work = None, None
    if deterministic:
        gather_fin = gather_sum_flat_grad_(flat, group, async_op=True)
    elif _world(group) > 1:
        work = dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group, async_op=True)
    stream = torch.cuda.current_stream(flat.device) if flat.is_cuda else None

    def finish():
        with torch.cuda.stream(stream) if stream is not None else contextlib.nullcontext():
            if gather_fin is not None:
                gather_fin()  # waits for the gather, then adds in rank order
            if work is not None:
                work.wait()  # the current stream (or, on the CPU, the host) waits for the sum
            dweight, dbias = split_flat_grad(flat, D, W, weight.dtype, bias_dtype)
            _accumulate(weight, dweight)
            if bias is not None:
                _accumulate(bias, dbias)

    torch.autograd.Variable._execution_engine.queue_callback(finish)
    return None, None


class _ShardedFn(torch.autograd.Function):
    """causal_conv1d_fn on this rank's batch shard whose weight/bias gradients are the sum over all
    ranks (computed by the backward kernel as one fp32 vector and all-reduced once). Mirrors the
    reference's `_CausalConv1dFn` (causal_conv1d.py:544-576) otherwise."""

    @staticmethod
    def forward(ctx, x, weight, bias, seq_idx, initial_states, return_final_states, silu, group, overlap,
                deterministic):
        from .causal_conv1d import _fwd

        final_states = None
        if return_final_states:
            final_states = torch.empty(x.shape[0], weight.shape[1] - 1, x.shape[2], device=x.device,
                                       dtype=x.dtype)
        out = _fwd(x, weight, bias, seq_idx, initial_states, final_states, silu)
        ctx.save_for_backward(x, weight, bias, seq_idx, initial_states)
        ctx.silu, ctx.group, ctx.overlap, ctx.deterministic = silu, group, overlap, deterministic
        # The deferred reduce adds to these leaves' .grad after the backward pass.
        ctx.leaves = (weight, bias) if overlap else None
        ctx.return_final_states = return_final_states
        return (out, final_states) if return_final_states else out

    @staticmethod
    def backward(ctx, dout, *args):
        from .causal_conv1d import _bwd, _channels_contiguous, _tma_layout

        x, weight, bias, seq_idx, initial_states = ctx.saved_tensors
        dfinal_states = args[0] if ctx.return_final_states else None
        if dfinal_states is not None:
            dfinal_states = dfinal_states.contiguous()
        D, W = weight.shape
        flat = torch.empty(flat_grad_size(D, W), device=x.device, dtype=torch.float32)
        need_dinit = initial_states is not None and ctx.needs_input_grad[4]
        dout = _tma_layout(_channels_contiguous(dout), W)
        dx, _, _, dinit = _bwd(x, weight, bias, seq_idx, initial_states, dout, dfinal_states,
                               need_dinit, ctx.silu, grad_f32=flat)
        if ctx.overlap:
            weight, bias = ctx.leaves
        dweight, dbias = reduce_weight_grads(flat, weight, bias, ctx.group, deferred=ctx.overlap,
                                             deterministic=ctx.deterministic)
        if bias is None:
            dbias = None
        return dx, dweight, dbias, None, dinit, None, None, None, None, None


def sharded_causal_conv1d_fn(
    x: Tensor,
    weight: Tensor,
    bias: Tensor | None = None,
    seq_idx: Tensor | None = None,
    initial_states: Tensor | None = None,
    return_final_states: bool = False,
    final_states_out: Tensor | None = None,
    activation: str | None = None,
    group=None,
    overlap_grad_reduce: bool = False,
    deterministic_grad_reduce: bool = False,
) -> Tensor | tuple[Tensor, Tensor]:
    """Data-parallel causal_conv1d_fn. The arguments are the reference's (causal_conv1d.py:579-588)
    for this rank's rows: `x`, `seq_idx`, `initial_states` and `final_states_out` hold this rank's
    batch shard (see shard_rows), and the results are the shard's. After backward,
    weight.grad / bias.grad hold the gradient summed over every rank of `group` (identical on all
    ranks).

    overlap_grad_reduce: run the gradient all-reduce asynchronously and add its result to the leaf
    weight / bias .grad at the end of the backward pass (see the module docstring); requires leaf
    weight and bias.

    deterministic_grad_reduce: sum the ranks' gradients in rank order (all-gather, then add) so
    they have the same bits on every rank and in every run at a given world size."""
    from .causal_conv1d import _channels_contiguous, _check_inputs, _tma_layout

    if activation not in (None, "silu", "swish"):
        raise NotImplementedError("activation must be None, silu, or swish")
    if seq_idx is not None:
        assert not return_final_states, "cannot return final states if seq_idx is not None"
    if final_states_out is not None:
        assert return_final_states, "final_states_out requires return_final_states=True"
    _check_inputs(x, weight, bias, seq_idx, initial_states)

    x = _channels_contiguous(x)
    weight = weight.contiguous()
    bias = bias.contiguous() if bias is not None else None
    seq_idx = seq_idx.to(torch.int32).contiguous() if seq_idx is not None else None
    initial_states = initial_states.contiguous() if initial_states is not None else None
    silu = activation is not None
    if overlap_grad_reduce and not (weight.is_leaf and (bias is None or bias.is_leaf)):
        raise ValueError("overlap_grad_reduce needs contiguous leaf weight and bias tensors")

    needs_grad = torch.is_grad_enabled() and any(
        t is not None and t.requires_grad for t in (x, weight, bias, initial_states))
    if needs_grad:
        x = _tma_layout(x, weight.shape[1])
        result = _ShardedFn.apply(x, weight, bias, seq_idx, initial_states, return_final_states, silu,
                                  group, overlap_grad_reduce, deterministic_grad_reduce)
    else:
        from .causal_conv1d import _fwd

        final_states = None
        if return_final_states:
            final_states = torch.empty(x.shape[0], weight.shape[1] - 1, x.shape[2], device=x.device,
                                       dtype=x.dtype)
        out = _fwd(x, weight, bias, seq_idx, initial_states, final_states, silu)
        result = (out, final_states) if return_final_states else out
    if final_states_out is not None:
        out, final_states = result
        result = out, final_states_out.copy_(final_states)
    return result
