"""Batch-sharded data parallelism for the causal conv1d (one process per GPU).

Rows of the batch are independent, so each rank runs the forward and backward on its own slice of
the batch with no exchange of activations. The only exchange is the weight/bias gradient: each
rank's backward writes its gradient as one fp32 vector [dweight (D, W) row-major, dbias (D)]
(`cc1d_bwd`'s `grad_f32` output), and one all-reduce (sum) over the process group combines it; over
NCCL on NVLink that is D * (W + 1) * 4 bytes per step (20 KB at D = 1024, W = 4).

The reference implementation has no distributed code; this is the data-parallel layer above its
`causal_conv1d_fn` (causal_conv1d_triton/causal_conv1d.py:579-639).
"""

from __future__ import annotations

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


def allreduce_flat_grad_(flat: Tensor, group=None) -> Tensor:
    """Sums the flat fp32 gradient vector over the ranks of `group`, in place."""
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    return flat


def split_flat_grad(flat: Tensor, dim: int, width: int, weight_dtype, bias_dtype=None):
    """(dweight (dim, width), dbias (dim) or None) from the flat vector, in the parameters' dtypes."""
    dweight = flat[: dim * width].view(dim, width)
    dweight = dweight if weight_dtype == torch.float32 else dweight.to(weight_dtype)
    dbias = None
    if bias_dtype is not None:
        dbias = flat[dim * width: dim * (width + 1)]
        dbias = dbias if bias_dtype == torch.float32 else dbias.to(bias_dtype)
    return dweight, dbias


class _ShardedFn(torch.autograd.Function):
    """causal_conv1d_fn on this rank's batch shard whose weight/bias gradients are the sum over all
    ranks (computed by the backward kernel as one fp32 vector and all-reduced once)."""

    @staticmethod
    def forward(ctx, x, weight, bias, initial_states, silu, group):
        from .causal_conv1d import _fwd

        out = _fwd(x, weight, bias, None, initial_states, None, silu)
        ctx.save_for_backward(x, weight, bias, initial_states)
        ctx.silu, ctx.group = silu, group
        return out

    @staticmethod
    def backward(ctx, dout):
        from .causal_conv1d import _bwd, _channels_contiguous

        x, weight, bias, initial_states = ctx.saved_tensors
        D, W = weight.shape
        flat = torch.empty(flat_grad_size(D, W), device=x.device, dtype=torch.float32)
        need_dinit = initial_states is not None and ctx.needs_input_grad[3]
        dx, _, _, dinit = _bwd(x, weight, bias, None, initial_states, _channels_contiguous(dout),
                               None, need_dinit, ctx.silu, grad_f32=flat)
        allreduce_flat_grad_(flat, ctx.group)
        dweight, dbias = split_flat_grad(flat, D, W, weight.dtype,
                                         bias.dtype if bias is not None else None)
        return dx, dweight, dbias, dinit, None, None


def sharded_causal_conv1d_fn(x: Tensor, weight: Tensor, bias: Tensor | None = None,
                             initial_states: Tensor | None = None,
                             activation: str | None = None, group=None) -> Tensor:
    """Data-parallel causal_conv1d_fn: `x` is this rank's batch shard (see shard_rows); the
    returned output is the shard's output, and after backward weight.grad / bias.grad hold the
    gradient summed over every rank of `group` (identical on all ranks)."""
    from .causal_conv1d import _channels_contiguous, _check_inputs

    if activation not in (None, "silu", "swish"):
        raise NotImplementedError("activation must be None, silu, or swish")
    _check_inputs(x, weight, bias, None, initial_states)
    x = _channels_contiguous(x)
    weight = weight.contiguous()
    bias = bias.contiguous() if bias is not None else None
    initial_states = initial_states.contiguous() if initial_states is not None else None
    return _ShardedFn.apply(x, weight, bias, initial_states, activation is not None, group)
