"""torch.library registration of the causal conv1d, for torch.compile and other graph tracers.

`causal_conv1d_b200::fwd` and `causal_conv1d_b200::bwd` wrap the same host launchers as
causal_conv1d_fn (and so the same C ABI and CUDA kernels). Each has a fake (meta) implementation for
shape propagation, and fwd's autograd formula calls bwd, so a traced graph keeps the op opaque and
differentiable. Absent optional outputs are returned as empty tensors, since custom ops return
tensors only. The reference notes dynamo compatibility as a concern of its host code
(causal_conv1d_triton/causal_conv1d.py:390); this module is the registration it does not have.
"""

from __future__ import annotations

import torch
from torch import Tensor

from .causal_conv1d import _bwd, _channels_contiguous, _check_inputs, _fwd


@torch.library.custom_op("causal_conv1d_b200::fwd", mutates_args=())
def fwd_op(x: Tensor, weight: Tensor, bias: Tensor | None, seq_idx: Tensor | None,
           initial_states: Tensor | None, return_final_states: bool, silu: bool
           ) -> tuple[Tensor, Tensor]:
    final = None
    if return_final_states:
        final = torch.empty(x.shape[0], weight.shape[1] - 1, x.shape[2], device=x.device,
                            dtype=x.dtype)
    out = _fwd(x, weight, bias, seq_idx, initial_states, final, silu)
    return out, final if final is not None else x.new_empty(0)


@fwd_op.register_fake
def _(x, weight, bias, seq_idx, initial_states, return_final_states, silu):
    out = torch.empty_like(x, memory_format=torch.contiguous_format)
    if return_final_states:
        final = x.new_empty(x.shape[0], weight.shape[1] - 1, x.shape[2])
    else:
        final = x.new_empty(0)
    return out, final


@torch.library.custom_op("causal_conv1d_b200::bwd", mutates_args=())
def bwd_op(x: Tensor, weight: Tensor, bias: Tensor | None, seq_idx: Tensor | None,
           initial_states: Tensor | None, dout: Tensor, dfinal_states: Tensor | None,
           need_dinit: bool, silu: bool) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    # Outputs of a custom op may not alias one another: separate weight / bias gradient buffers.
    dx, dweight, dbias, dinit = _bwd(x, weight, bias, seq_idx, initial_states,
                                     _channels_contiguous(dout), dfinal_states, need_dinit, silu,
                                     fuse_param_grads=False)
    return (dx, dweight, dbias if dbias is not None else x.new_empty(0),
            dinit if dinit is not None else x.new_empty(0))


@bwd_op.register_fake
def _(x, weight, bias, seq_idx, initial_states, dout, dfinal_states, need_dinit, silu):
    dx = torch.empty_like(x, memory_format=torch.contiguous_format)
    dweight = torch.empty_like(weight)
    dbias = torch.empty_like(bias) if bias is not None else x.new_empty(0)
    dinit = torch.empty_like(initial_states) if need_dinit else x.new_empty(0)
    return dx, dweight, dbias, dinit


def _setup_context(ctx, inputs, output):
    x, weight, bias, seq_idx, initial_states, return_final_states, silu = inputs
    ctx.save_for_backward(x, weight, bias, seq_idx, initial_states)
    ctx.return_final_states, ctx.silu = return_final_states, silu


def _backward(ctx, dout, dfinal):
    x, weight, bias, seq_idx, initial_states = ctx.saved_tensors
    dfinal = dfinal.contiguous() if ctx.return_final_states and dfinal is not None else None
    need_dinit = initial_states is not None and ctx.needs_input_grad[4]
    dx, dweight, dbias, dinit = bwd_op(x, weight, bias, seq_idx, initial_states, dout, dfinal,
                                       need_dinit, ctx.silu)
    return (dx, dweight, dbias if bias is not None else None, None,
            dinit if need_dinit else None, None, None)


fwd_op.register_autograd(_backward, setup_context=_setup_context)


def causal_conv1d_fn_op(x: Tensor, weight: Tensor, bias: Tensor | None = None,
                        seq_idx: Tensor | None = None, initial_states: Tensor | None = None,
                        return_final_states: bool = False, activation: str | None = None):
    """causal_conv1d_fn through the registered custom op (traceable by torch.compile).

    Same arguments and results as causal_conv1d_fn except final_states_out, which a functional op
    cannot write; copy the returned final states instead.
    """
    if activation not in (None, "silu", "swish"):
        raise NotImplementedError("activation must be None, silu, or swish")
    if seq_idx is not None:
        assert not return_final_states, "cannot return final states if seq_idx is not None"
    _check_inputs(x, weight, bias, seq_idx, initial_states)
    x = _channels_contiguous(x)
    weight = weight.contiguous()
    bias = bias.contiguous() if bias is not None else None
    seq_idx = seq_idx.to(torch.int32).contiguous() if seq_idx is not None else None
    initial_states = initial_states.contiguous() if initial_states is not None else None
    out, final = fwd_op(x, weight, bias, seq_idx, initial_states, return_final_states,
                        activation is not None)
    return (out, final) if return_final_states else out
