"""The causal conv over the xBC slice of a Mamba-2 in_proj output, fused with the block's splits.

In a Mamba-2 block the in_proj output `zxbcdt` (batch, seqlen, d_in_proj) holds [z | xBC | dt]
along channels; the conv runs on xBC and its output is split into the SSM's x, B and C. Written
with torch.split around causal_conv1d_fn, the backward first concatenates the gradients of x, B and
C into one dout (a full read and write of xBC's size), then concatenates dz, dxBC and ddt into
d(zxbcdt) (another read and write of xBC's size, plus dz and ddt). `split_conv1d` does neither:
the conv backward reads the gradients of x, B and C where they lie (C entry cc1d_bwd_split) and
writes dxBC straight into its slice of d(zxbcdt), so only dz and ddt are copied in, with the
library's vectorised channel-block copy (cc1d_copy_channels; torch's element-wise copy into the
strided slice ran at 1.9 TB/s on B200). The forward reads xBC in place (its row stride is
d_in_proj) and returns z and dt as views of zxbcdt and x, B, C as views of the conv output, exactly
as the splits do.

The reference contains only the conv; its README names the Mamba block as the caller
(causal_conv1d_triton README.md:3-4). Every value equals the unfused composition bit for bit: the
same kernels compute the same elements, only where dout is read from and dx written to differs.
"""

from __future__ import annotations

from typing import Sequence

import torch
from torch import Tensor

from .causal_conv1d import _bwd_split, _check_inputs, _copy_channels, _fwd, _tma_layout


class _SplitConv1dFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, zxbcdt, weight, bias, seq_idx, initial_states, d_z, xbc_split, silu):
        d_xbc = sum(xbc_split)
        # A slice the TMA kernels cannot address is copied once, as causal_conv1d_fn does, and the
        # copy serves the backward too.
        xbc = _tma_layout(zxbcdt[..., d_z:d_z + d_xbc], weight.shape[1])
        out = _fwd(xbc, weight, bias, seq_idx, initial_states, None, silu)
        ctx.save_for_backward(zxbcdt, weight, bias, seq_idx, initial_states, xbc)
        ctx.d_z, ctx.xbc_split, ctx.silu = d_z, xbc_split, silu
        parts = out.split(list(xbc_split), dim=-1)
        return (zxbcdt[..., :d_z], *parts, zxbcdt[..., d_z + d_xbc:])

    @staticmethod
    def backward(ctx, dz, *grads):
        zxbcdt, weight, bias, seq_idx, initial_states, xbc = ctx.saved_tensors
        dparts, ddt = grads[:-1], grads[-1]
        d_z, split = ctx.d_z, ctx.xbc_split
        d_xbc = sum(split)
        B, T, d_in = zxbcdt.shape
        dzx = torch.empty(B, T, d_in, device=zxbcdt.device, dtype=zxbcdt.dtype)
        head, tail = dzx[..., :d_z], dzx[..., d_z + d_xbc:]
        for dst, g in ((head, dz), (tail, ddt)):
            if dst.shape[-1]:
                _copy_channels(dst, g) if g is not None else dst.zero_()
        pieces = []
        for g, w in zip(dparts, split):
            if g is None:
                g = torch.zeros(B, T, w, device=zxbcdt.device, dtype=zxbcdt.dtype)
            elif g.stride(-1) != 1:
                g = g.contiguous()
            pieces.append(g)
        need_dinit = initial_states is not None and ctx.needs_input_grad[4]
        dweight, dbias, dinit = _bwd_split(xbc, weight, bias, seq_idx, initial_states, pieces,
                                           need_dinit, ctx.silu, dzx[..., d_z:d_z + d_xbc])
        return (dzx, dweight, dbias if bias is not None else None, None,
                dinit if need_dinit else None, None, None, None)


def split_conv1d(zxbcdt: Tensor, weight: Tensor, bias: Tensor | None = None, *, d_z: int,
                 xbc_split: Sequence[int], seq_idx: Tensor | None = None,
                 initial_states: Tensor | None = None, activation: str | None = None):
    """Split `zxbcdt` = [z | xBC | dt] along channels, run the causal conv on xBC and split its
    output; returns (z, *xbc_parts, dt).

    zxbcdt: (batch, seqlen, d_in_proj), channel stride 1; z is channels [0, d_z), xBC the next
        sum(xbc_split) channels, dt the rest.
    weight, bias, seq_idx, initial_states, activation: as for causal_conv1d_fn over xBC
        (weight (sum(xbc_split), width)).
    Equal to
        z, xBC, dt = zxbcdt.split([d_z, sum(xbc_split), rest], -1)
        parts = causal_conv1d_fn(xBC, weight, bias, seq_idx, initial_states, activation=activation)
                .split(xbc_split, -1)
    in values and gradients, bit for bit; the backward skips both concatenations of the unfused
    form (module docstring).
    """
    if activation not in (None, "silu", "swish"):
        raise NotImplementedError("activation must be None, silu, or swish")
    assert zxbcdt.ndim == 3 and zxbcdt.stride(2) == 1, "zxbcdt must be (batch, seqlen, d_in_proj), channel stride 1"
    xbc_split = tuple(int(w) for w in xbc_split)
    d_xbc = sum(xbc_split)
    assert d_z >= 0 and all(w > 0 for w in xbc_split) and d_z + d_xbc <= zxbcdt.shape[2]
    xbc = zxbcdt[..., d_z:d_z + d_xbc]
    _check_inputs(xbc, weight, bias, seq_idx, initial_states)
    weight = weight.contiguous()
    bias = bias.contiguous() if bias is not None else None
    seq_idx = seq_idx.to(torch.int32).contiguous() if seq_idx is not None else None
    initial_states = initial_states.contiguous() if initial_states is not None else None
    return _SplitConv1dFn.apply(zxbcdt, weight, bias, seq_idx, initial_states, d_z, xbc_split,
                                activation is not None)
