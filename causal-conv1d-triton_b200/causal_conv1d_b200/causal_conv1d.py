"""Causal depthwise conv1d over channels-last inputs, with forward and backward, on B200 (sm_100a).

    out[b, t, d] = act(bias[d] + sum_k weight[d, k] * x[b, t - (W - 1) + k, d])

where positions t < 0 read `initial_states` (or zero). A drop-in replacement for
jxiong21029/causal-conv1d-triton's `causal_conv1d_fn` (causal_conv1d_triton/causal_conv1d.py:579-639):
same signature, argument meaning, asserts and return values. x is (batch, seqlen, dim) and the
states are (batch, width - 1, dim): the inputs preceding x[:, 0]. Any width >= 2 (up to 256);
fp32/fp16/bf16 inputs, fp32 accumulation.

The kernels are hand-written CUDA for sm_100a behind the C ABI of include/causal_conv1d_b200.h,
called through the package's bindings (`_native`: ctypes, a CPython binding of the hot entry
points, and torch-side forward/backward launchers in C++). This module keeps the host-side logic of
the reference: the argument checks and the empty-input cases. Its autograd Function is C++
(`ConvFn` in csrc/cc1d_torch_ext.cpp), which spares each call the Python Function machinery.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _native
from ._native import DTYPE_CODE, check, fast, lib, tex

_FLOAT = (torch.float32, torch.float16, torch.bfloat16)


def _check_inputs(x, weight, bias, seq_idx, initial_states):
    """The reference's shape/device asserts (causal_conv1d.py:397-408)."""
    assert x.ndim == 3, "x must be (batch, seqlen, dim)"
    B, T, D = x.shape
    assert weight.ndim == 2 and weight.shape[0] == D, "weight must be (dim, width)"
    W = weight.shape[1]
    assert W >= 2, "width must be >= 2"
    assert x.is_cuda and weight.device == x.device
    assert bias is None or bias.shape == (D,)
    assert initial_states is None or initial_states.shape == (B, W - 1, D)
    assert seq_idx is None or seq_idx.shape == (B, T)
    # The reference computes offsets within one batch element in int32; the same inputs are
    # rejected here so that both accept exactly the same calls.
    assert (T + W) * max(x.stride(1), D) < 2**31


def _channels_contiguous(t: Tensor) -> Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


def _tma_layout(t: Tensor, width: int) -> Tensor:
    """`t` itself, or a fresh contiguous copy when its base or batch/time strides are not the
    16-byte multiples the TMA kernels need while its rows are (channels x element size a multiple of
    16 bytes) and the width is one those kernels cover (<= 16), e.g. a column slice at an odd
    offset. The copy is one pass over t; the per-element generic kernels it avoids ran ~5x slower on
    B200 (B=8 T=8192 D=1024 W=4 bf16, forward + backward). Differentiable (a clone)."""
    B, T, D = t.shape
    es = t.element_size()
    if width > 16 or (D * es) % 16 != 0 or t.numel() == 0:
        return t
    aligned = (t.data_ptr() % 16 == 0 and (t.stride(1) * es) % 16 == 0
               and (B == 1 or (t.stride(0) * es) % 16 == 0))
    return t if aligned else t.clone(memory_format=torch.contiguous_format)


def _as_float(t: Tensor | None) -> Tensor | None:
    """Parameters in a float type the kernels do not read (e.g. float64) are passed as fp32."""
    if t is None or t.dtype in _FLOAT:
        return t
    return t.float()


def _ptr(t: Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _code(t: Tensor | None) -> int:
    return 0 if t is None else DTYPE_CODE[t.dtype]


# torch's current raw stream and device through its C bindings when present (a fraction of a
# microsecond, against several for torch.cuda.current_stream / current_device, which matters for
# the small shapes where every call is host-bound).
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)
_raw_device = getattr(torch._C, "_cuda_getDevice", None)


def _stream(device) -> int:
    if _raw_stream is not None:
        return _raw_stream(device.index)
    return torch.cuda.current_stream(device).cuda_stream


def _current_device() -> int:
    return _raw_device() if _raw_device is not None else torch.cuda.current_device()


class _DeviceGuard:
    """Makes `device` current for the C calls, which launch on the current device (the reference
    launches under torch.cuda.device(x.device), causal_conv1d.py:448)."""

    __slots__ = ("idx", "prev")

    def __init__(self, device):
        self.idx = device.index

    def __enter__(self):
        self.prev = _current_device()
        if self.prev != self.idx:
            torch.cuda.set_device(self.idx)

    def __exit__(self, *exc):
        if self.prev != self.idx:
            torch.cuda.set_device(self.prev)


def _fwd(x, weight, bias, seq_idx, initial_states, final_states, silu):
    """Host launcher of the forward (the reference's `_fwd`, causal_conv1d.py:433-472): the output
    allocation, device guard and stream come from the torch-side launcher (csrc/cc1d_torch_ext.cpp),
    which calls cc1d_fwd."""
    if x.dtype not in _FLOAT:
        raise TypeError(f"x must be float32, float16 or bfloat16, got {x.dtype}")
    rc, out = tex.fwd(x, weight, bias, seq_idx, initial_states, final_states, bool(silu))
    if rc:
        check(rc, "causal_conv1d forward")
    return out


def _bwd(x, weight, bias, seq_idx, initial_states, dout, dfinal_states, need_dinit, silu,
         grad_f32=None, fuse_param_grads=True):
    """Host launcher of the backward (the reference's `_bwd`, causal_conv1d.py:475-541), through the
    torch-side launcher (csrc/cc1d_torch_ext.cpp): it allocates dx, dinit, the gradients and the
    workspace (cc1d_bwd_workspace_bytes) with torch's allocator and calls cc1d_bwd.

    Returns (dx, dweight, dbias, dinit). With `grad_f32` (a contiguous fp32 tensor of D * (W + 1)
    elements) the weight/bias gradients are written there as [dweight (D, W), dbias (D)] instead,
    and dweight/dbias are returned as None. With fp32 weight and bias and `fuse_param_grads`,
    dweight and dbias are views of one fp32 buffer (one allocation fewer per call).
    """
    rc, dx, dweight, dbias, dinit = tex.bwd(x, weight, bias, seq_idx, initial_states, dout, dfinal_states,
                                            bool(need_dinit), bool(silu), grad_f32, bool(fuse_param_grads))
    if rc:
        check(rc, "causal_conv1d backward")
    return dx, dweight, dbias, dinit


def _copy_channels(dst, src):
    """dst[...] = src for two (B, T, C) tensors with channel stride 1 and any batch/time strides,
    through the library's vectorised copy (cc1d_copy_channels)."""
    assert dst.shape == src.shape and dst.dtype == src.dtype and dst.dim() == 3
    if src.stride(2) != 1:
        src = src.contiguous()
    assert dst.stride(2) == 1
    B, T, C = dst.shape
    with _DeviceGuard(dst.device):
        check(lib.cc1d_copy_channels(dst.data_ptr(), dst.stride(0), dst.stride(1), src.data_ptr(), src.stride(0),
                                     src.stride(1), B, T, C, dst.element_size(), _stream(dst.device)),
              "cc1d_copy_channels")


def _bwd_split(x, weight, bias, seq_idx, initial_states, dout_pieces, need_dinit, silu, dx):
    """Backward with dout given as channel pieces and dx written into a caller's view.

    dout_pieces: (B, T, w_i) tensors with channel stride 1 whose widths sum to D, in channel order
    (at most CC1D_MAX_DOUT_PIECES). dx: a (B, T, D) view with channel stride 1 (for instance a
    channel slice of a wider gradient buffer), written in place. Returns (dweight, dbias, dinit).
    Uses cc1d_bwd_split, which reads the pieces where they lie and writes dx at its strides; when
    the layout is outside its fast path (CC1D_ERR_LAYOUT, reported before any device work) the
    pieces are concatenated and the ordinary backward runs, with dx copied into place.
    """
    B, T, D = x.shape
    W = weight.shape[1]
    assert sum(p.shape[-1] for p in dout_pieces) == D and dx.shape == (B, T, D) and dx.stride(2) == 1
    if len(dout_pieces) <= _native.CC1D_MAX_DOUT_PIECES:
        dinit = torch.empty_like(initial_states) if need_dinit else None
        w, b, init = _as_float(weight), _as_float(bias), _as_float(initial_states)
        dinit_k = _as_float(dinit)
        dweight = torch.empty_like(w)
        dbias = torch.empty_like(b) if b is not None else None
        p0 = dout_pieces[0]
        with _DeviceGuard(x.device):
            ws_bytes = lib.cc1d_bwd_workspace_bytes(
                x.data_ptr(), x.stride(0), x.stride(1), p0.data_ptr(), p0.stride(0), p0.stride(1),
                B, T, D, W, DTYPE_CODE[x.dtype],
            )
            if ws_bytes < 0:
                check(_native.CC1D_ERR_INVALID, "causal_conv1d backward workspace")
            workspace = torch.empty(max(1, ws_bytes // 4), device=x.device, dtype=torch.float32)
            pieces = (_native.DoutPiece * len(dout_pieces))(
                *[_native.DoutPiece(p.data_ptr(), p.stride(0), p.stride(1), p.shape[2]) for p in dout_pieces])
            rc = lib.cc1d_bwd_split(
                x.data_ptr(), x.stride(0), x.stride(1), w.data_ptr(), _ptr(b), _ptr(init), _ptr(seq_idx),
                pieces, len(dout_pieces), None, dx.data_ptr(), dx.stride(0), dx.stride(1), _ptr(dweight),
                _ptr(dbias), _ptr(dinit_k), None, workspace.data_ptr(), ws_bytes, B, T, D, W,
                DTYPE_CODE[x.dtype], DTYPE_CODE[w.dtype], _code(b), _code(init), int(silu),
                _stream(x.device),
            )
        if rc != _native.CC1D_ERR_LAYOUT:
            check(rc, "causal_conv1d split backward")
            if dinit is not None and dinit_k is not dinit:
                dinit.copy_(dinit_k)
            if dweight.dtype != weight.dtype:
                dweight = dweight.to(weight.dtype)
            if dbias is not None and dbias.dtype != bias.dtype:
                dbias = dbias.to(bias.dtype)
            return dweight, dbias, dinit
    dout = torch.cat([p.contiguous() for p in dout_pieces], dim=-1)
    dx_full, dweight, dbias, dinit = _bwd(x, weight, bias, seq_idx, initial_states, dout, None, need_dinit, silu)
    dx.copy_(dx_full)
    return dweight, dbias, dinit


def causal_conv1d_fn(
    x: Tensor,
    weight: Tensor,
    bias: Tensor | None = None,
    seq_idx: Tensor | None = None,
    initial_states: Tensor | None = None,
    return_final_states: bool = False,
    final_states_out: Tensor | None = None,
    activation: str | None = None,
) -> Tensor | tuple[Tensor, Tensor]:
    """Causal depthwise conv1d over channels-last inputs.

    x: (batch, seqlen, dim); must be contiguous along dim
    weight: (dim, width), width >= 2
    bias: (dim,)
    seq_idx: (batch, seqlen) integer sequence ids for packed sequences. Positions with negative ids
        are considered padding, and give zero outputs. Can be combined with initial_states, which
        count as part of seq_idx[:, 0]'s sequence, but cannot be combined with return_final_states
    initial_states: (batch, width - 1, dim), the inputs preceding x[:, 0]
    return_final_states: also return the last width - 1 rows of concat(initial_states, x), i.e. the
        initial_states for continuing the sequence; supports grad
    final_states_out: optional (batch, width - 1, dim) buffer to copy the final states into
    activation: None, "silu", or "swish"

    Returns out of shape (batch, seqlen, dim) and dtype x.dtype, or (out, final_states).
    """
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

    needs_grad = torch.is_grad_enabled() and any(
        t is not None and t.requires_grad for t in (x, weight, bias, initial_states)
    )
    if needs_grad:
        # The forward reads any layout; the backward's kernels need 16-byte aligned x, so a
        # misaligned x is copied once here and the copy is what the backward keeps.
        x = _tma_layout(x, weight.shape[1])
        # The reference's `_CausalConv1dFn` (causal_conv1d.py:544-576) as a C++ autograd Function
        # (`ConvFn`, csrc/cc1d_torch_ext.cpp): same saved tensors, need_dinit rule and gradients. A
        # failing library call inside it raises RuntimeError with the library's message.
        res = tex.conv_fn(x, weight, bias, seq_idx, initial_states, return_final_states, silu)
        result = (res[0], res[1]) if return_final_states else res[0]
    else:
        final_states = None
        if return_final_states:
            final_states = torch.empty(
                x.shape[0], weight.shape[1] - 1, x.shape[2], device=x.device, dtype=x.dtype
            )
        out = _fwd(x, weight, bias, seq_idx, initial_states, final_states, silu)
        result = (out, final_states) if return_final_states else out

    if final_states_out is not None:
        out, final_states = result
        result = out, final_states_out.copy_(final_states)
    return result


def causal_conv1d_update(
    x: Tensor,
    conv_state: Tensor,
    weight: Tensor,
    bias: Tensor | None = None,
    activation: str | None = None,
    conv_state_indices: Tensor | None = None,
) -> Tensor:
    """Decode step: run the new rows `x` through the conv, continuing from `conv_state`.

    x: (batch, dim) for one new row per batch entry, or (batch, seqlen, dim) for several;
        contiguous along dim
    conv_state: (n_slots, width - 1, dim), the inputs preceding x (the reference's state layout,
        causal_conv1d.py:597-599); updated in place to the last width - 1 rows of
        concat(conv_state, x), i.e. the final_states the forward would return
    weight: (dim, width); bias: (dim,); activation: None, "silu" or "swish"
    conv_state_indices: optional (batch,) integer slot of each batch entry in conv_state; a
        negative slot leaves that entry's output unwritten and its state untouched

    Returns the output rows, shaped like x, in x's dtype: the same values causal_conv1d_fn gives for
    these rows with initial_states=conv_state. The reference has no decode kernel; this is its
    single-step companion. Not differentiable (inference only).
    """
    if activation not in (None, "silu", "swish"):
        raise NotImplementedError("activation must be None, silu, or swish")
    squeeze = x.ndim == 2
    if squeeze:
        x = x.unsqueeze(1)
    assert x.ndim == 3, "x must be (batch, dim) or (batch, seqlen, dim)"
    B, L, D = x.shape
    assert weight.ndim == 2 and weight.shape[0] == D, "weight must be (dim, width)"
    W = weight.shape[1]
    assert W >= 2, "width must be >= 2"
    assert x.is_cuda and weight.device == x.device and conv_state.device == x.device
    assert conv_state.ndim == 3 and conv_state.shape[1:] == (W - 1, D)
    assert conv_state.is_contiguous(), "conv_state must be contiguous (it is updated in place)"
    assert bias is None or bias.shape == (D,)
    if conv_state_indices is None:
        assert conv_state.shape[0] >= B
    else:
        assert conv_state_indices.shape == (B,)
        conv_state_indices = conv_state_indices.to(device=x.device, dtype=torch.int32).contiguous()
    if x.dtype not in _FLOAT or conv_state.dtype not in _FLOAT:
        raise TypeError("x and conv_state must be float32, float16 or bfloat16")
    x = _channels_contiguous(x)
    w, b = _as_float(weight.contiguous()), _as_float(bias.contiguous() if bias is not None else None)
    out = torch.empty(B, L, D, device=x.device, dtype=x.dtype)
    with _DeviceGuard(x.device):
        rc = fast.update(
            x.data_ptr(), x.stride(0), x.stride(1), conv_state.data_ptr(),
            _ptr(conv_state_indices), w.data_ptr(), _ptr(b), out.data_ptr(), B, L, D, W,
            DTYPE_CODE[x.dtype], DTYPE_CODE[conv_state.dtype], DTYPE_CODE[w.dtype], _code(b),
            int(activation is not None), _stream(x.device),
        )
    if rc:
        check(rc, "causal_conv1d update")
    return out.squeeze(1) if squeeze else out


def seq_idx_from_cu_seqlens(cu_seqlens: Tensor, seqlen: int) -> Tensor:
    """seq_idx (int32) for packed variable-length sequences, built on the device.

    cu_seqlens: (n_seqs + 1,) for a single packed row, or (batch, n_seqs + 1) for one set of
        boundaries per row; non-decreasing from 0. Row b's sequences are [cu[i], cu[i+1]).
    seqlen: length T of each packed row.

    Returns (batch, seqlen) int32 (batch = 1 for 1-D cu_seqlens): each position's sequence id, and
    -1 (padding: zero output in causal_conv1d_fn) at or past the last boundary.
    """
    cu = cu_seqlens.unsqueeze(0) if cu_seqlens.ndim == 1 else cu_seqlens
    assert cu.ndim == 2 and cu.shape[1] >= 2, "cu_seqlens must be (n_seqs + 1,) or (batch, n_seqs + 1)"
    assert cu.is_cuda, "cu_seqlens must be on a CUDA device"
    cu = cu.to(torch.int32).contiguous()
    B, n1 = cu.shape
    seq_idx = torch.empty(B, seqlen, device=cu.device, dtype=torch.int32)
    with _DeviceGuard(cu.device):
        check(lib.cc1d_seq_idx_from_cu_seqlens(cu.data_ptr(), n1 - 1, seq_idx.data_ptr(), B, seqlen,
                                               _stream(cu.device)),
              "seq_idx_from_cu_seqlens")
    return seq_idx
