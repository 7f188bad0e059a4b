"""Python front end of the CPU oracle (oracle/cc1d_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker the CUDA path is compared against and the timed CPU
baseline. Only tests/, __graft_entry__.smoke() and bench.py (cpu_baseline leg and `--impl
reference` arm) may import this module. The product package never imports it.

The C restatement follows jxiong21029/causal-conv1d-triton, causal_conv1d_triton/causal_conv1d.py:
forward `_fwd_kernel` (causal_conv1d.py:44-164), backward `_bwd_kernel` + `_reduce_partials_kernel`
(causal_conv1d.py:167-374), and the host-side empty-input cases of `_fwd`/`_bwd`
(causal_conv1d.py:433-444, 475-489), which are restated here in Python. All arithmetic is fp32 on
fp32 copies of the inputs (bf16/fp16 -> fp32 is exact); callers round to the output dtype.

The oracle is pinned against outputs of the reference itself, run under the Triton CPU
interpreter, in tests/golden/ (tests/test_oracle_golden.py).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libcc1d_oracle.so")
_lib = None
_lock = threading.Lock()

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i64 = ctypes.c_int64


def build(force: bool = False) -> str:
    """Compile the C oracle with the Makefile beside this file; returns the library path."""
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
        os.path.join(_HERE, "cc1d_oracle.c")
    ):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                build()
            lib = ctypes.CDLL(_LIB_PATH)
            lib.cc1d_oracle_fwd.argtypes = [_f32p, _f32p, _f32p, _f32p, _i32p, _f32p, _f32p,
                                            _i64, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int]
            lib.cc1d_oracle_fwd.restype = None
            lib.cc1d_oracle_bwd.argtypes = [_f32p, _f32p, _f32p, _f32p, _i32p, _f32p, _f32p,
                                            _f32p, _f32p, _f32p, _f32p,
                                            _i64, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int]
            lib.cc1d_oracle_bwd.restype = None
            lib.cc1d_oracle_update.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p,
                                               _i64, _i64, _i64, _i64, ctypes.c_int]
            lib.cc1d_oracle_update.restype = None
            _lib = lib
    return _lib


def _f32(a):
    """Contiguous fp32 numpy copy of a numpy array or (CPU/CUDA) torch tensor, or None."""
    if a is None:
        return None
    if hasattr(a, "detach"):
        a = a.detach().float().cpu().numpy()
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a):
    if a is None:
        return None
    if hasattr(a, "detach"):
        a = a.detach().cpu().numpy()
    return np.ascontiguousarray(a, dtype=np.int32)


def _p(a, typ=_f32p):
    return None if a is None else a.ctypes.data_as(typ)


def fwd(x, weight, bias=None, initial_states=None, seq_idx=None, silu=False,
        return_final_states=False, nthreads=0):
    """Forward of causal_conv1d_fn in fp32. Returns out (B, T, D), plus final_states (B, W-1, D)
    when return_final_states. T == 0 follows _fwd (causal_conv1d.py:437-444)."""
    x, w, b, init = _f32(x), _f32(weight), _f32(bias), _f32(initial_states)
    seq = _i32(seq_idx)
    B, T, D = x.shape
    W = w.shape[1]
    out = np.zeros((B, T, D), np.float32)
    final = np.zeros((B, W - 1, D), np.float32) if return_final_states else None
    if T == 0:
        if final is not None and init is not None:
            final[...] = init
    else:
        _load().cc1d_oracle_fwd(_p(x), _p(w), _p(b), _p(init), _p(seq, _i32p), _p(out),
                                _p(final), B, T, D, W, int(bool(silu)), int(nthreads))
    return (out, final) if return_final_states else out


def bwd(x, weight, bias, initial_states, seq_idx, dout, dfinal_states=None, need_dinit=False,
        silu=False, nthreads=0):
    """Backward of causal_conv1d_fn in fp32. Returns (dx, dweight, dbias, dinit); dbias is None
    without bias, dinit is None unless need_dinit. T == 0 follows _bwd (causal_conv1d.py:480-489)."""
    x, w, b, init = _f32(x), _f32(weight), _f32(bias), _f32(initial_states)
    seq, dy, dfin = _i32(seq_idx), _f32(dout), _f32(dfinal_states)
    B, T, D = x.shape
    W = w.shape[1]
    dx = np.zeros((B, T, D), np.float32)
    dw = np.zeros((D, W), np.float32)
    db = np.zeros((D,), np.float32) if b is not None else None
    dinit = np.zeros((B, W - 1, D), np.float32) if need_dinit else None
    if T == 0:
        if dinit is not None and dfin is not None:
            dinit[...] = dfin
    else:
        _load().cc1d_oracle_bwd(_p(x), _p(w), _p(b), _p(init), _p(seq, _i32p), _p(dy),
                                _p(dfin), _p(dx), _p(dw), _p(db), _p(dinit),
                                B, T, D, W, int(bool(silu)), int(nthreads))
    return dx, dw, db, dinit


def update(x, conv_state, weight, bias=None, silu=False):
    """Decode step(s): x (B, L, D) new rows, conv_state (B, W-1, D). Returns (out, new_state)."""
    x, st, w, b = _f32(x), _f32(conv_state).copy(), _f32(weight), _f32(bias)
    B, L, D = x.shape
    W = w.shape[1]
    out = np.zeros((B, L, D), np.float32)
    _load().cc1d_oracle_update(_p(x), _p(st), _p(w), _p(b), _p(out), B, L, D, W, int(bool(silu)))
    return out, st
