"""Bindings of libcausal_conv1d_b200.so, the C ABI declared in include/causal_conv1d_b200.h.

`lib` binds every entry point with ctypes. `fast` is the package's CPython binding of the hot
launch entry points (cc1d_fwd, cc1d_bwd_workspace_bytes, cc1d_bwd, cc1d_update; built from
csrc/cc1d_pyfast.c), which parses arguments in a fraction of ctypes' per-call time. `tex` holds
the forward and backward launchers written in C++ against torch (csrc/cc1d_torch_ext.cpp): they
allocate the outputs and the workspace with torch's allocator and call cc1d_fwd / cc1d_bwd, which
keeps the per-call host time of the autograd path low. All three reach the same loaded library and
are built in-tree by causal-conv1d-triton_b200/build.py. Importing this module without them raises
ImportError: there is no CPU or Python fallback for the kernels.
"""

from __future__ import annotations

import ctypes
import os

import torch

LIB_NAME = "libcausal_conv1d_b200.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

# Element type codes (CC1D_F32, CC1D_F16, CC1D_BF16).
DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

CC1D_OK = 0
CC1D_ERR_INVALID = 1
CC1D_ERR_UNSUPPORTED = 2
CC1D_ERR_WORKSPACE = 3
CC1D_ERR_CUDA = 4
CC1D_ERR_SCRATCH_LIMIT = 5
CC1D_ERR_LAYOUT = 6
CC1D_MAX_DOUT_PIECES = 4


class DoutPiece(ctypes.Structure):
    """cc1d_dout_piece: one channel range of dout in its own tensor."""

    _fields_ = [("ptr", ctypes.c_void_p), ("stride_batch", ctypes.c_int64),
                ("stride_time", ctypes.c_int64), ("channels", ctypes.c_int64)]


# Every symbol the header declares, with its ctypes signature.
_P, _I64, _I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
SIGNATURES = {
    "cc1d_abi_version": ([], _I),
    "cc1d_fwd": ([_P, _I64, _I64, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64,
                  _I, _I, _I, _I, _I, _P], _I),
    "cc1d_seq_idx_from_cu_seqlens": ([_P, _I64, _P, _I64, _I64, _P], _I),
    "cc1d_update": ([_P, _I64, _I64, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64,
                     _I, _I, _I, _I, _I, _P], _I),
    "cc1d_bwd_workspace_bytes": ([_P, _I64, _I64, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I],
                                 _I64),
    "cc1d_bwd": ([_P, _I64, _I64, _P, _P, _P, _P, _P, _I64, _I64, _P, _P, _P, _P, _P, _P,
                  _P, _I64, _I64, _I64, _I64, _I64, _I, _I, _I, _I, _I, _P], _I),
    "cc1d_bwd_noalloc": ([_P, _I64, _I64, _P, _P, _P, _P, _P, _I64, _I64, _P, _P, _P, _P, _P, _P,
                          _I64, _I64, _I64, _I64, _I, _I, _I, _I, _I, _P], _I),
    "cc1d_bwd_split": ([_P, _I64, _I64, _P, _P, _P, _P, ctypes.POINTER(DoutPiece), _I, _P, _P, _I64,
                        _I64, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I, _I, _I, _I,
                        _I, _P], _I),
    "cc1d_copy_channels": ([_P, _I64, _I64, _P, _I64, _I64, _I64, _I64, _I64, _I, _P], _I),
    "cc1d_selftest_wait_timeout": ([_P], _I),
    "cc1d_status": ([ctypes.POINTER(ctypes.c_uint32), _I], _I),
    "cc1d_error_string": ([_I], ctypes.c_char_p),
    "cc1d_last_cuda_error": ([], _I),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build the CUDA library first "
            "(python causal-conv1d-triton_b200/build.py, or __graft_entry__.build())"
        )
    lib = ctypes.CDLL(LIB_PATH)
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    return lib


lib = _load()

try:
    from . import _cc1d_fast as fast  # noqa: E402  (links libcausal_conv1d_b200.so, loaded above)
except ImportError as e:  # pragma: no cover - only without a build
    raise ImportError(f"the package's CPython binding is missing ({e}): build the CUDA library first "
                      "(python causal-conv1d-triton_b200/build.py)") from e


try:
    import torch  # noqa: E402,F401  (the launchers below link torch's libraries)

    from . import _cc1d_torch as tex  # noqa: E402  (torch-side forward/backward launchers)
except ImportError as e:  # pragma: no cover - only without a build
    raise ImportError(f"the package's torch launchers are missing ({e}): build the CUDA library first "
                      "(python causal-conv1d-triton_b200/build.py)") from e


class CausalConv1dError(RuntimeError):
    """A non-zero status returned by the C ABI."""


def check(code: int, what: str) -> None:
    if code != CC1D_OK:
        msg = lib.cc1d_error_string(code).decode()
        if code == CC1D_ERR_CUDA:
            msg += f" (cudaError {lib.cc1d_last_cuda_error()})"
        raise CausalConv1dError(f"{what}: {msg}")


def status(clear: bool = False) -> int:
    """Device status word of the current device (synchronises it); bit 0 = a kernel timed out."""
    v = ctypes.c_uint32(0)
    check(lib.cc1d_status(ctypes.byref(v), int(clear)), "cc1d_status")
    return v.value
