"""CPU-side checks of the C-ABI library and of the host logic (no GPU needed).

- libcausal_conv1d_b200.so loads on a machine without a GPU and exports every function that
  include/causal_conv1d_b200.h declares, with the signatures the ctypes binding uses.
- The error codes and strings are stable.
- causal_conv1d_fn raises the reference's errors for bad arguments before touching a device
  (causal_conv1d_triton/causal_conv1d.py:605-611).
"""

import ctypes
import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "causal_conv1d_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(cc1d_\w+)\s*\(", src)))


def test_header_declares_the_abi():
    names = declared_functions()
    for n in ["cc1d_fwd", "cc1d_bwd", "cc1d_bwd_workspace_bytes", "cc1d_status",
              "cc1d_error_string", "cc1d_last_cuda_error", "cc1d_abi_version"]:
        assert n in names


def test_library_exports_every_declared_symbol():
    from causal_conv1d_b200 import _native

    lib = ctypes.CDLL(_native.LIB_PATH)
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
        assert name in _native.SIGNATURES, f"{name} has no ctypes signature in _native"


def test_abi_version_and_error_strings():
    from causal_conv1d_b200 import _native

    assert _native.lib.cc1d_abi_version() == 2
    assert _native.lib.cc1d_error_string(0) == b"success"
    for code in (1, 2, 3, 4, 5, 6):
        assert len(_native.lib.cc1d_error_string(code)) > 5
    assert _native.lib.cc1d_error_string(99) == b"unknown error"


def test_split_backward_rejects_bad_pieces_without_device_work():
    """cc1d_bwd_split validates its pieces (count, widths, coverage of dim) before any CUDA call."""
    from causal_conv1d_b200 import _native

    lib, P = _native.lib, _native.DoutPiece

    def call(pieces, dim=256):
        arr = (P * max(1, len(pieces)))(*pieces)
        return lib.cc1d_bwd_split(None, 0, 0, None, None, None, None, arr, len(pieces), None, None, 0, 0,
                                  None, None, None, None, None, 0, 2, 8, dim, 4, 2, 0, 0, 0, 1, None)

    assert call([]) == _native.CC1D_ERR_INVALID
    assert call([P(None, 0, 0, 128)] * 5, dim=640) == _native.CC1D_ERR_INVALID  # above the limit
    assert call([P(None, 0, 0, 128), P(None, 0, 0, 0), P(None, 0, 0, 128)]) == _native.CC1D_ERR_INVALID
    assert call([P(None, 0, 0, 128), P(None, 0, 0, 64)]) == _native.CC1D_ERR_INVALID  # 192 != 256


def test_invalid_sizes_rejected_without_device_work():
    """Argument checks run before any CUDA call."""
    from causal_conv1d_b200 import _native

    lib = _native.lib
    # width 1 is invalid, width 257 unsupported, negative sizes invalid, bad dtype code invalid
    assert lib.cc1d_bwd_workspace_bytes(None, 0, 0, None, 0, 0, 1, 8, 8, 1, 2) == -1
    assert lib.cc1d_bwd_workspace_bytes(None, 0, 0, None, 0, 0, 1, 8, 8, 257, 2) == -1
    assert lib.cc1d_bwd_workspace_bytes(None, 0, 0, None, 0, 0, -1, 8, 8, 4, 2) == -1
    assert lib.cc1d_bwd_workspace_bytes(None, 0, 0, None, 0, 0, 1, 8, 8, 4, 7) == -1
    # empty inputs need no workspace
    assert lib.cc1d_bwd_workspace_bytes(None, 0, 0, None, 0, 0, 0, 8, 8, 4, 2) == 0
    rc = lib.cc1d_fwd(None, 0, 0, None, None, None, None, None, None, 1, 8, 8, 300,
                      2, 0, 0, 0, 1, None)
    assert rc == _native.CC1D_ERR_UNSUPPORTED
    rc = lib.cc1d_fwd(None, 0, 0, None, None, None, None, None, None, 1, 8, 8, 4,
                      9, 0, 0, 0, 1, None)
    assert rc == _native.CC1D_ERR_INVALID


def test_api_errors_match_reference():
    from causal_conv1d_b200 import causal_conv1d_fn

    x = torch.randn(2, 8, 4)
    w = torch.randn(4, 3)
    with pytest.raises(NotImplementedError):
        causal_conv1d_fn(x, w, activation="relu")
    with pytest.raises(AssertionError):
        causal_conv1d_fn(x, w, seq_idx=torch.zeros(2, 8, dtype=torch.int32),
                         return_final_states=True)
    with pytest.raises(AssertionError):
        causal_conv1d_fn(x, w, final_states_out=torch.empty(2, 2, 4))
    with pytest.raises(AssertionError):  # weight must be (dim, width)
        causal_conv1d_fn(x, torch.randn(5, 3))
    with pytest.raises(AssertionError):  # width >= 2
        causal_conv1d_fn(x, torch.randn(4, 1))
    with pytest.raises(AssertionError):  # x must be on a CUDA device
        causal_conv1d_fn(x, w)


def test_split_conv1d_argument_errors():
    """split_conv1d checks its arguments on the host before any device work."""
    from causal_conv1d_b200 import split_conv1d

    zx = torch.randn(2, 8, 20)
    w = torch.randn(12, 4)
    with pytest.raises(NotImplementedError):
        split_conv1d(zx, w, d_z=4, xbc_split=(8, 2, 2), activation="gelu")
    with pytest.raises(AssertionError):  # zxbcdt must be 3-D
        split_conv1d(zx[0], w, d_z=4, xbc_split=(8, 2, 2))
    with pytest.raises(AssertionError):  # z + xBC wider than zxbcdt
        split_conv1d(zx, w, d_z=10, xbc_split=(8, 2, 2))
    with pytest.raises(AssertionError):  # empty piece
        split_conv1d(zx, w, d_z=4, xbc_split=(12, 0))
    with pytest.raises(AssertionError):  # weight rows must equal sum(xbc_split)
        split_conv1d(zx, torch.randn(10, 4), d_z=4, xbc_split=(8, 2, 2))
    with pytest.raises(AssertionError):  # zxbcdt must be on a CUDA device
        split_conv1d(zx, w, d_z=4, xbc_split=(8, 2, 2))


def test_copy_channels_rejects_bad_arguments():
    from causal_conv1d_b200 import _native

    lib = _native.lib
    assert lib.cc1d_copy_channels(None, 0, 0, None, 0, 0, 1, 1, 1, 3, None) == _native.CC1D_ERR_INVALID
    assert lib.cc1d_copy_channels(None, 0, 0, None, 0, 0, -1, 1, 1, 2, None) == _native.CC1D_ERR_INVALID
    assert lib.cc1d_copy_channels(None, 0, 0, None, 0, 0, 0, 8, 8, 2, None) == _native.CC1D_OK  # empty


def test_tma_layout_routing():
    """Host logic: a misaligned x whose rows are 16-byte multiples is copied once (contiguous,
    16-byte aligned) for the TMA kernels; aligned tensors, rows of other sizes and widths above 16
    are passed through unchanged."""
    from causal_conv1d_b200.causal_conv1d import _tma_layout

    x = torch.randn(2, 8, 16).to(torch.bfloat16)
    assert _tma_layout(x, 4) is x
    wide = torch.zeros(2, 8, 17, dtype=torch.bfloat16)
    sl = wide[..., 1:]  # odd channel offset: base 2 bytes past alignment
    y = _tma_layout(sl, 4)
    assert y is not sl and y.is_contiguous() and y.data_ptr() % 16 == 0 and torch.equal(y, sl)
    assert _tma_layout(sl, 17) is sl  # width beyond the TMA kernels
    odd = torch.zeros(2, 8, 13, dtype=torch.bfloat16)[..., 1:]  # 12 channels: 24-byte rows
    assert _tma_layout(odd, 4) is odd
    leaf = torch.zeros(2, 8, 17, dtype=torch.bfloat16, requires_grad=True)
    copied = _tma_layout(leaf[..., 1:], 4)  # misaligned view of a leaf: copied
    assert copied.data_ptr() != leaf.data_ptr()
    copied.float().sum().backward()  # the copy is differentiable
    assert (leaf.grad[..., 1:] == 1).all() and (leaf.grad[..., 0] == 0).all()


def test_fast_binding_checks_arguments_and_returns_abi_codes():
    """The package's CPython binding of the hot entry points (csrc/cc1d_pyfast.c) loads without a
    GPU, rejects a wrong argument count or type with a Python error, and returns the C ABI's own
    codes: an invalid dtype code or width is refused before any CUDA call."""
    from causal_conv1d_b200 import _native

    fast = _native.fast
    fwd = [1, 2, 3, 4, None, None, None, 5, None, 1, 2, 3, 4, 9, 0, 0, 0, 1, 0]
    assert fast.fwd(*fwd) == _native.CC1D_ERR_INVALID  # dtype code 9
    assert _native.lib.cc1d_fwd(*fwd) == _native.CC1D_ERR_INVALID
    bwd = [1, 2, 3, 4, None, None, None, 5, 6, 7, None, 8, 9, None, None, None, 10, 11,
           1, 2, 3, 4, 9, 0, 0, 0, 1, 0]
    assert fast.bwd(*bwd) == _native.CC1D_ERR_INVALID
    bwd_w = list(bwd)
    bwd_w[21], bwd_w[22] = 300, 2  # width 300 > 256, bf16
    assert fast.bwd(*bwd_w) == _native.lib.cc1d_bwd(*bwd_w) == _native.CC1D_ERR_UNSUPPORTED
    assert fast.bwd_workspace_bytes(1, 2, 3, 4, 5, 6, 1, 2, 3, 1, 2) == -1  # width 1
    upd = [1, 2, 3, 4, None, 5, None, 6, 1, 1, 3, 4, 9, 0, 0, 0, 1, 0]
    assert fast.update(*upd) == _native.CC1D_ERR_INVALID
    with pytest.raises(TypeError):
        fast.fwd(*fwd[:-1])
    with pytest.raises(TypeError):
        fast.bwd(*bwd, 0)
    with pytest.raises(TypeError):
        fast.fwd(*(["x"] + fwd[1:]))


def test_torch_launchers_load_and_expose_forward_and_backward():
    """The torch-side launchers (csrc/cc1d_torch_ext.cpp) load on the CPU, linked against the same
    library, with the forward and backward entry points the autograd path calls."""
    from causal_conv1d_b200 import _native

    tex = _native.tex
    assert callable(tex.fwd) and callable(tex.bwd)
    assert "fwd(" in tex.fwd.__doc__ and "bwd(" in tex.bwd.__doc__
    import os

    assert os.path.dirname(tex.__file__) == os.path.dirname(_native.LIB_PATH)
