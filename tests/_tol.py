"""Parity tolerances, as the task's correctness contract states them.

- final_states, the zero outputs at seq_idx padding rows and every tap the seq_idx mask removes
  are bit-exact (checked with exact equality where a test isolates them).
- bf16 / fp16 outputs and gradients: within 1e-2 relative / 1e-2 absolute of the fp32 CPU
  oracle, i.e. |actual - expected| <= 1e-2 + 1e-2 * |expected|, where the kernel's result is
  compared in fp32 after rounding to its own dtype.
- fp32 outputs: within 1e-5 (same form, 1e-5 for both terms).
- The tolerance is chosen by the dtype of x, the precision the whole call computes in: an fp32
  dweight from a bf16 call is held to the bf16 tolerance.
- dweight / dbias are sums over all B*T rows, so their rounding error grows with the magnitude
  of the sum rather than of each element: they are held to the same tolerance scaled by the
  largest |expected| entry, |actual - expected| <= tol * max(1, max|expected|).
"""

import numpy as np

TOL = {"f32": 1e-5, "f16": 1e-2, "bf16": 1e-2}


def dtype_key(dt) -> str:
    s = str(dt)
    if "bfloat16" in s or s == "bf16":
        return "bf16"
    if "float16" in s or s == "f16":
        return "f16"
    return "f32"


def _np(a):
    if hasattr(a, "detach"):
        a = a.detach().float().cpu().numpy()
    return np.asarray(a, dtype=np.float64)


def assert_close(actual, expected, dt, what=""):
    tol = TOL[dtype_key(dt)]
    a, e = _np(actual), _np(expected)
    assert a.shape == e.shape, f"{what}: shape {a.shape} != {e.shape}"
    err = np.abs(a - e)
    bound = tol + tol * np.abs(e)
    bad = ~(err <= bound)
    if bad.any():
        i = np.unravel_index(np.argmax(np.where(bad, err - bound, -np.inf)), a.shape)
        raise AssertionError(
            f"{what}: {bad.sum()} of {a.size} elements outside tol {tol}; worst at {i}: "
            f"actual {a[i]!r} expected {e[i]!r}"
        )


def assert_close_sum(actual, expected, dt, what=""):
    tol = TOL[dtype_key(dt)]
    a, e = _np(actual), _np(expected)
    assert a.shape == e.shape, f"{what}: shape {a.shape} != {e.shape}"
    scale = max(1.0, float(np.abs(e).max()) if e.size else 1.0)
    err = np.abs(a - e)
    bad = ~(err <= tol * scale)
    if bad.any():
        i = np.unravel_index(np.argmax(err), a.shape)
        raise AssertionError(
            f"{what}: {bad.sum()} of {a.size} elements outside tol {tol}*{scale:.3g}; worst at "
            f"{i}: actual {a[i]!r} expected {e[i]!r}"
        )


def assert_bitexact(actual, expected, what=""):
    a, e = _np(actual), _np(expected)
    assert a.shape == e.shape, f"{what}: shape {a.shape} != {e.shape}"
    assert np.array_equal(a, e), f"{what}: not bit-exact, max diff {np.abs(a - e).max()}"
