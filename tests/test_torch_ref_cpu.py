"""The torch fp32 restatement used by the full-shape GPU parity tests (tests/_torch_ref.py) agrees
with the pinned C oracle and with the reference's own golden vectors, on the CPU.

The oracle is pinned to outputs of the reference (tests/test_oracle_golden.py); this ties the
second checker to it, so a disagreement at full size points at the CUDA path, not the checker.
"""

import numpy as np
import pytest
import torch

from _golden import CASES, CASE_IDS
from _tol import assert_close, assert_close_sum
from _torch_ref import backward_chunk, forward_chunk
from oracle import oracle

# fp32 reference vs fp32 oracle: both compute in fp32 with different summation orders.
TOL = "f32"


def _case(seed, B, T, D, W, bias, init, seq, dfinal, silu):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, D, generator=g)
    w = torch.randn(D, W, generator=g) * W ** -0.5
    b = torch.randn(D, generator=g) * 0.3 if bias else None
    st = torch.randn(B, W - 1, D, generator=g) if init else None
    s = None
    if seq:
        s = torch.zeros(B, T, dtype=torch.int32)
        for r in range(B):
            cuts = sorted(torch.randint(1, T, (3,), generator=g).tolist())
            for i, c in enumerate(cuts):
                s[r, c:] = i + 1
            s[r, T - 5:] = -1
    dy = torch.randn(B, T, D, generator=g)
    df = torch.randn(B, W - 1, D, generator=g) if dfinal else None
    return x, w, b, st, s, dy, df, silu


CASES_CPU = [
    (0, 2, 64, 24, 4, True, True, False, True, True),
    (1, 3, 50, 16, 8, True, True, True, False, True),
    (2, 2, 33, 8, 3, False, False, True, False, False),
    (3, 2, 2, 8, 5, True, True, False, True, True),  # T < W - 1: dfinal reaches the init rows
    (4, 1, 40, 12, 2, True, False, False, False, True),
]


@pytest.mark.parametrize("case", CASES_CPU)
def test_torch_ref_matches_oracle(case):
    x, w, b, st, s, dy, df, silu = _case(*case)
    _, out = forward_chunk(x, w, b, st, s, silu)
    eo = oracle.fwd(x, w, b, st, s, silu=silu)
    assert_close(out, eo, TOL, "out")
    dx, dinit, dw, db = backward_chunk(x, w, b, st, s, dy, df, silu)
    edx, edw, edb, edi = oracle.bwd(x, w, b, st, s, dy, df, need_dinit=st is not None, silu=silu)
    assert_close(dx, edx, TOL, "dx")
    assert_close_sum(dw, edw, TOL, "dweight")
    if b is not None:
        assert_close_sum(db, edb, TOL, "dbias")
    if st is not None:
        assert_close(dinit, edi, TOL, "dinit")


@pytest.mark.parametrize("idx", range(len(CASES)), ids=CASE_IDS)
def test_torch_ref_matches_reference_golden(idx):
    """Against the vectors the reference itself produced (bf16/fp16 cases at their own tolerance:
    the golden outputs are rounded to the input dtype)."""
    meta, a = CASES[idx]
    if meta["T"] == 0:
        pytest.skip("T = 0 is a host-side case (no kernel arithmetic)")
    t = {k: torch.from_numpy(np.asarray(v)) for k, v in a.items()}
    dt = meta["x_dtype"]
    silu = meta["silu"]
    x, w = t["x"], t["weight"]
    b, st, s = t.get("bias"), t.get("initial_states"), t.get("seq_idx")
    _, out = forward_chunk(x, w, b, st, s, silu)
    assert_close(out, t["out"], dt, "out")
    if "dout" in t:
        dx, dinit, dw, db = backward_chunk(x, w, b, st, s, t["dout"], t.get("dfinal_states"), silu)
        assert_close(dx, t["dx"], dt, "dx")
        assert_close_sum(dw, t["dweight"], dt, "dweight")
        if "dbias" in t:
            assert_close_sum(db, t["dbias"], dt, "dbias")
        if "dinit" in t:
            assert_close(dinit, t["dinit"], dt, "dinit")
