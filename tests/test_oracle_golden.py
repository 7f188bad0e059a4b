"""Pins the CPU oracle (oracle/) to outputs of the reference implementation itself.

tests/golden/reference_vectors.npz holds inputs and outputs of the reference's own `_fwd`/`_bwd`
(causal_conv1d_triton/causal_conv1d.py:433-541) run under the Triton CPU interpreter; see
tests/golden/make_golden.py. Every case is recomputed by the oracle and compared within the
parity tolerance of the case's dtype, with final_states and seq_idx padding zeros bit-exact.
"""

import numpy as np
import pytest
import torch

from _golden import CASES, CASE_IDS
from _tol import assert_bitexact, assert_close, assert_close_sum
from oracle import oracle

DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def _round(a, dt):
    return torch.from_numpy(np.asarray(a, np.float32)).to(DT[dt]).float().numpy()


@pytest.mark.parametrize("case", CASES, ids=CASE_IDS)
def test_oracle_matches_reference(case):
    m, g = case
    xdt, wdt = m["x_dtype"], m["w_dtype"]
    res = oracle.fwd(g["x"], g["weight"], g.get("bias"), g.get("initial_states"), g.get("seq_idx"),
                     silu=m["silu"], return_final_states=m["return_final_states"])
    out, final = res if m["return_final_states"] else (res, None)
    assert_close(_round(out, xdt), g["out"], xdt, "out")
    if final is not None:
        assert_bitexact(_round(final, xdt), g["final_states"], "final_states")
    if m["seq"] and m["T"] > 0:
        pad = g["seq_idx"] < 0
        assert (g["out"][pad] == 0).all() and (out[pad] == 0).all()

    dx, dw, db, dinit = oracle.bwd(g["x"], g["weight"], g.get("bias"), g.get("initial_states"),
                                   g.get("seq_idx"), g["dout"], g.get("dfinal_states"),
                                   need_dinit=m["need_dinit"], silu=m["silu"])
    assert_close(_round(dx, xdt), g["dx"], xdt, "dx")
    assert_close_sum(_round(dw, wdt), g["dweight"], xdt, "dweight")
    if m["bias"]:
        assert_close_sum(_round(db, wdt), g["dbias"], xdt, "dbias")
    if m["need_dinit"]:
        assert_close(_round(dinit, xdt), g["dinit"], xdt, "dinit")
    if m["seq"] and m["T"] > 0:
        # A padding row only feeds outputs at padding rows, whose gradient is zero.
        pad = g["seq_idx"] < 0
        assert (g["dx"][pad] == 0).all() and (dx[pad] == 0).all()


def test_oracle_catches_planted_error():
    """A mistake planted in the oracle's output (on the CPU) must fail the comparison."""
    m, g = CASES[0]
    out = oracle.fwd(g["x"], g["weight"], g.get("bias"), None, None, silu=m["silu"])
    out = out.copy()
    out[0, 5, 3] += 0.5
    with pytest.raises(AssertionError):
        assert_close(_round(out, m["x_dtype"]), g["out"], m["x_dtype"], "out")
