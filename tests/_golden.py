"""Loader for tests/golden/reference_vectors.npz (written by tests/golden/make_golden.py from the
reference implementation run under the Triton CPU interpreter)."""

import json
import os

import numpy as np

PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_vectors.npz")


def load_cases():
    z = np.load(PATH)
    metas = json.loads(str(z["__meta__"]))
    cases = []
    for m in metas:
        pre = m["name"] + "/"
        arrs = {k[len(pre):]: z[k] for k in z.files if k.startswith(pre)}
        cases.append((m, arrs))
    return cases


CASES = load_cases()
CASE_IDS = [m["name"] for m, _ in CASES]
