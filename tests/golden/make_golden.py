"""Generate golden input/output vectors from the reference implementation itself.

Runs jxiong21029/causal-conv1d-triton's own host launchers `_fwd` and `_bwd`
(causal_conv1d_triton/causal_conv1d.py:433-541) under the Triton CPU interpreter
(TRITON_INTERPRET=1), on small seeded inputs, and writes inputs and outputs to
tests/golden/reference_vectors.npz. The reference lives only in the build container, so this
script runs there; the committed .npz is what the tests read (on any machine).

Two things the reference needs a GPU for are replaced, as the interpreter cannot supply them:
`_num_sms` (causal_conv1d.py:389) returns 148 (a B200's SM count; it only sets the chunking) and
`torch.cuda.device` (causal_conv1d.py:448, 498) becomes a null context. `causal_conv1d_fn`
itself asserts `x.is_cuda` (causal_conv1d.py:403), so the public API's argument handling
(causal_conv1d.py:605-634, 544-576) is restated in `run_case` around the two launchers.

Usage: python tests/golden/make_golden.py --ref /path/to/causal-conv1d-triton
"""

from __future__ import annotations

import argparse
import contextlib
import json
import os
import sys
import time

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "reference_vectors.npz")

DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}

# name: (B, T, D, W, x dtype, weight/bias dtype, bias, silu, init, seq, final, dfinal, need_dinit)
CASES = [
    ("bf16_bias_silu", 2, 64, 48, 4, "bf16", "f32", True, True, False, False, False, False, False),
    ("f32_plain", 2, 40, 24, 4, "f32", "f32", False, False, False, False, False, False, False),
    ("f16_w2_bias_silu", 2, 33, 32, 2, "f16", "f32", True, True, False, False, False, False, False),
    ("bf16_w3_state_chain", 2, 50, 40, 3, "bf16", "f32", True, True, True, False, True, True, True),
    ("f32_w5_short_T", 2, 3, 16, 5, "f32", "f32", True, False, True, False, True, True, True),
    ("bf16_w8_bias_silu", 1, 100, 40, 8, "bf16", "f32", True, True, False, False, False, False, False),
    ("bf16_seq_init", 2, 96, 32, 4, "bf16", "f32", True, True, True, True, False, False, True),
    ("f32_w3_seq", 2, 80, 24, 3, "f32", "f32", True, True, False, True, False, False, False),
    ("f32_odd_D", 2, 37, 13, 4, "f32", "f32", True, True, True, False, True, True, True),
    ("bf16_T1_state", 2, 1, 16, 4, "bf16", "f32", False, False, True, False, True, True, True),
    ("f32_w9", 1, 45, 16, 9, "f32", "f32", True, True, True, False, True, False, True),
    ("bf16_long_chunks", 1, 300, 32, 4, "bf16", "f32", True, True, True, False, True, True, True),
    ("bf16_bf16_weight", 2, 48, 24, 4, "bf16", "bf16", True, True, False, False, False, False, False),
    ("f16_seq_noinit_w4", 1, 120, 16, 4, "f16", "f32", False, True, False, True, False, False, False),
    ("f32_T0_state", 2, 0, 8, 4, "f32", "f32", True, False, True, False, True, True, True),
]


def load_reference(path):
    sys.path.insert(0, path)
    import causal_conv1d_triton.causal_conv1d as cc

    cc._num_sms = lambda idx: 148
    torch.cuda.device = lambda d: contextlib.nullcontext()
    return cc


def make_seq(B, T, gen):
    """Consecutive sequences with lengths drawn from [1, T//3 + 1], then a padded tail of -1."""
    seq = torch.empty(B, T, dtype=torch.int32)
    for b in range(B):
        pad = int(torch.randint(0, max(1, T // 8), (1,), generator=gen))
        t, sid = 0, 0
        while t < T - pad:
            n = int(torch.randint(1, T // 3 + 2, (1,), generator=gen))
            seq[b, t:min(t + n, T - pad)] = sid
            t += n
            sid += 1
        seq[b, T - pad:] = -1
    return seq


def run_case(cc, i, spec):
    name, B, T, D, W, xdt, wdt, has_bias, silu, has_init, has_seq, ret_final, has_dfinal, need_dinit = spec
    gen = torch.Generator().manual_seed(1000 + i)
    x = torch.randn(B, T, D, generator=gen).to(DT[xdt])
    weight = (torch.randn(D, W, generator=gen) / W**0.5).to(DT[wdt])
    bias = (torch.randn(D, generator=gen) * 0.3).to(DT[wdt]) if has_bias else None
    init = torch.randn(B, W - 1, D, generator=gen).to(DT[xdt]) if has_init else None
    seq = make_seq(B, T, gen) if has_seq else None
    dout = torch.randn(B, T, D, generator=gen).to(DT[xdt])
    dfinal = torch.randn(B, W - 1, D, generator=gen).to(DT[xdt]) if has_dfinal else None

    # causal_conv1d_fn's argument handling (causal_conv1d.py:605-618) and
    # _CausalConv1dFn.forward/backward (causal_conv1d.py:546-576).
    final = torch.empty(B, W - 1, D, dtype=x.dtype) if ret_final else None
    out = cc._fwd(x, weight, bias, seq, init, final, silu)
    dx, dweight, dbias, dinit = cc._bwd(x, weight, bias, seq, init, dout, dfinal, need_dinit, silu)

    rec = {"x": x, "weight": weight, "bias": bias, "initial_states": init, "seq_idx": seq,
           "dout": dout, "dfinal_states": dfinal, "out": out, "final_states": final, "dx": dx,
           "dweight": dweight, "dbias": dbias, "dinit": dinit}
    arrays = {}
    for k, v in rec.items():
        if v is None:
            continue
        arrays[f"{name}/{k}"] = v.numpy() if v.dtype == torch.int32 else v.float().numpy()
    meta = {"name": name, "B": B, "T": T, "D": D, "W": W, "x_dtype": xdt, "w_dtype": wdt,
            "bias": has_bias, "silu": silu, "init": has_init, "seq": has_seq,
            "return_final_states": ret_final, "dfinal": has_dfinal, "need_dinit": need_dinit}
    return arrays, meta


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True,
                    help="checkout of jxiong21029/causal-conv1d-triton (the directory holding the "
                         "causal_conv1d_triton package)")
    args = ap.parse_args()
    cc = load_reference(args.ref)
    arrays, metas = {}, []
    for i, spec in enumerate(CASES):
        t0 = time.time()
        a, m = run_case(cc, i, spec)
        arrays.update(a)
        metas.append(m)
        print(f"{m['name']}: {time.time() - t0:.1f}s", flush=True)
    arrays["__meta__"] = np.array(json.dumps(metas))
    np.savez_compressed(OUT, **arrays)
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
