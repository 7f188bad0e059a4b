"""Decode-time state update (causal_conv1d_update, C entry cc1d_update) on the GPU.

- Token-by-token decoding equals the forward with initial states (causal_conv1d_fn), exactly:
  both compute every output element with the same fp32 operations in the same order.
- Multi-row updates, slot indices (including a negative slot that must be left untouched), fp32
  and widths on both sides of the TMA forward's range are checked against the CPU oracle.
"""

import numpy as np
import pytest
import torch

from _tol import assert_bitexact, assert_close
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("W", [2, 4, 8])
def test_decode_steps_equal_forward(dt, W):
    from causal_conv1d_b200 import causal_conv1d_fn, causal_conv1d_update

    g = torch.Generator().manual_seed(W)
    B, T, D = 3, 24, 256
    x = torch.randn(B, T, D, generator=g).to(dt).to(DEV)
    w = (torch.randn(D, W, generator=g) / W**0.5).to(DEV)
    b = (torch.randn(D, generator=g) * 0.3).to(DEV)
    init = torch.randn(B, W - 1, D, generator=g).to(dt).to(DEV)
    full, final = causal_conv1d_fn(x, w, b, initial_states=init, return_final_states=True,
                                   activation="silu")
    state = init.clone()
    outs = [causal_conv1d_update(x[:, t], state, w, b, activation="silu") for t in range(T)]
    assert torch.equal(torch.stack(outs, 1), full)
    assert torch.equal(state, final)


@pytest.mark.parametrize("L", [1, 3, 10])
@pytest.mark.parametrize("W", [4, 12])
def test_update_matches_oracle_with_slots(L, W):
    from causal_conv1d_b200 import causal_conv1d_update

    g = torch.Generator().manual_seed(L * 31 + W)
    B, D, n_slots = 4, 72, 6
    x = torch.randn(B, L, D, generator=g).to(torch.bfloat16)
    w = torch.randn(D, W, generator=g) / W**0.5
    b = torch.randn(D, generator=g) * 0.3
    state0 = torch.randn(n_slots, W - 1, D, generator=g).to(torch.bfloat16)
    slots = torch.tensor([5, 0, -1, 2], dtype=torch.int32)
    sd = state0.to(DEV)
    out = causal_conv1d_update(x.to(DEV), sd, w.to(DEV), b.to(DEV), activation="silu",
                               conv_state_indices=slots.to(DEV))
    out, sd = out.cpu(), sd.cpu()
    for i, s in enumerate(slots.tolist()):
        if s < 0:
            continue
        ro, rs = oracle.update(x[i:i + 1], state0[s:s + 1], w, b, silu=True)
        assert_close(out[i:i + 1], torch.from_numpy(ro).to(torch.bfloat16).float(), "bf16", "out")
        assert_bitexact(sd[s:s + 1], torch.from_numpy(rs).to(torch.bfloat16).float(), "state")
    untouched = [s for s in range(n_slots) if s not in slots.tolist()]
    assert torch.equal(sd[untouched], state0[untouched])


def test_update_fp32_no_activation():
    from causal_conv1d_b200 import causal_conv1d_update

    g = torch.Generator().manual_seed(2)
    B, L, D, W = 2, 5, 40, 3
    x = torch.randn(B, L, D, generator=g)
    w = torch.randn(D, W, generator=g)
    st = torch.randn(B, W - 1, D, generator=g)
    sd = st.to(DEV)
    out = causal_conv1d_update(x.to(DEV), sd, w.to(DEV)).cpu()
    ro, rs = oracle.update(x, st, w, None, silu=False)
    assert_close(out, ro, "f32", "out")
    assert_bitexact(sd.cpu(), rs, "state")


@pytest.mark.parametrize("case", ["odd_dim", "dim_6_mod_4", "fp32_state", "odd_row_stride", "vec_path"])
def test_update_paths_match_oracle(case):
    """The vector decode kernel (D and the strides multiples of 4 bf16 channels, x and state of one
    type) and the general one (every other case) give the oracle's results."""
    from causal_conv1d_b200 import causal_conv1d_update

    g = torch.Generator().manual_seed(len(case))
    B, L, W = 3, 4, 4
    D = {"odd_dim": 37, "dim_6_mod_4": 66}.get(case, 64)
    sdt = torch.float32 if case == "fp32_state" else torch.bfloat16
    x = torch.randn(B, L, D, generator=g).to(torch.bfloat16)
    w = torch.randn(D, W, generator=g) / W**0.5
    b = torch.randn(D, generator=g) * 0.3
    st = torch.randn(B, W - 1, D, generator=g).to(sdt)
    xd = x.to(DEV)
    if case == "odd_row_stride":  # x read as a column slice of a wider buffer: row stride D + 1
        wide = torch.zeros(B, L, D + 1, dtype=torch.bfloat16, device=DEV)
        wide[..., 1:] = xd
        xd = wide[..., 1:]
    sd = st.to(DEV)
    out = causal_conv1d_update(xd, sd, w.to(DEV), b.to(DEV), activation="silu").cpu()
    ro, rs = oracle.update(x, st.float(), w, b, silu=True)
    assert_close(out, torch.from_numpy(ro).to(torch.bfloat16).float(), "bf16", "out")
    assert_bitexact(sd.cpu().float(), torch.from_numpy(rs).to(sdt).float(), "state")


def _seq_idx_reference(cu, T):
    out = np.full(T, -1, np.int32)
    for i in range(len(cu) - 1):
        out[cu[i]:cu[i + 1]] = i
    return out


@pytest.mark.parametrize("rows", [1, 3])
def test_seq_idx_from_cu_seqlens(rows):
    from causal_conv1d_b200 import seq_idx_from_cu_seqlens

    g = torch.Generator().manual_seed(rows)
    T, n = 5000, 9
    cus = []
    for _ in range(rows):
        lens = torch.randint(0, 900, (n,), generator=g)
        cu = torch.cat([torch.zeros(1, dtype=torch.long), torch.cumsum(lens, 0)]).clamp(max=T)
        cus.append(cu)
    cu = torch.stack(cus) if rows > 1 else cus[0]
    got = seq_idx_from_cu_seqlens(cu.to(DEV), T).cpu().numpy()
    for r in range(rows):
        ref = _seq_idx_reference(cus[r].tolist(), T)
        # empty sequences (equal boundaries) contain no position, so ids can skip a value
        assert np.array_equal(got[r], ref)


def test_varlen_via_cu_seqlens_matches_per_sequence_calls():
    """Packing sequences with seq_idx from cu_seqlens equals running each sequence alone."""
    from causal_conv1d_b200 import causal_conv1d_fn, seq_idx_from_cu_seqlens

    g = torch.Generator().manual_seed(11)
    lens = [37, 200, 5, 130]
    T, D, W = sum(lens) + 20, 136, 4
    x = torch.randn(1, T, D, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(D, W, generator=g) * 0.5).to(DEV)
    b = torch.randn(D, generator=g).to(DEV)
    cu = torch.tensor([0] + list(np.cumsum(lens)), device=DEV)
    seq = seq_idx_from_cu_seqlens(cu, T)
    packed = causal_conv1d_fn(x, w, b, seq_idx=seq, activation="silu")
    start = 0
    for n in lens:
        alone = causal_conv1d_fn(x[:, start:start + n], w, b, activation="silu")
        assert torch.equal(packed[:, start:start + n], alone)
        start += n
    assert (packed[:, start:] == 0).all()
