"""Plain PyTorch fp32 restatement of the reference's forward and backward, for the full-shape
parity tests. TEST INFRASTRUCTURE ONLY.

The C oracle (oracle/) is the pinned checker, but at the BASELINE configurations' full sizes
(up to 4.3e9 elements per tensor) it would take minutes per tensor on the host. This module
restates the same per-element semantics with torch tensor operations on the GPU, in fp32, over
chunks of batch rows, so every element of every output can be checked; the tests also compare
sampled rows against the oracle, which ties the two checkers together.

Semantics follow jxiong21029/causal-conv1d-triton, causal_conv1d_triton/causal_conv1d.py:
  forward  `_fwd_kernel` :129-143 (taps oldest first, seq_idx mask, bias, padding rows to zero,
           SiLU) and the loaders :17-41 (rows t < 0 read initial_states and carry seq_idx[b, 0];
           other rows outside [0, T) are zero with seq id -1);
  backward `_bwd_kernel` :274-321 (dz from the recomputed z, dx as the anti-causal conv masked to
           the same sequence, dfinal_states added to the last W-1 rows of concat(init, x), the
           dinit rows, dweight / dbias sums).
The weight / bias gradient sums accumulate in fp64.
"""

from __future__ import annotations

import torch


def _seq_ext(seq, has_init, pad):
    """(b, pad + T) sequence ids of rows -pad .. T-1 (None without seq_idx)."""
    if seq is None:
        return None
    b = seq.shape[0]
    pre = seq[:, :1].expand(b, pad) if has_init else torch.full((b, pad), -1, dtype=seq.dtype,
                                                                 device=seq.device)
    return torch.cat([pre, seq], 1)


def forward_chunk(x, weight, bias, init, seq, silu):
    """Returns (z, out) in fp32 for a chunk of batch rows: z is the pre-activation (zero at
    padding rows), out = act(z)."""
    b, T, D = x.shape
    W = weight.shape[1]
    pad = W - 1
    wf = weight.float()
    xf = x.float()
    pre = init.float() if init is not None else torch.zeros(b, pad, D, device=x.device)
    xp = torch.cat([pre, xf], 1)  # row e <-> t = e - pad
    sp = _seq_ext(seq, init is not None, pad)
    z = xf * wf[:, pad]
    for k in range(pad):
        tap = xp[:, k:k + T] * wf[:, k]
        if seq is not None:
            tap = torch.where((sp[:, k:k + T] == seq).unsqueeze(-1), tap, 0.0)
        z = z + tap
    if bias is not None:
        z = z + bias.float()
    if seq is not None:
        z = torch.where((seq < 0).unsqueeze(-1), 0.0, z)
    out = z * torch.sigmoid(z) if silu else z
    return z, out


def backward_chunk(x, weight, bias, init, seq, dout, dfinal, silu):
    """Returns (dx, dinit, dweight_f64, dbias_f64) for a chunk of batch rows: dx (b, T, D) and
    dinit (b, W-1, D) in fp32 (dinit None without init), the weight / bias gradient sums of this
    chunk in fp64."""
    b, T, D = x.shape
    W = weight.shape[1]
    pad = W - 1
    wf = weight.float()
    z, _ = forward_chunk(x, weight, bias, init, seq, silu)
    dz = dout.float()
    if silu:
        s = torch.sigmoid(z)
        dz = dz * s * (1 + z * (1 - s))
    if seq is not None:
        dz = torch.where((seq < 0).unsqueeze(-1), 0.0, dz)
    zeros = torch.zeros(b, pad, D, device=x.device)
    dz_ext = torch.cat([zeros, dz, zeros], 1)  # index i <-> row i - pad
    sp = _seq_ext(seq, init is not None, pad)  # rows -pad .. T-1
    sp2 = None
    if seq is not None:
        sp2 = torch.cat([sp, torch.full((b, pad), -1, dtype=sp.dtype, device=sp.device)], 1)
    # G[r] = sum_j w[pad - j] dz[r + j] for rows r = -pad .. T-1 (j >= 1 masked to r's sequence).
    G = dz_ext[:, 0:T + pad] * wf[:, pad]
    for j in range(1, W):
        term = dz_ext[:, j:j + T + pad] * wf[:, pad - j]
        if seq is not None:
            term = torch.where((sp2[:, j:j + T + pad] == sp).unsqueeze(-1), term, 0.0)
        G = G + term
    dinit_rows = G[:, :pad]
    dx = G[:, pad:].clone()
    dinit = dinit_rows.clone() if init is not None else None
    if dfinal is not None:  # final[p] = concat(init, x)[T - pad + p]
        for p in range(pad):
            r = T - pad + p
            if r >= 0:
                dx[:, r] += dfinal[:, p].float()
            elif dinit is not None:
                dinit[:, r + pad] += dfinal[:, p].float()
    pre = init.float() if init is not None else torch.zeros(b, pad, D, device=x.device)
    xp = torch.cat([pre, x.float()], 1)
    dw = torch.empty(D, W, dtype=torch.float64, device=x.device)
    for k in range(W):
        prod = dz * xp[:, k:k + T]
        if seq is not None and k < pad:
            prod = torch.where((sp[:, k:k + T] == seq).unsqueeze(-1), prod, 0.0)
        dw[:, k] = prod.sum(dim=(0, 1), dtype=torch.float64)
    db = dz.sum(dim=(0, 1), dtype=torch.float64) if bias is not None else None
    return dx, dinit, dw, db
