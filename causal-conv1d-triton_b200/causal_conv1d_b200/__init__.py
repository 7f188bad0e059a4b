"""B200-native (sm_100a) causal depthwise conv1d over channels-last inputs.

Drop-in for jxiong21029/causal-conv1d-triton (`from causal_conv1d_triton import causal_conv1d_fn`,
causal_conv1d_triton/__init__.py:1-3): `from causal_conv1d_b200 import causal_conv1d_fn`.
"""

from .causal_conv1d import causal_conv1d_fn, causal_conv1d_update, seq_idx_from_cu_seqlens
from .split_conv1d import split_conv1d

__all__ = ["causal_conv1d_fn", "causal_conv1d_update", "seq_idx_from_cu_seqlens", "split_conv1d"]
