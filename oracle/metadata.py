"""Per-row key bounds of the varlen path, restated in numpy (test oracle only).

The reference imports ``SwitchAttentionMetadata`` / ``build_switch_attention_metadata``
from a ``metadata`` module that is not part of the repository
(``swiattn_gqa_prefill_varlen.py:27``).  Its fields and lengths are fixed by the
wrapper's validation (``:360-374``: seven int32 vectors of lengths
``(Sq, Skv, Sq, Skv, Sq, Sq, Sq)``) and their meaning by the kernel
(``:134-137`` row bounds, ``:186-196`` legality ``start <= key < end`` with
``end`` exclusive).  For one sequence the bounds must reduce to the fixed-length
kernel's masks (``swiattn_gqa_prefill.py:145-158``: full ``key <= t``, local
``t - W + 1 <= key <= t``); for packed sequences the same masks apply inside
each segment.  This file states exactly that.
"""
from __future__ import annotations

import numpy as np


def build_metadata(q_len: int, kv_len: int, window: int, cu_seqlens=None) -> dict[str, np.ndarray]:
    if cu_seqlens is None:
        cu = np.array([0, q_len], dtype=np.int64)
    else:
        cu = np.asarray(cu_seqlens, dtype=np.int64)
        assert cu[0] == 0 and cu[-1] == q_len and kv_len == q_len
    t = np.arange(q_len, dtype=np.int64)
    seg = np.searchsorted(cu, t, side="right") - 1
    seg_start = cu[seg]
    q_positions = t - seg_start
    full_starts = seg_start
    local_starts = np.maximum(seg_start, t - window + 1)
    causal_ends = t + 1
    if cu_seqlens is None:
        kv_t = np.arange(kv_len, dtype=np.int64)
        kv_positions = kv_t
        kv_segment_ids = np.zeros(kv_len, dtype=np.int64)
    else:
        kv_positions = q_positions
        kv_segment_ids = seg
    out = {
        "q_positions": q_positions,
        "kv_positions": kv_positions,
        "q_segment_ids": seg,
        "kv_segment_ids": kv_segment_ids,
        "full_starts": full_starts,
        "local_starts": local_starts,
        "causal_ends": causal_ends,
    }
    return {k: v.astype(np.int32) for k, v in out.items()}
