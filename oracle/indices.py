"""Index compaction and capacity buckets, restated in numpy (test oracle only).

Follows ``swiattn_gqa_prefill_varlen.py`` of the reference:

* ``compact_mask``      -- ``build_switch_query_indices`` (:306-322): the
  positions where the mask is True (full branch) and where it is False (local
  branch), each in increasing order, as int32;
* ``bucket_capacity``   -- the power-of-two capacity of ``_prepare_indices``
  (:287-292);
* ``prepare_indices``   -- ``_prepare_indices`` (:271-304): -1 padding to the
  capacity, range and strict-increase validation with the reference messages;
* ``router_mask``       -- the routing decision that produces the mask (the
  router itself is outside the reference, ``README.md:85``, which fixes only
  the convention True = full attention): FP32 ``score > threshold``, or FP32
  ``logit_full - logit_local > threshold`` for ``(local, full)`` logit pairs.
"""
from __future__ import annotations

import math

import numpy as np

ERR_RANGE = "query index is outside [0, sequence_length)"
ERR_ORDER = "query indices must be strictly increasing"
ERR_COVER = "full and local query lists must cover the sequence"


def compact_mask(mask: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """``positions[mask], positions[~mask]`` (reference :321-322) for one row."""
    mask = np.asarray(mask, dtype=bool)
    assert mask.ndim == 1
    positions = np.arange(mask.size, dtype=np.int32)
    return positions[mask], positions[~mask]


def compact_mask_batched(mask: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Per-row compaction of a ``[B, S]`` mask into -1 padded ``[B, S]`` lists.

    Returns ``(full, local, counts)`` with ``counts[b] = (n_full, n_local)``.
    """
    mask = np.asarray(mask, dtype=bool)
    B, S = mask.shape
    full = np.full((B, S), -1, dtype=np.int32)
    local = np.full((B, S), -1, dtype=np.int32)
    counts = np.zeros((B, 2), dtype=np.int32)
    for b in range(B):
        f, l = compact_mask(mask[b])
        full[b, : f.size] = f
        local[b, : l.size] = l
        counts[b] = (f.size, l.size)
    return full, local, counts


def router_mask(router: np.ndarray, *, pair: bool, threshold: float = 0.0) -> np.ndarray:
    """Bool ``[B, S]`` routing mask of FP32 router outputs (``[B, S]`` or ``[B, S, 2]``).

    BF16 inputs are widened to FP32 exactly by the caller; the subtraction and
    the comparison are single FP32 operations, and NaN compares false (local).
    """
    r = np.asarray(router, dtype=np.float32)
    thr = np.float32(threshold)
    if pair:
        return (r[..., 1] - r[..., 0]) > thr
    return r > thr


def bucket_capacity(count: int, block_m: int) -> int:
    """Capacity bucket of ``_prepare_indices`` (reference :287-292).

    ``block_m << (bit_length(ceil(count / block_m)) - 1)``, doubled when that is
    still below ``count``: the smallest ``block_m * 2**j`` holding ``count``.
    """
    if count == 0:
        return 0
    padded = block_m << max(0, math.ceil(count / block_m).bit_length() - 1)
    if padded < count:
        padded <<= 1
    return padded


def prepare_indices(indices: np.ndarray, *, seq_len: int, block_m: int) -> tuple[np.ndarray, int]:
    """``_prepare_indices`` for one row (reference :271-304).

    Returns ``(padded[1, cap], count)``; raises ``ValueError`` with the reference
    message when an index is out of range or the list is not strictly increasing.
    """
    idx = np.asarray(indices, dtype=np.int32).reshape(1, -1)
    count = idx.shape[1]
    if count == 0:
        return idx, 0
    cap = bucket_capacity(count, block_m)
    padded = np.full((1, cap), -1, dtype=np.int32)
    padded[:, :count] = idx
    body = padded[:, :count]
    if bool(((body < 0) | (body >= seq_len)).any()):
        raise ValueError(ERR_RANGE)
    if count > 1 and bool((body[:, 1:] <= body[:, :-1]).any()):
        raise ValueError(ERR_ORDER)
    return padded, count
