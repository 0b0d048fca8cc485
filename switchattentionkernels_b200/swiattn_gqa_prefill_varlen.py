"""Drop-in for the reference module ``swiattn_gqa_prefill_varlen`` (BF16 forward
prefill of Switch Attention GQA, varlen/metadata variant).

Same public names, signatures, return values and exceptions as
``swiattn_gqa_prefill_varlen.py:251-446`` of YushengZhao/SwitchAttentionKernels.
Underneath, the two TileLang branch launches are replaced by one persistent
sm_100a kernel (tcgen05 MMAs with TMEM accumulators, TMA-fed K/V ring, routed-Q
gather) reached through the C ABI of ``libswattn_b200.so``.

``block_m`` / ``block_k`` / ``num_stages`` / ``threads`` keep the reference's
accepted values and assertion messages (``:67-71``); the sm_100a kernel uses its
own tiling (256 routed rows x 128 keys), so they do not change the result.
``block_m`` still selects the capacity bucket of ``_prepare_indices``.
"""
from __future__ import annotations

from typing import Tuple

import torch

from . import _core
from .metadata import SwitchAttentionMetadata, build_switch_attention_metadata

__all__ = [
    "SwitchAttentionMetadata",
    "build_switch_attention_metadata",
    "build_switch_query_indices",
    "switch_gqa_prefill_forward",
]


def _validate_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    _core.validate_qkv(q, k, v)


def _prepare_indices(indices: torch.Tensor, *, seq_len: int, block_m: int) -> Tuple[torch.Tensor, torch.Tensor]:
    return _core.prepare_indices(indices, seq_len=seq_len, block_m=block_m)


def build_switch_query_indices(full_mask: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Compact a B=1 hard route mask into sorted full and local query positions.

    ``True`` routes to full causal attention and ``False`` to sliding-window
    attention (reference ``swiattn_gqa_prefill_varlen.py:306-322``).
    """
    return _core.build_switch_query_indices(full_mask)


def switch_gqa_prefill_forward(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    full_query_indices: torch.Tensor,
    local_query_indices: torch.Tensor,
    *,
    metadata: SwitchAttentionMetadata | None = None,
    window_size: int = 1024,
    sm_scale: float | None = None,
    block_m: int = 64,
    block_k: int = 64,
    num_stages: int = 1,
    threads: int = 128,
    validate: bool = True,
    query_counts: torch.Tensor | None = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Run Switch Attention prefill forward.

    Returns BF16 output ``[B, Sq, Hq, 128]`` and FP32 log2-LSE ``[B, Sq, Hq]``.  The
    two index lists must be sorted, disjoint, and together cover every query
    position exactly once.  Without ``metadata`` the rows use the single-sequence
    bounds (full: keys ``0..t``; local: keys ``t-W+1..t``), which is what the
    reference's default metadata encodes.  ``validate=False`` skips the index
    range / order checks and their device-to-host read.  ``query_counts``
    (extension): int32 ``[B, 2]`` per-row list lengths from
    ``build_switch_query_indices_batched``; the lists are then ``-1`` padded rows.
    """
    assert block_m == 64, "the qualified schedule is BM64"
    assert block_k == 64, "the qualified schedule is BK64"
    assert num_stages == 1, "the qualified schedule uses one stage"
    assert threads == 128, "the qualified schedule uses 128 threads"
    return _core.forward(q, k, v, full_query_indices, local_query_indices, metadata=metadata,
                         window_size=window_size, sm_scale=sm_scale, validate=validate, query_counts=query_counts)
