"""Fixed-length Switch Attention GQA prefill (the reference's
``swiattn_gqa_prefill.py`` kernel, whose Python entry point is documented in
``README.md:60-83`` of YushengZhao/SwitchAttentionKernels).

``switch_gqa_prefill_forward(q, k, v, full_query_indices, local_query_indices,
window_size=1024)`` with the README's tensor contract.  The fixed-length kernel of
the reference takes a batch of index lists (``QueryIndices[batch, cap]``,
``swiattn_gqa_prefill.py:64-65``); here ``B > 1`` takes ``[B, N]`` lists padded
with ``-1`` (see ``build_switch_query_indices_batched``).

``block_m`` / ``block_k`` keep the values the reference kernel accepts
(``swiattn_gqa_prefill.py:39-40``) and do not change the result.
"""
from __future__ import annotations

from typing import Tuple

import torch

from . import _core

__all__ = ["build_switch_query_indices", "build_switch_query_indices_batched", "switch_gqa_prefill_forward"]

build_switch_query_indices = _core.build_switch_query_indices
build_switch_query_indices_batched = _core.build_switch_query_indices_batched


def switch_gqa_prefill_forward(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    full_query_indices: torch.Tensor,
    local_query_indices: torch.Tensor,
    *,
    window_size: int = 1024,
    sm_scale: float | None = None,
    block_m: int = 64,
    block_k: int = 64,
    num_stages: int = 2,
    threads: int = 128,
    validate: bool = True,
    query_counts: torch.Tensor | None = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """BF16 output ``[B, Sq, Hq, 128]`` and FP32 log2-LSE ``[B, Sq, Hq]``."""
    assert block_m in (64, 128), "qualified query tiles are BM64/BM128"
    assert block_k in (64, 128), "qualified key tiles are BK64/BK128"
    return _core.forward(q, k, v, full_query_indices, local_query_indices, window_size=window_size,
                         sm_scale=sm_scale, validate=validate, query_counts=query_counts)
