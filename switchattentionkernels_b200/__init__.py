"""B200-native (sm_100a) Switch Attention GQA prefill.

Public API (drop-in for YushengZhao/SwitchAttentionKernels):

* ``build_switch_query_indices(full_mask)``
* ``switch_gqa_prefill_forward(q, k, v, full_query_indices, local_query_indices, *, metadata=None, ...)``
* ``SwitchAttentionMetadata``, ``build_switch_attention_metadata``

Extensions: ``build_switch_query_indices_batched`` (B > 1 routing masks),
``build_switch_query_indices_from_router`` (router scores or logits compacted
in one kernel), ``sharded_switch_gqa_prefill_forward`` (one process per GPU,
(batch, KV group) units sharded across ranks, optional NCCL all-gather of
O/LSE), ``context_parallel.context_parallel_switch_gqa_prefill_forward``
(one long packed batch split by rows across ranks) and
``switch_gqa_decode_forward`` (one new token per sequence against a KV cache).
"""
from ._core import build_switch_query_indices_batched, build_switch_query_indices_from_router
from .decode import switch_gqa_decode_forward
from .metadata import SwitchAttentionMetadata, build_switch_attention_metadata, cu_seqlens_from_lengths
from .swiattn_gqa_prefill_varlen import build_switch_query_indices, switch_gqa_prefill_forward

__all__ = [
    "SwitchAttentionMetadata",
    "build_switch_attention_metadata",
    "build_switch_query_indices",
    "build_switch_query_indices_batched",
    "build_switch_query_indices_from_router",
    "cu_seqlens_from_lengths",
    "switch_gqa_decode_forward",
    "switch_gqa_prefill_forward",
]
