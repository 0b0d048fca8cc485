"""Position metadata for varlen (packed) Switch Attention prefill.

The reference imports ``SwitchAttentionMetadata`` and
``build_switch_attention_metadata`` from a ``metadata`` module that its
repository does not contain (``swiattn_gqa_prefill_varlen.py:27``).  The field
names, dtypes and lengths below are the ones its wrapper validates
(``swiattn_gqa_prefill_varlen.py:360-383``: seven contiguous int32 vectors of
lengths ``(Sq, Skv, Sq, Skv, Sq, Sq, Sq)``) and the call signature is the one it
uses (``:353-359``).  The kernel consumes ``full_starts`` / ``local_starts`` as
inclusive lower key bounds and ``causal_ends`` as the exclusive upper bound of
each query row (``:134-137,186-196``).

For one sequence the bounds reproduce the fixed-length masks
(``swiattn_gqa_prefill.py:145-158``).  ``cu_seqlens`` (an addition: the
reference's builder is not available) packs several sequences: row ``t`` of
segment ``s`` attends inside its own segment only.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native


@dataclass(frozen=True)
class SwitchAttentionMetadata:
    q_positions: torch.Tensor     # int32 [Sq]   position of each query row inside its sequence
    kv_positions: torch.Tensor    # int32 [Skv]  position of each key row inside its sequence
    q_segment_ids: torch.Tensor   # int32 [Sq]   sequence index of each query row
    kv_segment_ids: torch.Tensor  # int32 [Skv]  sequence index of each key row
    full_starts: torch.Tensor     # int32 [Sq]   first key of a full-attention row
    local_starts: torch.Tensor    # int32 [Sq]   first key of a sliding-window row
    causal_ends: torch.Tensor     # int32 [Sq]   one past the last key of a row


def build_switch_attention_metadata(q_len: int, kv_len: int, *, device, window_size: int,
                                    cu_seqlens: torch.Tensor | None = None) -> SwitchAttentionMetadata:
    """Build the per-row key bounds on ``device`` with one CUDA kernel.

    ``cu_seqlens``: optional int32 ``[nseq + 1]`` cumulative sequence lengths
    (``cu_seqlens[0] == 0``, ``cu_seqlens[-1] == q_len``; requires ``kv_len == q_len``).
    """
    if window_size <= 0:
        raise ValueError("window_size must be positive")
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("metadata must be built on a supported accelerator device")
    cu = None
    nseg = 0
    if cu_seqlens is not None:
        cu = torch.as_tensor(cu_seqlens).to(device=device, dtype=torch.int32).contiguous()
        if cu.ndim != 1 or cu.numel() < 2:
            raise ValueError("cu_seqlens must be a 1-D tensor with at least two entries")
        if kv_len != q_len:
            raise ValueError("packed metadata requires kv_len == q_len")
        nseg = cu.numel() - 1
    mk = lambda n: torch.empty(n, dtype=torch.int32, device=device)  # noqa: E731
    qp, kp, qs, ks, fs, ls, ce = mk(q_len), mk(kv_len), mk(q_len), mk(kv_len), mk(q_len), mk(q_len), mk(q_len)
    lib = _native.load()
    with torch.cuda.device(device):
        rc = lib.swa_build_metadata(_native.ptr(cu), nseg, q_len, kv_len, int(window_size), _native.ptr(qp),
                                    _native.ptr(kp), _native.ptr(qs), _native.ptr(ks), _native.ptr(fs),
                                    _native.ptr(ls), _native.ptr(ce), _native.stream_ptr(device))
    _native.check(rc, "build_switch_attention_metadata")
    return SwitchAttentionMetadata(qp, kp, qs, ks, fs, ls, ce)


def cu_seqlens_from_lengths(lengths, device=None) -> torch.Tensor:
    """int32 ``[len(lengths) + 1]`` cumulative sequence lengths."""
    lengths = torch.as_tensor(lengths, dtype=torch.int64)
    cu = torch.zeros(lengths.numel() + 1, dtype=torch.int64)
    cu[1:] = torch.cumsum(lengths, 0)
    return cu.to(dtype=torch.int32, device=device)
