"""Host side of the Switch Attention prefill path: validation, index lists,
capacity buckets and the launch of the sm_100a kernels through the C ABI.

Error types and messages are the reference's
(``swiattn_gqa_prefill_varlen.py:251-304,313-320,345-393``).  Deliberate
supersets of the reference's accepted inputs:

* any ``Hq % Hkv == 0`` (the reference wrapper only accepts Hq=32, Hkv=8,
  ``:266-267``, although its kernels support any group size);
* ``B >= 1`` (the reference wrapper only accepts B=1, ``:346-347``; its
  fixed-length kernel already takes ``QueryIndices[batch, cap]``,
  ``swiattn_gqa_prefill.py:64-65``).  For ``B > 1`` the index lists are
  ``[B, N]`` int32 tensors whose rows end in ``-1`` padding, as produced by
  ``build_switch_query_indices_batched``.
"""
from __future__ import annotations

import ctypes
import math
import os

import torch

from . import _native
from .metadata import SwitchAttentionMetadata

LOG2E = 1.4426950408889634

ERR_RANGE = "query index is outside [0, sequence_length)"
ERR_ORDER = "query indices must be strictly increasing"
ERR_COVER = "full and local query lists must cover the sequence"
ERR_PAD = "query index padding (-1) must be trailing"
ERR_META = "invalid Switch Attention position metadata"

# When set (environment variable SWA_CHECK_STATUS=1), every forward call reads
# back the kernel's status word and raises if a device-side wait timed out.
# Without it no call synchronises; a caller that wants the status passes a
# device int32 tensor as ``status_out`` and reads it after its own synchronisation.
CHECK_DEVICE_STATUS = os.environ.get("SWA_CHECK_STATUS", "0") == "1"


# --------------------------------------------------------------------------- validation
def validate_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    """``_validate_qkv`` (reference ``swiattn_gqa_prefill_varlen.py:251-269``) minus the Hq=32/Hkv=8 pin."""
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise TypeError("Switch Attention prefill requires BF16 Q/K/V")
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise ValueError("Q/K/V must be tensors on a supported accelerator device")
    if not (q.is_contiguous() and k.is_contiguous() and v.is_contiguous()):
        raise ValueError("Q/K/V must be contiguous")
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("Q/K/V must use [B,S,H,D] layout")
    if k.shape != v.shape:
        raise ValueError("K and V must have identical shapes")
    if q.shape[0] != k.shape[0]:
        raise ValueError("Q and KV batch sizes must match")
    if q.shape[3] != 128 or k.shape[3] != 128:
        raise ValueError("the first kernel is specialized for head_dim=128")
    if q.shape[2] % k.shape[2]:
        raise ValueError("query heads must be divisible by KV heads")
    if not (q.device == k.device == v.device):
        raise ValueError("Q/K/V must be on the same device")


def bucket_capacity(count: int, block_m: int) -> int:
    """Capacity bucket (reference ``swiattn_gqa_prefill_varlen.py:287-292``)."""
    if count == 0:
        return 0
    padded = block_m << max(0, math.ceil(count / block_m).bit_length() - 1)
    if padded < count:
        padded <<= 1
    return padded


def _check_status_out(status_out, dev) -> None:
    if status_out is None:
        return
    if (not isinstance(status_out, torch.Tensor) or status_out.dtype != torch.int32 or status_out.device != dev
            or status_out.numel() < 1):
        raise ValueError("status_out must be an int32 tensor with at least one element on the device of Q")


def publish_status(status_word: torch.Tensor, status_out) -> None:
    """Hand the launch's device status word to the caller without a host sync.

    ``status_word`` is a one-element int32 device tensor that the launch's kernels
    write; it is copied into ``status_out[0]`` on the current stream.  A non-zero
    value (``_native.STATUS_*`` bits; ``STATUS_TIMEOUT`` = a device-side wait gave
    up) means the outputs of that call are undefined.  With SWA_CHECK_STATUS=1 the
    word is also read back here and raised as an exception.
    """
    if status_out is not None:
        status_out.view(-1)[:1].copy_(status_word.view(-1)[:1])
    if CHECK_DEVICE_STATUS:
        _raise_status(int(status_word.item()))


def _raise_status(status: int) -> None:
    order = [
        (_native.STATUS_FULL_RANGE, ERR_RANGE),
        (_native.STATUS_FULL_PAD, ERR_PAD),
        (_native.STATUS_FULL_ORDER, ERR_ORDER),
        (_native.STATUS_LOCAL_RANGE, ERR_RANGE),
        (_native.STATUS_LOCAL_PAD, ERR_PAD),
        (_native.STATUS_LOCAL_ORDER, ERR_ORDER),
        (_native.STATUS_COVER, ERR_COVER),
    ]
    for bit, msg in order:
        if status & bit:
            raise ValueError(msg)
    if status & _native.STATUS_TIMEOUT:
        raise RuntimeError("Switch Attention kernel: a device-side wait timed out")


# --------------------------------------------------------------------------- index lists
def build_switch_query_indices(full_mask: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Compact a B=1 hard route mask into sorted full and local query positions.

    Same contract as the reference (``swiattn_gqa_prefill_varlen.py:306-322``):
    ``True`` routes a position to full causal attention, ``False`` to the sliding
    window; both outputs are int32 and strictly increasing.  Computed by one
    ballot/scan CUDA kernel; one device-to-host read sizes the outputs (the
    reference's ``positions[mask]`` performs the same synchronisation).
    """
    if full_mask.ndim == 2:
        if full_mask.shape[0] != 1:
            raise ValueError("the first kernel supports B=1 routing")
        full_mask = full_mask[0]
    if full_mask.ndim != 1 or full_mask.dtype != torch.bool or not full_mask.is_cuda:
        raise TypeError("full_mask must be a device-resident bool tensor with shape [S] or [1,S]")
    full, local, counts = build_switch_query_indices_batched(full_mask.unsqueeze(0))
    n_full, n_local = (int(x) for x in counts[0].tolist())
    return full[0, :n_full], local[0, :n_local]


def build_switch_query_indices_batched(full_mask: torch.Tensor):
    """``[B, S]`` bool mask -> ``(full [B,S], local [B,S], counts [B,2])`` on the device, no host sync.

    Row ``b`` of ``full`` / ``local`` holds the routed positions in increasing
    order followed by ``-1``; ``counts[b] = (n_full, n_local)``.
    """
    if full_mask.ndim != 2 or full_mask.dtype != torch.bool or not full_mask.is_cuda:
        raise TypeError("full_mask must be a device-resident bool tensor with shape [B,S]")
    mask = full_mask.contiguous()
    B, S = mask.shape
    dev = mask.device
    full = torch.empty((B, S), dtype=torch.int32, device=dev)
    local = torch.empty((B, S), dtype=torch.int32, device=dev)
    counts = torch.zeros((B, 2), dtype=torch.int32, device=dev)
    if B == 0 or S == 0:
        return full, local, counts
    lib = _native.load()
    nws = int(lib.swa_compact_workspace_elems(B, S))
    ws = torch.empty(max(nws, 1), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        rc = lib.swa_compact_mask_ws(_native.ptr(mask), B, S, _native.ptr(full), _native.ptr(local),
                                     _native.ptr(counts), _native.ptr(ws), nws, _native.stream_ptr(dev))
    _native.check(rc, "build_switch_query_indices")
    return full, local, counts


def build_switch_query_indices_from_router(router_out: torch.Tensor, *, threshold: float = 0.0, pair: bool = False):
    """Router output -> ``(full [B,S], local [B,S], counts [B,2])`` in one kernel, no mask buffer.

    The reference leaves the router outside the kernel and compacts the bool
    mask it yields (``README.md:85``); this fuses that step with the compaction.
    ``router_out``: device-resident BF16 or FP32.  ``pair=False``: ``[S]`` or
    ``[B, S]`` scores, a token goes to full attention iff ``score > threshold``.
    ``pair=True``: ``[S, 2]`` or ``[B, S, 2]`` logits ``(local, full)``, full iff
    ``logit_full - logit_local > threshold`` (0: argmax with ties to local).
    Compared in FP32; NaN routes to local.  Outputs as
    ``build_switch_query_indices_batched`` (a 1-D / 2-D input is one batch row).
    """
    if not isinstance(router_out, torch.Tensor) or not router_out.is_cuda:
        raise TypeError("router_out must be a device-resident tensor")
    if router_out.dtype == torch.bfloat16:
        dtype = _native.ROUTER_BF16
    elif router_out.dtype == torch.float32:
        dtype = _native.ROUTER_F32
    else:
        raise TypeError("router_out must be bfloat16 or float32")
    r = router_out
    if pair:
        if r.ndim == 2:
            r = r.unsqueeze(0)
        if r.ndim != 3 or r.shape[2] != 2:
            raise ValueError("with pair=True router_out must have shape [S, 2] or [B, S, 2]")
    else:
        if r.ndim == 1:
            r = r.unsqueeze(0)
        if r.ndim != 2:
            raise ValueError("router_out must have shape [S] or [B, S]")
    r = r.contiguous()
    B, S = int(r.shape[0]), int(r.shape[1])
    dev = r.device
    full = torch.empty((B, S), dtype=torch.int32, device=dev)
    local = torch.empty((B, S), dtype=torch.int32, device=dev)
    counts = torch.zeros((B, 2), dtype=torch.int32, device=dev)
    if B == 0 or S == 0:
        return full, local, counts
    lib = _native.load()
    nws = int(lib.swa_compact_workspace_elems(B, S))
    ws = torch.empty(max(nws, 1), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        rc = lib.swa_compact_router_ws(_native.ptr(r), dtype, 1 if pair else 0, float(threshold), B, S,
                                       _native.ptr(full), _native.ptr(local), _native.ptr(counts),
                                       _native.ptr(ws), nws, _native.stream_ptr(dev))
    _native.check(rc, "build_switch_query_indices_from_router")
    return full, local, counts


def prepare_indices(indices: torch.Tensor, *, seq_len: int, block_m: int) -> tuple[torch.Tensor, torch.Tensor]:
    """``_prepare_indices`` (reference ``swiattn_gqa_prefill_varlen.py:271-304``).

    Returns ``(padded [1, cap], count [1])`` with ``cap`` the power-of-two
    capacity bucket and ``-1`` fill; raises the reference's ``ValueError`` for an
    out-of-range or non-increasing list (one device-to-host read, as in the
    reference).
    """
    if indices.ndim == 1:
        indices = indices.unsqueeze(0)
    if indices.ndim != 2 or indices.shape[0] != 1:
        raise ValueError("the first kernel accepts one batch of query indices")
    if indices.device.type != "cuda":
        raise ValueError("query indices must be on a supported accelerator device")
    indices = indices.to(dtype=torch.int32).contiguous()
    count = int(indices.shape[1])
    dev = indices.device
    if count == 0:
        return indices, torch.zeros((1,), dtype=torch.int32, device=dev)
    cap = bucket_capacity(count, block_m)
    padded = torch.empty((1, cap), dtype=torch.int32, device=dev)
    count_t = torch.empty((1,), dtype=torch.int32, device=dev)
    status = torch.zeros((1,), dtype=torch.int32, device=dev)
    lib = _native.load()
    with torch.cuda.device(dev):
        rc = lib.swa_prepare_indices(_native.ptr(indices), 1, count, int(seq_len), 0, cap, _native.ptr(padded),
                                     _native.ptr(count_t), _native.ptr(status), _native.STATUS_FULL_RANGE,
                                     _native.STATUS_FULL_ORDER, 0, _native.stream_ptr(dev))
    _native.check(rc, "_prepare_indices")
    st = int(status.item())
    if st & _native.STATUS_FULL_RANGE:
        raise ValueError(ERR_RANGE)
    if st & _native.STATUS_FULL_ORDER:
        raise ValueError(ERR_ORDER)
    return padded, count_t


# --------------------------------------------------------------------------- forward
def _check_metadata(metadata: SwitchAttentionMetadata, q: torch.Tensor, q_len: int, kv_len: int) -> None:
    """Metadata validation of the reference wrapper (``swiattn_gqa_prefill_varlen.py:360-383``)."""
    tensors = (metadata.q_positions, metadata.kv_positions, metadata.q_segment_ids, metadata.kv_segment_ids,
               metadata.full_starts, metadata.local_starts, metadata.causal_ends)
    expected = (q_len, kv_len, q_len, kv_len, q_len, q_len, q_len)
    for t, n in zip(tensors, expected):
        if (t.device != q.device or t.dtype != torch.int32 or t.ndim != 1 or t.numel() != n
                or not t.is_contiguous()):
            raise ValueError(ERR_META)


def _index_rows(indices: torch.Tensor, B: int, device: torch.device, name: str) -> torch.Tensor:
    if not isinstance(indices, torch.Tensor):
        raise TypeError(f"{name} must be a tensor")
    if indices.device.type != "cuda":
        raise ValueError("query indices must be on a supported accelerator device")
    if indices.device != device:
        raise ValueError("query indices must be on the same device as Q")
    if B == 1:
        if indices.ndim == 1:
            indices = indices.unsqueeze(0)
        if indices.ndim != 2 or indices.shape[0] != 1:
            raise ValueError("the first kernel accepts one batch of query indices")
    elif indices.ndim != 2 or indices.shape[0] != B:
        raise ValueError(f"{name} must have shape [B, N] (rows padded with -1) when B > 1")
    return indices.to(dtype=torch.int32).contiguous()


_SM_COUNTS: dict = {}


def _num_sms(lib, dev) -> int:
    idx = dev.index if dev.index is not None else (torch.cuda.current_device() if dev.type == "cuda" else 0)
    if idx not in _SM_COUNTS:
        _SM_COUNTS[idx] = int(lib.swa_num_sms(idx))
    return _SM_COUNTS[idx]


def split_plan(B: int, kv_len: int, Hq: int, Hkv: int, n_full: int, n_local: int, window_size: int, device, *,
               n_bg: int = 0, request_tiles: int = 0) -> tuple[int, int]:
    """``(split_tiles, scratch_bytes)`` of a launch's key split (``swa_prefill_split_plan``):
    ``(0, 0)`` when long full-causal units are not split.  ``n_full`` / ``n_local``:
    the largest per-row counts (or the list capacities); ``n_bg``: units of the
    launch (0: all ``B * Hkv``); ``request_tiles`` > 0 asks for that piece length."""
    lib = _native.load()
    dev = torch.device(device)
    tiles = ctypes.c_int(0)
    nbytes = int(lib.swa_prefill_split_plan(B, kv_len, Hq, Hkv, n_full, n_local, n_bg, int(window_size),
                                            _num_sms(lib, dev), int(request_tiles), ctypes.byref(tiles)))
    return (tiles.value, nbytes) if nbytes else (0, 0)


def forward(q, k, v, full_query_indices, local_query_indices, *, metadata=None, window_size=1024, sm_scale=None,
            validate=True, query_counts=None, bg_list=None, out=None, lse=None, prefill_events=None,
            status_out=None, key_split="auto", max_counts=None):
    """Both branches of Switch Attention GQA prefill (see ``switch_gqa_prefill_forward``).

    ``query_counts``: optional int32 ``[B, 2]`` device tensor of per-row
    ``(n_full, n_local)`` as returned by ``build_switch_query_indices_batched``;
    the lists are then read as ``-1`` padded rows for any ``B`` and, with
    ``validate=False``, no validation kernel runs.
    ``bg_list`` (``b * Hkv + g`` ids) restricts the launch to those (batch, KV
    group) units; ``out`` / ``lse`` may be given to write into existing buffers
    (rows outside the computed units are left untouched).
    ``prefill_events``: optional pair of CUDA events recorded on the current
    stream right before and after the prefill kernel launch (kernel timing).
    ``status_out``: optional int32 device tensor; element 0 receives the call's
    status word on the current stream (no host sync): 0 when the results are
    valid; otherwise the validation bits of an unvalidated call
    (``validate=False``: the kernel then wrote nothing) or ``STATUS_TIMEOUT``
    (a device-side wait gave up; O / LSE are undefined).
    ``key_split``: ``"auto"`` (default) lets the launch split long full-causal
    units over several SMs when few such units would otherwise outlast the
    rest of the work (``swa_prefill_split_plan``; a scratch buffer is then
    allocated for the partial rows); an int asks for pieces of about that many
    128-key tiles; ``None`` / ``0`` never splits.  The plan needs the largest
    per-row counts: the list lengths for the reference's ``B == 1`` form, the
    counts read back with the validation status otherwise, or ``max_counts``
    (``(n_full, n_local)`` known on the host, for callers that skip
    validation); without any of these it sees only the list capacities.
    """
    validate_qkv(q, k, v)
    if window_size <= 0:
        raise ValueError("window_size must be positive")
    host_counts = None
    if max_counts is not None:
        if len(max_counts) != 2 or int(max_counts[0]) < 0 or int(max_counts[1]) < 0:
            raise ValueError("max_counts must be a pair of non-negative counts (n_full, n_local)")
        host_counts = (int(max_counts[0]), int(max_counts[1]))
    if key_split not in (None, False, "auto") and (isinstance(key_split, (str, bool)) or int(key_split) < 0):
        raise ValueError("key_split must be 'auto', None or a non-negative number of key tiles")
    B, q_len, Hq, D = q.shape
    kv_len, Hkv = k.shape[1], k.shape[2]
    dev = q.device
    if metadata is not None:
        _check_metadata(metadata, q, q_len, kv_len)
    padded = B > 1 or query_counts is not None
    full = _index_rows(full_query_indices, B, dev, "full_query_indices")
    local = _index_rows(local_query_indices, B, dev, "local_query_indices")
    scale = (sm_scale if sm_scale is not None else (1.0 / D) ** 0.5) * LOG2E
    if not scale > 0:
        raise ValueError("sm_scale must be positive")
    if query_counts is not None:
        if (query_counts.device != dev or query_counts.dtype != torch.int32 or tuple(query_counts.shape) != (B, 2)
                or not query_counts.is_contiguous()):
            raise ValueError("query_counts must be a contiguous int32 [B, 2] tensor on the device of Q")

    n_full, n_local = int(full.shape[1]), int(local.shape[1])
    if not padded and not validate and n_full + n_local != q_len:
        raise ValueError(ERR_COVER)
    if bg_list is not None:
        bg_list = torch.as_tensor(bg_list, dtype=torch.int32)
        if bg_list.ndim != 1 or bg_list.numel() == 0:
            raise ValueError("bg_list must be a non-empty 1-D list of b * Hkv + g unit ids")
        if bool(((bg_list < 0) | (bg_list >= B * Hkv)).any()):
            raise ValueError("bg_list entries must lie in [0, B * Hkv)")
    _check_status_out(status_out, dev)
    lib = _native.load()
    stream = _native.stream_ptr(dev)
    ws = torch.zeros(4 + 2 * B, dtype=torch.int32, device=dev)
    status = ws[2:3]
    counts = ws[4:]
    gate = None
    counts_arg, batch_major = None, 0
    with torch.cuda.device(dev):
        if not padded:
            # the reference's form: B == 1, every entry of each list is a routed row
            if validate:
                for t, n, rb, ob in ((full, n_full, _native.STATUS_FULL_RANGE, _native.STATUS_FULL_ORDER),
                                     (local, n_local, _native.STATUS_LOCAL_RANGE, _native.STATUS_LOCAL_ORDER)):
                    if n:
                        _native.check(lib.swa_prepare_indices(_native.ptr(t), 1, n, q_len, 0, 0, None,
                                                              _native.ptr(counts), _native.ptr(status), rb, ob, 0,
                                                              stream), "index validation")
                _raise_status(int(status.item()))
            host_counts = (n_full, n_local)
            if n_full + n_local != q_len:
                raise ValueError(ERR_COVER)
        elif validate or query_counts is None:
            for t, n, row, rb, ob, pb in (
                    (full, n_full, 0, _native.STATUS_FULL_RANGE, _native.STATUS_FULL_ORDER, _native.STATUS_FULL_PAD),
                    (local, n_local, 1, _native.STATUS_LOCAL_RANGE, _native.STATUS_LOCAL_ORDER,
                     _native.STATUS_LOCAL_PAD)):
                _native.check(lib.swa_prepare_indices(_native.ptr(t) if n else None, B, n, q_len, 1, 0, None,
                                                      _native.ptr(counts[row * B:(row + 1) * B]),
                                                      _native.ptr(status), rb, ob, pb, stream), "index validation")
            _native.check(lib.swa_check_cover(_native.ptr(counts), B, q_len, _native.ptr(status), stream),
                          "coverage check")
            if validate:
                vals = ws[2:].tolist()  # status and the per-row counts in one read
                _raise_status(int(vals[0]))
                host_counts = (max(vals[2:2 + B]), max(vals[2 + B:2 + 2 * B]))
            else:
                gate = status
            counts_arg = counts
        else:
            counts_arg, batch_major = query_counts, 1
        if out is None:
            out = torch.empty_like(q)
        if lse is None:
            lse = torch.empty(q.shape[:3], dtype=torch.float32, device=dev)
        if metadata is not None:
            fs, ls, ce = metadata.full_starts, metadata.local_starts, metadata.causal_ends
        else:
            fs = ls = ce = None
        n_bg = 0
        if bg_list is not None:
            bg_list = bg_list.to(device=dev).contiguous()
            n_bg = int(bg_list.numel())
        split_tiles, scratch, scratch_bytes = 0, None, 0
        if key_split:
            request = 0 if key_split == "auto" else int(key_split)
            cf, cl = host_counts if host_counts is not None else (n_full, n_local)
            split_tiles, scratch_bytes = split_plan(B, kv_len, Hq, Hkv, min(cf, n_full), min(cl, n_local), window_size,
                                                    dev, n_bg=n_bg, request_tiles=request)
            if scratch_bytes:
                scratch = torch.empty(scratch_bytes, dtype=torch.uint8, device=dev)
        args = (_native.ptr(q), _native.ptr(k), _native.ptr(v),
                _native.ptr(full) if n_full else None, _native.ptr(local) if n_local else None,
                n_full, n_local, n_full, n_local,
                _native.ptr(counts_arg), batch_major, n_full, n_local,
                _native.ptr(fs), _native.ptr(ls), _native.ptr(ce),
                _native.ptr(bg_list), n_bg,
                _native.ptr(out), _native.ptr(lse),
                B, q_len, kv_len, Hq, Hkv, D, int(window_size), float(scale),
                _native.ptr(gate), _native.ptr(ws), ws.numel() * 4)
        if prefill_events is not None:
            prefill_events[0].record()
        if split_tiles:
            rc = lib.swa_prefill_forward_split(*args, split_tiles, _native.ptr(scratch), scratch_bytes, stream)
        else:
            rc = lib.swa_prefill_forward(*args, stream)
        _native.check(rc, "switch_gqa_prefill_forward")
        if prefill_events is not None:
            prefill_events[1].record()
        if status_out is not None or CHECK_DEVICE_STATUS:
            # ws[1]: kernel status (timeout); ws[2]: validation bits of the gated launch
            publish_status(torch.bitwise_or(ws[1:2], ws[2:3]), status_out)
    return out, lse
