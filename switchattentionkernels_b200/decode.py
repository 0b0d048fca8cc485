"""Switch Attention GQA decode step: one new query token per sequence.

Not part of the reference (its kernels are prefill only); this is the decode
counterpart of the same routing: each sequence's new token attends either to
all of its cached keys (full causal attention) or to the last ``window_size``
of them (sliding window), with the scale, the log2-domain softmax and the LSE
convention of the prefill path (reference ``swiattn_gqa_prefill.py:145-158``
at the last position ``t = L - 1``).  One CUDA launch pair: the split-KV
kernel (TMA K/V ring, ``mma.sync`` tiles, online softmax per split) and the
merge of the splits.
"""
from __future__ import annotations

import torch

from . import _core, _native
from ._core import LOG2E


def _scales(x, B: int, Hkv: int, dev, name: str) -> torch.Tensor:
    """FP32 ``[B, Hkv]`` contiguous scales on ``dev`` from a number, ``[Hkv]`` or ``[B, Hkv]``."""
    t = torch.as_tensor(x, dtype=torch.float32, device=dev)
    if t.ndim == 0:
        t = t.expand(B, Hkv)
    elif t.ndim == 1 and t.shape[0] == Hkv:
        t = t.unsqueeze(0).expand(B, Hkv)
    if tuple(t.shape) != (B, Hkv):
        raise ValueError(f"{name} must be a number, [Hkv] or [B, Hkv]")
    return t.contiguous()


def switch_gqa_decode_forward(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                              seq_lens: torch.Tensor, route_full: torch.Tensor, *, window_size: int = 1024,
                              sm_scale: float | None = None, status_out: torch.Tensor | None = None,
                              k_scale: torch.Tensor | float | None = None, v_scale: torch.Tensor | float | None = None):
    """Attention of each sequence's new token over its KV cache.

    ``q``: BF16 ``[B, Hq, 128]`` (or ``[B, 1, Hq, 128]``); ``k_cache`` / ``v_cache``:
    BF16 ``[B, Smax, Hkv, 128]`` with the new token's K/V already at row
    ``seq_lens[b] - 1``; ``seq_lens``: int32 ``[B]`` (``1 <= L <= Smax``; a
    sequence with ``L = 0`` has no key and gets O = NaN, LSE = -inf, as a prefill
    row whose key range is empty);
    ``route_full``: bool ``[B]``, True = full causal attention, False = the
    sliding window of the last ``window_size`` keys.  Returns ``(O, LSE)``:
    BF16 ``[B, Hq, 128]`` and FP32 ``[B, Hq]`` (log2 units), shaped like ``q``.
    ``status_out``: optional int32 device tensor whose element 0 receives the
    launch's status word on the current stream (no host sync); non-zero
    (``STATUS_TIMEOUT``) means the outputs are undefined.

    FP8 cache: ``k_cache`` / ``v_cache`` of dtype ``torch.float8_e4m3fn`` with
    ``k_scale`` / ``v_scale`` (FP32 ``[B, Hkv]``, ``[Hkv]`` or a number): the
    attention uses ``k_cache * k_scale`` and ``v_cache * v_scale``.  Half the bytes
    of the BF16 step; the products run in FP16, so ``q`` must lie within the FP16
    range.
    """
    squeeze = q.ndim == 4
    if squeeze:
        if q.shape[1] != 1:
            raise ValueError("decode takes one query token per sequence")
        q = q[:, 0]
    fp8 = isinstance(k_cache, torch.Tensor) and k_cache.dtype == torch.float8_e4m3fn
    cache_dtype = torch.float8_e4m3fn if fp8 else torch.bfloat16
    if not isinstance(q, torch.Tensor) or q.dtype != torch.bfloat16 or not q.is_cuda:
        raise TypeError("q must be a device-resident bfloat16 tensor")
    for name, t in (("k_cache", k_cache), ("v_cache", v_cache)):
        if not isinstance(t, torch.Tensor) or t.dtype != cache_dtype or not t.is_cuda:
            raise TypeError(f"{name} must be a device-resident bfloat16 tensor, or float8_e4m3fn for both caches")
    for name, t in (("q", q), ("k_cache", k_cache), ("v_cache", v_cache)):
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if q.ndim != 3 or k_cache.ndim != 4 or v_cache.shape != k_cache.shape:
        raise ValueError("expected q [B, Hq, 128] and k_cache / v_cache [B, Smax, Hkv, 128]")
    B, Hq, D = q.shape
    Bk, Smax, Hkv, Dk = k_cache.shape
    if D != 128 or Dk != 128:
        raise ValueError("head_dim must be 128")
    if Bk != B:
        raise ValueError("q and the KV cache must have the same batch size")
    if Hq % Hkv != 0:
        raise ValueError("query heads must be divisible by KV heads")
    if window_size <= 0:
        raise ValueError("window_size must be positive")
    dev = q.device
    if k_cache.device != dev or v_cache.device != dev:
        raise ValueError("q and the KV cache must be on the same device")
    if seq_lens.device != dev or seq_lens.dtype != torch.int32 or tuple(seq_lens.shape) != (B,):
        raise ValueError("seq_lens must be an int32 [B] tensor on the device of q")
    if route_full.device != dev or route_full.dtype != torch.bool or tuple(route_full.shape) != (B,):
        raise ValueError("route_full must be a bool [B] tensor on the device of q")
    scale = (sm_scale if sm_scale is not None else (1.0 / D) ** 0.5) * LOG2E
    if not scale > 0:
        raise ValueError("sm_scale must be positive")
    if fp8:
        if k_scale is None or v_scale is None:
            raise ValueError("an FP8 KV cache needs k_scale and v_scale")
        k_scale = _scales(k_scale, B, Hkv, dev, "k_scale")
        v_scale = _scales(v_scale, B, Hkv, dev, "v_scale")
    elif k_scale is not None or v_scale is not None:
        raise ValueError("k_scale / v_scale apply to an FP8 KV cache only")
    _core._check_status_out(status_out, dev)
    lib = _native.load()
    out = torch.empty_like(q)
    lse = torch.empty((B, Hq), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        nbytes = int(lib.swa_decode_workspace_bytes(B, Smax, Hq, Hkv))
        if nbytes <= 0:
            raise RuntimeError("decode workspace size query failed: " +
                               lib.swa_last_error_string().decode(errors="replace"))
        ws = torch.empty((nbytes + 15) // 16 * 4, dtype=torch.int32, device=dev)
        route = route_full.contiguous().view(torch.uint8)
        if fp8:
            rc = lib.swa_decode_forward_fp8(_native.ptr(q), _native.ptr(k_cache), _native.ptr(v_cache),
                                            _native.ptr(k_scale), _native.ptr(v_scale),
                                            _native.ptr(seq_lens.contiguous()), _native.ptr(route), _native.ptr(out),
                                            _native.ptr(lse), B, Smax, Hq, Hkv, D, int(window_size), float(scale),
                                            _native.ptr(ws), ws.numel() * 4, _native.stream_ptr(dev))
        else:
            rc = lib.swa_decode_forward(_native.ptr(q), _native.ptr(k_cache), _native.ptr(v_cache),
                                        _native.ptr(seq_lens.contiguous()), _native.ptr(route), _native.ptr(out),
                                        _native.ptr(lse), B, Smax, Hq, Hkv, D, int(window_size), float(scale),
                                        _native.ptr(ws), ws.numel() * 4, _native.stream_ptr(dev))
    _native.check(rc, "switch_gqa_decode_forward")
    if status_out is not None or _core.CHECK_DEVICE_STATUS:
        _core.publish_status(ws[0:1], status_out)
    if squeeze:
        return out.unsqueeze(1), lse.unsqueeze(1)
    return out, lse
