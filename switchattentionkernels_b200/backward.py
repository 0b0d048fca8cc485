"""Switch Attention GQA prefill backward, and the forward + backward as one
autograd function.

The reference is forward only (``swiattn_gqa_prefill_varlen.py:14``); these are
the gradients of its forward with respect to q, k and v, computed from the
forward's output and its log2-domain LSE (the reason the forward returns it).
Three CUDA launches: ``rowsum(dO * O)``, the dQ pass over each branch's routed
rows, and the dK / dV pass over 64-key tiles.
"""
from __future__ import annotations

import torch

from . import _core, _native
from ._core import LOG2E


def _lists(full, local, query_counts, B, dev):
    """Index lists as -1 padded ``[B, N]`` rows and int32 ``[B, 2]`` counts on ``dev``."""
    if query_counts is not None:
        if (query_counts.device != dev or query_counts.dtype != torch.int32
                or tuple(query_counts.shape) != (B, 2)):
            raise ValueError("query_counts must be an int32 [B, 2] tensor on the device of Q")
        f = full.to(dtype=torch.int32).contiguous()
        l = local.to(dtype=torch.int32).contiguous()
        if f.ndim != 2 or l.ndim != 2 or f.shape[0] != B or l.shape[0] != B:
            raise ValueError("with query_counts the index lists must be [B, N]")
        return f, l, query_counts.contiguous()
    if B != 1:
        raise ValueError("B > 1 needs -1 padded [B, N] lists and query_counts")
    f = full.reshape(1, -1).to(device=dev, dtype=torch.int32).contiguous()
    l = local.reshape(1, -1).to(device=dev, dtype=torch.int32).contiguous()
    counts = torch.tensor([[f.shape[1], l.shape[1]]], dtype=torch.int32, device=dev)
    return f, l, counts


def switch_gqa_prefill_backward(q, k, v, out, lse, dout, full_query_indices, local_query_indices, *, metadata=None,
                                window_size: int = 1024, sm_scale: float | None = None, query_counts=None,
                                status_out=None):
    """``(dq, dk, dv)`` of ``switch_gqa_prefill_forward`` for the upstream gradient ``dout``.

    ``q`` / ``k`` / ``v`` / ``out`` / ``dout``: contiguous BF16 as in the forward;
    ``lse``: the forward's FP32 ``[B, Sq, Hq]`` (log2 units).  Index lists: the
    forward's (1-D for ``B == 1``, or -1 padded ``[B, N]`` with ``query_counts``).
    Returns BF16 tensors shaped like ``q``, ``k`` and ``v``.  ``status_out``:
    optional int32 device tensor whose element 0 receives the launch's status word
    on the current stream (no host sync); non-zero (``STATUS_TIMEOUT``) means the
    gradients are undefined.
    """
    _core.validate_qkv(q, k, v)
    for name, t in (("out", out), ("dout", dout)):
        if t.dtype != torch.bfloat16 or t.shape != q.shape or not t.is_contiguous() or t.device != q.device:
            raise ValueError(f"{name} must be a contiguous bfloat16 tensor shaped like q on its device")
    B, Sq, Hq, D = q.shape
    Skv, Hkv = k.shape[1], k.shape[2]
    if (lse.dtype != torch.float32 or tuple(lse.shape) != (B, Sq, Hq) or not lse.is_contiguous()
            or lse.device != q.device):
        raise ValueError("lse must be the forward's contiguous float32 [B, Sq, Hq] tensor")
    if window_size <= 0:
        raise ValueError("window_size must be positive")
    dev = q.device
    if metadata is not None:
        _core._check_metadata(metadata, q, Sq, Skv)
    scale = (sm_scale if sm_scale is not None else (1.0 / D) ** 0.5) * LOG2E
    if not scale > 0:
        raise ValueError("sm_scale must be positive")
    _core._check_status_out(status_out, dev)
    f, l, counts = _lists(full_query_indices, local_query_indices, query_counts, B, dev)
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    fs = ls = ce = None
    if metadata is not None:
        fs, ls, ce = metadata.full_starts, metadata.local_starts, metadata.causal_ends
    lib = _native.load()
    ws_bytes = lib.swa_backward_workspace_bytes(B, Hq, int(f.shape[1]), int(l.shape[1]))
    ws = torch.empty((ws_bytes + 15) // 16 * 4, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        rc = lib.swa_prefill_backward(
            _native.ptr(q), _native.ptr(k), _native.ptr(v), _native.ptr(out), _native.ptr(lse), _native.ptr(dout),
            _native.ptr(f) if f.shape[1] else None, _native.ptr(l) if l.shape[1] else None,
            int(f.shape[1]), int(l.shape[1]), _native.ptr(counts), _native.ptr(fs), _native.ptr(ls), _native.ptr(ce),
            _native.ptr(dq), _native.ptr(dk), _native.ptr(dv), B, Sq, Skv, Hq, Hkv, D, int(window_size),
            float(scale), _native.ptr(ws), ws.numel() * 4, _native.stream_ptr(dev))
    _native.check(rc, "switch_gqa_prefill_backward")
    if status_out is not None or _core.CHECK_DEVICE_STATUS:
        _core.publish_status(ws[0:1], status_out)
    return dq, dk, dv


class _SwitchAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, full, local, metadata, window_size, sm_scale, query_counts):
        out, lse = _core.forward(q, k, v, full, local, metadata=metadata, window_size=window_size, sm_scale=sm_scale,
                                 query_counts=query_counts)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.lists = (full, local, query_counts)
        ctx.opts = (metadata, window_size, sm_scale)
        ctx.mark_non_differentiable(lse)
        return out, lse

    @staticmethod
    def backward(ctx, dout, _dlse):
        q, k, v, out, lse = ctx.saved_tensors
        full, local, counts = ctx.lists
        metadata, window_size, sm_scale = ctx.opts
        dq, dk, dv = switch_gqa_prefill_backward(q, k, v, out, lse, dout.contiguous(), full, local,
                                                 metadata=metadata, window_size=window_size, sm_scale=sm_scale,
                                                 query_counts=counts)
        return dq, dk, dv, None, None, None, None, None, None


def switch_gqa_prefill_attention(q, k, v, full_query_indices, local_query_indices, *, metadata=None,
                                 window_size: int = 1024, sm_scale: float | None = None, query_counts=None):
    """``switch_gqa_prefill_forward`` as a differentiable op: ``(O, LSE)`` with gradients for q, k and v."""
    return _SwitchAttention.apply(q, k, v, full_query_indices, local_query_indices, metadata, window_size, sm_scale,
                                  query_counts)
