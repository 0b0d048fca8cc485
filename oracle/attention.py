"""Switch Attention GQA prefill, restated on the CPU in FP32 torch (test oracle only).

Reference semantics (YushengZhao/SwitchAttentionKernels):

* scale: ``scale_log2 = (sm_scale or 1/sqrt(D)) * log2(e)``
  (``swiattn_gqa_prefill.py:43-46``, ``swiattn_gqa_prefill_varlen.py:73-76``);
* GQA head map: query head ``h`` reads KV head ``h // (Hq / Hkv)``
  (``swiattn_gqa_prefill.py:88``, ``swiattn_gqa_prefill_varlen.py:124``);
* legality of key ``j`` for a row at position ``t`` (``swiattn_gqa_prefill.py:145-158``):
  full ``0 <= j <= t``, local ``max(t - W + 1, 0) <= j <= t``, and ``j < Skv``;
  with metadata (``swiattn_gqa_prefill_varlen.py:134-137,186-196``):
  ``start[t] <= j < causal_ends[t]`` and ``j < Skv`` where ``start`` is
  ``full_starts`` or ``local_starts``;
* output: ``O = softmax_2(scale_log2 * q k^T) v`` and the log2-domain
  ``LSE = log2(sum_j 2^(scale_log2 * s_j))`` (``swiattn_gqa_prefill_varlen.py:207-241``);
  a row with no legal key yields ``O = 0/0`` (NaN) and ``LSE = -inf`` exactly as the
  kernel's ``acc_o / row_sum`` and ``log2(row_sum)`` do;
* rows are written at their original positions (``:243-249``).

``prefill_dense`` computes the exact FP32 result (the accuracy reference).
``prefill_rows`` runs on the device of its inputs: the GPU tests evaluate the
same FP32 restatement on the GPU to check every row of the full-size workloads
(cuBLAS FP32 with TF32 off; the tests check it against the CPU evaluation on a
sample of rows).
``prefill_tiled`` replays the kernel loop tile by tile -- union key range of a
query tile (``swiattn_gqa_prefill.py:95-105``, varlen ``:142-154``), running max
initialised to ``-2**30`` (``:132``), ``exp2`` rescaling, P rounded to BF16 before
``P @ V`` (``:187``, varlen ``:225``), final division and log2 (``:201-206``) -- to
show how far the reference's own rounding sits from the exact result.
"""
from __future__ import annotations

import math

import numpy as np
import torch

LOG2E = 1.4426950408889634


def scale_log2_of(sm_scale, dim: int) -> float:
    return (sm_scale if sm_scale is not None else (1.0 / dim) ** 0.5) * LOG2E


def row_bounds(pos: np.ndarray, is_local: bool, window: int, skv: int, metadata=None) -> tuple[np.ndarray, np.ndarray]:
    """Half-open legal key range ``[lo, hi)`` of each row (before clipping to ``[0, Skv)``)."""
    pos = np.asarray(pos, dtype=np.int64)
    if metadata is None:
        hi = pos + 1
        lo = np.maximum(pos - window + 1, 0) if is_local else np.zeros_like(pos)
    else:
        starts = np.asarray(metadata["local_starts" if is_local else "full_starts"], dtype=np.int64)
        ends = np.asarray(metadata["causal_ends"], dtype=np.int64)
        lo = starts[pos]
        hi = ends[pos]
    lo = np.maximum(lo, 0)
    hi = np.minimum(hi, skv)
    return lo, hi


def legal_key_counts(full_lists, local_lists, *, window: int, skv: int, metadata=None) -> int:
    """Total number of legal (row, key) pairs for one query head, summed over batches."""
    total = 0
    for fl, ll in zip(full_lists, local_lists):
        for is_local, lst in ((False, fl), (True, ll)):
            lo, hi = row_bounds(lst, is_local, window, skv, metadata)
            total += int(np.maximum(hi - lo, 0).sum())
    return total


def prefill_rows(q, k, v, b: int, positions, is_local: bool, *, window: int, sm_scale=None, metadata=None,
                 budget_bytes: int = 1 << 28):
    """Exact FP32 rows of one branch: ``(O [n, Hq, D], LSE [n, Hq])`` for ``positions`` of batch ``b``.

    ``positions`` must be increasing (chunks take the union key range of
    consecutive rows, like the kernel's query tiles).
    """
    B, Sq, Hq, D = q.shape
    Skv, Hkv = k.shape[1], k.shape[2]
    r = Hq // Hkv
    sl2 = scale_log2_of(sm_scale, D)
    dev = q.device
    pos = np.asarray(positions, dtype=np.int64)
    O = torch.empty((pos.size, Hq, D), dtype=torch.float32, device=dev)
    LSE = torch.empty((pos.size, Hq), dtype=torch.float32, device=dev)
    if pos.size == 0:
        return O, LSE
    lo, hi = row_bounds(pos, is_local, window, Skv, metadata)
    c = 0
    while c < pos.size:
        span_guess = int(hi[min(c + 63, pos.size - 1)] - lo[c]) + 1
        n = max(1, min(64, budget_bytes // max(1, 4 * Hq * max(span_guess, 1))))
        sl = slice(c, c + n)
        p, l, h = pos[sl], lo[sl], hi[sl]
        n = p.size
        c += n
        L0, L1 = int(l.min()), int(h.max())
        if L1 <= L0:
            O[sl] = float("nan")
            LSE[sl] = float("-inf")
            continue
        qc = q[b, torch.from_numpy(p).to(dev)].float().view(n, Hkv, r, D)
        kc = k[b, L0:L1].float()
        vc = v[b, L0:L1].float()
        s = torch.einsum("ngrd,lgd->ngrl", qc, kc) * sl2
        keys = torch.arange(L0, L1, device=dev)
        lo_t = torch.from_numpy(l).to(dev)[:, None]
        hi_t = torch.from_numpy(h).to(dev)[:, None]
        legal = (keys[None, :] >= lo_t) & (keys[None, :] < hi_t)
        s = s.masked_fill(~legal[:, None, None, :], float("-inf"))
        m = s.amax(dim=-1, keepdim=True)
        m_safe = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
        pe = torch.exp2(s - m_safe)
        den = pe.sum(dim=-1, keepdim=True)
        num = torch.einsum("ngrl,lgd->ngrd", pe, vc)
        O[sl] = (num / den).reshape(n, Hq, D)
        LSE[sl] = (m_safe + torch.log2(den)).squeeze(-1).reshape(n, Hq)
    return O, LSE


def prefill_backward(q, k, v, dout, full_lists, local_lists, *, window: int, sm_scale=None, metadata=None):
    """FP32 ``(dq, dk, dv)`` of the prefill forward for the upstream gradient ``dout``.

    Autograd over the same restatement as ``prefill_rows`` (masks of
    ``swiattn_gqa_prefill.py:145-158`` / metadata bounds, scaled softmax, P V);
    the reference itself is forward only.  Rows without a legal key carry no
    gradient.  Small cases only: one dense ``[rows, heads, Skv]`` score block per
    (batch, branch).
    """
    B, Sq, Hq, D = q.shape
    Skv, Hkv = k.shape[1], k.shape[2]
    r = Hq // Hkv
    scale = sm_scale if sm_scale is not None else (1.0 / D) ** 0.5
    qf = q.detach().float().clone().requires_grad_(True)
    kf = k.detach().float().clone().requires_grad_(True)
    vf = v.detach().float().clone().requires_grad_(True)
    loss = torch.zeros(())
    for b in range(B):
        for is_local, lst in ((False, full_lists[b]), (True, local_lists[b])):
            pos = np.asarray(lst, dtype=np.int64)
            if pos.size == 0:
                continue
            lo, hi = row_bounds(pos, is_local, window, Skv, metadata)
            keep = hi > lo
            pos, lo, hi = pos[keep], lo[keep], hi[keep]
            if pos.size == 0:
                continue
            n = pos.size
            qc = qf[b, torch.from_numpy(pos)].view(n, Hkv, r, D)
            s = torch.einsum("ngrd,lgd->ngrl", qc, kf[b]) * scale
            keys = torch.arange(Skv)
            legal = (keys[None, :] >= torch.from_numpy(lo)[:, None]) & (keys[None, :] < torch.from_numpy(hi)[:, None])
            s = s.masked_fill(~legal[:, None, None, :], float("-inf"))
            o = torch.einsum("ngrl,lgd->ngrd", torch.softmax(s, dim=-1), vf[b]).reshape(n, Hq, D)
            loss = loss + (o * dout[b, torch.from_numpy(pos)].float()).sum()
    loss.backward()
    zero = lambda t, g: g if g is not None else torch.zeros_like(t)  # noqa: E731
    return zero(qf, qf.grad), zero(kf, kf.grad), zero(vf, vf.grad)


def decode_rows(q, k, v, seq_lens, route_full, *, window: int, sm_scale=None):
    """Exact FP32 decode step: ``(O [B, Hq, D], LSE [B, Hq])``.

    The row semantics of the reference kernels (``swiattn_gqa_prefill.py:145-158``:
    full rows see keys ``[0, t]``, local rows ``[t - W + 1, t]``) at the last
    position ``t = L - 1`` of each sequence, ``L = seq_lens[b]``; ``q`` is
    ``[B, Hq, D]``, ``k`` / ``v`` are ``[B, Smax, Hkv, D]``.  The reference itself is
    prefill only; this is its formula for one row per sequence.
    """
    B, Hq, D = q.shape
    Hkv = k.shape[2]
    r = Hq // Hkv
    sl2 = scale_log2_of(sm_scale, D)
    O = torch.empty((B, Hq, D), dtype=torch.float32)
    LSE = torch.empty((B, Hq), dtype=torch.float32)
    for b in range(B):
        L = int(seq_lens[b])
        lo = 0 if bool(route_full[b]) else max(0, L - window)
        qb = q[b].float().view(Hkv, r, D)
        kb = k[b, lo:L].float()
        vb = v[b, lo:L].float()
        s = torch.einsum("grd,lgd->grl", qb, kb) * sl2
        m = s.amax(dim=-1, keepdim=True)
        pe = torch.exp2(s - m)
        den = pe.sum(dim=-1, keepdim=True)
        O[b] = (torch.einsum("grl,lgd->grd", pe, vb) / den).reshape(Hq, D)
        LSE[b] = (m + torch.log2(den)).reshape(Hq)
    return O, LSE


def prefill_dense(q, k, v, full_lists, local_lists, *, window: int, sm_scale=None, metadata=None,
                  subset=None, budget_bytes: int = 1 << 28):
    """Exact FP32 result.  ``q``: ``[B,Sq,Hq,D]``, ``k``/``v``: ``[B,Skv,Hkv,D]`` (any float dtype, CPU).

    ``full_lists`` / ``local_lists``: per batch, 1-D int arrays of positions.
    ``subset``: optional per batch array of positions to compute (others stay NaN).
    Returns ``(O, LSE)`` as FP32 tensors ``[B,Sq,Hq,D]`` / ``[B,Sq,Hq]``.
    """
    B, Sq, Hq, D = q.shape
    O = torch.full((B, Sq, Hq, D), float("nan"), dtype=torch.float32)
    LSE = torch.full((B, Sq, Hq), float("nan"), dtype=torch.float32)
    for b in range(B):
        for is_local, lst in ((False, full_lists[b]), (True, local_lists[b])):
            pos = np.asarray(lst, dtype=np.int64)
            if subset is not None:
                pos = pos[np.isin(pos, np.asarray(subset[b]))]
            if pos.size == 0:
                continue
            o, lse = prefill_rows(q, k, v, b, pos, is_local, window=window, sm_scale=sm_scale, metadata=metadata,
                                  budget_bytes=budget_bytes)
            O[b, torch.from_numpy(pos)] = o
            LSE[b, torch.from_numpy(pos)] = lse
    return O, LSE


def prefill_tiled(q, k, v, full_list, local_list, *, window: int, sm_scale=None, metadata=None,
                  block_m: int = 64, block_k: int = 64):
    """Tile-by-tile replay of the reference branch kernel for ``B = 1`` (small cases only).

    Follows ``swiattn_gqa_prefill.py:86-214`` (fixed) and, when ``metadata`` is
    given, ``swiattn_gqa_prefill_varlen.py:122-249``; all query heads of a tile are
    processed together (the kernel's grid z axis).
    """
    B, Sq, Hq, D = q.shape
    assert B == 1
    Skv, Hkv = k.shape[1], k.shape[2]
    r = Hq // Hkv
    sl2 = scale_log2_of(sm_scale, D)
    O = torch.full((Sq, Hq, D), float("nan"), dtype=torch.float32)
    LSE = torch.full((Sq, Hq), float("nan"), dtype=torch.float32)
    kv_head = torch.arange(Hq) // r
    for is_local, lst in ((False, full_list), (True, local_list)):
        idx = np.asarray(lst, dtype=np.int64)
        count = idx.size
        if count == 0:
            continue
        cap = -(-count // block_m) * block_m
        for q0 in range(0, cap, block_m):
            slots = np.arange(q0, q0 + block_m)
            valid = slots < count
            qpos = np.where(valid, idx[np.minimum(slots, count - 1)], 0)
            first_slot = min(q0, max(count - 1, 0))
            last_slot = min(q0 + block_m - 1, max(count - 1, 0))
            first_q = max(int(idx[first_slot]), 0)
            last_q = max(int(idx[last_slot]), 0)
            if metadata is None:
                first_key = max(first_q - window + 1, 0) if is_local else 0
                last_key = min(last_q + 1, Skv)
                lo = np.maximum(qpos - window + 1, 0) if is_local else np.zeros_like(qpos)
                hi = qpos + 1
            else:
                starts = np.asarray(metadata["local_starts" if is_local else "full_starts"], dtype=np.int64)
                ends = np.asarray(metadata["causal_ends"], dtype=np.int64)
                first_key = int(starts[first_q]) if q0 < count else Skv
                last_key = min(int(ends[last_q]), Skv) if q0 < count else 0
                lo, hi = starts[qpos], ends[qpos]
            first_block = first_key // block_k
            last_block = -(-last_key // block_k)
            nblocks = max(last_block - first_block, 0)
            qt = q[0, torch.from_numpy(np.clip(qpos, 0, Sq - 1))].float()            # [BM, Hq, D]
            acc_o = torch.zeros(block_m, Hq, D)
            row_sum = torch.zeros(block_m, Hq)
            row_max = torch.full((block_m, Hq), -(2.0 ** 30))
            lo_t = torch.from_numpy(lo)[:, None]
            hi_t = torch.from_numpy(hi)[:, None]
            valid_t = torch.from_numpy(valid)[:, None]
            for jb in range(nblocks):
                key0 = (first_block + jb) * block_k
                keys = torch.arange(key0, key0 + block_k)
                safe = keys.clamp(0, Skv - 1)
                kt = k[0, safe].float()[:, kv_head]                                    # [BK, Hq, D]
                vt = v[0, safe].float()[:, kv_head]
                legal = valid_t & (keys[None, :] < Skv) & (keys[None, :] >= lo_t) & (keys[None, :] < hi_t)
                acc_s = torch.einsum("mhd,nhd->mhn", qt, kt)
                acc_s = torch.where(legal[:, None, :], acc_s, torch.tensor(float("-inf")))
                prev = row_max
                row_max = torch.maximum(prev, acc_s.amax(dim=-1))
                alpha = torch.exp2((prev - row_max) * sl2)
                pe = torch.exp2(acc_s * sl2 - (row_max * sl2)[..., None])
                row_sum = row_sum * alpha + pe.sum(dim=-1)
                acc_o = acc_o * alpha[..., None]
                acc_o = acc_o + torch.einsum("mhn,nhd->mhd", pe.to(torch.bfloat16).float(), vt)
            out = acc_o / row_sum[..., None]
            lse = torch.log2(row_sum) + row_max * sl2
            sel = torch.from_numpy(qpos[valid])
            O[sel] = out[torch.from_numpy(valid)]
            LSE[sel] = lse[torch.from_numpy(valid)]
    return O[None], LSE[None]
