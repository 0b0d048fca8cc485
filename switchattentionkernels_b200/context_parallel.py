"""Context parallelism for packed (varlen) Switch Attention prefill.

One long packed batch (``B == 1``, ``S`` tokens, optionally several sequences
given by ``cu_seqlens``) is split over the ranks of a process group by rows.
The token axis is cut into ``2N`` chunks and rank ``r`` holds chunks ``r`` and
``2N - 1 - r`` ("zigzag"): a causal row's cost grows with its position, and
pairing an early chunk with a late one evens out the ranks.  With uniform
chunks this is exact for one causal sequence; for packed sequences, where cost
restarts at every sequence start, the chunks can instead be cut at equal
quantiles of a per-row cost (``row_costs``, e.g. ``cp_row_costs`` of the routing
mask), which gives every rank the same number of legal (row, key) entries.

Each rank owns Q, K and V of its rows.  K and V are exchanged once, in one of
two ways: ``KVExchange`` -- every rank's K/V buffer of the whole token axis in
symmetric memory, each rank writing its two chunks straight into every rank's
buffer at their token offsets with one copy kernel of plain peer stores over
NVLink, between two device barriers of all ranks -- or, for any backend,
``cp_gather_kv``: an all-gather of the shards (NCCL over NVLink for CUDA
tensors) followed by one pass of chunk copies into token order.  Every rank
then runs the prefill kernel on its own query rows against the whole token
axis.  The
per-row key bounds (``full_starts`` / ``local_starts`` / ``causal_ends``) are those
of the rows' global positions, so a local row's legal keys are exactly the ones
it has without the split.

This is the layout the reference's varlen kernel prepares its metadata for:
local query rows addressing a gathered KV axis
(``swiattn_gqa_prefill_varlen.py:139-141,179-182``); the reference itself has no
distributed code.  Rows of one rank are in increasing global order, so key
bounds are non-decreasing along the local rows, which the kernel's work units
(union key range of their first and last routed row) require.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

import ctypes

from . import _core, _native
from .metadata import SwitchAttentionMetadata, build_switch_attention_metadata


def cp_row_costs(full_mask, window: int, cu_seqlens=None) -> np.ndarray:
    """Legal keys of every row of a packed batch (``full_mask``: bool ``[S]``, True = full branch)."""
    m = np.asarray(full_mask, dtype=bool).reshape(-1)
    S = m.size
    t = np.arange(S, dtype=np.int64)
    if cu_seqlens is None:
        start = np.zeros(S, dtype=np.int64)
    else:
        cu = np.asarray(cu_seqlens, dtype=np.int64)
        start = cu[np.searchsorted(cu, t, side="right") - 1]
    lo = np.where(m, start, np.maximum(start, t - window + 1))
    return (t + 1 - lo).astype(np.float64)


@dataclass(frozen=True)
class ContextParallelPlan:
    """Row split of a ``total_len``-token packed batch over ``world`` ranks."""
    total_len: int
    world: int
    bounds: np.ndarray  # 2 * world + 1 chunk boundaries: chunk c is rows [bounds[c], bounds[c + 1])

    def rows(self, rank: int) -> np.ndarray:
        """Global rows held by ``rank`` (increasing): chunks ``rank`` and ``2 * world - 1 - rank``."""
        if not 0 <= rank < self.world:
            raise ValueError("rank must lie in [0, world)")
        b = self.bounds
        c = 2 * self.world - 1 - rank
        return np.concatenate([np.arange(b[rank], b[rank + 1], dtype=np.int64),
                               np.arange(b[c], b[c + 1], dtype=np.int64)])

    @property
    def capacity(self) -> int:
        """Rows of the largest shard."""
        return max(int(self.rows(r).size) for r in range(self.world))


def make_cp_plan(total_len: int, world: int, row_costs=None) -> ContextParallelPlan:
    """Zigzag split into ``2 * world`` chunks: uniform, or of equal total ``row_costs``.

    Deterministic, so every rank computes the same plan from the same inputs.
    """
    if world <= 0:
        raise ValueError("world size must be positive")
    if total_len <= 0:
        raise ValueError("total_len must be positive")
    n = 2 * world
    if row_costs is None:
        b = (np.arange(n + 1, dtype=np.int64) * total_len) // n
    else:
        c = np.asarray(row_costs, dtype=np.float64).reshape(-1)
        if c.size != total_len or not np.all(np.isfinite(c)) or np.any(c < 0):
            raise ValueError("row_costs must hold total_len finite non-negative numbers")
        cum = np.concatenate([[0.0], np.cumsum(c)])
        if cum[-1] <= 0:
            b = (np.arange(n + 1, dtype=np.int64) * total_len) // n
        else:
            inner = np.searchsorted(cum, cum[-1] * np.arange(1, n) / n, side="left")
            b = np.concatenate([[0], np.minimum(inner, total_len), [total_len]]).astype(np.int64)
            b = np.maximum.accumulate(b)
    return ContextParallelPlan(total_len=int(total_len), world=int(world), bounds=b)


def cp_shard_rows(total_len: int, world: int, rank: int, row_costs=None) -> np.ndarray:
    """Global rows held by ``rank`` under ``make_cp_plan(total_len, world, row_costs)``."""
    return make_cp_plan(total_len, world, row_costs).rows(rank)


def cp_gather_kv(k: torch.Tensor, v: torch.Tensor, plan: ContextParallelPlan, *, group=None):
    """All-gather this rank's K/V rows (``[1, L_r, Hkv, D]``) into ``[1, S, Hkv, D]`` in token order.

    One collective per tensor on shards of the largest shard's length (a shard
    is sent in place when it has that length; padding rows are never read),
    then ``2 * world`` contiguous chunk copies into token order.  With one rank
    the shard already is the whole axis and nothing moves.  (A batch of NCCL
    point-to-point transfers straight into the token-order slots measured
    slower than this on two B200s: 0.55 ms against 0.47 ms for config 4.)
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if world != plan.world:
        raise ValueError("the plan was made for a different world size")
    rows = plan.rows(rank)
    for t in (k, v):
        if t.ndim != 4 or t.shape[0] != 1 or t.shape[1] != rows.size:
            raise ValueError(f"K/V shards must have shape [1, {rows.size}, Hkv, D] on rank {rank}")
    if world == 1:
        return k.contiguous(), v.contiguous()
    cap = plan.capacity
    b = plan.bounds
    n = 2 * world
    out = []
    for t in (k, v):
        tail = tuple(t.shape[2:])
        if rows.size == cap and t.is_contiguous():
            shard = t[0]
        else:
            shard = t.new_empty((cap,) + tail)
            shard[:rows.size] = t[0]
        buf = t.new_empty((world * cap,) + tail)
        dist.all_gather_into_tensor(buf, shard, group=group)
        full = t.new_empty((1, plan.total_len) + tail)
        for c in range(n):
            lo, hi = int(b[c]), int(b[c + 1])
            if hi == lo:
                continue
            r = c if c < world else n - 1 - c
            off = r * cap + (0 if c < world else int(b[r + 1] - b[r]))
            full[0, lo:hi].copy_(buf[off:off + hi - lo])
        out.append(full)
    return out[0], out[1]


class KVExchange:
    """K and V of the whole token axis (``[1, S, Hkv, D]`` each) on every rank of
    ``group``, in symmetric memory, filled by ``exchange``: each rank stores its
    two zigzag chunks into every rank's buffers at the chunks' token offsets
    (``swa_broadcast_bytes``: every word read once, stored to all ranks, plain
    stores to the peers' memory over NVLink), with a device barrier of all ranks
    before (nobody still reads the previous contents) and after (every chunk has
    landed).  No staging buffer, no collective, no reorder pass.  Allocated once
    per shape and reused; ``k`` / ``v`` are this rank's buffers, which the prefill
    kernel then reads from this GPU's own memory.  One rank: plain device buffers.
    """

    def __init__(self, total_len: int, hkv: int, *, device, group=None, head_dim: int = 128,
                 dtype=torch.bfloat16):
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("KVExchange needs CUDA tensors (use cp_gather_kv on other backends)")
        shape = (1, total_len, hkv, head_dim)
        self.shape = shape
        self.group = group
        self.world = 1 if not dist.is_initialized() else dist.get_world_size(group)
        self.rank = 0 if not dist.is_initialized() else dist.get_rank(group)
        self._handles = None
        if self.world == 1:
            self.k = torch.empty(shape, dtype=dtype, device=device)
            self.v = torch.empty(shape, dtype=dtype, device=device)
            kp, vp = [self.k.data_ptr()], [self.v.data_ptr()]
        else:
            import torch.distributed._symmetric_memory as symm_mem

            g = group if group is not None else dist.group.WORLD
            if self.world > 8:
                raise ValueError("KVExchange: at most 8 ranks")
            self.k = symm_mem.empty(shape, dtype=dtype, device=device)
            self.v = symm_mem.empty(shape, dtype=dtype, device=device)
            hk = symm_mem.rendezvous(self.k, g)
            hv = symm_mem.rendezvous(self.v, g)
            self._handles = (hk, hv)
            kp, vp = list(hk.buffer_ptrs), list(hv.buffer_ptrs)
        self._ptrs = (kp, vp)
        self._row_bytes = hkv * head_dim * torch.empty((), dtype=dtype).element_size()

    def barrier(self) -> None:
        """Device-side barrier of all ranks on the current stream (no-op for one rank)."""
        if self._handles is not None:
            self._handles[0].barrier(channel=0)

    def exchange(self, k: torch.Tensor, v: torch.Tensor, plan: ContextParallelPlan):
        """This rank's K/V rows (``[1, L_r, Hkv, D]``, ``plan.rows(rank)``) into every
        rank's buffers; returns this rank's ``(k, v)`` of the whole token axis."""
        if plan.world != self.world or plan.total_len != self.shape[1]:
            raise ValueError("the plan was made for a different world size or token count")
        rows = plan.rows(self.rank)
        for t in (k, v):
            if (t.ndim != 4 or t.shape[0] != 1 or t.shape[1] != rows.size or tuple(t.shape[2:]) != self.shape[2:]
                    or t.dtype != self.k.dtype or t.device != self.k.device):
                raise ValueError(f"K/V shards must be [1, {rows.size}, {self.shape[2]}, {self.shape[3]}] "
                                 f"{self.k.dtype} on {self.k.device}")
        lib = _native.load()
        b = plan.bounds
        r, n = self.rank, 2 * self.world
        first = int(b[r + 1] - b[r])
        chunks = ((int(b[r]), int(b[r + 1]), 0), (int(b[n - 1 - r]), int(b[n - r]), first))
        self.barrier()
        stream = _native.stream_ptr(self.k.device)
        with torch.cuda.device(self.k.device):
            for t, ptrs in ((k.contiguous(), self._ptrs[0]), (v.contiguous(), self._ptrs[1])):
                for lo, hi, off in chunks:
                    if hi == lo:
                        continue
                    nbytes = (hi - lo) * self._row_bytes
                    dsts = (ctypes.c_void_p * len(ptrs))(*[p + lo * self._row_bytes for p in ptrs])
                    rc = lib.swa_broadcast_bytes(ctypes.c_void_p(t.data_ptr() + off * self._row_bytes), nbytes,
                                                 dsts, len(ptrs), stream)
                    _native.check(rc, "swa_broadcast_bytes")
        self.barrier()
        return self.k, self.v


def cp_metadata(total_len: int, rows: np.ndarray, *, device, window_size: int,
                cu_seqlens: torch.Tensor | None = None) -> SwitchAttentionMetadata:
    """Key bounds of the local query ``rows`` (global row ids) against the whole token axis."""
    g = build_switch_attention_metadata(total_len, total_len, device=device, window_size=window_size,
                                        cu_seqlens=cu_seqlens)
    idx = torch.from_numpy(np.ascontiguousarray(rows, dtype=np.int64)).to(device)
    pick = lambda t: t.index_select(0, idx).contiguous()  # noqa: E731
    return SwitchAttentionMetadata(q_positions=pick(g.q_positions), kv_positions=g.kv_positions,
                                   q_segment_ids=pick(g.q_segment_ids), kv_segment_ids=g.kv_segment_ids,
                                   full_starts=pick(g.full_starts), local_starts=pick(g.local_starts),
                                   causal_ends=pick(g.causal_ends))


def context_parallel_switch_gqa_prefill_forward(q, k, v, full_query_indices, local_query_indices, *, total_len: int,
                                                cu_seqlens=None, window_size: int = 1024, sm_scale=None,
                                                group=None, validate: bool = True, row_costs=None,
                                                plan: ContextParallelPlan | None = None,
                                                metadata: SwitchAttentionMetadata | None = None,
                                                kv_exchange: KVExchange | None = None):
    """Switch Attention prefill of this rank's rows of a context-parallel packed batch.

    ``q`` / ``k`` / ``v``: ``[1, L_r, H, 128]`` -- the rows ``plan.rows(rank)`` of the
    packed batch, in that order (``plan`` defaults to ``make_cp_plan(total_len,
    world, row_costs)``).  ``full_query_indices`` / ``local_query_indices``:
    increasing local row indices (``0 .. L_r - 1``) routed to each branch, e.g.
    ``build_switch_query_indices`` of the local rows' routing mask.
    ``cu_seqlens``: sequence boundaries of the whole packed batch (global rows).
    ``metadata``: the local rows' key bounds, ``cp_metadata(total_len,
    plan.rows(rank), ...)``; built here when not given (it depends only on the
    batch, so a caller running several layers builds it once).
    Returns ``(O, LSE)`` of the local rows, ``[1, L_r, Hq, 128]`` BF16 and
    ``[1, L_r, Hq]`` FP32 (log2 units), equal to those rows of the unsplit forward.
    ``kv_exchange``: a ``KVExchange`` of this batch's shape and group, which
    exchanges K/V by peer stores through symmetric memory; without it, the NCCL
    all-gather of ``cp_gather_kv``.
    Every rank takes part in the K/V exchange, also one that holds no rows.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if plan is None:
        plan = make_cp_plan(total_len, world, row_costs)
    elif plan.total_len != total_len:
        raise ValueError("the plan was made for a different total_len")
    rows = plan.rows(rank)
    if q.ndim != 4 or q.shape[0] != 1 or q.shape[1] != rows.size:
        raise ValueError(f"Q shard must have shape [1, {rows.size}, Hq, D] on rank {rank}")
    if kv_exchange is not None:
        k_full, v_full = kv_exchange.exchange(k, v, plan)
    else:
        k_full, v_full = cp_gather_kv(k, v, plan, group=group)
    if rows.size == 0:
        return torch.empty_like(q), torch.empty(q.shape[:3], dtype=torch.float32, device=q.device)
    md = metadata
    if md is None:
        md = cp_metadata(total_len, rows, device=q.device, window_size=window_size, cu_seqlens=cu_seqlens)
    return _core.forward(q, k_full, v_full, full_query_indices, local_query_indices, metadata=md,
                         window_size=window_size, sm_scale=sm_scale, validate=validate)
