"""Multi-GPU driver: one prefill sharded over the ranks of a process group.

The unit of work is a (batch b, KV group g) pair: it reads ``q[b, :, g*r:(g+1)*r]``,
``k/v[b, :, g]`` and batch b's index lists, and writes the same slice of O/LSE,
so units are independent and need no communication.  Units are assigned to
ranks by longest-processing-time-first on their cost (the legal score entries
of batch b).  Two ways to run a rank's share:

* replicated inputs: every rank holds the whole q/k/v and the kernel computes
  only the rank's units (its ``bg_list``): ``sharded_switch_gqa_prefill_forward``;
* unit-major inputs: a rank holds only its units, as ``[n, S, r, 128]`` q and
  ``[n, S, 1, 128]`` k / v (``take_units``), which is the ordinary forward with
  ``B = n`` sequences of ``r`` query heads over one KV head -- the shape in which
  a head-sharded model layer produces them, and the only bytes a rank needs.

Only when the caller asks for a replicated result is there communication:
either the prefill kernel's epilogue stores every O / LSE row into every rank's
row-major ``[B, S, Hq, ...]`` buffer over NVLink as it is produced
(``forward_units_replicated`` with ``ReplicaBuffers`` in symmetric memory: the
transfer overlaps the attention itself), or one NCCL all-gather of O (BF16) and
LSE (FP32) after the launch followed by one scatter kernel into the row-major
layout (``gather_units_to_rows``; any backend that implements ``all_gather``).

The reference has no distributed code; this driver implements the sharding
that its per-(batch, head) grid (``swiattn_gqa_prefill.py:69``) admits.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Sequence

import numpy as np
import torch
import torch.distributed as dist

from . import _core, _native


def unit_costs(full_lists: Sequence[np.ndarray], local_lists: Sequence[np.ndarray], *, hkv: int, skv: int,
               window: int, metadata=None) -> np.ndarray:
    """Cost of every unit ``b * hkv + g``: legal (row, key) entries of batch b.

    Without ``metadata`` a row at position t has the fixed-length key ranges
    (full ``[0, t]``, local ``[t - W + 1, t]``, clipped to ``[0, Skv)``).  With
    ``metadata`` (a ``SwitchAttentionMetadata`` or a dict of its arrays) the
    ranges are the per-row bounds ``[start, causal_end)`` the kernel uses, so
    packed sequences are costed by their own lengths.
    """
    bounds = None
    if metadata is not None:
        def arr(name):
            a = metadata[name] if isinstance(metadata, dict) else getattr(metadata, name)
            return a.detach().cpu().numpy() if isinstance(a, torch.Tensor) else np.asarray(a)
        ends = np.minimum(arr("causal_ends").astype(np.int64), skv)
        bounds = (np.maximum(arr("full_starts").astype(np.int64), 0),
                  np.maximum(arr("local_starts").astype(np.int64), 0), ends)
    B = len(full_lists)
    costs = np.zeros(B * hkv, dtype=np.float64)
    for b in range(B):
        f = np.asarray(full_lists[b], dtype=np.int64)
        l = np.asarray(local_lists[b], dtype=np.int64)
        if bounds is None:
            n = float(np.minimum(f + 1, skv).sum())
            n += float(np.maximum(np.minimum(l + 1, skv) - np.maximum(l - window + 1, 0), 0).sum())
        else:
            fs, ls, ce = bounds
            n = float(np.maximum(ce[f] - fs[f], 0).sum()) + float(np.maximum(ce[l] - ls[l], 0).sum())
        costs[b * hkv:(b + 1) * hkv] = n
    return costs


def plan_units(costs: Sequence[float], world: int) -> list[list[int]]:
    """Longest-processing-time-first assignment of unit ids to ``world`` ranks.

    Deterministic: units in decreasing cost (ties: lower id first) go to the
    least-loaded rank (ties: lower rank).  Each rank's list is returned sorted.
    """
    if world <= 0:
        raise ValueError("world size must be positive")
    order = sorted(range(len(costs)), key=lambda u: (-float(costs[u]), u))
    load = [0.0] * world
    plan: list[list[int]] = [[] for _ in range(world)]
    for u in order:
        r = min(range(world), key=lambda i: (load[i], i))
        plan[r].append(u)
        load[r] += float(costs[u])
    return [sorted(p) for p in plan]


def _host_lists(full, local, query_counts, B):
    """Index lists on the host (one device-to-host copy) for the cost model."""
    f = full.detach().to("cpu")
    l = local.detach().to("cpu")
    if f.ndim == 1:
        f = f.unsqueeze(0)
        l = l.unsqueeze(0)
    fl, ll = [], []
    for b in range(B):
        fb, lb = f[b].numpy(), l[b].numpy()
        fl.append(fb[fb >= 0] if (B > 1 or query_counts is not None) else fb)
        ll.append(lb[lb >= 0] if (B > 1 or query_counts is not None) else lb)
    return fl, ll


def slot_map(plan: list[list[int]], n_slots: int | None = None) -> list[int]:
    """Unit id of every slot of an all-gathered unit-major buffer: rank p's units
    fill slots ``[p * n, p * n + len(plan[p]))`` (``n`` = the largest share), -1 pads."""
    n = max((len(p) for p in plan), default=0) if n_slots is None else n_slots
    ids = []
    for p in plan:
        ids.extend(list(p) + [-1] * (n - len(p)))
    return ids


_ID_CACHE: dict = {}


def _device_ids(unit_ids: Sequence[int], device: torch.device) -> torch.Tensor:
    """int32 device copy of a slot -> unit map, made once per (map, device): later
    calls enqueue no host-to-device copy."""
    key = (tuple(int(u) for u in unit_ids), device)
    t = _ID_CACHE.get(key)
    if t is None:
        if len(_ID_CACHE) > 256:
            _ID_CACHE.clear()
        t = torch.tensor(key[0], dtype=torch.int32).to(device)
        _ID_CACHE[key] = t
    return t


def _move_units(src: torch.Tensor, dst: torch.Tensor, unit_ids: Sequence[int], *, hkv: int, to_rows: bool) -> None:
    """Copy between a row-major ``[B, S, H, ...]`` tensor and a unit-major
    ``[n, S, r, ...]`` one (``H = hkv * r``); slots with unit id -1 are skipped.

    CUDA tensors: one ``swa_scatter_units`` / ``swa_gather_units`` kernel.  CPU
    tensors (the host-side tests over gloo): the same move by torch indexing.
    """
    rows, units = (dst, src) if to_rows else (src, dst)
    B, S, H = rows.shape[:3]
    r = H // hkv
    if units.shape[1] != S or units.shape[2] != r or units.shape[0] < len(unit_ids):
        raise ValueError("unit-major tensor must be [n, S, Hq / Hkv, ...] with a slot per unit id")
    if rows.dtype != units.dtype or not rows.is_contiguous() or not units.is_contiguous():
        raise ValueError("row-major and unit-major tensors must be contiguous and of one dtype")
    if rows.device.type == "cuda":
        lib = _native.load()
        ids = _device_ids(unit_ids, rows.device)
        chunk = r * rows[0, 0, 0].numel() * rows.element_size()
        fn = lib.swa_scatter_units if to_rows else lib.swa_gather_units
        with torch.cuda.device(rows.device):
            rc = fn(_native.ptr(src), _native.ptr(ids), len(unit_ids), S, hkv, chunk, H * chunk // r,
                    _native.ptr(dst), _native.stream_ptr(rows.device))
        _native.check(rc, "swa_scatter_units" if to_rows else "swa_gather_units")
        return
    view = rows.view(B, S, hkv, r, *rows.shape[3:])
    for i, u in enumerate(unit_ids):
        if u < 0:
            continue
        b, g = divmod(int(u), hkv)
        if to_rows:
            view[b, :, g].copy_(units[i])
        else:
            units[i].copy_(view[b, :, g])


def take_units(x: torch.Tensor, unit_ids: Sequence[int], *, hkv: int, slots: int | None = None) -> torch.Tensor:
    """Unit-major copy ``[max(n, slots), S, r, ...]`` of the units' slices of a
    row-major ``[B, S, H, ...]`` tensor (``r = H / hkv``; k / v: ``H = hkv``, r = 1)."""
    B, S, H = x.shape[:3]
    n = max(len(unit_ids), slots or 0)
    out = x.new_empty((n, S, H // hkv, *x.shape[3:]))
    _move_units(x, out, list(unit_ids), hkv=hkv, to_rows=False)
    return out


def all_gather_units(o_u: torch.Tensor, lse_u: torch.Tensor, plan: list[list[int]], *, group=None,
                     bufs: dict | None = None):
    """Every rank's unit-major outputs on every rank: ``([world * n, S, r, 128],
    [world * n, S, r])`` with rank p's units in slots ``[p * n, p * n + len(plan[p]))``
    (``n`` = the largest share).  One ``all_gather_into_tensor`` per tensor; at one
    rank (or without a process group) the inputs themselves.  ``bufs``: optional
    dict that keeps the receive buffers across calls."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    n_max = max(len(p) for p in plan)
    _, S, r, D = o_u.shape
    if o_u.shape[0] < n_max or lse_u.shape[0] < n_max:
        raise ValueError("o_u / lse_u need a slot for each unit of the largest share")
    send_o, send_l = o_u[:n_max], lse_u[:n_max]
    if world == 1:
        return send_o, send_l
    bufs = bufs if bufs is not None else {}
    key = (world, n_max, S, r, D, o_u.device)
    if bufs.get("key") != key:
        bufs.clear()
        bufs["key"] = key
        bufs["o"] = o_u.new_empty((world * n_max, S, r, D))
        bufs["l"] = lse_u.new_empty((world * n_max, S, r))
    dist.all_gather_into_tensor(bufs["o"], send_o, group=group)
    dist.all_gather_into_tensor(bufs["l"], send_l, group=group)
    return bufs["o"], bufs["l"]


def scatter_gathered(got_o: torch.Tensor, got_l: torch.Tensor, plan: list[list[int]], *, hkv: int,
                     out: torch.Tensor, lse: torch.Tensor) -> None:
    """Write all-gathered unit-major slots (``all_gather_units``) into row-major
    ``out`` ``[B, S, Hq, 128]`` / ``lse`` ``[B, S, Hq]``: one scatter kernel each."""
    n_max = max(len(p) for p in plan)
    ids = slot_map(plan, n_max)
    _move_units(got_o, out, ids, hkv=hkv, to_rows=True)
    _move_units(got_l, lse, ids, hkv=hkv, to_rows=True)


def gather_units_to_rows(o_u: torch.Tensor, lse_u: torch.Tensor, plan: list[list[int]], *, B: int, hkv: int,
                         out: torch.Tensor | None = None, lse: torch.Tensor | None = None, group=None,
                         _bufs: dict | None = None):
    """Replicate every rank's unit-major outputs on every rank, in row-major form.

    ``o_u`` ``[n, S, r, 128]`` / ``lse_u`` ``[n, S, r]``: this rank's units
    (``plan[rank]`` in order) in their first slots, ``n`` at least the largest
    share (slots past the rank's units are sent but never read).  One
    ``all_gather_into_tensor`` per tensor, then one scatter kernel each into
    ``out`` ``[B, S, Hq, 128]`` / ``lse`` ``[B, S, Hq]`` (allocated when None).
    """
    _, S, r, D = o_u.shape
    if out is None:
        out = o_u.new_empty((B, S, hkv * r, D))
    if lse is None:
        lse = lse_u.new_empty((B, S, hkv * r))
    if max(len(p) for p in plan) == 0:
        return out, lse
    got_o, got_l = all_gather_units(o_u, lse_u, plan, group=group, bufs=_bufs)
    scatter_gathered(got_o, got_l, plan, hkv=hkv, out=out, lse=lse)
    return out, lse


def gather_units(out: torch.Tensor, lse: torch.Tensor, plan: list[list[int]], *, hkv: int, group=None) -> None:
    """All-gather the O/LSE slices of every rank's units into ``out`` / ``lse`` in place
    (replicated-input form: this rank's units are already in place in ``out`` / ``lse``)."""
    rank = dist.get_rank(group)
    n_max = max(len(p) for p in plan)
    if n_max == 0:
        return
    stage_o = take_units(out, plan[rank], hkv=hkv, slots=n_max)
    stage_l = take_units(lse, plan[rank], hkv=hkv, slots=n_max)
    gather_units_to_rows(stage_o, stage_l, plan, B=out.shape[0], hkv=hkv, out=out, lse=lse, group=group)


def sharded_switch_gqa_prefill_forward(q, k, v, full_query_indices, local_query_indices, *, window_size=1024,
                                       sm_scale=None, metadata=None, query_counts=None, group=None,
                                       gather: bool = False, validate: bool = True, costs=None,
                                       compute: Callable | None = None):
    """Switch Attention prefill with (batch, KV group) units sharded over ``group``.

    Every rank passes the same (replicated) q/k/v and index lists.  Returns
    ``(out, lse, plan)``: ``plan[rank]`` lists the unit ids ``b * Hkv + g`` this
    rank computed.  Without ``gather`` only those slices of ``out`` / ``lse`` are
    defined on a rank; with ``gather=True`` every rank ends with the full result.
    ``costs`` (per unit) may be supplied to skip the host copy of the lists;
    ``compute(bg_list)`` replaces the kernel call (host-side tests).
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B = q.shape[0]
    hkv = k.shape[2]
    if costs is None:
        fl, ll = _host_lists(full_query_indices, local_query_indices, query_counts, B)
        costs = unit_costs(fl, ll, hkv=hkv, skv=k.shape[1], window=window_size, metadata=metadata)
    plan = plan_units(costs, world)
    mine = plan[rank]
    if compute is None:
        def compute(bg):
            out = torch.empty_like(q)
            lse = torch.empty(q.shape[:3], dtype=torch.float32, device=q.device)
            if bg:
                _core.forward(q, k, v, full_query_indices, local_query_indices, metadata=metadata,
                              window_size=window_size, sm_scale=sm_scale, validate=validate,
                              query_counts=query_counts, bg_list=bg, out=out, lse=lse)
            return out, lse
    out, lse = compute(mine)
    if gather and world > 1:
        gather_units(out, lse, plan, hkv=hkv, group=group)
    return out, lse, plan


class ReplicaBuffers:
    """Row-major O ``[B, S, Hq, 128]`` (BF16) and LSE ``[B, S, Hq]`` (FP32) of one
    sharded problem, on every rank of ``group``, in symmetric memory.

    Every rank's kernel writes its units' rows into all ranks' buffers directly
    (peer pointers over NVLink), so after ``forward_units_replicated`` every rank
    holds the whole result.  Allocated once per problem shape and reused across
    calls; ``out`` / ``lse`` are this rank's buffers.
    """

    def __init__(self, B: int, S: int, Hq: int, *, device, group=None):
        device = torch.device(device)
        self.shape = (B, S, Hq)
        single = not dist.is_initialized() or dist.get_world_size(group) == 1
        self._h_out = None
        if single:
            # one rank: plain device buffers, nothing to share
            self.out = torch.empty((B, S, Hq, 128), dtype=torch.bfloat16, device=device)
            self.lse = torch.empty((B, S, Hq), dtype=torch.float32, device=device)
            self.world = 1
            out_ptrs, lse_ptrs = [self.out.data_ptr()], [self.lse.data_ptr()]
        else:
            import torch.distributed._symmetric_memory as symm_mem

            if group is None:
                group = dist.group.WORLD
            self.out = symm_mem.empty((B, S, Hq, 128), dtype=torch.bfloat16, device=device)
            self.lse = symm_mem.empty((B, S, Hq), dtype=torch.float32, device=device)
            self._h_out = symm_mem.rendezvous(self.out, group)
            self._h_lse = symm_mem.rendezvous(self.lse, group)
            self.world = int(self._h_out.world_size)
            if self.world > 8:
                raise ValueError("at most 8 ranks can share replicated outputs")
            out_ptrs = list(self._h_out.buffer_ptrs)
            lse_ptrs = list(self._h_lse.buffer_ptrs)
        self._rep_out = (ctypes.c_void_p * self.world)(*out_ptrs)
        self._rep_lse = (ctypes.c_void_p * self.world)(*lse_ptrs)

    def barrier(self) -> None:
        """Device-side barrier of all ranks on the current stream: every rank's
        earlier writes into the buffers are complete and visible afterwards (a
        no-op with one rank: stream order suffices)."""
        if self._h_out is not None:
            self._h_out.barrier(channel=0)


def forward_units_replicated(q_u, k_u, v_u, full_u, local_u, counts_u, units: Sequence[int], rep: ReplicaBuffers, *,
                             hkv: int, window_size: int = 1024, sm_scale: float | None = None, metadata=None,
                             out=None, lse=None, barrier: bool = True, status_out=None):
    """This rank's units (unit-major, see ``take_units``) through the prefill
    kernel, every output row written into all ranks' ``rep`` buffers.

    ``full_u`` / ``local_u`` / ``counts_u``: the units' -1 padded index lists and
    ``[n, 2]`` counts (``build_switch_query_indices_batched`` of the units' mask
    rows).  ``units``: the global unit ids ``b * hkv + g`` of the n units, in order.
    ``out`` / ``lse``: optional unit-major outputs (not written when None).  With
    ``barrier`` (the default) the call starts with a device barrier of all ranks
    (nobody still reads the buffers' previous contents) and ends with one (every
    rank's rows have landed); without it those are the caller's.
    """
    _core.validate_qkv(q_u, k_u, v_u)
    n, S, r, D = q_u.shape
    if k_u.shape[2] != 1 or k_u.shape[0] != n or len(units) != n:
        raise ValueError("unit-major inputs: q [n, S, Hq/Hkv, 128], k / v [n, S, 1, 128], one unit id per row")
    B, S_rep, Hq = rep.shape
    if S_rep != S or Hq != hkv * r:
        raise ValueError("replica buffers do not match the problem")
    dev = q_u.device
    _core._check_status_out(status_out, dev)
    if counts_u.dtype != torch.int32 or tuple(counts_u.shape) != (n, 2) or counts_u.device != dev:
        raise ValueError("counts_u must be an int32 [n, 2] tensor on the device of q_u")
    f = full_u.to(dtype=torch.int32).contiguous()
    l = local_u.to(dtype=torch.int32).contiguous()
    scale = (sm_scale if sm_scale is not None else (1.0 / D) ** 0.5) * _core.LOG2E
    if not scale > 0:
        raise ValueError("sm_scale must be positive")
    fs = ls = ce = None
    if metadata is not None:
        _core._check_metadata(metadata, q_u, S, k_u.shape[1])
        fs, ls, ce = metadata.full_starts, metadata.local_starts, metadata.causal_ends
    gid = _device_ids(units, dev)
    ws = torch.zeros(4, dtype=torch.int32, device=dev)
    lib = _native.load()
    if barrier:
        rep.barrier()
    with torch.cuda.device(dev):
        rc = lib.swa_prefill_forward_replicated(
            _native.ptr(q_u), _native.ptr(k_u), _native.ptr(v_u),
            _native.ptr(f) if f.shape[1] else None, _native.ptr(l) if l.shape[1] else None,
            int(f.shape[1]), int(l.shape[1]), _native.ptr(counts_u.contiguous()),
            _native.ptr(fs), _native.ptr(ls), _native.ptr(ce), _native.ptr(gid),
            n, S, k_u.shape[1], r, D, int(window_size), float(scale), hkv, rep.world,
            ctypes.cast(rep._rep_out, ctypes.c_void_p), ctypes.cast(rep._rep_lse, ctypes.c_void_p),
            _native.ptr(out), _native.ptr(lse),
            _native.ptr(ws), ws.numel() * 4, _native.stream_ptr(dev))
    _native.check(rc, "forward_units_replicated")
    if barrier:
        rep.barrier()
    if status_out is not None or _core.CHECK_DEVICE_STATUS:
        _core.publish_status(ws[1:2], status_out)
    return rep.out, rep.lse
