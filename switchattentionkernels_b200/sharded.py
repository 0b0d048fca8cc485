"""Multi-GPU driver: one prefill sharded over the ranks of a process group.

The unit of work is a (batch b, KV group g) pair: it reads ``q[b, :, g*r:(g+1)*r]``,
``k/v[b, :, g]`` and batch b's index lists, and writes the same slice of O/LSE,
so units are independent and need no communication.  Units are assigned to
ranks by longest-processing-time-first on their cost (the legal score entries
of batch b), every rank computes only its own units (the kernel's ``bg_list``),
and -- only when the caller asks for a replicated result -- one all-gather moves
O (BF16) and LSE (FP32) of every unit to every rank (NCCL over NVLink for CUDA
tensors; any backend that implements ``all_gather``).

The reference has no distributed code; this driver implements the sharding
that its per-(batch, head) grid (``swiattn_gqa_prefill.py:69``) admits.
"""
from __future__ import annotations

from typing import Callable, Sequence

import numpy as np
import torch
import torch.distributed as dist

from . import _core


def unit_costs(full_lists: Sequence[np.ndarray], local_lists: Sequence[np.ndarray], *, hkv: int, skv: int,
               window: int) -> np.ndarray:
    """Cost of every unit ``b * hkv + g``: legal (row, key) entries of batch b."""
    B = len(full_lists)
    costs = np.zeros(B * hkv, dtype=np.float64)
    for b in range(B):
        f = np.asarray(full_lists[b], dtype=np.int64)
        l = np.asarray(local_lists[b], dtype=np.int64)
        n = float(np.minimum(f + 1, skv).sum())
        n += float(np.maximum(np.minimum(l + 1, skv) - np.maximum(l - window + 1, 0), 0).sum())
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


def gather_units(out: torch.Tensor, lse: torch.Tensor, plan: list[list[int]], *, hkv: int, group=None) -> None:
    """All-gather the O/LSE slices of every rank's units into ``out`` / ``lse`` in place."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B, S, Hq, D = out.shape
    r = Hq // hkv
    n_max = max(len(p) for p in plan)
    if n_max == 0:
        return
    # staging slots past a rank's own units are sent but never read: no fill
    stage_o = out.new_empty((n_max, S, r, D))
    stage_l = lse.new_empty((n_max, S, r))
    for i, u in enumerate(plan[rank]):
        b, g = divmod(u, hkv)
        stage_o[i].copy_(out[b, :, g * r:(g + 1) * r, :])
        stage_l[i].copy_(lse[b, :, g * r:(g + 1) * r])
    # one collective per tensor straight into a [world, n_max, ...] buffer
    got_o = out.new_empty((world, n_max, S, r, D))
    got_l = lse.new_empty((world, n_max, S, r))
    dist.all_gather_into_tensor(got_o.view(world * n_max, S, r, D), stage_o, group=group)
    dist.all_gather_into_tensor(got_l.view(world * n_max, S, r), stage_l, group=group)
    for p in range(world):
        if p == rank:
            continue
        for i, u in enumerate(plan[p]):
            b, g = divmod(u, hkv)
            out[b, :, g * r:(g + 1) * r, :].copy_(got_o[p][i])
            lse[b, :, g * r:(g + 1) * r].copy_(got_l[p][i])


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
        costs = unit_costs(fl, ll, hkv=hkv, skv=k.shape[1], window=window_size)
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
