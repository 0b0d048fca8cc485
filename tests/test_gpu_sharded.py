"""The sharded (multi-GPU) path's device side, on one GPU.

Each rank of ``sharded_switch_gqa_prefill_forward`` launches the kernel on its
own (batch, KV group) units (``bg_list``).  Here the units of a 4-rank plan are
computed one rank after another into the same buffers; the union must equal the
unsharded launch bit for bit (each unit's computation does not depend on which
other units the launch holds).  The collective part runs through a one-rank
NCCL group.  Two-rank collectives and failure handling are covered on CPU
(``test_sharded_gloo.py``).
"""
from __future__ import annotations

import datetime
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist

from _parity import device_lists, lists_from_mask
from switchattentionkernels_b200 import _core
from switchattentionkernels_b200.sharded import plan_units, sharded_switch_gqa_prefill_forward, unit_costs

pytestmark = pytest.mark.gpu


def _inputs(dev, B=3, S=900, Hq=16, Hkv=4, seed=21):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, S, Hq, 128, generator=g).bfloat16().to(dev)
    k = torch.randn(B, S, Hkv, 128, generator=g).bfloat16().to(dev)
    v = torch.randn(B, S, Hkv, 128, generator=g).bfloat16().to(dev)
    mask = torch.rand(B, S, generator=g) < torch.tensor([0.1, 0.5, 0.9]).unsqueeze(1)
    return q, k, v, mask


def test_units_of_a_plan_compose_to_the_full_result(cuda_device):
    q, k, v, mask = _inputs(cuda_device)
    B, Hkv, W = q.shape[0], k.shape[2], 200
    full, local = lists_from_mask(mask)
    fi, li = device_lists(full, local, cuda_device, B)
    ref_o, ref_l = _core.forward(q, k, v, fi, li, window_size=W)
    plan = plan_units(unit_costs(full, local, hkv=Hkv, skv=k.shape[1], window=W), 4)
    assert sorted(u for p in plan for u in p) == list(range(B * Hkv))
    out = torch.full_like(q, float("nan"))
    lse = torch.full(q.shape[:3], float("nan"), device=cuda_device)
    for units in plan:
        if units:
            _core.forward(q, k, v, fi, li, window_size=W, bg_list=units, out=out, lse=lse)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_o)
    assert torch.equal(lse, ref_l)


def test_sharded_forward_one_rank_nccl(cuda_device):
    if dist.is_initialized():
        pytest.skip("a process group is already initialised")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", str(29400 + (os.getpid() % 500)))
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60),
                            device_id=cuda_device)
    try:
        q, k, v, mask = _inputs(cuda_device, seed=22)
        W = 300
        full, local = lists_from_mask(mask)
        fi, li = device_lists(full, local, cuda_device, q.shape[0])
        out, lse, plan = sharded_switch_gqa_prefill_forward(q, k, v, fi, li, window_size=W, gather=True)
        ref_o, ref_l = _core.forward(q, k, v, fi, li, window_size=W)
        torch.cuda.synchronize()
        assert plan == [list(range(q.shape[0] * k.shape[2]))]
        assert torch.equal(out, ref_o) and torch.equal(lse, ref_l)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("Hq,Hkv", [(16, 4), (8, 8), (12, 2)])
def test_unit_moves_round_trip(cuda_device, Hq, Hkv):
    # swa_gather_units / swa_scatter_units: a rank's unit slices out of row-major
    # tensors and back, bit for bit (O rows of r * 256 bytes, LSE rows of r * 4
    # bytes: the 16-byte and the 4-byte word paths), padding slots skipped
    from switchattentionkernels_b200 import sharded

    g = torch.Generator().manual_seed(Hq + Hkv)
    B, S = 3, 257
    o = torch.randn(B, S, Hq, 128, generator=g).bfloat16().to(cuda_device)
    l = torch.randn(B, S, Hq, generator=g).to(cuda_device)
    units = [5 % (B * Hkv), 0, B * Hkv - 1]
    o_u = sharded.take_units(o, units, hkv=Hkv, slots=5)
    l_u = sharded.take_units(l, units, hkv=Hkv, slots=5)
    r = Hq // Hkv
    for i, u in enumerate(units):
        b, gg = divmod(u, Hkv)
        assert torch.equal(o_u[i], o[b, :, gg * r:(gg + 1) * r]) and torch.equal(l_u[i], l[b, :, gg * r:(gg + 1) * r])
    o2 = torch.zeros_like(o)
    l2 = torch.zeros_like(l)
    sharded._move_units(o_u, o2, units + [-1, -1], hkv=Hkv, to_rows=True)
    sharded._move_units(l_u, l2, units + [-1, -1], hkv=Hkv, to_rows=True)
    torch.cuda.synchronize()
    o_v, o2_v = o.view(B, S, Hkv, r, 128), o2.view(B, S, Hkv, r, 128)
    for u in range(B * Hkv):
        b, gg = divmod(u, Hkv)
        if u in units:
            assert torch.equal(o2_v[b, :, gg], o_v[b, :, gg])
        else:
            assert not o2_v[b, :, gg].any()


def test_unit_major_forward_equals_row_major_slices(cuda_device):
    # a rank's units held unit-major ([n, S, r, 128] q, [n, S, 1, 128] k / v, the units'
    # mask rows) through the ordinary forward: bit-equal to those units' slices of the
    # row-major launch; the gather (one rank: scatter only) rebuilds the whole result
    from switchattentionkernels_b200 import build_switch_query_indices_batched, sharded

    q, k, v, mask = _inputs(cuda_device, seed=23)
    B, S, Hq, _ = q.shape
    Hkv, W = k.shape[2], 150
    r = Hq // Hkv
    full, local, counts = build_switch_query_indices_batched(mask.to(cuda_device))
    ref_o, ref_l = _core.forward(q, k, v, full, local, window_size=W, query_counts=counts)
    fl, ll = lists_from_mask(mask)
    plan = plan_units(unit_costs(fl, ll, hkv=Hkv, skv=S, window=W), 3)
    n_max = max(len(p) for p in plan)
    o_all = torch.empty((3 * n_max, S, r, 128), dtype=torch.bfloat16, device=cuda_device)
    l_all = torch.empty((3 * n_max, S, r), dtype=torch.float32, device=cuda_device)
    for rank, units in enumerate(plan):
        q_u, k_u, v_u = (sharded.take_units(t, units, hkv=Hkv) for t in (q, k, v))
        m_u = mask[torch.tensor([u // Hkv for u in units])].to(cuda_device)
        f_u, l_u, c_u = build_switch_query_indices_batched(m_u)
        o_u, lse_u = _core.forward(q_u, k_u, v_u, f_u, l_u, window_size=W, query_counts=c_u)
        torch.cuda.synchronize()
        for i, u in enumerate(units):
            b, g = divmod(u, Hkv)
            assert torch.equal(o_u[i], ref_o[b, :, g * r:(g + 1) * r]), f"unit {u} O"
            assert torch.equal(lse_u[i], ref_l[b, :, g * r:(g + 1) * r]), f"unit {u} LSE"
        o_all[rank * n_max:rank * n_max + len(units)] = o_u
        l_all[rank * n_max:rank * n_max + len(units)] = lse_u
    out = torch.full_like(q, float("nan"))
    lse = torch.full((B, S, Hq), float("nan"), device=cuda_device)
    sharded.scatter_gathered(o_all, l_all, plan, hkv=Hkv, out=out, lse=lse)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_o) and torch.equal(lse, ref_l)


class _LocalReplicas:
    """Stand-in for ReplicaBuffers on one GPU: several row-major buffers of this
    device (the kernel path is the same; the peer pointers come from symmetric
    memory in the multi-GPU case)."""

    def __init__(self, B, S, Hq, dev, copies):
        import ctypes

        self.shape = (B, S, Hq)
        self.outs = [torch.full((B, S, Hq, 128), float("nan"), dtype=torch.bfloat16, device=dev) for _ in range(copies)]
        self.lses = [torch.full((B, S, Hq), float("nan"), device=dev) for _ in range(copies)]
        self.world = copies
        self._rep_out = (ctypes.c_void_p * copies)(*[t.data_ptr() for t in self.outs])
        self._rep_lse = (ctypes.c_void_p * copies)(*[t.data_ptr() for t in self.lses])
        self.out, self.lse = self.outs[0], self.lses[0]

    def barrier(self):
        pass


def test_replicated_epilogue_writes_every_copy(cuda_device):
    # each "rank" of a 3-rank plan runs its unit-major units through the replicating
    # launch; every row-major copy must equal the row-major forward bit for bit
    from switchattentionkernels_b200 import build_switch_query_indices_batched, sharded

    q, k, v, mask = _inputs(cuda_device, seed=24)
    B, S, Hq, _ = q.shape
    Hkv, W = k.shape[2], 170
    full, local, counts = build_switch_query_indices_batched(mask.to(cuda_device))
    ref_o, ref_l = _core.forward(q, k, v, full, local, window_size=W, query_counts=counts)
    fl, ll = lists_from_mask(mask)
    plan = plan_units(unit_costs(fl, ll, hkv=Hkv, skv=S, window=W), 3)
    rep = _LocalReplicas(B, S, Hq, cuda_device, copies=3)
    for units in plan:
        q_u, k_u, v_u = (sharded.take_units(t, units, hkv=Hkv) for t in (q, k, v))
        m_u = mask[torch.tensor([u // Hkv for u in units])].to(cuda_device)
        f_u, l_u, c_u = build_switch_query_indices_batched(m_u)
        o_u = torch.empty_like(q_u)
        lse_u = torch.empty(q_u.shape[:3], device=cuda_device)
        sharded.forward_units_replicated(q_u, k_u, v_u, f_u, l_u, c_u, units, rep, hkv=Hkv, window_size=W,
                                         out=o_u, lse=lse_u, barrier=False)
        torch.cuda.synchronize()
        for i, u in enumerate(units):
            b, g = divmod(u, Hkv)
            r = Hq // Hkv
            assert torch.equal(o_u[i], ref_o[b, :, g * r:(g + 1) * r]), f"unit {u}: unit-major O"
            assert torch.equal(lse_u[i], ref_l[b, :, g * r:(g + 1) * r]), f"unit {u}: unit-major LSE"
    for t in range(3):
        assert torch.equal(rep.outs[t], ref_o), f"copy {t}: O"
        assert torch.equal(rep.lses[t], ref_l), f"copy {t}: LSE"


def _replica_worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from switchattentionkernels_b200 import build_switch_query_indices_batched, sharded

        q, k, v, mask = _inputs(dev, seed=25)
        B, S, Hq, _ = q.shape
        Hkv, W = k.shape[2], 260
        fl, ll = lists_from_mask(mask)
        plan = plan_units(unit_costs(fl, ll, hkv=Hkv, skv=S, window=W), world)
        units = plan[rank]
        q_u, k_u, v_u = (sharded.take_units(t, units, hkv=Hkv) for t in (q, k, v))
        m_u = mask[torch.tensor([u // Hkv for u in units])].to(dev)
        f_u, l_u, c_u = build_switch_query_indices_batched(m_u)
        rep = sharded.ReplicaBuffers(B, S, Hq, device=dev)
        for _ in range(2):  # the buffers are reused across calls
            out, lse = sharded.forward_units_replicated(q_u, k_u, v_u, f_u, l_u, c_u, units, rep, hkv=Hkv,
                                                        window_size=W)
        full, local, counts = build_switch_query_indices_batched(mask.to(dev))
        ref_o, ref_l = _core.forward(q, k, v, full, local, window_size=W, query_counts=counts)
        torch.cuda.synchronize()
        ok = bool(torch.equal(out, ref_o) and torch.equal(lse, ref_l))
        result_q.put((rank, "ok" if ok else "mismatch"))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        result_q.put((rank, "error:" + type(e).__name__ + ":" + str(e)[:300]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def test_replicated_outputs_two_gpus():
    # every rank's kernel writes its units' rows into both ranks' symmetric-memory
    # buffers over NVLink; each rank must end with the whole row-major result
    import multiprocessing as mp_std
    import socket

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp_std.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_replica_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    assert res == [(0, "ok"), (1, "ok")], res
