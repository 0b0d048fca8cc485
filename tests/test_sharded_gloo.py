"""Host logic of the multi-GPU driver on CPU ranks (gloo, world size 2): unit
planning, the O/LSE all-gather, and failure behaviour.  The kernel call is
replaced by the CPU oracle computing exactly the rank's units."""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import attention as oracle_attn
from oracle import indices as oracle_idx
from switchattentionkernels_b200 import sharded


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    g = torch.Generator().manual_seed(0)
    B, S, Hq, Hkv = 3, 96, 4, 2
    q = torch.randn(B, S, Hq, 128, generator=g).bfloat16()
    k = torch.randn(B, S, Hkv, 128, generator=g).bfloat16()
    v = torch.randn(B, S, Hkv, 128, generator=g).bfloat16()
    mask = np.random.default_rng(1).random((B, S)) < np.array([[0.1], [0.5], [0.9]])
    full = [oracle_idx.compact_mask(m)[0] for m in mask]
    local = [oracle_idx.compact_mask(m)[1] for m in mask]
    return q, k, v, full, local


def _worker(rank, world, port, mode, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        q, k, v, full, local = _inputs()
        W = 20
        hkv = k.shape[2]
        r = q.shape[2] // hkv
        costs = sharded.unit_costs(full, local, hkv=hkv, skv=k.shape[1], window=W)

        def compute(bg):
            out = torch.full(q.shape, float("nan"), dtype=torch.bfloat16)
            lse = torch.full(q.shape[:3], float("nan"))
            O, L = oracle_attn.prefill_dense(q, k, v, full, local, window=W)
            for u in bg:
                b, g = divmod(u, hkv)
                out[b, :, g * r:(g + 1) * r] = O[b, :, g * r:(g + 1) * r].bfloat16()
                lse[b, :, g * r:(g + 1) * r] = L[b, :, g * r:(g + 1) * r]
            return out, lse

        if mode == "unit_major":
            # a rank holds only its units, unit-major: [n, S, r, 128] q and [n, S, 1, 128]
            # k / v with each unit's batch lists; the forward over them is the ordinary
            # forward with B = n, Hq = r, Hkv = 1
            plan = sharded.plan_units(costs, world)
            mine = plan[rank]
            n_max = max(len(x) for x in plan)
            q_u, k_u, v_u = (sharded.take_units(t, mine, hkv=hkv, slots=n_max) for t in (q, k, v))
            fl = [full[u // hkv] for u in mine] + [np.zeros(0, np.int32)] * (n_max - len(mine))
            ll = [local[u // hkv] for u in mine] + [np.arange(q.shape[1], dtype=np.int32)] * (n_max - len(mine))
            O_u, L_u = oracle_attn.prefill_dense(q_u, k_u, v_u, fl, ll, window=W)
            out, lse = sharded.gather_units_to_rows(O_u.bfloat16(), L_u, plan, B=q.shape[0], hkv=hkv)
            O, L = oracle_attn.prefill_dense(q, k, v, full, local, window=W)
            ok = bool(torch.equal(out, O.bfloat16()) and torch.equal(lse, L))
            result_q.put((rank, "ok" if ok else "mismatch", plan))
            return
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before its launch")
        out, lse, plan = sharded.sharded_switch_gqa_prefill_forward(
            q, k, v, None, None, window_size=W, group=None, gather=True, costs=costs, compute=compute)
        O, L = oracle_attn.prefill_dense(q, k, v, full, local, window=W)
        ok = bool(torch.equal(out, O.bfloat16()) and torch.equal(lse, L))
        result_q.put((rank, "ok" if ok else "mismatch", plan))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        result_q.put((rank, "error:" + type(e).__name__ + ":" + str(e)[:200], None))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(2):
        rank, status, plan = q.get(timeout=120)
        results[rank] = (status, plan)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


def test_plan_is_lpt_and_deterministic():
    costs = [5, 9, 1, 9, 3, 7, 2, 8]
    plan = sharded.plan_units(costs, 3)
    assert sorted(u for p in plan for u in p) == list(range(8))
    loads = [sum(costs[u] for u in p) for p in plan]
    assert max(loads) - min(loads) <= max(costs)
    assert plan == sharded.plan_units(costs, 3)
    assert sharded.plan_units(costs, 1) == [list(range(8))]
    assert sharded.plan_units([1.0] * 4, 8)[4:] == [[], [], [], []]


def test_unit_costs_match_oracle_counts():
    _, k, _, full, local = _inputs()
    costs = sharded.unit_costs(full, local, hkv=2, skv=k.shape[1], window=20)
    for b in range(3):
        n = oracle_attn.legal_key_counts([full[b]], [local[b]], window=20, skv=k.shape[1])
        assert costs[2 * b] == costs[2 * b + 1] == n


def test_sharded_gather_two_ranks():
    res = _run("ok")
    assert res[0][0] == "ok" and res[1][0] == "ok", res
    plan = res[0][1]
    assert plan == res[1][1]
    assert sorted(u for p in plan for u in p) == list(range(6))


def test_failing_rank_surfaces_as_error_not_hang():
    res = _run("fail")
    assert res[1][0].startswith("error:RuntimeError")
    assert res[0][0].startswith("error:"), res  # the surviving rank's collective times out and raises


def test_unit_costs_with_metadata_match_oracle_counts():
    # packed sequences: costs come from the per-row bounds, not from raw positions
    from oracle import metadata as oracle_meta

    rng = np.random.default_rng(5)
    cu = np.array([0, 40, 41, 150, 200])
    S = int(cu[-1])
    md = oracle_meta.build_metadata(S, S, 16, cu)
    fl, ll = [], []
    for b in range(2):
        m = rng.random(S) < 0.3
        fl.append(np.nonzero(m)[0].astype(np.int32))
        ll.append(np.nonzero(~m)[0].astype(np.int32))
    costs = sharded.unit_costs(fl, ll, hkv=3, skv=S, window=16, metadata=md)
    plain = sharded.unit_costs(fl, ll, hkv=3, skv=S, window=16)
    for b in range(2):
        n = oracle_attn.legal_key_counts([fl[b]], [ll[b]], window=16, skv=S, metadata=md)
        assert (costs[3 * b:3 * b + 3] == n).all()
    assert (costs < plain).all()  # full rows of later sequences no longer count earlier sequences' keys


def test_unit_major_shards_compose_to_the_whole_result():
    res = _run("unit_major")
    assert res[0][0] == "ok" and res[1][0] == "ok", res
    assert sorted(u for p in res[0][1] for u in p) == list(range(6))
