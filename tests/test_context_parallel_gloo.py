"""Context-parallel host logic on CPU ranks (gloo): the zigzag row split, the
K/V all-gather into token order, and the composition (each
rank's rows against the gathered K/V with the rows' global key bounds) checked
against the unsplit FP32 oracle.  The kernel itself runs in the GPU tests."""
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
from oracle import metadata as oracle_md
from switchattentionkernels_b200 import context_parallel as cp


def _check_partition(plan):
    S, world = plan.total_len, plan.world
    shards = [plan.rows(r) for r in range(world)]
    assert np.array_equal(np.sort(np.concatenate(shards)), np.arange(S))
    for rows in shards:
        assert np.all(np.diff(rows) > 0)
    assert plan.capacity == max(s.size for s in shards)
    return shards


@pytest.mark.parametrize("S,world", [(64, 1), (1000, 2), (1001, 2), (4097, 3), (8192, 4), (130, 8), (17, 8), (1, 2)])
def test_zigzag_rows_partition_the_token_axis(S, world):
    shards = _check_partition(cp.make_cp_plan(S, world))
    sizes = [s.size for s in shards]
    assert max(sizes) - min(sizes) <= 2
    assert np.array_equal(shards[0], cp.cp_shard_rows(S, world, 0))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_cost_balanced_zigzag_on_packed_sequences(world):
    rng = np.random.default_rng(world)
    lengths = rng.integers(512, 8193, size=16)
    cu = np.concatenate([[0], np.cumsum(lengths)])
    S = int(cu[-1])
    mask = rng.random(S) < 0.3
    costs = cp.cp_row_costs(mask, 4096, cu)
    plan = cp.make_cp_plan(S, world, costs)
    shards = _check_partition(plan)
    load = [costs[r].sum() for r in shards]
    # one row of granularity per chunk boundary: at most 2 * max row cost away from the mean
    assert max(load) - min(load) <= 4 * costs.max()
    uniform = [costs[r].sum() for r in _check_partition(cp.make_cp_plan(S, world))]
    assert max(load) / np.mean(load) < max(uniform) / np.mean(uniform)


def test_row_costs_are_the_legal_keys():
    cu = np.array([0, 5, 12])
    mask = np.array([1, 0, 1, 0, 0, 1, 0, 0, 0, 1, 0, 0], dtype=bool)
    got = cp.cp_row_costs(mask, 3, cu)
    pos = np.array([0, 1, 2, 3, 4, 0, 1, 2, 3, 4, 5, 6])
    want = np.where(mask, pos + 1, np.minimum(pos + 1, 3))
    assert np.array_equal(got, want)


def test_zigzag_balances_causal_work():
    S, world = 1 << 16, 8
    pos = np.arange(S, dtype=np.float64)
    costs = [float((pos[cp.cp_shard_rows(S, world, r)] + 1).sum()) for r in range(world)]
    assert max(costs) / min(costs) < 1.01
    # contiguous blocks would be 15x apart
    block = S // world
    naive = [float((pos[r * block:(r + 1) * block] + 1).sum()) for r in range(world)]
    assert max(naive) / min(naive) > 10


def test_bad_arguments():
    with pytest.raises(ValueError):
        cp.cp_shard_rows(100, 2, 2)
    with pytest.raises(ValueError):
        cp.make_cp_plan(0, 2)
    with pytest.raises(ValueError):
        cp.make_cp_plan(10, 0)
    with pytest.raises(ValueError):
        cp.make_cp_plan(10, 2, row_costs=np.ones(9))
    with pytest.raises(ValueError):
        cp.make_cp_plan(10, 2, row_costs=-np.ones(10))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(S=301):
    g = torch.Generator().manual_seed(5)
    Hq, Hkv = 4, 2
    q = torch.randn(1, S, Hq, 128, generator=g).bfloat16()
    k = torch.randn(1, S, Hkv, 128, generator=g).bfloat16()
    v = torch.randn(1, S, Hkv, 128, generator=g).bfloat16()
    mask = np.random.default_rng(6).random(S) < 0.4
    cu = np.array([0, 90, 91, 240, S]) if S > 240 else np.array([0, S])
    return q, k, v, mask, cu


def _worker(rank, world, port, mode, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        q, k, v, mask, cu = _problem(1 if mode == "tiny" else 301)
        S = q.shape[1]
        W = 37
        plan = cp.make_cp_plan(S, world, cp.cp_row_costs(mask, W, cu) if mode == "compose" else None)
        rows = plan.rows(rank)
        idx = torch.from_numpy(rows)
        k_full, v_full = cp.cp_gather_kv(k[:, idx].contiguous(), v[:, idx].contiguous(), plan)
        gathered = bool(torch.equal(k_full, k) and torch.equal(v_full, v))
        if mode in ("gather", "tiny"):
            result_q.put((rank, "ok" if gathered else "gather mismatch"))
            return
        md = oracle_md.build_metadata(S, S, W, cu)
        # the rows' own key bounds against the whole token axis (what cp_metadata builds on the device)
        md_local = {key: (val[rows] if key in ("q_positions", "q_segment_ids", "full_starts", "local_starts",
                                                 "causal_ends") else val) for key, val in md.items()}
        lmask = mask[rows]
        full_local, local_local = np.nonzero(lmask)[0], np.nonzero(~lmask)[0]
        O, L = oracle_attn.prefill_dense(q[:, idx], k_full, v_full, [full_local], [local_local], window=W,
                                         metadata=md_local)
        Og, Lg = oracle_attn.prefill_dense(q, k, v, [np.nonzero(mask)[0]], [np.nonzero(~mask)[0]], window=W,
                                           metadata=md)
        ok = gathered and torch.allclose(O[0], Og[0, idx], atol=1e-5, rtol=0) and torch.allclose(
            L[0], Lg[0, idx], atol=1e-5, rtol=0)
        result_q.put((rank, "ok" if ok else "mismatch"))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        result_q.put((rank, "error:" + type(e).__name__ + ":" + str(e)[:200]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    return sorted(res)


@pytest.mark.parametrize("world", [2, 3])
def test_kv_exchange_restores_token_order(world):
    assert _run(world, "gather") == [(r, "ok") for r in range(world)]


def test_kv_exchange_with_a_rank_that_holds_no_rows():
    # one token over two ranks: rank 1 holds nothing and still takes part in the exchange
    assert cp.make_cp_plan(1, 2).rows(1).size == 0
    assert _run(2, "tiny") == [(0, "ok"), (1, "ok")]


def test_context_parallel_rows_equal_the_unsplit_oracle():
    assert _run(2, "compose") == [(0, "ok"), (1, "ok")]
