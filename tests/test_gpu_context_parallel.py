"""Context-parallel prefill on the GPU: the per-rank key bounds, every rank's rows
(emulated on one GPU against the whole K/V, which is what the all-gather
delivers) against the FP32 oracle and the unsplit launch, a one-rank NCCL group
through the public entry point, and -- when the box has two GPUs -- two NCCL
ranks with the real K/V all-gather."""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from _parity import compare, oracle_subset
from oracle import metadata as oracle_md
from switchattentionkernels_b200 import _core, context_parallel as cp
from switchattentionkernels_b200.metadata import build_switch_attention_metadata

pytestmark = pytest.mark.gpu


def _problem(dev, S=2600, Hq=8, Hkv=2, seed=31, p=0.4):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(1, S, Hq, 128, generator=g).bfloat16()
    k = torch.randn(1, S, Hkv, 128, generator=g).bfloat16()
    v = torch.randn(1, S, Hkv, 128, generator=g).bfloat16()
    mask = torch.rand(S, generator=g) < p
    cu = np.array([0, 700, 701, 1900, S], dtype=np.int64)
    return q.to(dev), k.to(dev), v.to(dev), mask.numpy(), cu


def _lists(mask_rows, dev):
    f = np.nonzero(mask_rows)[0]
    l = np.nonzero(~mask_rows)[0]
    return (torch.from_numpy(f).to(device=dev, dtype=torch.int32),
            torch.from_numpy(l).to(device=dev, dtype=torch.int32))


@pytest.mark.parametrize("world", [2, 4])
def test_cp_metadata_is_the_rows_global_bounds(cuda_device, world):
    S, W = 2600, 300
    cu = np.array([0, 700, 701, 1900, S], dtype=np.int64)
    ref = oracle_md.build_metadata(S, S, W, cu)
    for rank in range(world):
        rows = cp.cp_shard_rows(S, world, rank)
        md = cp.cp_metadata(S, rows, device=cuda_device, window_size=W,
                            cu_seqlens=torch.from_numpy(cu).int())
        for name in ("q_positions", "q_segment_ids", "full_starts", "local_starts", "causal_ends"):
            assert np.array_equal(getattr(md, name).cpu().numpy(), ref[name][rows]), name
        for name in ("kv_positions", "kv_segment_ids"):
            assert np.array_equal(getattr(md, name).cpu().numpy(), ref[name]), name


@pytest.mark.parametrize("world,balanced", [(2, False), (3, False), (4, True)])
def test_cp_rows_match_the_oracle_and_the_unsplit_launch(cuda_device, world, balanced):
    dev = cuda_device
    q, k, v, mask, cu = _problem(dev, seed=30 + world)
    S, W = q.shape[1], 300
    cu_t = torch.from_numpy(cu).int()
    md_all = build_switch_attention_metadata(S, S, device=dev, window_size=W, cu_seqlens=cu_t)
    fa, la = _lists(mask, dev)
    ref_o, ref_l = _core.forward(q, k, v, fa, la, metadata=md_all, window_size=W)
    O, L = oracle_subset(q, k, v, [np.nonzero(mask)[0]], [np.nonzero(~mask)[0]], W,
                         metadata=oracle_md.build_metadata(S, S, W, cu))
    plan = cp.make_cp_plan(S, world, cp.cp_row_costs(mask, W, cu) if balanced else None)
    for rank in range(world):
        rows = plan.rows(rank)
        idx = torch.from_numpy(rows).to(dev)
        md = cp.cp_metadata(S, rows, device=dev, window_size=W, cu_seqlens=cu_t)
        fl, ll = _lists(mask[rows], dev)
        o, l = _core.forward(q.index_select(1, idx).contiguous(), k, v, fl, ll, metadata=md, window_size=W)
        torch.cuda.synchronize()
        ridx = torch.from_numpy(rows)
        compare(o[0], l[0], O[0, ridx], L[0, ridx], label=f"rank {rank} vs oracle")
        compare(o[0], l[0], ref_o[0].float().cpu()[ridx], ref_l[0].cpu()[ridx], label=f"rank {rank} vs unsplit")


def test_cp_one_rank_nccl_equals_the_plain_forward(cuda_device):
    if dist.is_initialized():
        pytest.skip("a process group is already initialised")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ["MASTER_PORT"] = str(29900 + (os.getpid() % 500))
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60),
                            device_id=cuda_device)
    try:
        q, k, v, mask, cu = _problem(cuda_device, S=1500, seed=40)
        S, W = q.shape[1], 200
        cu_t = torch.from_numpy(np.array([0, 500, S])).int()
        fl, ll = _lists(mask, cuda_device)
        o, l = cp.context_parallel_switch_gqa_prefill_forward(q, k, v, fl, ll, total_len=S, cu_seqlens=cu_t,
                                                              window_size=W)
        md = build_switch_attention_metadata(S, S, device=cuda_device, window_size=W, cu_seqlens=cu_t)
        ref_o, ref_l = _core.forward(q, k, v, fl, ll, metadata=md, window_size=W)
        torch.cuda.synchronize()
        assert torch.equal(o, ref_o) and torch.equal(l, ref_l)
    finally:
        dist.destroy_process_group()


def test_cp_kv_exchange_one_rank(cuda_device):
    # one rank: the exchange copies the shard (two zigzag chunks) into its own
    # buffer; the forward through it equals the plain forward bit for bit
    dev = cuda_device
    q, k, v, mask, cu = _problem(dev, S=1500, seed=44)
    S, W = q.shape[1], 200
    cu_t = torch.from_numpy(np.array([0, 500, S])).int()
    plan = cp.make_cp_plan(S, 1)
    kvx = cp.KVExchange(S, k.shape[2], device=dev)
    k_full, v_full = kvx.exchange(k, v, plan)
    torch.cuda.synchronize()
    assert torch.equal(k_full, k) and torch.equal(v_full, v)
    md = build_switch_attention_metadata(S, S, device=dev, window_size=W, cu_seqlens=cu_t)
    fl, ll = _lists(mask, dev)
    o1, l1 = _core.forward(q, k_full, v_full, fl, ll, metadata=md, window_size=W)
    o0, l0 = _core.forward(q, k, v, fl, ll, metadata=md, window_size=W)
    torch.cuda.synchronize()
    assert torch.equal(o0, o1) and torch.equal(l0, l1)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_gpu_worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        q, k, v, mask, cu = _problem(dev, seed=50)
        S, W = q.shape[1], 300
        cu_t = torch.from_numpy(cu).int()
        costs = cp.cp_row_costs(mask, W, cu)
        rows = cp.make_cp_plan(S, world, costs).rows(rank)
        idx = torch.from_numpy(rows).to(dev)
        fl, ll = _lists(mask[rows], dev)
        o, l = cp.context_parallel_switch_gqa_prefill_forward(
            q.index_select(1, idx).contiguous(), k.index_select(1, idx).contiguous(),
            v.index_select(1, idx).contiguous(), fl, ll, total_len=S, cu_seqlens=cu_t, window_size=W,
            row_costs=costs)
        md = build_switch_attention_metadata(S, S, device=dev, window_size=W, cu_seqlens=cu_t)
        fa, la = _lists(mask, dev)
        ref_o, ref_l = _core.forward(q, k, v, fa, la, metadata=md, window_size=W)
        torch.cuda.synchronize()
        ridx = torch.from_numpy(rows)
        compare(o[0], l[0], ref_o[0].float().cpu()[ridx], ref_l[0].cpu()[ridx], label=f"rank {rank}")
        # the symmetric-memory exchange: the whole K/V axis on every rank, and the same
        # rows bit for bit as through the NCCL all-gather (twice: the buffers are reused)
        plan = cp.make_cp_plan(S, world, costs)
        kvx = cp.KVExchange(S, k.shape[2], device=dev)
        kl, vl = k.index_select(1, idx).contiguous(), v.index_select(1, idx).contiguous()
        for _ in range(2):
            k_full, v_full = kvx.exchange(kl, vl, plan)
            torch.cuda.synchronize()
            assert torch.equal(k_full, k) and torch.equal(v_full, v), "exchanged K/V differ"
            o2, l2 = cp.context_parallel_switch_gqa_prefill_forward(
                q.index_select(1, idx).contiguous(), kl, vl, fl, ll, total_len=S, cu_seqlens=cu_t, window_size=W,
                plan=plan, kv_exchange=kvx)
            torch.cuda.synchronize()
            assert torch.equal(o2, o) and torch.equal(l2, l), "symmetric-memory exchange changed the rows"
        del kvx, k_full, v_full
        result_q.put((rank, "ok"))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        result_q.put((rank, "error:" + type(e).__name__ + ":" + str(e)[:300]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def test_cp_two_gpus_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_gpu_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    assert res == [(0, "ok"), (1, "ok")]
