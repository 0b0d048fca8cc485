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
