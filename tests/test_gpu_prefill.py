"""Parity of the sm_100a prefill kernel against the FP32 CPU oracle (GPU)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _parity import compare, device_lists, lists_from_mask, oracle_subset
from oracle import metadata as oracle_meta
from switchattentionkernels_b200 import swiattn_gqa_prefill as fixed
from switchattentionkernels_b200 import swiattn_gqa_prefill_varlen as varlen
from switchattentionkernels_b200 import workloads

pytestmark = pytest.mark.gpu


def _rand_qkv(B, Sq, Skv, Hq, Hkv, seed, dev, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, Sq, Hq, 128, generator=g) * scale).bfloat16()
    k = (torch.randn(B, Skv, Hkv, 128, generator=g) * scale).bfloat16()
    v = (torch.randn(B, Skv, Hkv, 128, generator=g) * scale).bfloat16()
    return q.to(dev), k.to(dev), v.to(dev)


def _run(q, k, v, mask, window, label, sm_scale=None, module=fixed):
    B = q.shape[0]
    full, local = lists_from_mask(mask)
    fi, li = device_lists(full, local, q.device, B)
    O, LSE = module.switch_gqa_prefill_forward(q, k, v, fi, li, window_size=window, sm_scale=sm_scale)
    torch.cuda.synchronize()
    O_ref, LSE_ref = oracle_subset(q, k, v, full, local, window, sm_scale=sm_scale)
    return compare(O, LSE, O_ref, LSE_ref, label=label)


def test_config1_full_parity(cuda_device):
    w = workloads.make_inputs(1, device=cuda_device)
    _run(w["q"], w["k"], w["v"], w["mask"], w["window"], "config1")


@pytest.mark.parametrize("p_full", [0.0, 1.0, 0.5])
def test_all_full_all_local(cuda_device, p_full):
    q, k, v = _rand_qkv(1, 1024, 1024, 8, 2, 11, cuda_device)
    mask = torch.rand(1, 1024, generator=torch.Generator().manual_seed(3)) < p_full
    _run(q, k, v, mask, 256, f"p_full={p_full}")


@pytest.mark.parametrize("window", [1, 127, 128, 129, 5000])
def test_window_edges(cuda_device, window):
    q, k, v = _rand_qkv(1, 777, 777, 4, 1, 5, cuda_device)
    mask = torch.rand(1, 777, generator=torch.Generator().manual_seed(window)) < 0.3
    _run(q, k, v, mask, window, f"window={window}")


@pytest.mark.parametrize("n_full", [1, 63, 64, 65, 128, 129, 255, 256, 257])
def test_bucket_boundary_counts(cuda_device, n_full):
    S = 640
    q, k, v = _rand_qkv(1, S, S, 8, 2, n_full, cuda_device)
    rng = np.random.default_rng(n_full)
    pos = rng.choice(S, size=n_full, replace=False)
    mask = torch.zeros(1, S, dtype=torch.bool)
    mask[0, torch.from_numpy(pos)] = True
    _run(q, k, v, mask, 100, f"n_full={n_full}")


def test_first_last_positions_routed(cuda_device):
    S = 1000
    q, k, v = _rand_qkv(1, S, S, 8, 2, 21, cuda_device)
    mask = torch.zeros(1, S, dtype=torch.bool)
    mask[0, [0, 1, S - 2, S - 1]] = True
    _run(q, k, v, mask, 64, "first/last full")
    _run(q, k, v, ~mask, 64, "first/last local")


@pytest.mark.parametrize("Sq,Skv", [(500, 700), (700, 500), (300, 1), (129, 129)])
def test_unequal_lengths_and_partial_tiles(cuda_device, Sq, Skv):
    q, k, v = _rand_qkv(1, Sq, Skv, 8, 4, Sq + Skv, cuda_device)
    mask = torch.rand(1, Sq, generator=torch.Generator().manual_seed(Sq)) < 0.4
    _run(q, k, v, mask, 96, f"Sq={Sq},Skv={Skv}")


@pytest.mark.parametrize("Hq,Hkv", [(4, 4), (8, 4), (16, 2), (16, 1), (6, 2), (12, 2), (64, 8), (48, 3)])
def test_gqa_group_sizes(cuda_device, Hq, Hkv):
    q, k, v = _rand_qkv(1, 600, 600, Hq, Hkv, Hq * 7 + Hkv, cuda_device)
    mask = torch.rand(1, 600, generator=torch.Generator().manual_seed(Hq)) < 0.35
    _run(q, k, v, mask, 200, f"Hq={Hq},Hkv={Hkv}")


@pytest.mark.parametrize("Hq,Hkv,S", [(64, 1, 300), (128, 1, 200), (256, 1, 150), (96, 3, 200)])
def test_large_gqa_groups(cuda_device, Hq, Hkv, S):
    # 64 heads per KV head: one Q box covers two positions; 128: one position per
    # tile; 256: a position's heads span both tiles of a unit; 32 (96/3): 4 per tile
    q, k, v = _rand_qkv(1, S, S, Hq, Hkv, 17 + Hq, cuda_device)
    mask = torch.rand(1, S, generator=torch.Generator().manual_seed(Hq)) < 0.5
    _run(q, k, v, mask, 64, f"Hq={Hq} Hkv={Hkv}")


@pytest.mark.parametrize("B,Hq,Hkv", [(3, 48, 4), (5, 16, 2), (2, 96, 6)])
def test_many_groups_unit_order(cuda_device, B, Hq, Hkv):
    # more (batch, KV group) groups than the kernel keeps for the tail, so the
    # local units of the first groups run between full units; 48/4 also gives
    # three head blocks per group; rows with no full row, all full rows and mixed
    S = 640
    q, k, v = _rand_qkv(B, S, S, Hq, Hkv, 40 + B + Hq, cuda_device)
    dens = torch.tensor([[0.0], [1.0], [0.3], [0.6], [0.05]])[:B]
    mask = torch.rand(B, S, generator=torch.Generator().manual_seed(B * Hkv)) < dens
    _run(q, k, v, mask, 96, f"B={B} Hq={Hq} Hkv={Hkv}")


def test_batched_padded_lists(cuda_device):
    B, S = 3, 900
    q, k, v = _rand_qkv(B, S, S, 8, 2, 33, cuda_device)
    g = torch.Generator().manual_seed(4)
    mask = torch.rand(B, S, generator=g) < torch.tensor([[0.1], [0.5], [0.9]])
    _run(q, k, v, mask, 128, "B=3")


def test_sm_scale(cuda_device):
    q, k, v = _rand_qkv(1, 512, 512, 8, 2, 44, cuda_device)
    mask = torch.rand(1, 512, generator=torch.Generator().manual_seed(9)) < 0.5
    _run(q, k, v, mask, 64, "sm_scale", sm_scale=0.05)


def test_varlen_metadata(cuda_device):
    lengths = [37, 300, 1, 129, 640, 77]
    S = sum(lengths)
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    q, k, v = _rand_qkv(1, S, S, 16, 2, 55, cuda_device)
    mask = torch.rand(1, S, generator=torch.Generator().manual_seed(10)) < 0.3
    W = 200
    meta = varlen.build_switch_attention_metadata(S, S, device=cuda_device, window_size=W,
                                                  cu_seqlens=torch.from_numpy(cu))
    ref_meta = oracle_meta.build_metadata(S, S, W, cu)
    for name, arr in ref_meta.items():
        assert np.array_equal(getattr(meta, name).cpu().numpy(), arr), name
    full, local = lists_from_mask(mask)
    fi, li = device_lists(full, local, cuda_device, 1)
    O, LSE = varlen.switch_gqa_prefill_forward(q, k, v, fi, li, metadata=meta, window_size=W)
    torch.cuda.synchronize()
    O_ref, LSE_ref = oracle_subset(q, k, v, full, local, W, metadata=ref_meta)
    compare(O, LSE, O_ref, LSE_ref, label="varlen")


def test_varlen_default_metadata_matches_fixed(cuda_device):
    q, k, v = _rand_qkv(1, 800, 800, 8, 2, 66, cuda_device)
    mask = torch.rand(1, 800, generator=torch.Generator().manual_seed(12)) < 0.4
    full, local = lists_from_mask(mask)
    fi, li = device_lists(full, local, cuda_device, 1)
    O1, L1 = varlen.switch_gqa_prefill_forward(q, k, v, fi, li, window_size=150)
    meta = varlen.build_switch_attention_metadata(800, 800, device=cuda_device, window_size=150)
    O2, L2 = varlen.switch_gqa_prefill_forward(q, k, v, fi, li, metadata=meta, window_size=150)
    torch.cuda.synchronize()
    assert torch.equal(O1, O2) and torch.equal(L1, L2)


def test_config2_full_parity(cuda_device):
    w = workloads.make_inputs(2, device=cuda_device)
    _run(w["q"], w["k"], w["v"], w["mask"], w["window"], "config2")


@pytest.mark.parametrize("Sq,Skv,W,Hq,Hkv", [(900, 300, 64, 8, 2), (700, 500, 96, 8, 4), (1200, 200, 1, 4, 1)])
def test_rows_without_keys_fixed_length(cuda_device, Sq, Skv, W, Hq, Hkv):
    # local rows at t >= Skv + W - 1 have no legal key; they share units with
    # rows that have keys (full rows, and local rows below the threshold)
    q, k, v = _rand_qkv(1, Sq, Skv, Hq, Hkv, Sq * 3 + W, cuda_device)
    mask = torch.rand(1, Sq, generator=torch.Generator().manual_seed(Sq + W)) < 0.5
    full, local = lists_from_mask(mask)
    assert (local[0] >= Skv + W - 1).any() and (local[0] < Skv + W - 1).any()
    fi, li = device_lists(full, local, cuda_device, 1)
    O, LSE = fixed.switch_gqa_prefill_forward(q, k, v, fi, li, window_size=W)
    torch.cuda.synchronize()
    O_ref, LSE_ref = oracle_subset(q, k, v, full, local, W)
    empty = torch.isneginf(LSE_ref)
    assert empty.any() and (~empty).any()
    compare(O, LSE, O_ref, LSE_ref, label=f"Sq={Sq} Skv={Skv} W={W}")


def test_rows_without_keys_varlen_metadata(cuda_device):
    # metadata rows with start == end (first row of a sequence given no key) and
    # start > end (last row of a sequence); the bounds stay monotone along the
    # rows, as every metadata builder produces them
    lengths = [130, 1, 257, 64, 300]
    S = sum(lengths)
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    W = 48
    q, k, v = _rand_qkv(1, S, S, 16, 4, 77, cuda_device)
    ref_meta = oracle_meta.build_metadata(S, S, W, cu)
    fs, ls, ce = (ref_meta[n].copy() for n in ("full_starts", "local_starts", "causal_ends"))
    for s in cu[1:-1]:
        ce[s] = s                      # start == end at a sequence start
    for e in cu[2:]:
        if e - 1 not in cu:
            fs[e - 1] = ls[e - 1] = e  # start > end at a sequence end
            ce[e - 1] = e - 1
    for arr in (fs, ls, ce):
        assert (np.diff(arr.astype(np.int64)) >= 0).all()
    ref_meta = dict(ref_meta, full_starts=fs, local_starts=ls, causal_ends=ce)
    meta = varlen.SwitchAttentionMetadata(**{n: torch.from_numpy(a).to(cuda_device) for n, a in ref_meta.items()})
    for p_full in (0.0, 0.4, 1.0):
        mask = torch.rand(1, S, generator=torch.Generator().manual_seed(int(p_full * 10))) < p_full
        full, local = lists_from_mask(mask)
        fi, li = device_lists(full, local, cuda_device, 1)
        O, LSE = varlen.switch_gqa_prefill_forward(q, k, v, fi, li, metadata=meta, window_size=W)
        torch.cuda.synchronize()
        O_ref, LSE_ref = oracle_subset(q, k, v, full, local, W, metadata=ref_meta)
        assert torch.isneginf(LSE_ref).any()
        compare(O, LSE, O_ref, LSE_ref, label=f"varlen empty rows p_full={p_full}")
