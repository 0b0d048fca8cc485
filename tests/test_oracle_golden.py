"""The CPU oracle against the golden vectors produced by the reference's own host
code (tests/golden/make_golden.py), and internal consistency of the oracle."""
from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from oracle import attention as oracle_attn
from oracle import indices as oracle_idx
from oracle import metadata as oracle_meta

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(GOLDEN, "reference_host.json")) as fh:
        record = json.load(fh)
    arrays = np.load(os.path.join(GOLDEN, "reference_host.npz"))
    return record, arrays


def test_compaction_matches_reference(golden):
    record, arrays = golden
    assert record["compaction"]
    for case in record["compaction"]:
        key = case["key"]
        mask = np.unpackbits(arrays[key + "_mask"])[: case["S"]].astype(bool)
        f, l = oracle_idx.compact_mask(mask)
        assert case["full_dtype"] == "torch.int32" and case["local_dtype"] == "torch.int32"
        assert np.array_equal(f, arrays[key + "_full"]), key
        assert np.array_equal(l, arrays[key + "_local"]), key


def test_prepare_matches_reference(golden):
    record, arrays = golden
    for case in record["prepare"]:
        key = case["key"]
        idx = arrays[key + "_in"]
        padded, count = oracle_idx.prepare_indices(idx, seq_len=case["seq_len"], block_m=case["block_m"])
        assert list(padded.shape) == case["padded_shape"], key
        assert np.array_equal(padded, arrays[key + "_padded"]), key
        assert count == int(arrays[key + "_count"][0]), key


def test_prepare_errors_match_reference(golden):
    record, _ = golden
    for case in record["prepare_errors"]:
        vals = np.asarray(case["values"], dtype=np.int32)
        if vals.ndim != 1:
            continue  # batch-shape error: host-side check of the product API (test_host_api)
        with pytest.raises(ValueError) as ei:
            oracle_idx.prepare_indices(vals, seq_len=case["seq_len"], block_m=64)
        assert case["error"]["type"] == "ValueError"
        assert str(ei.value) == case["error"]["message"], case["case"]


def test_bucket_capacity_matches_reference_dispatch(golden):
    record, arrays = golden
    for case in record["forward"]:
        mask = np.unpackbits(arrays[case["key"] + "_mask"])[: case["S"]].astype(bool)
        f, l = oracle_idx.compact_mask(mask)
        launches = {bool(x["is_local"]): x for x in case["launches"]}
        for is_local, lst in ((False, f), (True, l)):
            if lst.size == 0:
                assert is_local not in launches  # empty branch: no launch (reference :402,424)
                continue
            x = launches[is_local]
            assert x["num_queries"] == oracle_idx.bucket_capacity(lst.size, case["block_m"])
            assert x["query_count"] == [lst.size]
            got = np.asarray(x["query_indices"][0])
            assert np.array_equal(got[: lst.size], lst) and (got[lst.size:] == -1).all()
            assert x["window_size"] == case["window"]
            assert x["sm_scale"] == case["sm_scale"]


def test_tiled_replay_close_to_exact():
    """The reference's tile loop (BF16 P, running max) sits within the stated tolerance of the exact result."""
    g = torch.Generator().manual_seed(1)
    S, Hq, Hkv, W = 384, 8, 2, 100
    q = torch.randn(1, S, Hq, 128, generator=g).bfloat16()
    k = torch.randn(1, S, Hkv, 128, generator=g).bfloat16()
    v = torch.randn(1, S, Hkv, 128, generator=g).bfloat16()
    mask = np.random.default_rng(2).random(S) < 0.3
    f, l = oracle_idx.compact_mask(mask)
    O, L = oracle_attn.prefill_dense(q, k, v, [f], [l], window=W)
    for bm, bk in ((64, 64), (128, 128), (64, 128)):
        O2, L2 = oracle_attn.prefill_tiled(q, k, v, f, l, window=W, block_m=bm, block_k=bk)
        assert (O - O2).abs().max().item() < 2e-2
        assert (O - O2).abs().mean().item() < 2e-3
        assert (L - L2).abs().max().item() < 1e-4


def test_tiled_replay_metadata_equals_fixed():
    g = torch.Generator().manual_seed(3)
    S = 200
    q = torch.randn(1, S, 4, 128, generator=g).bfloat16()
    k = torch.randn(1, S, 2, 128, generator=g).bfloat16()
    v = torch.randn(1, S, 2, 128, generator=g).bfloat16()
    mask = np.random.default_rng(4).random(S) < 0.5
    f, l = oracle_idx.compact_mask(mask)
    meta = oracle_meta.build_metadata(S, S, 37)
    O1, L1 = oracle_attn.prefill_tiled(q, k, v, f, l, window=37)
    O2, L2 = oracle_attn.prefill_tiled(q, k, v, f, l, window=37, metadata=meta)
    assert torch.equal(O1, O2) and torch.equal(L1, L2)


def test_metadata_oracle_semantics():
    cu = np.array([0, 5, 5 + 300, 5 + 300 + 17])
    meta = oracle_meta.build_metadata(int(cu[-1]), int(cu[-1]), 64, cu)
    for s in range(len(cu) - 1):
        for t in range(cu[s], cu[s + 1]):
            assert meta["q_segment_ids"][t] == s
            assert meta["q_positions"][t] == t - cu[s]
            assert meta["full_starts"][t] == cu[s]
            assert meta["local_starts"][t] == max(cu[s], t - 63)
            assert meta["causal_ends"][t] == t + 1
    single = oracle_meta.build_metadata(50, 70, 8)
    assert np.array_equal(single["kv_positions"], np.arange(70))
    assert np.array_equal(single["local_starts"], np.maximum(np.arange(50) - 7, 0))
    assert all(len(single[n]) == L for n, L in zip(
        ["q_positions", "kv_positions", "q_segment_ids", "kv_segment_ids", "full_starts", "local_starts",
         "causal_ends"], [50, 70, 50, 70, 50, 50, 50]))


def test_empty_rows_give_nan_and_minus_inf():
    """A row with no legal key: O = 0/0 and LSE = log2(0) + m, as in the kernel."""
    q = torch.randn(1, 4, 2, 128).bfloat16()
    k = torch.randn(1, 2, 1, 128).bfloat16()
    v = torch.randn(1, 2, 1, 128).bfloat16()
    meta = oracle_meta.build_metadata(4, 2, 4)
    meta["full_starts"][3] = 5  # start beyond every key
    O, L = oracle_attn.prefill_dense(q, k, v, [np.array([3])], [np.array([0, 1, 2])], window=4, metadata=meta)
    assert torch.isnan(O[0, 3]).all() and torch.isneginf(L[0, 3]).all()
    assert torch.isfinite(L[0, :3]).all()
