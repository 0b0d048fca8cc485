"""Routing-mask compaction and capacity-bucket preparation on the GPU: bit-exact
against the numpy oracle (which is itself pinned to the reference's code)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import indices as oracle_idx
from switchattentionkernels_b200 import swiattn_gqa_prefill_varlen as varlen
from switchattentionkernels_b200 import build_switch_query_indices_batched
from switchattentionkernels_b200 import workloads

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("S", [1, 2, 15, 16, 17, 1000, 16384, 16385, 65537])
@pytest.mark.parametrize("p", [0.0, 0.3, 1.0])
def test_compaction_bit_exact(cuda_device, S, p):
    g = torch.Generator().manual_seed(S)
    mask = torch.rand(S, generator=g) < p
    f, l = varlen.build_switch_query_indices(mask.to(cuda_device))
    rf, rl = oracle_idx.compact_mask(mask.numpy())
    assert f.dtype == torch.int32 and l.dtype == torch.int32
    assert np.array_equal(f.cpu().numpy(), rf)
    assert np.array_equal(l.cpu().numpy(), rl)


def test_compaction_batched_and_unaligned(cuda_device):
    g = torch.Generator().manual_seed(7)
    base = torch.rand(5, 3001, generator=g) < 0.4
    # a view starting at an odd byte offset exercises the unaligned load path
    big = torch.zeros(5 * 3001 + 3, dtype=torch.bool)
    big[3:] = base.flatten()
    mask = big[3:].view(5, 3001).to(cuda_device)
    full, local, counts = build_switch_query_indices_batched(mask)
    rf, rl, rc = oracle_idx.compact_mask_batched(base.numpy())
    assert np.array_equal(full.cpu().numpy(), rf)
    assert np.array_equal(local.cpu().numpy(), rl)
    assert np.array_equal(counts.cpu().numpy(), rc)


@pytest.mark.parametrize("cfg_id", [1, 2, 3, 4, 5])
def test_compaction_benchmark_configs(cuda_device, cfg_id):
    w = workloads.make_inputs(cfg_id, device="cpu") if cfg_id in (1, 2) else None
    if w is None:
        cfg = workloads.CONFIGS[cfg_id]
        S = cfg.S or 70000
        g = torch.Generator().manual_seed(cfg.seed)
        mask = torch.rand(cfg.B, S, generator=g) < cfg.p_full
    else:
        mask = w["mask"]
    full, local, counts = build_switch_query_indices_batched(mask.to(cuda_device))
    rf, rl, rc = oracle_idx.compact_mask_batched(mask.numpy())
    assert np.array_equal(full.cpu().numpy(), rf)
    assert np.array_equal(local.cpu().numpy(), rl)
    assert np.array_equal(counts.cpu().numpy(), rc)


@pytest.mark.parametrize("count", [1, 63, 64, 65, 128, 129, 1000, 4097])
@pytest.mark.parametrize("block_m", [64, 128])
def test_prepare_indices_buckets(cuda_device, count, block_m):
    rng = np.random.default_rng(count)
    idx = np.sort(rng.choice(5000, size=count, replace=False)).astype(np.int32)
    padded, cnt = varlen._prepare_indices(torch.from_numpy(idx).to(cuda_device), seq_len=5000, block_m=block_m)
    rp, rc = oracle_idx.prepare_indices(idx, seq_len=5000, block_m=block_m)
    assert np.array_equal(padded.cpu().numpy(), rp)
    assert int(cnt.item()) == rc and cnt.dtype == torch.int32 and cnt.shape == (1,)


@pytest.mark.parametrize("bad,msg", [
    ([3, 2, 5], oracle_idx.ERR_ORDER),
    ([1, 1, 5], oracle_idx.ERR_ORDER),
    ([-1, 2, 5], oracle_idx.ERR_RANGE),
    ([0, 2, 5000], oracle_idx.ERR_RANGE),
])
def test_prepare_indices_errors(cuda_device, bad, msg):
    with pytest.raises(ValueError, match=msg.replace("(", r"\(").replace(")", r"\)").replace("[", r"\[")):
        varlen._prepare_indices(torch.tensor(bad, dtype=torch.int32, device=cuda_device), seq_len=5000,
                                block_m=64)
