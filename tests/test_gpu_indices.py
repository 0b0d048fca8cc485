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


def _router_case(B, S, dtype, pair, seed):
    g = torch.Generator().manual_seed(seed)
    shape = (B, S, 2) if pair else (B, S)
    r = torch.randn(shape, generator=g).to(dtype)
    flat = r.view(-1)
    if flat.numel() > 20:
        flat[3] = float("nan")
        flat[10:14] = 0.0        # ties (pairs) and scores equal to a zero threshold
    return r


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("pair", [False, True])
@pytest.mark.parametrize("B,S", [(1, 1), (1, 17), (2, 1000), (3, 16384), (1, 16385), (2, 40001)])
@pytest.mark.parametrize("threshold", [0.0, 0.7])
def test_router_compaction_bit_exact(cuda_device, dtype, pair, B, S, threshold):
    from switchattentionkernels_b200 import build_switch_query_indices_from_router
    r = _router_case(B, S, dtype, pair, seed=B * 100003 + S)
    full, local, counts = build_switch_query_indices_from_router(r.to(cuda_device), threshold=threshold, pair=pair)
    mask = oracle_idx.router_mask(r.float().numpy(), pair=pair, threshold=threshold)
    rf, rl, rc = oracle_idx.compact_mask_batched(mask)
    assert np.array_equal(full.cpu().numpy(), rf)
    assert np.array_equal(local.cpu().numpy(), rl)
    assert np.array_equal(counts.cpu().numpy(), rc)


@pytest.mark.parametrize("pair", [False, True])
def test_router_compaction_unaligned_and_1d(cuda_device, pair):
    from switchattentionkernels_b200 import build_switch_query_indices_from_router
    S = 5003
    per = 2 if pair else 1
    g = torch.Generator().manual_seed(11)
    big = torch.randn(S * per + 1, generator=g).to(torch.bfloat16).to(cuda_device)
    r = big[1:].view(S, 2) if pair else big[1:]   # starts 2 bytes past a 16-byte boundary
    full, local, counts = build_switch_query_indices_from_router(r, threshold=0.1, pair=pair)
    mask = oracle_idx.router_mask(r.float().cpu().numpy()[None], pair=pair, threshold=0.1)
    rf, rl, rc = oracle_idx.compact_mask_batched(mask)
    assert np.array_equal(full.cpu().numpy(), rf) and np.array_equal(local.cpu().numpy(), rl)
    assert np.array_equal(counts.cpu().numpy(), rc)


def test_router_compaction_errors(cuda_device):
    from switchattentionkernels_b200 import build_switch_query_indices_from_router
    with pytest.raises(TypeError):
        build_switch_query_indices_from_router(torch.zeros(10, dtype=torch.float16, device=cuda_device))
    with pytest.raises(ValueError):
        build_switch_query_indices_from_router(torch.zeros(2, 10, 3, device=cuda_device), pair=True)
    with pytest.raises(TypeError):
        build_switch_query_indices_from_router(torch.zeros(10))


@pytest.mark.parametrize("B,S,p", [(1, 1 << 20, 0.3), (3, 100003, 0.5), (2, 4097, 0.5), (2, 70000, 0.0),
                                   (2, 70000, 1.0)])
def test_chunked_compaction_bit_exact(cuda_device, B, S, p):
    # rows longer than one 4096-token chunk are split over several CTAs
    g = torch.Generator().manual_seed(B + S)
    mask = torch.rand(B, S, generator=g) < p
    full, local, counts = build_switch_query_indices_batched(mask.to(cuda_device))
    rf, rl, rc = oracle_idx.compact_mask_batched(mask.numpy())
    assert np.array_equal(counts.cpu().numpy(), rc)
    assert np.array_equal(full.cpu().numpy(), rf)
    assert np.array_equal(local.cpu().numpy(), rl)


def test_chunked_compaction_unaligned_rows(cuda_device):
    B, S = 3, 9001   # odd row length: rows 1 and 2 start off a 16-byte boundary
    g = torch.Generator().manual_seed(5)
    mask = torch.rand(B, S, generator=g) < 0.4
    full, local, counts = build_switch_query_indices_batched(mask.to(cuda_device))
    rf, rl, rc = oracle_idx.compact_mask_batched(mask.numpy())
    assert np.array_equal(full.cpu().numpy(), rf) and np.array_equal(local.cpu().numpy(), rl)
    assert np.array_equal(counts.cpu().numpy(), rc)


def test_chunked_and_single_cta_paths_agree(cuda_device):
    from switchattentionkernels_b200 import _native
    lib = _native.load()
    B, S = 2, 50000
    g = torch.Generator().manual_seed(9)
    mask = (torch.rand(B, S, generator=g) < 0.2).to(cuda_device)
    outs = []
    for chunked in (False, True):
        full = torch.empty(B, S, dtype=torch.int32, device=cuda_device)
        local = torch.empty_like(full)
        counts = torch.empty(B, 2, dtype=torch.int32, device=cuda_device)
        if chunked:
            n = int(lib.swa_compact_workspace_elems(B, S))
            assert n == B * ((S + 4095) // 4096)
            ws = torch.empty(n, dtype=torch.int32, device=cuda_device)
            rc = lib.swa_compact_mask_ws(_native.ptr(mask), B, S, _native.ptr(full), _native.ptr(local),
                                         _native.ptr(counts), _native.ptr(ws), n, _native.stream_ptr(cuda_device))
            assert lib.swa_compact_mask_ws(_native.ptr(mask), B, S, _native.ptr(full), _native.ptr(local),
                                           _native.ptr(counts), _native.ptr(ws), n - 1,
                                           _native.stream_ptr(cuda_device)) != 0   # workspace too small
        else:
            rc = lib.swa_compact_mask(_native.ptr(mask), B, S, _native.ptr(full), _native.ptr(local),
                                      _native.ptr(counts), _native.stream_ptr(cuda_device))
        assert rc == 0
        outs.append((full.cpu(), local.cpu(), counts.cpu()))
    for a, b in zip(*outs):
        assert torch.equal(a, b)
