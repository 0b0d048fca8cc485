"""The allocation-free entry point (swa_prefill_forward_noalloc), called through
the C ABI, must give the same output as the regular entry point: bit for bit,
since both run the same prefill kernel on the same units.

It exists for callers that may not allocate device memory at attention time
(the library keeps its scratch in a fixed array instead of a caller workspace).
This file is collected last so that a run stopping at the first failure has
already run every other test; it also passes on its own in a fresh process.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import metadata as oracle_meta
from oracle import indices as oracle_idx
from switchattentionkernels_b200 import _core, _native

pytestmark = pytest.mark.gpu

LOG2E = 1.4426950408889634


def _inputs(dev, B=3, S=700, Hq=8, Hkv=2, seed=77):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, S, Hq, 128, generator=g).bfloat16().to(dev)
    k = torch.randn(B, S, Hkv, 128, generator=g).bfloat16().to(dev)
    v = torch.randn(B, S, Hkv, 128, generator=g).bfloat16().to(dev)
    mask = np.random.default_rng(seed).random((B, S)) < np.linspace(0.1, 0.9, B)[:, None]
    full, local, _ = oracle_idx.compact_mask_batched(mask)
    nf = max(1, int((full >= 0).sum(1).max()))
    nl = max(1, int((local >= 0).sum(1).max()))
    full_t = torch.from_numpy(np.ascontiguousarray(full[:, :nf])).to(dev)
    local_t = torch.from_numpy(np.ascontiguousarray(local[:, :nl])).to(dev)
    return q, k, v, full_t, local_t


def _noalloc(lib, q, k, v, full, local, window, out, lse, status, metadata=None):
    B, S, Hq, D = q.shape
    fs = ls = ce = None
    if metadata is not None:
        fs, ls, ce = metadata.full_starts, metadata.local_starts, metadata.causal_ends
    rc = lib.swa_prefill_forward_noalloc(
        _native.ptr(q), _native.ptr(k), _native.ptr(v), _native.ptr(full), _native.ptr(local),
        full.shape[1], local.shape[1], _native.ptr(fs), _native.ptr(ls), _native.ptr(ce), _native.ptr(out),
        _native.ptr(lse), B, S, k.shape[1], Hq, k.shape[2], D, window, (D ** -0.5) * LOG2E, _native.ptr(status),
        _native.stream_ptr(q.device))
    assert rc == 0, lib.swa_last_error_string()


def _same(out, lse, ref_o, ref_l, label):
    # identical bits, NaN rows included (rows without a legal key)
    assert torch.equal(out.view(torch.int16), ref_o.view(torch.int16)), f"{label}: O differs"
    assert torch.equal(lse.view(torch.int32), ref_l.view(torch.int32)), f"{label}: LSE differs"


def test_noalloc_matches_regular_entry_point_twice(cuda_device):
    lib = _native.load()
    q, k, v, full, local = _inputs(cuda_device)
    W = 96
    ref_o, ref_l = _core.forward(q, k, v, full, local, window_size=W)
    for call in range(2):  # two calls in a row: the shared scratch must be reset each time
        out = torch.full_like(q, float("nan"))
        lse = torch.full(q.shape[:3], float("nan"), device=cuda_device)
        status = torch.full((2,), -1, dtype=torch.int32, device=cuda_device)
        _noalloc(lib, q, k, v, full, local, W, out, lse, status)
        torch.cuda.synchronize()
        assert status.tolist() == [0, 0], f"call {call}: status {status.tolist()}"
        _same(out, lse, ref_o, ref_l, f"call {call}")


def test_noalloc_matches_regular_entry_point_with_metadata(cuda_device):
    # packed sequences: per-row key bounds from the varlen metadata
    lib = _native.load()
    lengths = [200, 1, 333, 166]
    S = sum(lengths)
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    W = 80
    q, k, v, full, local = _inputs(cuda_device, B=1, S=S, Hq=16, Hkv=4, seed=78)
    md = {n: torch.from_numpy(a).to(cuda_device) for n, a in oracle_meta.build_metadata(S, S, W, cu).items()}
    meta = _core.SwitchAttentionMetadata(**md)
    ref_o, ref_l = _core.forward(q, k, v, full, local, metadata=meta, window_size=W)
    for call in range(2):
        out = torch.full_like(q, float("nan"))
        lse = torch.full(q.shape[:3], float("nan"), device=cuda_device)
        status = torch.full((2,), -1, dtype=torch.int32, device=cuda_device)
        _noalloc(lib, q, k, v, full, local, W, out, lse, status, metadata=meta)
        torch.cuda.synchronize()
        assert status.tolist() == [0, 0], f"call {call}: status {status.tolist()}"
        _same(out, lse, ref_o, ref_l, f"metadata call {call}")


def test_noalloc_rejects_batch_beyond_maximum(cuda_device):
    lib = _native.load()
    limit = lib.swa_noalloc_max_batch()
    assert limit == 2046
    q, k, v, full, local = _inputs(cuda_device, B=1, S=64)
    out = torch.empty_like(q)
    lse = torch.empty(q.shape[:3], device=cuda_device)
    rc = lib.swa_prefill_forward_noalloc(
        _native.ptr(q), _native.ptr(k), _native.ptr(v), _native.ptr(full), _native.ptr(local),
        full.shape[1], local.shape[1], None, None, None, _native.ptr(out), _native.ptr(lse),
        limit + 1, 64, 64, 8, 2, 128, 16, 0.1, None, _native.stream_ptr(cuda_device))
    assert rc == -1
    assert b"swa_noalloc_max_batch" in lib.swa_last_error_string()


def test_noalloc_reports_invalid_indices(cuda_device):
    lib = _native.load()
    q, k, v, full, local = _inputs(cuda_device, B=2, S=300)
    bad_full = full.clone()
    bad_full[1, 0] = 299  # breaks strict increase in row 1
    out = torch.empty_like(q)
    lse = torch.empty(q.shape[:3], device=cuda_device)
    status = torch.zeros((2,), dtype=torch.int32, device=cuda_device)
    _noalloc(lib, q, k, v, bad_full, local, 32, out, lse, status)
    torch.cuda.synchronize()
    assert status[0].item() & _native.STATUS_FULL_ORDER
