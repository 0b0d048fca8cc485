"""Key-split pieces of long full-causal units (swa_prefill_forward_split) on the GPU.

A forced small piece length (``key_split=2`` tiles) splits every full-branch unit
of more than two 128-key tiles into pieces that run on different CTAs; the merge
kernel combines their partial O / LSE.  Every row is checked against the FP32
oracle with the stated tolerances (rows without a legal key: O = NaN, LSE =
-inf), and against the unsplit launch (each piece rounds P to BF16 against its
own running max, so the two agree to rounding, not bit for bit).  The automatic
plan is checked on a shape where it splits: one (batch, KV group) unit of a
16K-token sequence with a handful of full-causal rows.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from _parity import compare, compare_every_row_on_device, device_lists, lists_from_mask, oracle_subset
from oracle import metadata as oracle_meta
from switchattentionkernels_b200 import _core, _native
from switchattentionkernels_b200 import swiattn_gqa_prefill_varlen as varlen

pytestmark = pytest.mark.gpu

SPLIT_VS_UNSPLIT_O = 1e-2
SPLIT_VS_UNSPLIT_LSE = 1e-3


def _rand_qkv(B, Sq, Skv, Hq, Hkv, seed, dev):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Sq, Hq, 128, generator=g).bfloat16()
    k = torch.randn(B, Skv, Hkv, 128, generator=g).bfloat16()
    v = torch.randn(B, Skv, Hkv, 128, generator=g).bfloat16()
    return q.to(dev), k.to(dev), v.to(dev)


def _close_to_unsplit(O, LSE, O0, L0, label):
    fin = torch.isfinite(L0)
    assert torch.equal(fin, torch.isfinite(LSE)), f"{label}: rows without keys differ"
    assert torch.isnan(O[~fin]).all(), f"{label}: rows without keys must be NaN"
    assert (O[fin].float() - O0[fin].float()).abs().max().item() <= SPLIT_VS_UNSPLIT_O, f"{label}: O vs unsplit"
    assert (LSE[fin] - L0[fin]).abs().max().item() <= SPLIT_VS_UNSPLIT_LSE, f"{label}: LSE vs unsplit"


class _SplitSpy:
    """Records the split_tiles argument of every swa_prefill_forward_split call."""

    def __init__(self, monkeypatch):
        self.tiles = []
        lib = _native.load()
        real = lib.swa_prefill_forward_split

        def spy(*args):
            self.tiles.append(args[-4])
            return real(*args)

        monkeypatch.setattr(lib, "swa_prefill_forward_split", spy)


def _plan(q, k, n_full, n_local, window, request, n_bg=0):
    lib = _native.load()
    tiles = ctypes.c_int(0)
    nbytes = lib.swa_prefill_split_plan(q.shape[0], k.shape[1], q.shape[2], k.shape[2], n_full, n_local, n_bg, window,
                                        lib.swa_num_sms(q.device.index or 0), request, ctypes.byref(tiles))
    return int(nbytes), tiles.value


@pytest.mark.parametrize("B,Sq,Skv,Hq,Hkv,W,p_full", [
    (1, 1500, 1500, 8, 2, 100, 0.5),
    (2, 2100, 2100, 16, 2, 300, 0.3),   # B > 1 (padded lists), 8 query heads per KV head
    (1, 700, 500, 8, 4, 96, 0.6),       # Sq > Skv: local rows without a key
    (1, 1000, 1000, 32, 1, 64, 0.8),    # 32 heads per KV head: 8 positions per unit
])
def test_forced_split_matches_oracle_and_unsplit(cuda_device, monkeypatch, B, Sq, Skv, Hq, Hkv, W, p_full):
    q, k, v = _rand_qkv(B, Sq, Skv, Hq, Hkv, Sq + Hq + W, cuda_device)
    mask = torch.rand(B, Sq, generator=torch.Generator().manual_seed(Sq * 7 + W)) < p_full
    full, local = lists_from_mask(mask)
    fi, li = device_lists(full, local, cuda_device, B)
    nbytes, tiles = _plan(q, k, fi.shape[-1], li.shape[-1], W, 2)
    assert tiles == 2 and nbytes > 0
    O0, L0 = _core.forward(q, k, v, fi, li, window_size=W, key_split=None)
    spy = _SplitSpy(monkeypatch)
    for call in range(2):  # a second call on fresh outputs
        O, LSE = _core.forward(q, k, v, fi, li, window_size=W, key_split=2)
        assert spy.tiles == [2] * (call + 1)
        torch.cuda.synchronize()
        O_ref, LSE_ref = oracle_subset(q, k, v, full, local, W)
        compare(O, LSE, O_ref, LSE_ref, label=f"split call {call}")
        _close_to_unsplit(O, LSE, O0, L0, f"split call {call}")


def test_forced_split_on_a_unit_subset(cuda_device):
    # bg_list: only some (batch, KV group) units are computed; the others stay untouched
    B, S, Hq, Hkv, W = 2, 1200, 8, 2, 128
    q, k, v = _rand_qkv(B, S, S, Hq, Hkv, 5, cuda_device)
    mask = torch.rand(B, S, generator=torch.Generator().manual_seed(6)) < 0.5
    full, local = lists_from_mask(mask)
    fi, li = device_lists(full, local, cuda_device, B)
    out = torch.full_like(q, 7.0)
    lse = torch.full(q.shape[:3], 7.0, device=cuda_device)
    units = [3, 0]
    _core.forward(q, k, v, fi, li, window_size=W, key_split=2, bg_list=units, out=out, lse=lse)
    torch.cuda.synchronize()
    O_ref, LSE_ref = oracle_subset(q, k, v, full, local, W)
    r = Hq // Hkv
    for u in range(B * Hkv):
        b, g = divmod(u, Hkv)
        heads = slice(g * r, (g + 1) * r)
        if u in units:
            compare(out[b:b + 1, :, heads], lse[b:b + 1, :, heads], O_ref[b:b + 1, :, heads],
                    LSE_ref[b:b + 1, :, heads], label=f"unit {u}")
        else:
            assert (out[b, :, heads] == 7.0).all() and (lse[b, :, heads] == 7.0).all(), f"unit {u} written"


def test_forced_split_varlen_rows_without_keys(cuda_device):
    # metadata with start == end and start > end rows: every piece of such a row is
    # empty, and the merge writes O = NaN, LSE = -inf
    lengths = [700, 1, 900, 400]
    S = sum(lengths)
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    W = 64
    q, k, v = _rand_qkv(1, S, S, 16, 4, 78, cuda_device)
    ref_meta = oracle_meta.build_metadata(S, S, W, cu)
    fs, ls, ce = (ref_meta[n].copy() for n in ("full_starts", "local_starts", "causal_ends"))
    for s in cu[1:-1]:
        ce[s] = s
    for e in cu[2:]:
        if e - 1 not in cu:
            fs[e - 1] = ls[e - 1] = e
            ce[e - 1] = e - 1
    ref_meta = dict(ref_meta, full_starts=fs, local_starts=ls, causal_ends=ce)
    meta = varlen.SwitchAttentionMetadata(**{n: torch.from_numpy(a).to(cuda_device) for n, a in ref_meta.items()})
    mask = torch.rand(1, S, generator=torch.Generator().manual_seed(9)) < 0.6
    full, local = lists_from_mask(mask)
    fi, li = device_lists(full, local, cuda_device, 1)
    O0, L0 = _core.forward(q, k, v, fi, li, metadata=meta, window_size=W, key_split=None)
    O, LSE = _core.forward(q, k, v, fi, li, metadata=meta, window_size=W, key_split=2)
    torch.cuda.synchronize()
    O_ref, LSE_ref = oracle_subset(q, k, v, full, local, W, metadata=ref_meta)
    assert torch.isneginf(LSE_ref).any()
    compare(O, LSE, O_ref, LSE_ref, label="varlen split")
    _close_to_unsplit(O, LSE, O0, L0, "varlen split")


def test_automatic_split_on_few_long_full_units(cuda_device, monkeypatch):
    # one unit of a 16K-token sequence with ~80 full-causal rows: three full units of
    # up to 128 key tiles against ~500 short window units, so the plan splits them
    B, S, Hq, Hkv, W = 1, 16384, 8, 1, 256
    q, k, v = _rand_qkv(B, S, S, Hq, Hkv, 11, cuda_device)
    mask = torch.rand(B, S, generator=torch.Generator().manual_seed(12)) < 0.005
    full, local = lists_from_mask(mask)
    fi, li = device_lists(full, local, cuda_device, B)
    nbytes, tiles = _plan(q, k, fi.shape[-1], li.shape[-1], W, 0)
    assert nbytes > 0 and 0 < tiles < 128, (nbytes, tiles)
    O0, L0 = _core.forward(q, k, v, fi, li, window_size=W, key_split=None)
    spy = _SplitSpy(monkeypatch)
    O, LSE = _core.forward(q, k, v, fi, li, window_size=W)  # "auto": the list lengths are the counts
    assert spy.tiles == [tiles]
    torch.cuda.synchronize()
    compare_every_row_on_device(O, LSE, q, k, v, full, local, W, label="auto split")
    _close_to_unsplit(O, LSE, O0, L0, "auto split")
    # the same unit through [B, S] padded lists and device counts (no validation):
    # the plan sees the counts only through max_counts
    fp, lp, counts = _core.build_switch_query_indices_batched(mask.to(cuda_device))
    O2, L2 = _core.forward(q, k, v, fp, lp, window_size=W, validate=False, query_counts=counts)
    assert spy.tiles == [tiles]  # list capacities only: no split
    O3, L3 = _core.forward(q, k, v, fp, lp, window_size=W, validate=False, query_counts=counts,
                           max_counts=(len(full[0]), len(local[0])))
    assert spy.tiles == [tiles, tiles]
    torch.cuda.synchronize()
    assert torch.equal(O2.view(torch.int16), O0.view(torch.int16)) and torch.equal(L2, L0)
    assert torch.equal(O3.view(torch.int16), O.view(torch.int16)) and torch.equal(L3, LSE)


def test_split_pieces_write_the_scratch(cuda_device):
    # through the C ABI with a zeroed scratch: the pieces' partial LSE slots are
    # written (so the split ran), and the merged rows match the unsplit launch
    B, S, Hq, Hkv, W = 1, 3000, 8, 2, 128
    q, k, v = _rand_qkv(B, S, S, Hq, Hkv, 21, cuda_device)
    mask = torch.rand(B, S, generator=torch.Generator().manual_seed(22)) < 0.3
    full, local = lists_from_mask(mask)
    fi, li = device_lists(full, local, cuda_device, B)
    nf, nl = fi.numel(), li.numel()
    nbytes, tiles = _plan(q, k, nf, nl, W, 3)
    assert tiles == 3
    lib = _native.load()
    scratch = torch.zeros(nbytes, dtype=torch.uint8, device=cuda_device)
    ws = torch.zeros(4, dtype=torch.int32, device=cuda_device)
    out = torch.empty_like(q)
    lse = torch.empty(q.shape[:3], dtype=torch.float32, device=cuda_device)
    rc = lib.swa_prefill_forward_split(
        _native.ptr(q), _native.ptr(k), _native.ptr(v), _native.ptr(fi), _native.ptr(li), nf, nl, nf, nl,
        None, 0, nf, nl, None, None, None, None, 0, _native.ptr(out), _native.ptr(lse), B, S, S, Hq, Hkv, 128, W,
        (128 ** -0.5) * 1.4426950408889634, None, _native.ptr(ws), ws.numel() * 4, tiles, _native.ptr(scratch),
        nbytes, _native.stream_ptr(cuda_device))
    assert rc == 0, lib.swa_last_error_string()
    torch.cuda.synchronize()
    assert ws[1].item() == 0
    slots = nbytes // (256 * 4 * 129)
    written = int((scratch[: slots * 1024].view(torch.float32) != 0).sum())
    assert written > 0
    O0, L0 = _core.forward(q, k, v, fi, li, window_size=W, key_split=None)
    _close_to_unsplit(out, lse, O0, L0, "ABI split")
    O_ref, LSE_ref = oracle_subset(q, k, v, full, local, W)
    compare(out, lse, O_ref, LSE_ref, label="ABI split")
