"""The FP32 attention oracle against torch's own attention.

The reference's kernels only lower for Hopper, so no reference output exists to
pin the attention numerics to.  This checks the oracle's restatement of the
routed masks (full rows: causal; local rows: causal sliding window of W keys,
both per row) and its log2 LSE against scaled_dot_product_attention with the
equivalent per-row boolean mask, on mixed routing, GQA and a non-default scale.
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import attention as oracle_attn


@pytest.mark.parametrize("S,Hq,Hkv,W,p_full,sm_scale", [
    (64, 4, 2, 9, 0.3, None), (97, 8, 2, 32, 0.5, 0.05), (50, 6, 3, 1, 0.5, None), (40, 4, 4, 100, 0.2, None),
])
def test_prefill_dense_matches_sdpa(S, Hq, Hkv, W, p_full, sm_scale):
    g = torch.Generator().manual_seed(S + Hq + W)
    B, D = 2, 128
    q = torch.randn(B, S, Hq, D, generator=g)
    k = torch.randn(B, S, Hkv, D, generator=g)
    v = torch.randn(B, S, Hkv, D, generator=g)
    mask = torch.rand(B, S, generator=g) < p_full
    full = [np.nonzero(mask[b].numpy())[0] for b in range(B)]
    local = [np.nonzero(~mask[b].numpy())[0] for b in range(B)]
    O, L = oracle_attn.prefill_dense(q, k, v, full, local, window=W, sm_scale=sm_scale)

    scale = sm_scale if sm_scale is not None else 1.0 / math.sqrt(D)
    r = Hq // Hkv
    t = torch.arange(S)
    causal = t[None, :] <= t[:, None]
    in_window = t[None, :] > t[:, None] - W
    for b in range(B):
        allowed = causal & (mask[b][:, None] | in_window)  # [S rows, S keys]
        qh = q[b].transpose(0, 1)                               # [Hq, S, D]
        kh = k[b].repeat_interleave(r, 1).transpose(0, 1)
        vh = v[b].repeat_interleave(r, 1).transpose(0, 1)
        want_o = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=allowed, scale=scale).transpose(0, 1)
        s = (qh @ kh.transpose(1, 2)) * scale
        s = s.masked_fill(~allowed, float("-inf"))
        want_lse = (torch.logsumexp(s, dim=-1) / math.log(2.0)).transpose(0, 1)  # log2 units, [S, Hq]
        assert torch.allclose(O[b], want_o, atol=2e-5, rtol=1e-5), (O[b] - want_o).abs().max()
        assert torch.allclose(L[b], want_lse, atol=2e-5, rtol=1e-5), (L[b] - want_lse).abs().max()


def test_every_row_helper_passes_the_oracle_and_catches_a_planted_error():
    # The helper the GPU tests use to check every row, run here on CPU tensors:
    # the oracle's own result passes, one row moved by 0.05 fails, and a row
    # without a legal key (Sq > Skv, local branch) must be NaN / -inf.
    import sys
    import os
    sys.path.insert(0, os.path.dirname(__file__))
    from _parity import compare_every_row_on_device

    g = torch.Generator().manual_seed(5)
    B, Sq, Skv, Hq, Hkv, D, W = 2, 90, 60, 4, 2, 128, 8
    q = torch.randn(B, Sq, Hq, D, generator=g).bfloat16()
    k = torch.randn(B, Skv, Hkv, D, generator=g).bfloat16()
    v = torch.randn(B, Skv, Hkv, D, generator=g).bfloat16()
    mask = torch.rand(B, Sq, generator=g) < 0.4
    full = [np.nonzero(mask[b].numpy())[0] for b in range(B)]
    local = [np.nonzero(~mask[b].numpy())[0] for b in range(B)]
    O, L = oracle_attn.prefill_dense(q, k, v, full, local, window=W)
    assert torch.isneginf(L).any()  # local rows past Skv + W - 1 have no legal key
    o_max, o_mean, l_max, rows = compare_every_row_on_device(O, L, q, k, v, full, local, W, label="self")
    assert rows == B * Sq and o_max == 0.0 and l_max == 0.0
    bad = O.clone()
    bad[1, int(full[1][0])] += 0.05
    with pytest.raises(AssertionError, match="O max-abs"):
        compare_every_row_on_device(bad, L, q, k, v, full, local, W, label="planted")
    fin = torch.isfinite(L)
    empty_row = torch.nonzero(~fin[0, :, 0])[0, 0]
    bad_l = L.clone()
    bad_l[0, empty_row] = 0.0
    with pytest.raises(AssertionError, match="LSE = -inf"):
        compare_every_row_on_device(O, bad_l, q, k, v, full, local, W, label="planted")
