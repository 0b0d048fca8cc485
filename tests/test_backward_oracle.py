"""The backward oracle is pinned to torch's own attention gradients
(scaled_dot_product_attention with the same causal / sliding-window masks)."""
from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import attention as oracle_attn


@pytest.mark.parametrize("window", [1 << 20, 9])
def test_prefill_backward_matches_sdpa(window):
    g = torch.Generator().manual_seed(4)
    B, S, Hq, Hkv = 2, 40, 4, 2
    q = torch.randn(B, S, Hq, 128, generator=g)
    k = torch.randn(B, S, Hkv, 128, generator=g)
    v = torch.randn(B, S, Hkv, 128, generator=g)
    dout = torch.randn(B, S, Hq, 128, generator=g)
    # every row on one branch: full for window = 2^20 (plain causal), local otherwise
    rows = np.arange(S)
    full = [rows if window > S else rows[:0]] * B
    local = [rows[:0] if window > S else rows] * B
    dq, dk, dv = oracle_attn.prefill_backward(q, k, v, dout, full, local, window=window)
    qt = q.clone().requires_grad_(True)
    kt = k.clone().requires_grad_(True)
    vt = v.clone().requires_grad_(True)
    t = torch.arange(S)
    allowed = (t[None, :] <= t[:, None]) & (t[None, :] > t[:, None] - window)
    o = F.scaled_dot_product_attention(qt.transpose(1, 2), kt.repeat_interleave(Hq // Hkv, 2).transpose(1, 2),
                                       vt.repeat_interleave(Hq // Hkv, 2).transpose(1, 2), attn_mask=allowed)
    (o.transpose(1, 2) * dout).sum().backward()
    for got, want in ((dq, qt.grad), (dk, kt.grad), (dv, vt.grad)):
        assert torch.allclose(got, want, atol=2e-4, rtol=1e-4), (got - want).abs().max()
