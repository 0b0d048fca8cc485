"""The oracle's routing decision from router outputs, pinned to the plain torch
expressions a router would use (the router is outside the reference, which
fixes only the convention True = full attention, README.md:85)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import indices as oracle_idx


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("threshold", [0.0, 0.25, -1.5])
def test_router_mask_matches_torch(dtype, threshold):
    g = torch.Generator().manual_seed(3)
    scores = torch.randn(3, 777, generator=g).to(dtype)
    logits = torch.randn(3, 777, 2, generator=g).to(dtype)
    scores[0, :5] = float("nan")
    logits[1, :7, 0] = logits[1, :7, 1]           # ties route to local
    logits[2, :3, 1] = float("nan")
    want_s = scores.float() > threshold
    want_p = (logits[..., 1].float() - logits[..., 0].float()) > threshold
    got_s = oracle_idx.router_mask(scores.float().numpy(), pair=False, threshold=threshold)
    got_p = oracle_idx.router_mask(logits.float().numpy(), pair=True, threshold=threshold)
    assert np.array_equal(got_s, want_s.numpy())
    assert np.array_equal(got_p, want_p.numpy())
    assert not got_s[0, :5].any() and not got_p[2, :3].any()   # NaN routes to local
    if threshold >= 0:
        assert not got_p[1, :7].any()                           # ties route to local
