"""The decode-step oracle is the prefill oracle's row at each sequence's last
position (t = L - 1), for both branches."""
from __future__ import annotations

import numpy as np
import torch

from oracle import attention as oracle_attn


def test_decode_rows_equal_prefill_rows_at_the_last_position():
    g = torch.Generator().manual_seed(2)
    B, Smax, Hq, Hkv, W = 4, 300, 8, 2, 37
    k = torch.randn(B, Smax, Hkv, 128, generator=g).bfloat16()
    v = torch.randn(B, Smax, Hkv, 128, generator=g).bfloat16()
    qfull = torch.randn(B, Smax, Hq, 128, generator=g).bfloat16()
    seq_lens = np.array([1, 37, 38, 300])
    route = np.array([True, False, True, False])
    q = torch.stack([qfull[b, seq_lens[b] - 1] for b in range(B)])
    O, L = oracle_attn.decode_rows(q, k, v, seq_lens, route, window=W)
    for b in range(B):
        t = int(seq_lens[b]) - 1
        o, lse = oracle_attn.prefill_rows(qfull, k, v, b, [t], not route[b], window=W)
        assert torch.allclose(O[b], o[0], atol=1e-5, rtol=0)
        assert torch.allclose(L[b], lse[0], atol=1e-5, rtol=0)
