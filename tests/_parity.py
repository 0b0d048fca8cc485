"""Shared helpers of the parity tests: run the CUDA path, run the CPU oracle on
the same inputs, compare with the stated tolerances."""
from __future__ import annotations

import numpy as np
import torch

from oracle import attention as oracle_attn
from oracle import indices as oracle_idx

# Tolerances against the FP32 oracle (BF16 output, P rounded to BF16 before P V).
O_MAX_ABS = 2e-2
O_MEAN_ABS = 2e-3
LSE_MAX_ABS = 1e-3


def lists_from_mask(mask: torch.Tensor):
    m = mask.cpu().numpy().astype(bool)
    full, local = [], []
    for b in range(m.shape[0]):
        f, l = oracle_idx.compact_mask(m[b])
        full.append(f)
        local.append(l)
    return full, local


def device_lists(full, local, device, B):
    """Index tensors in the forward's input format (1-D for B=1, -1 padded [B, N] otherwise)."""
    if B == 1:
        return (torch.from_numpy(full[0]).to(device), torch.from_numpy(local[0]).to(device))
    nf = max(1, max(len(x) for x in full))
    nl = max(1, max(len(x) for x in local))
    F = torch.full((B, nf), -1, dtype=torch.int32)
    L = torch.full((B, nl), -1, dtype=torch.int32)
    for b in range(B):
        F[b, :len(full[b])] = torch.from_numpy(full[b])
        L[b, :len(local[b])] = torch.from_numpy(local[b])
    return F.to(device), L.to(device)


def compare(O, LSE, O_ref, LSE_ref, rows=None, label=""):
    """Compare with the oracle: within tolerance where it is defined (finite LSE),
    and exactly ``O = NaN``, ``LSE = -inf`` on the rows where it has no legal key
    (the reference's ``0/0`` and ``log2(0)``, ``swiattn_gqa_prefill.py:201-206``).

    ``rows`` (bool, the shape of ``LSE``) restricts the comparison to a subset.
    """
    O = O.float().cpu()
    LSE = LSE.float().cpu()
    O_ref = O_ref.float()
    LSE_ref = LSE_ref.float()
    scope = torch.ones_like(LSE_ref, dtype=torch.bool) if rows is None else rows
    empty = scope & torch.isneginf(LSE_ref)
    if empty.any():
        assert torch.isneginf(LSE[empty]).all(), f"{label}: rows without a legal key must have LSE = -inf"
        assert torch.isnan(O[empty]).all(), f"{label}: rows without a legal key must have O = NaN"
    sel = scope & torch.isfinite(LSE_ref)
    assert sel.any(), f"{label}: nothing to compare"
    o_err = (O[sel] - O_ref[sel]).abs()
    l_err = (LSE[sel] - LSE_ref[sel]).abs()
    o_max, o_mean, l_max = o_err.max().item(), o_err.mean().item(), l_err.max().item()
    assert torch.isfinite(O[sel]).all(), f"{label}: non-finite output rows"
    assert o_max <= O_MAX_ABS, f"{label}: O max-abs {o_max:.3e} > {O_MAX_ABS}"
    assert o_mean <= O_MEAN_ABS, f"{label}: O mean-abs {o_mean:.3e} > {O_MEAN_ABS}"
    assert l_max <= LSE_MAX_ABS, f"{label}: LSE max-abs {l_max:.3e} > {LSE_MAX_ABS}"
    return o_max, o_mean, l_max


def compare_every_row_on_device(O, LSE, q, k, v, full, local, window, metadata=None, label="",
                                rows_per_slice: int = 8192):
    """Every routed row of a full-size result against the FP32 restatement evaluated
    on the result's own GPU (``oracle.attention.prefill_rows`` on device tensors),
    slice by slice, with the tolerances of ``compare``; rows without a legal key
    must be exactly ``O = NaN``, ``LSE = -inf``.  Returns ``(o_max, o_mean, l_max, rows)``.
    """
    assert not torch.backends.cuda.matmul.allow_tf32, "the device oracle needs IEEE FP32 GEMMs"
    dev = q.device
    o_max = l_max = 0.0
    o_sum = 0.0
    o_cnt = 0
    rows = 0
    for b in range(len(full)):
        for is_local, lst in ((False, full[b]), (True, local[b])):
            pos_all = np.asarray(lst, dtype=np.int64)
            for s0 in range(0, pos_all.size, rows_per_slice):
                pos = pos_all[s0:s0 + rows_per_slice]
                o_ref, l_ref = oracle_attn.prefill_rows(q, k, v, b, pos, is_local, window=window, metadata=metadata,
                                                        budget_bytes=1 << 30)
                pt = torch.from_numpy(pos).to(dev)
                o = O[b, pt].float()
                lse = LSE[b, pt].float()
                empty = torch.isneginf(l_ref)
                if empty.any():
                    assert torch.isneginf(lse[empty]).all().item(), f"{label}: rows without a legal key need LSE = -inf"
                    assert torch.isnan(o[empty]).all().item(), f"{label}: rows without a legal key need O = NaN"
                fin = ~empty
                err = (o - o_ref).abs()[fin]
                assert torch.isfinite(err).all().item(), f"{label}: non-finite output rows (batch {b})"
                o_max = max(o_max, err.max().item()) if err.numel() else o_max
                if not fin.any():
                    rows += pos.size
                    continue
                o_sum += err.double().sum().item()
                o_cnt += err.numel()
                l_max = max(l_max, (lse - l_ref).abs()[fin].max().item())
                rows += pos.size
    assert o_cnt > 0, f"{label}: nothing to compare"
    o_mean = o_sum / o_cnt
    assert o_max <= O_MAX_ABS, f"{label}: O max-abs {o_max:.3e} > {O_MAX_ABS}"
    assert o_mean <= O_MEAN_ABS, f"{label}: O mean-abs {o_mean:.3e} > {O_MEAN_ABS}"
    assert l_max <= LSE_MAX_ABS, f"{label}: LSE max-abs {l_max:.3e} > {LSE_MAX_ABS}"
    return o_max, o_mean, l_max, rows


def oracle_subset(q, k, v, full, local, window, subset=None, metadata=None, sm_scale=None):
    return oracle_attn.prefill_dense(q.cpu(), k.cpu(), v.cpu(), full, local, window=window, subset=subset,
                                     metadata=metadata, sm_scale=sm_scale)


def sample_positions(S: int, n: int, seed: int, must=()):
    rng = np.random.default_rng(seed)
    pick = set(rng.choice(S, size=min(n, S), replace=False).tolist())
    pick.update(p for p in must if 0 <= p < S)
    return np.array(sorted(pick), dtype=np.int64)
