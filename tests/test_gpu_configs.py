"""Parity at the BASELINE workload sizes (configs 3, 4, 5) on the GPU.

The CUDA path runs on the whole workload; the FP32 CPU oracle checks a seeded
sample of positions per sequence (all heads of each sampled position, in either
branch), which includes the first and last positions, the first positions of
varlen sequences and positions next to routing switches.  Size-independent
properties are checked on every row: every routed row has at least one legal key
in these workloads, so every output row and LSE must be finite.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _parity import compare, device_lists, lists_from_mask, oracle_subset, sample_positions
from oracle import metadata as oracle_meta
from switchattentionkernels_b200 import swiattn_gqa_prefill as fixed
from switchattentionkernels_b200 import swiattn_gqa_prefill_varlen as varlen
from switchattentionkernels_b200 import workloads

pytestmark = pytest.mark.gpu


def _switch_positions(mask_row: np.ndarray, limit: int = 8):
    """A few positions where the routing changes branch (both sides of the switch)."""
    sw = np.nonzero(mask_row[1:] != mask_row[:-1])[0]
    picks = sw[:: max(1, sw.size // limit)][:limit] if sw.size else sw
    return [int(p) for p in picks] + [int(p) + 1 for p in picks]


def _check_all_rows_finite(O, LSE, label):
    assert torch.isfinite(LSE).all().item(), f"{label}: non-finite LSE"
    assert torch.isfinite(O.float()).all().item(), f"{label}: non-finite output"


def _sampled_parity(w, O, LSE, n_per_batch, seed, label, metadata=None, extra=()):
    q, k, v, mask, W = w["q"], w["k"], w["v"], w["mask"], w["window"]
    B, S = mask.shape
    full, local = lists_from_mask(mask)
    m = mask.numpy()
    subset = [sample_positions(S, n_per_batch, seed + b, must=[0, S - 1, *extra, *_switch_positions(m[b])])
              for b in range(B)]
    O_ref, LSE_ref = oracle_subset(q, k, v, full, local, W, subset=subset, metadata=metadata)
    sel = torch.zeros(LSE_ref.shape, dtype=torch.bool)
    for b in range(B):
        sel[b, torch.from_numpy(subset[b])] = True
    return compare(O, LSE, O_ref, LSE_ref, rows=sel, label=label)


def test_config3_sampled_parity(cuda_device):
    w = workloads.make_inputs(3, device=cuda_device, on_device=True)
    B = w["q"].shape[0]
    full, local = lists_from_mask(w["mask"])
    fi, li = device_lists(full, local, cuda_device, B)
    O, LSE = fixed.switch_gqa_prefill_forward(w["q"], w["k"], w["v"], fi, li, window_size=w["window"])
    torch.cuda.synchronize()
    _check_all_rows_finite(O, LSE, "config3")
    O, LSE = O.cpu(), LSE.cpu()
    w_cpu = dict(w, q=w["q"].cpu(), k=w["k"].cpu(), v=w["v"].cpu())
    _sampled_parity(w_cpu, O, LSE, 24, 300, "config3")


def test_config4_varlen_sampled_parity(cuda_device):
    w = workloads.make_inputs(4, device=cuda_device)
    cu = w["cu_seqlens"].numpy()
    S = int(cu[-1])
    W = w["window"]
    meta = varlen.build_switch_attention_metadata(S, S, device=cuda_device, window_size=W,
                                                  cu_seqlens=w["cu_seqlens"])
    full, local = lists_from_mask(w["mask"])
    fi, li = device_lists(full, local, cuda_device, 1)
    O, LSE = varlen.switch_gqa_prefill_forward(w["q"], w["k"], w["v"], fi, li, metadata=meta, window_size=W)
    torch.cuda.synchronize()
    _check_all_rows_finite(O, LSE, "config4")
    ref_meta = oracle_meta.build_metadata(S, S, W, cu)
    starts = [int(x) for x in cu[:-1]]
    ends = [int(x) - 1 for x in cu[1:]]
    w_cpu = dict(w, q=w["q"].cpu(), k=w["k"].cpu(), v=w["v"].cpu())
    _sampled_parity(w_cpu, O.cpu(), LSE.cpu(), 32, 400, "config4", metadata=ref_meta,
                    extra=starts[:8] + ends[:8])


@pytest.mark.parametrize("p_full", [0.0, 0.01, 1.0])
def test_config5_long_context_sampled_parity(cuda_device, p_full):
    w = workloads.make_inputs(5, device=cuda_device, p_full=p_full, on_device=True)
    B = w["q"].shape[0]
    full, local = lists_from_mask(w["mask"])
    fi, li = device_lists(full, local, cuda_device, B)
    O, LSE = fixed.switch_gqa_prefill_forward(w["q"], w["k"], w["v"], fi, li, window_size=w["window"])
    torch.cuda.synchronize()
    _check_all_rows_finite(O, LSE, f"config5 p_full={p_full}")
    w_cpu = dict(w, q=w["q"].cpu(), k=w["k"].cpu(), v=w["v"].cpu())
    _sampled_parity(w_cpu, O.cpu(), LSE.cpu(), 8, 500, f"config5 p_full={p_full}")
