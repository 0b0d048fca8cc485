"""Parity at the BASELINE workload sizes (configs 3, 4, 5) on the GPU.

The CUDA path runs on the whole workload.  Two checks follow:

* every routed row (all heads) against the FP32 restatement of the oracle
  evaluated on the same GPU (``compare_every_row_on_device``), with the stated
  tolerances; rows without a legal key (none in these workloads) would have to be
  O = NaN, LSE = -inf;
* a seeded sample of positions per sequence against the oracle evaluated on the
  CPU (the first and last positions, the first positions of varlen sequences and
  positions next to routing switches), and on those rows the GPU evaluation of
  the oracle against the CPU one (FP32 vs FP32, 1e-4), which ties the every-row
  check to the CPU restatement.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _parity import compare, compare_every_row_on_device, device_lists, lists_from_mask, oracle_subset, sample_positions
from oracle import attention as oracle_attn
from oracle import metadata as oracle_meta
from switchattentionkernels_b200 import swiattn_gqa_prefill as fixed
from switchattentionkernels_b200 import swiattn_gqa_prefill_varlen as varlen
from switchattentionkernels_b200 import workloads

pytestmark = pytest.mark.gpu

ORACLE_DEVICE_VS_CPU = 1e-4


def _switch_positions(mask_row: np.ndarray, limit: int = 8):
    """A few positions where the routing changes branch (both sides of the switch)."""
    sw = np.nonzero(mask_row[1:] != mask_row[:-1])[0]
    picks = sw[:: max(1, sw.size // limit)][:limit] if sw.size else sw
    return [int(p) for p in picks] + [int(p) + 1 for p in picks]


def _check_all_rows_finite(O, LSE, label):
    assert torch.isfinite(LSE).all().item(), f"{label}: non-finite LSE"
    assert torch.isfinite(O.float()).all().item(), f"{label}: non-finite output"


def _sampled_parity(w_dev, O, LSE, n_per_batch, seed, label, metadata=None, extra=()):
    """CPU-oracle parity on a sample of positions, and the device oracle against the CPU one there."""
    q, k, v = w_dev["q"].cpu(), w_dev["k"].cpu(), w_dev["v"].cpu()
    mask, W = w_dev["mask"], w_dev["window"]
    B, S = mask.shape
    full, local = lists_from_mask(mask)
    m = mask.cpu().numpy()
    subset = [sample_positions(S, n_per_batch, seed + b, must=[0, S - 1, *extra, *_switch_positions(m[b])])
              for b in range(B)]
    O_ref, LSE_ref = oracle_subset(q, k, v, full, local, W, subset=subset, metadata=metadata)
    sel = torch.zeros(LSE_ref.shape, dtype=torch.bool)
    for b in range(B):
        sel[b, torch.from_numpy(subset[b])] = True
    compare(O, LSE, O_ref, LSE_ref, rows=sel, label=label)
    for b in range(B):
        for is_local, lst in ((False, full[b]), (True, local[b])):
            pos = lst[np.isin(lst, subset[b])]
            if pos.size == 0:
                continue
            o_d, l_d = oracle_attn.prefill_rows(w_dev["q"], w_dev["k"], w_dev["v"], b, pos, is_local, window=W,
                                                metadata=metadata)
            pt = torch.from_numpy(pos)
            assert (o_d.cpu() - O_ref[b, pt]).abs().max().item() <= ORACLE_DEVICE_VS_CPU, f"{label}: device oracle O"
            assert (l_d.cpu() - LSE_ref[b, pt]).abs().max().item() <= ORACLE_DEVICE_VS_CPU, f"{label}: device oracle LSE"


def test_config3_parity(cuda_device):
    w = workloads.make_inputs(3, device=cuda_device, on_device=True)
    B = w["q"].shape[0]
    full, local = lists_from_mask(w["mask"])
    fi, li = device_lists(full, local, cuda_device, B)
    O, LSE = fixed.switch_gqa_prefill_forward(w["q"], w["k"], w["v"], fi, li, window_size=w["window"])
    torch.cuda.synchronize()
    _check_all_rows_finite(O, LSE, "config3")
    compare_every_row_on_device(O, LSE, w["q"], w["k"], w["v"], full, local, w["window"], label="config3 every row")
    _sampled_parity(w, O.cpu(), LSE.cpu(), 24, 300, "config3")


def test_config4_varlen_parity(cuda_device):
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
    compare_every_row_on_device(O, LSE, w["q"], w["k"], w["v"], full, local, W, metadata=ref_meta,
                                label="config4 every row")
    starts = [int(x) for x in cu[:-1]]
    ends = [int(x) - 1 for x in cu[1:]]
    _sampled_parity(w, O.cpu(), LSE.cpu(), 32, 400, "config4", metadata=ref_meta, extra=starts[:8] + ends[:8])


@pytest.mark.parametrize("p_full", [0.0, 0.01, 1.0])
def test_config5_long_context_parity(cuda_device, p_full):
    w = workloads.make_inputs(5, device=cuda_device, p_full=p_full, on_device=True)
    B = w["q"].shape[0]
    full, local = lists_from_mask(w["mask"])
    fi, li = device_lists(full, local, cuda_device, B)
    O, LSE = fixed.switch_gqa_prefill_forward(w["q"], w["k"], w["v"], fi, li, window_size=w["window"])
    torch.cuda.synchronize()
    _check_all_rows_finite(O, LSE, f"config5 p_full={p_full}")
    compare_every_row_on_device(O, LSE, w["q"], w["k"], w["v"], full, local, w["window"],
                                label=f"config5 p_full={p_full} every row")
    _sampled_parity(w, O.cpu(), LSE.cpu(), 8, 500, f"config5 p_full={p_full}")
