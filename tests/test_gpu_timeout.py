"""Failure detection on the GPU without a fault: a bounded device wait runs out.

The library's test hook makes the first CTA withhold one K/V tile load (the flag
its MMA issuer waits on is never set).  The kernel's bounded wait gives up after
about a second, every role leaves its loop, tensor memory is released and the
launch reports SWA_STATUS_TIMEOUT, which the Python layer raises.  A normal
launch on the same CUDA context afterwards must still give correct results.
"""
from __future__ import annotations

import pytest
import torch

from _parity import compare, device_lists, lists_from_mask, oracle_subset
from switchattentionkernels_b200 import _core, _native

pytestmark = pytest.mark.gpu


def test_wait_that_runs_out_reports_timeout_and_context_stays_usable(cuda_device):
    lib = _native.load()
    g = torch.Generator().manual_seed(91)
    q = torch.randn(1, 600, 8, 128, generator=g).bfloat16().to(cuda_device)
    k = torch.randn(1, 600, 2, 128, generator=g).bfloat16().to(cuda_device)
    v = torch.randn(1, 600, 2, 128, generator=g).bfloat16().to(cuda_device)
    mask = torch.rand(1, 600, generator=g) < 0.4
    full, local = lists_from_mask(mask)
    fi, li = device_lists(full, local, cuda_device, 1)
    lib.swa_test_withhold_kv_load(1)
    try:
        with pytest.raises(RuntimeError, match="timed out"):
            _core.forward(q, k, v, fi, li, window_size=100)
    finally:
        lib.swa_test_withhold_kv_load(0)
    torch.cuda.synchronize()
    out, lse = _core.forward(q, k, v, fi, li, window_size=100)
    torch.cuda.synchronize()
    O_ref, L_ref = oracle_subset(q, k, v, full, local, 100)
    compare(out, lse, O_ref, L_ref, label="after timeout")
