"""Prefill backward on the GPU against the FP32 autograd oracle (itself pinned
to torch's attention gradients).  Gradients have no natural unit, so the
tolerance is relative to the oracle's magnitude: max-abs error <= 3 % of the
largest oracle gradient and mean-abs error <= 1 % of its mean magnitude (BF16
operands for P and dS and BF16 outputs; a layout or masking error is of the
order of the gradient itself)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _parity import device_lists, lists_from_mask
from oracle import attention as oracle_attn
from oracle import metadata as oracle_md
from switchattentionkernels_b200 import _core
from switchattentionkernels_b200.backward import switch_gqa_prefill_attention, switch_gqa_prefill_backward
from switchattentionkernels_b200.metadata import build_switch_attention_metadata

pytestmark = pytest.mark.gpu

MAX_REL = 0.03
MEAN_REL = 0.01


def _close(got, want, label):
    got = got.float().cpu()
    err = (got - want).abs()
    scale_max = want.abs().max().item()
    scale_mean = want.abs().mean().item()
    assert torch.isfinite(got).all(), f"{label}: non-finite"
    assert err.max().item() <= MAX_REL * scale_max + 1e-4, \
        f"{label}: max-abs {err.max().item():.3e} vs {MAX_REL} x {scale_max:.3e}"
    assert err.mean().item() <= MEAN_REL * scale_mean + 1e-5, \
        f"{label}: mean-abs {err.mean().item():.3e} vs {MEAN_REL} x {scale_mean:.3e}"


def _run(dev, B, S, Hq, Hkv, W, p, seed, sm_scale=None, cu=None):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, S, Hq, 128, generator=g).bfloat16()
    k = torch.randn(B, S, Hkv, 128, generator=g).bfloat16()
    v = torch.randn(B, S, Hkv, 128, generator=g).bfloat16()
    dout = torch.randn(B, S, Hq, 128, generator=g).bfloat16()
    mask = torch.rand(B, S, generator=g) < p
    full, local = lists_from_mask(mask)
    md = md_or = None
    if cu is not None:
        md = build_switch_attention_metadata(S, S, device=dev, window_size=W, cu_seqlens=torch.tensor(cu).int())
        md_or = oracle_md.build_metadata(S, S, W, np.asarray(cu))
    qd, kd, vd, dod = (t.to(dev) for t in (q, k, v, dout))
    if B == 1:
        fi, li = device_lists(full, local, dev, B)
        counts = None
    else:
        fi, li, counts = _core.build_switch_query_indices_batched(mask.to(dev))
    out, lse = _core.forward(qd, kd, vd, fi, li, metadata=md, window_size=W, sm_scale=sm_scale, query_counts=counts)
    dq, dk, dv = switch_gqa_prefill_backward(qd, kd, vd, out, lse, dod, fi, li, metadata=md, window_size=W,
                                             sm_scale=sm_scale, query_counts=counts)
    torch.cuda.synchronize()
    rq, rk, rv = oracle_attn.prefill_backward(q, k, v, dout, full, local, window=W, sm_scale=sm_scale, metadata=md_or)
    label = f"B={B} S={S} Hq={Hq} Hkv={Hkv} W={W} p={p}"
    _close(dq, rq, label + " dq")
    _close(dk, rk, label + " dk")
    _close(dv, rv, label + " dv")


@pytest.mark.parametrize("B,S,Hq,Hkv,W,p", [
    (1, 200, 4, 2, 64, 0.3), (1, 700, 8, 2, 100, 0.5), (2, 513, 4, 1, 37, 0.2), (3, 300, 16, 4, 1000, 0.7),
    (1, 1000, 8, 8, 128, 0.0), (1, 1000, 8, 8, 128, 1.0), (2, 333, 32, 1, 50, 0.4), (1, 260, 6, 3, 1, 0.5),
    (1, 2048, 8, 2, 1024, 0.125),  # config 3's window and routing density, many tiles per CTA
])
def test_backward_matches_oracle(cuda_device, B, S, Hq, Hkv, W, p):
    _run(cuda_device, B, S, Hq, Hkv, W, p, seed=B * 131 + S + Hq + W)


def test_backward_varlen_metadata_and_scale(cuda_device):
    _run(cuda_device, 1, 900, 8, 2, 150, 0.4, seed=7, sm_scale=0.07, cu=[0, 300, 301, 650, 900])


def test_autograd_function(cuda_device):
    dev = cuda_device
    g = torch.Generator().manual_seed(9)
    S, Hq, Hkv, W = 300, 8, 2, 64
    q = torch.randn(1, S, Hq, 128, generator=g).bfloat16().to(dev).requires_grad_(True)
    k = torch.randn(1, S, Hkv, 128, generator=g).bfloat16().to(dev).requires_grad_(True)
    v = torch.randn(1, S, Hkv, 128, generator=g).bfloat16().to(dev).requires_grad_(True)
    mask = torch.rand(1, S, generator=g) < 0.5
    full, local = lists_from_mask(mask)
    fi, li = device_lists(full, local, dev, 1)
    out, lse = switch_gqa_prefill_attention(q, k, v, fi, li, window_size=W)
    dout = torch.randn(out.shape, generator=g).bfloat16().to(dev)
    (out.float() * dout.float()).sum().backward()
    dq, dk, dv = switch_gqa_prefill_backward(q.detach(), k.detach(), v.detach(), out.detach(), lse, dout, fi, li,
                                             window_size=W)
    assert torch.equal(q.grad, dq) and torch.equal(k.grad, dk) and torch.equal(v.grad, dv)


def test_backward_context_parallel_rows(cuda_device):
    # one rank's rows of a zigzag split against the whole K/V axis: Sq != Skv, per-row
    # key bounds from the metadata (the layout context_parallel.py hands the kernels)
    from switchattentionkernels_b200 import context_parallel as cp

    dev = cuda_device
    g = torch.Generator().manual_seed(13)
    S, Hq, Hkv, W = 900, 8, 2, 150
    cu = np.array([0, 300, 301, 650, S])
    q = torch.randn(1, S, Hq, 128, generator=g).bfloat16()
    k = torch.randn(1, S, Hkv, 128, generator=g).bfloat16()
    v = torch.randn(1, S, Hkv, 128, generator=g).bfloat16()
    dout = torch.randn(1, S, Hq, 128, generator=g).bfloat16()
    mask = (torch.rand(S, generator=g) < 0.4).numpy()
    rows = cp.make_cp_plan(S, 2, cp.cp_row_costs(mask, W, cu)).rows(1)
    idx = torch.from_numpy(rows)
    md = cp.cp_metadata(S, rows, device=dev, window_size=W, cu_seqlens=torch.from_numpy(cu).int())
    lmask = mask[rows]
    full, local = np.nonzero(lmask)[0].astype(np.int32), np.nonzero(~lmask)[0].astype(np.int32)
    fi = torch.from_numpy(full)[None].to(dev)
    li = torch.from_numpy(local)[None].to(dev)
    ql, dol = q[:, idx].contiguous(), dout[:, idx].contiguous()
    qd, kd, vd, dod = (t.to(dev) for t in (ql, k, v, dol))
    out, lse = _core.forward(qd, kd, vd, fi, li, metadata=md, window_size=W)
    dq, dk, dv = switch_gqa_prefill_backward(qd, kd, vd, out, lse, dod, fi, li, metadata=md, window_size=W)
    torch.cuda.synchronize()
    full_md = oracle_md.build_metadata(S, S, W, cu)
    md_rows = {key: (val[rows] if key in ("q_positions", "q_segment_ids", "full_starts", "local_starts",
                                           "causal_ends") else val) for key, val in full_md.items()}
    rq, rk, rv = oracle_attn.prefill_backward(ql, k, v, dol, [full], [local], window=W, metadata=md_rows)
    _close(dq, rq, "context-parallel rows dq")
    _close(dk, rk, "context-parallel rows dk")
    _close(dv, rv, "context-parallel rows dv")


def test_backward_rows_without_keys(cuda_device):
    # metadata rows with start == end (a sequence's first row) and start > end (its
    # last row): the forward gives O = NaN and LSE = -inf there, and those rows
    # carry no gradient; every gradient must stay finite
    dev = cuda_device
    g = torch.Generator().manual_seed(21)
    cu = np.array([0, 200, 201, 520, 700])
    S, Hq, Hkv, W = int(cu[-1]), 8, 2, 96
    md_or = oracle_md.build_metadata(S, S, W, cu)
    fs, ls, ce = (md_or[n].copy() for n in ("full_starts", "local_starts", "causal_ends"))
    for s in cu[1:-1]:
        ce[s] = s
    for e in cu[2:]:
        if e - 1 not in cu:
            fs[e - 1] = ls[e - 1] = e
            ce[e - 1] = e - 1
    md_or = dict(md_or, full_starts=fs, local_starts=ls, causal_ends=ce)
    md = _core.SwitchAttentionMetadata(**{n: torch.from_numpy(a).to(dev) for n, a in md_or.items()})
    q = torch.randn(1, S, Hq, 128, generator=g).bfloat16()
    k = torch.randn(1, S, Hkv, 128, generator=g).bfloat16()
    v = torch.randn(1, S, Hkv, 128, generator=g).bfloat16()
    dout = torch.randn(1, S, Hq, 128, generator=g).bfloat16()
    mask = torch.rand(1, S, generator=g) < 0.4
    full, local = lists_from_mask(mask)
    fi, li = device_lists(full, local, dev, 1)
    qd, kd, vd, dod = (t.to(dev) for t in (q, k, v, dout))
    out, lse = _core.forward(qd, kd, vd, fi, li, metadata=md, window_size=W)
    assert torch.isneginf(lse).any()
    dq, dk, dv = switch_gqa_prefill_backward(qd, kd, vd, out, lse, dod, fi, li, metadata=md, window_size=W)
    torch.cuda.synchronize()
    rq, rk, rv = oracle_attn.prefill_backward(q, k, v, dout, full, local, window=W, metadata=md_or)
    _close(dq, rq, "rows without keys dq")
    _close(dk, rk, "rows without keys dk")
    _close(dv, rv, "rows without keys dv")
