"""Decode step on the GPU against the FP32 oracle (and the prefill kernel's row
at the same position), with the tolerances of the prefill path."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _parity import O_MAX_ABS, O_MEAN_ABS, LSE_MAX_ABS
from oracle import attention as oracle_attn
from switchattentionkernels_b200 import _core
from switchattentionkernels_b200.decode import switch_gqa_decode_forward

pytestmark = pytest.mark.gpu


def _case(dev, B, Smax, Hq, Hkv, seed, lens=None, p_full=0.5):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, 128, generator=g).bfloat16()
    k = torch.randn(B, Smax, Hkv, 128, generator=g).bfloat16()
    v = torch.randn(B, Smax, Hkv, 128, generator=g).bfloat16()
    if lens is None:
        lens = torch.randint(1, Smax + 1, (B,), generator=g)
        lens[0] = Smax
        if B > 1:
            lens[1] = 1
    lens = torch.as_tensor(lens, dtype=torch.int32)
    route = torch.rand(B, generator=g) < p_full
    return q, k, v, lens, route


def _check(O, L, Oref, Lref, label):
    O = O.float().cpu()
    L = L.cpu()
    err = (O - Oref).abs()
    assert torch.isfinite(O).all(), label
    assert err.max().item() <= O_MAX_ABS, f"{label}: O max-abs {err.max().item():.3e}"
    assert err.mean().item() <= O_MEAN_ABS, f"{label}: O mean-abs {err.mean().item():.3e}"
    lerr = (L - Lref).abs().max().item()
    assert lerr <= LSE_MAX_ABS, f"{label}: LSE max-abs {lerr:.3e}"


@pytest.mark.parametrize("B,Smax,Hq,Hkv,W", [
    (1, 1, 8, 2, 16), (3, 100, 8, 2, 1), (5, 1000, 32, 8, 200), (4, 5000, 64, 8, 4096), (2, 3000, 32, 1, 512),
    (7, 777, 6, 3, 64), (3, 2049, 40, 8, 1000), (33, 700, 32, 8, 128), (2, 20000, 32, 4, 2048),
])
def test_decode_matches_oracle(cuda_device, B, Smax, Hq, Hkv, W):
    q, k, v, lens, route = _case(cuda_device, B, Smax, Hq, Hkv, seed=B * 7919 + Smax + W)
    O, L = switch_gqa_decode_forward(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device),
                                     lens.to(cuda_device), route.to(cuda_device), window_size=W)
    torch.cuda.synchronize()
    Oref, Lref = oracle_attn.decode_rows(q, k, v, lens.numpy(), route.numpy(), window=W)
    _check(O, L, Oref, Lref, f"B={B} Smax={Smax} Hq={Hq} Hkv={Hkv} W={W}")


@pytest.mark.parametrize("p_full", [0.0, 1.0])
def test_decode_all_one_branch_and_sm_scale(cuda_device, p_full):
    q, k, v, lens, route = _case(cuda_device, 6, 2500, 16, 4, seed=3, p_full=p_full)
    O, L = switch_gqa_decode_forward(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device),
                                     lens.to(cuda_device), route.to(cuda_device), window_size=300, sm_scale=0.05)
    Oref, Lref = oracle_attn.decode_rows(q, k, v, lens.numpy(), route.numpy(), window=300, sm_scale=0.05)
    _check(O, L, Oref, Lref, f"p_full={p_full}")


def test_decode_equals_the_prefill_row_at_the_last_position(cuda_device):
    dev = cuda_device
    B, S, Hq, Hkv, W = 3, 1500, 16, 4, 300
    g = torch.Generator().manual_seed(17)
    qf = torch.randn(B, S, Hq, 128, generator=g).bfloat16().to(dev)
    k = torch.randn(B, S, Hkv, 128, generator=g).bfloat16().to(dev)
    v = torch.randn(B, S, Hkv, 128, generator=g).bfloat16().to(dev)
    route = torch.tensor([True, False, True])
    # the prefill path with every position routed like the last one
    mask = route[:, None].expand(B, S).to(dev).contiguous()
    full, local, counts = _core.build_switch_query_indices_batched(mask)
    Op, Lp = _core.forward(qf, k, v, full, local, window_size=W, query_counts=counts)
    lens = torch.full((B,), S, dtype=torch.int32, device=dev)
    O, L = switch_gqa_decode_forward(qf[:, -1].contiguous(), k, v, lens, route.to(dev), window_size=W)
    torch.cuda.synchronize()
    _check(O, L, Op[:, -1].float().cpu(), Lp[:, -1].cpu(), "decode vs prefill row")


@pytest.mark.parametrize("W", [64, 5000])
def test_decode_sequence_without_keys(cuda_device, W):
    # a sequence with no cached key (L = 0) has a row sum of 0: O = NaN and LSE = -inf,
    # as the prefill writes a row whose key range is empty; the other sequences are
    # unaffected (one of them spans many splits, merged by the last CTA to finish)
    dev = cuda_device
    q, k, v, _, route = _case(dev, 3, 6000, 32, 4, seed=91 + W)
    lens = torch.tensor([0, 6000, 37], dtype=torch.int32)
    route[:] = torch.tensor([True, True, False])
    O, L = switch_gqa_decode_forward(q.to(dev), k.to(dev), v.to(dev), lens.to(dev), route.to(dev), window_size=W)
    torch.cuda.synchronize()
    O = O.float().cpu()
    L = L.cpu()
    assert torch.isnan(O[0]).all() and torch.isneginf(L[0]).all()
    Oref, Lref = oracle_attn.decode_rows(q[1:], k[1:], v[1:], lens[1:].numpy(), route[1:].numpy(), window=W)
    _check(O[1:], L[1:], Oref, Lref, f"L = 0 beside others, W={W}")


def test_decode_arguments(cuda_device):
    dev = cuda_device
    q = torch.zeros(2, 8, 128, dtype=torch.bfloat16, device=dev)
    k = torch.zeros(2, 10, 2, 128, dtype=torch.bfloat16, device=dev)
    lens = torch.ones(2, dtype=torch.int32, device=dev)
    route = torch.ones(2, dtype=torch.bool, device=dev)
    with pytest.raises(ValueError):
        switch_gqa_decode_forward(q, k, k, lens, route, window_size=0)
    with pytest.raises(ValueError):
        switch_gqa_decode_forward(q, k, k, lens.long(), route)
    with pytest.raises(TypeError):
        switch_gqa_decode_forward(q.float(), k, k, lens, route)
    O, L = switch_gqa_decode_forward(q.unsqueeze(1), k, k, lens, route)
    assert O.shape == (2, 1, 8, 128) and L.shape == (2, 1, 8)


def _fp8_cache(k, v, seed):
    """FP8 e4m3 caches with per-(b, KV head) scales (amax / 448, as a quantiser would
    choose them) and the dequantised FP32 values the oracle sees."""
    g = torch.Generator().manual_seed(seed)
    B, _, Hkv, _ = k.shape
    ks = (k.float().abs().amax(dim=(1, 3)) / 448.0) * (0.5 + torch.rand(B, Hkv, generator=g))
    vs = (v.float().abs().amax(dim=(1, 3)) / 448.0) * (0.5 + torch.rand(B, Hkv, generator=g))
    k8 = (k.float() / ks[:, None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    v8 = (v.float() / vs[:, None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    kd = k8.float() * ks[:, None, :, None]
    vd = v8.float() * vs[:, None, :, None]
    return k8, v8, ks, vs, kd, vd


@pytest.mark.parametrize("B,Smax,Hq,Hkv,W", [
    (1, 1, 8, 2, 16), (3, 100, 8, 2, 1), (5, 1000, 32, 8, 200), (2, 3000, 32, 1, 512), (7, 777, 6, 3, 64),
    (33, 700, 32, 8, 128), (2, 20000, 32, 4, 2048),
])
def test_decode_fp8_cache_matches_oracle(cuda_device, B, Smax, Hq, Hkv, W):
    # FP8 e4m3 K/V with per-(b, KV head) scales: the oracle attends over the
    # dequantised cache; the kernel's FP16 products keep the prefill tolerances
    q, k, v, lens, route = _case(cuda_device, B, Smax, Hq, Hkv, seed=B * 31 + Smax + W)
    k8, v8, ks, vs, kd, vd = _fp8_cache(k, v, seed=B + W)
    O, L = switch_gqa_decode_forward(q.to(cuda_device), k8.to(cuda_device), v8.to(cuda_device),
                                     lens.to(cuda_device), route.to(cuda_device), window_size=W,
                                     k_scale=ks.to(cuda_device), v_scale=vs.to(cuda_device))
    torch.cuda.synchronize()
    Oref, Lref = oracle_attn.decode_rows(q, kd, vd, lens.numpy(), route.numpy(), window=W)
    _check(O, L, Oref, Lref, f"fp8 B={B} Smax={Smax} Hq={Hq} Hkv={Hkv} W={W}")


def test_decode_fp8_scale_forms_and_bf16_agreement(cuda_device):
    # one number, [Hkv] and [B, Hkv] scales give the same result; with power-of-two
    # scales the dequantised cache is exact in BF16, and the BF16 step on it agrees
    q, k, v, lens, route = _case(cuda_device, 4, 1500, 16, 4, seed=12)
    k8 = (k.float() * 4).clamp(-448, 448).to(torch.float8_e4m3fn)
    v8 = (v.float() * 4).clamp(-448, 448).to(torch.float8_e4m3fn)
    dev = cuda_device
    args = (q.to(dev), k8.to(dev), v8.to(dev), lens.to(dev), route.to(dev))
    outs = [switch_gqa_decode_forward(*args, window_size=200, k_scale=s, v_scale=s)
            for s in (0.25, torch.full((4,), 0.25), torch.full((4, 4), 0.25))]
    torch.cuda.synchronize()
    for O, L in outs[1:]:
        assert torch.equal(O, outs[0][0]) and torch.equal(L, outs[0][1])
    kb = (k8.float() * 0.25).bfloat16().to(dev)
    vb = (v8.float() * 0.25).bfloat16().to(dev)
    Ob, Lb = switch_gqa_decode_forward(q.to(dev), kb, vb, lens.to(dev), route.to(dev), window_size=200)
    torch.cuda.synchronize()
    _check(outs[0][0], outs[0][1], Ob.float().cpu(), Lb.cpu(), "fp8 vs bf16 on the same values")
    with pytest.raises(ValueError):
        switch_gqa_decode_forward(*args, window_size=200)  # scales are required
