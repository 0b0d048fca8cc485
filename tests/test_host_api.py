"""Host-side behaviour of the product API (CPU only): error types and messages
against the reference fixtures, capacity buckets, workload generators, and the
C-ABI library's exported symbols."""
from __future__ import annotations

import ctypes
import json
import os
import re

import numpy as np
import pytest
import torch
from torch.overrides import TorchFunctionMode

from oracle import attention as oracle_attn
from oracle import indices as oracle_idx
from switchattentionkernels_b200 import _core, _native, workloads
from switchattentionkernels_b200 import swiattn_gqa_prefill_varlen as varlen

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")


class HostAsCuda(torch.Tensor):
    """CPU tensor that reports a CUDA device, to reach the host-side checks without a GPU."""

    @property
    def is_cuda(self):
        return True

    @property
    def device(self):
        return torch.device("cuda", 0)


class CpuFactories(TorchFunctionMode):
    def __torch_function__(self, func, types_, args=(), kwargs=None):
        kwargs = dict(kwargs or {})
        if "device" in kwargs:
            kwargs["device"] = "cpu"
        return func(*args, **kwargs)


def dev(t):
    return t.as_subclass(HostAsCuda)


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(GOLDEN, "reference_host.json")) as fh:
        return json.load(fh)


def _err(fn):
    try:
        fn()
    except Exception as e:  # noqa: BLE001
        return {"type": type(e).__name__, "message": str(e)}
    return None


def test_validate_qkv_messages_match_reference(golden):
    def qkv(qs, ks, vs, qd=torch.bfloat16):
        return (dev(torch.zeros(qs, dtype=qd)), dev(torch.zeros(ks, dtype=torch.bfloat16)),
                dev(torch.zeros(vs, dtype=torch.bfloat16)))
    cases = {
        "ok": qkv((1, 8, 32, 128), (1, 8, 8, 128), (1, 8, 8, 128)),
        "fp16_q": qkv((1, 8, 32, 128), (1, 8, 8, 128), (1, 8, 8, 128), qd=torch.float16),
        "rank3": qkv((8, 32, 128), (8, 8, 128), (8, 8, 128)),
        "kv_mismatch": qkv((1, 8, 32, 128), (1, 8, 8, 128), (1, 9, 8, 128)),
        "batch_mismatch": qkv((2, 8, 32, 128), (1, 8, 8, 128), (1, 8, 8, 128)),
        "dim64": qkv((1, 8, 32, 64), (1, 8, 8, 64), (1, 8, 8, 64)),
        "hq16_hkv4": qkv((1, 8, 16, 128), (1, 8, 4, 128), (1, 8, 4, 128)),
    }
    ref = {c["case"]: c["error"] for c in golden["qkv_errors"]}
    for name, (q, k, v) in cases.items():
        got = _err(lambda: varlen._validate_qkv(q, k, v))
        if name == "hq16_hkv4":
            # deliberate superset: the reference wrapper pins Hq=32/Hkv=8, its kernels do not
            assert ref[name]["message"] == "the qualified kernel requires Hq=32 and Hkv=8"
            assert got is None
        else:
            assert got == ref[name], name
    nc = dev(torch.zeros(1, 8, 32, 256, dtype=torch.bfloat16)[..., ::2])
    ok = dev(torch.zeros(1, 8, 8, 128, dtype=torch.bfloat16))
    assert _err(lambda: varlen._validate_qkv(nc, ok, ok)) == ref["non_contiguous"]
    cpu = torch.zeros(1, 8, 32, 128, dtype=torch.bfloat16)
    cpu_kv = torch.zeros(1, 8, 8, 128, dtype=torch.bfloat16)
    assert _err(lambda: varlen._validate_qkv(cpu, cpu_kv, cpu_kv)) == ref["cpu_tensors"]


def test_mask_errors_match_reference(golden):
    ref = {c["case"]: c["error"] for c in golden["mask_errors"]}
    assert _err(lambda: varlen.build_switch_query_indices(dev(torch.zeros(2, 8, dtype=torch.bool)))) == ref["batch2"]
    assert _err(lambda: varlen.build_switch_query_indices(dev(torch.zeros(8, dtype=torch.int32)))) == ref["int_mask"]
    assert _err(lambda: varlen.build_switch_query_indices(dev(torch.zeros(1, 1, 8, dtype=torch.bool)))) == ref["3d"]
    assert _err(lambda: varlen.build_switch_query_indices(torch.zeros(8, dtype=torch.bool))) == ref["cpu_tensor"]


def test_prepare_batch_error_matches_reference(golden):
    ref = {c["case"]: c["error"] for c in golden["prepare_errors"]}
    with CpuFactories():
        got = _err(lambda: varlen._prepare_indices(dev(torch.tensor([[0, 1], [0, 1]], dtype=torch.int32)),
                                                   seq_len=10, block_m=64))
    assert got == ref["two_batches"]


def test_forward_host_errors_match_reference(golden):
    ref = {c["case"]: c for c in golden["forward_errors"]}
    S = 64
    q = dev(torch.zeros(1, S, 32, 128, dtype=torch.bfloat16))
    k = dev(torch.zeros(1, S, 8, 128, dtype=torch.bfloat16))
    pos = torch.arange(S, dtype=torch.int32)
    with CpuFactories():
        got = _err(lambda: varlen.switch_gqa_prefill_forward(q, k, k, dev(pos[:10]), dev(pos[10:]), window_size=0))
        assert got == ref["window_zero"]["error"]
        bad = varlen.SwitchAttentionMetadata(*[dev(torch.zeros(S + 1, dtype=torch.int32))] * 7)
        got = _err(lambda: varlen.switch_gqa_prefill_forward(q, k, k, dev(pos[:10]), dev(pos[10:]), metadata=bad,
                                                             window_size=16))
        assert got == ref["bad_metadata"]["error"]
        got = _err(lambda: varlen.switch_gqa_prefill_forward(q, k, k, dev(pos[:10]), dev(pos[20:]), window_size=16,
                                                             validate=False))
        assert got == ref["not_covering"]["error"]
    # every reference error case launched nothing
    assert all(c["launches"] == 0 for c in golden["forward_errors"])


def test_reference_schedule_arguments_still_validated():
    q = dev(torch.zeros(1, 8, 32, 128, dtype=torch.bfloat16))
    with pytest.raises(AssertionError, match="BM64"):
        varlen.switch_gqa_prefill_forward(q, q, q, q, q, block_m=128)
    with pytest.raises(AssertionError, match="one stage"):
        varlen.switch_gqa_prefill_forward(q, q, q, q, q, num_stages=2)


@pytest.mark.parametrize("count", [0, 1, 63, 64, 65, 128, 129, 1000, 70000])
@pytest.mark.parametrize("block_m", [64, 128])
def test_bucket_capacity_matches_oracle(count, block_m):
    assert _core.bucket_capacity(count, block_m) == oracle_idx.bucket_capacity(count, block_m)


def test_library_exports_every_header_symbol():
    header = open(os.path.join(ROOT, "include", "swattn_b200.h")).read()
    declared = set(re.findall(r"^(?:int|int64_t|size_t|void|const char\*)\s+(swa_\w+)\(", header, flags=re.M))
    assert declared == set(_native.EXPORTED)
    lib = _native.load()  # loads without a GPU; no compute call is made
    for name in declared:
        assert hasattr(lib, name), name
    assert lib.swa_abi_version() == 1
    raw = ctypes.CDLL(_native.LIB_PATH)
    for name in declared:
        assert ctypes.cast(getattr(raw, name), ctypes.c_void_p).value


def test_effective_flops_counter_matches_oracle():
    rng = np.random.default_rng(0)
    for S, W in ((1000, 100), (4096, 4096), (777, 1)):
        mask = rng.random((2, S)) < 0.3
        full = [oracle_idx.compact_mask(m)[0] for m in mask]
        local = [oracle_idx.compact_mask(m)[1] for m in mask]
        n = oracle_attn.legal_key_counts(full, local, window=W, skv=S)
        assert workloads.effective_flops(mask, W, S, hq=8) == 4.0 * 128 * 8 * n
    cu = np.array([0, 100, 350, 351])
    mask = rng.random((1, 351)) < 0.5
    from oracle import metadata as om
    meta = om.build_metadata(351, 351, 64, cu)
    f, l = oracle_idx.compact_mask(mask[0])
    n = oracle_attn.legal_key_counts([f], [l], window=64, skv=351, metadata=meta)
    assert workloads.effective_flops(mask, 64, 351, hq=2, cu_seqlens=cu) == 4.0 * 128 * 2 * n


def test_markov_mask_statistics():
    u = np.random.default_rng(5).random((2, 400001))
    m = workloads.markov_mask(u, 0.125, 0.02)
    frac = m.mean()
    switches = (m[:, 1:] != m[:, :-1]).mean()
    assert abs(frac - 0.125) < 0.02
    assert abs(switches - 0.02) < 0.003


def test_config_shapes():
    c = workloads.CONFIGS
    assert (c[1].B, c[1].S, c[1].Hq, c[1].Hkv, c[1].window, c[1].p_full, c[1].seed) == (1, 1024, 8, 2, 256, 0.25, 0)
    assert (c[2].B, c[2].S, c[2].Hq, c[2].Hkv, c[2].window, c[2].p_full) == (1, 8192, 32, 8, 1024, 0.5)
    assert (c[3].B, c[3].S, c[3].Hq, c[3].Hkv, c[3].window, c[3].scale) == (4, 32768, 32, 8, 1024, 0.5)
    assert (c[4].Hq, c[4].Hkv, c[4].window, c[4].varlen) == (64, 8, 4096, (16, 512, 8192))
    assert (c[5].B, c[5].S, c[5].Hq, c[5].Hkv, c[5].window, c[5].p_sweep) == (2, 131072, 32, 4, 2048, (0.0, 0.01, 1.0))
    w = workloads.make_inputs(1)
    assert w["q"].shape == (1, 1024, 8, 128) and w["q"].dtype == torch.bfloat16
    assert w["mask"].shape == (1, 1024) and w["mask"].dtype == torch.bool
    lengths = workloads.varlen_lengths(c[4])
    assert lengths.size == 16 and lengths.min() >= 512 and lengths.max() <= 8192


def test_backward_workspace_query():
    # host arithmetic only: status word, then per (list slot, head) a 16-byte record,
    # a 4-byte position and the 256-byte Q and dO rows, each section 256-byte aligned
    lib = _native.load()
    for B, Hq, fs, ls in [(1, 32, 4096, 28672), (3, 16, 7, 300), (2, 8, 0, 5), (1, 1, 1, 0)]:
        rows = B * Hq * (fs + ls)
        got = lib.swa_backward_workspace_bytes(B, Hq, fs, ls)
        assert rows * 532 <= got <= rows * 532 + 256 * 6
    assert lib.swa_backward_workspace_bytes(0, 8, 4, 4) == 0
    assert lib.swa_backward_workspace_bytes(2, 8, -1, 4) == 0


def _plan(lib, B, Skv, Hq, Hkv, full_cap, local_cap, n_bg, window, request=0, sms=148):
    tiles = ctypes.c_int(-1)
    nbytes = lib.swa_prefill_split_plan(B, Skv, Hq, Hkv, full_cap, local_cap, n_bg, window, sms, request,
                                        ctypes.byref(tiles))
    return int(nbytes), tiles.value


def test_key_split_plan():
    # host arithmetic only: which launches split long full-causal units, and the scratch they need
    lib = _native.load()
    # config 3 at 1 and 8 GPUs (unit-major shards: B = units, Hkv = 1): never split
    assert _plan(lib, 4, 32768, 32, 8, 4300, 28672, 0, 1024) == (0, 0)
    assert _plan(lib, 4, 32768, 4, 1, 4300, 28672, 0, 1024) == (0, 0)
    # config 5 at p_full 1.0 / 0.0 / 0.01 on one GPU (8 units): no split
    assert _plan(lib, 2, 131072, 32, 4, 131072, 0, 0, 2048) == (0, 0)
    assert _plan(lib, 2, 131072, 32, 4, 0, 131072, 0, 2048) == (0, 0)
    assert _plan(lib, 2, 131072, 32, 4, 1400, 130000, 0, 2048) == (0, 0)
    # config 5 at p_full 0.01, one unit per GPU (8 GPUs): the 1024-tile full units are split
    nbytes, tiles = _plan(lib, 1, 131072, 8, 1, 1400, 130000, 0, 2048)
    assert 32 <= tiles < 1024
    pieces = -(-1024 // tiles)
    slots = -(-1400 // 32) * pieces
    assert nbytes == slots * 256 * 4 * (1 + 128)
    # the same share seen through list capacities only (lists padded to S): no split,
    # and a requested split keeps its scratch within 512 MiB (the longest units only)
    assert _plan(lib, 1, 131072, 8, 1, 131072, 131072, 0, 2048) == (0, 0)
    nbytes, tiles = _plan(lib, 1, 131072, 8, 1, 131072, 131072, 0, 2048, request=512)
    assert tiles == 512 and 0 < nbytes <= 512 << 20 and nbytes % (2 * 256 * 4 * 129) == 0
    # a requested piece length is honoured; none when no unit can be that long
    nbytes, tiles = _plan(lib, 2, 1000, 8, 2, 300, 700, 0, 64, request=2)
    # 4 (b, g) units x 5 position blocks x 4 pieces of 2 of the 8 tiles
    assert tiles == 2 and nbytes == 4 * (-(-300 // 64)) * 4 * 256 * 4 * 129
    assert _plan(lib, 2, 1000, 8, 2, 300, 700, 0, 64, request=8) == (0, 0)
    assert _plan(lib, 2, 1000, 8, 2, 0, 1000, 0, 64, request=2) == (0, 0)
    # bad shapes plan nothing
    assert _plan(lib, 0, 1000, 8, 2, 300, 700, 0, 64, request=2) == (0, 0)


def test_key_split_arguments_validated():
    S = 64
    q = dev(torch.zeros(1, S, 8, 128, dtype=torch.bfloat16))
    k = dev(torch.zeros(1, S, 2, 128, dtype=torch.bfloat16))
    pos = torch.arange(S, dtype=torch.int32)
    with CpuFactories():
        for bad in ("always", -1, True):
            got = _err(lambda: _core.forward(q, k, k, dev(pos[:10]), dev(pos[10:]), window_size=16, key_split=bad))
            assert got["type"] == "ValueError" and "key_split" in got["message"], (bad, got)
        for bad in ((1,), (-1, 5), (1, 2, 3)):
            got = _err(lambda: _core.forward(q, k, k, dev(pos[:10]), dev(pos[10:]), window_size=16, max_counts=bad))
            assert got["type"] == "ValueError" and "max_counts" in got["message"], (bad, got)
