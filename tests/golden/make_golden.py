"""Generate golden vectors by executing the reference's own Python on the CPU.

Run from the repository root in a container that has the reference checkout:

    python tests/golden/make_golden.py /path/to/SwitchAttentionKernels

It imports ``swiattn_gqa_prefill_varlen.py`` of YushengZhao/SwitchAttentionKernels
unchanged and calls its host functions -- ``build_switch_query_indices``,
``_prepare_indices``, ``_validate_qkv`` and ``switch_gqa_prefill_forward`` -- on
CPU tensors.  Three stand-ins make that possible without a GPU and without the
TileLang JIT:

* a CPU tensor subclass that reports ``is_cuda == True`` / ``device == cuda:0``
  (the reference rejects non-CUDA tensors), together with a torch-function mode
  that turns ``device=`` arguments of factory calls back into ``cpu``;
* a minimal ``tilelang`` module whose ``jit`` decorator records each branch
  launch (its arguments) instead of compiling the TileLang kernel;
* the ``metadata`` module the reference imports but does not ship
  (``swiattn_gqa_prefill_varlen.py:27``): a dataclass with the seven fields the
  wrapper reads; every forward fixture passes metadata explicitly.

The kernel itself is never executed (it lowers only for Hopper); the fixtures
pin the index compaction, the capacity buckets, the dispatch decisions
(which branch launches, with which capacity and count) and the validation
errors.  Output: ``tests/golden/reference_host.npz`` + ``reference_host.json``.
"""
from __future__ import annotations

import dataclasses
import importlib.util
import json
import os
import sys
import types

import numpy as np
import torch
from torch.overrides import TorchFunctionMode

HERE = os.path.dirname(os.path.abspath(__file__))


class HostAsCuda(torch.Tensor):
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


def dev(t: torch.Tensor) -> torch.Tensor:
    return t.as_subclass(HostAsCuda)


LAUNCHES: list[dict] = []


def _install_stubs():
    tl = types.ModuleType("tilelang")

    class PassConfigKey:
        TL_DISABLE_TMA_LOWER = "tl.disable_tma_lower"
        TL_DISABLE_WARP_SPECIALIZED = "tl.disable_warp_specialized"
        TL_ENABLE_FAST_MATH = "tl.enable_fast_math"

    def jit(pass_configs=None):
        def deco(fn):
            def record(*args, **kwargs):
                names = ["Q", "K", "V", "QueryIndices", "QueryCount", "FullStarts", "LocalStarts", "CausalEnds",
                         "Output", "Lse", "heads", "dim", "num_queries", "kv_group", "window_size", "sm_scale"]
                bound = dict(zip(names, args))
                bound.update(kwargs)
                LAUNCHES.append({
                    "is_local": bool(bound.get("is_local", False)),
                    "query_indices": np.asarray(bound["QueryIndices"].as_subclass(torch.Tensor)).tolist(),
                    "query_count": np.asarray(bound["QueryCount"].as_subclass(torch.Tensor)).tolist(),
                    "heads": int(bound["heads"]),
                    "dim": int(bound["dim"]),
                    "num_queries": int(bound["num_queries"]),
                    "kv_group": int(bound["kv_group"]),
                    "window_size": int(bound["window_size"]),
                    "sm_scale": None if bound["sm_scale"] is None else float(bound["sm_scale"]),
                    "block_M": int(bound["block_M"]),
                    "block_K": int(bound["block_K"]),
                    "num_stages": int(bound["num_stages"]),
                    "threads": int(bound["threads"]),
                })
            return record
        return deco

    tl.PassConfigKey = PassConfigKey
    tl.jit = jit
    lang = types.ModuleType("tilelang.language")
    tl.language = lang
    sys.modules["tilelang"] = tl
    sys.modules["tilelang.language"] = lang

    pkg = types.ModuleType("swiref")
    pkg.__path__ = []
    sys.modules["swiref"] = pkg
    meta = types.ModuleType("swiref.metadata")

    @dataclasses.dataclass
    class SwitchAttentionMetadata:
        q_positions: torch.Tensor
        kv_positions: torch.Tensor
        q_segment_ids: torch.Tensor
        kv_segment_ids: torch.Tensor
        full_starts: torch.Tensor
        local_starts: torch.Tensor
        causal_ends: torch.Tensor

    def build_switch_attention_metadata(*a, **k):
        raise NotImplementedError("fixtures pass metadata explicitly")

    meta.SwitchAttentionMetadata = SwitchAttentionMetadata
    meta.build_switch_attention_metadata = build_switch_attention_metadata
    sys.modules["swiref.metadata"] = meta
    return SwitchAttentionMetadata


def load_reference(ref_dir: str):
    Meta = _install_stubs()
    path = os.path.join(ref_dir, "swiattn_gqa_prefill_varlen.py")
    spec = importlib.util.spec_from_file_location("swiref.swiattn_gqa_prefill_varlen", path)
    mod = importlib.util.module_from_spec(spec)
    mod.__package__ = "swiref"
    spec.loader.exec_module(mod)
    return mod, Meta


def capture_error(fn):
    try:
        fn()
    except Exception as e:  # noqa: BLE001 - the fixture records whatever the reference raises
        return {"type": type(e).__name__, "message": str(e)}
    return None


def single_metadata(Meta, q_len, kv_len, window):
    t = torch.arange(q_len, dtype=torch.int32)
    return Meta(
        q_positions=dev(t.clone()), kv_positions=dev(torch.arange(kv_len, dtype=torch.int32)),
        q_segment_ids=dev(torch.zeros(q_len, dtype=torch.int32)),
        kv_segment_ids=dev(torch.zeros(kv_len, dtype=torch.int32)),
        full_starts=dev(torch.zeros(q_len, dtype=torch.int32)),
        local_starts=dev(torch.clamp(t - window + 1, min=0).to(torch.int32)),
        causal_ends=dev((t + 1).to(torch.int32)))


def main(ref_dir: str):
    ref, Meta = load_reference(ref_dir)
    arrays: dict[str, np.ndarray] = {}
    record: dict = {"compaction": [], "prepare": [], "prepare_errors": [], "mask_errors": [],
                    "qkv_errors": [], "forward": [], "forward_errors": []}
    rng = np.random.default_rng(20260101)
    with CpuFactories():
        # 1. build_switch_query_indices (swiattn_gqa_prefill_varlen.py:306-322)
        cases = [(1, 0.5), (2, 0.5), (15, 0.3), (16, 0.3), (17, 0.7), (100, 0.0), (100, 1.0), (1000, 0.25),
                 (4097, 0.5), (16385, 0.125)]
        for i, (S, p) in enumerate(cases):
            mask = rng.random(S) < p
            for shape2d in (False, True):
                m = torch.from_numpy(mask)
                if shape2d:
                    m = m.unsqueeze(0)
                f, l = ref.build_switch_query_indices(dev(m))
                key = f"compaction_{i}_{int(shape2d)}"
                arrays[key + "_mask"] = np.packbits(mask)
                arrays[key + "_full"] = np.asarray(f.as_subclass(torch.Tensor))
                arrays[key + "_local"] = np.asarray(l.as_subclass(torch.Tensor))
                record["compaction"].append({"key": key, "S": S, "p": p, "shape2d": shape2d,
                                             "full_dtype": str(f.dtype), "local_dtype": str(l.dtype)})
        for desc, t in (("batch2", torch.zeros(2, 8, dtype=torch.bool)),
                        ("int_mask", torch.zeros(8, dtype=torch.int32)),
                        ("3d", torch.zeros(1, 1, 8, dtype=torch.bool))):
            record["mask_errors"].append({"case": desc, "error": capture_error(
                lambda t=t: ref.build_switch_query_indices(dev(t)))})
        record["mask_errors"].append({"case": "cpu_tensor", "error": capture_error(
            lambda: ref.build_switch_query_indices(torch.zeros(8, dtype=torch.bool)))})

        # 2. _prepare_indices (swiattn_gqa_prefill_varlen.py:271-304)
        for count in (0, 1, 2, 63, 64, 65, 127, 128, 129, 255, 256, 257, 1000, 4096, 4097):
            for block_m in (64, 128):
                idx = np.sort(rng.choice(10000, size=count, replace=False)).astype(np.int32)
                padded, cnt = ref._prepare_indices(dev(torch.from_numpy(idx)), seq_len=10000, block_m=block_m)
                key = f"prepare_{count}_{block_m}"
                arrays[key + "_in"] = idx
                arrays[key + "_padded"] = np.asarray(padded.as_subclass(torch.Tensor))
                arrays[key + "_count"] = np.asarray(cnt.as_subclass(torch.Tensor))
                record["prepare"].append({"key": key, "count": count, "block_m": block_m, "seq_len": 10000,
                                          "padded_shape": list(padded.shape)})
        for desc, vals, seq_len in (("descending", [5, 3, 9], 100), ("duplicate", [1, 1, 2], 100),
                                    ("negative", [-1, 3, 4], 100), ("too_large", [0, 5, 100], 100),
                                    ("range_and_order", [7, 3, 200], 100)):
            record["prepare_errors"].append({"case": desc, "values": vals, "seq_len": seq_len, "error": capture_error(
                lambda v=vals, s=seq_len: ref._prepare_indices(dev(torch.tensor(v, dtype=torch.int32)),
                                                               seq_len=s, block_m=64))})
        record["prepare_errors"].append({"case": "two_batches", "values": [[0, 1], [0, 1]], "seq_len": 10,
                                         "error": capture_error(lambda: ref._prepare_indices(
                                             dev(torch.tensor([[0, 1], [0, 1]], dtype=torch.int32)),
                                             seq_len=10, block_m=64))})

        # 3. _validate_qkv (swiattn_gqa_prefill_varlen.py:251-269)
        def qkv(qs, ks, vs, qd=torch.bfloat16, kd=torch.bfloat16, vd=torch.bfloat16):
            return (dev(torch.zeros(qs, dtype=qd)), dev(torch.zeros(ks, dtype=kd)), dev(torch.zeros(vs, dtype=vd)))
        qkv_cases = {
            "ok": qkv((1, 8, 32, 128), (1, 8, 8, 128), (1, 8, 8, 128)),
            "fp16_q": qkv((1, 8, 32, 128), (1, 8, 8, 128), (1, 8, 8, 128), qd=torch.float16),
            "rank3": qkv((8, 32, 128), (8, 8, 128), (8, 8, 128)),
            "kv_mismatch": qkv((1, 8, 32, 128), (1, 8, 8, 128), (1, 9, 8, 128)),
            "batch_mismatch": qkv((2, 8, 32, 128), (1, 8, 8, 128), (1, 8, 8, 128)),
            "dim64": qkv((1, 8, 32, 64), (1, 8, 8, 64), (1, 8, 8, 64)),
            "hq16_hkv4": qkv((1, 8, 16, 128), (1, 8, 4, 128), (1, 8, 4, 128)),
        }
        for name, (q, k, v) in qkv_cases.items():
            record["qkv_errors"].append({"case": name, "error": capture_error(lambda q=q, k=k, v=v: ref._validate_qkv(q, k, v))})
        nc = torch.zeros(1, 8, 32, 256, dtype=torch.bfloat16)[..., ::2]
        record["qkv_errors"].append({"case": "non_contiguous", "error": capture_error(lambda: ref._validate_qkv(
            dev(nc), dev(torch.zeros(1, 8, 8, 128, dtype=torch.bfloat16)), dev(torch.zeros(1, 8, 8, 128, dtype=torch.bfloat16))))})
        record["qkv_errors"].append({"case": "cpu_tensors", "error": capture_error(lambda: ref._validate_qkv(
            torch.zeros(1, 8, 32, 128, dtype=torch.bfloat16), torch.zeros(1, 8, 8, 128, dtype=torch.bfloat16),
            torch.zeros(1, 8, 8, 128, dtype=torch.bfloat16)))})

        # 4. switch_gqa_prefill_forward dispatch (swiattn_gqa_prefill_varlen.py:324-446)
        for i, (S, p, window, block_m, sm_scale) in enumerate(
                [(256, 0.25, 64, 64, None), (256, 0.0, 32, 64, None), (256, 1.0, 32, 64, 0.1),
                 (320, 0.5, 1000, 64, None), (130, 0.5, 7, 64, None)]):
            mask = rng.random(S) < p
            pos = np.arange(S, dtype=np.int32)
            f, l = pos[mask], pos[~mask]
            q = dev(torch.zeros(1, S, 32, 128, dtype=torch.bfloat16))
            k = dev(torch.zeros(1, S, 8, 128, dtype=torch.bfloat16))
            meta = single_metadata(Meta, S, S, window)
            LAUNCHES.clear()
            ref.switch_gqa_prefill_forward(q, k, k, dev(torch.from_numpy(f)), dev(torch.from_numpy(l)),
                                           metadata=meta, window_size=window, sm_scale=sm_scale, block_m=block_m)
            key = f"forward_{i}"
            arrays[key + "_mask"] = np.packbits(mask)
            record["forward"].append({"key": key, "S": S, "window": window, "block_m": block_m,
                                      "sm_scale": sm_scale, "launches": list(LAUNCHES)})

        S = 64
        q = dev(torch.zeros(1, S, 32, 128, dtype=torch.bfloat16))
        k = dev(torch.zeros(1, S, 8, 128, dtype=torch.bfloat16))
        meta = single_metadata(Meta, S, S, 16)
        all_pos = torch.arange(S, dtype=torch.int32)
        err_cases = {
            "not_covering": lambda: ref.switch_gqa_prefill_forward(q, k, k, dev(all_pos[:10]), dev(all_pos[20:]),
                                                                   metadata=meta, window_size=16),
            "window_zero": lambda: ref.switch_gqa_prefill_forward(q, k, k, dev(all_pos[:10]), dev(all_pos[10:]),
                                                                  metadata=meta, window_size=0),
            "batch2": lambda: ref.switch_gqa_prefill_forward(
                dev(torch.zeros(2, S, 32, 128, dtype=torch.bfloat16)), dev(torch.zeros(2, S, 8, 128, dtype=torch.bfloat16)),
                dev(torch.zeros(2, S, 8, 128, dtype=torch.bfloat16)), dev(all_pos[:10]), dev(all_pos[10:]),
                metadata=meta, window_size=16),
            "bad_metadata": lambda: ref.switch_gqa_prefill_forward(
                q, k, k, dev(all_pos[:10]), dev(all_pos[10:]), window_size=16,
                metadata=Meta(*[dev(torch.zeros(S + 1, dtype=torch.int32))] * 7)),
            "unsorted_full": lambda: ref.switch_gqa_prefill_forward(
                q, k, k, dev(torch.tensor([5, 3], dtype=torch.int32)),
                dev(torch.tensor([i for i in range(S) if i not in (3, 5)], dtype=torch.int32)),
                metadata=meta, window_size=16),
            "range_local": lambda: ref.switch_gqa_prefill_forward(
                q, k, k, dev(all_pos[:10]), dev(torch.arange(10, S + 1, dtype=torch.int32)),
                metadata=meta, window_size=16),
            "range_full_and_cover": lambda: ref.switch_gqa_prefill_forward(
                q, k, k, dev(torch.tensor([0, 99], dtype=torch.int32)), dev(all_pos[10:]),
                metadata=meta, window_size=16),
        }
        for name, fn in err_cases.items():
            LAUNCHES.clear()
            record["forward_errors"].append({"case": name, "error": capture_error(fn), "launches": len(LAUNCHES)})

    np.savez_compressed(os.path.join(HERE, "reference_host.npz"), **arrays)
    with open(os.path.join(HERE, "reference_host.json"), "w") as fh:
        json.dump(record, fh, indent=1)
    print("wrote", len(arrays), "arrays;", {k: len(v) for k, v in record.items()})


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference checkout directory>")
    main(sys.argv[1])
