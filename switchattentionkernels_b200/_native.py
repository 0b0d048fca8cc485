"""ctypes binding of libswattn_b200.so (C ABI: include/swattn_b200.h).

The library is loaded on first use.  There is no fallback: when the shared
object is missing or the device is not an sm_100 GPU the calls raise.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libswattn_b200.so")

SWA_OK = 0
STATUS_FULL_RANGE = 1 << 0
STATUS_FULL_ORDER = 1 << 1
STATUS_LOCAL_RANGE = 1 << 2
STATUS_LOCAL_ORDER = 1 << 3
STATUS_FULL_PAD = 1 << 4
STATUS_LOCAL_PAD = 1 << 5
STATUS_COVER = 1 << 6
STATUS_TIMEOUT = 1 << 16
ROUTER_BF16 = 1
ROUTER_F32 = 2

EXPORTED = (
    "swa_abi_version",
    "swa_last_error_string",
    "swa_num_sms",
    "swa_compact_mask",
    "swa_compact_router",
    "swa_compact_workspace_elems",
    "swa_compact_mask_ws",
    "swa_compact_router_ws",
    "swa_prepare_indices",
    "swa_check_cover",
    "swa_build_metadata",
    "swa_prefill_forward",
    "swa_noalloc_max_batch",
    "swa_prefill_forward_noalloc",
    "swa_test_withhold_kv_load",
    "swa_decode_workspace_bytes",
    "swa_decode_forward",
    "swa_prefill_backward",
    "swa_backward_workspace_bytes",
    "swa_broadcast_bytes",
    "swa_scatter_units",
    "swa_gather_units",
    "swa_prefill_forward_replicated",
    "swa_decode_forward_fp8",
    "swa_prefill_split_plan",
    "swa_prefill_forward_split",
)

_lock = threading.Lock()
_lib = None

_p = ctypes.c_void_p
_i = ctypes.c_int
_sz = ctypes.c_size_t
_f = ctypes.c_float


def _declare(lib) -> None:
    lib.swa_abi_version.restype = _i
    lib.swa_abi_version.argtypes = []
    lib.swa_last_error_string.restype = ctypes.c_char_p
    lib.swa_last_error_string.argtypes = []
    lib.swa_num_sms.restype = _i
    lib.swa_num_sms.argtypes = [_i]
    lib.swa_compact_mask.restype = _i
    lib.swa_compact_mask.argtypes = [_p, _i, _i, _p, _p, _p, _p]
    lib.swa_compact_router.restype = _i
    lib.swa_compact_router.argtypes = [_p, _i, _i, _f, _i, _i, _p, _p, _p, _p]
    lib.swa_compact_workspace_elems.restype = ctypes.c_int64
    lib.swa_compact_workspace_elems.argtypes = [_i, _i]
    lib.swa_compact_mask_ws.restype = _i
    lib.swa_compact_mask_ws.argtypes = [_p, _i, _i, _p, _p, _p, _p, ctypes.c_int64, _p]
    lib.swa_compact_router_ws.restype = _i
    lib.swa_compact_router_ws.argtypes = [_p, _i, _i, _f, _i, _i, _p, _p, _p, _p, ctypes.c_int64, _p]
    lib.swa_prepare_indices.restype = _i
    lib.swa_prepare_indices.argtypes = [_p, _i, _i, _i, _i, _i, _p, _p, _p, _i, _i, _i, _p]
    lib.swa_check_cover.restype = _i
    lib.swa_check_cover.argtypes = [_p, _i, _i, _p, _p]
    lib.swa_build_metadata.restype = _i
    lib.swa_build_metadata.argtypes = [_p, _i, _i, _i, _i, _p, _p, _p, _p, _p, _p, _p, _p]
    lib.swa_prefill_forward.restype = _i
    lib.swa_prefill_forward.argtypes = [
        _p, _p, _p,            # q, k, v
        _p, _p,                # full_idx, local_idx
        _i, _i, _i, _i,        # strides, caps
        _p, _i, _i, _i,        # counts, counts_batch_major, count_full, count_local
        _p, _p, _p,            # full_starts, local_starts, causal_ends
        _p, _i,                # bg_list, n_bg
        _p, _p,                # out, lse
        _i, _i, _i, _i, _i, _i,  # B, Sq, Skv, Hq, Hkv, head_dim
        _i, _f,                # window, scale_log2
        _p, _p, _sz,           # gate, workspace, workspace_bytes
        _p,                    # stream
    ]
    lib.swa_prefill_split_plan.restype = _sz
    lib.swa_prefill_split_plan.argtypes = [_i, _i, _i, _i, _i, _i, _i, _i, _i, _i, ctypes.POINTER(_i)]
    lib.swa_prefill_forward_split.restype = _i
    lib.swa_prefill_forward_split.argtypes = list(lib.swa_prefill_forward.argtypes[:-1]) + [
        _i, _p, _sz,           # split_tiles, scratch, scratch_bytes
        _p,                    # stream
    ]
    lib.swa_noalloc_max_batch.restype = _i
    lib.swa_noalloc_max_batch.argtypes = []
    lib.swa_prefill_forward_noalloc.restype = _i
    lib.swa_prefill_forward_noalloc.argtypes = [
        _p, _p, _p,            # q, k, v
        _p, _p, _i, _i,        # full_idx, local_idx, full_stride, local_stride
        _p, _p, _p,            # full_starts, local_starts, causal_ends
        _p, _p,                # out, lse
        _i, _i, _i, _i, _i, _i,  # B, Sq, Skv, Hq, Hkv, head_dim
        _i, _f,                # window, scale_log2
        _p, _p,                # status_out, stream
    ]
    lib.swa_test_withhold_kv_load.restype = None
    lib.swa_test_withhold_kv_load.argtypes = [_i]
    lib.swa_prefill_backward.restype = _i
    lib.swa_prefill_backward.argtypes = [
        _p, _p, _p, _p, _p, _p,  # q, k, v, o, lse, dout
        _p, _p, _i, _i, _p,      # full_idx, local_idx, full_stride, local_stride, counts
        _p, _p, _p,              # full_starts, local_starts, causal_ends
        _p, _p, _p,              # dq, dk, dv
        _i, _i, _i, _i, _i, _i,  # B, Sq, Skv, Hq, Hkv, head_dim
        _i, _f,                  # window, scale_log2
        _p, _sz, _p,             # workspace, workspace_bytes, stream
    ]
    lib.swa_backward_workspace_bytes.restype = _sz
    lib.swa_backward_workspace_bytes.argtypes = [_i, _i, _i, _i]
    lib.swa_decode_workspace_bytes.restype = _sz
    lib.swa_decode_workspace_bytes.argtypes = [_i, _i, _i, _i]
    lib.swa_decode_forward.restype = _i
    lib.swa_decode_forward.argtypes = [
        _p, _p, _p, _p, _p,    # q, k_cache, v_cache, seq_lens, route
        _p, _p,                # out, lse
        _i, _i, _i, _i, _i,    # B, Smax, Hq, Hkv, head_dim
        _i, _f,                # window, scale_log2
        _p, _sz, _p,           # workspace, workspace_bytes, stream
    ]
    lib.swa_decode_forward_fp8.restype = _i
    lib.swa_decode_forward_fp8.argtypes = [
        _p, _p, _p, _p, _p,    # q, k_cache, v_cache, k_scale, v_scale
        _p, _p,                # seq_lens, route
        _p, _p,                # out, lse
        _i, _i, _i, _i, _i,    # B, Smax, Hq, Hkv, head_dim
        _i, _f,                # window, scale_log2
        _p, _sz, _p,           # workspace, workspace_bytes, stream
    ]
    lib.swa_prefill_forward_replicated.restype = _i
    lib.swa_prefill_forward_replicated.argtypes = [
        _p, _p, _p,            # q, k, v (unit-major)
        _p, _p, _i, _i,        # full_idx, local_idx, full_stride, local_stride
        _p, _p, _p, _p,        # counts [B, 2], full_starts, local_starts, causal_ends
        _p,                    # unit_gid
        _i, _i, _i, _i, _i,    # B, Sq, Skv, Hq, head_dim
        _i, _f,                # window, scale_log2
        _i, _i, _p, _p,        # rep_hkv, n_rep, rep_out[], rep_lse[]
        _p, _p,                # out, lse (nullable)
        _p, _sz, _p,           # workspace, workspace_bytes, stream
    ]
    for name in ("swa_scatter_units", "swa_gather_units"):
        fn = getattr(lib, name)
        fn.restype = _i
        fn.argtypes = [_p, _p, _i, _i, _i, _i, _i, _p, _p]  # src, unit_of_slot, n_slots, S, hkv, chunk, row, dst, stream
    lib.swa_broadcast_bytes.restype = _i
    lib.swa_broadcast_bytes.argtypes = [_p, _sz, _p, _i, _p]  # src, bytes, dsts[], n_dst, stream


def load():
    """Load (once) and return the native library; raise if it is not built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with `python -m switchattentionkernels_b200.build`")
                lib = ctypes.CDLL(LIB_PATH)
                _declare(lib)
                if lib.swa_abi_version() != 1:
                    raise RuntimeError("libswattn_b200 ABI version mismatch")
                _lib = lib
    return _lib


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_ptr(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def check(rc: int, what: str) -> None:
    if rc != SWA_OK:
        msg = load().swa_last_error_string().decode(errors="replace")
        if rc == -1:
            raise ValueError(f"{what}: {msg}")
        raise RuntimeError(f"{what} failed ({rc}): {msg}")
