"""Seeded synthetic workloads of the Switch Attention prefill benchmark and the
effective-work counter.

The five configurations are the benchmark's named shapes: q/k/v i.i.d. N(0,1)
BF16 (config 3 scales them by 0.5), a routing mask per (batch, position) with
``True`` = full causal attention, window sizes and head counts as listed in
``CONFIGS``.  No public dataset is involved.  Values are drawn from a torch
generator seeded with the config's seed, in the order q, k, v, mask (config 4
draws its sequence lengths first).  Small configs draw on the CPU; large ones
may draw on the GPU (``on_device=True``), which is seeded the same way but gives
different numbers than the CPU stream.

Effective work counts only legal (row, key) score entries: a full row at
in-sequence position ``i`` sees ``i + 1`` keys, a local row ``min(i + 1, W)``;
FLOPs = ``4 * D * sum over heads and rows``.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch


@dataclass(frozen=True)
class Config:
    name: str
    B: int
    S: int
    Hq: int
    Hkv: int
    window: int
    p_full: float
    seed: int
    scale: float = 1.0
    markov_switch: float | None = None      # mean per-step switch probability of a 2-state chain
    varlen: tuple[int, int, int] | None = None  # (n_seqs, min_len, max_len)
    p_sweep: tuple[float, ...] = field(default_factory=tuple)


CONFIGS = {
    1: Config("c1_b1_s1024_hq8_hkv2_w256", 1, 1024, 8, 2, 256, 0.25, 0),
    2: Config("c2_b1_s8192_hq32_hkv8_w1024", 1, 8192, 32, 8, 1024, 0.5, 1),
    3: Config("c3_b4_s32768_hq32_hkv8_w1024_markov", 4, 32768, 32, 8, 1024, 0.125, 2, scale=0.5,
              markov_switch=0.02),
    4: Config("c4_varlen16_hq64_hkv8_w4096", 1, 0, 64, 8, 4096, 0.3, 3, varlen=(16, 512, 8192)),
    5: Config("c5_b2_s131072_hq32_hkv4_w2048", 2, 131072, 32, 4, 2048, 0.01, 4, p_sweep=(0.0, 0.01, 1.0)),
}

HEAD_DIM = 128


def markov_mask(u: np.ndarray, p_full: float, switch: float) -> np.ndarray:
    """Two-state routing chain per row of ``u`` (uniform draws, ``[B, S + 1]``).

    Stationary full fraction ``p_full``, mean per-step switch probability
    ``switch``: P(local -> full) = switch / (2 (1 - p_full)),
    P(full -> local) = switch / (2 p_full).  Column 0 draws the initial state.
    """
    a = switch / (2.0 * (1.0 - p_full))
    b = switch / (2.0 * p_full)
    B, S1 = u.shape
    out = np.zeros((B, S1 - 1), dtype=bool)
    for r in range(B):
        state = bool(u[r, 0] < p_full)
        row = u[r, 1:]
        for t in range(S1 - 1):
            out[r, t] = state
            if state:
                if row[t] < b:
                    state = False
            elif row[t] < a:
                state = True
    return out


def varlen_lengths(cfg: Config) -> np.ndarray:
    n, lo, hi = cfg.varlen
    g = torch.Generator().manual_seed(cfg.seed)
    return torch.randint(lo, hi + 1, (n,), generator=g).numpy().astype(np.int64)


def make_inputs(cfg_id: int, *, device="cpu", p_full: float | None = None, on_device: bool = False,
                batch_override: int | None = None, seed_offset: int = 0):
    """q, k, v (BF16), mask (bool [B, S]) and, for config 4, ``cu_seqlens``.

    ``batch_override`` draws a batch of a different size with the same recipe
    (used for weak-scaling runs, where each GPU gets its own copy of the batch);
    ``seed_offset`` shifts the seed (one independent draw per GPU).
    """
    cfg = CONFIGS[cfg_id]
    if seed_offset:
        from dataclasses import replace
        cfg = replace(cfg, seed=cfg.seed + seed_offset)
    p = cfg.p_full if p_full is None else p_full
    gen_dev = torch.device(device) if on_device else torch.device("cpu")
    g = torch.Generator(device=gen_dev).manual_seed(cfg.seed)
    cu = None
    if cfg.varlen is not None:
        lengths = varlen_lengths(cfg)
        g = torch.Generator(device=gen_dev).manual_seed(cfg.seed + 1000)
        S = int(lengths.sum())
        B = 1
        cu = np.zeros(lengths.size + 1, dtype=np.int64)
        cu[1:] = np.cumsum(lengths)
    else:
        S = cfg.S
        B = batch_override or cfg.B
    q = torch.randn((B, S, cfg.Hq, HEAD_DIM), generator=g, device=gen_dev, dtype=torch.float32)
    q = (q * cfg.scale).to(torch.bfloat16) if cfg.scale != 1.0 else q.to(torch.bfloat16)
    k = torch.randn((B, S, cfg.Hkv, HEAD_DIM), generator=g, device=gen_dev, dtype=torch.float32)
    k = (k * cfg.scale).to(torch.bfloat16) if cfg.scale != 1.0 else k.to(torch.bfloat16)
    v = torch.randn((B, S, cfg.Hkv, HEAD_DIM), generator=g, device=gen_dev, dtype=torch.float32)
    v = (v * cfg.scale).to(torch.bfloat16) if cfg.scale != 1.0 else v.to(torch.bfloat16)
    if cfg.markov_switch is not None:
        u = torch.rand((B, S + 1), generator=g, device=gen_dev, dtype=torch.float64).cpu().numpy()
        mask = torch.from_numpy(markov_mask(u, p, cfg.markov_switch))
    else:
        mask = (torch.rand((B, S), generator=g, device=gen_dev, dtype=torch.float32) < p).cpu()
    out = {
        "cfg": cfg, "q": q.to(device), "k": k.to(device), "v": v.to(device), "mask": mask,
        "window": cfg.window, "p_full": p,
        "cu_seqlens": None if cu is None else torch.from_numpy(cu.astype(np.int32)),
    }
    return out


def legal_keys_per_row(mask: np.ndarray, window: int, skv: int, cu_seqlens=None) -> np.ndarray:
    """Number of legal keys of every (batch, position) row, ``[B, S]`` int64."""
    mask = np.asarray(mask, dtype=bool)
    B, S = mask.shape
    t = np.arange(S, dtype=np.int64)
    if cu_seqlens is None:
        start = np.zeros(S, dtype=np.int64)
    else:
        cu = np.asarray(cu_seqlens, dtype=np.int64)
        start = cu[np.searchsorted(cu, t, side="right") - 1]
    hi = np.minimum(t + 1, skv)
    lo_full = start
    lo_local = np.maximum(start, t - window + 1)
    n_full = np.maximum(hi - lo_full, 0)
    n_local = np.maximum(hi - lo_local, 0)
    return np.where(mask, n_full[None, :], n_local[None, :])


def effective_flops(mask, window: int, skv: int, hq: int, cu_seqlens=None, head_dim: int = HEAD_DIM) -> float:
    """``4 * D * N_eff`` with ``N_eff`` = legal (row, key) entries summed over heads."""
    n_eff = int(legal_keys_per_row(mask, window, skv, cu_seqlens).sum()) * hq
    return 4.0 * head_dim * n_eff
