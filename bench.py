#!/usr/bin/env python
"""Switch Attention GQA prefill benchmark on B200: effective TFLOP/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: config 3, the 32K-token mixed-routing batch (B=4, S=32768, Hq=32,
Hkv=8, D=128, W=1024, q/k/v ~ 0.5*N(0,1) BF16, two-state Markov routing with
stationary p_full=0.125).  Effective work counts only legal score entries
(4*D per entry and head).

The batch's 32 (batch, KV group) units are sharded over the N ranks
(longest-processing-time first on their legal-entry cost; strong scaling: the
batch is fixed as N grows).  A rank holds only its units, unit-major
([units, S, Hq/Hkv, 128] q, [units, S, 1, 128] k / v, the units' mask rows),
and one step is the hot path over them: routing-mask compaction and the
persistent prefill kernel.  No collective is in the data path.

``value`` = effective FLOP of the batch / the slowest rank's device-timed step
(inputs resident in HBM, no host sync inside a step).  ``gather`` = the same
with every step ending in the NCCL all-gather of every rank's O and LSE and the
scatter kernel into [B, S, Hq, ...] on every rank (a replicated result).
``e2e`` = the same metric through the public API from pinned host buffers: every
step copies the rank's own units (q/k/v/mask) host->device, runs
build_switch_query_indices_batched + switch_gqa_prefill_forward (validating, as
the reference does) and copies the rank's O and LSE back; consecutive steps are
pipelined over a copy-in, a compute and a copy-out stream (two device input
slots), as a serving loop would run them.  The copy byte counts are summed over
the ranks.  ``steady`` repeats the device-timed step back to back for at least
two seconds with its own clock record.  At N=1 the line also carries the same
kernel on the row-major [B, S, Hq, 128] layout (``standard_layout``), one
backward step (dQ, dK, dV) and one decode step over a BF16 and over an FP8
cache.  ``--replicas`` instead gives every rank its own 4 sequences (weak
scaling); ``--cp`` times context-parallel prefill of one packed batch.  ``--impl reference`` times the
CPU restatement of the reference path (the reference kernels are Hopper-only
TileLang programs and cannot run on B200 or on a CPU).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from switchattentionkernels_b200 import workloads  # noqa: E402

METRIC = "effective TFLOP/s (unmasked entries) & % BF16 TC peak at 1/2/4/8 B200"
UNIT = "TFLOP/s"
CONFIG_ID = 3
FALLBACK_PEAK_TFLOPS = 1590.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample budget")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences per GPU (default: the workload's 4); smaller values give profiling-size cases")
    ap.add_argument("--cp", action="store_true",
                    help="instead of the default line: context-parallel prefill over the N ranks "
                         "(strong scaling; K/V exchange + kernel per step)")
    ap.add_argument("--replicas", action="store_true",
                    help="instead of the default line: every rank computes its own 4 sequences (weak scaling)")
    ap.add_argument("--steady-seconds", type=float, default=2.0,
                    help="length of the back-to-back steady-state block after the timed steps")
    ap.add_argument("--workload", type=int, choices=[3, 5], default=CONFIG_ID,
                    help="default line's workload: 3 (the headline) or 5 (two 131072-token sequences, Hkv 4)")
    ap.add_argument("--p-full", type=float, default=None, help="with --workload 5: routing density p_full")
    ap.add_argument("--p-sweep", type=str, default=None,
                    help="with --workload 5: comma-separated p_full values, one line each from one process")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the N=1 extras (standard-layout kernel, backward and decode steps)")
    ap.add_argument("--backward", action="store_true",
                    help="instead of the default line: the prefill backward (dQ, dK, dV) of the config-3 workload")
    ap.add_argument("--decode", action="store_true",
                    help="instead of the default line: one decode step (one new token per sequence) over a KV cache")
    ap.add_argument("--cp-config", type=int, choices=[4, 5], default=4,
                    help="--cp workload: 4 = the varlen packed batch, 5 = one 131072-token sequence of config 5")
    return ap.parse_args()


# --------------------------------------------------------------------------- helpers
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            d = json.load(fh)
        return float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    return FALLBACK_PEAK_TFLOPS, 1400.0, "fallback"


def profile_traffic(workload: str):
    """Per-launch DRAM traffic (bytes) of the prefill kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "prefill_config3_ncu.md")
    if not os.path.exists(path):
        return None
    with open(path) as fh:
        for line in fh:
            if line.startswith("traffic_bytes_per_launch_full_workload:"):
                try:
                    return float(line.split(":", 1)[1].strip().split()[0])
                except ValueError:
                    return None
    return None


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", f"swa_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        # nvidia-smi takes a moment to start: wait (at most 5 s) for its first sample so
        # that the samples cover the timed region that follows
        deadline = time.time() + 5.0
        while time.time() < deadline and os.path.getsize(self.path) == 0:
            time.sleep(0.05)

    def mark(self, which: str):
        """Wall-clock bounds of the timed region; only samples inside it are kept."""
        setattr(self, which, datetime.datetime.now())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        t_begin = getattr(self, "begin", None)
        t_end = getattr(self, "end", None)
        rows = []
        with open(self.path) as fh:
            for line in fh:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 10:
                    continue
                try:
                    ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f")
                except ValueError:
                    ts = None
                rows.append((ts, parts))
        inside = [r for r in rows if r[0] is not None and t_begin is not None and t_end is not None
                  and t_begin <= r[0] <= t_end]
        for _, parts in (inside or rows):  # all samples if the timestamps cannot be matched
            try:
                sms.append(float(parts[2]))
                maxes.append(float(parts[3]))
            except ValueError:
                continue
            for name, val in zip(names, parts[6:10]):
                if val.lower() == "active":
                    reasons.add(name)
        os.unlink(self.path)
        if not sms:
            return None
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes), "samples": len(sms),
                "reasons": sorted(reasons)}


def unit_flops(mask: np.ndarray, window: int, hq: int, skv: int) -> float:
    return workloads.effective_flops(mask, window, skv, hq)


def config3_dict(world: int, cfg_id: int = CONFIG_ID, p_full: float | None = None) -> dict:
    """``config`` of the default line: the same keys and values in both arms."""
    cfg = workloads.CONFIGS[cfg_id]
    p = cfg.p_full if p_full is None else p_full
    gib = (cfg.B * cfg.S * (cfg.Hq + 2 * cfg.Hkv) * 128 * 2) / 2**30
    return {"workload": cfg.name, "B": cfg.B, "S": cfg.S, "Hq": cfg.Hq, "Hkv": cfg.Hkv, "head_dim": 128,
            "window": cfg.window, "p_full": p,
            "routing": "markov(switch=0.02)" if cfg.markov_switch is not None else "bernoulli",
            "units": cfg.B * cfg.Hkv,
            "parallelism": f"(batch, KV group) units sharded over {world} rank(s), LPT on legal entries",
            "l2": f"inputs larger than L2 (q/k/v {gib:.1f} GiB)"}


# --------------------------------------------------------------------------- CPU baseline (oracle)
def cpu_oracle_sample(inputs, seconds: float, rng_seed: int = 123):
    """Time the CPU restatement on random 256-position blocks until ``seconds`` elapse."""
    from oracle import attention as oracle_attn  # test infrastructure: the CPU baseline only

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    q, k, v, mask, W = inputs["q_cpu"], inputs["k_cpu"], inputs["v_cpu"], inputs["mask"], inputs["window"]
    B, S, Hq, _ = q.shape
    rng = np.random.default_rng(rng_seed)
    flops = 0.0
    elapsed = 0.0
    blocks = 0
    while elapsed < seconds:
        b = int(rng.integers(B))
        p0 = int(rng.integers(0, S // 256)) * 256
        m = mask[b, p0:p0 + 256]
        pos = np.arange(p0, p0 + 256)
        t0 = time.perf_counter()
        for is_local, sel in ((False, m), (True, ~m)):
            if sel.any():
                oracle_attn.prefill_rows(q, k, v, b, pos[sel], is_local, window=W)
        elapsed += time.perf_counter() - t0
        keys = workloads.legal_keys_per_row(mask[b:b + 1, :], W, S)[0, p0:p0 + 256]
        flops += 4.0 * 128 * Hq * float(keys.sum())
        blocks += 1
    return {"value": flops / elapsed / 1e12, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{blocks} random 256-position blocks of config 3 (all {Hq} heads), "
                      f"{elapsed:.1f} s of FP32 torch on the host"}


def make_cpu_inputs(seed_offset: int = 0):
    w = workloads.make_inputs(CONFIG_ID, device="cpu")
    return {"q_cpu": w["q"], "k_cpu": w["k"], "v_cpu": w["v"], "mask": w["mask"].numpy(), "window": w["window"]}


def run_reference(args, world, rank):
    if rank != 0:
        return 0
    inputs = make_cpu_inputs()
    per_step = max(1.0, 60.0 / max(1, args.steps + args.warmup))
    for _ in range(args.warmup):
        cpu_oracle_sample(inputs, per_step / 4, rng_seed=7)
    samples = []
    for s in range(args.steps):
        res = cpu_oracle_sample(inputs, per_step, rng_seed=1000 + s)
        samples.append(res)
    value = statistics.fmean([r["value"] for r in samples])
    flops = workloads.effective_flops(inputs["mask"], inputs["window"], inputs["q_cpu"].shape[1],
                                      inputs["q_cpu"].shape[2])
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup,
        # one whole config-3 batch at the sampled rate (each step times a bounded sample)
        "ms_per_step": flops / (value * 1e12) * 1e3, "sample_seconds_per_step": per_step,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config3_dict(args.gpus),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": samples[0]["cores"], "kind": "port",
                         "sample": f"each step: {samples[0]['sample']}"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference kernels are TileLang programs that lower only for Hopper (T.wgmma_gemm); the "
                "reference path is timed as its CPU restatement (oracle/) on one host, whatever N is",
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------- GPU arm
def run_backward(args, world, rank, local_rank):
    """Prefill backward of the config-3 workload (``--batch`` sequences per GPU).

    One step = dQ, dK, dV from the forward's O and LSE for a random upstream
    gradient (pack pass, dQ pass, dK/dV pass).  ``value`` uses the usual
    convention of 2.5 x the forward's effective FLOP (five matrix products of
    the forward's size, over the legal entries only).
    """
    from switchattentionkernels_b200 import _core, build_switch_query_indices_batched
    from switchattentionkernels_b200.backward import switch_gqa_prefill_backward

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    w = workloads.make_inputs(CONFIG_ID, device=dev, on_device=True, seed_offset=1000 * rank,
                              batch_override=args.batch)
    cfg = w["cfg"]
    q, k, v, mask, W = w["q"], w["k"], w["v"], w["mask"], w["window"]
    full, local, counts = build_switch_query_indices_batched(mask.to(dev))
    out, lse = _core.forward(q, k, v, full, local, window_size=W, query_counts=counts)
    g = torch.Generator(device=dev).manual_seed(5 + rank)
    dout = torch.randn(out.shape, generator=g, device=dev).bfloat16()
    flops = 2.5 * workloads.effective_flops(mask.numpy(), W, q.shape[1], q.shape[2])

    def step():
        switch_gqa_prefill_backward(q, k, v, out, lse, dout, full, local, window_size=W, query_counts=counts)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    clocks = ClockSampler(dev.index)
    clocks.start()
    clocks.mark("begin")
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    clocks.mark("end")
    clock_info = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.destroy_process_group()
    if rank == 0:
        peak_burst, _, peak_src = measured_peaks()
        value = flops * world / (ms * 1e-3) / 1e12
        print(json.dumps({
            "metric": "prefill backward: effective TFLOP/s (2.5 x forward, unmasked entries)", "value": value,
            "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": cfg.name, "B_per_gpu": q.shape[0], "effective_tflop_per_step": flops / 1e12},
            "roofline": {"bound": "tensor", "achieved": value / world, "peak": peak_burst, "unit": UNIT,
                         "frac": value / world / peak_burst, "peak_source": f"{peak_src} bf16_tflops (burst)"},
            "gpu_launches": 3 * args.steps,  # rowsum, dQ pass, dK/dV pass per step
            "clocks": clock_info,
        }), flush=True)
    return 0


DECODE_B, DECODE_SMAX, DECODE_HQ, DECODE_HKV, DECODE_W, DECODE_P = 64, 32768, 32, 8, 1024, 0.125


def hbm_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            hbm = float(json.load(fh).get("hbm_gbs", 0.0))
        if hbm > 0:
            return hbm, "measured hbm_gbs"
    return 6650.0, "fallback"


def make_decode_batch(dev, seed):
    """The decode step's batch: 64 sequences with 16K-32K cached keys each, Hq 32 /
    Hkv 8, each new token routed full with p = 0.125; returns q, k, v, lens, route
    and the legal K/V bytes one step reads."""
    B, Smax, Hq, Hkv, W, p_full = DECODE_B, DECODE_SMAX, DECODE_HQ, DECODE_HKV, DECODE_W, DECODE_P
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn((B, Hq, 128), generator=g, device=dev).bfloat16()
    k = torch.randn((B, Smax, Hkv, 128), generator=g, device=dev).bfloat16()
    v = torch.randn((B, Smax, Hkv, 128), generator=g, device=dev).bfloat16()
    lens = torch.randint(Smax // 2, Smax + 1, (B,), generator=g, device=dev, dtype=torch.int32)
    route = torch.rand((B,), generator=g, device=dev) < p_full
    L = lens.cpu().numpy().astype(np.int64)
    keys = np.where(route.cpu().numpy(), L, np.minimum(L, W))
    kv_bytes = float(keys.sum()) * Hkv * 128 * 2 * 2
    return q, k, v, lens, route, kv_bytes


def time_steps(fn, steps, stream=None):
    """Average milliseconds of ``fn`` over ``steps`` back-to-back calls (CUDA events)."""
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        fn()
    t1.record(stream)
    torch.cuda.synchronize()
    return t0.elapsed_time(t1) / steps


def run_decode(args, world, rank, local_rank):
    """Decode step of the config-3 model shape: 64 sequences with 16K-32K cached
    keys each, Hq 32 / Hkv 8, W 1024, each new token routed full with p = 0.125.

    HBM-bound: ``value`` = legal K/V bytes read per step / step time (GB/s),
    against the measured copy bandwidth; ``tokens_per_s`` = sequences / step
    time.  With N ranks every rank runs its own batch (weak scaling).
    """
    from switchattentionkernels_b200.decode import switch_gqa_decode_forward

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    B, W = DECODE_B, DECODE_W
    q, k, v, lens, route, kv_bytes = make_decode_batch(dev, 11 + rank)
    for _ in range(args.warmup):
        switch_gqa_decode_forward(q, k, v, lens, route, window_size=W)
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    clocks = ClockSampler(dev.index)
    clocks.start()
    clocks.mark("begin")
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        switch_gqa_decode_forward(q, k, v, lens, route, window_size=W)
    t1.record()
    torch.cuda.synchronize()
    clocks.mark("end")
    clock_info = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.destroy_process_group()
    if rank == 0:
        peak, hbm_src = hbm_peak()
        gbs = kv_bytes * world / (ms * 1e-3) / 1e9
        print(json.dumps({
            "metric": "decode step: legal K/V bytes read per second", "value": gbs, "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "tokens_per_s": B * world / (ms * 1e-3),
            "config": {"workload": "decode: 64 sequences, 16K-32K cached keys, Hq 32, Hkv 8, W 1024, p_full 0.125",
                       "kv_bytes_per_step": kv_bytes},
            "roofline": {"bound": "hbm", "achieved": gbs / world, "peak": peak, "unit": "GB/s",
                         "frac": gbs / world / peak, "peak_source": hbm_src},
            "gpu_launches": 2 * args.steps,  # split-KV kernel + merge per step
            "clocks": clock_info,
        }), flush=True)
    return 0


def run_cp(args, world, rank, local_rank):
    """Context-parallel prefill of one packed batch over ``world`` ranks.

    Workload: config 4 (16 packed sequences) or, with ``--cp-config 5``, the first
    131072-token sequence of config 5.

    Every rank draws the same batch and keeps only its rows of Q, K and V (zigzag
    chunks of equal legal-entry cost, ``context_parallel.make_cp_plan``).  One
    step is the public context-parallel forward (one attention layer): the K/V
    exchange (``KVExchange``: peer stores into every rank's symmetric-memory
    buffer) and the prefill kernel on the rank's rows.  The rows' key bounds
    depend only on the batch and are built once, before the steps.  ``value`` =
    effective FLOP of the whole batch / the slowest rank's step time (strong
    scaling: the batch is fixed as N grows); at N > 1 ``kv_exchange_nccl`` is the
    same step with the NCCL all-gather instead, and ``kv_exchange`` times the two
    exchanges alone.
    """
    import torch.distributed as dist
    from switchattentionkernels_b200 import context_parallel as cp

    cfg_id = args.cp_config
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    w = workloads.make_inputs(cfg_id, device=dev, on_device=True)
    cfg = w["cfg"]
    q, k, v, mask, W, cu = w["q"][:1], w["k"][:1], w["v"][:1], w["mask"][0].numpy(), w["window"], w["cu_seqlens"]
    if cu is None:
        cu = torch.tensor([0, q.shape[1]], dtype=torch.int32)
    S, Hq, Hkv = q.shape[1], q.shape[2], k.shape[2]
    flops_total = workloads.effective_flops(mask[None, :], W, S, Hq, cu_seqlens=cu.numpy())
    if world == 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(29700 + os.getpid() % 200))
        dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    plan = cp.make_cp_plan(S, world, cp.cp_row_costs(mask, W, cu.numpy()))
    rows = plan.rows(rank)
    idx = torch.from_numpy(rows).to(dev)
    ql, kl, vl = (t.index_select(1, idx).contiguous() for t in (q, k, v))
    del q, k, v
    lm = mask[rows]
    fl = torch.from_numpy(np.nonzero(lm)[0]).to(device=dev, dtype=torch.int32)
    ll = torch.from_numpy(np.nonzero(~lm)[0]).to(device=dev, dtype=torch.int32)

    md = cp.cp_metadata(S, rows, device=dev, window_size=W, cu_seqlens=cu)

    # K/V exchange: symmetric memory and peer stores (one rank: nothing to exchange)
    kvx = cp.KVExchange(S, Hkv, device=dev) if world > 1 else None

    def step(exchange=kvx):
        cp.context_parallel_switch_gqa_prefill_forward(ql, kl, vl, fl, ll, total_len=S, cu_seqlens=cu,
                                                       window_size=W, validate=False, plan=plan, metadata=md,
                                                       kv_exchange=exchange)

    def timed(fn, n):
        torch.cuda.synchronize()
        dist.barrier()
        a = torch.cuda.Event(enable_timing=True)
        z = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n):
            fn()
        z.record()
        torch.cuda.synchronize()
        t = torch.tensor([a.elapsed_time(z) / n], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    extra = {}
    if kvx is not None:
        # the same step with the NCCL all-gather + reorder, and each exchange alone
        for _ in range(2):
            step(None)
        extra["kv_exchange_nccl"] = {"ms_per_step": timed(lambda: step(None), args.steps)}
        extra["kv_exchange_nccl"]["value"] = flops_total / (extra["kv_exchange_nccl"]["ms_per_step"] * 1e-3) / 1e12
        sent = 2 * kl.numel() * kl.element_size() * (world - 1)  # this rank's K and V to every peer
        ex_ms = timed(lambda: kvx.exchange(kl, vl, plan), args.steps)
        nc_ms = timed(lambda: cp.cp_gather_kv(kl, vl, plan), args.steps)
        extra["kv_exchange"] = {"what": "every rank stores its K/V chunks into every rank's symmetric-memory "
                                        "buffer (one copy kernel per chunk, plain peer stores), between two "
                                        "device barriers",
                                "ms": ex_ms, "bytes_to_peers_rank0": sent, "gbs_per_rank": sent / (ex_ms * 1e6),
                                "nccl_all_gather_and_reorder_ms": nc_ms,
                                "reference_nvlink_peer_copy_gbs": 770.0}

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    clocks = ClockSampler(dev.index)
    clocks.start()
    clocks.mark("begin")
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    clocks.mark("end")
    dist.barrier()
    clock_info = clocks.stop()
    ms = torch.tensor([t0.elapsed_time(t1) / args.steps], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms_max = float(ms.item())
    if world == 1:
        dist.destroy_process_group()
    if rank == 0:
        peak_burst, _, peak_src = measured_peaks()
        value = flops_total / (ms_max * 1e-3) / 1e12
        print(json.dumps({
            "metric": "effective TFLOP/s, context-parallel varlen prefill", "value": value, "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": cfg.name, "tokens": S, "sequences": int(cu.numel() - 1), "Hq": Hq, "Hkv": Hkv,
                       "window": W, "p_full": cfg.p_full,
                       "parallelism": f"context parallel over {world} ranks: cost-balanced zigzag rows, "
                                      + ("K/V exchanged by peer stores through symmetric memory" if world > 1
                                         else "no exchange"),
                       "rows_per_rank_max": plan.capacity,
                       "effective_tflop_per_step": flops_total / 1e12},
            "pct_of_bf16_peak_per_gpu": 100.0 * value / world / peak_burst, "peak_source": peak_src,
            # the prefill kernel, plus at N > 1 four exchange copy kernels (two chunks of K and V), per step
            "gpu_launches": args.steps * (5 if world > 1 else 1),
            "clocks": clock_info,
            **extra,
        }), flush=True)
    return 0


def run_replicas(args, world, rank, local_rank):
    """Weak scaling: every rank draws its own 4 sequences (seed offset by rank) and
    computes all of their (batch, KV group) units; no collective."""
    from switchattentionkernels_b200 import _core, build_switch_query_indices_batched, switch_gqa_prefill_forward

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    cfg = workloads.CONFIGS[CONFIG_ID]
    # each rank draws its own 4 sequences of the global batch (seed offset by rank)
    w = workloads.make_inputs(CONFIG_ID, device=dev, on_device=True, seed_offset=1000 * rank,
                              batch_override=args.batch)
    q, k, v, mask_cpu, W = w["q"], w["k"], w["v"], w["mask"], w["window"]
    B, S, Hq, D = q.shape
    mask_np = mask_cpu.numpy()
    mask_dev = mask_cpu.to(dev)
    flops_rank = unit_flops(mask_np, W, Hq, S)
    out = torch.empty_like(q)
    lse = torch.empty(q.shape[:3], dtype=torch.float32, device=dev)

    stream = torch.cuda.current_stream(dev)
    pf_events = []

    def step(record=False):
        full, local, counts = build_switch_query_indices_batched(mask_dev)
        ev = None
        if record:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            pf_events.append(ev)
        _core.forward(q, k, v, full, local, window_size=W, validate=False, query_counts=counts, out=out, lse=lse,
                      prefill_events=ev)

    launches_per_step = 3  # mask compaction (two launches for rows over 4096 tokens) + prefill kernel
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    clocks = ClockSampler(dev.index)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    clocks.mark("begin")
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        step(record=True)
    t1.record(stream)
    torch.cuda.synchronize()
    clocks.mark("end")
    barrier()
    clock_info = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    pf_ms = [a.elapsed_time(b) for a, b in pf_events]
    pf_avg = statistics.fmean(pf_ms)

    # e2e through the public API from pinned host buffers.  Every step copies its
    # inputs host->device, runs compaction + the (validating) public forward, and
    # copies O and LSE back; the steps are pipelined over three streams (copy in,
    # compute, copy out, two device slots), as a serving loop would run them, so the
    # copies of neighbouring steps overlap the compute of this one.
    e2e = None
    if not args.no_e2e:
        hq = q.cpu().pin_memory()
        hk = k.cpu().pin_memory()
        hv = v.cpu().pin_memory()
        hm = mask_cpu.pin_memory()
        ho = torch.empty(out.shape, dtype=out.dtype).pin_memory()
        hl = torch.empty(lse.shape, dtype=lse.dtype).pin_memory()
        s_in = torch.cuda.Stream(dev)
        s_out = torch.cuda.Stream(dev)
        slots = [(torch.empty_like(q), torch.empty_like(k), torch.empty_like(v),
                  torch.empty(hm.shape, dtype=hm.dtype, device=dev)) for _ in range(2)]

        def e2e_run(n):
            in_done = [torch.cuda.Event() for _ in range(n)]
            comp_done = [torch.cuda.Event() for _ in range(n)]

            def copy_in(i):
                with torch.cuda.stream(s_in):
                    if i >= 2:
                        s_in.wait_event(comp_done[i - 2])  # slot i % 2 no longer read
                    dq, dk, dv, dm = slots[i % 2]
                    dq.copy_(hq, non_blocking=True)
                    dk.copy_(hk, non_blocking=True)
                    dv.copy_(hv, non_blocking=True)
                    dm.copy_(hm, non_blocking=True)
                    in_done[i].record(s_in)

            copy_in(0)
            for i in range(n):
                if i + 1 < n:
                    copy_in(i + 1)
                stream.wait_event(in_done[i])
                dq, dk, dv, dm = slots[i % 2]
                full, local, cnt = build_switch_query_indices_batched(dm)
                o, l_ = switch_gqa_prefill_forward(dq, dk, dv, full, local, window_size=W, query_counts=cnt)
                comp_done[i].record(stream)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(comp_done[i])
                    o.record_stream(s_out)
                    l_.record_stream(s_out)
                    ho.copy_(o, non_blocking=True)
                    hl.copy_(l_, non_blocking=True)

        e2e_run(min(2, args.warmup) + 1)
        torch.cuda.synchronize()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        s_in.wait_event(e0)
        e2e_run(args.steps)
        e1.record(s_out)
        torch.cuda.synchronize()
        barrier()
        e2e_ms = e0.elapsed_time(e1) / args.steps
        h2d = hq.numel() * 2 + hk.numel() * 2 + hv.numel() * 2 + hm.numel()
        d2h = ho.numel() * 2 + hl.numel() * 4
        e2e = {"ms": e2e_ms, "h2d": h2d, "d2h": d2h}

    # max over ranks / sums over ranks
    vals = torch.tensor([ms, pf_avg, flops_rank, e2e["ms"] if e2e else 0.0], dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as dist
        mx = vals.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = vals.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        ms_max, pf_max, flops_total, e2e_ms_max = mx[0].item(), mx[1].item(), sm[2].item(), mx[3].item()
    else:
        ms_max, pf_max, flops_total, e2e_ms_max = ms, pf_avg, flops_rank, (e2e["ms"] if e2e else 0.0)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # rank 0 at N=1 only: the CPU restatement on a bounded sample of the same workload
        cpu_inputs = {"q_cpu": q.cpu(), "k_cpu": k.cpu(), "v_cpu": v.cpu(), "mask": mask_np, "window": W}
        cpu = cpu_oracle_sample(cpu_inputs, args.cpu_seconds)

    if rank == 0:
        peak_burst, peak_sustained, peak_src = measured_peaks()
        achieved = flops_rank / (pf_avg * 1e-3) / 1e12
        traffic = profile_traffic(cfg.name)
        value = flops_total / (ms_max * 1e-3) / 1e12
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "weak",
            "mode": "replicas",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": cfg.name, "B_per_gpu": B, "S": S, "Hq": Hq, "Hkv": k.shape[2], "head_dim": D,
                       "window": W, "p_full": cfg.p_full, "routing": "markov(switch=0.02)",
                       "parallelism": f"(batch, kv-group) units, {B} sequences per GPU",
                       "l2": "inputs larger than L2 (q/k/v 1.5 GiB per GPU)",
                       "effective_tflop_per_step": flops_total / 1e12},
            "pct_of_bf16_peak": 100.0 * value / world / peak_burst,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_burst, "unit": UNIT,
                         "frac": achieved / peak_burst, "traffic": traffic,
                         "kernel": "switch_prefill_kernel", "kernel_ms": pf_avg,
                         "peak_source": f"{peak_src} bf16_tflops (burst)",
                         "frac_of_sustained": achieved / peak_sustained},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clock_info,
        }
        if e2e is not None:
            line["e2e"] = {"value": flops_total / (e2e_ms_max * 1e-3) / 1e12, "unit": UNIT,
                           "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                           "ms_per_step": e2e_ms_max}
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def run_default(args, world, rank, local_rank):
    """Config 3's (batch, KV group) units sharded over the ranks (see the module docstring)."""
    import math

    import torch.distributed as dist
    from switchattentionkernels_b200 import (_core, build_switch_query_indices_batched, sharded,
                                             switch_gqa_prefill_forward)

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    multi = world > 1
    K, WU = args.steps, args.warmup

    def barrier():
        if multi:
            dist.barrier()

    def reduce(vals, op):
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        if multi:
            dist.all_reduce(t, op=op)
        return t.tolist()

    # every rank draws the same batch and keeps its own units
    w = workloads.make_inputs(args.workload, device=dev, on_device=True, p_full=args.p_full)
    q, k, v, mask_cpu, W = w["q"], w["k"], w["v"], w["mask"], w["window"]
    B, S, Hq, D = q.shape
    Hkv = k.shape[2]
    r = Hq // Hkv
    mask_np = mask_cpu.numpy()
    fl = [np.nonzero(m)[0] for m in mask_np]
    ll = [np.nonzero(~m)[0] for m in mask_np]
    costs = sharded.unit_costs(fl, ll, hkv=Hkv, skv=S, window=W)
    plan = sharded.plan_units(costs, world)
    mine = plan[rank]
    n, n_max = len(mine), max(len(p) for p in plan)
    flops_total = workloads.effective_flops(mask_np, W, S, Hq)
    flops_rank = 4.0 * D * r * float(sum(costs[u] for u in mine))
    q_u = sharded.take_units(q, mine, hkv=Hkv)
    k_u = sharded.take_units(k, mine, hkv=Hkv)
    v_u = sharded.take_units(v, mine, hkv=Hkv)
    mask_u_cpu = mask_cpu[torch.tensor([u // Hkv for u in mine], dtype=torch.long)].contiguous()
    mask_u = mask_u_cpu.to(dev)
    # the rank's largest per-unit counts, known on the host: the launch's key-split plan
    # (long full-causal units over several SMs) needs them and the step reads none back
    unit_counts = ((int(mask_u_cpu.sum(1).max()), int((~mask_u_cpu).sum(1).max())) if n else (0, 0))
    split_tiles = _core.split_plan(n, S, r, 1, unit_counts[0], unit_counts[1], W, dev)[0] if n else 0
    o_u = torch.empty((n_max, S, r, D), dtype=torch.bfloat16, device=dev)
    l_u = torch.empty((n_max, S, r), dtype=torch.float32, device=dev)
    if multi:
        del q, k, v
    torch.cuda.synchronize()

    stream = torch.cuda.current_stream(dev)
    pf_events = []

    def step(record=False):
        if n == 0:
            return
        full, local, counts = build_switch_query_indices_batched(mask_u)
        ev = None
        if record:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            pf_events.append(ev)
        _core.forward(q_u, k_u, v_u, full, local, window_size=W, validate=False, query_counts=counts,
                      out=o_u[:n], lse=l_u[:n], prefill_events=ev, max_counts=unit_counts)

    # mask compaction (two launches: rows over 4096 tokens) + the prefill kernel (+ the
    # merge of key-split pieces)
    launches_per_step = 3 + (1 if split_tiles else 0)
    for _ in range(WU):
        step()
    torch.cuda.synchronize()
    barrier()
    clocks = ClockSampler(dev.index)
    clocks.start()
    clocks.mark("begin")
    ms = time_steps(lambda: step(record=True), K, stream)
    clocks.mark("end")
    barrier()
    clock_info = clocks.stop()
    pf_avg = statistics.fmean([a.elapsed_time(b) for a, b in pf_events]) if pf_events else 0.0

    # the same step with a replicated result, fused: the kernel's epilogue writes every
    # row into every rank's row-major buffer (symmetric memory, over NVLink)
    rep = sharded.ReplicaBuffers(B, S, Hq, device=dev)
    f_events = []

    def step_fused(record=False):
        if n == 0:
            rep.barrier()
            rep.barrier()
            return
        full, local, counts = build_switch_query_indices_batched(mask_u)
        e = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) if record else None
        rep.barrier()  # nobody still reads the buffers' previous contents
        if e:
            e[0].record(stream)
        sharded.forward_units_replicated(q_u, k_u, v_u, full, local, counts, mine, rep, hkv=Hkv, window_size=W,
                                         barrier=False)
        if e:
            e[1].record(stream)
            f_events.append(e)
        rep.barrier()  # every rank's rows have landed everywhere

    for _ in range(2):
        step_fused()
    torch.cuda.synchronize()
    barrier()
    fu_ms = time_steps(lambda: step_fused(record=True), K, stream)
    barrier()
    fu_kernel = statistics.fmean([a.elapsed_time(b) for a, b in f_events]) if f_events else 0.0
    del rep

    # the same with the replication after the launch: NCCL all-gather of every rank's
    # unit-major O / LSE + the scatter kernel
    out_all = torch.empty((B, S, Hq, D), dtype=torch.bfloat16, device=dev)
    lse_all = torch.empty((B, S, Hq), dtype=torch.float32, device=dev)
    gbufs = {}
    g_events = []

    def step_gather(record=False):
        step()
        e = [torch.cuda.Event(enable_timing=True) for _ in range(3)] if record else None
        if e:
            e[0].record(stream)
        got_o, got_l = sharded.all_gather_units(o_u, l_u, plan, bufs=gbufs)
        if e:
            e[1].record(stream)
        sharded.scatter_gathered(got_o, got_l, plan, hkv=Hkv, out=out_all, lse=lse_all)
        if e:
            e[2].record(stream)
            g_events.append(e)

    for _ in range(2):
        step_gather()
    torch.cuda.synchronize()
    barrier()
    g_ms = time_steps(lambda: step_gather(record=True), K, stream)
    barrier()
    coll_ms = statistics.fmean([a.elapsed_time(b) for a, b, _ in g_events])
    scat_ms = statistics.fmean([b.elapsed_time(c) for _, b, c in g_events])
    del gbufs

    # steady state: back-to-back steps for at least --steady-seconds, own clock record
    ms_max0 = reduce([ms], dist.ReduceOp.MAX)[0] if multi else ms
    n_steady = max(K, int(math.ceil(args.steady_seconds * 1000.0 / max(ms_max0, 1e-3))))
    barrier()
    torch.cuda.synchronize()
    clocks2 = ClockSampler(dev.index)
    clocks2.start()
    clocks2.mark("begin")
    st_ms = time_steps(step, n_steady, stream)
    clocks2.mark("end")
    barrier()
    steady_clocks = clocks2.stop()

    # e2e through the public API from pinned host buffers (the rank's own units)
    e2e = None
    if not args.no_e2e:
        hq, hk, hv = (t.cpu().pin_memory() for t in (q_u, k_u, v_u))
        hm = mask_u_cpu.pin_memory()
        ho = torch.empty((n, S, r, D), dtype=torch.bfloat16).pin_memory()
        hl = torch.empty((n, S, r), dtype=torch.float32).pin_memory()
        s_in = torch.cuda.Stream(dev)
        s_out = torch.cuda.Stream(dev)
        slots = [(torch.empty_like(q_u), torch.empty_like(k_u), torch.empty_like(v_u),
                  torch.empty(hm.shape, dtype=hm.dtype, device=dev)) for _ in range(2)]

        def e2e_run(count):
            if n == 0:
                return
            in_done = [torch.cuda.Event() for _ in range(count)]
            comp_done = [torch.cuda.Event() for _ in range(count)]

            def copy_in(i):
                with torch.cuda.stream(s_in):
                    if i >= 2:
                        s_in.wait_event(comp_done[i - 2])  # slot i % 2 no longer read
                    dq, dk, dv, dm = slots[i % 2]
                    dq.copy_(hq, non_blocking=True)
                    dk.copy_(hk, non_blocking=True)
                    dv.copy_(hv, non_blocking=True)
                    dm.copy_(hm, non_blocking=True)
                    in_done[i].record(s_in)

            copy_in(0)
            for i in range(count):
                if i + 1 < count:
                    copy_in(i + 1)
                stream.wait_event(in_done[i])
                dq, dk, dv, dm = slots[i % 2]
                full, local, cnt = build_switch_query_indices_batched(dm)
                o, l_ = switch_gqa_prefill_forward(dq, dk, dv, full, local, window_size=W, query_counts=cnt)
                comp_done[i].record(stream)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(comp_done[i])
                    o.record_stream(s_out)
                    l_.record_stream(s_out)
                    ho.copy_(o, non_blocking=True)
                    hl.copy_(l_, non_blocking=True)

        e2e_run(min(2, WU) + 1)
        torch.cuda.synchronize()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        s_in.wait_event(e0)
        e2e_run(K)
        e1.record(s_out)
        torch.cuda.synchronize()
        barrier()
        e2e = {"ms": e0.elapsed_time(e1) / K,
               "h2d": (hq.numel() + hk.numel() + hv.numel()) * 2 + hm.numel(),
               "d2h": ho.numel() * 2 + hl.numel() * 4}

    # N = 1 extras: the row-major layout of the single-GPU API, one backward and one decode step
    extras = {}
    if not multi and not args.no_extras and args.workload == CONFIG_ID:
        from switchattentionkernels_b200.backward import switch_gqa_prefill_backward
        from switchattentionkernels_b200.decode import switch_gqa_decode_forward

        mask_dev = mask_cpu.to(dev)
        full, local, counts = build_switch_query_indices_batched(mask_dev)
        out = torch.empty_like(q)
        lse = torch.empty((B, S, Hq), dtype=torch.float32, device=dev)
        std_events = []

        def step_std():
            f, l_, c = build_switch_query_indices_batched(mask_dev)
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            std_events.append(ev)
            _core.forward(q, k, v, f, l_, window_size=W, validate=False, query_counts=c, out=out, lse=lse,
                          prefill_events=ev)

        for _ in range(WU):
            step_std()
        torch.cuda.synchronize()
        std_events.clear()
        std_ms = time_steps(step_std, K, stream)
        std_k = statistics.fmean([a.elapsed_time(b) for a, b in std_events])
        extras["standard_layout"] = {"value": flops_total / (std_ms * 1e-3) / 1e12, "unit": UNIT,
                                     "ms_per_step": std_ms, "kernel_ms": std_k,
                                     "layout": "q [B, S, Hq, 128], k / v [B, S, Hkv, 128] (the single-GPU API)"}
        peak_burst, _, peak_src = measured_peaks()
        g = torch.Generator(device=dev).manual_seed(5)
        dout = torch.randn(out.shape, generator=g, device=dev).bfloat16()

        def step_bwd():
            switch_gqa_prefill_backward(q, k, v, out, lse, dout, full, local, window_size=W, query_counts=counts)

        for _ in range(2):
            step_bwd()
        torch.cuda.synchronize()
        nb = max(3, K // 4)
        b_ms = time_steps(step_bwd, nb, stream)
        bval = 2.5 * flops_total / (b_ms * 1e-3) / 1e12
        extras["backward"] = {
            "metric": "prefill backward (dQ, dK, dV): effective TFLOP/s, 2.5 x the forward's legal-entry FLOP",
            "value": bval, "unit": UNIT, "ms_per_step": b_ms, "steps": nb,
            "roofline": {"bound": "tensor", "achieved": bval, "peak": peak_burst, "unit": UNIT,
                         "frac": bval / peak_burst, "peak_source": f"{peak_src} bf16_tflops (burst)"},
            "gpu_launches_per_step": 3}
        del dout
        dq_, dk_, dv_, dl, dr, kv_bytes = make_decode_batch(dev, 11)

        def step_dec():
            switch_gqa_decode_forward(dq_, dk_, dv_, dl, dr, window_size=DECODE_W)

        for _ in range(2):
            step_dec()
        torch.cuda.synchronize()
        nd = max(5, K // 2)
        d_ms = time_steps(step_dec, nd, stream)
        gbs = kv_bytes / (d_ms * 1e-3) / 1e9
        hpk, hsrc = hbm_peak()
        extras["decode"] = {
            "metric": "decode step (one new token per sequence): legal K/V bytes read per second",
            "value": gbs, "unit": "GB/s", "ms_per_step": d_ms, "steps": nd,
            "tokens_per_s": DECODE_B / (d_ms * 1e-3),
            "workload": f"{DECODE_B} sequences, 16K-32K cached keys, Hq {DECODE_HQ}, Hkv {DECODE_HKV}, "
                        f"W {DECODE_W}, p_full {DECODE_P}",
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hpk, "unit": "GB/s", "frac": gbs / hpk,
                         "peak_source": hsrc},
            "gpu_launches_per_step": 2}
        # the same batch with an FP8 e4m3 cache, per-(sequence, KV head) scales
        ks_ = dk_.float().abs().amax(dim=(1, 3)) / 448.0
        vs_ = dv_.float().abs().amax(dim=(1, 3)) / 448.0
        dk8 = (dk_.float() / ks_[:, None, :, None]).to(torch.float8_e4m3fn)
        dv8 = (dv_.float() / vs_[:, None, :, None]).to(torch.float8_e4m3fn)
        del dk_, dv_

        def step_dec8():
            switch_gqa_decode_forward(dq_, dk8, dv8, dl, dr, window_size=DECODE_W, k_scale=ks_, v_scale=vs_)

        for _ in range(2):
            step_dec8()
        torch.cuda.synchronize()
        d8_ms = time_steps(step_dec8, nd, stream)
        gbs8 = kv_bytes / 2 / (d8_ms * 1e-3) / 1e9
        extras["decode_fp8"] = {
            "metric": "decode step over an FP8 e4m3 KV cache: legal K/V bytes read per second",
            "value": gbs8, "unit": "GB/s", "ms_per_step": d8_ms, "steps": nd,
            "tokens_per_s": DECODE_B / (d8_ms * 1e-3), "speedup_vs_bf16_cache": d_ms / d8_ms,
            "workload": "the decode batch above, K/V quantised per (sequence, KV head)",
            "roofline": {"bound": "hbm", "achieved": gbs8, "peak": hpk, "unit": "GB/s", "frac": gbs8 / hpk,
                         "peak_source": hsrc},
            "gpu_launches_per_step": 2}
        del dq_, dk8, dv8

    e2e_ms = e2e["ms"] if e2e else 0.0
    mx = reduce([ms, g_ms, coll_ms, scat_ms, st_ms, e2e_ms, pf_avg, fu_ms, fu_kernel], dist.ReduceOp.MAX)
    sm = reduce([flops_rank, pf_avg, float(e2e["h2d"] if e2e else 0), float(e2e["d2h"] if e2e else 0)],
                dist.ReduceOp.SUM)
    ms_max, g_ms_max, coll_max, scat_max, st_max, e2e_max, pf_max, fu_max, fu_kernel_max = mx
    flops_sum, pf_sum, h2d_sum, d2h_sum = sm

    cpu = None
    if rank == 0 and not multi and not args.no_cpu_baseline and args.workload == CONFIG_ID:
        # rank 0 at N=1 only: the CPU restatement on a bounded sample of the same workload
        cpu_inputs = {"q_cpu": q.cpu(), "k_cpu": k.cpu(), "v_cpu": v.cpu(), "mask": mask_np, "window": W}
        cpu = cpu_oracle_sample(cpu_inputs, args.cpu_seconds)

    if rank == 0:
        peak_burst, peak_sustained, peak_src = measured_peaks()
        value = flops_total / (ms_max * 1e-3) / 1e12
        achieved = flops_sum / (pf_sum * 1e-3) / 1e12 if pf_sum > 0 else 0.0
        recv = (world - 1) * n_max * S * r * (D * 2 + 4)
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": WU,
            "ms_per_step": ms_max, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic", "config": config3_dict(world, args.workload, w["p_full"]),
            "units_per_rank": [len(p) for p in plan],
            "key_split_tiles_rank0": split_tiles,
            "layout": "each rank holds its units unit-major: q [units, S, Hq/Hkv, 128], k / v [units, S, 1, 128]",
            "effective_tflop_per_step": flops_total / 1e12,
            "pct_of_bf16_peak_per_gpu": 100.0 * value / world / peak_burst,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_burst, "unit": UNIT,
                         "frac": achieved / peak_burst, "traffic": profile_traffic(config3_dict(1)["workload"]) if args.workload == CONFIG_ID else None,
                         "kernel": "switch_prefill_kernel", "kernel_ms": pf_max,
                         "peak_source": f"{peak_src} bf16_tflops (burst)",
                         "frac_of_sustained": achieved / peak_sustained},
            "gather": {"value": flops_total / (fu_max * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": fu_max,
                       "kernel_ms": fu_kernel_max,
                       "bytes_to_peers_rank0": (world - 1) * n * S * r * (D * 2 + 4),
                       "what": "replicated result: the prefill epilogue stores every O/LSE row into every rank's "
                               "row-major buffer (symmetric memory, peer stores over NVLink) during the "
                               "attention itself; a device barrier of all ranks before and after each step"},
            "gather_nccl": {"value": flops_total / (g_ms_max * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": g_ms_max,
                       "all_gather_ms": coll_max, "scatter_ms": scat_max,
                       "bytes_received_per_rank": recv,
                       "all_gather_gbs_per_rank": recv / (coll_max * 1e-3) / 1e9 if recv and coll_max > 0 else None,
                       "reference_nvlink_peer_copy_gbs": 770.0,
                       "what": "every step ends with NCCL all_gather_into_tensor of every rank's unit-major O and "
                               "LSE and the scatter kernel into [B, S, Hq, ...] on every rank"},
            "steady": {"value": flops_total / (st_max * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": st_max,
                       "steps": n_steady, "clocks": steady_clocks,
                       "mcycles_per_step": (st_max * 1e-3 * steady_clocks["sm_mhz"] * 1e6 / 1e6
                                            if steady_clocks else None)},
            "gpu_launches": launches_per_step * K,  # rank 0: compaction (2) + prefill (+ merge), every step
            "clocks": clock_info,
        }
        if e2e is not None:
            line["e2e"] = {"value": flops_total / (e2e_max * 1e-3) / 1e12, "unit": UNIT,
                           "h2d_bytes_per_step": int(h2d_sum), "d2h_bytes_per_step": int(d2h_sum),
                           "ms_per_step": e2e_max,
                           "what": "every step: the rank's own units' q/k/v/mask host->device, compaction + "
                                   "validating public forward, its O/LSE device->host (bytes summed over ranks)"}
        if cpu is not None:
            line["cpu_baseline"] = cpu
        line.update(extras)
        print(json.dumps(line), flush=True)
    return 0

def main():
    args = parse_args()
    world, rank, local_rank = dist_env()
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.impl == "reference":
            return run_reference(args, world, rank)
        if args.decode:
            return run_decode(args, world, rank, local_rank)
        if args.backward:
            return run_backward(args, world, rank, local_rank)
        if args.cp:
            return run_cp(args, world, rank, local_rank)
        if args.replicas:
            return run_replicas(args, world, rank, local_rank)
        if args.p_sweep:
            for pv in args.p_sweep.split(","):
                args.p_full = float(pv)
                run_default(args, world, rank, local_rank)
                torch.cuda.empty_cache()
            return 0
        return run_default(args, world, rank, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            if dist.is_initialized():
                dist.destroy_process_group()



if __name__ == "__main__":
    sys.exit(main())
