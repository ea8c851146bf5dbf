"""Benchmark of the FA2 forward hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg3|cfg3c|cfg2|cfg2c|cfg1|cfg4|cfg5|bwd3|bwd3c|d128_3|d128_3c]
                    [--no-legs] [--no-cpu-baseline] [--ring-layout contiguous|zigzag]

Metric: FA2 forward TFLOP/s per B200 (fp16, D=64), FLOPs =
4·B·H·N²·D halved for causal (reference benchmarks/benchmark_throughput.py:23-31).
A step is one forward_flash2 call over one batch. The default workload is
BASELINE config 3 (B=2, H=8, N=4096, D=64, non-causal: the headline). With N
GPUs (torchrun) every rank runs its own config-3 batch of (b,h) slices of a
global B=2·N problem (head sharding, no communication): weak scaling, so the
N=1 line is the single-GPU headline.

Timing of ``value``: W untimed warm-up steps, then K steps between CUDA events
on the launching stream, bracketed by a barrier and a device synchronize; the
max over ranks is reported. Steps rotate through enough independent input
sets that their total footprint is over 3x the 126 MB L2, so every step reads
its inputs from HBM. Beside it: ``median`` (median of per-call CUDA-event
times), ``same_method`` (the reference benchmark's own method: median of 100
after 25 warm-up on one input set, benchmarks/benchmark_throughput.py:34-54),
``e2e`` (the step through the public API with inputs copied from pinned host
memory and the output read back), ``naive`` (forward_naive, timed as the
reference benchmark does, :125-136), ``peak_mem_mb`` (peak allocated memory of
forward_flash2 with and without ``out=`` against unfused torch attention,
:170-197) and ``cfg1``.

Multi-GPU legs (``cfg4``, ``cfg5`` sub-objects, at every N, on by default for
the config-3 workloads): config 4 (B16 H32 N8192 causal, 512 slices split
over the ranks: strong scaling) and config 5 (B1 H8 N131072 causal, sequence
sharded, NCCL ring, contiguous and zig-zag layouts). Each leg times its step,
the same problem on one GPU (rank 0 alone, for the efficiency), and checks
sampled output rows of every rank against the CPU fp32 oracle.

``--impl reference`` runs the reference's CPU math path (torch fp32
matmul-softmax-matmul on all host threads, the oracle port) on the same
workload and, when a GPU and the reference kernels built from its own sources
(oracle/_ref) are present, also times those kernels and PyTorch SDPA. That
process loads no code of this package.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

L2_BYTES = 126 * 1024 * 1024
D = 64
TOL_MAX, TOL_MEAN = 2e-3, 2e-4  # north-star tolerance against the fp32 oracle

WORKLOADS = {
    # name: (B, H, N, causal, description)
    "cfg1": (1, 2, 128, False, "BASELINE config 1: B1 H2 N128 D64 non-causal"),
    "cfg2": (2, 8, 1024, False, "BASELINE config 2: B2 H8 N1024 D64 non-causal"),
    "cfg2c": (2, 8, 1024, True, "BASELINE config 2: B2 H8 N1024 D64 causal"),
    "cfg3": (2, 8, 4096, False, "BASELINE config 3: B2 H8 N4096 D64 non-causal (headline)"),
    "cfg3c": (2, 8, 4096, True, "BASELINE config 3: B2 H8 N4096 D64 causal"),
    "cfg4": (16, 32, 8192, True, "BASELINE config 4: B16 H32 N8192 D64 causal, 512 slices split over ranks"),
    "cfg5": (1, 8, 131072, True, "BASELINE config 5: B1 H8 N131072 D64 causal, sequence sharded, NCCL ring"),
}

# Extension workloads (no reference counterpart: the reference is forward-only
# and head_dim 64 only): name -> (B, H, N, D, causal, backward, description)
EXT_WORKLOADS = {
    "bwd3": (2, 8, 4096, 64, False, True, "FA2 backward on the config-3 shape: B2 H8 N4096 D64 non-causal"),
    "bwd3c": (2, 8, 4096, 64, True, True, "FA2 backward on the config-3 shape: B2 H8 N4096 D64 causal"),
    "d128_3": (2, 8, 4096, 128, False, False, "FA2 forward, head_dim 128: B2 H8 N4096 D128 non-causal"),
    "d128_3c": (2, 8, 4096, 128, True, False, "FA2 forward, head_dim 128: B2 H8 N4096 D128 causal"),
    "sk20": (1, 20, 4096, 64, False, False,
             "FA2 forward on a 2.16-wave grid (320 units on 148 SMs), stream-K schedule: B1 H20 N4096 D64 non-causal"),
}


def flops(B, H, N, D_, causal):
    return (2.0 if causal else 4.0) * B * H * N * N * D_


def median(xs):
    s = sorted(xs)
    return s[len(s) // 2]


# ----------------------------------------------------------------------------
# distributed plumbing
# ----------------------------------------------------------------------------
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_dist(world, backend):
    if world > 1 and not torch.distributed.is_initialized():
        import datetime

        torch.distributed.init_process_group(backend, timeout=datetime.timedelta(seconds=120))


def barrier(world, device=None):
    if world > 1:
        if device is not None:
            torch.distributed.barrier(device_ids=[device.index])
        else:
            torch.distributed.barrier()


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t)
    return float(t.item())


# ----------------------------------------------------------------------------
# clocks during the timed region
# ----------------------------------------------------------------------------
class ClockSampler:
    """Polls SM clock and throttle reasons through NVML in a thread.

    ``mark()`` splits the samples taken so far (the timed region) from those
    of an untimed sustained pass of the same step that follows it, so a short
    timed region still gets a clock reading."""

    REASONS = {
        "sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, index: int, period_s: float = 0.0005):
        self.samples, self.reasons = [], set()
        self.n_timed = None
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        self._period = period_s
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None

    def _sample(self):
        nv = self._nv
        self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
        mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
        for name, bit in self.REASONS.items():
            if mask & bit:
                self.reasons.add(name)

    def _loop(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            time.sleep(self._period)

    def __enter__(self):
        if self._nv is not None:
            self._t = threading.Thread(target=self._loop, daemon=True)
            self._t.start()
        return self

    def mark(self):
        self.n_timed = len(self.samples)

    def __exit__(self, *exc):
        self._stop.set()
        if self._t is not None:
            self._t.join()
            if not self.samples:
                try:
                    self._sample()
                except Exception:
                    pass

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        return {"sm_mhz": median(self.samples), "sm_max_mhz": self.max_mhz,
                "sm_mhz_min": min(self.samples), "reasons": sorted(self.reasons),
                "samples": len(self.samples),
                "samples_timed_region": self.n_timed if self.n_timed is not None else len(self.samples),
                "window": "timed region plus an untimed sustained pass of the same step right after it"}


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), \
            float(d["hbm_gbs"]), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


def profiled_traffic(kernel: str, workload: str):
    """DRAM bytes per launch from the committed ncu summary, if present."""
    f = ROOT / "profiles" / f"{kernel}_{workload}.txt"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


# ----------------------------------------------------------------------------
# seeded synthetic inputs, generated on the device
# ----------------------------------------------------------------------------
def dev_slices(idx, N, seed, device, scale=1.0):
    """q, k, v [len(idx), N, D] fp16: i.i.d. N(0,1)·scale, each (b,h) slice
    (and tensor) from its own CUDA generator, so values do not depend on how
    slices are sharded over ranks."""
    g = torch.Generator(device=device)
    out = []
    for name in range(3):
        t = torch.empty(len(idx), N, D, dtype=torch.float16, device=device)
        for r, s in enumerate(idx):
            g.manual_seed((seed * 1_000_003 + s) * 4 + name)
            t[r] = torch.randn(N, D, generator=g, device=device) * scale
        out.append(t)
    return out


RING_BLOCK = 1024  # rows per generator block of the sequence-sharded inputs


def dev_rows(row0, nrows, H, seed, device, scale, heads=None):
    """q, k, v [1, len(heads), nrows, D] fp16 for global rows [row0, row0+nrows)
    of a [1, H, N, D] problem: each (1024-row block, head, tensor) draws from
    its own CUDA generator, so any rank can produce any rows."""
    assert row0 % RING_BLOCK == 0 and nrows % RING_BLOCK == 0
    heads = list(range(H)) if heads is None else heads
    g = torch.Generator(device=device)
    out = []
    for name in range(3):
        t = torch.empty(1, len(heads), nrows, D, dtype=torch.float16, device=device)
        for hi, h in enumerate(heads):
            for b in range(nrows // RING_BLOCK):
                blk = row0 // RING_BLOCK + b
                g.manual_seed((seed * 1_000_003 + blk * H + h) * 4 + name)
                t[0, hi, b * RING_BLOCK:(b + 1) * RING_BLOCK] = \
                    torch.randn(RING_BLOCK, D, generator=g, device=device) * scale
        out.append(t)
    return out


def rank_slices(workload, world, rank):
    from flashlite_b200.parallel_attn import shard_range

    B, H, N, causal, _ = WORKLOADS[workload]
    if workload == "cfg4":  # strong scaling: fixed 512 slices split over ranks
        return shard_range(B * H, world, rank), B * H, N, causal, "strong"
    per = B * H  # weak scaling: each rank owns one config-sized batch
    return range(rank * per, (rank + 1) * per), per * world, N, causal, "weak"


def l2_flush_buffer(device):
    return torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=device)


def time_steps_flushed(step, steps, warmup, flush, stream):
    """Per-step CUDA-event times (ms), each step preceded by an untimed write
    of a buffer larger than L2."""
    for _ in range(warmup):
        step()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    for a, b in evs:
        flush.zero_()
        a.record(stream)
        step()
        b.record(stream)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


def median_ms_ref_method(fn, warm=25, runs=100):
    """benchmarks/benchmark_throughput.py:34-54: median of `runs` CUDA-event
    timings after `warm` calls (inputs stay in L2 between calls)."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    es = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(runs)]
    for a, b in es:
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize()
    return median([a.elapsed_time(b) for a, b in es])


# ----------------------------------------------------------------------------
# parity of sampled rows against the CPU fp32 oracle (the checker)
# ----------------------------------------------------------------------------
def row_errors(out_rows, q_all, k_all, v_all, rows, sm_scale, causal):
    """(max-abs, sum-abs, count) of out_rows [S, R, D] against the oracle's
    rows of q_all/k_all/v_all [S, N, D] (host or device tensors)."""
    from oracle.attention_oracle import attention_rows_fp32

    ref = attention_rows_fp32(q_all.cpu(), k_all.cpu(), v_all.cpu(), rows, sm_scale, causal)
    err = (out_rows.float().cpu() - ref).abs()
    return float(err.max()), float(err.sum()), err.numel()


def reduce_errors(errs, world, device):
    mx = max_over_ranks(max(e[0] for e in errs), world, device)
    tot = sum_over_ranks(sum(e[1] for e in errs), world, device)
    cnt = sum_over_ranks(float(sum(e[2] for e in errs)), world, device)
    mean = tot / max(cnt, 1.0)
    return {"max_abs": mx, "mean_abs": mean, "values_checked": int(cnt),
            "ok": bool(mx <= TOL_MAX and mean <= TOL_MEAN), "tolerance": [TOL_MAX, TOL_MEAN]}


# ----------------------------------------------------------------------------
# multi-GPU legs: config 4 (head sharded) and config 5 (ring)
# ----------------------------------------------------------------------------
def leg_cfg4(world, rank, device, steps, warmup, flush, stream):
    """512 (b,h) slices of N=8192 causal split over ranks."""
    from flashlite_b200 import flash_attn_wmma as fa
    from flashlite_b200.parallel_attn import shard_range

    B, H, N, causal, desc = WORKLOADS["cfg4"]
    total, scale, seed = B * H, 0.125, 4

    def run_on(idx):
        q, k, v = dev_slices(idx, N, seed, device)
        shape = (1, len(idx), N, D)
        q, k, v = (t.view(shape) for t in (q, k, v))
        o = torch.empty_like(q)
        ts = time_steps_flushed(lambda: fa.forward_flash2(q, k, v, scale, causal, out=o),
                                steps, warmup, flush, stream)
        return q, k, v, o, ts

    mine = shard_range(total, world, rank)
    q, k, v, o, ts = run_on(mine)
    ms = max_over_ranks(median(ts), world, device)
    # parity: first and last slice of this rank, rows spread over the sequence
    rows = torch.tensor([0, 1, 127, 128, N // 2 - 1, N // 2, N - 129, N - 1])
    errs = []
    for i in (0, len(mine) - 1):
        errs.append(row_errors(o[0, i][rows][None], q[0, i][None], k[0, i][None], v[0, i][None],
                               rows, scale, causal))
    parity = reduce_errors(errs, world, device)
    del q, k, v, o
    # the same problem on one GPU (rank 0 alone), for the efficiency
    barrier(world, device)
    t1 = None
    if world == 1:
        t1 = ms
    elif rank == 0:
        *_, ts1 = run_on(range(total))
        t1 = median(ts1)
    barrier(world, device)
    torch.cuda.empty_cache()
    f = flops(B, H, N, D, causal)
    res = {"workload": desc, "scaling": "strong", "slices_per_rank": len(mine),
           "ms_per_step": round(ms, 4), "tflops": round(f / (ms * 1e-3) / 1e12, 2),
           "timing": f"median of {steps} steps after {warmup} warm-up, L2 flushed between steps, max over ranks",
           "parity": parity}
    if rank == 0:
        res["one_gpu_ms"] = round(t1, 4)
        res["efficiency"] = round(t1 / (world * ms), 4)
    return res


def ring_inputs(world, rank, layout, N, H, seed, scale, device):
    """This rank's q, k, v and the global query rows each local row holds."""
    if layout == "zigzag" and world > 1:
        from flashlite_b200.parallel_attn import zigzag_chunks

        c = N // (2 * world)
        parts = [dev_rows(ch * c, c, H, seed, device, scale) for ch in zigzag_chunks(rank, world)]
        q, k, v = (torch.stack([parts[0][i], parts[1][i]]) for i in range(3))
        starts = [ch * c for ch in zigzag_chunks(rank, world)]
        return q, k, v, starts, c
    nb = N // world
    q, k, v = dev_rows(rank * nb, nb, H, seed, device, scale)
    return q, k, v, [rank * nb], nb


def ring_breakdown(per, ms):
    """Names the step that limits a ring from every rank's [compute ms,
    exchange-wait ms] of one step and the step time: the rank that computes
    most sets the step, so its wait is exchange the ring failed to hide
    (lightly loaded ranks also wait, on their busier neighbours)."""
    comp = [c for c, _ in per]
    crit = max(range(len(per)), key=lambda r: comp[r])
    c_max, c_min = max(comp), min(comp)
    out = {"compute_ms_max": round(c_max, 4), "compute_ms_min": round(c_min, 4),
           "exposed_exchange_ms_max": round(max(w for _, w in per), 4),
           "busiest_rank": crit, "busiest_rank_exchange_wait_ms": round(per[crit][1], 4)}
    if per[crit][1] > 0.1 * ms:
        out["limiting_step"] = "K/V exchange not hidden behind the busiest rank's block compute"
    elif c_max > 1.15 * c_min:
        out["limiting_step"] = ("causal load imbalance: the rank holding the last rows computes "
                                f"{c_max / max(c_min, 1e-9):.2f}x the lightest rank's blocks")
    else:
        out["limiting_step"] = "block compute (the ring's per-step kernel launches on N/P-row blocks)"
    return out


def leg_cfg5(world, rank, device, steps, warmup, flush, stream, layout):
    """B1 H8 N131072 causal, sequence sharded over ranks."""
    from flashlite_b200 import flash_attn_wmma as fa
    from flashlite_b200.parallel_attn import RingAttention, ZigzagRingAttention

    B, H, N, causal, desc = WORKLOADS["cfg5"]
    scale, seed, sm_scale = 0.5, 5, 0.125
    q, k, v, starts, rows_per_part = ring_inputs(world, rank, layout, N, H, seed, scale, device)
    out = torch.empty_like(q)
    o_acc = torch.empty(q.shape, dtype=torch.float32, device=device)
    lse = torch.empty(q.shape[:-1], dtype=torch.float32, device=device)
    ring = None
    launches = [0]  # this rank's kernel launches in its timed steps
    if world > 1:
        def block(*a):
            launches[0] += 1
            fa.forward_block(*a)

        def finalize(*a):
            launches[0] += 1
            fa.ring_finalize(*a)

        cls = ZigzagRingAttention if layout == "zigzag" else RingAttention
        ring = cls(block_fn=block, finalize_fn=finalize)

    def step(events=None):
        if ring is None:
            fa.forward_flash2(q, k, v, sm_scale, causal, out=out)
        else:
            ring.forward(q, k, v, sm_scale, causal, out=out, o_acc=o_acc, lse=lse, events=events)

    ts = time_steps_flushed(step, steps, warmup, flush, stream)
    per_step = launches[0] / (steps + warmup) if ring is not None else 1.0
    ms = max_over_ranks(median(ts), world, device)
    breakdown = None
    if ring is not None:
        # one instrumented step: block compute vs exchange wait per ring step
        flush.zero_()
        evs = []
        step(evs)
        torch.cuda.synchronize()
        comp = sum(e[0].elapsed_time(e[1]) for e in evs)
        wait = sum(e[1].elapsed_time(e[2]) for e in evs)
        # every rank's (compute, exchange wait); the rank that computes most
        # sets the step, so its wait is the exchange time the ring failed to
        # hide (lightly loaded ranks wait on their busier neighbours instead)
        per = torch.zeros(world, 2, dtype=torch.float64, device=device)
        per[rank, 0], per[rank, 1] = comp, wait
        if world > 1:
            torch.distributed.all_reduce(per)
        breakdown = ring_breakdown(per.cpu().tolist(), ms)
    # parity: sampled rows of this rank (first and last rows of each part) on
    # the first and last head, against the oracle over the whole causal prefix
    errs = []
    for hh in (0, H - 1):
        last = max(starts) + rows_per_part
        kq, kk, kv = dev_rows(0, last, H, seed, device, scale, heads=[hh])
        for pi, st in enumerate(starts):
            loc = torch.tensor([0, rows_per_part // 2, rows_per_part - 1])
            glob = loc + st
            got = (out[pi, 0, hh] if q.dim() == 5 else out[0, hh])[loc]
            errs.append(row_errors(got[None], kq[0, 0][None], kk[0, 0][None], kv[0, 0][None],
                                   glob, sm_scale, causal))
        del kq, kk, kv
    parity = reduce_errors(errs, world, device)
    del q, k, v, out, o_acc, lse
    if ring is not None:
        del ring
    barrier(world, device)
    t1 = None
    if world == 1:
        t1 = ms
    elif rank == 0:
        qa, ka, va = dev_rows(0, N, H, seed, device, scale)
        oa = torch.empty_like(qa)
        t1 = median(time_steps_flushed(lambda: fa.forward_flash2(qa, ka, va, sm_scale, causal, out=oa),
                                       steps, warmup, flush, stream))
        del qa, ka, va, oa
    barrier(world, device)
    torch.cuda.empty_cache()
    f = flops(B, H, N, D, causal)
    res = {"workload": desc, "scaling": "strong",
           "layout": (layout if world > 1 else "single GPU"),
           "gpu_launches_per_step": per_step,
           "ms_per_step": round(ms, 4), "tflops": round(f / (ms * 1e-3) / 1e12, 2),
           "timing": f"median of {steps} steps after {warmup} warm-up, L2 flushed between steps, max over ranks",
           "parity": parity}
    if breakdown is not None:
        res["breakdown"] = breakdown
    if layout == "contiguous" and world > 1:
        res["causal_speedup_cap"] = round(world * world / (2 * world - 1), 3)
    if rank == 0:
        res["one_gpu_ms"] = round(t1, 4)
        res["efficiency"] = round(t1 / (world * ms), 4)
    return res


def _leg(fn, *a):
    """Runs one leg; an exception is recorded in the leg's own entry so that
    the line still carries the headline. (A failure on every rank leaves the
    ranks in step; one on a single rank ends its peers' next collective
    through the process group's timeout.)"""
    try:
        return fn(*a)
    except Exception as exc:  # reported, not hidden: the entry says what failed
        if torch.cuda.is_available() and torch.cuda.is_initialized():
            torch.cuda.synchronize()
        return {"error": f"{type(exc).__name__}: {str(exc)[:300]}"}


def run_legs(world, rank, device, stream):
    flush = l2_flush_buffer(device)
    legs = {"cfg4": _leg(leg_cfg4, world, rank, device, 5, 3, flush, stream)}
    layouts = ["contiguous", "zigzag"] if world > 1 else ["contiguous"]
    legs["cfg5"] = {lay: _leg(leg_cfg5, world, rank, device, 3, 2, flush, stream, lay) for lay in layouts}
    del flush
    torch.cuda.empty_cache()
    return legs


# ----------------------------------------------------------------------------
# single-GPU extras: naive path, peak memory, config 1
# ----------------------------------------------------------------------------
def naive_timing(q, k, v, sm_scale, causal, f):
    """forward_naive with the reference benchmark's iteration counts (:129-131)."""
    from flashlite_b200 import flash_attn_wmma as fa

    N = q.shape[2]
    warm, runs = (5, 20) if N <= 1024 else (2, 5)
    ms = median_ms_ref_method(lambda: fa.forward_naive(q, k, v, sm_scale, causal), warm, runs)
    return {"ms": round(ms, 4), "tflops": round(f / (ms * 1e-3) / 1e12, 3),
            "timing": f"median of {runs} after {warm} warm-up (benchmarks/benchmark_throughput.py:129-132)"}


def peak_memory(device, causal):
    """benchmarks/benchmark_throughput.py:170-197 (B2 H8, N 512..4096): peak
    allocated MB of unfused torch attention, forward_flash2 and
    forward_flash2(out=) with q, k, v (and out) already allocated."""
    from flashlite_b200 import flash_attn_wmma as fa

    res = {}
    for N in (512, 1024, 2048, 4096):
        q, k, v = (torch.randn(2, 8, N, D, dtype=torch.float16, device=device) for _ in range(3))
        buf = torch.empty_like(q)
        sm = 1.0 / math.sqrt(D)

        def peak(fn):
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
            torch.cuda.reset_peak_memory_stats(device)
            r = fn()
            torch.cuda.synchronize()
            del r
            return round(torch.cuda.max_memory_allocated(device) / 2**20, 2)

        def unfused():
            s = torch.matmul(q, k.transpose(-2, -1)) * sm
            return torch.matmul(torch.softmax(s, dim=-1), v)

        res[str(N)] = {"unfused_torch": peak(unfused),
                       "forward_flash2": peak(lambda: fa.forward_flash2(q, k, v, sm, causal)),
                       "forward_flash2_out": peak(lambda: fa.forward_flash2(q, k, v, sm, causal, out=buf))}
        del q, k, v, buf
    torch.cuda.empty_cache()
    return res


def cfg1_line(device, with_cpu):
    """BASELINE config 1 (B1 H2 N128 non-causal, seed 0, scale 1/8): GPU
    timings of both kernels with the reference's method, and the CPU oracle."""
    from flashlite_b200 import flash_attn_wmma as fa

    B, H, N, causal, desc = WORKLOADS["cfg1"]
    q, k, v = (t.to(device) for t in dev_slices(range(B * H), N, 0, device))
    q, k, v = (t.view(B, H, N, D) for t in (q, k, v))
    out = torch.empty_like(q)
    f = flops(B, H, N, D, causal)
    ms = median_ms_ref_method(lambda: fa.forward_flash2(q, k, v, 0.125, causal, out=out))
    res = {"workload": desc, "flash2": {"ms": round(ms, 5), "tflops": round(f / (ms * 1e-3) / 1e12, 4)},
           "naive": naive_timing(q, k, v, 0.125, causal, f)}
    if with_cpu:
        res["cpu_baseline"] = cpu_baseline("cfg1")
    return res


# ----------------------------------------------------------------------------
# our arm
# ----------------------------------------------------------------------------
def run_ours(args):
    world, rank, local = dist_env()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    init_dist(world, "nccl")
    from flashlite_b200 import flash_attn_wmma as fa

    slices, total_slices, N, causal, scaling = rank_slices(args.workload, world, rank)
    S = len(slices)
    sm_scale = 0.125
    base = dev_slices(slices, N, seed=0, device=device)
    shape = (1, S, N, D)
    set_bytes = 4 * base[0].numel() * 2
    n_sets = max(2, math.ceil(3 * L2_BYTES / set_bytes))
    n_sets = min(n_sets, max(2, int(0.25 * torch.cuda.get_device_properties(device).total_memory // set_bytes)))
    sets = []
    for i in range(n_sets):  # distinct buffers, same values: keeps every step's bytes cold in L2
        q, k, v = (t.view(shape) if i == 0 else t.view(shape).clone() for t in base)
        sets.append((q, k, v, torch.empty_like(q)))
    del base
    stream = torch.cuda.current_stream(device)

    def step(i):
        q, k, v, o = sets[i % n_sets]
        fa.forward_flash2(q, k, v, sm_scale, causal, out=o)

    clk = ClockSampler(device.index if device.index is not None else 0)  # NVML set-up before timing
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(device)
    barrier(world, device)
    torch.cuda.synchronize(device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with clk:
        # A ~4 ms spin on the stream before the start event: by the time the
        # GPU reaches ev0 the host has queued all K steps (~25 us each through
        # the binding, with the clock sampler's thread sharing the GIL), so
        # the timed region holds device time only.
        torch.cuda._sleep(8_000_000)
        ev0.record(stream)
        for i in range(args.steps):
            step(i)
        ev1.record(stream)
        torch.cuda.synchronize(device)
        clk.mark()
        # untimed sustained pass of the same step (~0.3 s) for the clock reading
        t_end = time.perf_counter() + 0.3
        i = 0
        while time.perf_counter() < t_end:
            for _ in range(20):
                step(i)
                i += 1
            torch.cuda.synchronize(device)
    barrier(world, device)
    torch.cuda.synchronize(device)
    ms_local = ev0.elapsed_time(ev1)
    err = fa.device_error()
    ms = max_over_ranks(ms_local, world, device)
    per_rank_flops = flops(1, S, N, D, causal)
    total_flops = per_rank_flops * world
    ms_step = ms / args.steps
    value = total_flops / (ms_step * 1e-3) / 1e12

    # ---- per-call CUDA-event times: median beside the mean above ----
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    torch.cuda._sleep(8_000_000)
    for i, (a, b) in enumerate(evs):
        a.record(stream)
        step(i)
        b.record(stream)
    torch.cuda.synchronize(device)
    med_ms = max_over_ranks(median([a.elapsed_time(b) for a, b in evs]), world, device)

    # ---- the reference benchmark's method: one input set, L2 warm ----
    q0, k0, v0, o0 = sets[0]
    same_ms = max_over_ranks(median_ms_ref_method(
        lambda: fa.forward_flash2(q0, k0, v0, sm_scale, causal, out=o0)), world, device)

    # ---- end to end through the public API: pinned host in, host out ----
    # Every step copies its Q, K, V from pinned host memory and its O back.
    # Serial: copy in, compute, copy out, one after the other. Pipelined (the
    # reported e2e): two device buffer sets; step i+1's copies in run on a
    # copy stream while step i computes, step i's copy out on a third stream.
    # Q, K and V of a step sit in one pinned host buffer and travel as one
    # copy (one 24 MiB copy runs at ~54 GB/s, three 8 MiB copies back to back
    # at ~48-52 on this host link); the call gets contiguous views of it.
    qkv_p = torch.stack((q0, k0, v0)).cpu().pin_memory()
    ops = [torch.empty_like(qkv_p[0]).pin_memory() for _ in range(2)]
    dbuf = [(torch.empty_like(qkv_p, device=device), torch.empty_like(q0)) for _ in range(2)]

    def e2e_serial(nsteps):
        dqkv, do = dbuf[0]
        for _ in range(nsteps):
            dqkv.copy_(qkv_p, non_blocking=True)
            fa.forward_flash2(dqkv[0], dqkv[1], dqkv[2], sm_scale, causal, out=do)
            ops[0].copy_(do, non_blocking=True)

    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def e2e_pipelined(nsteps, start_ev):
        s_in.wait_event(start_ev)
        for i in range(nsteps):
            b = i % 2
            dqkv, do = dbuf[b]
            with torch.cuda.stream(s_in):
                if i >= 2:
                    s_in.wait_event(ev_done[b])  # step i-2 has read these inputs
                dqkv.copy_(qkv_p, non_blocking=True)
                ev_in[b].record(s_in)
            stream.wait_event(ev_in[b])
            if i >= 2:
                stream.wait_event(ev_out[b])  # step i-2's output has been copied out
            fa.forward_flash2(dqkv[0], dqkv[1], dqkv[2], sm_scale, causal, out=do)
            ev_done[b].record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_done[b])
                ops[b].copy_(do, non_blocking=True)
                ev_out[b].record(s_out)
        for b in range(2):
            stream.wait_event(ev_out[b])

    e_steps = max(3, min(args.steps, 50))

    def timed(fn):
        for _ in range(3):  # warm-up
            e0 = torch.cuda.Event()
            e0.record(stream)
            fn(2, e0) if fn is e2e_pipelined else fn(2)
        torch.cuda.synchronize(device)
        barrier(world, device)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        fn(e_steps, t0) if fn is e2e_pipelined else fn(e_steps)
        t1.record(stream)
        torch.cuda.synchronize(device)
        return max_over_ranks(t0.elapsed_time(t1) / e_steps, world, device)

    es_ms = timed(e2e_serial)
    e_ms = timed(e2e_pipelined)
    e2e_value = total_flops / (e_ms * 1e-3) / 1e12
    e2e_serial_value = total_flops / (es_ms * 1e-3) / 1e12
    ok = all(torch.isfinite(o.float()).all().item() for o in ops)
    del dbuf, sets

    extras = {}
    if rank == 0 and args.workload != "cfg4":
        extras["naive"] = naive_timing(q0, k0, v0, sm_scale, causal, per_rank_flops)
        extras["peak_mem_mb"] = peak_memory(device, causal)
        extras["cfg1"] = cfg1_line(device, with_cpu=(world == 1 and not args.no_cpu_baseline))
    del q0, k0, v0, o0
    torch.cuda.empty_cache()
    legs = None
    if not args.no_legs and args.workload in ("cfg3", "cfg3c"):
        legs = run_legs(world, rank, device, stream)

    peak_burst, peak_sust, hbm, peak_kind = measured_peaks()
    achieved = per_rank_flops / (ms_step * 1e-3) / 1e12  # per launch per GPU
    alg_bytes = 4 * S * N * D * 2
    traffic = profiled_traffic("flash2_fwd", args.workload)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.workload)

    if rank == 0:
        B0, H0, N0, c0, desc = WORKLOADS[args.workload]
        line = {
            "metric": "FA2 fwd TFLOP/s per B200 (fp16, D=64)",
            "value": round(value, 2),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_step, 5),
            "higher_is_better": True,
            "scaling": scaling,
            "vs_baseline": None,
            "dtype": "fp16 (fp32 accumulate)",
            "data": "synthetic: seeded i.i.d. N(0,1) fp16 Q/K/V generated on the device per (b,h) slice",
            "config": {
                "workload": desc,
                "B_per_rank": 1, "H_per_rank": S, "slices_total": total_slices,
                "N": N, "D": D, "causal": causal, "sm_scale": sm_scale,
                "parallelism": f"head-sharded x{world}, no collective" if world > 1 else "single GPU",
                "l2": f"{n_sets} rotating input sets, {n_sets * set_bytes / 2**20:.0f} MiB > 126 MB L2",
            },
            "median": {"ms_per_call": round(med_ms, 5),
                       "value": round(total_flops / (med_ms * 1e-3) / 1e12, 2),
                       "timing": "median of per-call CUDA-event times over K calls (same rotating sets)"},
            "same_method": {"ms": round(same_ms, 5),
                            "value_per_gpu": round(per_rank_flops / (same_ms * 1e-3) / 1e12, 2),
                            "timing": "median of 100 after 25 warm-up, one input set, L2 warm "
                                      "(benchmarks/benchmark_throughput.py:34-54)"},
            "pct_of_peak": round(100 * achieved / peak_burst, 2),
            "hbm_gbs": round(alg_bytes / (ms_step * 1e-3) / 1e9, 1),
            "roofline": {
                "bound": "tensor", "achieved": round(achieved, 2), "peak": peak_burst,
                "unit": "TFLOP/s", "frac": round(achieved / peak_burst, 4),
                "peak_kind": f"{peak_kind} bf16 dense burst (sustained {peak_sust})",
                "traffic": traffic,
                "alg_bytes": alg_bytes,
                "hbm_frac": round(alg_bytes / (ms_step * 1e-3) / 1e9 / hbm, 4),
            },
            "e2e": {"value": round(e2e_value, 2), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": qkv_p.numel() * 2, "d2h_bytes_per_step": ops[0].numel() * 2,
                    "ms_per_step": round(e_ms, 4), "output_finite": bool(ok),
                    "mode": "pipelined: step i+1's host-to-device copy (Q, K, V in one pinned "
                            "buffer) and step i-1's device-to-host copy overlap step i's kernel "
                            "(two buffer sets)",
                    "serial_value": round(e2e_serial_value, 2), "serial_ms_per_step": round(es_ms, 4)},
            "gpu_launches": args.steps,
            "clocks": clk.summary(),
            "device_error": int(err),
            "cpu_baseline": cpu,
        }
        line.update(extras)
        if legs is not None:
            line.update(legs)
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


# ----------------------------------------------------------------------------
# extension workloads: backward, head_dim 128 (single GPU or weak-scaled copies)
# ----------------------------------------------------------------------------
def run_ext(args):
    world, rank, local = dist_env()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    init_dist(world, "nccl")
    from flashlite_b200 import flash_attn_wmma as fa

    B, H, N, Dx, causal, bwd, desc = EXT_WORKLOADS[args.workload]
    sm_scale = 0.0  # 1/sqrt(D)
    g = torch.Generator().manual_seed(7 + rank)
    host = [torch.randn(B, H, N, Dx, generator=g).half() for _ in range(4 if bwd else 3)]
    tensor_bytes = host[0].numel() * 2
    in_bytes = (6 if bwd else 3) * tensor_bytes  # bwd: q, k, v, out, dout (+ lse)
    n_sets = max(2, math.ceil(3 * L2_BYTES / in_bytes))
    sets = []
    for i in range(n_sets):
        q, k, v = (t.to(device) for t in host[:3])
        if bwd:
            do = host[3].to(device)
            out, lse = fa.forward_flash2_ex(q, k, v, sm_scale, causal, return_lse=True)
            sets.append((q, k, v, out, do, lse))
        else:
            sets.append((q, k, v, torch.empty_like(q)))
    stream = torch.cuda.current_stream(device)

    def step(i):
        t = sets[i % n_sets]
        if bwd:
            return fa.backward_flash2(*t, sm_scale, causal)
        return fa.forward_flash2_ex(t[0], t[1], t[2], sm_scale, causal, out=t[3])

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(device)
    barrier(world, device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index if device.index is not None else 0) as clk:
        ev0.record(stream)
        for i in range(args.steps):
            step(i)
        ev1.record(stream)
        torch.cuda.synchronize(device)
        clk.mark()
    barrier(world, device)
    ms_step = max_over_ranks(ev0.elapsed_time(ev1), world, device) / args.steps
    err = fa.device_error()
    # FLOPs: forward 4·B·H·N²·D (halved causal); backward 2.5x that (five GEMMs to two)
    f_step = (2.5 if bwd else 1.0) * flops(B, H, N, Dx, causal)
    value = world * f_step / (ms_step * 1e-3) / 1e12

    # end to end through the public API: inputs from pinned host memory, the
    # results (dq, dk, dv or out) read back each step, serially
    pinned = [t.pin_memory() for t in host]
    dev = [torch.empty_like(t, device=device) for t in host]
    lse_h = sets[0][5].cpu().pin_memory() if bwd else None
    out_h = sets[0][3].cpu().pin_memory() if bwd else None
    lse_d = torch.empty_like(sets[0][5]) if bwd else None
    out_d = torch.empty_like(sets[0][3]) if bwd else None
    res_h = [torch.empty_like(host[0]).pin_memory() for _ in range(3 if bwd else 1)]

    def e2e(n):
        for _ in range(n):
            for d_, h_ in zip(dev, pinned):
                d_.copy_(h_, non_blocking=True)
            if bwd:
                out_d.copy_(out_h, non_blocking=True)
                lse_d.copy_(lse_h, non_blocking=True)
                res = fa.backward_flash2(dev[0], dev[1], dev[2], out_d, dev[3], lse_d, sm_scale, causal)
            else:
                res = (fa.forward_flash2_ex(dev[0], dev[1], dev[2], sm_scale, causal)[0],)
            for r_h, r in zip(res_h, res):
                r_h.copy_(r, non_blocking=True)

    e_steps = max(3, min(args.steps, 30))
    e2e(3)
    torch.cuda.synchronize(device)
    barrier(world, device)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    e2e(e_steps)
    t1.record(stream)
    torch.cuda.synchronize(device)
    e_ms = max_over_ranks(t0.elapsed_time(t1) / e_steps, world, device)
    h2d = sum(t.numel() * t.element_size() for t in host) + (
        (out_h.numel() * 2 + lse_h.numel() * 4) if bwd else 0)
    d2h = sum(t.numel() * 2 for t in res_h)

    peak_burst, peak_sust, hbm, peak_kind = measured_peaks()
    achieved = f_step / (ms_step * 1e-3) / 1e12
    kernel = "flash2_bwd" if bwd else "flash2_fwd"
    if rank == 0:
        line = {
            "metric": ("FA2 bwd" if bwd else "FA2 fwd") + f" TFLOP/s per B200 (fp16, D={Dx})",
            "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16 (fp32 accumulate)",
            "data": "synthetic: seeded i.i.d. N(0,1) fp16 inputs generated on host",
            "config": {"workload": desc, "B": B, "H": H, "N": N, "D": Dx, "causal": causal,
                       "sm_scale": "1/sqrt(D)",
                       "flops_per_step": f_step,
                       "parallelism": f"independent copies x{world}" if world > 1 else "single GPU",
                       "l2": f"{n_sets} rotating input sets, {n_sets * in_bytes / 2**20:.0f} MiB > 126 MB L2"},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak_burst,
                         "unit": "TFLOP/s", "frac": round(achieved / peak_burst, 4),
                         "peak_kind": f"{peak_kind} bf16 dense burst (sustained {peak_sust})",
                         "traffic": profiled_traffic(kernel, args.workload)},
            "e2e": {"value": round(world * f_step / (e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e_ms, 4),
                    "mode": "serial: copies in, the call, results out"},
            "gpu_launches": args.steps * (3 if bwd else 1),
            "clocks": clk.summary(),
            "device_error": int(err),
            "cpu_baseline": None,
            "note": "no reference counterpart (the reference is forward-only and head_dim 64 only)",
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


# ----------------------------------------------------------------------------
# config 5 as the main workload: sequence-sharded ring attention
# ----------------------------------------------------------------------------
def run_ring(args):
    world, rank, local = dist_env()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    init_dist(world, "nccl")
    from flashlite_b200 import flash_attn_wmma as fa

    stream = torch.cuda.current_stream(device)
    flush = l2_flush_buffer(device)
    with ClockSampler(device.index) as clk:
        leg = leg_cfg5(world, rank, device, args.steps, args.warmup, flush, stream, args.ring_layout)
        clk.mark()
    err = fa.device_error()
    peak_burst, peak_sust, _, peak_kind = measured_peaks()
    if rank == 0:
        value = leg["tflops"]
        per_gpu = value / world
        line = {
            "metric": "FA2 fwd TFLOP/s per B200 (fp16, D=64)", "value": value,
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": leg["ms_per_step"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp16 (fp32 accumulate)",
            "data": "synthetic: seeded i.i.d. N(0,1)*0.5 fp16 Q/K/V generated on the device per 1024-row block",
            "config": {"workload": WORKLOADS["cfg5"][4], "N": 131072, "D": D, "causal": True,
                       "parallelism": (f"ring x{world} (NCCL send/recv), {args.ring_layout} layout"
                                       if world > 1 else "single GPU"),
                       "l2": "buffer larger than L2 written between timed steps (untimed)"},
            "pct_of_peak": round(100 * per_gpu / peak_burst, 2),
            "roofline": {"bound": "tensor", "achieved": round(per_gpu, 2), "peak": peak_burst,
                         "unit": "TFLOP/s", "frac": round(per_gpu / peak_burst, 4),
                         "peak_kind": f"{peak_kind} bf16 dense burst (sustained {peak_sust})",
                         "traffic": None, "note": "per GPU"},
            "cfg5": leg,
            "gpu_launches": int(round(args.steps * leg["gpu_launches_per_step"])),
            "clocks": clk.summary(),
            "device_error": int(err),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


# ----------------------------------------------------------------------------
# CPU baseline (oracle port, torch fp32 on host cores)
# ----------------------------------------------------------------------------
def cpu_step(workload):
    """One CPU pass of the workload: (callable, FLOPs, description).

    torch fp32 matmul-softmax-matmul (the oracle port). Configs 1-3 run in
    full. Config 4 is sampled by slices (2 of 512) and config 5 by query rows
    (its full score matrix would need 64 GB): the last 256 rows of one head,
    each attending to its whole causal prefix."""
    from oracle.attention_oracle import attention_fp32, attention_rows_fp32, make_qkv

    B, H, N, causal, _ = WORKLOADS[workload]
    if workload == "cfg5":
        R = 256
        q, k, v = make_qkv(1, 1, N, 64, seed=0, scale=0.5)
        q3, k3, v3 = (t.view(1, N, 64) for t in (q, k, v))
        rows = torch.arange(N - R, N)
        f = float(sum(4 * (int(r) + 1) * 64 for r in rows))
        return (lambda: attention_rows_fp32(q3, k3, v3, rows, 0.125, True), f,
                f"last {R} query rows of 1 of the {H} heads (N={N}, causal), row-sampled")
    n_slices = 2 if workload == "cfg4" else B * H
    q, k, v = make_qkv(1, n_slices, N, 64, seed=0)
    what = (f"{n_slices} of the workload's {B * H} (b,h) slices" if n_slices < B * H
            else f"all {n_slices} (b,h) slices")
    return (lambda: attention_fp32(q, k, v, 0.125, causal), flops(1, n_slices, N, 64, causal),
            f"{what} (N={N}, causal={causal})")


def use_all_host_cores() -> int:
    """torchrun sets OMP_NUM_THREADS=1 for every rank; the CPU arm runs on rank
    0 alone and may use every core this process is allowed on."""
    n = len(os.sched_getaffinity(0))
    torch.set_num_threads(n)
    return n


def cpu_baseline(workload, reps=3):
    use_all_host_cores()
    fn, f, desc = cpu_step(workload)
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    t = median(ts)
    return {"value": round(f / t / 1e12, 5), "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{desc}; torch fp32 matmul-softmax-matmul, median of {reps}: {t * 1e3:.1f} ms"}


def run_reference(args):
    world, rank, local = dist_env()
    if rank != 0:
        return  # the reference arm runs on rank 0 only
    use_all_host_cores()
    fn, f, desc = cpu_step(args.workload)
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    dt = (time.perf_counter() - t0) / args.steps
    value = f / dt / 1e12
    B, H, N, causal, _ = WORKLOADS[args.workload]
    sample = f"{desc} per step; torch fp32 matmul-softmax-matmul on host cores"
    line = {
        "metric": "FA2 fwd TFLOP/s per B200 (fp16, D=64)", "impl": "reference",
        "value": round(value, 5), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic: seeded i.i.d. N(0,1) fp16 Q/K/V generated on host",
        "config": {"workload": WORKLOADS[args.workload][4], "sample": desc, "N": N,
                   "D": 64, "causal": causal,
                   "same_config": args.workload in ("cfg1", "cfg2", "cfg2c", "cfg3", "cfg3c")},
        "cpu_baseline": {"value": round(value, 5), "unit": "TFLOP/s",
                         "cores": torch.get_num_threads(), "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    line["reference_gpu_kernels"] = reference_gpu(args.workload)
    print(json.dumps(line), flush=True)


def reference_gpu(workload):
    """Times the reference's WMMA kernels (built from its own sources for
    sm_100a into oracle/_ref) and PyTorch SDPA-flash, the reference's own
    comparator (benchmarks/benchmark_throughput.py:99-104), on this GPU, with
    the reference benchmark's method. Loads nothing of this package."""
    if not torch.cuda.is_available():
        return {"unavailable": "no GPU"}
    from oracle import build_ref

    B, H, N, causal, _ = WORKLOADS[workload]
    if workload in ("cfg4", "cfg5"):
        return {"unavailable": f"not timed for {workload}"}
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(0)
    q, k, v = (torch.randn(B, H, N, 64, device=dev, dtype=torch.float16, generator=g) for _ in range(3))
    out = torch.empty_like(q)
    f = flops(B, H, N, 64, causal)
    res = {"timing": "median of 100 after 25 warm-up, L2 warm (the reference benchmark's method)"}
    mod = build_ref.load()
    if mod is None:
        res["wmma"] = {"unavailable": "oracle/_ref not built"}
    else:
        ms = median_ms_ref_method(lambda: mod.forward_flash2(q, k, v, 0.125, causal, out=out))
        res["wmma"] = {"ms": round(ms, 4), "tflops": round(f / ms / 1e9, 2)}
        warm, runs = (5, 20) if N <= 1024 else (2, 5)
        ms = median_ms_ref_method(lambda: mod.forward_naive(q, k, v, 0.125, causal), warm, runs)
        res["naive"] = {"ms": round(ms, 4), "tflops": round(f / ms / 1e9, 3)}
    try:
        from torch.nn.attention import SDPBackend, sdpa_kernel
        import torch.nn.functional as F

        def sdpa():
            with sdpa_kernel([SDPBackend.FLASH_ATTENTION]):
                return F.scaled_dot_product_attention(q, k, v, is_causal=causal, scale=0.125)

        ms = median_ms_ref_method(sdpa)
        res["sdpa_flash"] = {"ms": round(ms, 4), "tflops": round(f / ms / 1e9, 2)}
    except Exception as exc:  # backend may be unavailable
        res["sdpa_flash"] = {"unavailable": str(exc)[:120]}
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="cfg3", choices=sorted(WORKLOADS) + sorted(EXT_WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-legs", action="store_true",
                    help="skip the config-4 / config-5 sub-measurements of the config-3 workloads")
    ap.add_argument("--ring-layout", default="contiguous", choices=["contiguous", "zigzag"],
                    help="sequence layout of --workload cfg5 on 2+ GPUs (config 5 fixes contiguous blocks)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    world, _, _ = dist_env()
    if world != args.gpus and not (world == 1 and args.gpus == 1):
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)
    if args.impl == "reference" and args.workload in EXT_WORKLOADS:
        if dist_env()[1] == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the reference is forward-only and "
                              "takes head_dim 64 only: no counterpart for " + args.workload}))
    elif args.impl == "reference":
        run_reference(args)
    elif args.workload in EXT_WORKLOADS:
        run_ext(args)
    elif args.workload == "cfg5":
        run_ring(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
