"""Benchmark of the FA2 forward hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg3|cfg3c|cfg2|cfg2c|cfg4|cfg5|bwd3|bwd3c|d128_3|d128_3c]

(bwd3/bwd3c: the backward pass, d128_3/d128_3c: the head_dim-128 forward, on
the config-3 shape; extensions without a reference counterpart.)

Metric: FA2 forward TFLOP/s per B200 (fp16, D=64), FLOPs =
4·B·H·N²·D halved for causal (reference benchmarks/benchmark_throughput.py:23-31).
A step is one forward_flash2 call over one batch. The default workload is
BASELINE config 3 (B=2, H=8, N=4096, D=64, non-causal: the headline). With N
GPUs (torchrun) every rank runs its own config-3 batch of (b,h) slices of a
global B=2·N problem (head sharding, no communication): weak scaling.

Timing: W untimed warm-up steps, then K steps between CUDA events on the
launching stream, bracketed by a barrier and a device synchronize; the max
over ranks is reported. Steps rotate through enough independent input sets
that their total footprint is over 3x the 126 MB L2, so every step reads its
inputs from HBM. ``e2e`` repeats the measurement through the public API with
the inputs copied from pinned host memory and the output read back each step.

``--impl reference`` runs the reference's CPU math path (torch fp32
matmul-softmax-matmul on all host threads, the oracle port) on a bounded
sample of the same workload, and, when a GPU and the reference kernels built
from its own sources (oracle/_ref) are present, also times those kernels.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

L2_BYTES = 126 * 1024 * 1024

WORKLOADS = {
    # name: (B, H, N, causal, description)
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
}


def flops(B, H, N, D, causal):
    return (2.0 if causal else 4.0) * B * H * N * N * D


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


# ----------------------------------------------------------------------------
# clocks during the timed region
# ----------------------------------------------------------------------------
class ClockSampler:
    """Polls SM clock and throttle reasons through NVML in a thread."""

    REASONS = {
        "sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, index: int, period_s: float = 0.002):
        self.samples, self.reasons = [], set()
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
        s = sorted(self.samples)
        return {"sm_mhz": s[len(s) // 2], "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(s)}


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
# our arm
# ----------------------------------------------------------------------------
def rank_slices(workload, world, rank):
    B, H, N, causal, _ = WORKLOADS[workload]
    if workload == "cfg4":  # strong scaling: fixed 512 slices split over ranks
        total = B * H
        assert total % world == 0
        per = total // world
        return range(rank * per, (rank + 1) * per), total, N, causal, "strong"
    per = B * H  # weak scaling: each rank owns one config-sized batch
    return range(rank * per, (rank + 1) * per), per * world, N, causal, "weak"


def make_inputs(slices, N, seed, device=None):
    from oracle.attention_oracle import make_qkv  # seeded host generator (shared with tests)

    q, k, v = make_qkv(1, len(slices), N, 64, seed=seed, slices=slices)
    shape = (1, len(slices), N, 64)
    return q.view(shape), k.view(shape), v.view(shape)


def run_ours(args):
    world, rank, local = dist_env()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    init_dist(world, "nccl")
    from flashlite_b200 import flash_attn_wmma as fa

    slices, total_slices, N, causal, scaling = rank_slices(args.workload, world, rank)
    S = len(slices)
    D = 64
    sm_scale = 0.125
    qh, kh, vh = make_inputs(slices, N, seed=0)
    set_bytes = 4 * qh.numel() * 2
    n_sets = max(2, math.ceil(3 * L2_BYTES / set_bytes))
    n_sets = min(n_sets, max(2, int(0.25 * torch.cuda.get_device_properties(device).total_memory // set_bytes)))
    sets = []
    for i in range(n_sets):
        if i == 0:
            q, k, v = (t.to(device) for t in (qh, kh, vh))
        else:  # distinct buffers, same values: keeps every step's bytes cold in L2
            q, k, v = (t.clone() for t in sets[0][:3])
        sets.append((q, k, v, torch.empty_like(q)))
    stream = torch.cuda.current_stream(device)

    def step(i):
        q, k, v, o = sets[i % n_sets]
        fa.forward_flash2(q, k, v, sm_scale, causal, out=o)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(device)
    barrier(world, device)
    torch.cuda.synchronize(device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index if device.index is not None else 0) as clk:
        ev0.record(stream)
        for i in range(args.steps):
            step(i)
        ev1.record(stream)
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

    # ---- end to end through the public API: pinned host in, host out ----
    # Every step copies its Q, K, V from pinned host memory and its O back.
    # Serial: copy in, compute, copy out, one after the other. Pipelined (the
    # reported e2e): two device buffer sets; step i+1's copies in run on a
    # copy stream while step i computes, step i's copy out on a third stream.
    qp, kp, vp = (t.pin_memory() for t in (qh, kh, vh))
    ops = [torch.empty_like(qh).pin_memory() for _ in range(2)]
    dbuf = [tuple(torch.empty_like(sets[0][0]) for _ in range(4)) for _ in range(2)]

    def e2e_serial(nsteps):
        dq, dk, dv, do = dbuf[0]
        for _ in range(nsteps):
            dq.copy_(qp, non_blocking=True)
            dk.copy_(kp, non_blocking=True)
            dv.copy_(vp, non_blocking=True)
            fa.forward_flash2(dq, dk, dv, sm_scale, causal, out=do)
            ops[0].copy_(do, non_blocking=True)

    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def e2e_pipelined(nsteps, start_ev):
        s_in.wait_event(start_ev)
        for i in range(nsteps):
            b = i % 2
            dq, dk, dv, do = dbuf[b]
            with torch.cuda.stream(s_in):
                if i >= 2:
                    s_in.wait_event(ev_done[b])  # step i-2 has read these inputs
                dq.copy_(qp, non_blocking=True)
                dk.copy_(kp, non_blocking=True)
                dv.copy_(vp, non_blocking=True)
                ev_in[b].record(s_in)
            stream.wait_event(ev_in[b])
            if i >= 2:
                stream.wait_event(ev_out[b])  # step i-2's output has been copied out
            fa.forward_flash2(dq, dk, dv, sm_scale, causal, out=do)
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

    peak_burst, peak_sust, hbm, peak_kind = measured_peaks()
    achieved = per_rank_flops / (ms_step * 1e-3) / 1e12  # per launch per GPU
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
            "data": "synthetic: seeded i.i.d. N(0,1) fp16 Q/K/V generated on host",
            "config": {
                "workload": desc,
                "B_per_rank": 1, "H_per_rank": S, "slices_total": total_slices,
                "N": N, "D": D, "causal": causal, "sm_scale": sm_scale,
                "parallelism": f"head-sharded x{world}, no collective" if world > 1 else "single GPU",
                "l2": f"{n_sets} rotating input sets, {n_sets * set_bytes / 2**20:.0f} MiB > 126 MB L2",
            },
            "pct_of_peak": round(100 * achieved / peak_burst, 2),
            "roofline": {
                "bound": "tensor", "achieved": round(achieved, 2), "peak": peak_burst,
                "unit": "TFLOP/s", "frac": round(achieved / peak_burst, 4),
                "peak_kind": f"{peak_kind} bf16 dense burst (sustained {peak_sust})",
                "traffic": traffic,
                "alg_bytes": 4 * S * N * D * 2,
            },
            "e2e": {"value": round(e2e_value, 2), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": 3 * qh.numel() * 2, "d2h_bytes_per_step": qh.numel() * 2,
                    "ms_per_step": round(e_ms, 4), "output_finite": bool(ok),
                    "mode": "pipelined: step i+1's host-to-device copies and step i-1's "
                            "device-to-host copy overlap step i's kernel (two buffer sets)",
                    "serial_value": round(e2e_serial_value, 2), "serial_ms_per_step": round(es_ms, 4)},
            "gpu_launches": args.steps,
            "clocks": clk.summary(),
            "device_error": int(err),
            "cpu_baseline": cpu,
        }
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

    B, H, N, D, causal, bwd, desc = EXT_WORKLOADS[args.workload]
    sm_scale = 0.0  # 1/sqrt(D)
    g = torch.Generator().manual_seed(7 + rank)
    host = [torch.randn(B, H, N, D, generator=g).half() for _ in range(4 if bwd else 3)]
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
    barrier(world, device)
    ms_step = max_over_ranks(ev0.elapsed_time(ev1), world, device) / args.steps
    err = fa.device_error()
    # FLOPs: forward 4·B·H·N²·D (halved causal); backward 2.5x that (five GEMMs to two)
    f_step = (2.5 if bwd else 1.0) * flops(B, H, N, D, causal)
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
            "metric": ("FA2 bwd" if bwd else "FA2 fwd") + f" TFLOP/s per B200 (fp16, D={D})",
            "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16 (fp32 accumulate)",
            "data": "synthetic: seeded i.i.d. N(0,1) fp16 inputs generated on host",
            "config": {"workload": desc, "B": B, "H": H, "N": N, "D": D, "causal": causal,
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
# config 5: sequence-sharded ring attention (strong scaling over ranks)
# ----------------------------------------------------------------------------
def run_ring(args):
    world, rank, local = dist_env()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    init_dist(world, "nccl")
    from flashlite_b200 import flash_attn_wmma as fa
    from flashlite_b200.parallel_attn import RingAttention, ZigzagRingAttention

    B, H, N, causal, desc = WORKLOADS["cfg5"]
    D, sm_scale = 64, 0.125
    # causal rings use the zig-zag layout (rank r holds chunks r and 2P-1-r of
    # 2P), which gives every rank the same work; --ring-layout contiguous keeps
    # one contiguous block per rank
    zigzag = world > 1 and causal and args.ring_layout == "zigzag"
    assert N % (2 * world) == 0
    nb = N // world
    shape = (2, B, H, nb // 2, D) if zigzag else (B, H, nb, D)
    g = torch.Generator(device=device).manual_seed(1000 + rank)
    q, k, v = ((torch.randn(*shape, generator=g, device=device) * 0.5).to(torch.float16)
               for _ in range(3))
    out = torch.empty_like(q)
    o_acc = torch.empty(*shape, dtype=torch.float32, device=device)
    lse = torch.empty(*shape[:-1], dtype=torch.float32, device=device)
    ring = (ZigzagRingAttention() if zigzag else RingAttention()) if world > 1 else None
    flush = torch.empty(256 * 2**20, dtype=torch.uint8, device=device)

    def step():
        if ring is None:
            fa.forward_flash2(q, k, v, sm_scale, causal, out=out)
        else:
            ring.forward(q, k, v, sm_scale, causal, out=out, o_acc=o_acc, lse=lse)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    barrier(world, device)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    with ClockSampler(device.index) as clk:
        for a, b in evs:
            flush.zero_()  # untimed: evicts this rank's blocks from L2
            a.record()
            step()
            b.record()
        torch.cuda.synchronize(device)
    barrier(world, device)
    ms_local = sum(a.elapsed_time(b) for a, b in evs)
    ms = max_over_ranks(ms_local, world, device)
    ms_step = ms / args.steps
    total_flops = flops(B, H, N, D, causal)
    value = total_flops / (ms_step * 1e-3) / 1e12

    # end to end: this rank's blocks from pinned host memory, output back
    qp, kp, vp = (t.cpu().pin_memory() for t in (q, k, v))
    op = torch.empty_like(qp).pin_memory()

    def e2e_step():
        q.copy_(qp, non_blocking=True)
        k.copy_(kp, non_blocking=True)
        v.copy_(vp, non_blocking=True)
        step()
        op.copy_(out, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize(device)
    barrier(world, device)
    e_steps = max(2, min(args.steps, 5))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e_steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize(device)
    e_ms = max_over_ranks(e0.elapsed_time(e1) / e_steps, world, device)
    err = fa.device_error()
    peak_burst, peak_sust, _, peak_kind = measured_peaks()
    per_gpu = value / world
    if rank == 0:
        line = {
            "metric": "FA2 fwd TFLOP/s per B200 (fp16, D=64)", "value": round(value, 2),
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp16 (fp32 accumulate)",
            "data": "synthetic: seeded i.i.d. N(0,1)*0.5 fp16 Q/K/V generated per rank on device",
            "config": {"workload": desc, "B": B, "H": H, "N": N, "D": D, "causal": True,
                       "rows_per_rank": nb,
                       "parallelism": (f"ring x{world} (NCCL send/recv), "
                                       f"{'zig-zag' if zigzag else 'contiguous'} layout")
                       if world > 1 else "single GPU",
                       "l2": "256 MiB buffer written between timed steps (untimed)"},
            "pct_of_peak": round(100 * per_gpu / peak_burst, 2),
            "roofline": {"bound": "tensor", "achieved": round(per_gpu, 2), "peak": peak_burst,
                         "unit": "TFLOP/s", "frac": round(per_gpu / peak_burst, 4),
                         "peak_kind": f"{peak_kind} bf16 dense burst (sustained {peak_sust})",
                         "traffic": None,
                         "note": "per GPU" + ("; causal contiguous blocks cap the ideal ring speedup at P^2/(2P-1)"
                                           if world > 1 and causal and not zigzag else "")},
            "e2e": {"value": round(total_flops / (e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": 3 * q.numel() * 2, "d2h_bytes_per_step": q.numel() * 2,
                    "ms_per_step": round(e_ms, 3)},
            "gpu_launches": args.steps * (world if world > 1 else 1),
            "clocks": clk.summary(),
            "device_error": int(err),
        }
        print(json.dumps(line), flush=True)
    if ring is not None:
        del ring
    if world > 1:
        torch.distributed.destroy_process_group()


# ----------------------------------------------------------------------------
# CPU baseline (oracle port, torch fp32 on host cores)
# ----------------------------------------------------------------------------
def cpu_step(workload):
    """One bounded CPU sample of the workload: (callable, FLOPs, description).

    torch fp32 matmul-softmax-matmul (the oracle port). Config 5 is sampled
    by query rows (its full score matrix would need 64 GB): the last 256 rows
    of one head, each attending to its whole causal prefix."""
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
    n_slices = {"cfg2": 16, "cfg2c": 16, "cfg3": 4, "cfg3c": 4, "cfg4": 1}[workload]
    q, k, v = make_qkv(1, n_slices, N, 64, seed=0)
    return (lambda: attention_fp32(q, k, v, 0.125, causal), flops(1, n_slices, N, 64, causal),
            f"{n_slices} of the workload's (b,h) slices (N={N}, causal={causal})")


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
    t = sorted(ts)[len(ts) // 2]
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
                   "D": 64, "causal": causal},
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
    comparator (benchmarks/benchmark_throughput.py:99-104), on this GPU."""
    if not torch.cuda.is_available():
        return {"unavailable": "no GPU"}
    from oracle import build_ref

    B, H, N, causal, _ = WORKLOADS[workload]
    if workload == "cfg4":
        return {"unavailable": "not timed for cfg4"}
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(0)
    q, k, v = (torch.randn(B, H, N, 64, device=dev, dtype=torch.float16, generator=g) for _ in range(3))
    out = torch.empty_like(q)
    f = flops(B, H, N, 64, causal)

    def median_ms(fn, warm=25, runs=100):  # benchmarks/benchmark_throughput.py:34-54
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        es = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(runs)]
        for a, b in es:
            a.record()
            fn()
            b.record()
        torch.cuda.synchronize()
        ts = sorted(a.elapsed_time(b) for a, b in es)
        return ts[len(ts) // 2]

    res = {"timing": "median of 100 after 25 warm-up, L2 warm (the reference benchmark's method)"}
    mod = build_ref.load()
    if mod is None:
        res["wmma"] = {"unavailable": "oracle/_ref not built"}
    else:
        ms = median_ms(lambda: mod.forward_flash2(q, k, v, 0.125, causal, out=out))
        res["wmma"] = {"ms": round(ms, 4), "tflops": round(f / ms / 1e9, 2)}
    try:
        from torch.nn.attention import SDPBackend, sdpa_kernel
        import torch.nn.functional as F

        def sdpa():
            with sdpa_kernel([SDPBackend.FLASH_ATTENTION]):
                return F.scaled_dot_product_attention(q, k, v, is_causal=causal, scale=0.125)

        ms = median_ms(sdpa)
        res["sdpa_flash"] = {"ms": round(ms, 4), "tflops": round(f / ms / 1e9, 2)}
    except Exception as exc:  # backend may be unavailable
        res["sdpa_flash"] = {"unavailable": str(exc)[:120]}
    from flashlite_b200 import flash_attn_wmma as fa

    ms = median_ms(lambda: fa.forward_flash2(q, k, v, 0.125, causal, out=out))
    res["flashlite_b200_same_method"] = {"ms": round(ms, 4), "tflops": round(f / ms / 1e9, 2)}
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="cfg3", choices=sorted(WORKLOADS) + sorted(EXT_WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ring-layout", default="zigzag", choices=["zigzag", "contiguous"],
                    help="sequence layout of the config-5 ring on 2+ GPUs")
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
