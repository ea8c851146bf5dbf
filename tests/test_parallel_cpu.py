"""CPU tests of the multi-GPU host logic over gloo ranks (no GPU needed).

* head sharding: shard_range splits (b,h) slices contiguously and evenly;
* ring attention: RingAttention's schedule, double-buffered send/recv and
  merge order, run on world sizes 2 and 4 with a host implementation of the
  block step, reproduce full attention of every rank's query block;
* zig-zag ring: every rank holds chunks r and 2P-1-r, computes the same
  number of key blocks, and reproduces full attention of its two chunks;
* failure: a rank that raises before the ring leaves the others with an
  error from the process group's timeout, not a hang.
"""
import datetime
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flashlite_b200.parallel_attn import (RingAttention, ZigzagRingAttention, ring_schedule,
                                          shard_range, zigzag_chunks, zigzag_pairs)
from oracle.attention_oracle import attention_fp32, block_attention_lse, merge_lse


def cpu_block_fn(q, k, v, o_acc, lse, q_offset, kv_offset, sm_scale, is_causal, first):
    """Host stand-in for the CUDA forward_block (same contract)."""
    o_b, l_b = block_attention_lse(q, k, v, q_offset, kv_offset, sm_scale, is_causal)
    if first:
        o_acc.copy_(o_b)
        lse.copy_(l_b)
    else:
        o_m, l_m = merge_lse(o_acc, lse, o_b, l_b)
        o_acc.copy_(o_m)
        lse.copy_(l_m)


def cpu_finalize_fn(o_acc, out):
    out.copy_(o_acc.to(out.dtype))


def test_shard_range_even_and_ragged():
    assert [len(shard_range(512, 8, r)) for r in range(8)] == [64] * 8
    assert shard_range(512, 8, 3) == range(192, 256)
    parts = [shard_range(10, 4, r) for r in range(4)]
    assert [len(p) for p in parts] == [3, 3, 2, 2]
    assert sum(len(p) for p in parts) == 10 and parts[-1].stop == 10
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_ring_schedule():
    assert ring_schedule(0, 4, True) == [(0, True), (3, False), (2, False), (1, False)]
    assert ring_schedule(2, 4, True) == [(2, True), (1, True), (0, True), (3, False)]
    assert all(c for _, c in ring_schedule(1, 3, False))


def test_zigzag_schedule_is_balanced():
    for world in (2, 4, 8):
        assert sorted(c for r in range(world) for c in zigzag_chunks(r, world)) == list(range(2 * world))
        work = []
        for r in range(world):
            pairs = [zigzag_pairs(r, (r - s) % world, world, True) for s in range(world)]
            assert all(len(p) == 2 for p in pairs[1:])   # equal work at every later step
            work.append(sum(len(p) for p in pairs))
        assert len(set(work)) == 1
        assert all(len(zigzag_pairs(r, s, world, False)) == 4 for r in range(world) for s in range(world))


def _zigzag_worker(rank, world, port, causal, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=30))
        torch.manual_seed(0)
        c, H, D = 12, 2, 16
        q, k, v = (torch.randn(1, H, 2 * world * c, D) for _ in range(3))
        full = attention_fp32(q, k, v, 0.25, causal)
        own = zigzag_chunks(rank, world)
        pick = lambda t: torch.stack([t[:, :, i * c:(i + 1) * c] for i in own]).contiguous()
        ring = ZigzagRingAttention(block_fn=cpu_block_fn, finalize_fn=cpu_finalize_fn)
        out = ring.forward(pick(q), pick(k), pick(v), 0.25, causal)
        out2 = ring.forward(pick(q), pick(k), pick(v), 0.25, causal)  # buffers reused
        err = max((out - pick(full)).abs().max().item(), (out2 - out).abs().max().item())
        results[rank] = err
        dist.destroy_process_group()
    except Exception:  # report, never hang the parent
        results[rank] = traceback.format_exc()


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("causal", [True, False])
def test_zigzag_ring_attention_gloo(world, causal):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_zigzag_worker, args=(r, world, port, causal, results))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0, "zig-zag ring worker did not finish"
    for r in range(world):
        assert isinstance(results[r], float), results[r]
        assert results[r] < 1e-5, (r, results[r])


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _ring_worker(rank, world, port, causal, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=30))
        torch.manual_seed(0)
        nb, H, D = 24, 2, 16
        q, k, v = (torch.randn(1, H, nb * world, D) for _ in range(3))
        full = attention_fp32(q, k, v, 0.25, causal)
        sl = slice(rank * nb, (rank + 1) * nb)
        ring = RingAttention(block_fn=cpu_block_fn, finalize_fn=cpu_finalize_fn)
        out = ring.forward(q[:, :, sl].contiguous(), k[:, :, sl].contiguous(),
                           v[:, :, sl].contiguous(), 0.25, causal,
                           out=torch.empty(1, H, nb, D))
        err = (out - full[:, :, sl]).abs().max().item()
        results[rank] = err
        dist.destroy_process_group()
    except Exception:  # report, never hang the parent
        results[rank] = traceback.format_exc()


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("causal", [False, True])
def test_ring_attention_gloo(world, causal):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_ring_worker, args=(r, world, port, causal, results))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0, "ring worker did not finish"
    for r in range(world):
        assert isinstance(results[r], float), results[r]
        assert results[r] < 1e-5, (r, results[r])


def _failing_worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        results[rank] = "raised"
        raise SystemExit(0)  # leaves between steps, before the ring starts
    try:
        q = torch.zeros(1, 1, 8, 4)
        RingAttention(block_fn=cpu_block_fn, finalize_fn=cpu_finalize_fn).forward(
            q, q.clone(), q.clone(), 0.5, True)
        results[rank] = "completed"
    except Exception as exc:  # the expected outcome: an error, not a hang
        results[rank] = "error: " + type(exc).__name__


def test_ring_peer_failure_is_an_error_not_a_hang():
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("a surviving rank hung instead of raising")
    assert results[1] == "raised"
    assert str(results[0]).startswith("error"), results[0]


def test_bench_reference_arm_for_extensions_is_unavailable():
    # the backward and head_dim-128 workloads have no reference counterpart:
    # the reference arm prints its `unavailable` line and exits 0
    import json
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    for w in ("bwd3", "d128_3"):
        r = subprocess.run([sys.executable, str(root / "bench.py"), "--impl", "reference", "--workload", w,
                            "--steps", "1", "--warmup", "3"], capture_output=True, text=True, timeout=300,
                           cwd=str(root))
        assert r.returncode == 0, r.stderr
        line = json.loads(r.stdout.strip().splitlines()[-1])
        assert line["impl"] == "reference" and "unavailable" in line
