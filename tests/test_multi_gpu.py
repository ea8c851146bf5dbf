"""Head sharding, ring and zig-zag ring attention on 2+ GPUs over NCCL (one
process per GPU).

The CPU suite covers the same host logic with gloo ranks
(test_parallel_cpu.py); this file runs the CUDA kernels with real NCCL
send/recv between GPUs and compares every rank's rows against the CPU fp32
oracle of the whole sequence. Skipped on a box with fewer than two GPUs.
"""
import os
import socket
from datetime import timedelta

import pytest
import torch

from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu

H, N, D = 4, 1536, 64


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, causal, results):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        from flashlite_b200.parallel_attn import (RingAttention, ZigzagRingAttention,
                                                  head_sharded_forward, shard_range, zigzag_chunks)

        q, k, v = (t.to(dev) for t in orc.make_qkv(1, H, N, D, seed=31))
        nb = N // world
        rows = slice(rank * nb, (rank + 1) * nb)
        blk = [t[:, :, rows].contiguous() for t in (q, k, v)]
        ring = RingAttention()
        ring_out = ring.forward(*blk, 0.125, causal)
        ring_out2 = ring.forward(*blk, 0.125, causal)  # second call reuses the ring buffers
        heads = shard_range(H, world, rank)
        hs = [t[:, heads.start:heads.stop].contiguous() for t in (q, k, v)]
        head_out = head_sharded_forward(*hs, 0.125, causal)
        # zig-zag layout: chunks r and 2P-1-r of 2P
        c = N // (2 * world)
        own = zigzag_chunks(rank, world)
        zz = [torch.stack([t[:, :, i * c:(i + 1) * c] for i in own]).contiguous() for t in (q, k, v)]
        zz_out = ZigzagRingAttention().forward(*zz, 0.125, causal)
        torch.cuda.synchronize()
        dist.barrier()
        results.put((rank, ring_out.cpu(), ring_out2.cpu(), head_out.cpu(), zz_out.cpu()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("causal", [False, True])
def test_ring_and_head_sharding_match_oracle(causal):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, causal, results))
             for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(world):
            rank, a, b, c, z = results.get(timeout=240)
            got[rank] = (a, b, c, z)
    finally:
        for p in procs:
            p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]

    q, k, v = orc.make_qkv(1, H, N, D, seed=31)
    ref = orc.attention_fp32(q, k, v, 0.125, causal)
    nb = N // world
    cz = N // (2 * world)
    for rank, (ring_out, ring_out2, head_out, zz_out) in got.items():
        for a, ch in enumerate((rank, 2 * world - 1 - rank)):
            mx, mean = orc.error_metrics(zz_out[a], ref[:, :, ch * cz:(ch + 1) * cz])
            assert mx <= orc.MAX_ABS_TOL and mean <= orc.MEAN_ABS_TOL, ("zigzag", rank, a, mx, mean)
        want = ref[:, :, rank * nb:(rank + 1) * nb]
        mx, mean = orc.error_metrics(ring_out, want)
        assert mx <= orc.MAX_ABS_TOL and mean <= orc.MEAN_ABS_TOL, (rank, mx, mean)
        assert torch.equal(ring_out, ring_out2)
        heads = range(rank * H // world, (rank + 1) * H // world)
        mx, mean = orc.error_metrics(head_out, ref[:, heads.start:heads.stop])
        assert mx <= orc.MAX_ABS_TOL and mean <= orc.MEAN_ABS_TOL, (rank, mx, mean)
