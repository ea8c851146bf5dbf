"""GPU parity of the stream-K schedule (csrc/fl_flash2_sk.cu) against the oracle.

Non-causal head_dim-64 grids with more units (pairs of 128-row query tiles)
than SMs, whose last wave would leave SMs idle, run as stream-K: each CTA
takes an equal share of the concatenated KV steps, and a unit cut between
two CTAs is merged by whichever piece finishes last. Covered: shapes the cost
model sends there, ragged key and query lengths, an odd number of query
tiles (a unit with one tile), the LSE output, the [B, N, H, D] layout, shapes
it would not pick run in the forced mode (FL_STREAMK=2, in a subprocess:
BASELINE config 3, tails of a few steps per CTA, units that are never cut,
units without a second tile), repeatability, graph capture (with and without
a workspace for the capturing stream), concurrent streams and the cap on
cached workspaces. Same tolerance as
forward_flash2: max-abs <= 2e-3, mean-abs <= 2e-4 against fp32 attention.
"""
import os
import subprocess
import sys
import threading
from pathlib import Path

import pytest
import torch

from flashlite_b200 import flash_attn_wmma as fa
from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def _check(out, ref, tag):
    assert not torch.isnan(out.float()).any(), f"NaN in output {tag}"
    mx, mean = orc.error_metrics(out, ref)
    assert mx <= orc.MAX_ABS_TOL and mean <= orc.MEAN_ABS_TOL, f"{tag}: max-abs {mx:.3e} mean-abs {mean:.3e}"


@pytest.mark.parametrize("B,H,N", [
    (1, 14, 4096),  # 224 units on 148 SMs (1.51 waves)
    (1, 20, 4096),  # 2.16 waves
    (1, 20, 4000),  # ragged keys and queries
    (1, 20, 3968),  # 31 query tiles: each slice's last unit has one tile
    (1, 6, 8192),   # 64-step units, 1.30 waves
    (3, 9, 2944),   # 23 query tiles, 27 slices
], ids=lambda v: str(v))
def test_streamk_shapes(cuda, B, H, N):
    q, k, v = orc.make_qkv(B, H, N, 64, seed=N + H)
    ref = orc.attention_fp32(q, k, v, 0.125, False)
    out = fa.forward_flash2(q.to(cuda), k.to(cuda), v.to(cuda), 0.125, False)
    torch.cuda.synchronize()
    assert fa.device_error() == 0
    _check(out.cpu(), ref, f"B{B} H{H} N{N}")


def test_streamk_lse_and_ex(cuda):
    """forward_flash2_ex with N_k != N_q and the LSE output, on a stream-K grid."""
    B, H, Nq, Nk = 1, 20, 4096, 3000
    q, _, _ = orc.make_qkv(B, H, Nq, 64, seed=3)
    _, k, v = orc.make_qkv(B, H, Nk, 64, seed=4)
    o_ref, lse_ref = orc.block_attention_lse(q, k, v, 0, 0, 0.125, False)
    out, lse = fa.forward_flash2_ex(q.to(cuda), k.to(cuda), v.to(cuda), 0.125, False, return_lse=True)
    torch.cuda.synchronize()
    assert fa.device_error() == 0
    _check(out.cpu(), o_ref, "ex")
    assert (lse.cpu() - lse_ref).abs().max().item() < 1e-3


def test_streamk_repeatable(cuda):
    """The piece that merges a cut unit varies from run to run; the bits do not."""
    q, k, v = (t.to(cuda) for t in orc.make_qkv(1, 20, 4096, 64, seed=8))
    first = fa.forward_flash2(q, k, v, 0.125, False)
    for _ in range(5):
        again = fa.forward_flash2(q, k, v, 0.125, False)
        torch.cuda.synchronize()
        assert torch.equal(first, again)


def test_streamk_concurrent_streams(cuda):
    """Each stream has its own workspace: four threads on four streams give
    the single-stream bits."""
    q, k, v = (t.to(cuda) for t in orc.make_qkv(1, 20, 4096, 64, seed=12))
    ref = fa.forward_flash2(q, k, v, 0.125, False)
    torch.cuda.synchronize()
    results, errors = [None] * 4, []

    def work(i):
        try:
            s = torch.cuda.Stream(cuda)
            with torch.cuda.stream(s):
                outs = [fa.forward_flash2(q, k, v, 0.125, False) for _ in range(20)]
            s.synchronize()
            results[i] = outs[-1]
        except Exception as e:  # surfaced in the main thread below
            errors.append(e)

    threads = [threading.Thread(target=work, args=(i,)) for i in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    assert fa.device_error() == 0
    for r in results:
        assert torch.equal(r, ref)


def test_streamk_graph_capture(cuda):
    """A stream that already has a workspace captures the stream-K launch
    (replays give the eager bits); a stream without one captures the
    one-unit-per-CTA launch (no allocation while capturing), which agrees
    within the tolerance."""
    q, k, v = (t.to(cuda) for t in orc.make_qkv(1, 20, 4096, 64, seed=14))
    s = torch.cuda.Stream(cuda)
    with torch.cuda.stream(s):
        eager = fa.forward_flash2(q, k, v, 0.125, False)
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        out = fa.forward_flash2(q, k, v, 0.125, False)
    for _ in range(3):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
    fresh = torch.cuda.Stream(cuda)
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2, stream=fresh):
        out2 = fa.forward_flash2(q, k, v, 0.125, False)
    g2.replay()
    torch.cuda.synchronize()
    assert fa.device_error() == 0
    mx, mean = orc.error_metrics(out2.cpu(), eager.cpu().float())
    assert mx <= orc.MAX_ABS_TOL and mean <= orc.MEAN_ABS_TOL


_FORCED = r"""
import sys, torch
sys.path.insert(0, {root!r})
from flashlite_b200 import flash_attn_wmma as fa
from oracle import attention_oracle as orc
for (B, H, N) in [(2, 8, 4096), (1, 150, 256), (1, 148, 512), (1, 75, 1152), (1, 149, 128), (2, 8, 1000)]:
    q, k, v = orc.make_qkv(B, H, N, 64, seed=B + H + N)
    ref = orc.attention_fp32(q, k, v, 0.125, False)
    out = fa.forward_flash2(q.cuda(), k.cuda(), v.cuda(), 0.125, False)
    again = fa.forward_flash2(q.cuda(), k.cuda(), v.cuda(), 0.125, False)
    torch.cuda.synchronize()
    assert fa.device_error() == 0, (B, H, N)
    assert torch.equal(out, again), (B, H, N)
    mx, mean = orc.error_metrics(out.cpu(), ref)
    assert mx <= orc.MAX_ABS_TOL and mean <= orc.MEAN_ABS_TOL, (B, H, N, mx, mean)
print("forced stream-K ok")
"""


def test_streamk_forced_small_tails(cuda):
    """FL_STREAMK=2 takes stream-K wherever a grid has more units than SMs:
    config 3 (which the cost model leaves on one unit per CTA), 150 units of
    2 steps (CTAs of 2 or 3 steps, units cut in two), 296 units that split
    into whole units only, units with one query tile (N = 128 and 1152), and
    a grid of one tile per CTA that keeps its own schedule."""
    env = dict(os.environ, FL_STREAMK="2")
    r = subprocess.run([sys.executable, "-c", _FORCED.format(root=str(ROOT))], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "forced stream-K ok" in r.stdout


def test_streamk_workspaces_are_capped(cuda):
    """A caller that makes a new stream per request: at most 8 streams per
    device keep a stream-K workspace (19.7 MB each); calls on further streams
    run the one-unit-per-CTA schedule. Every result stays correct and the
    library's device memory stays bounded."""
    B, H, N = 1, 20, 4096
    q, k, v = orc.make_qkv(B, H, N, 64, seed=21)
    ref = orc.attention_fp32(q, k, v, 0.125, False)
    qd, kd, vd = (t.to(cuda) for t in (q, k, v))
    outs = [torch.empty_like(qd) for _ in range(12)]
    streams = [torch.cuda.Stream(cuda) for _ in range(12)]
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(cuda)[0]
    for s, o in zip(streams, outs):
        with torch.cuda.stream(s):
            fa.forward_flash2(qd, kd, vd, 0.125, False, out=o)
    torch.cuda.synchronize()
    grown = free0 - torch.cuda.mem_get_info(cuda)[0]
    assert fa.device_error() == 0
    assert grown <= 8 * 20 * 2**20 + (4 << 20), f"device memory grew by {grown / 2**20:.1f} MiB"
    for i, o in enumerate(outs):
        _check(o.cpu(), ref, f"stream {i}")


def test_streamk_bnhd_layout(cuda):
    """The [B, N, H, D] layout on a stream-K grid gives the [B, H, N, D] bits
    (same cut points; only the tensor maps' strides differ), LSE included."""
    B, H, N = 1, 20, 4096
    q, k, v = (t.to(cuda) for t in orc.make_qkv(B, H, N, 64, seed=23))
    ref, lse_ref = fa.forward_flash2_ex(q, k, v, 0.125, False, return_lse=True)
    qt, kt, vt = (t.transpose(1, 2).contiguous() for t in (q, k, v))
    out, lse = fa.forward_flash2_ex(qt, kt, vt, 0.125, False, return_lse=True, layout="bnhd")
    torch.cuda.synchronize()
    assert fa.device_error() == 0
    assert torch.equal(out.transpose(1, 2), ref)
    assert torch.equal(lse, lse_ref)
