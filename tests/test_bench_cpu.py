"""Host-side logic of bench.py (no GPU): seeded inputs that do not depend on
sharding, the config-4 shard ranges, the config-5 ring layouts, and the
reference arm loading no code of this package."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def test_dev_slices_do_not_depend_on_sharding():
    full = bench.dev_slices(range(6), 64, seed=3, device="cpu")
    part = bench.dev_slices(range(2, 5), 64, seed=3, device="cpu")
    for f, p in zip(full, part):
        assert torch.equal(f[2:5], p)
    assert not torch.equal(full[0], full[1])  # q and k differ


def test_dev_rows_do_not_depend_on_sharding():
    H = 3
    full = bench.dev_rows(0, 4 * bench.RING_BLOCK, H, seed=5, device="cpu", scale=0.5)
    part = bench.dev_rows(bench.RING_BLOCK, 2 * bench.RING_BLOCK, H, seed=5, device="cpu", scale=0.5)
    one = bench.dev_rows(0, 4 * bench.RING_BLOCK, H, seed=5, device="cpu", scale=0.5, heads=[2])
    for f, p, o in zip(full, part, one):
        assert torch.equal(f[:, :, bench.RING_BLOCK:3 * bench.RING_BLOCK], p)
        assert torch.equal(f[:, 2:3], o)
    assert abs(float(full[0].float().std()) - 0.5) < 0.02


def test_cfg4_slices_cover_512_once_at_every_world_size():
    for world in (1, 2, 4, 8):
        seen = []
        for r in range(world):
            sl, total, N, causal, scaling = bench.rank_slices("cfg4", world, r)
            assert (total, N, causal, scaling) == (512, 8192, True, "strong")
            seen.extend(sl)
        assert seen == list(range(512))


def test_weak_scaling_keeps_config3_per_rank():
    for world in (1, 8):
        sl, total, N, causal, scaling = bench.rank_slices("cfg3", world, world - 1)
        assert len(sl) == 16 and total == 16 * world and scaling == "weak" and N == 4096


def test_ring_layout_rows_cover_the_sequence():
    """Contiguous and zig-zag layouts give every global row to exactly one rank."""
    from flashlite_b200.parallel_attn import zigzag_chunks

    N = 16 * bench.RING_BLOCK
    for world in (2, 4, 8):
        cont, zz = [], []
        nb = N // world
        c = N // (2 * world)
        for r in range(world):
            cont.extend(range(r * nb, (r + 1) * nb))
            for ch in zigzag_chunks(r, world):
                zz.extend(range(ch * c, (ch + 1) * c))
        assert sorted(cont) == list(range(N)) and sorted(zz) == list(range(N))


def test_cpu_step_runs_configs_1_to_3_in_full():
    for w in ("cfg1", "cfg2", "cfg3"):
        _, f, desc = bench.cpu_step(w)
        B, H, N, causal, _ = bench.WORKLOADS[w]
        assert f == bench.flops(B, H, N, 64, causal)
        assert desc.startswith("all ")


def test_reference_arm_loads_no_package_code():
    code = (
        "import sys, json, argparse; sys.path.insert(0, %r); import bench\n"
        "a = argparse.Namespace(workload='cfg1', steps=1, warmup=3, impl='reference')\n"
        "bench.run_reference(a)\n"
        "assert not [m for m in sys.modules if m.startswith('flashlite_b200')], 'package loaded'\n"
    ) % str(ROOT)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300,
                       env={"CUDA_VISIBLE_DEVICES": "", "PATH": "/usr/bin:/bin"})
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["config"]["same_config"] is True
    assert line["value"] > 0 and line["e2e"]["h2d_bytes_per_step"] == 0


def test_failed_leg_is_reported_in_its_own_entry():
    def broken(*_):
        raise RuntimeError("leg failed")

    assert bench._leg(broken, 1, 2) == {"error": "RuntimeError: leg failed"}
    assert bench._leg(lambda a, b: {"ok": a + b}, 1, 2) == {"ok": 3}


def test_ring_breakdown_names_the_limit():
    # 4 ranks of a contiguous causal ring: the light ranks wait on their
    # neighbours, the busiest hardly at all -> imbalance, not the exchange
    per = [[1.5, 6.3], [4.0, 4.0], [7.0, 1.2], [9.8, 0.3]]
    out = bench.ring_breakdown(per, 11.0)
    assert out["busiest_rank"] == 3 and out["limiting_step"].startswith("causal load imbalance")
    # the busiest rank waits > 10 % of the step: the exchange is exposed
    assert bench.ring_breakdown([[9.8, 2.0], [9.5, 0.1]], 11.0)["limiting_step"].startswith("K/V exchange")
    # balanced, hidden exchange: block compute
    assert bench.ring_breakdown([[6.4, 0.01], [6.5, 0.01]], 6.5)["limiting_step"].startswith("block compute")


def test_leg_parity_check_flags_a_wrong_output():
    """The legs' row check against the oracle: exact rows pass, a mistake
    planted in the compared output (on the CPU) fails the tolerance."""
    from oracle.attention_oracle import attention_rows_fp32

    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(1, 512, 64, generator=g).half() for _ in range(3))
    rows = torch.tensor([0, 100, 511])
    good = attention_rows_fp32(q, k, v, rows, 0.125, True).half()
    e = bench.row_errors(good, q, k, v, rows, 0.125, True)
    ok = bench.reduce_errors([e], 1, None)
    assert ok["ok"] and ok["values_checked"] == 3 * 64
    bad = good.clone()
    bad[0, 1, 5] += 0.01
    assert not bench.reduce_errors([bench.row_errors(bad, q, k, v, rows, 0.125, True)], 1, None)["ok"]
