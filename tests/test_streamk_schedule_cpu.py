"""Bookkeeping of the stream-K schedule, checked on the CPU.

csrc/fl_flash2_sk.cu gives CTA c of G the KV steps [c S / G, (c+1) S / G) of
the S = units * n_ktiles steps laid end to end (sk_range), walks them as
segments of single units (sk_seg), finds the CTA that holds a step by
sk_cta_of, stores the pieces of a unit cut between CTAs in slots
(c, first or last segment of c, tile) and counts their arrivals in a word per
(CTA holding the unit's first step, tile). The merge is correct only if the
ranges partition the steps, the slots of all pieces in flight are distinct,
each counter word belongs to one cut unit, and no unit has more pieces than
the 8-bit arrival count holds. This test restates those integer formulas and
checks the invariants over many grid sizes; the GPU tests check the outputs.
"""
import random


def sk_range(total, grid, c):
    return total * c // grid, total * (c + 1) // grid


def sk_cta_of(total, grid, x):
    return ((x + 1) * grid - 1) // total


def segments(total, grid, nkv, c):
    w, w_end = sk_range(total, grid, c)
    out = []
    while w < w_end:
        u, k0 = divmod(w, nkv)
        k1 = min(nkv, k0 + (w_end - w))
        out.append((u, k0, k1))
        w += k1 - k0
    return out


def check(units, nkv, sms=148):
    total = units * nkv
    grid = min(sms, total)  # launch_flash2_sk: every CTA gets a step
    seen = [0] * total
    slots, counters, pieces = {}, {}, {}
    for c in range(grid):
        segs = segments(total, grid, nkv, c)
        assert segs, "every CTA has a step"
        if units >= sms:  # the only grids launch_flash2 sends here
            assert len(segs) <= 3 or all(k0 == 0 and k1 == nkv for (_, k0, k1) in segs[1:-1])
        for si, (u, k0, k1) in enumerate(segs):
            for k in range(k0, k1):
                seen[u * nkv + k] += 1
            if k0 == 0 and k1 == nkv:
                continue  # a whole unit: stored directly
            u0 = u * nkv
            c_first = sk_cta_of(total, grid, u0)
            m = sk_cta_of(total, grid, u0 + nkv - 1) - c_first + 1
            pc = c - c_first
            assert 0 <= pc < m and m >= 2
            assert m <= 255, "arrival count is 8 bits"
            # the kernel's slot_of: first (0) or last (1) segment of the piece's CTA
            last_seg = 1 if (pc == 0 and total * c // grid != u0) else 0
            # the formula agrees with the CTA's own view: slot 1 iff not its first segment
            assert last_seg == (1 if si > 0 else 0)
            for tile in (0, 1):
                slot = (c * 2 + last_seg) * 2 + tile
                assert slot < 4 * grid
                assert slot not in slots, (units, nkv, c, slot)
                slots[slot] = (u, pc)
                key = c_first * 2 + tile
                assert counters.setdefault(key, u) == u, "one cut unit per counter word"
                assert key < 2 * grid
            pieces.setdefault(u, set()).add(pc)
    assert all(v == 1 for v in seen), "ranges partition the steps"
    for u, pcs in pieces.items():
        u0 = u * nkv
        m = sk_cta_of(total, grid, u0 + nkv - 1) - sk_cta_of(total, grid, u0) + 1
        assert pcs == set(range(m)), "every piece of a cut unit is stored once"


def test_cta_of_inverts_range():
    rng = random.Random(1)
    for _ in range(2000):
        grid = rng.randint(1, 300)
        total = rng.randint(grid, 100_000)
        for _ in range(20):
            x = rng.randrange(total)
            c = sk_cta_of(total, grid, x)
            lo, hi = sk_range(total, grid, c)
            assert lo <= x < hi


def test_schedule_invariants_on_launched_shapes():
    # units >= SMs (two query tiles per CTA): the grids launch_flash2 sends to stream-K
    for units, nkv in [(256, 32), (320, 32), (224, 32), (512, 64), (150, 2), (296, 4), (149, 1),
                       (375, 9), (148, 7), (1000, 3), (161, 64)]:
        check(units, nkv)
    rng = random.Random(7)
    for _ in range(300):
        check(rng.randint(148, 3000), rng.randint(1, 80))


def test_schedule_invariants_other_sm_counts():
    rng = random.Random(9)
    for _ in range(200):
        sms = rng.randint(1, 200)
        check(rng.randint(sms, sms * 6), rng.randint(1, 40), sms)
