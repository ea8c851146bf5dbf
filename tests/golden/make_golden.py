"""Generate the golden vectors in this directory.

Each golden_*.npz holds seeded fp16 inputs (regenerable from ``seed`` and
``input_scale`` with oracle.attention_oracle.make_qkv), the scale and causal
flag, and the fp32 attention output computed in float64 and rounded to fp32
(independent of the fp32 oracle's own summation order). Shapes follow the
BASELINE configs that a CPU finishes in milliseconds plus the edge cases the
reference never tested (odd N, N < 64).

Run from the repository root:  python tests/golden/make_golden.py
"""
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle.attention_oracle import make_qkv  # noqa: E402

CASES = [
    # name, B, H, N, D, seed, input_scale, sm_scale, causal
    ("cfg1_b1h2n128", 1, 2, 128, 64, 0, 1.0, 0.125, False),
    ("b1h2n128_causal", 1, 2, 128, 64, 0, 1.0, 0.125, True),
    ("b2h1n200_causal", 2, 1, 200, 64, 11, 1.0, 0.125, True),
    ("b1h1n37", 1, 1, 37, 64, 12, 1.0, 0.0, False),
    ("b1h2n256_half_scale_causal", 1, 2, 256, 64, 13, 0.5, 0.125, True),
]


def exact(q, k, v, scale, causal):
    qd, kd, vd = (t.to(torch.float64) for t in (q, k, v))
    s = qd @ kd.transpose(-2, -1) * scale
    if causal:
        n = s.shape[-1]
        s = s.masked_fill(torch.ones(n, n, dtype=torch.bool).triu(1), float("-inf"))
    return (torch.softmax(s, -1) @ vd).to(torch.float32)


def main():
    for name, B, H, N, D, seed, iscale, sm, causal in CASES:
        q, k, v = make_qkv(B, H, N, D, seed=seed, scale=iscale)
        scale = sm if sm != 0.0 else float(np.float32(1.0) / np.sqrt(np.float32(D)))
        out = exact(q, k, v, scale, causal)
        np.savez_compressed(
            Path(__file__).parent / f"golden_{name}.npz", q=q.numpy(), k=k.numpy(), v=v.numpy(),
            sm_scale=np.float64(sm), is_causal=np.bool_(causal), seed=np.int64(seed),
            input_scale=np.float64(iscale), out_fp32=out.numpy())
        print("wrote", name)


if __name__ == "__main__":
    main()
