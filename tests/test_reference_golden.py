"""CPU: pin the oracle on outputs of the reference kernels themselves.

tests/golden/ref_*.npz hold what thebigblender/FlashLite's forward_flash2 and
forward_naive (built from its own sources for sm_100a, oracle/build_ref.py)
returned on a B200 for the inputs of the matching golden_*.npz; they were
recorded with tests/golden/make_ref_golden.py. The fp32 oracle must agree
with both within the north-star tolerance, and so must the exact (float64)
outputs stored with the inputs.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import attention_oracle as orc

GOLDEN = Path(__file__).resolve().parent / "golden"
PAIRS = sorted(GOLDEN.glob("ref_*.npz"))


def test_reference_outputs_present():
    assert len(PAIRS) == len(list(GOLDEN.glob("golden_*.npz")))


@pytest.mark.parametrize("path", PAIRS, ids=lambda p: p.stem)
def test_oracle_matches_reference_outputs(path):
    ref = np.load(path)
    g = np.load(GOLDEN / path.name.replace("ref_", "golden_"))
    q, k, v = (torch.from_numpy(g[n]) for n in ("q", "k", "v"))
    out = orc.attention_fp32(q, k, v, float(g["sm_scale"]), bool(g["is_causal"]))
    for name in ("flash2", "naive"):
        r = torch.from_numpy(ref[name].astype(np.float32))
        mx, mean = orc.error_metrics(r, out)
        assert mx <= orc.MAX_ABS_TOL and mean <= orc.MEAN_ABS_TOL, (name, mx, mean)
    # the reference's tiled numerics restated on the host track its kernel
    tiled = torch.from_numpy(orc.flash2_tiled_reference(q, k, v, float(g["sm_scale"]),
                                                        bool(g["is_causal"])).astype(np.float32))
    mx, _ = orc.error_metrics(tiled, torch.from_numpy(ref["flash2"].astype(np.float32)))
    assert mx <= 2e-3, mx
