"""GPU parity against the reference kernels themselves.

oracle/_ref holds thebigblender/FlashLite's own extension built from its
sources for sm_100a (oracle/build_ref.py). On the same inputs:
  * the reference's forward_flash2/forward_naive meet the tolerance against
    the fp32 oracle (this pins the oracle on the reference itself, including
    its N >= 2048 Br=128 kernel that its own tests never ran);
  * our forward_flash2/forward_naive agree with the reference's outputs.
Skipped when oracle/_ref was not built (no reference tree at build time).
"""
import math

import pytest
import torch

from flashlite_b200 import flash_attn_wmma as fa
from oracle import attention_oracle as orc
from oracle import build_ref

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref_mod():
    mod = build_ref.load()
    if mod is None:
        pytest.skip("reference kernels (oracle/_ref) not built")
    return mod


CASES = [(1, 4, 128, False), (2, 8, 512, True), (2, 8, 1024, False), (2, 8, 1024, True),
         (2, 8, 2048, True), (2, 8, 4096, False), (2, 8, 4096, True), (1, 2, 1000, True)]


@pytest.mark.parametrize("B,H,N,causal", CASES)
def test_flash2_matches_reference_kernel(cuda, ref_mod, B, H, N, causal):
    q, k, v = orc.make_qkv(B, H, N, 64, seed=100 + N)
    oracle = orc.attention_fp32(q, k, v, 0.125, causal)
    qd, kd, vd = (t.to(cuda) for t in (q, k, v))
    ref = ref_mod.forward_flash2(qd, kd, vd, 0.125, causal).cpu()
    ours = fa.forward_flash2(qd, kd, vd, 0.125, causal).cpu()
    mx_r, mean_r = orc.error_metrics(ref, oracle)
    assert mx_r <= orc.MAX_ABS_TOL and mean_r <= orc.MEAN_ABS_TOL, ("reference vs oracle", mx_r, mean_r)
    mx_o, mean_o = orc.error_metrics(ours, oracle)
    assert mx_o <= orc.MAX_ABS_TOL and mean_o <= orc.MEAN_ABS_TOL, ("ours vs oracle", mx_o, mean_o)
    mx, mean = orc.error_metrics(ours, ref)
    assert mx <= orc.MAX_ABS_TOL and mean <= orc.MEAN_ABS_TOL, ("ours vs reference", mx, mean)


@pytest.mark.parametrize("B,H,N,causal", [(1, 4, 256, False), (2, 8, 512, True), (1, 2, 1000, True)])
def test_naive_matches_reference_kernel(cuda, ref_mod, B, H, N, causal):
    q, k, v = orc.make_qkv(B, H, N, 64, seed=7 + N)
    qd, kd, vd = (t.to(cuda) for t in (q, k, v))
    scale = 1.0 / math.sqrt(64)
    ref = ref_mod.forward_naive(qd, kd, vd, scale, causal).cpu()
    ours = fa.forward_naive(qd, kd, vd, scale, causal).cpu()
    mx, mean = orc.error_metrics(ours, ref)
    assert mx <= orc.MAX_ABS_TOL and mean <= orc.MEAN_ABS_TOL, (mx, mean)


def test_same_error_messages_as_reference(cuda, ref_mod):
    z = torch.zeros(1, 2, 128, 32, dtype=torch.float16, device=cuda)
    msgs = []
    for mod in (ref_mod, fa):
        with pytest.raises(RuntimeError) as ei:
            mod.forward_flash2(z, z, z)
        msgs.append(str(ei.value))
    assert "FlashLite WMMA kernel currently requires head_dim == 64" in msgs[0]
    assert "FlashLite WMMA kernel currently requires head_dim == 64" in msgs[1]
