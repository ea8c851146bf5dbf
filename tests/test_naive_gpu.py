"""GPU parity of the naive CUDA-core kernel (forward_naive) against the oracle.

Matrix of the reference (thebigblender/FlashLite tests/test_correctness.py:29-58)
plus head dims other than 64 (the reference naive path accepts any D) and a
sequence longer than one shared-memory chunk of scores."""
import math

import pytest
import torch

from flashlite_b200 import flash_attn_wmma as fa
from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu


def _run(cuda, B, H, N, D, causal, seed=42, sm_scale=None):
    q, k, v = orc.make_qkv(B, H, N, D, seed=seed)
    scale = 1.0 / math.sqrt(D) if sm_scale is None else sm_scale
    ref = orc.attention_fp32(q, k, v, scale, causal)
    out = fa.forward_naive(q.to(cuda), k.to(cuda), v.to(cuda), scale, causal)
    torch.cuda.synchronize()
    mx, mean = orc.error_metrics(out, ref)
    assert out.dtype == torch.float16 and out.shape == q.shape
    assert mx <= orc.MAX_ABS_TOL and mean <= orc.MEAN_ABS_TOL, (mx, mean)


@pytest.mark.parametrize("batch_size", [1, 2])
@pytest.mark.parametrize("num_heads", [4, 8])
@pytest.mark.parametrize("seq_len", [128, 256, 512])
@pytest.mark.parametrize("is_causal", [False, True])
def test_reference_matrix(cuda, batch_size, num_heads, seq_len, is_causal):
    _run(cuda, batch_size, num_heads, seq_len, 64, is_causal)


@pytest.mark.parametrize("D", [8, 16, 36, 80, 128, 256, 520, 1024])
def test_other_head_dims(cuda, D):
    # multiples of 8 take the 16-byte-load form (1 to 16 chunks of q per
    # lane); 36 takes the scalar form
    _run(cuda, 1, 2, 200, D, True, seed=D)


def test_unaligned_tensors_take_the_scalar_form(cuda):
    """Tensors that start 2 bytes past a 16-byte boundary cannot use 16-byte
    loads; the result must not change."""
    B, H, N, D = 1, 2, 300, 64
    q, k, v = orc.make_qkv(B, H, N, D, seed=11)
    ref = orc.attention_fp32(q, k, v, 0.125, False)

    def shifted(t):
        buf = torch.empty(t.numel() + 1, dtype=t.dtype, device=cuda)
        view = buf[1:].view(t.shape)
        view.copy_(t.to(cuda))
        assert view.data_ptr() % 16 == 2
        return view

    out = fa.forward_naive(shifted(q), shifted(k), shifted(v), 0.125, False)
    aligned = fa.forward_naive(q.to(cuda), k.to(cuda), v.to(cuda), 0.125, False)
    torch.cuda.synchronize()
    mx, mean = orc.error_metrics(out, ref)
    assert mx <= orc.MAX_ABS_TOL and mean <= orc.MEAN_ABS_TOL, (mx, mean)
    mx2, _ = orc.error_metrics(aligned, ref)
    assert mx2 <= orc.MAX_ABS_TOL


@pytest.mark.parametrize("causal", [False, True])
def test_longer_than_one_chunk(cuda, causal):
    _run(cuda, 1, 1, 5000, 64, causal, seed=7)


def test_default_scale(cuda):
    _run(cuda, 1, 2, 100, 64, False, seed=3, sm_scale=0.0)
