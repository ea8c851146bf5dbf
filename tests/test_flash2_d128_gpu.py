"""GPU parity of the head_dim 128 kernel (forward_flash2_ex, forward_block).

The reference takes head_dim 64 only (csrc/kernel_flash2.cu:756-757), so
these cases are checked against the CPU fp32 oracle alone, at the same
tolerance as the D = 64 kernel (max-abs <= 2e-3, mean-abs <= 2e-4). D = 128
runs its own instantiation (64-key KV tiles, two 64-column halves per
shared-memory tile), so the cases cover both dispatch classes (one / two
query tiles per CTA), ragged lengths, causal offsets, LSE, the [B, N, H, D]
layout, the conditional O rescale, and the ring-attention block step.
"""
import pytest
import torch

from flashlite_b200 import flash_attn_wmma as fa
from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu

D = 128


def _case(cuda, B, H, Nq, Nk, q_off, kv_off, causal, seed, sm_scale=0.0, input_scale=1.0):
    q, _, _ = orc.make_qkv(B, H, Nq, D, seed=seed, scale=input_scale)
    _, k, v = orc.make_qkv(B, H, Nk, D, seed=seed + 1, scale=input_scale)
    scale = sm_scale if sm_scale != 0.0 else D ** -0.5
    o_ref, lse_ref = orc.block_attention_lse(q, k, v, q_off, kv_off, scale, causal)
    out, lse = fa.forward_flash2_ex(q.to(cuda), k.to(cuda), v.to(cuda), sm_scale, causal,
                                    q_off, kv_off, return_lse=True)
    torch.cuda.synchronize()
    assert fa.device_error() == 0
    assert out.shape == (B, H, Nq, D)
    mx, mean = orc.error_metrics(out.cpu(), o_ref)
    assert mx <= orc.MAX_ABS_TOL and mean <= orc.MEAN_ABS_TOL, (mx, mean)
    fin = torch.isfinite(lse_ref)
    assert torch.equal(torch.isfinite(lse.cpu()), fin)
    if fin.any():
        assert (lse.cpu()[fin] - lse_ref[fin]).abs().max().item() < 1e-3
    return out, lse


@pytest.mark.parametrize("B,H,N,causal", [
    (1, 2, 128, False), (1, 2, 128, True),
    (2, 4, 1024, False), (2, 4, 1024, True),
    (1, 3, 1000, False), (1, 3, 1000, True),   # ragged last query and KV tiles
    (1, 2, 64, True), (1, 2, 37, False),       # shorter than one tile
])
def test_square(cuda, B, H, N, causal):
    _case(cuda, B, H, N, N, 0, 0, causal, seed=N + H)


@pytest.mark.parametrize("Nq,Nk,q_off,kv_off,causal", [
    (256, 640, 0, 0, False),       # more keys than queries
    (640, 200, 0, 0, False),       # fewer keys, ragged
    (300, 300, 300, 0, True),      # queries after all keys: full visibility
    (384, 512, 128, 0, True),      # diagonal band inside the key range
    (256, 256, 0, 512, True),      # every key after every query: zero rows, -inf LSE
])
def test_offsets_and_lengths(cuda, Nq, Nk, q_off, kv_off, causal):
    _case(cuda, 1, 4, Nq, Nk, q_off, kv_off, causal, seed=Nq + Nk)


@pytest.mark.parametrize("B,H,N,causal", [
    (4, 40, 1024, True),   # 160 slices x 4 tile pairs: two query tiles per CTA
    (2, 80, 1000, False),  # ragged rows and keys, two tiles per CTA
    (1, 160, 384, True),   # 3 query tiles: the second pair has one tile
])
def test_two_tile_dispatch(cuda, B, H, N, causal):
    _case(cuda, B, H, N, N, 0, 0, causal, seed=B * H + N)


def test_large_logits_rescale_path(cuda):
    # log2-domain logits with std ~11: the running maximum often grows by more
    # than 2^8 (O rescaled in TMEM); inputs scaled so |O| < 4
    _case(cuda, 1, 4, 1024, 1024, 0, 0, False, seed=3, sm_scale=1.4, input_scale=0.7)
    _case(cuda, 1, 4, 1024, 1024, 0, 0, True, seed=4, sm_scale=1.4, input_scale=0.7)


def test_repeatable_and_out_buffer(cuda):
    q, k, v = (t.to(cuda) for t in orc.make_qkv(4, 16, 1100, D, seed=10))
    first, _ = fa.forward_flash2_ex(q, k, v, 0.0, True)
    buf = torch.empty_like(q)
    again, _ = fa.forward_flash2_ex(q, k, v, 0.0, True, out=buf)
    torch.cuda.synchronize()
    assert again.data_ptr() == buf.data_ptr()
    assert torch.equal(first, again)


@pytest.mark.parametrize("B,H,N,causal", [(2, 8, 1024, False), (2, 8, 1024, True), (1, 3, 200, True)])
def test_bnhd_layout_equals_bhnd(cuda, B, H, N, causal):
    q, k, v = (t.to(cuda) for t in orc.make_qkv(B, H, N, D, seed=N + H))
    ref, lse_ref = fa.forward_flash2_ex(q, k, v, 0.0, causal, return_lse=True)
    qt, kt, vt = (t.transpose(1, 2).contiguous() for t in (q, k, v))
    out, lse = fa.forward_flash2_ex(qt, kt, vt, 0.0, causal, return_lse=True, layout="bnhd")
    torch.cuda.synchronize()
    assert out.shape == (B, N, H, D)
    assert torch.equal(out.transpose(1, 2), ref)
    assert torch.equal(lse, lse_ref)


def test_forward_flash2_keeps_reference_head_dim_check(cuda):
    q = torch.zeros(1, 2, 128, D, dtype=torch.float16, device=cuda)
    with pytest.raises(RuntimeError, match="requires head_dim == 64"):
        fa.forward_flash2(q, q, q)
    with pytest.raises(RuntimeError, match="head_dim 64 or 128"):
        z = torch.zeros(1, 2, 128, 96, dtype=torch.float16, device=cuda)
        fa.forward_flash2_ex(z, z, z)


def test_block_steps_merge_to_full_attention(cuda):
    # two causal ring steps (diagonal block, then the earlier block) merged
    # in (o_acc, lse) equal attention over the whole key range
    nb, H = 256, 4
    q, k, v = orc.make_qkv(1, H, 2 * nb, D, seed=21)
    scale = D ** -0.5
    full = orc.attention_fp32(q, k, v, scale, True)
    qd = q[:, :, nb:].contiguous().to(cuda)
    o_acc = torch.full((1, H, nb, D), 7.0, device=cuda)
    lse = torch.full((1, H, nb), 7.0, device=cuda)
    for step, (blk, first) in enumerate(((1, True), (0, False))):
        kd = k[:, :, blk * nb:(blk + 1) * nb].contiguous().to(cuda)
        vd = v[:, :, blk * nb:(blk + 1) * nb].contiguous().to(cuda)
        fa.forward_block(qd, kd, vd, o_acc, lse, nb, blk * nb, scale, True, first)
    out = torch.empty(1, H, nb, D, dtype=torch.float16, device=cuda)
    fa.ring_finalize(o_acc, out)
    torch.cuda.synchronize()
    assert fa.device_error() == 0
    mx, mean = orc.error_metrics(out.cpu(), full[:, :, nb:])
    assert mx <= orc.MAX_ABS_TOL and mean <= orc.MEAN_ABS_TOL, (mx, mean)
