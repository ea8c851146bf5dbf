"""GPU parity of forward_flash2_ex (no reference counterpart): N_k != N_q,
global query/key positions for the causal mask, optional log-sum-exp output.

Checked against the CPU oracle's block attention (oracle.block_attention_lse:
fp32 softmax over the visible keys, natural-log LSE, zero rows and -inf LSE
for rows without a visible key) at the same tolerance as forward_flash2.
Covers both dispatch classes (one / two query tiles per CTA), ragged lengths,
keys entirely before / after the queries, and the argument checks.
"""
import pytest
import torch

from flashlite_b200 import flash_attn_wmma as fa
from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu


def _case(cuda, B, H, Nq, Nk, q_off, kv_off, causal, seed):
    q, _, _ = orc.make_qkv(B, H, Nq, 64, seed=seed)
    _, k, v = orc.make_qkv(B, H, Nk, 64, seed=seed + 1)
    o_ref, lse_ref = orc.block_attention_lse(q, k, v, q_off, kv_off, 0.125, causal)
    out, lse = fa.forward_flash2_ex(q.to(cuda), k.to(cuda), v.to(cuda), 0.125, causal,
                                    q_off, kv_off, return_lse=True)
    torch.cuda.synchronize()
    assert fa.device_error() == 0
    mx, mean = orc.error_metrics(out.cpu(), o_ref)
    assert mx <= orc.MAX_ABS_TOL and mean <= orc.MEAN_ABS_TOL, (mx, mean)
    fin = torch.isfinite(lse_ref)
    assert torch.equal(torch.isfinite(lse.cpu()), fin)
    if fin.any():
        assert (lse.cpu()[fin] - lse_ref[fin]).abs().max().item() < 1e-3
    return out, lse


@pytest.mark.parametrize("Nq,Nk,q_off,kv_off,causal", [
    (256, 640, 0, 0, False),       # more keys than queries
    (640, 200, 0, 0, False),       # fewer keys, ragged
    (300, 300, 300, 0, True),      # queries after all keys: full visibility
    (384, 512, 128, 0, True),      # diagonal band inside the key range
    (256, 256, 0, 512, True),      # every key after every query: zero rows, -inf LSE
    (1000, 1000, 0, 0, True),      # plain causal, ragged
])
def test_offsets_and_lengths(cuda, Nq, Nk, q_off, kv_off, causal):
    _case(cuda, 1, 4, Nq, Nk, q_off, kv_off, causal, seed=Nq + Nk)


def test_two_tile_dispatch_with_lse(cuda):
    # 4*40 slices x 4 query-tile pairs >= 148: two query tiles per CTA
    _case(cuda, 4, 40, 1024, 768, 256, 0, True, seed=9)


@pytest.mark.parametrize("B,H,Nq,Nk", [
    (1, 160, 256, 100),    # one KV step per unit: every CTA share is whole units or one-step cuts
    (2, 80, 1000, 1000),   # ragged rows and keys, units cut between CTAs
    (1, 150, 512, 3000),   # more keys than queries
])
def test_full_pairs_many_ctas_with_lse(cuda, B, H, Nq, Nk):
    # non-causal, even query-tile count, >= 148 tile pairs: the persistent
    # launch, whose cut units merge (O, m, l) parts; LSE from the merged parts
    a, lse_a = _case(cuda, B, H, Nq, Nk, 0, 0, False, seed=Nq + H)
    q, _, _ = orc.make_qkv(B, H, Nq, 64, seed=Nq + H)
    _, k, v = orc.make_qkv(B, H, Nk, 64, seed=Nq + H + 1)
    b = fa.forward_flash2_ex(q.to(cuda), k.to(cuda), v.to(cuda), 0.125, False)[0]
    torch.cuda.synchronize()
    assert torch.equal(a, b)  # with or without LSE, the same bits


def test_matches_forward_flash2_when_plain(cuda):
    q, k, v = (t.to(cuda) for t in orc.make_qkv(2, 4, 512, 64, seed=4))
    for causal in (False, True):
        a = fa.forward_flash2(q, k, v, 0.125, causal)
        b, lse = fa.forward_flash2_ex(q, k, v, 0.125, causal)
        assert torch.equal(a, b)
        assert lse.numel() == 0


def test_out_buffer_and_errors(cuda):
    q, k, v = (t.to(cuda) for t in orc.make_qkv(1, 2, 256, 64, seed=2))
    buf = torch.empty_like(q)
    res, _ = fa.forward_flash2_ex(q, k[:, :, :128].contiguous(), v[:, :, :128].contiguous(),
                                  out=buf)
    assert res.data_ptr() == buf.data_ptr()
    with pytest.raises(RuntimeError, match="negative offset"):
        fa.forward_flash2_ex(q, k, v, 0.125, True, -1, 0)
    with pytest.raises(RuntimeError, match="Value dimensions must match Key"):
        fa.forward_flash2_ex(q, k, v[:, :, :128].contiguous())


@pytest.mark.parametrize("B,H,N,causal", [(2, 8, 1024, False), (2, 8, 1024, True), (4, 40, 1000, True),
                                          (1, 3, 200, False), (2, 80, 1000, False)])
def test_bnhd_layout_equals_bhnd(cuda, B, H, N, causal):
    # [B, N, H, D] (the flash_attn package's layout) through 4-D tensor maps:
    # the same arithmetic as [B, H, N, D], so the bits must agree
    q, k, v = (t.to(cuda) for t in orc.make_qkv(B, H, N, 64, seed=N + H))
    ref = fa.forward_flash2(q, k, v, 0.125, causal)
    qt, kt, vt = (t.transpose(1, 2).contiguous() for t in (q, k, v))
    out, lse = fa.forward_flash2_ex(qt, kt, vt, 0.125, causal, return_lse=True, layout="bnhd")
    _, lse_ref = fa.forward_flash2_ex(q, k, v, 0.125, causal, return_lse=True)
    torch.cuda.synchronize()
    assert out.shape == (B, N, H, 64) and lse.shape == (B, H, N)
    assert torch.equal(out.transpose(1, 2), ref)
    assert torch.equal(lse, lse_ref)


def test_bnhd_rejects_mismatched_shapes(cuda):
    q = torch.zeros(1, 128, 2, 64, dtype=torch.float16, device=cuda)
    k = torch.zeros(1, 128, 3, 64, dtype=torch.float16, device=cuda)
    with pytest.raises(RuntimeError, match=r"\[B, N_k, H, D\]"):
        fa.forward_flash2_ex(q, k, k, layout="bnhd")
    with pytest.raises(RuntimeError, match="layout must be"):
        fa.forward_flash2_ex(q, q, q, layout="nhd")
