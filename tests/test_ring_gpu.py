"""GPU parity of the ring-attention building blocks.

forward_block (the FA2 kernel in merge mode) against the oracle's block
attention and log-sum-exp merge, for diagonal, fully visible, fully masked
and ragged blocks; and a ring emulated in one process (the block loop of
RingAttention without communication) against full attention, including the
BASELINE config-5 shape on sampled rows with fewer heads.
"""
import ctypes

import pytest
import torch

from flashlite_b200 import flash_attn_wmma as fa
from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu


def _block(cuda, q, k, v, q_off, kv_off, causal, o_acc=None, lse=None, first=True, scale=0.125):
    qd, kd, vd = (t.to(cuda) for t in (q, k, v))
    B, H, Nq, D = q.shape
    if o_acc is None:
        o_acc = torch.full((B, H, Nq, D), 7.0, device=cuda)  # garbage: first must overwrite
        lse = torch.full((B, H, Nq), 7.0, device=cuda)
    fa.forward_block(qd, kd, vd, o_acc, lse, q_off, kv_off, scale, causal, first)
    torch.cuda.synchronize()
    assert fa.device_error() == 0
    return o_acc, lse


@pytest.mark.parametrize("Nq,Nk,q_off,kv_off,causal", [
    (256, 256, 512, 512, True),    # diagonal block
    (256, 384, 1024, 256, True),   # fully visible earlier block
    (200, 300, 300, 0, True),      # ragged, partially visible
    (256, 256, 0, 0, False),
    (130, 70, 0, 0, False),        # ragged non-causal
])
def test_block_matches_oracle(cuda, Nq, Nk, q_off, kv_off, causal):
    q, _, _ = orc.make_qkv(1, 4, Nq, 64, seed=Nq)
    _, k, v = orc.make_qkv(1, 4, Nk, 64, seed=Nk + 1)
    o, lse = _block(cuda, q, k, v, q_off, kv_off, causal)
    o_ref, lse_ref = orc.block_attention_lse(q, k, v, q_off, kv_off, 0.125, causal)
    assert (o.cpu() - o_ref).abs().max().item() < 2e-3
    fin = torch.isfinite(lse_ref)
    assert torch.equal(torch.isfinite(lse.cpu()), fin)
    assert (lse.cpu()[fin] - lse_ref[fin]).abs().max().item() < 1e-3


def test_fully_masked_block_gives_zero_and_neg_inf(cuda):
    q, k, v = orc.make_qkv(1, 2, 128, 64, seed=1)
    o, lse = _block(cuda, q, k, v, 0, 4096, True)  # every key after every query
    assert torch.all(o == 0) and torch.all(torch.isneginf(lse))


@pytest.mark.parametrize("P,causal", [(2, True), (4, True), (3, False)])
def test_ring_emulation_equals_full_attention(cuda, P, causal):
    nb, H = 256, 4
    q, k, v = orc.make_qkv(1, H, nb * P, 64, seed=P)
    full = orc.attention_fp32(q, k, v, 0.125, causal)
    for r in range(P):
        sl = slice(r * nb, (r + 1) * nb)
        qb = q[:, :, sl].contiguous()
        o_acc = lse = None
        for s in range(P):  # the order RingAttention visits blocks in
            src = (r - s) % P
            if causal and src > r:
                continue
            kb = k[:, :, src * nb:(src + 1) * nb].contiguous()
            vb = v[:, :, src * nb:(src + 1) * nb].contiguous()
            o_acc, lse = _block(cuda, qb, kb, vb, r * nb, src * nb, causal, o_acc, lse, first=(s == 0))
        out = torch.empty(1, H, nb, 64, dtype=torch.float16, device=cuda)
        fa.ring_finalize(o_acc, out)
        torch.cuda.synchronize()
        mx, mean = orc.error_metrics(out.cpu(), full[:, :, sl])
        assert mx <= orc.MAX_ABS_TOL and mean <= orc.MEAN_ABS_TOL, (r, mx, mean)


@pytest.mark.parametrize("P", [2, 4])
def test_zigzag_ring_emulation_equals_full_attention(cuda, P):
    """The zig-zag layout's block schedule (ZigzagRingAttention without the
    communication): rank r's two chunks against every rank's chunk pairs."""
    from flashlite_b200.parallel_attn import zigzag_chunks, zigzag_pairs

    c, H = 192, 2
    q, k, v = orc.make_qkv(1, H, 2 * P * c, 64, seed=10 + P)
    full = orc.attention_fp32(q, k, v, 0.125, True)
    chunk = lambda t, i: t[:, :, i * c:(i + 1) * c].contiguous()
    for r in range(P):
        own = zigzag_chunks(r, P)
        acc = [None, None]
        for s in range(P):
            src = (r - s) % P
            kc = zigzag_chunks(src, P)
            for a, b in zigzag_pairs(r, src, P, True):
                o_acc, lse = acc[a] if acc[a] is not None else (None, None)
                acc[a] = _block(cuda, chunk(q, own[a]), chunk(k, kc[b]), chunk(v, kc[b]),
                                own[a] * c, kc[b] * c, True, o_acc, lse, first=acc[a] is None)
        for a in range(2):
            out = torch.empty(1, H, c, 64, dtype=torch.float16, device=cuda)
            fa.ring_finalize(acc[a][0], out)
            torch.cuda.synchronize()
            mx, mean = orc.error_metrics(out.cpu(), chunk(full, own[a]))
            assert mx <= orc.MAX_ABS_TOL and mean <= orc.MEAN_ABS_TOL, (r, a, mx, mean)


@pytest.mark.slow
def test_config5_shape_sampled_rows(cuda):
    """BASELINE config 5 (B1 H8 N131072, inputs N(0,1)*0.5, causal) with 1 head,
    split into 8 contiguous blocks as on 8 ranks; last block, sampled rows."""
    P, N = 8, 131072
    nb = N // P
    q, k, v = orc.make_qkv(1, 1, N, 64, seed=5, scale=0.5)
    r = P - 1
    qb = q[:, :, r * nb:].contiguous()
    o_acc = lse = None
    for s in range(P):
        src = (r - s) % P
        kb = k[:, :, src * nb:(src + 1) * nb].contiguous()
        vb = v[:, :, src * nb:(src + 1) * nb].contiguous()
        o_acc, lse = _block(cuda, qb, kb, vb, r * nb, src * nb, True, o_acc, lse, first=(s == 0))
    out = torch.empty(1, 1, nb, 64, dtype=torch.float16, device=cuda)
    fa.ring_finalize(o_acc, out)
    rows = torch.tensor([0, 1, 777, nb // 2, nb - 1]) + r * nb
    ref = orc.attention_rows_fp32(q.view(1, N, 64), k.view(1, N, 64), v.view(1, N, 64), rows, 0.125, True)
    got = out.view(nb, 64)[rows - r * nb].cpu().float()
    assert (got - ref[0]).abs().max().item() <= orc.MAX_ABS_TOL


def test_block_c_abi_and_errors(cuda, fl_lib):
    q, k, v = (t.to(cuda) for t in orc.make_qkv(1, 2, 128, 64, seed=2))
    o = torch.empty(1, 2, 128, 64, device=cuda)
    lse = torch.empty(1, 2, 128, device=cuda)
    st = fl_lib.fl_flash2_fwd_block(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                    lse.data_ptr(), 2, 128, 128, 64, 0, 0, 0.125, 1, 1, None)
    assert st == 0, fl_lib.fl_last_error()
    assert fl_lib.fl_flash2_fwd_block(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                      lse.data_ptr(), 2, 128, 128, 32, 0, 0, 0.125, 1, 1, None) == 2
    assert fl_lib.fl_flash2_fwd_block(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                      lse.data_ptr(), 2, 128, 128, 64, -1, 0, 0.125, 1, 1, None) == 1
    torch.cuda.synchronize()
