"""GPU parity of the FA2 backward (backward_flash2 / fl_flash2_bwd).

No reference counterpart (the reference is forward-only): checked against
the CPU oracle's fp32 gradients (oracle.attention_backward_fp32, pinned to
torch.autograd in test_oracle.py) on the same fp16 inputs. The GPU gradients
come from fp16 operands (P and dS rounded to fp16 before their products, as
in FlashAttention-2) and the fp16 forward output, so the bound is relative:
max-abs error <= 1e-2 of max |ref| and mean-abs error <= 1e-2 of mean |ref|
for each of dq, dk, dv.
"""
import pytest
import torch

from flashlite_b200 import flash_attn_wmma as fa
from flashlite_b200.attention import flash_attention
from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu

MAX_REL, MEAN_REL = 1e-2, 1e-2


def _grads(cuda, B, H, N, causal, seed, sm_scale=0.0, input_scale=1.0):
    q, k, v = orc.make_qkv(B, H, N, 64, seed=seed, scale=input_scale)
    do = orc.make_qkv(B, H, N, 64, seed=seed + 100)[0]
    qd, kd, vd, dod = (t.to(cuda) for t in (q, k, v, do))
    out, lse = fa.forward_flash2_ex(qd, kd, vd, sm_scale, causal, return_lse=True)
    dq, dk, dv = fa.backward_flash2(qd, kd, vd, out, dod, lse, sm_scale, causal)
    torch.cuda.synchronize()
    assert fa.device_error() == 0
    ref = orc.attention_backward_fp32(q, k, v, do, sm_scale, causal)
    return (dq, dk, dv), ref


def _check(got, ref, tag):
    for name, g, r in zip(("dq", "dk", "dv"), got, ref):
        assert g.dtype == torch.float16 and not torch.isnan(g.float()).any(), (tag, name)
        mx, mean = orc.grad_error_metrics(g, r)
        assert mx <= MAX_REL and mean <= MEAN_REL, f"{tag} {name}: max {mx:.2e} mean {mean:.2e}"


@pytest.mark.parametrize("B,H,N", [(1, 2, 128), (2, 4, 256), (1, 3, 1000), (2, 8, 1024), (1, 2, 77)])
@pytest.mark.parametrize("causal", [False, True])
def test_backward_matches_oracle(cuda, B, H, N, causal):
    got, ref = _grads(cuda, B, H, N, causal, seed=N + H)
    _check(got, ref, f"B{B} H{H} N{N} causal={causal}")


def test_backward_scale_and_large_logits(cuda):
    got, ref = _grads(cuda, 1, 2, 512, False, seed=3, sm_scale=0.5)
    _check(got, ref, "scale 0.5")
    got, ref = _grads(cuda, 1, 2, 512, True, seed=4, sm_scale=1.4, input_scale=0.7)
    _check(got, ref, "large logits")


def test_backward_repeatable(cuda):
    q, k, v = (t.to(cuda) for t in orc.make_qkv(2, 4, 512, 64, seed=7))
    do = orc.make_qkv(2, 4, 512, 64, seed=8)[0].to(cuda)
    out, lse = fa.forward_flash2_ex(q, k, v, 0.0, True, return_lse=True)
    a = fa.backward_flash2(q, k, v, out, do, lse, 0.0, True)
    b = fa.backward_flash2(q, k, v, out, do, lse, 0.0, True)
    torch.cuda.synchronize()
    # dk, dv are summed in TMEM in a fixed order; dq adds key tiles through
    # global reductions whose order may vary, so only dk, dv must repeat bitwise
    assert torch.equal(a[1], b[1]) and torch.equal(a[2], b[2])
    mx, _ = orc.grad_error_metrics(a[0], b[0].float())
    assert mx < 1e-3


def test_autograd_wrapper(cuda):
    q, k, v = (t.to(cuda).requires_grad_(True) for t in orc.make_qkv(1, 2, 256, 64, seed=9))
    do = orc.make_qkv(1, 2, 256, 64, seed=10)[0].to(cuda)
    out = flash_attention(q, k, v, 0.0, True)
    out.backward(do)
    ref = orc.attention_backward_fp32(q, k, v, do, 0.0, True)
    _check((q.grad, k.grad, v.grad), ref, "autograd")


def test_backward_errors(cuda):
    q = torch.zeros(1, 2, 128, 64, dtype=torch.float16, device=cuda)
    lse = torch.zeros(1, 2, 128, device=cuda)
    with pytest.raises(RuntimeError, match="lse must hold"):
        fa.backward_flash2(q, q, q, q, q, lse[:, :, :64].contiguous())
    z = torch.zeros(1, 2, 128, 128, dtype=torch.float16, device=cuda)
    with pytest.raises(RuntimeError, match="head_dim == 64"):
        fa.backward_flash2(z, z, z, z, z, lse)


@pytest.mark.parametrize("causal", [False, True])
def test_backward_bnhd_layout(cuda, causal):
    # [B, N, H, D] tensors through 4-D tensor maps: the same arithmetic as
    # [B, H, N, D], so dk and dv repeat bitwise (dq up to reduction order)
    B, H, N = 2, 3, 640
    q, k, v = (t.to(cuda) for t in orc.make_qkv(B, H, N, 64, seed=21))
    do = orc.make_qkv(B, H, N, 64, seed=22)[0].to(cuda)
    out, lse = fa.forward_flash2_ex(q, k, v, 0.0, causal, return_lse=True)
    ref = fa.backward_flash2(q, k, v, out, do, lse, 0.0, causal)

    def t(x):
        return x.transpose(1, 2).contiguous()

    out_t, lse_t = fa.forward_flash2_ex(t(q), t(k), t(v), 0.0, causal, return_lse=True, layout="bnhd")
    got = fa.backward_flash2(t(q), t(k), t(v), out_t, t(do), lse_t, 0.0, causal, "bnhd")
    torch.cuda.synchronize()
    assert fa.device_error() == 0
    assert all(g.shape == (B, N, H, 64) for g in got)
    assert torch.equal(got[1].transpose(1, 2), ref[1]) and torch.equal(got[2].transpose(1, 2), ref[2])
    mx, _ = orc.grad_error_metrics(got[0].transpose(1, 2), ref[0].float())
    assert mx < 1e-3
    # and against the oracle through the autograd wrapper
    qg, kg, vg = (t(x).requires_grad_(True) for x in (q, k, v))
    flash_attention(qg, kg, vg, 0.0, causal, layout="bnhd").backward(t(do))
    oref = orc.attention_backward_fp32(q, k, v, do, 0.0, causal)
    _check((qg.grad.transpose(1, 2), kg.grad.transpose(1, 2), vg.grad.transpose(1, 2)), oref, "bnhd autograd")
