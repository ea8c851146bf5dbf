"""Autograd entry point over the B200 kernels.

``flash_attention(q, k, v, sm_scale=0.0, is_causal=False, layout="bhnd")``
returns softmax(sm_scale * q k^T [causal mask]) v for ``[B, H, N, 64]`` (or,
with ``layout="bnhd"``, ``[B, N, H, 64]``) fp16 CUDA tensors and is
differentiable: the forward is ``forward_flash2_ex`` with the
row log-sum-exp kept for backward, the backward is ``backward_flash2``
(tcgen05 FA2 backward). Neither has a reference counterpart: the reference
module is forward-only.
"""
from __future__ import annotations

import torch

from .flash_attn_wmma import backward_flash2, forward_flash2_ex


class _FlashAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, sm_scale, is_causal, layout):
        out, lse = forward_flash2_ex(q, k, v, sm_scale, is_causal, return_lse=True, layout=layout)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.sm_scale = sm_scale
        ctx.is_causal = is_causal
        ctx.layout = layout
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse = ctx.saved_tensors
        dq, dk, dv = backward_flash2(q, k, v, out, dout.contiguous(), lse, ctx.sm_scale, ctx.is_causal,
                                     ctx.layout)
        return dq, dk, dv, None, None, None


def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sm_scale: float = 0.0,
                    is_causal: bool = False, layout: str = "bhnd") -> torch.Tensor:
    """Differentiable FA2 attention; ``sm_scale == 0`` means ``1/sqrt(D)``."""
    return _FlashAttention.apply(q, k, v, sm_scale, is_causal, layout)
