"""Drop-in replacement of the reference module ``flash_attn_wmma``.

Same functions, argument names, defaults and error behaviour as
thebigblender/FlashLite ``csrc/flash_attn.cpp:4-29``:

* ``forward_flash2(q, k, v, sm_scale=0.0, is_causal=False, out=None)``
  FlashAttention-2 forward on ``[B, H, N, 64]`` fp16 CUDA tensors. With
  ``out`` given, the result is written there and ``out`` is returned (the
  zero-allocation form). ``sm_scale == 0`` means ``1/sqrt(D)``.
* ``forward_naive(q, k, v, sm_scale=0.0, is_causal=False)``
  unfused CUDA-core baseline, any head_dim up to 1024.

Invalid inputs raise ``RuntimeError`` with the reference's messages. The
functions are the C++ binding's own (``flashlite_b200._C``); there is no
Python or CPU fallback: importing this module without the built native code
raises ImportError.

Extra entry points (no reference counterpart):
``forward_flash2_ex(q, k, v, sm_scale=0.0, is_causal=False, q_offset=0,
kv_offset=0, out=None, return_lse=False, layout="bhnd") -> (out, lse)`` takes
head_dim 64 or 128, N_k != N_q and global positions (query row i at
q_offset + i, key row j at kv_offset + j), the ``[B, N, H, D]`` layout
(``layout="bnhd"``), and can return the per-row log-sum-exp;
``forward_block`` (head_dim 64 or 128) and ``ring_finalize`` are the
ring-attention steps; ``backward_flash2(q, k, v, out, dout, lse, sm_scale=0.0,
is_causal=False) -> (dq, dk, dv)`` is the FA2 backward (head_dim 64; ``lse`` from
``forward_flash2_ex(..., return_lse=True)``, wrapped for autograd by
``flashlite_b200.attention.flash_attention``); ``device_error`` reads the
error bits kernels raise when a bounded wait gives up.
"""
from __future__ import annotations

import torch  # noqa: F401  (loads libtorch/libc10 for the binding)

try:
    from ._C import (backward_flash2, device_error, forward_block, forward_flash2,
                     forward_flash2_ex, forward_naive, ring_finalize)
except ImportError as exc:  # pragma: no cover - exercised only on unbuilt trees
    raise ImportError(
        "flashlite_b200 native extension is not built; run `python -m flashlite_b200.build` "
        f"(or __graft_entry__.build()): {exc}"
    ) from exc

__all__ = ["forward_flash2", "forward_naive", "forward_flash2_ex", "forward_block", "ring_finalize",
           "backward_flash2", "device_error"]
