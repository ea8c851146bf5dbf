"""flashlite_b200: FlashAttention-2 forward for NVIDIA B200 (sm_100a).

Drop-in for the ``flash_attn_wmma`` extension of thebigblender/FlashLite::

    from flashlite_b200 import flash_attn_wmma
    out = flash_attn_wmma.forward_flash2(q, k, v, sm_scale=0.0, is_causal=False, out=None)
    out = flash_attn_wmma.forward_naive(q, k, v, sm_scale=0.0, is_causal=False)

Multi-GPU helpers live in :mod:`flashlite_b200.parallel_attn` (head sharding
and ring attention over NCCL). The native code is the in-tree
``libflashlite_b200.so`` (C ABI, ``include/flashlite_b200.h``) and the torch
binding ``_C``; importing this package fails loudly if they are missing.
"""
from __future__ import annotations

from pathlib import Path

import torch  # noqa: F401  (loads libtorch/libc10 for the binding)

_PKG = Path(__file__).resolve().parent
LIBRARY_PATH = _PKG / "libflashlite_b200.so"

try:
    from . import _C  # noqa: E402
except ImportError as exc:  # pragma: no cover - exercised only on broken installs
    raise ImportError(
        "flashlite_b200 native extension is not built; run `python -m flashlite_b200.build` "
        f"(or __graft_entry__.build()): {exc}"
    ) from exc

from . import flash_attn_wmma  # noqa: E402

__all__ = ["flash_attn_wmma", "LIBRARY_PATH"]
__version__ = "0.1.0"
