"""flashlite_b200: FlashAttention-2 forward for NVIDIA B200 (sm_100a).

Drop-in for the ``flash_attn_wmma`` extension of thebigblender/FlashLite::

    from flashlite_b200 import flash_attn_wmma
    out = flash_attn_wmma.forward_flash2(q, k, v, sm_scale=0.0, is_causal=False, out=None)
    out = flash_attn_wmma.forward_naive(q, k, v, sm_scale=0.0, is_causal=False)

Multi-GPU helpers live in :mod:`flashlite_b200.parallel_attn` (head sharding
and ring attention over NCCL). The native code is the in-tree
``libflashlite_b200.so`` (C ABI, ``include/flashlite_b200.h``) and the torch
binding ``_C``, built by ``python -m flashlite_b200.build``. Importing
``flash_attn_wmma`` fails loudly if they are missing; there is no fallback.
"""
from __future__ import annotations

from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIBRARY_PATH = _PKG / "libflashlite_b200.so"

__version__ = "0.1.0"


def __getattr__(name):
    # Lazy so that the build script (a submodule) can run before the native
    # extension exists; any use of the drop-in module imports it for real.
    if name == "flash_attn_wmma":
        import importlib

        return importlib.import_module(__name__ + ".flash_attn_wmma")
    raise AttributeError(name)


__all__ = ["flash_attn_wmma", "LIBRARY_PATH"]
