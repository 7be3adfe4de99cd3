"""Rebind the reference decoder to this library (the drop-in step).

``kani_tts/optimized_decode.py:14`` imports ``fused_rms_norm``,
``fused_silu_mul`` and ``fused_rope`` by name at import time, so replacing
``kani_tts.triton_kernels`` after that import has no effect.  This helper
covers both orders:

* before ``kani_tts.optimized_decode`` is imported it registers this
  package's module as ``kani_tts.triton_kernels`` in ``sys.modules``;
* after, it rebinds the three names inside ``kani_tts.optimized_decode``.

It also points ``kani_tts.static_cache.StaticLfm2HybridConvCache`` (and the
engine's imported name) at :class:`StaticKVCache`, whose ``update`` is the
kernel-backed KV write.
"""
from __future__ import annotations

import sys

from . import fused_kernels
from .static_cache import StaticKVCache

_NAMES = ("fused_rms_norm", "fused_silu_mul", "fused_rope")


def install_into_reference() -> list[str]:
    """Install the kernels into an importable reference package; return what was patched."""
    patched = []
    od = sys.modules.get("kani_tts.optimized_decode")
    if od is None:
        sys.modules["kani_tts.triton_kernels"] = fused_kernels
        patched.append("sys.modules['kani_tts.triton_kernels']")
    else:
        for name in _NAMES:
            setattr(od, name, getattr(fused_kernels, name))
            patched.append(f"kani_tts.optimized_decode.{name}")
    for modname in ("kani_tts.static_cache", "kani_tts.inference_engine"):
        mod = sys.modules.get(modname)
        if mod is not None and hasattr(mod, "StaticLfm2HybridConvCache"):
            mod.StaticLfm2HybridConvCache = StaticKVCache
            patched.append(f"{modname}.StaticLfm2HybridConvCache")
    return patched
