"""B200 (sm_100a) kernels for the KaniTTS per-token decode path.

Public surface:

* :mod:`kani_tts_b200.fused_kernels` — drop-in ``fused_rms_norm``,
  ``fused_silu_mul``, ``fused_rope`` (same signatures as
  ``kani_tts/triton_kernels.py``) and the fused ``fused_add_rms_norm``,
  ``kv_cache_write``, ``fused_rope_kv_write``;
* :class:`kani_tts_b200.static_cache.StaticKVCache` — the static cache with
  kernel-backed ``update`` / ``update_fused``;
* :mod:`kani_tts_b200.positions` — BemaTTS position schedule and
  learnable-alpha frequencies feeding the RoPE kernel;
* :func:`kani_tts_b200.install.install_into_reference` — rebinding of the
  reference decoder's kernel names to this library.

All compute goes through ``_lib/libkani_b200.so``; importing the ops fails if
it has not been built.
"""
from .fused_kernels import (  # noqa: F401
    fused_add_rms_norm,
    fused_rms_norm,
    fused_rope,
    fused_rope_kv_write,
    fused_silu_mul,
    kv_cache_write,
    launch_count,
)
from .static_cache import StaticKVCache  # noqa: F401
from . import positions  # noqa: F401

__version__ = "0.1.0"
