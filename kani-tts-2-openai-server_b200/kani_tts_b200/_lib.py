"""ctypes binding of ``libkani_b200.so`` (the C ABI in ``include/kani_b200.h``).

The shared library is the only implementation of the ops: there is no Triton,
CPU or eager fallback.  Loading fails loudly when the library has not been
built, and every op raises when it is handed a non-CUDA tensor.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libkani_b200.so"

KANI_DTYPE_F32 = 0
KANI_DTYPE_BF16 = 1
KANI_DTYPE_F16 = 2

KANI_FLAG_SLOT_OOB = 1
KANI_FLAG_FRAME_OOB = 2
KANI_FLAG_TIMEOUT = 4

_DTYPE_CODES = {
    torch.float32: KANI_DTYPE_F32,
    torch.bfloat16: KANI_DTYPE_BF16,
    torch.float16: KANI_DTYPE_F16,
}

_c_i32 = ctypes.c_int32
_c_i64 = ctypes.c_int64
_c_f32 = ctypes.c_float
_c_p = ctypes.c_void_p

# argument signatures, in header order
_SIGNATURES = {
    "kani_version": ([], ctypes.c_int),
    "kani_status_string": ([ctypes.c_int], ctypes.c_char_p),
    "kani_launch_count": ([], ctypes.c_uint64),
    "kani_set_wait_limit": ([_c_i64], ctypes.c_int),
    "kani_set_l2_prefetch": ([_c_p, _c_i64, _c_p, _c_i64], ctypes.c_int),
    "kani_rms_norm": ([_c_i32, _c_i32, _c_p, _c_i64, _c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_f32, _c_p],
                      ctypes.c_int),
    "kani_add_rms_norm": ([_c_i32, _c_i32, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_p, _c_i64, _c_p, _c_i64,
                           _c_i64, _c_i64, _c_f32, _c_p], ctypes.c_int),
    "kani_reduce_add_rms_norm": ([_c_i32, _c_i32, _c_p, _c_i64, _c_i64, _c_i32, _c_p, _c_i64, _c_p, _c_p, _c_i64,
                                  _c_p, _c_i64, _c_i64, _c_i64, _c_f32, _c_p], ctypes.c_int),
    "kani_silu_mul": ([_c_i32, _c_p, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_p], ctypes.c_int),
    "kani_rope_qk": ([_c_i32, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_p],
                     ctypes.c_int),
    "kani_kv_cache_write": ([_c_i32, _c_p, _c_p, _c_i64, _c_i32, _c_i32, _c_p, _c_p, _c_i64, _c_p, _c_i32,
                             _c_p, _c_p], ctypes.c_int),
    "kani_rope_kv_write": ([_c_i32, _c_i64, _c_i64, _c_i32, _c_i32, _c_i32,
                            _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_i64,
                            _c_p, _c_p,
                            _c_p, _c_p, _c_f32,
                            _c_p, _c_i64, _c_p, _c_i32,
                            _c_p, _c_i64, _c_i64,
                            _c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_i64,
                            _c_p, _c_p, _c_p], ctypes.c_int),
    "kani_decode_attention": ([_c_i32, _c_i64, _c_i32, _c_i32, _c_i32,
                               _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_i64,
                               _c_p, _c_f32, _c_p, _c_i64, _c_i64, _c_p, _c_p], ctypes.c_int),
    "kani_decode_attention_step": ([_c_i32, _c_i64, _c_i32, _c_i32, _c_i32,
                                    _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_i64,
                                    _c_p, _c_f32, _c_p, _c_i64, _c_i64, _c_p, _c_p], ctypes.c_int),
    "kani_short_conv_step": ([_c_i32, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_p, _c_i64, _c_i64, _c_i32, _c_i32,
                              _c_p], ctypes.c_int),
    "kani_sample_tokens": ([_c_i32, _c_p, _c_i64, _c_i64, _c_i32, _c_p,
                            _c_p, _c_i64, _c_i32,
                            _c_f32, _c_f32, _c_f32, _c_i32,
                            _c_p, ctypes.c_uint64, _c_p,
                            _c_p, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_p], ctypes.c_int),
    "kani_head_argmax": ([_c_i32, _c_p, _c_i64, _c_i64, _c_i32, _c_p, _c_i64, _c_i32,
                          _c_p, _c_p, _c_i64, _c_p, _c_p, _c_i64, _c_p], ctypes.c_int),
    "kani_head_argmax_norm": ([_c_i32, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_f32, _c_i64, _c_i32, _c_p, _c_i64,
                               _c_i32, _c_p, _c_p, _c_i64, _c_p, _c_p, _c_i64, _c_p], ctypes.c_int),
    "kani_head_argmax_noalloc": ([_c_i32, _c_p, _c_i64, _c_i64, _c_i32, _c_p, _c_i64, _c_i32,
                                  _c_p, _c_p, _c_i64, _c_p, _c_i64, _c_p], ctypes.c_int),
    "kani_head_argmax_tc": ([_c_i32, _c_p, _c_i64, _c_i64, _c_i32, _c_p, _c_i64, _c_i32,
                             _c_p, _c_p, _c_i64, _c_p, _c_p, _c_i64, _c_p, _c_p], ctypes.c_int),
    "kani_gemm_tc": ([_c_i32, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_f32, _c_p, _c_i64,
                      _c_i32, _c_i32, _c_i64, _c_i32, _c_p, _c_i64, _c_p, _c_p], ctypes.c_int),
    "kani_gemv": ([_c_i32, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_f32, _c_p, _c_i64,
                   _c_i32, _c_i32, _c_i64, _c_i32, _c_p, _c_i64, _c_p], ctypes.c_int),
    "kani_gemv_short_conv": ([_c_i32, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_f32, _c_p, _c_i64,
                              _c_i32, _c_i32, _c_i64, _c_p, _c_i64, _c_p, _c_i32, _c_p, _c_i64, _c_p], ctypes.c_int),
    "kani_decode_advance": ([_c_p, _c_p, _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_i32, _c_f32,
                             _c_p, _c_p, _c_p, _c_i64, _c_p], ctypes.c_int),
    "kani_gemv_rope_kv": ([_c_i32, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_f32, _c_p, _c_i64,
                           _c_i32, _c_i64, _c_i32, _c_i32, _c_i32, _c_p, _c_p, _c_p, _c_p, _c_f32, _c_p, _c_i64,
                           _c_p, _c_i32, _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_p,
                           _c_p, _c_p], ctypes.c_int),
    "kani_codec_codes": ([_c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_p, _c_p,
                          _c_p], ctypes.c_int),
}

EXPORTED_SYMBOLS = tuple(_SIGNATURES)


class KaniError(RuntimeError):
    """A kernel launch of the library failed (status from the C ABI)."""


_lib = None
_lib_lock = threading.Lock()


def load_library(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load (once) and return the shared library; raises if it is missing."""
    global _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise ImportError(
                f"{p} is missing: build it with `python -m kani_tts_b200._build` "
                "(or __graft_entry__.build()); there is no fallback implementation")
        lib = ctypes.CDLL(str(p))
        for name, (argtypes, restype) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = restype
        _lib = lib
        return lib


def status_string(code: int) -> str:
    return load_library().kani_status_string(code).decode()


def launch_count() -> int:
    return int(load_library().kani_launch_count())


def set_wait_limit(cycles: int) -> None:
    """Bound the kernels' on-chip TMA waits to `cycles` (0: the default ~1 s);
    a test of the timeout path (KANI_FLAG_TIMEOUT).  Process-wide."""
    check(load_library().kani_set_wait_limit(int(cycles)), "kani_set_wait_limit")


def set_l2_prefetch(ranges) -> None:
    """Name up to two device ranges ((address, bytes) pairs, 16-byte aligned)
    that the next decode GEMV / head / reduce + add + RMSNorm / SiLU·mul launch
    from this thread prefetches into L2 as it starts; ``None`` or ``()`` clears
    the hint."""
    r = list(ranges or ())
    if len(r) > 2:
        raise ValueError("at most two L2 prefetch ranges per launch")
    r += [(None, 0)] * (2 - len(r))
    check(load_library().kani_set_l2_prefetch(r[0][0], int(r[0][1]), r[1][0], int(r[1][1])),
          "kani_set_l2_prefetch")


def check(code: int, op: str) -> None:
    if code != 0:
        raise KaniError(f"{op} failed: {status_string(code)} (status {code})")


def dtype_code(t: torch.Tensor, what: str) -> int:
    try:
        return _DTYPE_CODES[t.dtype]
    except KeyError:
        raise TypeError(f"{what}: unsupported dtype {t.dtype} (expected float32, bfloat16 or float16)") from None


def require_cuda(t: torch.Tensor, what: str) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{what} must be a torch.Tensor, got {type(t).__name__}")
    if t.device.type != "cuda":
        raise ValueError(f"{what} must be a CUDA tensor (got device {t.device}); "
                         "these ops have no CPU implementation")


def stream_ptr(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


_err_flags: dict[int, torch.Tensor] = {}


def error_flag(device: torch.device) -> torch.Tensor:
    """Per-device int32 flag the kernels OR KANI_FLAG_* bits into.

    Allocated on first use; call once before CUDA-graph capture so the
    captured kernels point at a tensor that outlives the graph.
    """
    idx = device.index if device.index is not None else torch.cuda.current_device()
    f = _err_flags.get(idx)
    if f is None:
        f = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _err_flags[idx] = f
    return f


def read_and_clear_errors(device: torch.device) -> int:
    """Synchronising read of the device error flag (then reset to 0)."""
    f = error_flag(device)
    v = int(f.item())
    f.zero_()
    return v
