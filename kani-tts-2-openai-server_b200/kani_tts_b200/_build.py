"""Build the sm_100a shared library ``_lib/libkani_b200.so`` in-tree.

The library is plain CUDA C++ behind the C ABI declared in
``include/kani_b200.h``; it has no PyTorch dependency.  Run as
``python -m kani_tts_b200._build`` (from the package's parent directory) or
call :func:`build_library`.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC_DIR = PKG_DIR.parent / "csrc"
REPO_ROOT = PKG_DIR.parent.parent
INCLUDE_DIR = REPO_ROOT / "include"
LIB_DIR = PKG_DIR / "_lib"
LIB_PATH = LIB_DIR / "libkani_b200.so"

SOURCES = ["capi.cu", "rms_norm.cu", "silu_mul.cu", "rope_kv.cu", "decode_attn.cu", "short_conv.cu",
           "sampling.cu", "head_argmax.cu", "codec_codes.cu", "gemv.cu",
           "decode_advance.cu", "head_tc.cu", "gemm_tc.cu"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++20",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    # precise sqrt/div/sin/cos: the RoPE angle reaches thousands of radians
    "-prec-div=true", "-prec-sqrt=true", "-fmad=true",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    deps = [CSRC_DIR / s for s in SOURCES] + list(CSRC_DIR.glob("*.cuh")) + [INCLUDE_DIR / "kani_b200.h"]
    return any(d.stat().st_mtime > t for d in deps)


def build_library(force: bool = False, verbose: bool = False, ptxas_report: bool = False) -> Path:
    """Compile every source for sm_100a and link the shared library."""
    if not force and not _stale() and not ptxas_report:
        return LIB_PATH
    nvcc = _nvcc()
    obj_dir = PKG_DIR.parent / "_build"
    obj_dir.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    def compile_one(src: str):
        obj = obj_dir / (Path(src).stem + ".o")
        cmd = [nvcc, *NVCC_FLAGS, "-I", str(INCLUDE_DIR), "-I", str(CSRC_DIR), "-c",
               str(CSRC_DIR / src), "-o", str(obj)]
        if ptxas_report:
            cmd[1:1] = ["-Xptxas", "-v"]
        return src, obj, cmd, subprocess.run(cmd, capture_output=True, text=True)

    # one nvcc per source, as many at once as there are cores
    workers = max(1, min(len(SOURCES), os.cpu_count() or 1))
    with ThreadPoolExecutor(max_workers=workers) as pool:
        results = list(pool.map(compile_one, SOURCES))
    objs = []
    for src, obj, cmd, res in results:
        if verbose:
            print(" ".join(cmd), flush=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{res.stdout}\n{res.stderr}")
        if ptxas_report or verbose:
            sys.stdout.write(res.stderr)
        objs.append(str(obj))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    link = [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-Xcompiler", "-fPIC",
            *objs, "-o", str(tmp)]
    if verbose:
        print(" ".join(link), flush=True)
    res = subprocess.run(link, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build_library(force="--force" in sys.argv, verbose=True, ptxas_report="--ptxas" in sys.argv)
    print(LIB_PATH)
