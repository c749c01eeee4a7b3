"""Builds libb200attn.so (the C-ABI library) for sm_100a with nvcc.

Usage: python build.py [--debug]
The shared object is written next to the Python package
(``b200attn/libb200attn.so``) so that it travels with the source tree.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG_ROOT = HERE.parent
REPO = PKG_ROOT.parent
INCLUDE = REPO / "include"
OUT_DIR = PKG_ROOT / "b200attn"
LIB_NAME = "libb200attn.so"
BUILD_DIR = PKG_ROOT / "_build"

SOURCES = ["host_util.cu", "capi.cu", "kv_scatter.cu", "paged_decode.cu", "paged_decode_no_alloc.cu",
           "prefill_tc.cu", "qkv_proj.cu", "selftest.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found")
    return cand


def compile_one(src: str, flags: list[str]) -> Path:
    obj = BUILD_DIR / (Path(src).stem + ".o")
    cmd = [nvcc(), *ARCH, *flags, "-c", str(HERE / src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    if res.stderr.strip():
        sys.stderr.write(res.stderr)
    return obj


def build(debug: bool = False, verbose_ptxas: bool = False) -> Path:
    BUILD_DIR.mkdir(exist_ok=True)
    flags = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
             "-I", str(INCLUDE), "-I", str(HERE), "--expt-relaxed-constexpr"]
    if debug:
        flags += ["-DB200_DEBUG=1"]
    if verbose_ptxas:
        flags += ["-Xptxas", "-v"]
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: compile_one(s, flags), SOURCES))
    out = OUT_DIR / LIB_NAME
    tmp = out.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart_static"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    a = ap.parse_args()
    print(build(debug=a.debug, verbose_ptxas=a.ptxas_v))
