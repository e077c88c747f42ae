"""Build libwbk.so (the C-ABI kernel library) in-tree for sm_100a.

    python whisper-blaze_b200/csrc/build.py [--force] [--verbose]

Objects go to whisper-blaze_b200/_build/, the library to
whisper-blaze_b200/lib/libwbk.so. The CUDA runtime is linked statically so the
library does not depend on which libcudart the host process loaded first.
The quantiser unit is compiled with --use_fast_math, the flag set of the
reference's own quantiser build (setup.py:41-54); its scale division is the
explicit approximate quotient of wbk_fp8_quant.cuh, which the GEMM unit (IEEE
defaults, like every other unit) shares.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
REPO = os.path.dirname(PKG)
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "lib", "libwbk.so")
INCLUDE = os.path.join(REPO, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
               "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{HERE}"]

# source -> extra flags
UNITS = {
    "wbk_host.cpp": [],
    "wbk_quant.cu": ["--use_fast_math"],
    "wbk_norm.cu": [],
    "wbk_gemm.cu": [],
    "wbk_attn.cu": [],
}
HEADERS = [os.path.join(HERE, "wbk_common.cuh"), os.path.join(HERE, "wbk_sm100.cuh"),
           os.path.join(HERE, "wbk_fp8_quant.cuh"), os.path.join(INCLUDE, "wbk.h")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _compile(src: str, flags: list[str], force: bool, verbose: bool) -> tuple[str, str]:
    path = os.path.join(HERE, src)
    obj = os.path.join(BUILD, src + ".o")
    if not force and not _stale(obj, [path] + HEADERS + [__file__]):
        return obj, ""
    cmd = [nvcc()] + ARCH + NVCC_COMMON + flags + ["-c", path, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [nvcc(), "-O3", "-std=c++17", "-Xcompiler", "-fPIC", f"-I{INCLUDE}", f"-I{HERE}", "-c", path, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj, (r.stdout + r.stderr) if verbose else ""


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    with ThreadPoolExecutor(max_workers=len(UNITS)) as ex:
        results = list(ex.map(lambda kv: _compile(kv[0], kv[1], force, verbose), UNITS.items()))
    objs = [o for o, _ in results]
    for _, log in results:
        if log:
            print(log)
    if force or _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
    sys.exit(0)
