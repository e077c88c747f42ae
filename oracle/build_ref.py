"""Build the reference's own quantiser + norm kernels into oracle/_ref/ (GPU oracle).

TEST INFRASTRUCTURE ONLY. Compiles, from where they lie in the reference tree
(never copied), csrc/kernels/fp8_quantize.cu and csrc/kernels/layernorm_fused.cu
with the reference's own nvcc flags (setup.py:41-54: -O3 --use_fast_math and
the half-operator flags), retargeted from sm_90a to sm_100a, plus our binding
file oracle/ref_bindings.cpp, as a torch extension:

    oracle/_ref/wbk_reference_kernels.so

The reference's GEMM and attention kernels are not built: they are unbound or
broken upstream and do not compile for sm_100a. The build needs the reference
tree (present in the development container, absent on GPU boxes); the built
.so travels with the repository snapshot. `load()` imports the prebuilt file.

    python oracle/build_ref.py [--reference PATH]
"""
from __future__ import annotations

import argparse
import importlib.machinery
import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
NAME = "wbk_reference_kernels"
SO_PATH = os.path.join(OUT_DIR, NAME + ".so")
# The reference tree: WBK_REFERENCE_DIR, else a `reference` directory beside this repository.
DEFAULT_REFERENCE = os.environ.get("WBK_REFERENCE_DIR") or os.path.join(os.path.dirname(os.path.dirname(HERE)),
                                                                         "reference")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-std=c++17", "-O3", "--use_fast_math",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_HALF2_OPERATORS__",
    "-lineinfo", "-DCUDA_HAS_FP8",
]


def sources(reference: str) -> list[str]:
    return [os.path.join(HERE, "ref_bindings.cpp"),
            os.path.join(reference, "csrc", "kernels", "fp8_quantize.cu"),
            os.path.join(reference, "csrc", "kernels", "layernorm_fused.cu")]


def build(reference: str = DEFAULT_REFERENCE, verbose: bool = False) -> str | None:
    """Build when the reference tree is present; returns the .so path or None."""
    srcs = sources(reference)
    if not all(os.path.exists(s) for s in srcs):
        return SO_PATH if os.path.exists(SO_PATH) else None
    if os.path.exists(SO_PATH) and all(os.path.getmtime(SO_PATH) >= os.path.getmtime(s) for s in srcs + [__file__]):
        return SO_PATH
    from torch.utils.cpp_extension import load
    os.makedirs(OUT_DIR, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    load(name=NAME, sources=srcs, extra_include_paths=[os.path.join(reference, "csrc", "include")],
         extra_cflags=["-O3", "-std=c++17"], extra_cuda_cflags=NVCC_FLAGS, build_directory=OUT_DIR,
         verbose=verbose, with_cuda=True)
    return SO_PATH


def load():
    """Import the prebuilt reference-kernel extension (raises if absent)."""
    if not os.path.exists(SO_PATH):
        raise ImportError(f"{SO_PATH} is not built (run oracle/build_ref.py where the reference tree exists)")
    import torch  # noqa: F401  (the extension links against torch)
    loader = importlib.machinery.ExtensionFileLoader(NAME, SO_PATH)
    spec = importlib.util.spec_from_file_location(NAME, SO_PATH, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=DEFAULT_REFERENCE)
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.reference, a.verbose))
    sys.exit(0)
