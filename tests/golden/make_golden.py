"""Generate golden fixtures from the reference's own CUDA kernels (run on a B200).

    python tests/golden/make_golden.py [OUT_DIR]

Loads oracle/_ref/wbk_reference_kernels.so (the reference's fp8_quantize.cu
and layernorm_fused.cu, built unmodified for sm_100a by oracle/build_ref.py)
and records, for seeded inputs generated on the CPU:

  ref_scale_table.npz  the reference scale (compute_fp8_scale, i.e.
                       compute_scale_kernel + host max) for EVERY positive
                       finite fp16 amax value, for E4M3 (448) and E5M2 (57344);
  ref_quantise.npz     inputs, fp8 bytes, scales and dequantised outputs of
                       quantise_to_e4m3/_e5m2 and dequantise_e4m3/_e5m2;
  ref_norm.npz         layernorm_fused_impl (output and sum) and rmsnorm_fused.

All inputs have element counts that are multiples of 8 (the reference kernels
read 8 elements per thread with no tail handling).
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, REPO)

from oracle import build_ref  # noqa: E402


def randn(shape, seed, std=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g, dtype=torch.float32) * std).half()


def quant_cases():
    g = torch.Generator().manual_seed(1234)
    specials = torch.randint(0, 65536, (2048,), generator=g, dtype=torch.int32).to(torch.int16).view(torch.float16)
    specials = specials.clone()
    specials[:8] = torch.tensor([0.0, -0.0, float("nan"), float("inf"), -float("inf"), 65504.0, -65504.0, 6e-8])
    finite = torch.nan_to_num(specials.clone(), nan=0.0, posinf=0.0, neginf=0.0)
    wide = (randn((2048,), 11) * torch.exp2(torch.randint(-20, 12, (2048,), generator=g).float())).half()
    return {
        "randn_16x1024": randn((16, 1024), 1),
        "weights_32x512": randn((32, 512), 2, std=0.02),
        "specials_2048": specials,
        "finite_random_bits_2048": finite,
        "wide_range_2048": wide,
        "tiny_1024": (randn((1024,), 3) * 1e-6).half(),
        "zeros_256": torch.zeros(256, dtype=torch.float16),
    }


def main(out_dir: str) -> None:
    os.makedirs(out_dir, exist_ok=True)
    R = build_ref.load()
    dev = torch.device("cuda:0")

    # every positive finite fp16 value as an amax
    bits = np.arange(0x0001, 0x7C00, dtype=np.uint16)
    vals = torch.from_numpy(bits.view(np.float16).copy())
    table = {"amax_bits": bits}
    for name, mx in (("e4m3", 448.0), ("e5m2", 57344.0)):
        out = np.empty(len(bits), dtype=np.float32)
        xd = vals.to(dev)
        for i in range(len(bits)):
            out[i] = R.compute_fp8_scale(xd[i:i + 1], mx)
        table[f"scale_{name}"] = out
    np.savez_compressed(os.path.join(out_dir, "ref_scale_table.npz"), **table)

    quant = {}
    for name, x in quant_cases().items():
        xd = x.to(dev).contiguous()
        quant[f"{name}__x"] = x.numpy()
        for fmt, qfn, dqfn in (("e4m3", R.quantise_e4m3, R.dequantise_e4m3),
                               ("e5m2", R.quantise_e5m2, R.dequantise_e5m2)):
            q, s = qfn(xd)
            quant[f"{name}__q_{fmt}"] = q.cpu().numpy()
            quant[f"{name}__s_{fmt}"] = np.float32(s)
            quant[f"{name}__dq_{fmt}"] = dqfn(q, s, list(x.shape)).cpu().numpy()
    np.savez_compressed(os.path.join(out_dir, "ref_quantise.npz"), **quant)

    x, res = randn((24, 1280), 21), randn((24, 1280), 22)
    gamma = (1.0 + randn((1280,), 23, 0.1).float()).half()
    beta = randn((1280,), 24, 0.1)
    d = lambda t: t.to(dev).contiguous()  # noqa: E731
    ln_out, ln_sum = R.layernorm_fused_residual(d(x), d(res), d(gamma), d(beta), 1e-5)
    rms = R.rmsnorm_fused(d(x), d(res), d(gamma), 1e-5)
    np.savez_compressed(os.path.join(out_dir, "ref_norm.npz"), x=x.numpy(), res=res.numpy(), gamma=gamma.numpy(),
                        beta=beta.numpy(), ln_out=ln_out.cpu().numpy(), ln_sum=ln_sum.cpu().numpy(),
                        rms_out=rms.cpu().numpy())
    print("wrote", sorted(os.listdir(out_dir)))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__)))
