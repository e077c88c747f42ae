"""Precision configuration (mirror of whisper_blaze/precision.py, v0.1.17).

Same enum values, dataclasses, presets and errors as the reference
(whisper_blaze/precision.py:15-123), so configs, env vars and tests written
against it keep working. The reference's FP8 presets are deprecated aliases
of the FP16 config (precision.py:86-108) because it had no FP8 GEMM; they are
kept exactly so here. This build adds one real FP8 preset, `fp8_e4m3`, which
runs every encoder/decoder linear through the B200 FP8 GEMM.
"""
from __future__ import annotations

import warnings
from dataclasses import dataclass, field
from enum import Enum


class Precision(str, Enum):
    FP16 = "fp16"
    FP8_E4M3 = "fp8_e4m3"
    FP8_E5M2 = "fp8_e5m2"

    def is_fp8(self) -> bool:
        return self in (Precision.FP8_E4M3, Precision.FP8_E5M2)

    def max_val(self) -> float:
        return {Precision.FP16: 65504.0, Precision.FP8_E4M3: 448.0, Precision.FP8_E5M2: 57344.0}[self]

    def fmt(self) -> str:
        """Kernel format name of an fp8 precision ('e4m3' / 'e5m2')."""
        if not self.is_fp8():
            raise ValueError(f"{self} is not an fp8 precision")
        return "e4m3" if self is Precision.FP8_E4M3 else "e5m2"


@dataclass
class LayerPrecision:
    """Per-operation precision for one transformer layer."""
    weight: Precision = Precision.FP16
    activation: Precision = Precision.FP16

    def is_fp8(self) -> bool:
        return self.weight.is_fp8() or self.activation.is_fp8()


@dataclass
class PrecisionConfig:
    """Full model precision configuration, one LayerPrecision per layer group."""
    encoder_ffn: LayerPrecision = field(default_factory=LayerPrecision)
    encoder_attn_qkv: LayerPrecision = field(default_factory=LayerPrecision)
    encoder_attn_out: LayerPrecision = field(default_factory=LayerPrecision)
    decoder_self_attn: LayerPrecision = field(default_factory=LayerPrecision)
    decoder_cross_attn: LayerPrecision = field(default_factory=LayerPrecision)
    decoder_ffn: LayerPrecision = field(default_factory=LayerPrecision)

    def summary(self) -> str:
        lines = ["PrecisionConfig:"]
        for name, lp in self.__dict__.items():
            lines.append(f"  {name:<22} weight={lp.weight.value:<10} act={lp.activation.value}")
        return "\n".join(lines)


def full_fp16() -> PrecisionConfig:
    """All FP16. Maximum quality, no quantisation."""
    fp16 = LayerPrecision(Precision.FP16, Precision.FP16)
    return PrecisionConfig(encoder_ffn=fp16, encoder_attn_qkv=fp16, encoder_attn_out=fp16,
                           decoder_self_attn=fp16, decoder_cross_attn=fp16, decoder_ffn=fp16)


def fp8_e4m3() -> PrecisionConfig:
    """Every linear in FP8 E4M3 (weights and activations, per-tensor scales)."""
    fp8 = LayerPrecision(Precision.FP8_E4M3, Precision.FP8_E4M3)
    return PrecisionConfig(encoder_ffn=fp8, encoder_attn_qkv=fp8, encoder_attn_out=fp8,
                           decoder_self_attn=fp8, decoder_cross_attn=fp8, decoder_ffn=fp8)


def mixed_fp8() -> PrecisionConfig:
    """Deprecated alias for :func:`full_fp16` (kept as in the reference)."""
    warnings.warn("mixed_fp8() is deprecated: it returns the all-FP16 configuration. Use full_fp16(), "
                  "or fp8_e4m3() for FP8 linears.", DeprecationWarning, stacklevel=2)
    return full_fp16()


def aggressive_fp8() -> PrecisionConfig:
    """Deprecated alias for :func:`full_fp16` (kept as in the reference)."""
    warnings.warn("aggressive_fp8() is deprecated: it returns the all-FP16 configuration. Use full_fp16(), "
                  "or fp8_e4m3() for FP8 linears.", DeprecationWarning, stacklevel=2)
    return full_fp16()


PRESETS: dict[str, callable] = {
    "fp16": full_fp16,
    "mixed_fp8": mixed_fp8,
    "aggressive_fp8": aggressive_fp8,
    "fp8_e4m3": fp8_e4m3,
}


def from_name(name: str) -> PrecisionConfig:
    if name not in PRESETS:
        raise ValueError(f"Unknown precision preset '{name}'. Available: {list(PRESETS.keys())}")
    return PRESETS[name]()
