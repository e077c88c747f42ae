"""Install the B200 modules into a Hugging Face Whisper model.

Mirrors the reference's WhisperBlaze._patch_layers (whisper_blaze/model.py:334-350),
which swaps every supported nn.LayerNorm for BlazeLayerNorm, and adds what that
method leaves out: each nn.Linear of the encoder and decoder layers becomes a
BlazeLinear with the precision of its PrecisionConfig group
(whisper_blaze/precision.py:41-59 names the groups):

  WhisperEncoderLayer  self_attn.{q,k,v}_proj -> encoder_attn_qkv
                       self_attn.out_proj     -> encoder_attn_out
                       fc1, fc2               -> encoder_ffn
  WhisperDecoderLayer  self_attn.*            -> decoder_self_attn
                       encoder_attn.*         -> decoder_cross_attn
                       fc1, fc2               -> decoder_ffn

With an FP8 decoder_cross_attn group, each decoder layer's encoder_attn.k_proj and
v_proj are stacked into one FP8 linear (StackedKVProjection): the cross-attention
K/V of a generate call is one GEMM of width 2 x d_model per layer (config 4's
shape) instead of two.

Layers are recognised by class name, so transformers is not imported here.
A linear whose group is FP16 keeps the fp16 F.linear path of BlazeLinear
(bit-identical to nn.Linear); an FP8 group quantises its weight once, on the
GPU, at patch time.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch.nn as nn

from .modules import BlazeLayerNorm, BlazeLinear, StackedKVProjection
from .precision import LayerPrecision, PrecisionConfig

ENCODER_LAYER = "WhisperEncoderLayer"
DECODER_LAYER = "WhisperDecoderLayer"


def linear_group(layer_kind: str, path: str) -> Optional[str]:
    """PrecisionConfig field for the linear at `path` (relative to its layer), or None."""
    head, _, leaf = path.rpartition(".")
    if layer_kind == ENCODER_LAYER:
        if head == "self_attn":
            if leaf in ("q_proj", "k_proj", "v_proj"):
                return "encoder_attn_qkv"
            if leaf == "out_proj":
                return "encoder_attn_out"
        if head == "" and leaf in ("fc1", "fc2"):
            return "encoder_ffn"
    elif layer_kind == DECODER_LAYER:
        if head == "self_attn" and leaf in ("q_proj", "k_proj", "v_proj", "out_proj"):
            return "decoder_self_attn"
        if head == "encoder_attn" and leaf in ("q_proj", "k_proj", "v_proj", "out_proj"):
            return "decoder_cross_attn"
        if head == "" and leaf in ("fc1", "fc2"):
            return "decoder_ffn"
    return None


def _set_child(root: nn.Module, path: str, new: nn.Module) -> None:
    parent = root
    *heads, leaf = path.split(".")
    for h in heads:
        parent = getattr(parent, h)
    setattr(parent, leaf, new)


def patch_layers(model: nn.Module, precision: PrecisionConfig, layernorms: bool = True,
                 stack_cross_kv: bool = True) -> Dict[str, int]:
    """Swap the linears (by precision group) and, optionally, the LayerNorms of `model` in place.

    With stack_cross_kv and an FP8 decoder_cross_attn group, each decoder layer's
    encoder_attn.k_proj / v_proj become the two halves of one StackedKVProjection
    (registered as encoder_attn.kv_proj): one FP8 GEMM of width 2 x d_model per
    generate call and layer instead of two.

    Returns counts: patched_layernorms, patched_linears (k and v count as two),
    stacked_cross_kv, and one entry per group that received at least one FP8
    linear (``fp8_<group>``).
    """
    counts: Dict[str, int] = {"patched_layernorms": 0, "patched_linears": 0, "stacked_cross_kv": 0}
    for layer in list(model.modules()):
        kind = type(layer).__name__
        if kind not in (ENCODER_LAYER, DECODER_LAYER):
            continue
        stacked_paths = set()
        xattn = getattr(layer, "encoder_attn", None) if kind == DECODER_LAYER else None
        if (stack_cross_kv and xattn is not None and precision.decoder_cross_attn.is_fp8()
                and isinstance(getattr(xattn, "k_proj", None), nn.Linear)
                and isinstance(getattr(xattn, "v_proj", None), nn.Linear)):
            kv = StackedKVProjection(xattn.k_proj, xattn.v_proj, precision.decoder_cross_attn)
            xattn.kv_proj = kv
            xattn.k_proj = kv.half(0)
            xattn.v_proj = kv.half(1)
            stacked_paths = {"encoder_attn.k_proj", "encoder_attn.v_proj"}
            counts["patched_linears"] += 2
            counts["stacked_cross_kv"] += 1
            counts["fp8_decoder_cross_attn"] = counts.get("fp8_decoder_cross_attn", 0) + 2
        for path, child in list(layer.named_modules()):
            if path in stacked_paths or path.startswith("encoder_attn.kv_proj"):
                continue
            if not isinstance(child, nn.Linear):
                continue
            group = linear_group(kind, path)
            if group is None:
                continue
            lp: LayerPrecision = getattr(precision, group)
            w = child.weight.data.detach()
            b = child.bias.data.detach() if child.bias is not None else None
            _set_child(layer, path, BlazeLinear(w, b, lp))
            counts["patched_linears"] += 1
            if lp.is_fp8():
                counts[f"fp8_{group}"] = counts.get(f"fp8_{group}", 0) + 1
    if layernorms:
        for parent in list(model.modules()):
            for name, child in list(parent.named_children()):
                if isinstance(child, nn.LayerNorm) and BlazeLayerNorm.supports(child):
                    setattr(parent, name, BlazeLayerNorm.from_layernorm(child))
                    counts["patched_layernorms"] += 1
    return counts
