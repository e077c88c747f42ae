"""GPU parity of the FP8 encoder stack against the CPU oracle stack."""
import pytest
import torch

from conftest import randn_f16
from oracle import encoder as ref_encoder
from oracle import gemm
from whisper_blaze_b200.encoder import EncoderConfig, FP8EncoderStack, random_layer_weights

pytestmark = pytest.mark.gpu

STACK_GATE = 2e-2  # relative (max|y-ref|/max|ref|) after two layers and the final LayerNorm


def _layers(cfg, n, seed):
    g = torch.Generator().manual_seed(seed)
    return [random_layer_weights(cfg, g) for _ in range(n)]


@pytest.mark.parametrize("B,S", [(2, 64), (1, 1500)])
def test_two_layer_stack_matches_oracle(cuda_device, B, S):
    cfg = EncoderConfig(layers=2, seq_len=S)
    layers = _layers(cfg, 2, 5)
    stack = FP8EncoderStack(cfg, layers, cuda_device)
    h = randn_f16((B, S, cfg.d_model), 6)
    y = stack.forward(h.to(cuda_device)).float().cpu()
    ref = ref_encoder.encoder_stack_ref(h, [ref_encoder.quantise_layer(lw) for lw in layers], cfg.heads).float()
    rel = gemm.rel_error(y, ref)
    assert rel <= STACK_GATE, f"stack relative error {rel:.3e}"
    assert (y - ref).abs().mean().item() < 5e-3


def test_stack_is_deterministic_and_host_path_agrees(cuda_device):
    cfg = EncoderConfig(layers=3, seq_len=128)
    stack = FP8EncoderStack(cfg, _layers(cfg, 3, 9), cuda_device)
    h = randn_f16((4, 128, cfg.d_model), 10)
    y1 = stack.forward(h.to(cuda_device)).clone()
    y2 = stack.forward(h.to(cuda_device)).clone()
    assert torch.equal(y1, y2)
    y3 = stack.forward_host(h.pin_memory())
    assert torch.equal(y3, y1.cpu())
    assert torch.isfinite(y1.float()).all()
