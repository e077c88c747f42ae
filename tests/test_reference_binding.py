"""The reference's own model.py binds to this drop-in module unchanged (no GPU needed).

whisper_blaze/model.py does `import whisper_blaze_kernels as _kernels` inside a
try/except and calls the ops below with positional arguments. With this
repository's `whisper_blaze_kernels` on sys.path, importing the reference's
model.py (its package __init__ is skipped: it pulls in the audio processor)
must bind `_kernels` to this module, report the kernels as available, and
every call model.py makes must bind to the drop-in signature.

The reference tree is found through WBK_REFERENCE_DIR, else a `reference`
directory beside this repository; the test skips where it is absent (GPU boxes).
"""
import importlib
import inspect
import os
import sys
import types

import pytest

from oracle import build_ref

REF = build_ref.DEFAULT_REFERENCE
MODEL_PY = os.path.join(REF, "whisper_blaze", "model.py")

pytestmark = pytest.mark.skipif(not os.path.exists(MODEL_PY), reason="reference tree not present")

# (op, positional arguments as model.py passes them: whisper_blaze/model.py:76-78, :94-106, :161-162, :221-225)
CALLS = [
    ("quantise_e4m3", ("w_fp16",)),
    ("quantise_e5m2", ("w_fp16",)),
    ("dequantise_e4m3", ("a_fp8", "a_scale", "shape")),
    ("dequantise_e5m2", ("a_fp8", "a_scale", "shape")),
    ("layernorm_fused", ("x", "residual", "weight", "bias", "eps")),
    ("encoder_self_attn", ("Q", "K", "V")),
    ("decoder_cross_attn", ("Q", "K", "V")),
    ("decoder_self_attn", ("Q", "K", "V")),
]


@pytest.fixture
def reference_model():
    saved = {k: v for k, v in sys.modules.items() if k == "whisper_blaze" or k.startswith("whisper_blaze.")}
    for k in saved:
        del sys.modules[k]
    pkg = types.ModuleType("whisper_blaze")
    pkg.__path__ = [os.path.dirname(MODEL_PY)]  # a package without running its __init__
    sys.modules["whisper_blaze"] = pkg
    try:
        yield importlib.import_module("whisper_blaze.model")
    finally:
        for k in [k for k in sys.modules if k == "whisper_blaze" or k.startswith("whisper_blaze.")]:
            del sys.modules[k]
        sys.modules.update(saved)


def test_reference_model_binds_this_module(reference_model):
    import whisper_blaze_kernels
    assert reference_model._KERNELS_AVAILABLE is True
    assert reference_model._kernels is whisper_blaze_kernels
    assert os.path.dirname(whisper_blaze_kernels.__file__).endswith(os.path.join("whisper-blaze_b200",
                                                                                   "whisper_blaze_kernels"))


@pytest.mark.parametrize("op,args", CALLS)
def test_every_model_call_binds_to_the_drop_in_signature(reference_model, op, args):
    fn = getattr(reference_model._kernels, op)
    inspect.signature(fn).bind(*args)  # raises TypeError on an arity mismatch


def test_reference_layernorm_module_routes_cuda_fp16_to_the_kernel(reference_model):
    """BlazeLayerNorm.forward's kernel branch (model.py:155-162) calls layernorm_fused with
    (x, residual, weight, bias, eps); on a CPU tensor it takes torch's path, so here the
    call is made directly and must fail in the drop-in's own CUDA check, not on arity."""
    import torch
    ln = reference_model.BlazeLayerNorm(torch.ones(1280, dtype=torch.float16), torch.zeros(1280, dtype=torch.float16))
    x = torch.randn(2, 1280).half()
    y = ln(x)  # CPU: the reference's torch fallback
    assert y.shape == x.shape
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        reference_model._kernels.layernorm_fused(x, None, ln.weight, ln.bias, ln.eps)
