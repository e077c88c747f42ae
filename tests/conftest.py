import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "whisper-blaze_b200")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN_DIR = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built libwbk.so")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but no CUDA device is visible")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.fail(f"these kernels are built for sm_100a only; device is sm_{major}{minor}")
    return torch.device("cuda:0")


def seeded(seed: int):
    import torch
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def randn_f16(shape, seed: int, std: float = 1.0):
    """Seeded N(0, std) generated on the CPU in fp32, then rounded to fp16."""
    import torch
    return (torch.randn(*shape, generator=seeded(seed), dtype=torch.float32) * std).half()
