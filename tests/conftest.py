import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(REPO, "bare-metal-nllb_b200")
for p in (PKG_DIR, os.path.join(REPO, "oracle"), os.path.join(REPO, "tests"),
          os.path.join(REPO, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def _ensure_built():
    so = os.path.join(PKG_DIR, "libnllb_attn.so")
    if not os.path.exists(so):
        subprocess.run(["make", "-C", PKG_DIR], check=True, stdout=subprocess.DEVNULL)
    oso = os.path.join(REPO, "oracle", "_build", "liboracle.so")
    if not os.path.exists(oso):
        subprocess.run(["make", "-C", os.path.join(REPO, "oracle"), "oracle"], check=True,
                       stdout=subprocess.DEVNULL)


_ensure_built()


@pytest.fixture(scope="session")
def cuda_device():
    """Device 0 as a torch device; the GPU tests need it to exist."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    return torch.device("cuda:0")
