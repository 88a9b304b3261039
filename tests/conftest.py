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


@pytest.fixture(scope="session")
def synth_model_path(tmp_path_factory):
    """The seeded synthetic model: $NLLB_SYNTH_MODEL when set, else written
    once per session outside the repository (about 860 MB, ~30 s)."""
    from nllb_attn import synth_model as sm
    path = os.environ.get("NLLB_SYNTH_MODEL") or str(tmp_path_factory.mktemp("synth") / "synth_seed0.safetensors")
    return sm.ensure_model(path, seed=0)
