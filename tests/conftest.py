import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "glimpse-language_b200")
for p in (PKG, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA kernels)")
    # build the checker and the library in-tree when they are missing (no rebuild when present: the GPU box gets
    # the prebuilt files)
    if not os.path.exists(os.path.join(ROOT, "oracle", "_build", "libbonsai_oracle.so")):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=True)
    if not all(os.path.exists(os.path.join(PKG, "bonsai_b200", f)) for f in ("libbonsai_cuda.so", "libbonsai_synth.so")):
        subprocess.run(["make", "-s", "-j8", "-C", PKG], check=True)


def has_gpu():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def gpu():
    if not has_gpu():
        pytest.skip("no GPU")
    return 0
