import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(REPO, "stt-web_b200")
for p in (PKG_DIR, REPO, os.path.join(REPO, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    # Build both native libraries once per session (make is a no-op when up to date).
    if os.environ.get("STT_SKIP_BUILD") != "1":
        subprocess.check_call(["make", "-s", "-C", os.path.join(REPO, "oracle")], stdout=subprocess.DEVNULL)
        subprocess.check_call(["make", "-s", "-j4", "-C", PKG_DIR], stdout=subprocess.DEVNULL,
                              stderr=subprocess.DEVNULL)


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def tiny_meta():
    import json
    return json.load(open(os.path.join(GOLDEN, "tiny_ref_meta.json")))


@pytest.fixture(scope="session")
def tiny_ref_gguf():
    import numpy as np
    return np.fromfile(os.path.join(GOLDEN, "tiny_ref.gguf"), dtype=np.uint8)
