"""Shared test setup: import paths, the `gpu` marker, and the libraries the tests load.

CPU tests (-m "not gpu") cover the oracle against the golden fixtures and against the reference's
own compiled CPU code, the host logic, and the C ABI's exported surface.  GPU tests (-m gpu) are
the parity tests proper: they call libpt_b200.so through its C ABI and compare with the oracle.
"""
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "prime-tts_b200")
for p in (REPO, PKG, os.path.join(REPO, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def reference_dir():
    """The reference project's source tree: $PT_REFERENCE_DIR, else the `reference_path` recorded
    in BASELINE.json; None when it is not on this machine (the GPU box has none)."""
    import json
    d = os.environ.get("PT_REFERENCE_DIR")
    if not d:
        try:
            with open(os.path.join(REPO, "BASELINE.json")) as f:
                d = json.load(f).get("reference_path")
        except Exception:
            d = None
    return d if d and os.path.isdir(d) else None


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA library)")


def _make(path):
    subprocess.run(["make", "-s", "-C", path], check=True)


@pytest.fixture(scope="session", autouse=True)
def _built_libraries():
    """Build the oracle (always cheap) and the CUDA library when they are missing."""
    if not os.path.exists(os.path.join(REPO, "oracle", "liboracle.so")):
        _make(os.path.join(REPO, "oracle"))
    if not os.path.exists(os.path.join(PKG, "libpt_b200.so")):
        _make(PKG)
    yield


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def ref_available():
    return os.path.exists(os.path.join(REPO, "oracle", "_ref", "libptref.so"))
