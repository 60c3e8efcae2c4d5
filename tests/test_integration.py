"""The drop-in claim, checked at link level (CPU-only): the reference's own graph interpreter and
driver (runtime/v21/src/pt_v21_host.c + main_v21.c), compiled for its CUDA build with
-DPT_V21_CUDA, link against libpt_b200.so with every CUDA-layer symbol resolved by this library.
"""
import os
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
from conftest import reference_dir

_REF = reference_dir()


def test_reference_interpreter_links_against_library():
    if not _REF:
        pytest.skip("reference sources not present on this machine")
    out = os.path.join(REPO, "oracle", "_ref", "pt_v21_b200")
    if os.path.exists(out):
        os.remove(out)
    subprocess.run(["make", "-s", "-C", os.path.join(REPO, "oracle"), "interp", f"REF={_REF}"],
                   check=True)
    assert os.path.exists(out)
    ldd = subprocess.run(["ldd", out], capture_output=True, text=True).stdout
    assert "libpt_b200.so" in ldd and "not found" not in ldd
    # the interpreter resolves its CUDA layer here (no pt_v21_cuda.o was linked)
    nm = subprocess.run(["nm", "-u", out], capture_output=True, text=True).stdout
    for sym in ("pt_v21_conv", "pt_v21_convT", "pt_v21_matmul", "pt_v21_cuda_init"):
        assert sym in nm
    # it runs up to opening its (absent) trained container
    r = subprocess.run([out], capture_output=True, text=True, timeout=60)
    assert "v21.ptk" in (r.stdout + r.stderr)
