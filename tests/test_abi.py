"""The C ABI of libpt_b200.so (CPU-only: no compute call reaches a GPU).

* every entry point include/pt_b200.h declares is exported by the library;
* pt_ctx has exactly the reference interpreter's layout (runtime/v21/src/pt_v21.h:79-162), so the
  interpreter built with -DPT_V21_CUDA can hand its contexts to this library;
* a context that was never initialised for the GPU makes compute calls fail loudly (-1 and a
  message): the library has no CPU path.
"""
import ctypes as C
import os
import re
import subprocess
import tempfile

import numpy as np
import pytest

import pt_b200
from conftest import reference_dir

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HDR = os.path.join(REPO, "include", "pt_b200.h")
_REF = reference_dir()
REF_HDR_DIR = os.path.join(_REF, "runtime", "v21", "src") if _REF else None


def declared_symbols():
    text = open(HDR).read()
    return sorted(set(re.findall(r"^PT_B200_API [^(]*?\b((?:pt_v21|pt_b200)_\w+)\(", text, re.M)))


def test_header_declares_the_reference_boundary():
    names = set(declared_symbols())
    # the reference CUDA layer's symbols (runtime/v21/src/pt_v21.h:208-259)
    boundary = {"pt_v21_cuda_init", "pt_v21_cuda_prewarm", "pt_v21_cuda_shutdown", "pt_v21_conv",
                "pt_v21_convT", "pt_v21_matmul", "pt_v21_conv_pads_in_kernel",
                "pt_v21_devadd_run", "pt_v21_devleaky_run", "pt_v21_dev_upload",
                "pt_v21_dev_sync_host", "pt_v21_dev_alloc", "pt_v21_dev_free",
                "pt_v21_dev_reclaim", "pt_v21_cuda_active", "pt_v21_cuda_weights_mib",
                "pt_v21_cuda_keepwarm", "pt_v21_gpu_cur_freq", "pt_v21_gpu_max_freq"}
    assert boundary <= names, boundary - names


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", pt_b200.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    missing = set(declared_symbols()) - exported
    assert not missing, missing
    lib = pt_b200.lib()  # loads without a GPU and binds every signature
    for name in declared_symbols():
        assert hasattr(lib, name)


_FIELDS = [f for f, _ in pt_b200.PtCtx._fields_]


def _probe_offsets(include_line: str, incdir: str):
    src = ["#include <stdio.h>", "#include <stddef.h>", include_line, "int main(void){"]
    src.append('printf("sizeof %zu\\n", sizeof(struct pt_ctx));')
    for f in _FIELDS:
        src.append(f'printf("{f} %zu\\n", offsetof(struct pt_ctx, {f}));')
    src.append('printf("tv %zu\\n", sizeof(pt_tv)); return 0;}')
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "probe.c")
        exe = os.path.join(d, "probe")
        open(c, "w").write("\n".join(src))
        subprocess.run(["gcc", "-std=gnu11", "-I", incdir, c, "-o", exe], check=True)
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout
    return {k: int(v) for k, v in (l.split() for l in out.splitlines())}


def test_ctx_layout_matches_our_header_and_ctypes():
    got = _probe_offsets('#include "pt_b200.h"', os.path.join(REPO, "include"))
    assert got["sizeof"] == C.sizeof(pt_b200.PtCtx)
    assert got["tv"] == C.sizeof(pt_b200.PtTv)
    for f in _FIELDS:
        assert got[f] == getattr(pt_b200.PtCtx, f).offset, f


def test_ctx_layout_matches_the_reference_header():
    if not REF_HDR_DIR or not os.path.exists(os.path.join(REF_HDR_DIR, "pt_v21.h")):
        pytest.skip("reference header not present on this machine")
    ref = _probe_offsets('#include "pt_v21.h"', REF_HDR_DIR)
    ours = _probe_offsets('#include "pt_b200.h"', os.path.join(REPO, "include"))
    assert ref == ours


def test_uninitialised_context_fails_loudly():
    lib = pt_b200.lib()
    ctx = pt_b200.PtCtx()  # use_cuda == 0: the interpreter's --no-cuda context
    x = np.ones((1, 4, 8), np.float32)
    y = np.zeros((1, 4, 8), np.float32)
    w = np.zeros(4 * 1 * 4, np.float32)
    f = C.POINTER(C.c_float)
    rc = lib.pt_v21_conv(C.byref(ctx), x.ctypes.data_as(f), 8, 4, y.ctypes.data_as(f), 8, 8, 4, 1,
                         1, 0, 1, w.ctypes.data_as(f), None, 1, -1, -1, 0, 0, 0.0, 0.0)
    assert rc == -1
    assert b"no CPU path" in lib.pt_b200_last_error()
    assert np.all(y == 0)  # nothing was computed on the host
    rc = lib.pt_v21_convT(C.byref(ctx), x.ctypes.data_as(f), 8, 4, 8, y.ctypes.data_as(f), 8, 1, 1,
                          0, 1, w.ctypes.data_as(f), None, 1, -1, -1)
    assert rc == -1
    assert lib.pt_v21_conv_pads_in_kernel(C.byref(ctx)) == 1


def test_decoder_create_without_gpu_returns_null():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    w = pt_b200.make_decoder_weights(np.random.default_rng(0))
    cw = w.as_c()
    assert not pt_b200.lib().pt_b200_decoder_create(0, C.byref(cw))
