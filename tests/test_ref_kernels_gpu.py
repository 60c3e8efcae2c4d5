"""The reference's own CUDA kernels (runtime/v21/src/pt_v21_cuda.cu, recompiled for sm_100a by
`make -C oracle refcuda` into oracle/_ref/libptref_cuda.so) against this library, through the same
C ABI (pt_v21_conv / pt_v21_convT), on the same B200 and the same inputs: config 1, config 2 and
every distinct layer shape of the config-3 decoder.

Both libraries get the reference's steady state: weights resident on the device by container index
(the reference uploads the pt_ctx container table in pt_v21_cuda_init, pt_v21_cuda.cu:120-215;
this library caches by the same indices), host tensors in and out of every call, synchronous
calls.  Results must agree with the CPU oracle (reference path: its own claimed bit-identity with
the CPU kernels, pt_v21_cuda.cu:980-985; this library: the 1e-3 per-op gate).  The per-call times
are printed (`-s`); kernel-only times come from an ncu launch list of this test.
"""
import ctypes as C
import os
import time

import numpy as np
import pytest

import oracle
import pt_b200

REF = os.path.join(os.path.dirname(oracle.HERE), "oracle", "_ref", "libptref_cuda.so")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.exists(REF), reason="oracle/_ref/libptref_cuda.so not built")]

# (name, kind, cin, cout, K, dil or stride, T, epi): config 1, config 2, and the config-3 layers
CASES = [
    ("cfg1 conv 512->256 k7", "conv", 512, 256, 7, 1, 256, 1),
    ("cfg2 convT 512->256 k16 s4", "convT", 512, 256, 16, 4, 256, 0),
    ("conv_pre 192->512 k7 T226", "conv", 192, 512, 7, 1, 226, 1),
    ("ups.0 512->256 T226", "convT", 512, 256, 16, 4, 226, 0),
    ("L1 k3 d1 256ch T904", "conv", 256, 256, 3, 1, 904, 1),
    ("L1 k7 d3 256ch T904", "conv", 256, 256, 7, 3, 904, 1),
    ("L1 k11 d5 256ch T904", "conv", 256, 256, 11, 5, 904, 1),
    ("ups.1 256->128 T904", "convT", 256, 128, 16, 4, 904, 0),
    ("L2 k3 d1 128ch T3616", "conv", 128, 128, 3, 1, 3616, 1),
    ("L2 k11 d5 128ch T3616", "conv", 128, 128, 11, 5, 3616, 1),
    ("conv_post 128->72 k7 T3617", "conv", 128, 72, 7, 1, 3617, 0),
]


def _case_arrays(i, kind, cin, cout, K, ds, T):
    rng = np.random.default_rng(100 + i)
    x = rng.standard_normal((1, cin, T)).astype(np.float32)
    if kind == "conv":
        W = (0.02 * rng.standard_normal((cout, cin, K))).astype(np.float32)
        wp = pt_b200.pack_conv(W)
    else:
        W = (0.02 * rng.standard_normal((cin, cout, K))).astype(np.float32)
        wp = pt_b200.pack_convT(W, ds)
    b = (0.01 * rng.standard_normal(cout)).astype(np.float32)
    return x, W, wp, b


class _RefContext(pt_b200.Context):
    """pt_b200.Context's calls routed to the reference CUDA library, with a container table."""

    def __init__(self, records):
        self._lib = C.CDLL(REF)
        for name, (args, res) in pt_b200._SIGS.items():
            if name.startswith("pt_v21_") and hasattr(self._lib, name):
                f = getattr(self._lib, name)
                f.argtypes, f.restype = args, res
        self._keep = records
        n = len(records)
        self._ptrs = (C.c_void_p * n)(*[r.ctypes.data for r in records])
        self._lens = (C.c_int64 * n)(*[r.size for r in records])
        self.ctx = pt_b200.PtCtx()
        self.ctx.conv_pad_in = -1
        self.ctx.cont_f32 = C.cast(self._ptrs, C.c_void_p)
        self.ctx.cont_n = C.cast(self._lens, C.c_void_p)
        self.ctx.n_cont = n
        if self._lib.pt_v21_cuda_init(C.byref(self.ctx), 0) != 0:
            raise RuntimeError("reference pt_v21_cuda_init failed")
        self.device = 0

    def close(self):
        if self.ctx.use_cuda:
            self._lib.pt_v21_cuda_shutdown(C.byref(self.ctx))


@pytest.fixture(scope="module")
def setup():
    arrays = [_case_arrays(i, c[1], c[2], c[3], c[4], c[5], c[6]) for i, c in enumerate(CASES)]
    records = []
    for x, W, wp, b in arrays:
        records += [wp, b]
    ours = pt_b200.Context(0)
    ref = _RefContext(records)
    yield arrays, ours, ref
    ref.close()
    ours.close()


def _run(ctx, libfun, case, arr, i):
    name, kind, cin, cout, K, ds, T, epi = case
    x, W, wp, b = arr
    with _Routed(ctx, libfun):
        if kind == "conv":
            pad = ds * (K - 1) // 2
            return ctx.conv(x, wp, b, cout, K, pad, ds, epi0=epi, a0=0.1, wtab=2 * i, btab=2 * i + 1)
        return ctx.convT(x, wp, b, cout, K, ds, (K - ds) // 2, wtab=2 * i, btab=2 * i + 1)


class _Routed:
    """Temporarily point pt_b200.lib() at another ctypes library (the reference's)."""

    def __init__(self, ctx, libfun):
        self.libfun = libfun

    def __enter__(self):
        self.saved = pt_b200.lib
        if self.libfun is not None:
            pt_b200.lib = self.libfun

    def __exit__(self, *a):
        pt_b200.lib = self.saved


def _time(fn, n=5):
    fn()
    fn()
    ts = []
    for _ in range(n):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return 1e3 * float(np.median(ts))


def test_reference_kernels_vs_ours(setup):
    arrays, ours, ref = setup
    orc = oracle.CpuDecoder("oracle")
    lines = []
    for i, (case, arr) in enumerate(zip(CASES, arrays)):
        name, kind, cin, cout, K, ds, T, epi = case
        x, W, wp, b = arr
        y_ref = _run(ref, lambda: ref._lib, case, arr, i)
        y_us = _run(ours, None, case, arr, i)
        if kind == "conv":
            pad = ds * (K - 1) // 2
            y_orc = orc.conv(x, wp, b, cout, K, pad, ds, epi0=epi, a0=0.1)
        else:
            y_orc = orc.convT(x, wp, b, cout, K, ds, (K - ds) // 2)
        y_ref, y_us, y_orc = y_ref[0, :cout], y_us[0, :cout], y_orc[0, :cout]
        m_ref = oracle.metrics(y_ref, y_orc)
        m_us = oracle.metrics(y_us, y_orc)
        assert m_ref["max_rel"] <= 1e-5, (name, m_ref)
        assert m_us["max_rel"] <= 1e-3, (name, m_us)
        t_ref = _time(lambda: _run(ref, lambda: ref._lib, case, arr, i))
        t_us = _time(lambda: _run(ours, None, case, arr, i))
        lines.append(f"| {name} | {t_ref:.3f} | {t_us:.3f} | {t_ref / t_us:.1f} | "
                     f"{m_ref['max_rel']:.1e} | {m_us['max_rel']:.1e} |")
    print("\n| op (C ABI call, host tensors) | reference CUDA ms | ours ms | ratio | ref max_rel | "
          "ours max_rel |\n|---|---:|---:|---:|---:|---:|\n" + "\n".join(lines))
