"""Parity of the tensor-core Conv1d / ConvTranspose1d / MatMul entry points (pt_v21_conv,
pt_v21_convT, pt_v21_matmul through the C ABI) against the CPU oracle.

Tolerance: the reference's per-op gate, max|a-b| / max|b| <= 1e-3 (tests/v21_reference.py:
430-437, 502), with TF32 operands (10-bit mantissa, round-to-nearest) and fp32 accumulation.
"""
import ctypes as C

import numpy as np
import pytest

import oracle
import pt_b200
from golden.make_golden import CONV_CASES, CONVT_CASES, cfg1_inputs, cfg2_inputs, conv_inputs, convT_inputs

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.fixture(scope="module")
def ctx():
    c = pt_b200.Context(0)
    yield c
    c.close()


@pytest.fixture(scope="module")
def orc():
    return oracle.CpuDecoder("oracle")


def _close(y, ref, tol=TOL):
    m = oracle.metrics(y, ref)
    assert m["max_rel"] <= tol, m
    return m


def test_config1_conv_512_256_k7(ctx, orc):
    x, wp, b = cfg1_inputs()
    ref = orc.conv(x, wp, b, 256, 7, 3, 1, 1, 0, 0.1, 0.0)
    y = ctx.conv(x, wp, b, 256, 7, 3, 1, epi0=1, a0=0.1)
    m = _close(y, ref)
    assert m["sndr_db"] > 60


def test_config2_convT_512_256_k16_s4(ctx, orc):
    x, wp, b = cfg2_inputs()
    ref = orc.convT(x, wp, b, 256, 16, 4, 6)
    y = ctx.convT(x, wp, b, 256, 16, 4, 6)
    m = _close(y, ref)
    assert m["sndr_db"] > 60
    # the fused-epilogue extension: convT + LeakyReLU 0.1
    y2 = ctx.convT(x, wp, b, 256, 16, 4, 6, epi0=1, a0=0.1)
    _close(y2, np.where(ref >= 0, ref, np.float32(0.1) * ref))


@pytest.mark.parametrize("i", range(len(CONV_CASES)))
def test_conv_cases(ctx, orc, i):
    seed, B, cin, cout, K, pad, dil, T, e0, a0, e1, a1 = CONV_CASES[i]
    x, wp, b = conv_inputs(seed, B, cin, cout, K, T)
    ref = orc.conv(x, wp, b, cout, K, pad, dil, e0, e1, a0, a1)
    _close(ctx.conv(x, wp, b, cout, K, pad, dil, e0, e1, a0, a1), ref)
    _close(ctx.conv(x, wp, b, cout, K, pad, dil, e0, e1, a0, a1, padded_input=True), ref)


@pytest.mark.parametrize("i", range(len(CONVT_CASES)))
def test_convT_cases(ctx, orc, i):
    seed, B, cin, cout, K, s, pad, T = CONVT_CASES[i]
    x, wp, b = convT_inputs(seed, B, cin, cout, K, s, T)
    _close(ctx.convT(x, wp, b, cout, K, s, pad), orc.convT(x, wp, b, cout, K, s, pad))


# the decoder's own conv shapes at a ragged length (tiles partly filled, T not a multiple of 128)
@pytest.mark.parametrize("cin,cout,K,dil,T", [(192, 512, 7, 1, 226), (256, 256, 11, 5, 300),
                                               (128, 128, 3, 3, 1000), (128, 72, 7, 1, 161),
                                               (256, 256, 7, 3, 129), (128, 128, 11, 1, 5),
                                               (64, 64, 15, 5, 200)])   # halo 70: per-tap kernel
def test_decoder_conv_shapes(ctx, orc, cin, cout, K, dil, T):
    x, wp, b = conv_inputs(7 * cin + K + T, 1, cin, cout, K, T)
    pad = dil * (K - 1) // 2
    _close(ctx.conv(x, wp, b, cout, K, pad, dil, 1, 0, 0.1, 0.0),
           orc.conv(x, wp, b, cout, K, pad, dil, 1, 0, 0.1, 0.0))


@pytest.mark.parametrize("cin,cout,T", [(512, 256, 226), (256, 128, 904), (256, 128, 3)])
def test_decoder_upsampler_shapes(ctx, orc, cin, cout, T):
    x, wp, b = convT_inputs(cin + T, 1, cin, cout, 16, 4, T)
    _close(ctx.convT(x, wp, b, cout, 16, 4, 6), orc.convT(x, wp, b, cout, 16, 4, 6))


def test_resident_weights_reused(ctx, orc):
    x, wp, b = conv_inputs(41, 1, 64, 64, 3, 50)
    y1 = ctx.conv(x, wp, b, 64, 3, 1, 1, wtab=900, btab=901)
    y2 = ctx.conv(x, wp, b, 64, 3, 1, 1, wtab=900, btab=901)   # served from the device copy
    assert np.array_equal(y1, y2)
    _close(y1, orc.conv(x, wp, b, 64, 3, 1, 1))
    assert pt_b200.lib().pt_v21_cuda_weights_mib(ctx.ptr) > 0


def test_conv_chain_stays_on_device(ctx, orc):
    """conv_keep / conv_in_dev (pt_v21_host.c:3334-3366): the first conv's output never comes
    back to the host; the second conv reads it from the device."""
    lib = pt_b200.lib()
    x, w1, b1 = conv_inputs(51, 1, 64, 64, 3, 77)
    _, w2, b2 = conv_inputs(52, 1, 64, 32, 5, 77)
    ref = orc.conv(orc.conv(x, w1, b1, 64, 3, 1, 1, 1, 0, 0.1, 0.0), w2, b2, 32, 5, 2, 1)
    f = C.POINTER(C.c_float)
    c = ctx.ctx
    y1 = np.full((1, 64, 77), 7.0, np.float32)
    c.conv_pad_in = 1
    c.conv_keep = 1
    rc = lib.pt_v21_conv(ctx.ptr, x.ctypes.data_as(f), 77, 64, y1.ctypes.data_as(f), 77, 77, 64,
                         3, 1, 1, 1, w1.ctypes.data_as(f), b1.ctypes.data_as(f), 1, -1, -1, 1, 0,
                         0.1, 0.0)
    c.conv_keep = 0
    assert rc == 0 and c.conv_out_dev and np.all(y1 == 7.0)
    c.conv_in_dev = c.conv_out_dev
    c.conv_pad_in = 2
    y2 = np.empty((1, 32, 77), np.float32)
    rc = lib.pt_v21_conv(ctx.ptr, None, 77, 64, y2.ctypes.data_as(f), 77, 77, 32, 5, 1, 2, 1,
                         w2.ctypes.data_as(f), b2.ctypes.data_as(f), 1, -1, -1, 0, 0, 0.0, 0.0)
    c.conv_in_dev = None
    assert rc == 0
    assert c.chain_mark is None and c.g_arena_used == 0  # the chain's arena range was released
    _close(y2, ref, 2e-3)


def test_matmul(ctx):
    rng = np.random.default_rng(3)
    for m, k, n in [(37, 192, 70), (300, 96, 5), (8, 1, 300)]:
        A = rng.standard_normal((m, k)).astype(np.float32)
        B = rng.standard_normal((k, n)).astype(np.float32)
        ref = (A.astype(np.float64) @ B.astype(np.float64)).astype(np.float32)
        _close(ctx.matmul(A, B), ref)


def test_device_add_and_leaky(ctx):
    lib = pt_b200.lib()
    rng = np.random.default_rng(4)
    a = rng.standard_normal(10007).astype(np.float32)
    b = rng.standard_normal(10007).astype(np.float32)
    da = lib.pt_v21_dev_upload(ctx.ptr, a.ctypes.data, a.size)
    db = lib.pt_v21_dev_upload(ctx.ptr, b.ctypes.data, b.size)
    dy = lib.pt_v21_dev_alloc(ctx.ptr, a.size * 4)
    assert da and db and dy
    assert lib.pt_v21_devadd_run(ctx.ptr, da, db, dy, a.size, 1, C.c_float(0.1)) == 0
    y = np.empty_like(a)
    lib.pt_v21_dev_sync_host(ctx.ptr, y.ctypes.data, dy, a.size)
    s = a + b
    assert np.array_equal(y, np.where(s >= 0, s, np.float32(0.1) * s))
    for p in (da, db, dy):
        lib.pt_v21_dev_free(ctx.ptr, p)


def test_kernel_launch_counter(ctx):
    pt_b200.kernel_launches(reset=True)
    x, wp, b = conv_inputs(61, 1, 32, 32, 3, 64)
    ctx.conv(x, wp, b, 32, 3, 1, 1)
    assert pt_b200.kernel_launches() >= 2   # staging + tensor-core conv
