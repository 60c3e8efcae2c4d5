"""The CPU oracle is pinned before it is trusted (CPU-only tests).

1. Against tests/golden/golden_v21.npz, made by make_golden.py from the reference's own CPU code
   (runtime/v21/src/pt_v21_host.c compiled from its sources): bit-exact.
2. Against that compiled reference code directly (oracle/_ref/libptref.so, when it was built in
   this tree) on further seeded shapes: bit-exact.
3. The numpy packers (prime-tts_b200/pt_b200.py) against the oracle's C packers.
"""
import os

import numpy as np
import pytest

import oracle
import pt_b200
from golden.make_golden import (CONV_CASES, CONVT_CASES, cfg1_inputs, cfg2_inputs, conv_inputs,
                                convT_inputs, tail_inputs)

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_v21.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


@pytest.fixture(scope="module")
def orc():
    return oracle.CpuDecoder("oracle")


@pytest.mark.parametrize("i", range(len(CONV_CASES)))
def test_conv_matches_golden(orc, gold, i):
    seed, B, cin, cout, K, pad, dil, T, e0, a0, e1, a1 = CONV_CASES[i]
    x, wp, b = conv_inputs(seed, B, cin, cout, K, T)
    y = orc.conv(x, wp, b, cout, K, pad, dil, e0, e1, a0, a1)
    assert np.array_equal(y, gold[f"conv{i}"])


@pytest.mark.parametrize("i", range(len(CONVT_CASES)))
def test_convT_matches_golden(orc, gold, i):
    seed, B, cin, cout, K, s, pad, T = CONVT_CASES[i]
    x, wp, b = convT_inputs(seed, B, cin, cout, K, s, T)
    y = orc.convT(x, wp, b, cout, K, s, pad)
    assert np.array_equal(y, gold[f"convT{i}"])


def test_tail_matches_golden(orc, gold):
    pq = pt_b200.pqmf_synthesis_filter()
    assert np.array_equal(orc.tail(tail_inputs(30, 16 * 8 + 1), pq), gold["tail_T8"])
    assert np.array_equal(orc.tail(tail_inputs(31, 16 * 3 + 1), pq), gold["tail_T3"])


def test_package_config_generators_match_the_fixture_inputs():
    """bench.py's configs 1 and 2 (pt_b200.config1 / config2) draw exactly the inputs the golden
    fixtures were made from."""
    for ours, fixture in ((pt_b200.config1(), cfg1_inputs()), (pt_b200.config2(), cfg2_inputs())):
        for a, b in zip(ours, fixture):
            assert np.array_equal(a, b)


def test_config1_config2_match_golden(orc, gold):
    x, wp, b = cfg1_inputs()
    y1 = orc.conv(x, wp, b, 256, 7, 3, 1, 1, 0, 0.1, 0.0).ravel()
    assert np.array_equal(y1[gold["cfg1_idx"]], gold["cfg1_val"])
    assert y1.astype(np.float64).sum() == gold["cfg1_sum"][0]
    x, wp, b = cfg2_inputs()
    y2 = orc.convT(x, wp, b, 256, 16, 4, 6).ravel()
    assert np.array_equal(y2[gold["cfg2_idx"]], gold["cfg2_val"])
    assert (y2.astype(np.float64) ** 2).sum() == gold["cfg2_sum"][1]


@pytest.mark.parametrize("T", [8, 13])
def test_decode_matches_golden(orc, gold, T):
    w, z = pt_b200.config3(seed=2, T=T)
    assert np.array_equal(orc.decode(w, z), gold[f"decode_T{T}"])


# ---- against the compiled reference itself (present where the reference tree was) ----------
def _ref():
    if not os.path.exists(oracle.LIB_REF):
        pytest.skip("oracle/_ref/libptref.so not built (reference sources absent)")
    return oracle.CpuDecoder("reference")


@pytest.mark.parametrize("seed", range(6))
def test_conv_bit_exact_vs_reference(orc, seed):
    ref = _ref()
    rng = np.random.default_rng(100 + seed)
    B = int(rng.integers(1, 3))
    cin, cout = int(rng.integers(1, 40)), int(rng.integers(1, 40))
    K = int(rng.choice([1, 3, 5, 7, 11]))
    dil = int(rng.choice([1, 2, 3, 5]))
    pad = dil * (K - 1) // 2
    T = int(rng.integers(1, 50))
    x, wp, b = conv_inputs(1000 + seed, B, cin, cout, K, T)
    e0, e1 = int(rng.integers(0, 5)), int(rng.integers(0, 5))
    args = (x, wp, b, cout, K, pad, dil, e0, e1, 0.1, -0.3)
    assert np.array_equal(orc.conv(*args), ref.conv(*args))


@pytest.mark.parametrize("seed", range(6))
def test_convT_bit_exact_vs_reference(orc, seed):
    ref = _ref()
    rng = np.random.default_rng(200 + seed)
    B = int(rng.integers(1, 3))
    cin, cout = int(rng.integers(1, 30)), int(rng.integers(1, 30))
    s = int(rng.integers(1, 5))
    K = int(rng.integers(s, 4 * s + 1))
    pad = int(rng.integers(0, (K + 1) // 2))
    T = int(rng.integers(2, 30))
    if (T - 1) * s - 2 * pad + K <= 0:
        pytest.skip("empty output")
    x, wp, b = convT_inputs(2000 + seed, B, cin, cout, K, s, T)
    args = (x, wp, b, cout, K, s, pad)
    assert np.array_equal(orc.convT(*args), ref.convT(*args))


@pytest.mark.parametrize("Tp", [2, 17, 49, 113, 161])
def test_tail_bit_exact_vs_reference(orc, Tp):
    ref = _ref()
    post = tail_inputs(300 + Tp, Tp)
    pq = pt_b200.pqmf_synthesis_filter()
    assert np.array_equal(orc.tail(post, pq), ref.tail(post, pq))


def test_decode_bit_exact_vs_reference(orc):
    ref = _ref()
    w, z = pt_b200.config3(seed=7, T=5)
    assert np.array_equal(orc.decode(w, z), ref.decode(w, z))


# ---- packers -----------------------------------------------------------------------------
def test_numpy_packers_match_oracle_packers():
    import ctypes as C
    lib = C.CDLL(oracle.LIB_ORACLE)
    f = C.POINTER(C.c_float)
    rng = np.random.default_rng(5)
    W = rng.standard_normal((6, 5, 7)).astype(np.float32)     # conv [cout][cin][K]
    out = np.zeros(lib.or_packed_conv_elems(6, 5, 7) if False else 8 * 7 * 5, np.float32)
    lib.or_pack_conv(W.ctypes.data_as(f), 6, 5, 7, out.ctypes.data_as(f))
    assert np.array_equal(out, pt_b200.pack_conv(W).ravel())
    Wt = rng.standard_normal((5, 6, 10)).astype(np.float32)   # convT [cin][cout][K], s=4
    n = 4 * 8 * 3 * 5
    out = np.zeros(n, np.float32)
    lib.or_pack_convT(Wt.ctypes.data_as(f), 5, 6, 10, 4, out.ctypes.data_as(f))
    assert np.array_equal(out, pt_b200.pack_convT(Wt, 4).ravel())


def test_metrics_definition():
    ref = np.array([1.0, -2.0, 4.0], np.float32)
    est = ref + np.array([0.0, 0.01, -0.02], np.float32)
    m = oracle.metrics(est, ref)
    assert abs(m["max_rel"] - 0.02 / 4.0) < 1e-6
    assert abs(m["sndr_db"] - 10 * np.log10(21.0 / (0.01 ** 2 + 0.02 ** 2))) < 1e-3


def test_flops_accounting_matches_survey():
    # 32.578 GFLOP per request at T = 226 frames (conv stack ~99.86 %)
    assert abs(pt_b200.decoder_gflop(226) - 32.578) < 0.01
    assert pt_b200.conv_gflop(226) / pt_b200.decoder_gflop(226) > 0.998
