"""The live tensor-core rate probe (pt_b200_mma_rate): the conv roofline's denominator.

tcgen05.mma kind::tf32 at M128 x N256 x K8 retires 4,096 FLOP per SM clock on B200 (one
instruction per 128 cycles); the probe must measure that, one CTA per SM, and report a clock and
an aggregate rate consistent with it.  bench.py divides the conv stack's FLOP rate by the probe's
TFLOP/s for `frac_mma`.
"""
import pytest

import pt_b200

pytestmark = pytest.mark.gpu


def test_probe_measures_the_tf32_issue_rate():
    runs = [pt_b200.mma_rate(0) for _ in range(3)]
    print("\nkind::tf32 probe:", runs)
    for r in runs:
        assert 3900.0 <= r["flop_per_clk_sm"] <= 4200.0, r
        assert 500.0 <= r["sm_mhz"] <= 2100.0, r
        # aggregate = per-SM rate x 148 SMs x the clock the run held (the run's slowest CTA sets
        # the wall time, so the aggregate is at most that product)
        ideal = r["flop_per_clk_sm"] * 148 * r["sm_mhz"] * 1e6 / 1e12
        assert 0.9 * ideal <= r["tflops"] <= 1.01 * ideal, (r, ideal)


def test_probe_rejects_bad_arguments():
    import ctypes as C
    f, t, m = C.c_double(), C.c_double(), C.c_double()
    assert pt_b200.lib().pt_b200_mma_rate(0, 0, C.byref(f), C.byref(t), C.byref(m)) == -1
    assert b"bad arguments" in pt_b200.lib().pt_b200_last_error()
