"""Streaming window plans and the exactness argument, on the CPU.

The library's overlap-save plan (pt_b200_stream_plan, exact = 0) must be the reference driver's
loop (runtime/v21/src/main_v21.c:342-364, restated in oracle.overlap_save_windows).  The exact
plan keeps that emission schedule and widens every window to the decoder's receptive radius
(25 frames back, 24 ahead); decoding its windows with the CPU oracle and stitching them must give
the whole-utterance decode bit for bit, while the reference's (64, 16) scheme does not.
"""
import numpy as np
import pytest

import oracle
import pt_b200

CASES_T = [2, 20, 33, 48, 63, 64, 65, 96, 97, 100, 129, 1000]
SCHEMES = [(64, 16), (48, 16), (64, 8), (256, 16), (81, 25)]


@pytest.mark.parametrize("win,ctx", SCHEMES)
def test_overlap_save_plan_is_the_reference_loop(win, ctx):
    plan = pt_b200.stream_plan(CASES_T, win, ctx, exact=False)
    k, zo, wo = 0, 0, 0
    for T in CASES_T:
        olen = 0
        for a, we, lo, hi in oracle.overlap_save_windows(T, win, ctx):
            frames, z_off, z_ld, klo, khi, dst = plan[k]
            assert (frames, z_off, z_ld, klo, khi, dst) == (we, zo + a, T, lo, hi, wo + olen)
            olen += hi - lo
            k += 1
        assert olen == 256 * T   # the reference loop emits every sample once
        zo += 192 * T
        wo += 256 * T
    assert k == len(plan)


@pytest.mark.parametrize("win,ctx", SCHEMES)
def test_exact_plan_covers_and_has_full_context(win, ctx):
    plan = pt_b200.stream_plan(CASES_T, win, ctx, exact=True)
    step = max(1, win - 2 * ctx)
    cl, cr = max(ctx, 25), max(ctx, 24)
    k, zo, wo = 0, 0, 0
    for T in CASES_T:
        nxt = 0   # next sample of this stream to emit
        for e in range(0, T, step):
            frames, z_off, z_ld, klo, khi, dst = plan[k]
            a = z_off - zo
            e1 = min(T, e + step)
            assert z_ld == T and frames >= 2 and 0 <= a and a + frames <= T
            assert dst == wo + 256 * e == wo + nxt            # contiguous, in order
            assert (klo, khi) == (256 * (e - a), 256 * (e1 - a))
            assert e - a >= min(cl, e) and a + frames - e1 >= min(cr, T - e1)
            nxt = 256 * e1
            k += 1
        assert nxt == 256 * T
        zo += 192 * T
        wo += 256 * T
    assert k == len(plan)


@pytest.fixture(scope="module")
def weights():
    return pt_b200.config3()[0]


def test_exact_scheme_is_bit_exact_on_the_oracle(weights):
    """Stitched exact windows == whole decode, bitwise, on the reference-exact CPU oracle; the
    same windows with one frame less of right context already differ."""
    orc = oracle.CpuDecoder("oracle")
    T = 90
    z = np.random.default_rng(11).standard_normal((192, T)).astype(np.float32)
    full = orc.decode(weights, z)
    plan = pt_b200.stream_plan([T], 64, 16, exact=True)
    wins = [(int(r[1]), int(r[0]), int(r[3]), int(r[4])) for r in plan]
    got = oracle.stitch(lambda zz: orc.decode(weights, zz), z, wins)
    np.testing.assert_array_equal(got, full)
    # the interior window with its right context cut to 23 frames is no longer exact
    a, we, lo, hi = wins[1]
    short = orc.decode(weights, np.ascontiguousarray(z[:, a:a + we - (we - hi // 256 - 23)]))
    assert not np.array_equal(short[lo:hi], full[256 * 32: 256 * 64])


def test_reference_scheme_deviation_on_the_reference_cpu(weights, ref_available):
    """The reference's own CPU decoder, stitched with its (64, 16) overlap-save loop, deviates
    from its whole decode by far more than 1e-6 on these weights (the receptive radius is 25
    frames, the context 16)."""
    kind = "reference" if ref_available else "oracle"
    dec = oracle.CpuDecoder(kind)
    T = 80
    z = np.random.default_rng(12).standard_normal((192, T)).astype(np.float32)
    full = dec.decode(weights, z)
    got = oracle.stitch(lambda zz: dec.decode(weights, zz), z, oracle.overlap_save_windows(T, 64, 16))
    m = oracle.metrics(got, full)
    print(f"reference CPU ({kind}) overlap-save (64,16) vs whole decode, T={T}: "
          f"max|d| {m['max_abs']:.3e}  SNDR {m['sndr_db']:.1f} dB")
    assert got.shape == full.shape
    assert m["max_abs"] > 1e-6 and m["sndr_db"] > 20.0


# ---- carried-state streaming: the pass plan (pt_b200_carry_plan) -----------------------------

CARRY_CHUNKS = [1, 7, 32, 64, 1000]


@pytest.mark.parametrize("chunk", CARRY_CHUNKS)
def test_carry_plan_emits_every_sample_once_in_order(chunk):
    """Pass after pass, each stream's emitted ranges are contiguous, start at 0, never go back,
    and the stream's flush pass (the one after the pass that delivers its last frame) ends at
    256 T; the pass delivering the last frame still holds back the look-ahead."""
    n, lo, hi = pt_b200.carry_plan(CASES_T, chunk)
    assert n == -(-max(CASES_T) // chunk) + 1
    for s, T in enumerate(CASES_T):
        assert lo[0, s] == 0
        np.testing.assert_array_equal(lo[1:, s], hi[:-1, s])
        assert (hi[:, s] >= lo[:, s]).all()
        last = -(-T // chunk)
        assert hi[last, s] == 256 * T and (hi[last:, s] == 256 * T).all()
        assert hi[last - 1, s] < 256 * T


@pytest.mark.parametrize("chunk", CARRY_CHUNKS)
def test_carry_plan_emits_only_samples_whose_frames_have_arrived(chunk):
    """A sample of latent frame f needs frames up to f + 24 (the receptive radius): before a
    stream's last frame has arrived, a pass may emit only samples of frames <= arrived - 25."""
    n, lo, hi = pt_b200.carry_plan(CASES_T, chunk)
    for s, T in enumerate(CASES_T):
        for k in range(n):
            arrived = min(T, (k + 1) * chunk)
            if arrived < T and hi[k, s] > 0:
                assert (hi[k, s] - 1) // 256 <= arrived - 25, (T, chunk, k)


def test_carry_plan_delay_at_the_reference_chunk():
    """At 32 new frames per pass (the reference's 64-frame windows with 16 frames of context),
    a long stream's emission trails its arrived frames by at least the 24-frame look-ahead and
    at most 40 frames (the 16-row rounding of the level-1 resblock convs adds the rest)."""
    n, lo, hi = pt_b200.carry_plan([1000], 32)
    lag = [min(1000, 32 * (k + 1)) - hi[k, 0] / 256 for k in range(n - 1)]
    assert min(lag) >= 24.0 and max(lag) <= 40.0, lag


def test_carry_plan_rejects_bad_arguments():
    for T, chunk in (([1, 50], 32), ([50], 0), ([], 32)):
        Ta = np.ascontiguousarray(T, np.int64)
        assert pt_b200.lib().pt_b200_carry_plan(len(Ta), Ta.ctypes.data_as(pt_b200._i64p), chunk,
                                                None, None, 0) == -1


def test_carry_plan_rejects_sessions_past_the_32_bit_row_limit():
    """Epilogue offsets are 32-bit: a session whose level-2 tensors would pass 2^31 elements is
    refused by the planner with a message, before any device memory is touched.  The tensors hold
    a bounded window per stream, so the limit is a stream count, not a frame count."""
    T = np.full(2000, 600, np.int64)   # 1.2M frames: accepted, the windows are per stream
    assert pt_b200.lib().pt_b200_carry_plan(len(T), T.ctypes.data_as(pt_b200._i64p), 32, None,
                                            None, 0) == 20   # 19 with frames + the flush
    T = np.full(24000, 600, np.int64)  # ~20M level-2 window rows x 128 channels
    n = pt_b200.lib().pt_b200_carry_plan(len(T), T.ctypes.data_as(pt_b200._i64p), 32, None, None, 0)
    assert n == -1
    assert b"too large" in pt_b200.lib().pt_b200_last_error()


def test_carried_session_memory_is_bounded_per_stream():
    """A session's activations grow with the number of streams, not with their length: each
    stream keeps a fixed window of rows per resolution (pt_b200_carry_device_bytes); only the
    per-pass tables (a few KB per stream and pass) grow with the number of passes."""
    short = pt_b200.carry_device_bytes([400] * 8, 32)
    long = pt_b200.carry_device_bytes([4000] * 8, 32)   # 10 x the frames, 10 x the passes
    assert long < 1.5 * short, (short, long)
    assert pt_b200.carry_device_bytes([400] * 16, 32) > 1.8 * short
    T, _ = pt_b200.config5()
    b = pt_b200.carry_device_bytes(T, 32)
    print(f"\nconfig 5 carried session: {b / 1e9:.2f} GB for {len(T)} streams, {sum(T)} frames")
    assert b < 8e9, b
