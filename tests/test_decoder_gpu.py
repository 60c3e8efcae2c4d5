"""Parity of the iSTFT+PQMF tail kernel and of the batched device-resident decoder against the
CPU oracle (which is bit-exact to the reference's CPU path, tests/test_oracle.py).

Gates (tests/v21_reference.py:430-447, 502-505): SNDR >= 60 dB per waveform; the tail alone,
whose arithmetic stays within a microunit of the reference's, is held much tighter (max_rel
1e-5, 100 dB).
"""
import numpy as np
import pytest

import oracle
import pt_b200

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = pt_b200.Context(0)
    yield c
    c.close()


@pytest.fixture(scope="module")
def orc():
    return oracle.CpuDecoder("oracle")


@pytest.fixture(scope="module")
def cfg3():
    return pt_b200.config3(seed=2, T=226)


@pytest.fixture(scope="module")
def dec(cfg3):
    d = pt_b200.Decoder(cfg3[0], device=0)
    yield d
    d.close()


@pytest.mark.parametrize("Tp", [2, 17, 49, 129, 161, 1000, 3617])
def test_tail_matches_oracle(ctx, orc, Tp):
    rng = np.random.default_rng(Tp)
    post = (0.5 * rng.standard_normal((72, Tp))).astype(np.float32)
    pq = pt_b200.pqmf_synthesis_filter()
    ref = orc.tail(post, pq)
    y = ctx.istft_pqmf(post, pq)
    m = oracle.metrics(y, ref)
    # the kernel uses the hardware exp / sincos approximations and fp32 fused multiply-adds where
    # the reference rounds every step (measured: max_rel <= 4.3e-7, >= 132 dB at these sizes);
    # the gate leaves a 20x margin on the relative error and 30 dB on the SNDR
    assert m["max_rel"] <= 1e-5 and m["sndr_db"] >= 100, m


def test_config3_decoder(dec, orc, cfg3):
    w, z = cfg3
    ref = orc.decode(w, z)
    (y,) = dec.decode([z])
    assert y.shape == ref.shape == (256 * 226,)
    m = oracle.metrics(y, ref)
    print("config 3 decoder vs oracle:", m)
    assert m["sndr_db"] >= 60.0, m


def test_ragged_batch_each_request_matches_oracle(dec, orc, cfg3):
    w = cfg3[0]
    rng = np.random.default_rng(11)
    Ts = [2, 3, 17, 64, 129]
    zs = [rng.standard_normal((192, t)).astype(np.float32) for t in Ts]
    outs = dec.decode(zs)
    for z, y in zip(zs, outs):
        m = oracle.metrics(y, orc.decode(w, z))
        assert m["sndr_db"] >= 60.0, (z.shape, m)


def test_batch_invariance_bitwise(dec):
    """A request decodes to the same bits alone or anywhere inside a ragged batch."""
    rng = np.random.default_rng(12)
    Ts = [50, 7, 333, 128, 129, 2]
    zs = [rng.standard_normal((192, t)).astype(np.float32) for t in Ts]
    together = dec.decode(zs)
    for i in (0, 2, 5):
        (alone,) = dec.decode([zs[i]])
        assert np.array_equal(alone, together[i])
    again = dec.decode(zs[::-1])[::-1]
    for a, b in zip(again, together):
        assert np.array_equal(a, b)


def test_config4_batch_properties(dec, orc, cfg3):
    """The benchmark workload (64 requests, T ~ U{50..600}, seed 3): shapes, finiteness, the two
    shortest requests against the oracle, and two more against their solo decode."""
    T, zs = pt_b200.config4()
    outs = dec.decode(zs)
    assert [o.size for o in outs] == [256 * t for t in T]
    assert all(np.isfinite(o).all() for o in outs)
    order = np.argsort(T)
    for i in order[:2]:
        m = oracle.metrics(outs[i], orc.decode(cfg3[0], zs[i]))
        assert m["sndr_db"] >= 60.0, (T[i], m)
    for i in order[-2:]:
        (alone,) = dec.decode([zs[i]])
        assert np.array_equal(alone, outs[i])


def test_decode_single_request_via_context(ctx, dec, cfg3):
    """pt_v21_decode: the one-request driver shape on an interpreter context."""
    import ctypes as C
    z = cfg3[1][:, :40].copy()
    wav = np.empty(256 * 40, np.float32)
    f = C.POINTER(C.c_float)
    rc = pt_b200.lib().pt_v21_decode(ctx.ptr, dec.h, z.ctypes.data_as(f), 40, wav.ctypes.data_as(f))
    assert rc == 0
    (ref,) = dec.decode([z])
    assert np.array_equal(wav, ref)


def test_graph_replay_is_bitwise_and_counts_launches(dec):
    """The decode is captured as a CUDA graph on its second identical call and replayed after:
    every call returns the same bits, and a replay reports the same kernel count as an eager
    decode."""
    import torch
    T, zs = pt_b200.config4(seed=5, n=6, lo=30, hi=90)
    Ta = np.array(T, np.int64)
    dev = torch.device("cuda", 0)
    z = torch.from_numpy(np.concatenate([a.ravel() for a in zs])).to(dev)
    s = torch.cuda.Stream(device=dev)
    outs, counts = [], []
    wav = torch.empty(int(256 * Ta.sum()), device=dev)
    for _ in range(4):   # eager, capture + replay, replay, replay
        wav.fill_(float("nan"))
        pt_b200.kernel_launches(reset=True)
        dec.decode_device(Ta, z.data_ptr(), wav.data_ptr(), s.cuda_stream)
        dec.sync(s.cuda_stream)
        counts.append(pt_b200.kernel_launches())
        outs.append(wav.cpu().numpy().copy())
    for o in outs[1:]:
        np.testing.assert_array_equal(o, outs[0])
    assert np.isfinite(outs[0]).all()
    # the first decode of a new layout also clears the gap rows another layout may have used
    # (one more kernel); the replays launch exactly what an eager decode of the same plan does
    assert counts[1] > 0 and all(c == counts[1] for c in counts[1:]), counts
    assert counts[0] in (counts[1], counts[1] + 1), counts
    ref = dec.decode(zs)   # host entry point, separate buffers: its own eager decode
    np.testing.assert_array_equal(np.concatenate(ref), outs[0])


def test_decoder_from_container(tmp_path, orc):
    """A decoder created from a reference weight container (.ptk, fp16 conv weights) matches the
    oracle run on the same fp16-rounded weights; the one-call C entry gives the same bits."""
    import ctypes as C
    from ptk_writer import decoder_tensors, fp16_rounded, write_ptk
    w, z = pt_b200.config3(seed=2, T=120)
    path = str(tmp_path / "dec.ptk")
    write_ptk(path, decoder_tensors(w))
    d = pt_b200.Decoder.from_container(path)
    got = d.decode([z])[0]
    d.close()
    m = oracle.metrics(got, orc.decode(fp16_rounded(w), z))
    assert m["sndr_db"] >= 60.0, m
    h = pt_b200.lib().pt_b200_decoder_create_from_ptk(0, path.encode())
    assert h
    try:
        T = np.array([z.shape[1]], np.int64)
        zc = np.ascontiguousarray(z, np.float32)
        wav = np.empty(256 * z.shape[1], np.float32)
        rc = pt_b200.lib().pt_b200_decode_batch(h, None, 1, T.ctypes.data_as(C.POINTER(C.c_int64)),
                                                zc.ctypes.data, wav.ctypes.data)
        assert rc == 0
        np.testing.assert_array_equal(wav, got)
    finally:
        pt_b200.lib().pt_b200_decoder_destroy(h)


def test_pipelined_host_decodes_match_the_synchronous_ones(dec):
    """pt_b200_decode_batch_async: calls queued back to back (two staging slots in turn, each
    captured and replayed as its own graph, a bigger batch growing the slots midway) return the
    same bits as one synchronous host decode per batch, in every output buffer."""
    import torch
    batches = [pt_b200.config4(seed=s, n=5, lo=20, hi=70) for s in (7, 8)]
    batches.append(pt_b200.config4(seed=9, n=7, lo=60, hi=140))   # grows the staging slots
    calls = [0, 1, 0, 1, 0, 2, 2, 1, 2]
    zh, wh, refs = [], [], []
    for T, zs in batches:
        zh.append(torch.from_numpy(np.concatenate([a.ravel() for a in zs])).pin_memory())
        refs.append(np.concatenate(dec.decode(zs)))
    for b in calls:
        w = torch.full((int(256 * sum(batches[b][0])),), float("nan")).pin_memory()
        wh.append(w)
        dec.decode_async(np.array(batches[b][0], np.int64), zh[b].data_ptr(), w.data_ptr())
    dec.decode_async_wait()
    for b, w in zip(calls, wh):
        np.testing.assert_array_equal(w.numpy(), refs[b])


def test_switching_between_batches_reuses_plans_bitwise(dec):
    """Device decodes of different ragged batches in turn -- switching back to a recent batch's
    layout, replaying its captured graph, evicting the oldest layout when more than the kept
    number of layouts are in use -- give every batch the same bits as its first decode."""
    import torch
    dev = torch.device("cuda", 0)
    s = torch.cuda.Stream(device=dev)
    batches = [pt_b200.config4(seed=40 + k, n=3 + k, lo=20, hi=80) for k in range(6)]
    bufs = []
    for T, zs in batches:
        z = torch.from_numpy(np.concatenate([a.ravel() for a in zs])).to(dev)
        w = torch.empty(int(256 * sum(T)), device=dev)
        bufs.append((np.array(T, np.int64), z, w))
    first = {}
    order = [0, 1, 0, 1, 0, 1, 2, 3, 4, 5, 0, 2, 5, 5, 5, 1]
    for b in order:
        T, z, w = bufs[b]
        w.fill_(float("nan"))
        dec.decode_device(T, z.data_ptr(), w.data_ptr(), s.cuda_stream)
        dec.sync(s.cuda_stream)
        got = w.cpu().numpy()
        assert np.isfinite(got).all(), b
        if b in first:
            np.testing.assert_array_equal(got, first[b])
        else:
            first[b] = got
            ref = np.concatenate(dec.decode(batches[b][1]))
            np.testing.assert_array_equal(got, ref)
