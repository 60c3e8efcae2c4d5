"""The library's reader of the reference weight container (.ptk), on the CPU: a container written
in the exporter's layout (tests/ptk_writer.py) reads back as the fp16-rounded conv weights and the
exact fp32 records, with the PQMF filter unpacked from the final conv; malformed containers are
rejected with a message."""
import os
import struct

import numpy as np
import pytest

import pt_b200
from ptk_writer import decoder_tensors, fp16_rounded, write_ptk


@pytest.fixture(scope="module")
def weights():
    return pt_b200.config3()[0]


def _flat(a):
    return np.asarray(a, np.float32).ravel()


def test_container_roundtrip(tmp_path, weights):
    path = str(tmp_path / "dec.ptk")
    # unrelated records first, as in a full model container
    extra = [("enc.emb.wp#h", np.ones((8, 4), np.float32)), ("dtype.table", np.ones(3, np.float32))]
    write_ptk(path, decoder_tensors(weights, extra))
    got = pt_b200.load_ptk(path)
    ref = fp16_rounded(weights)
    np.testing.assert_array_equal(got.pre_w, _flat(ref.pre_w))
    np.testing.assert_array_equal(got.pre_b, _flat(ref.pre_b))
    for s in range(2):
        np.testing.assert_array_equal(got.ups_w[s], _flat(ref.ups_w[s]))
        np.testing.assert_array_equal(got.ups_b[s], _flat(ref.ups_b[s]))
    for r in range(6):
        for j in range(3):
            np.testing.assert_array_equal(got.rb_w1[r][j], _flat(ref.rb_w1[r][j]))
            np.testing.assert_array_equal(got.rb_b2[r][j], _flat(ref.rb_b2[r][j]))
    np.testing.assert_array_equal(got.post_w, _flat(ref.post_w))
    np.testing.assert_array_equal(got.pqmf.ravel(), _flat(weights.pqmf))


def test_fp16_widening_is_exact(tmp_path, weights):
    """Every fp16 value, subnormals included, widens to the same float numpy gives."""
    path = str(tmp_path / "h.ptk")
    vals = np.arange(65536, dtype=np.uint16).view(np.float16)
    vals = vals[np.isfinite(vals)].astype(np.float32)
    t = decoder_tensors(weights)
    n = np.asarray(weights.pre_w).size
    probe = np.resize(vals, n).reshape(np.asarray(weights.pre_w).shape)
    t[0] = ("dec.conv_pre.wp#h", probe)
    write_ptk(path, t)
    got = pt_b200.load_ptk(path)
    np.testing.assert_array_equal(got.pre_w, probe.ravel())


def test_bad_containers_are_rejected(tmp_path, weights):
    good = str(tmp_path / "g.ptk")
    write_ptk(good, decoder_tensors(weights))
    raw = open(good, "rb").read()
    bad_magic = str(tmp_path / "m.ptk")
    open(bad_magic, "wb").write(b"XXXX" + raw[4:])
    with pytest.raises(pt_b200.PtB200Error, match="magic"):
        pt_b200.load_ptk(bad_magic)
    missing = str(tmp_path / "x.ptk")
    write_ptk(missing, [t for t in decoder_tensors(weights) if not t[0].startswith("dec.ups.1.b")])
    with pytest.raises(pt_b200.PtB200Error, match="dec.ups.1.b"):
        pt_b200.load_ptk(missing)
    wrong = str(tmp_path / "w.ptk")
    write_ptk(wrong, [(n, a[:-1] if n == "dec.conv_pre.b" else a) for n, a in decoder_tensors(weights)])
    with pytest.raises(pt_b200.PtB200Error, match="dec.conv_pre.b"):
        pt_b200.load_ptk(wrong)
    with pytest.raises(pt_b200.PtB200Error, match="cannot open"):
        pt_b200.load_ptk(str(tmp_path / "absent.ptk"))
    trunc = str(tmp_path / "t.ptk")
    open(trunc, "wb").write(raw[:100])
    with pytest.raises(pt_b200.PtB200Error):
        pt_b200.load_ptk(trunc)
