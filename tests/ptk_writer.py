"""Writer of the reference's weight container (.ptk) for test fixtures -- a restatement of the
layout in tools/export_v21.py:1-40 and write_ptk (:232-253): header <IIIiq> (magic 0x50544B31,
version 2, n_tensor, reserved 0, data_bytes), n_tensor records <64si4x6qqq> (name, ndim, dims[6],
nelem, offset), zero padding to a 64-byte boundary, 64-byte aligned payloads; names ending in '#h'
carry fp16 payloads (decoder conv weights), everything else fp32."""
import struct

import numpy as np

MAGIC, VERSION = 0x50544B31, 2
HDR = struct.Struct("<IIIiq")
REC = struct.Struct("<64si4x6qqq")


def _a64(n):
    return (n + 63) // 64 * 64


def write_ptk(path, tensors):
    """tensors: [(name, array)]; '#h' names are stored fp16."""
    recs, off, payloads = [], 0, []
    for name, a in tensors:
        a = np.asarray(a)
        h = name.endswith("#h")
        b = (a.astype(np.float16) if h else a.astype(np.float32)).tobytes()
        dims = list(a.shape) + [0] * (6 - a.ndim)
        recs.append(REC.pack(name.encode(), a.ndim, *dims, a.size, off))
        payloads.append(b + b"\0" * (_a64(len(b)) - len(b)))
        off += _a64(len(b))
    hd = HDR.size + REC.size * len(tensors)
    with open(path, "wb") as f:
        f.write(HDR.pack(MAGIC, VERSION, len(tensors), 0, off))
        for r in recs:
            f.write(r)
        f.write(b"\0" * (_a64(hd) - hd))
        for p in payloads:
            f.write(p)


def decoder_tensors(w, extra=()):
    """The decoder records of a DecoderWeights (packed layouts), as the exporter names them
    (spec/v21_layers.json layers 3819-4065): conv weights fp16, biases / conv_post / PQMF fp32.
    The PQMF filter is the final 4 -> 1 conv, packed [1][63][4][4] (output channel 0 real)."""
    t = list(extra)
    t += [("dec.conv_pre.wp#h", w.pre_w), ("dec.conv_pre.b", w.pre_b)]
    for s in range(2):
        t += [(f"dec.ups.{s}.wp#h", w.ups_w[s]), (f"dec.ups.{s}.b", w.ups_b[s])]
        for rb in range(3):
            r = 3 * s + rb
            for j in range(3):
                t += [(f"dec.resblocks.{r}.convs1.{j}.wp#h", w.rb_w1[r][j]),
                      (f"dec.resblocks.{r}.convs1.{j}.b", w.rb_b1[r][j]),
                      (f"dec.resblocks.{r}.convs2.{j}.wp#h", w.rb_w2[r][j]),
                      (f"dec.resblocks.{r}.convs2.{j}.b", w.rb_b2[r][j])]
    t += [("dec.subband_conv_post.wp", w.post_w), ("dec.subband_conv_post.b", w.post_b)]
    pq = np.asarray(w.pqmf, np.float32).reshape(4, 63)
    packed = np.zeros((1, 63, 4, 4), np.float32)
    packed[0, :, :, 0] = pq.T
    t += [("dec.Conv.wp", packed), ("dec.Conv.b", np.zeros(4, np.float32))]
    return t


def fp16_rounded(w):
    """The weights a container stores: conv weights rounded to fp16, the rest fp32."""
    import copy
    r = copy.deepcopy(w)
    f = lambda a: np.asarray(a).astype(np.float16).astype(np.float32)
    r.pre_w = f(w.pre_w)
    r.ups_w = [f(a) for a in w.ups_w]
    r.rb_w1 = [[f(a) for a in row] for row in w.rb_w1]
    r.rb_w2 = [[f(a) for a in row] for row in w.rb_w2]
    return r
