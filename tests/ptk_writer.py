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


def _tail_tables():
    """Hann window, window-sum kernel (graph constants 4009 / 3617, from the oracle, which holds
    the values spec/v21_layers.json records) and the [9,16] cos / sin tables of the irfft bases
    (graph constants 3607 / 3612, not recorded by the spec: round_fp32(cos / sin(2 pi k n / 16)))."""
    import ctypes as C
    import oracle
    lib = C.CDLL(oracle.LIB_ORACLE)
    win, win2 = np.zeros(16, np.float32), np.zeros(16, np.float32)
    f = C.POINTER(C.c_float)
    lib.or_tail_constants(win.ctypes.data_as(f), win2.ctypes.data_as(f), None, None)
    k = np.arange(9, dtype=np.float64)[:, None]
    n = np.arange(16, dtype=np.float64)[None, :]
    ang = 2.0 * np.pi * k * n / 16.0
    return win, win2, np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def decoder_range_tensors(w):
    """Every container record the reference interpreter reads when it runs the decoder's node
    range (conv_pre .. the PQMF conv) and the constant-only nodes that build its irfft bases and
    zero-stuff kernel: the decoder records of `decoder_tensors`, the packed kernels of the three
    tail ConvTranspose nodes, the graph constants (values as spec/v21_layers.json records them;
    the PQMF filter is `w.pqmf`), and the `dtype.table` record (payload item size of every record,
    record order) that pt_v21_open requires (runtime/v21/src/pt_v21_host.c:1124-1147)."""
    import sys, os
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "prime-tts_b200"))
    import pt_b200
    win, win2, cos9, sin9 = _tail_tables()
    eye = np.zeros((16, 1, 16), np.float32)
    for i in range(16):
        eye[i, 0, i] = 1.0                        # overlap-add kernel, ONNX [Cin][Cout][K]
    stuff = np.zeros((4, 4, 4), np.float32)
    for i in range(4):
        stuff[i, i, 0] = 4.0                      # x4 zero-stuff with gain 4
    t = decoder_tensors(w)
    t += [("dec.ConvTranspose.wp", pt_b200.pack_convT(eye, 4)), ("dec.ConvTranspose.b", np.zeros(1, np.float32)),
          ("dec.ConvTranspose_1.wp", pt_b200.pack_convT(win2.reshape(1, 1, 16), 4)),
          ("dec.ConvTranspose_1.b", np.zeros(1, np.float32)),
          ("dec.ConvTranspose_2.wp", pt_b200.pack_convT(stuff, 4)),
          ("dec.ConvTranspose_2.b", np.zeros(4, np.float32))]
    sc = lambda v: np.array(v, np.float32)
    t += [("const.3530", np.full((9, 1), 2.0, np.float32)), ("const.3531", sc(1.0)),
          ("const.3607", cos9), ("const.3609", sc(16.0)), ("const.3612", sin9),
          ("const.3614", sc(16.0)), ("const.3616", eye), ("const.3617", win2.reshape(1, 1, 16)),
          ("const.3618", np.zeros((4, 4, 4), np.float32)), ("const.3867", sc(3.0)),
          ("const.3916", sc(3.0)), ("const.3970", sc(np.float32(np.pi))),
          ("const.4009", win.reshape(1, 16, 1)), ("const.4020", sc(1e-9)),
          ("const.4044", sc(4.0)), ("const.4062", sc(0.0)),
          ("const.4064", np.asarray(w.pqmf, np.float32).reshape(1, 4, 63))]
    sizes = [2.0 if name.endswith("#h") else 4.0 for name, _ in t] + [4.0]
    t.append(("dtype.table", np.array(sizes, np.float32)))
    return t
