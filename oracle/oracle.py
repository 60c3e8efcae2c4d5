"""ctypes front end of the CPU checker (TEST INFRASTRUCTURE).

Two libraries with the same entry points:

* ``liboracle.so``      -- the restatement in ``oracle/pt_oracle.c`` (always built);
* ``_ref/libptref.so``  -- the reference's own CPU code compiled from its sources by
  ``oracle/Makefile`` (``ref_harness.c``).  It is built in the development container, where the
  reference tree exists, and travels to the GPU box as a prebuilt binary.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_ORACLE = os.path.join(HERE, "liboracle.so")
LIB_REF = os.path.join(HERE, "_ref", "libptref.so")

_f = C.POINTER(C.c_float)
_i64 = C.c_int64


def build() -> None:
    """Compile liboracle.so (and _ref/libptref.so when the reference sources exist)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


class _DecW(C.Structure):
    """C mirror of ``or_dec_weights`` (oracle/pt_oracle.h)."""

    _fields_ = [
        ("pre_w", _f), ("pre_b", _f),
        ("ups_w", _f * 2), ("ups_b", _f * 2),
        ("rb_w1", (_f * 3) * 6), ("rb_b1", (_f * 3) * 6),
        ("rb_w2", (_f * 3) * 6), ("rb_b2", (_f * 3) * 6),
        ("post_w", _f), ("post_b", _f),
        ("pqmf", _f),
    ]


def _p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f)


class CpuDecoder:
    """One of the two CPU implementations, selected by ``kind`` ("oracle" or "reference")."""

    def __init__(self, kind: str = "oracle"):
        path = LIB_ORACLE if kind == "oracle" else LIB_REF
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        self.kind = kind
        self.lib = C.CDLL(path)
        pre = "or_" if kind == "oracle" else "ref_"
        self._conv = getattr(self.lib, pre + "conv")
        self._convT = getattr(self.lib, pre + "convT")
        self._tail = getattr(self.lib, pre + "tail")
        self._decode = getattr(self.lib, pre + "decode")
        self._tail.argtypes = [_f, _i64, _f, _f]
        self._tail.restype = C.c_int
        self._decode.argtypes = [C.POINTER(_DecW), _f, _i64, _f]
        self._decode.restype = C.c_int
        if kind == "oracle":
            self._conv.argtypes = [_f, _i64, _i64, _f, _i64, _i64, C.c_int, C.c_int, C.c_int,
                                   C.c_int, _f, _f, _i64, C.c_int, C.c_int, C.c_float, C.c_float]
            self._conv.restype = None
            self._convT.argtypes = [_f, _i64, _i64, _i64, _f, _i64, C.c_int, C.c_int, C.c_int,
                                    C.c_int, _f, _f, _i64]
            self._convT.restype = None
        else:
            self._conv.argtypes = [_f, _i64, _i64, _f, _i64, _i64, C.c_int, C.c_int, C.c_int,
                                   C.c_int, C.c_int, _f, _f, _i64, C.c_int, C.c_int, C.c_float,
                                   C.c_float]
            self._conv.restype = C.c_int
            self._convT.argtypes = [_f, _i64, _i64, _i64, _f, _i64, C.c_int, C.c_int, C.c_int,
                                    C.c_int, _f, _f, _i64]
            self._convT.restype = C.c_int

    # -- single ops, the reference's calling convention ------------------------------------
    def conv(self, x: np.ndarray, wp: np.ndarray, bias, cout: int, K: int, pad: int, dil: int = 1,
             epi0: int = 0, epi1: int = 0, a0: float = 0.0, a1: float = 0.0) -> np.ndarray:
        """x [B][cin][T] (unpadded) -> Y [B][cout4][Tout] exactly as pt_v21_conv_cpu writes it."""
        B, cin, T = x.shape
        ldx = T + 2 * pad
        xp = np.zeros((B, cin, ldx), np.float32)
        xp[:, :, pad:pad + T] = x
        Tout = T + 2 * pad - (K - 1) * dil
        c4 = (cout + 3) // 4 * 4
        y = np.empty((B, c4, Tout), np.float32)
        bp = _p(bias) if bias is not None else None
        if self.kind == "oracle":
            self._conv(_p(xp), ldx, cin, _p(y), Tout, Tout, cout, K, 1, dil, _p(wp), bp, B,
                       epi0, epi1, a0, a1)
        else:
            self._conv(_p(xp), ldx, cin, _p(y), Tout, Tout, cout, K, 1, pad, dil, _p(wp), bp, B,
                       epi0, epi1, a0, a1)
        return y

    def convT(self, x: np.ndarray, wp: np.ndarray, bias, cout: int, K: int, s: int,
              pad: int) -> np.ndarray:
        B, cin, T = x.shape
        x = np.ascontiguousarray(x, np.float32)
        Lout = (T - 1) * s - 2 * pad + K
        c4 = (cout + 3) // 4 * 4
        y = np.empty((B, c4, Lout), np.float32)
        bp = _p(bias) if bias is not None else None
        self._convT(_p(x), T, cin, T, _p(y), Lout, cout, s, pad, K, _p(wp), bp, B)
        return y

    def tail(self, post: np.ndarray, pqmf: np.ndarray) -> np.ndarray:
        post = np.ascontiguousarray(post, np.float32)
        assert post.shape[0] == 72
        Tp = post.shape[1]
        wav = np.empty(256 * (Tp - 1) // 16, np.float32)
        r = self._tail(_p(post), Tp, _p(np.ascontiguousarray(pqmf, np.float32)), _p(wav))
        if r != 0:
            raise RuntimeError(f"{self.kind} tail failed ({r})")
        return wav

    def decode(self, weights, z: np.ndarray) -> np.ndarray:
        """weights: prime-tts_b200 ``DecoderWeights`` (packed numpy arrays); z [192][T]."""
        z = np.ascontiguousarray(z, np.float32)
        T = z.shape[-1]
        wav = np.empty(256 * T, np.float32)
        dw = self._weights(weights)
        r = self._decode(C.byref(dw), _p(z), T, _p(wav))
        if r != 0:
            raise RuntimeError(f"{self.kind} decode failed ({r})")
        return wav

    def decode_checkpoints(self, weights, z: np.ndarray):
        """The oracle's decode with the output of each of its 40 conv nodes (or_decode_ckpt; the
        layer order and shapes of pt_b200_decoder_checkpoints): (list of 40 arrays, wav)."""
        if self.kind != "oracle":
            raise ValueError("checkpoints come from the restatement (kind='oracle')")
        z = np.ascontiguousarray(z, np.float32)
        T = z.shape[-1]
        ck = [np.empty(s, np.float32) for s in checkpoint_shapes(T)]
        arr = (_f * 40)(*[_p(a) for a in ck])
        fn = self.lib.or_decode_ckpt
        fn.argtypes = [C.POINTER(_DecW), _f, _i64, _f, C.POINTER(_f)]
        fn.restype = C.c_int
        wav = np.empty(256 * T, np.float32)
        dw = self._weights(weights)
        if fn(C.byref(dw), _p(z), T, _p(wav), arr) != 0:
            raise RuntimeError("oracle checkpoint decode failed")
        return ck, wav

    @staticmethod
    def _weights(weights):
        dw = _DecW()
        dw.pre_w, dw.pre_b = _p(weights.pre_w), _p(weights.pre_b)
        for i in range(2):
            dw.ups_w[i], dw.ups_b[i] = _p(weights.ups_w[i]), _p(weights.ups_b[i])
        for r in range(6):
            for j in range(3):
                dw.rb_w1[r][j] = _p(weights.rb_w1[r][j])
                dw.rb_b1[r][j] = _p(weights.rb_b1[r][j])
                dw.rb_w2[r][j] = _p(weights.rb_w2[r][j])
                dw.rb_b2[r][j] = _p(weights.rb_b2[r][j])
        dw.post_w, dw.post_b = _p(weights.post_w), _p(weights.post_b)
        dw.pqmf = _p(weights.pqmf)
        return dw


def checkpoint_shapes(T: int) -> list:
    """Shapes of the 40 per-layer checkpoints of a T-frame decode (conv launch order)."""
    out = [(512, T)]
    for s, (C_, L) in enumerate(((256, 4 * T), (128, 16 * T))):
        out += [(C_, L)] * 19
    out[38] = (128, 16 * T + 1)
    out.append((72, 16 * T + 1))
    return out


def checkpoint_names() -> list:
    """Names of the 40 checkpoints (graph layer names)."""
    names = ["conv_pre"]
    for s in range(2):
        names.append(f"ups.{s}")
        for rb in range(3):
            for j in range(3):
                names += [f"rb{3 * s + rb}.convs1.{j}", f"rb{3 * s + rb}.convs2.{j}"]
    names.append("conv_post")
    return names


def overlap_save_windows(T: int, win: int, ctx: int, hop: int = 256) -> list:
    """The reference's overlap-save stitch loop (runtime/v21/src/main_v21.c:342-364) for one
    utterance of T frames: [(a, win_eff, lo, hi)] -- window frames [a, a+win_eff), whose output
    samples [lo, hi) are appended to the stitched waveform in order."""
    out = []
    step = win - 2 * ctx
    if step < 1:
        step = 1
    a = 0
    while True:
        win_eff = win
        if a + win_eff > T:
            win_eff = T - a
        first, last = a == 0, a + win_eff >= T
        n = win_eff * hop
        lo = 0 if first else ctx * hop
        hi = n if last else (win_eff - ctx) * hop
        if hi > n:
            hi = n
        if hi > lo:
            out.append((a, win_eff, lo, hi))
        if last:
            break
        a += step
    return out


def stitch(decode, z: np.ndarray, windows: list) -> np.ndarray:
    """Decode each window's frames with ``decode(z_slice) -> wav`` and concatenate the kept
    samples, as the reference driver does with pt_v21_stream_chunk (main_v21.c:346-360)."""
    parts = []
    for a, we, lo, hi in windows:
        wav = decode(np.ascontiguousarray(z[:, a:a + we]))
        parts.append(wav[lo:hi])
    return np.concatenate(parts)


def metrics(est: np.ndarray, ref: np.ndarray) -> dict:
    """The reference's parity metrics (tests/v21_reference.py:430-447): max|a-b|/max|b| and
    SNDR = 10 log10(sum ref^2 / sum (est-ref)^2)."""
    est = np.asarray(est, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    err = est - ref
    den = float(np.max(np.abs(ref))) if ref.size else 0.0
    max_rel = float(np.max(np.abs(err))) / den if den > 0 else float(np.max(np.abs(err)))
    e2 = float(np.sum(err * err))
    sndr = float("inf") if e2 == 0 else 10.0 * np.log10(float(np.sum(ref * ref)) / e2)
    return {"max_rel": max_rel, "sndr_db": sndr, "max_abs": float(np.max(np.abs(err)))}
