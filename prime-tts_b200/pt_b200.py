"""Host-side mirror of the PrimeTTS v2.1 decoder hot path on B200 (ctypes over libpt_b200.so).

The compute lives in ``libpt_b200.so`` (C ABI declared in ``include/pt_b200.h``): the
reference's ``pt_v21_conv`` / ``pt_v21_convT`` / ``pt_v21_matmul`` entry points with the same
argument meaning and ``pt_ctx`` protocol (runtime/v21/src/pt_v21.h:208-259), plus the batched
device-resident decoder.  This module only marshals arguments; it has no compute path of its own
and raises when the library is missing or a call fails.

Also here: the reference container's packed weight layouts (tools/export_v21.py:88-121), the
4-band PQMF synthesis filter, and the seeded synthetic workloads of the benchmark configs.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass, field

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpt_b200.so")

_f = C.POINTER(C.c_float)
_i64 = C.c_int64
_i64p = C.POINTER(C.c_int64)


def build(verbose: bool = False) -> None:
    """Compile libpt_b200.so in place (nvcc, sm_100a)."""
    subprocess.run(["make", "-C", HERE] + ([] if verbose else ["-s"]), check=True)


# --------------------------------------------------------------------------------------------
# pt_ctx: layout of runtime/v21/src/pt_v21.h:79-162 (include/pt_b200.h mirrors it)
class PtTv(C.Structure):
    _fields_ = [("dt", C.c_int), ("ndim", C.c_int), ("d", C.c_int64 * 6), ("n", C.c_int64),
                ("p", C.c_void_p), ("dev", C.c_int), ("dev_res", C.c_int), ("dev_p", C.c_void_p),
                ("alive", C.c_int), ("base", C.c_void_p), ("view", C.c_int)]


class PtCtx(C.Structure):
    _fields_ = [
        ("use_cuda", C.c_int), ("map", C.c_void_p), ("maplen", C.c_size_t), ("base", C.c_char_p),
        ("n_tensor", C.c_uint32), ("cont_names", C.c_void_p), ("cont_f32", C.c_void_p),
        ("cont_isz", C.c_void_p), ("cont_n", C.c_void_p), ("cont_ndim", C.c_void_p),
        ("cont_path", C.c_char_p), ("cont_shared", C.c_void_p), ("cont_dims", C.c_void_p),
        ("n_cont", C.c_int), ("V", C.c_void_p), ("wav", C.c_void_p), ("wav_n", C.c_int64),
        ("ck_n", C.c_int), ("ck_ids", C.c_void_p), ("ck_dir", C.c_char * 512),
        ("dev_mode", C.c_int),
        ("n_conv", C.c_long), ("n_convT", C.c_long), ("n_matmul", C.c_long),
        ("n_alloc_fail", C.c_long),
        ("t_conv", C.c_double), ("t_convT", C.c_double), ("t_matmul", C.c_double),
        ("t_total", C.c_double),
        ("g_alloc_ms", C.c_double), ("g_copy_ms", C.c_double), ("g_kernel_ms", C.c_double),
        ("g_free_ms", C.c_double), ("g_calls", C.c_long), ("prof", C.c_int),
        ("prof_node_on", C.c_int), ("host_bytes_live", C.c_long), ("host_bytes_peak", C.c_long),
        ("pool", C.c_void_p * 64), ("pool_bytes", C.c_long), ("pool_cap", C.c_long),
        ("host_alloc_count", C.c_long), ("dev_bytes_weights", C.c_double),
        ("dev_bytes_arena", C.c_double), ("dev_bytes_stray", C.c_double),
        ("dev_bytes_res", C.c_double), ("devres_oom", C.c_int),
        ("arena_alloc_bytes", C.c_size_t), ("skip", C.c_void_p), ("fuse", C.c_int),
        ("run_from", C.c_int), ("run_to", C.c_int), ("stream_inject_id", C.c_int),
        ("stream_inject", C.c_void_p), ("stream_seeds", C.c_void_p), ("stream_nseeds", C.c_int),
        ("stream_state", C.c_void_p), ("prof_node", C.c_void_p),
        ("t_ekind", C.c_double * 96), ("n_ekind", C.c_long * 96),
        ("g_weights", C.c_void_p), ("g_arena", C.c_void_p), ("g_stream", C.c_void_p),
        ("g_arena_bytes", C.c_size_t), ("g_arena_used", C.c_size_t),
        ("conv_pad_in", C.c_int64), ("conv_in_dev", C.c_void_p), ("conv_keep", C.c_int),
        ("conv_keep_res", C.c_int), ("devadd_used", C.c_int), ("dev_live", C.c_int),
        ("conv_out_dev", C.c_void_p), ("chain_mark", C.c_void_p), ("devres", C.c_void_p),
    ]


class DecWeightsC(C.Structure):
    """``pt_b200_dec_weights`` (include/pt_b200.h)."""

    _fields_ = [
        ("pre_w", _f), ("pre_b", _f), ("ups_w", _f * 2), ("ups_b", _f * 2),
        ("rb_w1", (_f * 3) * 6), ("rb_b1", (_f * 3) * 6),
        ("rb_w2", (_f * 3) * 6), ("rb_b2", (_f * 3) * 6),
        ("post_w", _f), ("post_b", _f), ("pqmf", _f),
    ]


# exported C symbols and their ctypes signatures
class WindowC(C.Structure):
    """pt_b200_window: one streaming window (a latent column slice and the samples it keeps)."""
    _fields_ = [("frames", C.c_int64), ("z_off", C.c_int64), ("z_ld", C.c_int64),
                ("keep_lo", C.c_int64), ("keep_hi", C.c_int64), ("dst", C.c_int64)]


_SIGS = {
    "pt_v21_cuda_prewarm": ([], C.c_int),
    "pt_v21_cuda_init": ([C.c_void_p, C.c_int], C.c_int),
    "pt_v21_cuda_init_dev": ([C.c_void_p, C.c_int, C.c_int], C.c_int),
    "pt_v21_cuda_shutdown": ([C.c_void_p], None),
    "pt_v21_conv": ([C.c_void_p, _f, _i64, _i64, _f, _i64, _i64, C.c_int, C.c_int, C.c_int,
                     C.c_int, C.c_int, _f, _f, _i64, C.c_int, C.c_int, C.c_int, C.c_int,
                     C.c_float, C.c_float], C.c_int),
    "pt_v21_convT": ([C.c_void_p, _f, _i64, _i64, _i64, _f, _i64, C.c_int, C.c_int, C.c_int,
                      C.c_int, _f, _f, _i64, C.c_int, C.c_int], C.c_int),
    "pt_v21_convT_epi": ([C.c_void_p, _f, _i64, _i64, _i64, _f, _i64, C.c_int, C.c_int, C.c_int,
                          C.c_int, _f, _f, _i64, C.c_int, C.c_int, C.c_int, C.c_float], C.c_int),
    "pt_v21_matmul": ([C.c_void_p, _f, _i64, _i64, _i64, _f, _i64, _i64, _f, _i64], C.c_int),
    "pt_v21_conv_pads_in_kernel": ([C.c_void_p], C.c_int),
    "pt_v21_devadd_run": ([C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, _i64, C.c_int,
                           C.c_float], C.c_int),
    "pt_v21_devleaky_run": ([C.c_void_p, C.c_void_p, C.c_void_p, _i64, C.c_float], C.c_int),
    "pt_v21_dev_upload": ([C.c_void_p, C.c_void_p, _i64], C.c_void_p),
    "pt_v21_dev_sync_host": ([C.c_void_p, C.c_void_p, C.c_void_p, _i64], None),
    "pt_v21_dev_alloc": ([C.c_void_p, C.c_size_t], C.c_void_p),
    "pt_v21_dev_free": ([C.c_void_p, C.c_void_p], None),
    "pt_v21_dev_reclaim": ([C.c_void_p], None),
    "pt_v21_cuda_active": ([C.c_int], None),
    "pt_v21_cuda_weights_mib": ([C.c_void_p], C.c_double),
    "pt_v21_cuda_keepwarm": ([C.c_int], C.c_int),
    "pt_v21_gpu_cur_freq": ([], C.c_long),
    "pt_v21_gpu_max_freq": ([], C.c_long),
    "pt_v21_istft_pqmf": ([C.c_void_p, _f, _i64, _f, _f], C.c_int),
    "pt_v21_decode": ([C.c_void_p, C.c_void_p, _f, _i64, _f], C.c_int),
    "pt_b200_decoder_create": ([C.c_int, C.POINTER(DecWeightsC)], C.c_void_p),
    "pt_b200_decoder_destroy": ([C.c_void_p], None),
    "pt_b200_decode_batch": ([C.c_void_p, C.c_void_p, C.c_int, _i64p, C.c_void_p, C.c_void_p],
                             C.c_int),
    "pt_b200_decode_batch_device": ([C.c_void_p, C.c_void_p, C.c_int, _i64p, C.c_void_p,
                                     C.c_void_p], C.c_int),
    "pt_b200_decoder_sync": ([C.c_void_p, C.c_void_p], C.c_int),
    "pt_b200_decode_batch_async": ([C.c_void_p, C.c_int, _i64p, C.c_void_p, C.c_void_p], C.c_int),
    "pt_b200_decode_async_wait": ([C.c_void_p], C.c_int),
    "pt_b200_decode_async_streams": ([C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                      C.POINTER(C.c_void_p)], C.c_int),
    "pt_b200_decode_windows": ([C.c_void_p, C.c_void_p, C.c_int, C.POINTER(WindowC), C.c_void_p,
                                C.c_void_p], C.c_int),
    "pt_b200_stream_plan": ([C.c_int, _i64p, C.c_int, C.c_int, C.c_int, C.POINTER(WindowC),
                             _i64], _i64),
    "pt_b200_stream_decode": ([C.c_void_p, C.c_void_p, C.c_int, _i64p, C.c_void_p, C.c_int,
                               C.c_int, C.c_int, _i64, C.c_void_p], C.c_int),
    "pt_b200_carry_open": ([C.c_void_p, C.c_int, _i64p, C.c_int], C.c_void_p),
    "pt_b200_carry_passes": ([C.c_void_p], C.c_int),
    "pt_b200_carry_bytes": ([C.c_void_p], _i64),
    "pt_b200_carry_device_bytes": ([C.c_int, _i64p, C.c_int], _i64),
    "pt_b200_carry_run": ([C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p], C.c_int),
    "pt_b200_carry_reset": ([C.c_void_p], C.c_int),
    "pt_b200_carry_close": ([C.c_void_p], None),
    "pt_b200_stream_decode_carry": ([C.c_void_p, C.c_void_p, C.c_int, _i64p, C.c_void_p, C.c_int,
                                     C.c_void_p], C.c_int),
    "pt_b200_carry_plan": ([C.c_int, _i64p, C.c_int, _i64p, _i64p, _i64], _i64),
    "pt_b200_decoder_profile": ([C.c_void_p, C.c_int], C.c_int),
    "pt_b200_decoder_launch_times": ([C.c_void_p, C.c_int, C.POINTER(C.c_double),
                                      C.POINTER(C.c_double), C.POINTER(C.c_double),
                                      C.POINTER(C.c_int)], C.c_int),
    "pt_b200_decoder_checkpoints": ([C.c_void_p, _f, _i64, C.POINTER(_f), _f], C.c_int),
    "pt_b200_conv_noalloc": ([C.c_int, C.c_void_p, C.c_void_p, _i64, _i64, _i64, C.c_void_p,
                              C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                              C.c_int, C.c_float], C.c_int),
    "pt_b200_ptk_open": ([C.c_char_p], C.c_void_p),
    "pt_b200_ptk_decoder_weights": ([C.c_void_p, C.POINTER(DecWeightsC)], C.c_int),
    "pt_b200_ptk_close": ([C.c_void_p], None),
    "pt_b200_decoder_create_from_ptk": ([C.c_int, C.c_char_p], C.c_void_p),
    "pt_b200_mma_rate": ([C.c_int, C.c_int, C.POINTER(C.c_double), C.POINTER(C.c_double),
                          C.POINTER(C.c_double)], C.c_int),
    "pt_b200_last_error": ([], C.c_char_p),
    "pt_b200_kernel_launches": ([C.c_int], C.c_long),
}

_lib = None


def lib():
    """The loaded libpt_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(f"{LIB_PATH} is missing: run `make -C {HERE}` (no CPU path)")
        L = C.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


class PtB200Error(RuntimeError):
    pass


def _check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().pt_b200_last_error()
        raise PtB200Error(f"{what} failed: {msg.decode() if msg else rc}")


def _p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous, (a.dtype, a.flags)
    return a.ctypes.data_as(_f)


def mma_rate(device: int = 0, iters: int = 20000) -> dict:
    """The tensor core's kind::tf32 rate measured live (pt_b200_mma_rate): FLOP per SM clock,
    aggregate TFLOP/s and the SM clock (MHz) of the run."""
    f, t, m = C.c_double(), C.c_double(), C.c_double()
    _check(lib().pt_b200_mma_rate(device, iters, C.byref(f), C.byref(t), C.byref(m)),
           "pt_b200_mma_rate")
    return {"flop_per_clk_sm": f.value, "tflops": t.value, "sm_mhz": m.value}


def kernel_launches(reset: bool = False) -> int:
    return int(lib().pt_b200_kernel_launches(1 if reset else 0))


# --------------------------------------------------------------------------------------------
class Context:
    """One interpreter context (``pt_ctx``) bound to a GPU: the reference's per-request state."""

    def __init__(self, device: int = 0, verbose: bool = False):
        self.ctx = PtCtx()
        self.ctx.conv_pad_in = -1
        _check(lib().pt_v21_cuda_init_dev(C.byref(self.ctx), device, int(verbose)),
               "pt_v21_cuda_init_dev")
        self.device = device

    @property
    def ptr(self):
        return C.byref(self.ctx)

    def close(self) -> None:
        if self.ctx.use_cuda:
            lib().pt_v21_cuda_shutdown(C.byref(self.ctx))

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # -- the reference's op entry points ---------------------------------------------------
    def conv(self, x: np.ndarray, wp: np.ndarray, bias, cout: int, K: int, pad: int, dil: int = 1,
             epi0: int = 0, epi1: int = 0, a0: float = 0.0, a1: float = 0.0, wtab: int = -1,
             btab: int = -1, padded_input: bool = False) -> np.ndarray:
        """pt_v21_conv on x [B][cin][T].  padded_input=False hands the rows over unpadded
        (conv_pad_in = pad, the interpreter's CUDA path); True pads them on the host first."""
        x = np.ascontiguousarray(x, np.float32)
        B, cin, T = x.shape
        Tout = T + 2 * pad - (K - 1) * dil
        if padded_input:
            xp = np.zeros((B, cin, T + 2 * pad), np.float32)
            xp[:, :, pad:pad + T] = x
            x, ldx = xp, T + 2 * pad
            self.ctx.conv_pad_in = -1
        else:
            ldx = T
            self.ctx.conv_pad_in = pad
        c4 = (cout + 3) // 4 * 4
        y = np.empty((B, c4, Tout), np.float32)
        bp = _p(bias) if bias is not None else None
        rc = lib().pt_v21_conv(self.ptr, _p(x), ldx, cin, _p(y), Tout, Tout, cout, K, 1, pad, dil,
                               _p(wp), bp, B, wtab, btab, epi0, epi1, a0, a1)
        _check(rc, "pt_v21_conv")
        return y

    def convT(self, x: np.ndarray, wp: np.ndarray, bias, cout: int, K: int, s: int, pad: int,
              epi0: int = 0, a0: float = 0.0, wtab: int = -1, btab: int = -1) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        B, cin, T = x.shape
        Lout = (T - 1) * s - 2 * pad + K
        c4 = (cout + 3) // 4 * 4
        y = np.empty((B, c4, Lout), np.float32)
        bp = _p(bias) if bias is not None else None
        if epi0:
            rc = lib().pt_v21_convT_epi(self.ptr, _p(x), T, cin, T, _p(y), Lout, cout, s, pad, K,
                                        _p(wp), bp, B, wtab, btab, epi0, a0)
        else:
            rc = lib().pt_v21_convT(self.ptr, _p(x), T, cin, T, _p(y), Lout, cout, s, pad, K,
                                    _p(wp), bp, B, wtab, btab)
        _check(rc, "pt_v21_convT")
        return y

    def matmul(self, A: np.ndarray, B: np.ndarray) -> np.ndarray:
        A = np.ascontiguousarray(A, np.float32)
        B = np.ascontiguousarray(B, np.float32)
        m, k = A.shape
        k2, nn = B.shape
        assert k == k2
        Cm = np.empty((m, nn), np.float32)
        _check(lib().pt_v21_matmul(self.ptr, _p(A), m, k, k, _p(B), nn, nn, _p(Cm), nn),
               "pt_v21_matmul")
        return Cm

    def istft_pqmf(self, post: np.ndarray, pqmf: np.ndarray) -> np.ndarray:
        post = np.ascontiguousarray(post, np.float32)
        Tp = post.shape[-1]
        wav = np.empty(16 * (Tp - 1), np.float32)
        _check(lib().pt_v21_istft_pqmf(self.ptr, _p(post), Tp,
                                       _p(np.ascontiguousarray(pqmf, np.float32)), _p(wav)),
               "pt_v21_istft_pqmf")
        return wav


# --------------------------------------------------------------------------------------------
# packed layouts (tools/export_v21.py:88-121)
def r4(n: int) -> int:
    return (n + 3) // 4 * 4


def pack_conv(W: np.ndarray) -> np.ndarray:
    """ONNX conv weight [Cout][Cin][K] -> packed [Cout4/4][K][Cin][4]."""
    Cout, Cin, K = W.shape
    c4 = r4(Cout)
    Wp = np.zeros((c4, Cin, K), np.float32)
    Wp[:Cout] = W
    return np.ascontiguousarray(Wp.reshape(c4 // 4, 4, Cin, K).transpose(0, 3, 2, 1))


def pack_convT(W: np.ndarray, s: int) -> np.ndarray:
    """ONNX ConvTranspose weight [Cin][Cout][K] -> packed [s*Cout4/4][ntap][Cin][4]; phase r /
    channel c / tap j holds ONNX tap k = r + j*s."""
    Cin, Cout, K = W.shape
    c4, nt = r4(Cout), (K + s - 1) // s
    Wph = np.zeros((s * c4, Cin, nt), np.float32)
    for r in range(s):
        for j in range(nt):
            k = r + j * s
            if k < K:
                Wph[r * c4:r * c4 + Cout, :, j] = W[:, :, k].T
    return pack_conv(Wph)


def pqmf_synthesis_filter(taps: int = 62, cutoff: float = 0.142, beta: float = 9.0,
                          bands: int = 4) -> np.ndarray:
    """[1][bands][taps+1] cosine-modulated synthesis filters of a near-perfect-reconstruction
    pseudo-QMF bank (Nguyen 1994): a Kaiser-windowed ideal low-pass prototype, modulated by
    cos((2k+1) pi/(2K) (n - taps/2) - (-1)^k pi/4).  The trained model's filter is not in the
    reference tree, so this published design stands in for it (oracle and GPU use the same)."""
    n = np.arange(taps + 1, dtype=np.float64) - 0.5 * taps
    with np.errstate(invalid="ignore", divide="ignore"):
        proto = np.sin(np.pi * cutoff * n) / (np.pi * n)
    proto[taps // 2] = cutoff
    proto = proto * np.kaiser(taps + 1, beta)
    g = np.stack([2.0 * proto * np.cos((2 * k + 1) * (np.pi / (2 * bands)) * n
                                       - (-1) ** k * np.pi / 4) for k in range(bands)])
    return np.ascontiguousarray(g[None].astype(np.float32))


@dataclass
class DecoderWeights:
    """Decoder weights in the container's packed layouts (resblock r: kernel (3,7,11)[r%3])."""

    pre_w: np.ndarray
    pre_b: np.ndarray
    ups_w: list
    ups_b: list
    rb_w1: list
    rb_b1: list
    rb_w2: list
    rb_b2: list
    post_w: np.ndarray
    post_b: np.ndarray
    pqmf: np.ndarray
    _keep: list = field(default_factory=list, repr=False)

    def as_c(self) -> DecWeightsC:
        dw = DecWeightsC()
        dw.pre_w, dw.pre_b = _p(self.pre_w), _p(self.pre_b)
        for i in range(2):
            dw.ups_w[i], dw.ups_b[i] = _p(self.ups_w[i]), _p(self.ups_b[i])
        for r in range(6):
            for j in range(3):
                dw.rb_w1[r][j], dw.rb_b1[r][j] = _p(self.rb_w1[r][j]), _p(self.rb_b1[r][j])
                dw.rb_w2[r][j], dw.rb_b2[r][j] = _p(self.rb_w2[r][j]), _p(self.rb_b2[r][j])
        dw.post_w, dw.post_b, dw.pqmf = _p(self.post_w), _p(self.post_b), _p(self.pqmf)
        return dw


RB_KERNELS = (3, 7, 11)
RB_DILATIONS = (1, 3, 5)


def make_decoder_weights(rng: np.random.Generator, wstd: float = 0.02,
                         bstd: float = 0.01) -> DecoderWeights:
    """Random-init decoder of the v21_mbistft_16k architecture (config 3): each layer draws its
    ONNX-layout weight N(0, wstd^2) then its bias N(0, bstd^2), in graph order: conv_pre, ups.0,
    resblocks 0-2 (convs1.0-2 then convs2.0-2 per block), ups.1, resblocks 3-5, conv_post."""
    def conv(cout, cin, k):
        W = (wstd * rng.standard_normal((cout, cin, k))).astype(np.float32)
        b = (bstd * rng.standard_normal(cout)).astype(np.float32)
        return pack_conv(W), b

    def convT(cin, cout, k, s):
        W = (wstd * rng.standard_normal((cin, cout, k))).astype(np.float32)
        b = (bstd * rng.standard_normal(cout)).astype(np.float32)
        return pack_convT(W, s), b

    pre_w, pre_b = conv(512, 192, 7)
    ups_w, ups_b = [None, None], [None, None]
    rb_w1 = [[None] * 3 for _ in range(6)]
    rb_b1 = [[None] * 3 for _ in range(6)]
    rb_w2 = [[None] * 3 for _ in range(6)]
    rb_b2 = [[None] * 3 for _ in range(6)]
    for s, (cin, cout) in enumerate(((512, 256), (256, 128))):
        ups_w[s], ups_b[s] = convT(cin, cout, 16, 4)
        for rb in range(3):
            r = 3 * s + rb
            K = RB_KERNELS[rb]
            for j in range(3):
                rb_w1[r][j], rb_b1[r][j] = conv(cout, cout, K)
            for j in range(3):
                rb_w2[r][j], rb_b2[r][j] = conv(cout, cout, K)
    post_w, post_b = conv(72, 128, 7)
    return DecoderWeights(pre_w, pre_b, ups_w, ups_b, rb_w1, rb_b1, rb_w2, rb_b2, post_w, post_b,
                          pqmf_synthesis_filter())


def _conv_sizes():
    """Packed element counts of every decoder record, in DecoderWeights order."""
    n = {"pre_w": 512 * 7 * 192, "pre_b": 512, "post_w": 72 * 7 * 128, "post_b": 72}
    for s, (cin, c) in enumerate(((512, 256), (256, 128))):
        n[f"ups_w{s}"] = 4 * c * 4 * cin
        n[f"ups_b{s}"] = c
        for rb in range(3):
            K = RB_KERNELS[rb]
            n[f"rb{3 * s + rb}"] = (c * K * c, c)
    return n


def load_ptk(path: str) -> DecoderWeights:
    """Decoder weights read from a reference weight container (.ptk) by the library's reader
    (pt_b200_ptk_open: fp16 '#h' payloads widened to fp32; no GPU needed)."""
    h = lib().pt_b200_ptk_open(path.encode())
    if not h:
        raise PtB200Error(f"pt_b200_ptk_open: {lib().pt_b200_last_error().decode()}")
    try:
        cw = DecWeightsC()
        _check(lib().pt_b200_ptk_decoder_weights(h, C.byref(cw)), "pt_b200_ptk_decoder_weights")
        n = _conv_sizes()

        def arr(ptr, count):
            return np.ctypeslib.as_array(C.cast(ptr, C.POINTER(C.c_float)), (count,)).copy()

        rb_w1 = [[None] * 3 for _ in range(6)]
        rb_b1 = [[None] * 3 for _ in range(6)]
        rb_w2 = [[None] * 3 for _ in range(6)]
        rb_b2 = [[None] * 3 for _ in range(6)]
        for r in range(6):
            wn, bn = n[f"rb{r}"]
            for j in range(3):
                rb_w1[r][j], rb_b1[r][j] = arr(cw.rb_w1[r][j], wn), arr(cw.rb_b1[r][j], bn)
                rb_w2[r][j], rb_b2[r][j] = arr(cw.rb_w2[r][j], wn), arr(cw.rb_b2[r][j], bn)
        return DecoderWeights(arr(cw.pre_w, n["pre_w"]), arr(cw.pre_b, n["pre_b"]),
                              [arr(cw.ups_w[s], n[f"ups_w{s}"]) for s in range(2)],
                              [arr(cw.ups_b[s], n[f"ups_b{s}"]) for s in range(2)],
                              rb_w1, rb_b1, rb_w2, rb_b2,
                              arr(cw.post_w, n["post_w"]), arr(cw.post_b, n["post_b"]),
                              arr(cw.pqmf, 4 * 63).reshape(1, 4, 63))
    finally:
        lib().pt_b200_ptk_close(h)


def config1(seed: int = 0):
    """Config 1: one Conv1d 512 -> 256, k7, same padding, T = 256: x [1][512][256] ~ N(0,1), ONNX
    weight [256][512][7] ~ N(0, 0.02^2), bias ~ N(0, 0.01^2), from one generator; returns
    (x, packed weights, bias).  The conv is followed by LeakyReLU 0.1."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((1, 512, 256)).astype(np.float32)
    W = (0.02 * rng.standard_normal((256, 512, 7))).astype(np.float32)
    b = (0.01 * rng.standard_normal(256)).astype(np.float32)
    return x, pack_conv(W), b


def config2(seed: int = 1):
    """Config 2: one ConvTranspose1d 512 -> 256, k16, s4, p6, T_in = 256 -> 1024: x ~ N(0,1),
    ONNX weight [512][256][16] ~ N(0, 0.02^2), bias ~ N(0, 0.01^2); returns (x, packed weights,
    bias).  The convT is followed by LeakyReLU 0.1."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((1, 512, 256)).astype(np.float32)
    W = (0.02 * rng.standard_normal((512, 256, 16))).astype(np.float32)
    b = (0.01 * rng.standard_normal(256)).astype(np.float32)
    return x, pack_convT(W, 4), b


def config3(seed: int = 2, T: int = 226):
    """Config 3: latent z [192][T] ~ N(0,1), then the decoder weights, from one generator."""
    rng = np.random.default_rng(seed)
    z = rng.standard_normal((192, T)).astype(np.float32)
    return make_decoder_weights(rng), z


def config4(seed: int = 3, n: int = 64, lo: int = 50, hi: int = 600):
    """Config 4: n requests, T ~ U{lo..hi} (inclusive integers), z ~ N(0,1) per request."""
    rng = np.random.default_rng(seed)
    T = rng.integers(lo, hi + 1, size=n)
    zs = [rng.standard_normal((192, int(t))).astype(np.float32) for t in T]
    return [int(t) for t in T], zs


def config5(seed: int = 4, n: int = 512, lo: int = 100, hi: int = 1000):
    """Config 5: n streams, T ~ U{lo..hi} (inclusive integers), z ~ N(0,1) per stream; decoded in
    64-frame windows with 16 frames of context per side (step 32)."""
    return config4(seed, n, lo, hi)


STREAM_WIN, STREAM_CTX = 64, 16


def stream_plan(T, win: int = STREAM_WIN, ctx: int = STREAM_CTX, exact: bool = False) -> np.ndarray:
    """The library's window plan (pt_b200_stream_plan) as an int64 array of rows
    (frames, z_off, z_ld, keep_lo, keep_hi, dst) over concatenated latents / waveforms."""
    T = np.ascontiguousarray(T, np.int64)
    n = lib().pt_b200_stream_plan(len(T), T.ctypes.data_as(_i64p), win, ctx, int(exact), None, 0)
    if n < 0:
        _check(-1, "pt_b200_stream_plan")
    arr = (WindowC * max(n, 1))()
    lib().pt_b200_stream_plan(len(T), T.ctypes.data_as(_i64p), win, ctx, int(exact), arr, n)
    return np.array([[w.frames, w.z_off, w.z_ld, w.keep_lo, w.keep_hi, w.dst] for w in arr[:n]],
                    np.int64).reshape(-1, 6)


def carry_plan(T, chunk: int = STREAM_WIN - 2 * STREAM_CTX):
    """The carried-state pass plan (pt_b200_carry_plan, no GPU): (passes, lo, hi), lo / hi of
    shape [passes][streams] -- the samples [lo, hi) of each stream that each pass emits."""
    T = np.ascontiguousarray(T, np.int64)
    n = lib().pt_b200_carry_plan(len(T), T.ctypes.data_as(_i64p), chunk, None, None, 0)
    if n < 0:
        _check(-1, "pt_b200_carry_plan")
    lo = np.zeros((n, len(T)), np.int64)
    hi = np.zeros((n, len(T)), np.int64)
    lib().pt_b200_carry_plan(len(T), T.ctypes.data_as(_i64p), chunk, lo.ctypes.data_as(_i64p),
                             hi.ctypes.data_as(_i64p), lo.size)
    return int(n), lo, hi


def carry_device_bytes(T, chunk: int = STREAM_WIN - 2 * STREAM_CTX) -> int:
    """Device bytes a carried session of these streams holds (pt_b200_carry_device_bytes)."""
    T = np.ascontiguousarray(T, np.int64)
    b = lib().pt_b200_carry_device_bytes(len(T), T.ctypes.data_as(_i64p), chunk)
    if b < 0:
        _check(-1, "pt_b200_carry_device_bytes")
    return int(b)


class CarrySession:
    """A carried-state streaming session (pt_b200_carry_*): pass k feeds latent frames
    [k*chunk, (k+1)*chunk) of every stream and emits the samples whose inputs are complete."""

    def __init__(self, decoder: "Decoder", T, chunk: int = STREAM_WIN - 2 * STREAM_CTX):
        self.T = np.ascontiguousarray(T, np.int64)
        self.h = lib().pt_b200_carry_open(decoder.h, len(self.T), self.T.ctypes.data_as(_i64p),
                                          chunk)
        if not self.h:
            _check(-1, "pt_b200_carry_open")
        self.passes = lib().pt_b200_carry_passes(self.h)
        self.bytes = int(lib().pt_b200_carry_bytes(self.h))

    def run(self, k: int, z_dev: int, wav_dev: int, stream=None) -> None:
        _check(lib().pt_b200_carry_run(self.h, stream, k, z_dev, wav_dev), "pt_b200_carry_run")

    def run_all(self, z_dev: int, wav_dev: int, stream=None) -> None:
        """Rewind, then every pass (asynchronous on `stream`)."""
        _check(lib().pt_b200_carry_reset(self.h), "pt_b200_carry_reset")
        for k in range(self.passes):
            self.run(k, z_dev, wav_dev, stream)

    def close(self) -> None:
        if self.h:
            lib().pt_b200_carry_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def decoder_gflop(T: int) -> float:
    """Algorithmic GFLOP of one decoder request of T frames (2 x MACs; convT counted without the
    zero-stuffed MACs; the tail's einsum / OLA / PQMF included)."""
    macs = 512 * 192 * 7 * T                       # conv_pre
    for s, (cin, c) in enumerate(((512, 256), (256, 128))):
        Tin = T * (4 ** s)
        macs += cin * c * 16 * Tin                 # ups (useful MACs: K per input sample)
        L = 4 * Tin
        macs += 2 * 3 * sum(RB_KERNELS) * c * c * L
    Tp = 16 * T + 1
    macs += 72 * 128 * 7 * Tp                      # conv_post
    macs += 2 * 4 * 9 * 16 * Tp                    # einsum re + im
    macs += 4 * 16 * Tp                            # overlap-add
    macs += 63 * 4 * 256 * T                       # PQMF synthesis (4 bands x 63 taps)
    return 2.0 * macs / 1e9


def conv_gflop(T: int) -> float:
    """GFLOP of the conv stack alone (conv_pre, ups, MRF convs, conv_post)."""
    macs = 512 * 192 * 7 * T
    for s, (cin, c) in enumerate(((512, 256), (256, 128))):
        Tin = T * (4 ** s)
        macs += cin * c * 16 * Tin
        macs += 2 * 3 * sum(RB_KERNELS) * c * c * (4 * Tin)
    macs += 72 * 128 * 7 * (16 * T + 1)
    return 2.0 * macs / 1e9


# --------------------------------------------------------------------------------------------
class Decoder:
    """The batched device-resident decoder (pt_b200_decoder_*)."""

    def __init__(self, weights: DecoderWeights, device: int = 0):
        self.weights = weights
        self._cw = weights.as_c()
        h = lib().pt_b200_decoder_create(device, C.byref(self._cw))
        if not h:
            raise PtB200Error(f"pt_b200_decoder_create failed: {lib().pt_b200_last_error()}")
        self.h = h
        self.device = device

    @classmethod
    def from_container(cls, path: str, device: int = 0) -> "Decoder":
        """The decoder of a reference weight container (.ptk)."""
        return cls(load_ptk(path), device)

    def close(self) -> None:
        if self.h:
            lib().pt_b200_decoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def decode(self, zs: list) -> list:
        """Host in, host out: each z [192][T_i] -> wav [256*T_i]."""
        T = np.array([z.shape[-1] for z in zs], np.int64)
        zcat = np.ascontiguousarray(np.concatenate([np.ascontiguousarray(z, np.float32).ravel()
                                                    for z in zs]))
        wav = np.empty(int(256 * T.sum()), np.float32)
        _check(lib().pt_b200_decode_batch(self.h, None, len(zs), T.ctypes.data_as(_i64p),
                                          zcat.ctypes.data, wav.ctypes.data),
               "pt_b200_decode_batch")
        out, o = [], 0
        for t in T:
            out.append(wav[o:o + 256 * int(t)])
            o += 256 * int(t)
        return out

    def decode_host_ptr(self, T: np.ndarray, z_ptr: int, wav_ptr: int, stream=None) -> None:
        """Concatenated host buffers given by address (pinned buffers in bench.py)."""
        _check(lib().pt_b200_decode_batch(self.h, stream, len(T), T.ctypes.data_as(_i64p),
                                          z_ptr, wav_ptr), "pt_b200_decode_batch")

    def decode_async(self, T: np.ndarray, z_ptr: int, wav_ptr: int) -> None:
        """Pipelined host-buffer decode (pinned buffers): queue upload, decode and download and
        return; decode_async_wait() joins every queued call."""
        T = np.ascontiguousarray(T, np.int64)
        _check(lib().pt_b200_decode_batch_async(self.h, len(T), T.ctypes.data_as(_i64p), z_ptr,
                                                wav_ptr), "pt_b200_decode_batch_async")

    def decode_async_wait(self) -> None:
        _check(lib().pt_b200_decode_async_wait(self.h), "pt_b200_decode_async_wait")

    def async_streams(self):
        """(upload, decode, download) cudaStream_t handles of the pipelined entry point."""
        up, dec, down = C.c_void_p(), C.c_void_p(), C.c_void_p()
        _check(lib().pt_b200_decode_async_streams(self.h, C.byref(up), C.byref(dec),
                                                  C.byref(down)), "pt_b200_decode_async_streams")
        return up.value, dec.value, down.value

    def decode_device(self, T: np.ndarray, z_dev: int, wav_dev: int, stream=None) -> None:
        """Concatenated device buffers (addresses), asynchronous on `stream`."""
        _check(lib().pt_b200_decode_batch_device(self.h, stream, len(T),
                                                 T.ctypes.data_as(_i64p), z_dev, wav_dev),
               "pt_b200_decode_batch_device")

    def decode_windows(self, windows: np.ndarray, z_dev: int, wav_dev: int, stream=None) -> None:
        """Windows given as rows (frames, z_off, z_ld, keep_lo, keep_hi, dst); device buffers."""
        w = np.ascontiguousarray(windows, np.int64).reshape(-1, 6)
        arr = (WindowC * len(w))(*[WindowC(*map(int, r)) for r in w])
        _check(lib().pt_b200_decode_windows(self.h, stream, len(w), arr, z_dev, wav_dev),
               "pt_b200_decode_windows")

    def stream_device(self, T, z_dev: int, wav_dev: int, win: int = STREAM_WIN,
                      ctx: int = STREAM_CTX, exact: bool = False, max_frames: int = 0,
                      stream=None) -> None:
        """Decode and stitch every stream (concatenated [192][T_i] latents -> concatenated
        [256*T_i] waveforms, device buffers), asynchronous on `stream`."""
        T = np.ascontiguousarray(T, np.int64)
        _check(lib().pt_b200_stream_decode(self.h, stream, len(T), T.ctypes.data_as(_i64p), z_dev,
                                           win, ctx, int(exact), int(max_frames), wav_dev),
               "pt_b200_stream_decode")

    def stream(self, zs: list, win: int = STREAM_WIN, ctx: int = STREAM_CTX,
               exact: bool = False, max_frames: int = 0) -> list:
        """Host in, host out: each stream's z [192][T_i] -> stitched wav [256*T_i]."""
        import torch
        T = np.array([z.shape[-1] for z in zs], np.int64)
        zcat = np.concatenate([np.ascontiguousarray(z, np.float32).ravel() for z in zs])
        dev = torch.device("cuda", self.device)
        z_dev = torch.from_numpy(zcat).to(dev)
        wav_dev = torch.full((int(256 * T.sum()),), float("nan"), device=dev)
        s = torch.cuda.Stream(device=dev)
        self.stream_device(T, z_dev.data_ptr(), wav_dev.data_ptr(), win, ctx, exact, max_frames,
                           s.cuda_stream)
        self.sync(s.cuda_stream)
        wav = wav_dev.cpu().numpy()
        out, o = [], 0
        for t in T:
            out.append(wav[o:o + 256 * int(t)])
            o += 256 * int(t)
        return out

    def stream_carry_device(self, T, z_dev: int, wav_dev: int,
                            chunk: int = STREAM_WIN - 2 * STREAM_CTX, stream=None) -> None:
        """Carried-state streaming of every stream (device buffers laid out as for
        stream_device): open a session, run its passes, close it; synchronous."""
        T = np.ascontiguousarray(T, np.int64)
        _check(lib().pt_b200_stream_decode_carry(self.h, stream, len(T), T.ctypes.data_as(_i64p),
                                                 z_dev, chunk, wav_dev),
               "pt_b200_stream_decode_carry")

    def stream_carry(self, zs: list, chunk: int = STREAM_WIN - 2 * STREAM_CTX) -> list:
        """Host in, host out: each stream's z [192][T_i] -> its wav [256*T_i], carried state."""
        import torch
        T = np.array([z.shape[-1] for z in zs], np.int64)
        zcat = np.concatenate([np.ascontiguousarray(z, np.float32).ravel() for z in zs])
        dev = torch.device("cuda", self.device)
        z_dev = torch.from_numpy(zcat).to(dev)
        wav_dev = torch.full((int(256 * T.sum()),), float("nan"), device=dev)
        s = torch.cuda.Stream(device=dev)
        self.stream_carry_device(T, z_dev.data_ptr(), wav_dev.data_ptr(), chunk, s.cuda_stream)
        wav = wav_dev.cpu().numpy()
        out, o = [], 0
        for t in T:
            out.append(wav[o:o + 256 * int(t)])
            o += 256 * int(t)
        return out

    def sync(self, stream=None) -> None:
        _check(lib().pt_b200_decoder_sync(self.h, stream), "pt_b200_decoder_sync")

    def checkpoints(self, z: np.ndarray):
        """pt_b200_decoder_checkpoints: one request's 40 per-layer outputs (channel-major, no gap
        rows; shapes in include/pt_b200.h) and its waveform."""
        z = np.ascontiguousarray(z, np.float32)
        T = z.shape[-1]
        shapes = [(512, T)] + [(256, 4 * T)] * 19 + [(128, 16 * T)] * 19 + [(72, 16 * T + 1)]
        shapes[38] = (128, 16 * T + 1)
        ck = [np.empty(sh, np.float32) for sh in shapes]
        arr = (_f * len(ck))(*[_p(a) for a in ck])
        wav = np.empty(256 * T, np.float32)
        _check(lib().pt_b200_decoder_checkpoints(self.h, _p(z), T, arr, _p(wav)),
               "pt_b200_decoder_checkpoints")
        return ck, wav

    LAUNCH_KINDS = ("stage", "conv", "convT", "conv_post", "tail")

    def profile(self, enable: bool) -> None:
        _check(lib().pt_b200_decoder_profile(self.h, int(enable)), "pt_b200_decoder_profile")

    def launch_times(self) -> list:
        """[(kind, N tile, ms, algorithmic flops, algorithmic bytes)] for each launch of the last
        decode (call after sync; profiling must be on).  The N tile names the tensor-core conv
        instance (conv_tc_kernel<N tile, stages>), 0 for the other kernels."""
        n = 64
        ms, fl, by = (C.c_double * n)(), (C.c_double * n)(), (C.c_double * n)()
        kd = (C.c_int * n)()
        k = lib().pt_b200_decoder_launch_times(self.h, n, ms, fl, by, kd)
        if k < 0:
            _check(k, "pt_b200_decoder_launch_times")
        return [(self.LAUNCH_KINDS[kd[i] & 255], kd[i] >> 8, ms[i], fl[i], by[i])
                for i in range(k)]
