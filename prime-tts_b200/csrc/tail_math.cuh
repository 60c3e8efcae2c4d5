// tail_math.cuh -- the per-frame arithmetic of the MB-iSTFT tail (the Exp / Sin / Cos, einsum and
// Hann-window nodes among /dec/Reshape_6 .. /dec/Conv, ref/v21_graph_trace.txt 3957-4065), shared by the
// tail kernel (tail.cu) and conv_post's frames epilogue (conv_tc.cuh), so that both compute every
// windowed frame with the same operations in the same order and agree bit for bit.
#pragma once
#include <cmath>

namespace ptb {

// periodic Hann window and its square; the inverse real-DFT basis (cosine and sine rows, k-major
// 9 x 16, with the one-sided weights and the 1/16); defined and uploaded per device by tail.cu
extern __constant__ float c_win[16], c_win2[16];
extern __constant__ float c_bc[144], c_bs[144];

// magnitude / phase of one bin: re = exp(a) * cos(pi * sin(b)), im = exp(a) * sin(pi * sin(b))
// (the cosine and sine of the phase come from one sincos call).  F32: fp32 functions, the
// hardware approximations for exp and for the phase's sincos; otherwise double-precision ones
// rounded to fp32 (the reference's choice for small tensors).
template <bool F32>
__device__ __forceinline__ void tr_bin(float la, float lb, float &rv, float &iv) {
  float mag, sb, c, sn;
  if constexpr (F32) {
    mag = __expf(la);
    sb = sinf(lb);
  } else {
    mag = (float)exp((double)la);
    sb = (float)sin((double)lb);
  }
  const float ph = __fmul_rn(sb, 3.1415927410125732f);
  if constexpr (F32) {
    __sincosf(ph, &sn, &c);
  } else {
    double sd, cd;
    sincos((double)ph, &sd, &cd);
    sn = (float)sd;
    c = (float)cd;
  }
  rv = __fmul_rn(mag, c);
  iv = __fmul_rn(mag, sn);
}

// The 9 -> 16 basis sums of one (frame, band) (fp32 FMAs, k ascending, zero basis entries skipped),
// then the window; `out` receives the band's 16 samples.  Columns n and 16 - n come from one
// pair of sums: the tables are mirror-symmetric (bc[k][16 - n] = bc[k][n], bs[k][16 - n] =
// -bs[k][n]) except for entries below 1e-15 that stand for exact zeros (cos(pi / 2) in double is
// 6.1e-17), and the host checks that when it builds them.  The zero entries skipped are known in
// advance: the sine basis is exactly zero at k = 0 and at n = 0 (sin 0) and nowhere else, the
// cosine basis nowhere; the host checks both.
__device__ __forceinline__ void basis_sym(const float (&rv)[9], const float (&iv)[9], float *out) {
  float er[9], ei[9];
#pragma unroll
  for (int n = 0; n < 9; ++n) er[n] = ei[n] = 0.0f;
#pragma unroll
  for (int k = 0; k < 9; ++k) {
#pragma unroll
    for (int n = 0; n < 9; ++n) {
      er[n] = __fmaf_rn(c_bc[k * 16 + n], rv[k], er[n]);
      if (k != 0 && n != 0) ei[n] = __fmaf_rn(c_bs[k * 16 + n], iv[k], ei[n]);
    }
  }
#pragma unroll
  for (int n = 0; n < 9; ++n) out[n] = __fmul_rn(__fadd_rn(er[n], ei[n]), c_win[n]);
#pragma unroll
  for (int n = 9; n < 16; ++n) out[n] = __fmul_rn(__fsub_rn(er[16 - n], ei[16 - n]), c_win[n]);
}

// One (frame, band) from its 9 log-magnitudes `la` and 9 phase logits `lb` (fp32 functions):
// the 16 windowed samples of the band's inverse-DFT frame.
__device__ __forceinline__ void frame_band(const float (&la)[9], const float (&lb)[9],
                                           float (&out)[16]) {
  float rv[9], iv[9];
#pragma unroll
  for (int k = 0; k < 9; ++k) tr_bin<true>(la[k], lb[k], rv[k], iv[k]);
  basis_sym(rv, iv, out);
}

}  // namespace ptb
