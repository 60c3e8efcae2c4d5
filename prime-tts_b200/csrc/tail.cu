// tail.cu -- the MB-iSTFT + PQMF synthesis tail as one kernel (graph nodes /dec/Reshape_6 ..
// /dec/Conv, ref/v21_graph_trace.txt 3957-4065).
//
// Per request the conv_post output holds Tp frames x 72 channels = 4 subbands x (9 log-magnitudes,
// 9 phase logits).  One CTA produces kTailW consecutive output samples:
//   1. frames:  mag = exp(a), ph = pi * sin(b), re/im = mag * cos/sin(ph); the 9 -> 16 inverse
//      real-DFT basis contraction (the reference einsum, runtime/v21/src/pt_v21_host.c:
//      1963-1995, accumulates in double; here fp32 fused multiply-adds), re + im, times the
//      periodic Hann window;
//   2. overlap-add (hop 4, the eye(16) ConvTranspose) divided by the clipped window-sum
//      envelope (ConvTranspose_1 of ones with the Hann^2 kernel, Clip 1e-9, Div), trimmed [8:-8];
//   3. x4 zero-stuffed upsampling with gain 4 (ConvTranspose_2) folded into the 63-tap PQMF
//      synthesis conv: only taps landing on a stuffed sample (one in four) are evaluated.
// The tail is instruction-bound (its HBM bytes are small), so it trades the reference's exact
// operation order for fewer instructions where the result moves by less than a microunit: the
// magnitude's exp and the phase rotation's sincos use the hardware approximations (__expf;
// __sincosf on a phase in [-pi, pi], absolute error below 2^-21), the basis sums run in fp32
// FMAs and the PQMF taps fuse their multiply-adds; sin(b), whose argument is unbounded, stays
// the accurate sinf.  Against the reference's own order (the CPU oracle): max relative error
// 4.3e-7 and >= 132 dB on N(0, 0.25) spectra at Tp = 2 .. 3617 (the test gate: 1e-5, 100 dB);
// 148 -> 123 us per config-4 decode.
#include <cmath>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "tail_math.cuh"

namespace ptb {

constexpr int kTailW = 1024;                 // output samples per CTA (45.8 KB of shared memory)
// 9 warps: 8 frames x 36 bins in the magnitude / phase phase, the 576 (frame, band, half) basis
// items of a chunk in two rounds, the 276 staged overlap-add samples in one; the PQMF phase uses 8
constexpr int kTailThreads = 288;
constexpr int kTailP3 = 256;
constexpr int kTailF = kTailW / 16 + 8;      // staged frames (chunk + halo): NF <= W/16 + 5
constexpr int kTailM = kTailW / 4 + 20;      // staged trimmed-OLA samples per band

__constant__ float c_win[16], c_win2[16];   // declared in tail_math.cuh
__constant__ float c_bc[144], c_bs[144];   // the inverse real-DFT basis (cosine, sine rows)

// Frame rows are 68 floats (4 bands x 16 + 4 pad): the overlap-add reads 8 consecutive frames at
// one (band, sample) per warp and the stride of 68 puts those reads on 32 distinct banks.
constexpr int kFrStride = 68;
struct TailSmem {
  float re[kTailF][4][9], im[kTailF][4][9];   // per frame, band, bin
  float fr[kTailF][kFrStride];                 // windowed frames, [frame][band * 16 + n]
  float4 sm[kTailM];                           // trimmed OLA, 4 bands interleaved
  float4 h[63];                                // PQMF taps, 4 bands interleaved
  float win2[16];
};
// The frames variant reads windowed frames that conv_post's epilogue computed (the decoder's
// batched paths): no spectra, the frame rows staged straight from memory.
struct TailFrSmem {
  float fr[kTailF][kFrStride];
  float4 sm[kTailM];
  float4 h[63];
  float win2[16];
};

struct TailArgs {
  const float *post;      // element (channel c, frame f) of request r:
  long long st_t, st_c;   //   post[(row0[r] + f) * st_t + c * st_c]
  const long long *row0;  // per request (nullptr: 0)
  const long long *tp;    // per request frame count (nullptr: tp1)
  const long long *wav0;  // per request output offset (nullptr: 0): sample j goes to wav[wav0 + j]
  const long long *klo, *khi;   // per request kept samples [klo, khi) (nullptr: all)
  const long long *jbase;       // per request first sample of CTA 0 (nullptr: 0; a multiple of kTailW)
  long long tp1;
  const float *pqmf;      // [4][63]
  float *wav;
};

// Phase 1a loop of one thread: its bin's frames fl0, fl0 + 8, ... of [0, NF), two at a time, the
// next two frames' loads issued before this pair's math; frames outside [flo, fhi) are zeros.
template <bool F32>
__device__ __forceinline__ void bins_loop(const float *pc, long long st_t, long long cst,
                                          long long F0, int NF, int flo, int fhi, int fl0,
                                          float *pre, float *pim) {
  auto ld = [&](int f, float &x, float &y) {
    x = 0.0f;
    y = 0.0f;
    if (f < NF && f >= flo && f < fhi) {
      const float *pf = pc + (F0 + f) * st_t;
      x = pf[0];
      y = pf[9 * cst];
    }
  };
  float na, nb, na2, nb2;
  ld(fl0, na, nb);
  ld(fl0 + 8, na2, nb2);
  for (int fl = fl0; fl < NF; fl += 16) {
    const int fl2 = fl + 8;
    const bool v1 = fl >= flo && fl < fhi, v2 = fl2 < NF && fl2 >= flo && fl2 < fhi;
    const float la = na, lb = nb, la2 = na2, lb2 = nb2;
    ld(fl + 16, na, nb);
    ld(fl + 24, na2, nb2);
    float rv, iv, rv2, iv2;
    tr_bin<F32>(la, lb, rv, iv);
    tr_bin<F32>(la2, lb2, rv2, iv2);
    pre[fl * 36] = v1 ? rv : 0.0f;
    pim[fl * 36] = v1 ? iv : 0.0f;
    if (fl2 < NF) {
      pre[fl2 * 36] = v2 ? rv2 : 0.0f;
      pim[fl2 * 36] = v2 ? iv2 : 0.0f;
    }
  }
}

// FR = false: `post` holds conv_post's 72 channels per frame and the kernel runs phases 1-3.
// FR = true: `post` holds each frame's 64 windowed samples ([band * 16 + n], conv_post's frames
// epilogue, the same arithmetic as phases 1a-1b) and the kernel runs phases 2-3.
template <bool FR>
__global__ void __launch_bounds__(FR ? kTailP3 : kTailThreads, FR ? 8 : 4) tail_kernel(const TailArgs a) {
  extern __shared__ __align__(16) unsigned char tail_smem[];
  using Smem = typename std::conditional<FR, TailFrSmem, TailSmem>::type;
  Smem &S = *reinterpret_cast<Smem *>(tail_smem);
  auto &fr = S.fr;
  auto &sm = S.sm;
  const int req = blockIdx.y;
  const long long Tp = a.tp ? a.tp[req] : a.tp1;
  const long long nwav = 16 * (Tp - 1);
  const long long j0 = (a.jbase ? a.jbase[req] : 0) + (long long)blockIdx.x * kTailW;
  const long long keep_lo = a.klo ? a.klo[req] : 0, keep_hi = a.khi ? a.khi[req] : nwav;
  if (Tp < 2 || j0 >= nwav || j0 >= keep_hi || j0 + kTailW <= keep_lo) return;
  const long long Ls = 4 * (Tp - 1);
  const float *post = a.post + (a.row0 ? a.row0[req] : 0) * a.st_t;

  float *hf = reinterpret_cast<float *>(S.h);
  for (int i = threadIdx.x; i < 4 * 63; i += blockDim.x) hf[(i % 63) * 4 + i / 63] = a.pqmf[i];
  if (threadIdx.x < 16) S.win2[threadIdx.x] = c_win2[threadIdx.x];

  // trimmed-OLA samples m needed by outputs [j0, j0 + W): stuffed index 4m in [j - 31, j + 31];
  // m_lo_raw .. m_hi_raw before clipping to the signal, which is zero outside [0, Ls)
  const long long m_lo_raw = (j0 - 31 + 3) >> 2;
  long long m_lo = m_lo_raw;
  if (m_lo < 0) m_lo = 0;
  long long m_hi = (j0 + kTailW - 1 + 31) >> 2;
  if (m_hi > Ls - 1) m_hi = Ls - 1;
  // frames feeding OLA positions p = m + 8: q = p / 4 and its three predecessors
  const long long F0 = ((m_lo + 8) >> 2) - 3;
  const int NF = (int)(((m_hi + 8) >> 2) - F0 + 1);

  if constexpr (FR) {
    // ---- 1. the windowed frames F0 + fl in [0, Tp) that the overlap-add reads, 16 float4 a row
    for (int i = threadIdx.x; i < NF * 16; i += blockDim.x) {
      const int fl = i >> 4, c4 = i & 15;
      const long long qq = F0 + fl;
      if (qq >= 0 && qq < Tp)
        *reinterpret_cast<float4 *>(&fr[fl][4 * c4]) =
            __ldg(reinterpret_cast<const float4 *>(post + qq * a.st_t) + c4);
    }
    __syncthreads();
  } else {
    // ---- 1a. per (frame, band, bin): magnitude / phase -> re, im.  Thread t owns bin t % 36 of
    // frames t / 36, t / 36 + 8, ...: the bin's column, band and basis row are fixed per
    // thread, so the loop carries only pointers; two frames at a time (independent chains in
    // flight), the next two frames' loads issued before this pair's math.  Frames outside
    // [0, Tp) never reach the overlap-add: zeros.
    static_assert(kTailThreads == 288, "phase 1a maps 8 frames x 36 bins onto the threads");
    {
      const int rb = threadIdx.x % 36, fl0 = threadIdx.x / 36, b = rb / 9, k = rb - b * 9;
      const long long flo_l = -F0 > 0 ? -F0 : 0, fhi_l = Tp - F0 < NF ? Tp - F0 : NF;
      const int flo = (int)flo_l, fhi = (int)fhi_l;   // valid frames [flo, fhi) of [0, NF)
      const long long cst = a.st_c;
      const float *pc = post + (long long)(b * 18 + k) * cst;
      float *pre = &S.re[0][b][k], *pim = &S.im[0][b][k];
      // the fp32 / double choice is per request: one code path per CTA, not a branch per bin;
      // the reference switches Exp/Sin/Cos to fp32 libm only for tensors of >= 4096 elements
      if (36 * Tp >= 4096) bins_loop<true>(pc, a.st_t, cst, F0, NF, flo, fhi, fl0, pre, pim);
      else bins_loop<false>(pc, a.st_t, cst, F0, NF, flo, fhi, fl0, pre, pim);
    }
    __syncthreads();
    // ---- 1b. per (frame, band): the 9 -> 16 basis sums and the window (basis_sym: a thread loads
    // its frame's nine re / im values once and keeps 18 independent chains; the basis constants
    // are instruction operands).  Zero basis entries are skipped, as in the reference einsum,
    // and each bin sums k in ascending order.
    for (int it = threadIdx.x; it < NF * 4; it += blockDim.x) {
      const int fl = it >> 2, b = it & 3;
      basis_sym(S.re[fl][b], S.im[fl][b], &fr[fl][b * 16]);
    }
    __syncthreads();
  }

  // ---- 2. overlap-add / window-sum envelope, trimmed [8:-8]; frames outside [0, Tp) are absent.
  // sm[i] holds sample m_lo_raw + i; samples outside the signal (and the spare entries) are zero,
  // so phase 3 reads its whole window without bounds tests.
  // (request-relative indices fit 32 bits: the launchers cap the frame count)
  const int mlr = (int)m_lo_raw, mlo = (int)m_lo, mhi = (int)m_hi, f0 = (int)F0, tp = (int)Tp;
  for (int ml = threadIdx.x; ml < kTailM; ml += blockDim.x) {
    const int m = mlr + ml;
    if (m < mlo || m > mhi) {
      sm[ml] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      continue;
    }
    const int q = (m + 8) >> 2, r = (m + 8) & 3;
    float ola[4] = {0.0f, 0.0f, 0.0f, 0.0f}, env = 0.0f;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int qq = q - t;
      if (qq >= 0 && qq < tp) {
        const int fl = qq - f0;
#pragma unroll
        for (int b = 0; b < 4; ++b) ola[b] = __fadd_rn(ola[b], fr[fl][b * 16 + r + 4 * t]);
        env = __fadd_rn(env, S.win2[r + 4 * t]);
      }
    }
    const float ec = env > 1e-9f ? env : 1e-9f;
    // stored with the zero-stuffing gain 4 applied (a power of two: exact), as phase 3 uses it
    sm[ml] = make_float4(__fmul_rn(4.0f, __fdiv_rn(ola[0], ec)), __fmul_rn(4.0f, __fdiv_rn(ola[1], ec)),
                         __fmul_rn(4.0f, __fdiv_rn(ola[2], ec)), __fmul_rn(4.0f, __fdiv_rn(ola[3], ec)));
  }
  __syncthreads();

  // ---- 3. x4 zero-stuff (gain 4) + 63-tap PQMF synthesis, tap-major then band (conv order).
  // Polyphase: output j only meets taps k = k0 + 4s with (j + k - 31) divisible by 4.  A thread
  // takes output phase p = j mod 4 and four consecutive outputs of that phase (j = j0 + 16g + 4v
  // + p, v = 0..3); tap s of output v reads staged sample q0 + v + s, so the four outputs slide
  // over one window and each tap loads one new sample and one filter tap.  Each output sums
  // taps in ascending order, bands within a tap, as the reference conv does.
  float *wav = a.wav + (a.wav0 ? a.wav0[req] : 0);
  const int jn = (int)(nwav - j0 < kTailW ? nwav - j0 : kTailW);
  const int klo = (int)keep_lo, khi = (int)(keep_hi < nwav ? keep_hi : nwav);
  static_assert(kTailW == 16 * kTailP3 / 4, "phase 3 gives each of its threads four outputs");
  if (threadIdx.x >= kTailP3) return;
  const int p = threadIdx.x & 3, g = threadIdx.x >> 2;
  const int k0 = (31 - p) & 3;   // 16 taps k0 + 4s, 15 for k0 = 3 (phase 0)
  // j0 is a multiple of 4, so j + k0 - 31 is: the shift divides exactly
  const int q0 = (int)(((j0 + 16 * g + p + k0 - 31) >> 2) - m_lo_raw);
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  float4 x0 = sm[q0], x1 = sm[q0 + 1], x2 = sm[q0 + 2], x3 = sm[q0 + 3];
  auto tap = [](float t, const float4 h, const float4 x) {
    t = __fmaf_rn(h.x, x.x, t);
    t = __fmaf_rn(h.y, x.y, t);
    t = __fmaf_rn(h.z, x.z, t);
    return __fmaf_rn(h.w, x.w, t);
  };
  // (the reference skips zero inputs; adding h x 0 changes a sum only in the sign of an exact zero)
  // Fully unrolled, so the sliding window lives in renamed registers.
#pragma unroll
  for (int s = 0; s < 16; ++s) {
    if (s == 15 && k0 == 3) break;
    const float4 h4 = S.h[k0 + 4 * s];
    acc[0] = tap(acc[0], h4, x0);
    acc[1] = tap(acc[1], h4, x1);
    acc[2] = tap(acc[2], h4, x2);
    acc[3] = tap(acc[3], h4, x3);
    x0 = x1;
    x1 = x2;
    x2 = x3;
    if (s < 15) x3 = sm[q0 + s + 4];
  }
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    const int jj = 16 * g + 4 * v + p;
    const long long ju = j0 + jj;
    if (jj < jn && ju >= klo && ju < khi) wav[ju] = acc[v];
  }
}

// the basis / window constants, computed on the host exactly as the reference graph does
static int g_tail_err = 0;
static void tail_constants_init() {
  float bc[144], bs[144];
  static const float win[16] = {
      0.0f,        0.03806024789810181f, 0.1464466154575348f, 0.30865830183029175f,
      0.5f,        0.691341757774353f,   0.8535534143447876f, 0.961939811706543f,
      1.0f,        0.9619397521018982f,  0.853553295135498f,  0.6913415789604187f,
      0.5f,        0.3086581826210022f,  0.14644649624824524f, 0.03806021809577942f};
  static const float win2[16] = {
      0.0f,  0.0014485825086012483f, 0.02144661173224449f, 0.09526994824409485f,
      0.25f, 0.4779534339904785f,    0.7285534143447876f,  0.9253281950950623f,
      1.0f,  0.9253280758857727f,    0.7285532355308533f,  0.477953165769577f,
      0.25f, 0.09526987373828888f,   0.021446576341986656f, 0.0014485801802948117f};
  for (int k = 0; k < 9; ++k) {
    volatile float wk = (k == 0 || k == 8) ? 1.0f : 2.0f;
    for (int n = 0; n < 16; ++n) {
      const double ang = 2.0 * M_PI * (double)k * (double)n / 16.0;
      volatile float c = (float)cos(ang), s = (float)sin(ang);
      volatile float p1 = wk * c, p2 = (-wk) * s;
      bc[k * 16 + n] = p1 / 16.0f;
      bs[k * 16 + n] = p2 / 16.0f;
    }
  }
  for (int i = 0; i < 144; ++i) {
    // the kernels skip exactly these zero entries and mirror columns n and 16 - n (basis_sym)
    const int k = i / 16, n = i % 16;
    if (bc[i] == 0.0f || (bs[i] == 0.0f) != (k == 0 || n == 0)) g_tail_err = 2;
    if (n > 8 && (std::fabs(bc[i] - bc[k * 16 + 16 - n]) > 1e-15f ||
                  std::fabs(bs[i] + bs[k * 16 + 16 - n]) > 1e-15f))
      g_tail_err = 2;
  }
  if (cudaMemcpyToSymbol(c_bc, bc, sizeof(bc)) != cudaSuccess ||
      cudaMemcpyToSymbol(c_bs, bs, sizeof(bs)) != cudaSuccess ||
      cudaMemcpyToSymbol(c_win, win, sizeof(win)) != cudaSuccess ||
      cudaMemcpyToSymbol(c_win2, win2, sizeof(win2)) != cudaSuccess)
    g_tail_err = 1;
}

// constants are per device: initialise on every device that runs the tail
static int tail_ready() {
  static bool done[64] = {false};
  static std::mutex mu;
  int dev = 0;
  PTB_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(mu);
  if (dev < 0 || dev >= 64) return -1;
  if (!done[dev]) {
    g_tail_err = 0;
    tail_constants_init();
    PTB_REQUIRE(g_tail_err != 2,
                "pt_b200: iSTFT basis zeros or mirror symmetry differ from the kernels' assumption");
    PTB_REQUIRE(!g_tail_err, "pt_b200: tail constant upload failed");
    PTB_CUDA(cudaFuncSetAttribute(tail_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)sizeof(TailSmem)));
    PTB_CUDA(cudaFuncSetAttribute(tail_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)sizeof(TailFrSmem)));
    done[dev] = true;
  }
  return 0;
}

// constants on the calling thread's current device (call before a stream capture)
int tail_prepare() { return tail_ready(); }

// single request, channel-major post [72][Tp]
int tail_run(const float *post_dev, int64_t Tp, const float *pqmf_dev, float *wav_dev,
             cudaStream_t st) {
  if (tail_ready()) return -1;
  TailArgs a{};
  a.post = post_dev;
  a.st_t = 1;
  a.st_c = Tp;
  a.tp1 = Tp;
  PTB_REQUIRE(Tp >= 1 && Tp < (1LL << 26), "pt_b200: tail frame count %lld out of range", (long long)Tp);
  a.pqmf = pqmf_dev;
  a.wav = wav_dev;
  const long long nwav = 16 * (Tp - 1);
  dim3 grid((unsigned)((nwav + kTailW - 1) / kTailW), 1);
  tail_kernel<false><<<grid, kTailThreads, sizeof(TailSmem), st>>>(a);
  PTB_CUDA(cudaGetLastError());
  count_launch();
  return 0;
}

// batched requests, channels-last post rows (ld = row stride); per-request tables on the device,
// each request writing only its kept samples.  `chunks` CTAs of kTailW samples per request start
// at sample jbase[r] (all of a request's samples from 0 when jbase is null and chunks is 0).
// frames = 0: the rows hold conv_post's 72 channels; 1: each row's 64 windowed frame samples
// (conv_post's frames epilogue), and only the overlap-add and the PQMF run here.
int tail_run_rows(const float *post_dev, long long ld, const long long *row0, const long long *tp,
                  const long long *wav0, const long long *klo, const long long *khi,
                  const long long *jbase, long long chunks, int nreq, long long max_tp,
                  const float *pqmf_dev, float *wav_dev, cudaStream_t st, int frames) {
  if (tail_ready()) return -1;
  TailArgs a{};
  a.post = post_dev;
  a.st_t = ld;
  a.st_c = 1;
  a.row0 = row0;
  a.tp = tp;
  a.wav0 = wav0;
  a.klo = klo;
  a.khi = khi;
  a.jbase = jbase;
  a.pqmf = pqmf_dev;
  a.wav = wav_dev;
  PTB_REQUIRE(max_tp < (1LL << 26), "pt_b200: tail frame count %lld out of range", max_tp);
  const long long nwav = 16 * (max_tp - 1);
  if (chunks <= 0) chunks = (nwav + kTailW - 1) / kTailW;
  dim3 grid((unsigned)chunks, (unsigned)nreq);
  if (frames) {
    PTB_REQUIRE(ld % 4 == 0 && (reinterpret_cast<uintptr_t>(post_dev) & 15) == 0,
                "pt_b200: frame rows need 16-byte alignment");
    tail_kernel<true><<<grid, kTailP3, sizeof(TailFrSmem), st>>>(a);
  } else {
    tail_kernel<false><<<grid, kTailThreads, sizeof(TailSmem), st>>>(a);
  }
  PTB_CUDA(cudaGetLastError());
  count_launch();
  return 0;
}

}  // namespace ptb
