// tail.cu -- the MB-iSTFT + PQMF synthesis tail as one kernel (graph nodes /dec/Reshape_6 ..
// /dec/Conv, ref/v21_graph_trace.txt 3957-4065).
//
// Per request the conv_post output holds Tp frames x 72 channels = 4 subbands x (9 log-magnitudes,
// 9 phase logits).  One CTA produces kTailW consecutive output samples:
//   1. frames:  mag = exp(a), ph = pi * sin(b), re/im = mag * cos/sin(ph); the 9 -> 16 inverse
//      real-DFT basis contraction in double (the reference einsum's double accumulation,
//      runtime/v21/src/pt_v21_host.c:1963-1995), re + im, times the periodic Hann window;
//   2. overlap-add (hop 4, the eye(16) ConvTranspose) divided by the clipped window-sum
//      envelope (ConvTranspose_1 of ones with the Hann^2 kernel, Clip 1e-9, Div), trimmed [8:-8];
//   3. x4 zero-stuffed upsampling with gain 4 (ConvTranspose_2) folded into the 63-tap PQMF
//      synthesis conv: only taps landing on a stuffed sample (one in four) are evaluated.
// Every fp32 step keeps the reference's operation order (no FMA contraction), so apart from the
// exp/sin/cos implementations the tail reproduces the reference bit for bit.
#include <cmath>
#include <mutex>

#include "common.cuh"

namespace ptb {

constexpr int kTailW = 1024;                 // output samples per CTA
constexpr int kTailThreads = 256;
constexpr int kTailF = kTailW / 16 + 12;     // staged frames (chunk + halo)
constexpr int kTailM = kTailW / 4 + 20;      // staged trimmed-OLA samples per band

__constant__ float c_bc[144], c_bs[144], c_win[16], c_win2[16];

struct TailArgs {
  const float *post;      // element (channel c, frame f) of request r:
  long long st_t, st_c;   //   post[(row0[r] + f) * st_t + c * st_c]
  const long long *row0;  // per request (nullptr: 0)
  const long long *tp;    // per request frame count (nullptr: tp1)
  const long long *wav0;  // per request output offset (nullptr: 0)
  long long tp1;
  const float *pqmf;      // [4][63]
  float *wav;
};

__device__ __forceinline__ float tr_exp(float x, bool f32) { return f32 ? expf(x) : (float)exp((double)x); }
__device__ __forceinline__ float tr_sin(float x, bool f32) { return f32 ? sinf(x) : (float)sin((double)x); }
__device__ __forceinline__ float tr_cos(float x, bool f32) { return f32 ? cosf(x) : (float)cos((double)x); }

__global__ void __launch_bounds__(kTailThreads) tail_kernel(const TailArgs a) {
  __shared__ float fr[4][kTailF][16];
  __shared__ float sm[4][kTailM];
  __shared__ float h[4][63];
  const int req = blockIdx.y;
  const long long Tp = a.tp ? a.tp[req] : a.tp1;
  const long long nwav = 16 * (Tp - 1);
  const long long j0 = (long long)blockIdx.x * kTailW;
  if (Tp < 2 || j0 >= nwav) return;
  const long long Ls = 4 * (Tp - 1);
  const float *post = a.post + (a.row0 ? a.row0[req] : 0) * a.st_t;
  // the reference switches Exp/Sin/Cos to fp32 libm only for tensors of >= 4096 elements
  const bool f32 = 36 * Tp >= 4096;

  for (int i = threadIdx.x; i < 4 * 63; i += blockDim.x) h[i / 63][i % 63] = a.pqmf[i];

  // trimmed-OLA samples m needed by outputs [j0, j0 + W): stuffed index 4m in [j - 31, j + 31]
  long long m_lo = (j0 - 31 + 3) >> 2;
  if (m_lo < 0) m_lo = 0;
  long long m_hi = (j0 + kTailW - 1 + 31) >> 2;
  if (m_hi > Ls - 1) m_hi = Ls - 1;
  // frames feeding OLA positions p = m + 8: q = p / 4 and its three predecessors
  const long long F0 = ((m_lo + 8) >> 2) - 3;
  const int NF = (int)(((m_hi + 8) >> 2) - F0 + 1);

  // ---- 1. frames
  for (int it = threadIdx.x; it < 4 * NF; it += blockDim.x) {
    const int b = it / NF, fl = it - b * NF;
    const long long f = F0 + fl;
    float out[16];
    if (f >= 0 && f < Tp) {
      float re[9], im[9];
      const float *pf = post + f * a.st_t;
#pragma unroll
      for (int k = 0; k < 9; ++k) {
        const float mag = tr_exp(pf[(long long)(b * 18 + k) * a.st_c], f32);
        const float ph = __fmul_rn(tr_sin(pf[(long long)(b * 18 + 9 + k) * a.st_c], f32),
                                   3.1415927410125732f);
        re[k] = __fmul_rn(mag, tr_cos(ph, f32));
        im[k] = __fmul_rn(mag, tr_sin(ph, f32));
      }
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        double er = 0.0, ei = 0.0;
#pragma unroll
        for (int k = 0; k < 9; ++k) {
          const float bc = c_bc[k * 16 + n], bs = c_bs[k * 16 + n];
          if (bc != 0.0f) er = __dadd_rn(er, __dmul_rn((double)bc, (double)re[k]));
          if (bs != 0.0f) ei = __dadd_rn(ei, __dmul_rn((double)bs, (double)im[k]));
        }
        out[n] = __fmul_rn(__fadd_rn((float)er, (float)ei), c_win[n]);
      }
    } else {
#pragma unroll
      for (int n = 0; n < 16; ++n) out[n] = 0.0f;
    }
#pragma unroll
    for (int n = 0; n < 16; ++n) fr[b][fl][n] = out[n];
  }
  __syncthreads();

  // ---- 2. overlap-add / window-sum envelope, trimmed [8:-8]
  const int NM = (int)(m_hi - m_lo + 1);
  for (int it = threadIdx.x; it < 4 * NM; it += blockDim.x) {
    const int b = it / NM, ml = it - b * NM;
    const long long p = m_lo + ml + 8;
    const long long q = p >> 2;
    const int r = (int)(p & 3);
    float ola = 0.0f, env = 0.0f;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const long long qq = q - t;
      if (qq >= 0 && qq < Tp) {
        ola = __fadd_rn(ola, fr[b][qq - F0][r + 4 * t]);
        env = __fadd_rn(env, c_win2[r + 4 * t]);
      }
    }
    const float ec = env > 1e-9f ? env : 1e-9f;
    sm[b][ml] = __fdiv_rn(ola, ec);
  }
  __syncthreads();

  // ---- 3. x4 zero-stuff (gain 4) + 63-tap PQMF synthesis, tap-major then band (conv order)
  float *wav = a.wav + (a.wav0 ? a.wav0[req] : 0);
  for (int jj = threadIdx.x; jj < kTailW; jj += blockDim.x) {
    const long long j = j0 + jj;
    if (j >= nwav) break;
    float acc = 0.0f;
    const int k0 = (int)((31 - j) & 3);  // first tap with (j + k - 31) % 4 == 0
    for (int k = k0; k < 63; k += 4) {
      const long long i = j + k - 31;
      if (i < 0 || i >= nwav) continue;
      const int ml = (int)((i >> 2) - m_lo);
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const float x = __fmul_rn(4.0f, sm[b][ml]);
        if (x == 0.0f) continue;
        acc = __fadd_rn(acc, __fmul_rn(h[b][k], x));
      }
    }
    wav[j] = acc;
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
    PTB_REQUIRE(!g_tail_err, "pt_b200: tail constant upload failed");
    done[dev] = true;
  }
  return 0;
}

// single request, channel-major post [72][Tp]
int tail_run(const float *post_dev, int64_t Tp, const float *pqmf_dev, float *wav_dev,
             cudaStream_t st) {
  if (tail_ready()) return -1;
  TailArgs a{};
  a.post = post_dev;
  a.st_t = 1;
  a.st_c = Tp;
  a.tp1 = Tp;
  a.pqmf = pqmf_dev;
  a.wav = wav_dev;
  const long long nwav = 16 * (Tp - 1);
  dim3 grid((unsigned)((nwav + kTailW - 1) / kTailW), 1);
  tail_kernel<<<grid, kTailThreads, 0, st>>>(a);
  PTB_CUDA(cudaGetLastError());
  count_launch();
  return 0;
}

// batched requests, channels-last post rows (ld = row stride); per-request tables on the device
int tail_run_rows(const float *post_dev, long long ld, const long long *row0, const long long *tp,
                  const long long *wav0, int nreq, long long max_tp, const float *pqmf_dev,
                  float *wav_dev, cudaStream_t st) {
  if (tail_ready()) return -1;
  TailArgs a{};
  a.post = post_dev;
  a.st_t = ld;
  a.st_c = 1;
  a.row0 = row0;
  a.tp = tp;
  a.wav0 = wav0;
  a.pqmf = pqmf_dev;
  a.wav = wav_dev;
  const long long nwav = 16 * (max_tp - 1);
  dim3 grid((unsigned)((nwav + kTailW - 1) / kTailW), (unsigned)nreq);
  tail_kernel<<<grid, kTailThreads, 0, st>>>(a);
  PTB_CUDA(cudaGetLastError());
  count_launch();
  return 0;
}

}  // namespace ptb
