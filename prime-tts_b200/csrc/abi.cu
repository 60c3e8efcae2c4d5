// abi.cu -- the pt_v21_* C ABI (runtime/v21/src/pt_v21.h:208-259) on the tensor-core kernels.
//
// Per-context state hangs off pt_ctx::g_weights (a field the reference's CUDA layer owns and
// never uses); the stream and the bump arena use the reference's own fields (g_stream, g_arena,
// g_arena_bytes, g_arena_used) with the reference's mark/release discipline, so the interpreter's
// chain protocol (conv_keep / conv_in_dev / conv_out_dev / chain_mark) works unchanged.
#include <sched.h>
#include <time.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "../../include/pt_b200.h"
#include "common.cuh"

namespace ptb {
long launches(int reset);
int tail_run(const float *post_dev, int64_t Tp, const float *pqmf_dev, float *wav_dev,
             cudaStream_t st);
}  // namespace ptb

using namespace ptb;

namespace {

constexpr int kMaxDev = 64;

struct WEntry {
  float *w = nullptr;     // [n_pad][ntap][cin32], tf32
  float *bias = nullptr;  // [round_up(n_pad, 32)], zero padded
  int n_pad = 0, bn = 0, cin32 = 0, ntap = 0, rows4 = 0, cin = 0;
  const void *host = nullptr;
  size_t bytes = 0;
};

struct DevWeights {
  std::mutex mu;
  std::unordered_map<uint64_t, WEntry> map;
  size_t bytes = 0;
};
DevWeights g_dw[kMaxDev];
int g_active = 0;

struct Ctx {
  int device = 0;
  uint32_t *gerr = nullptr;       // device error word of this context
  uint32_t *gerr_host = nullptr;  // pinned mirror
  std::vector<void *> dev_blocks; // pt_v21_dev_alloc / dev_upload blocks
};

Ctx *ctx_of(pt_ctx *c) {
  if (!c || !c->use_cuda || !c->g_weights) {
    set_error("pt_b200: context is not initialised for the GPU (call pt_v21_cuda_init first); "
              "this library has no CPU path");
    return nullptr;
  }
  return static_cast<Ctx *>(c->g_weights);
}

double now_s() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

double wait_limit_s() {
  static double v = -1.0;
  if (v < 0) v = getenv("PT_B200_WAIT_S") ? atof(getenv("PT_B200_WAIT_S")) : 120.0;
  return v;
}

}  // namespace

// Poll the stream with a deadline (the reference's pt_wait, runtime/v21/src/pt_v21_cuda.cu:30-57,
// plus a limit): a stream that does not finish in time is reported, not waited on forever.
int ptb::wait_stream(cudaStream_t s) {
  const double t0 = now_s(), lim = wait_limit_s();
  for (unsigned it = 0;; ++it) {
    const cudaError_t e = cudaStreamQuery(s);
    if (e == cudaSuccess) return 0;
    if (e != cudaErrorNotReady) {
      set_error("pt_b200 cuda: %s while waiting for the stream", cudaGetErrorString(e));
      return -1;
    }
    if ((it & 63) == 0 && now_s() - t0 > lim) {
      set_error("pt_b200: stream did not finish within %.0f s", lim);
      return -1;
    }
    sched_yield();
  }
}

namespace {

// After a sync: report kernel-side errors (bounded waits that gave up, rejected arguments).
int check_gerr(Ctx *x) {
  if (*x->gerr_host) {
    set_error("pt_b200: device error word 0x%x (a bounded wait gave up or a kernel rejected its "
              "arguments)", *x->gerr_host);
    *x->gerr_host = 0;
    cudaMemset(x->gerr, 0, 4);
    return -1;
  }
  return 0;
}

// ---- arena: the reference's bump allocator with mark / release (pt_v21_cuda.cu:491-515)
void *arena_alloc(pt_ctx *c, size_t bytes) {
  const size_t off = (c->g_arena_used + 255) & ~(size_t)255;
  if (off + bytes > c->g_arena_bytes) return nullptr;
  c->g_arena_used = off + bytes;
  if (c->g_arena_used > c->arena_alloc_bytes) c->arena_alloc_bytes = c->g_arena_used;
  return static_cast<char *>(c->g_arena) + off;
}
void *arena_mark(pt_ctx *c) { return static_cast<char *>(c->g_arena) + c->g_arena_used; }
void arena_release(pt_ctx *c, void *mark) {
  c->g_arena_used = (size_t)(static_cast<char *>(mark) - static_cast<char *>(c->g_arena));
}

// Scratch from the arena, or an owned cudaMalloc when the arena is full (still correct).
struct Scratch {
  std::vector<void *> owned;
  ~Scratch() {
    for (void *p : owned) cudaFree(p);
  }
  void *get(pt_ctx *c, size_t bytes, bool *stray = nullptr) {
    void *p = arena_alloc(c, bytes);
    if (p) return p;
    if (cudaMalloc(&p, bytes ? bytes : 256) != cudaSuccess) return nullptr;
    owned.push_back(p);
    c->dev_bytes_stray += (double)bytes;
    if (stray) *stray = true;
    return p;
  }
};

enum WKind : uint64_t { WK_CONV = 1, WK_CONVT = 2 };

// Device copy of packed weights (+ bias) in the kernel's layout.  With wtab >= 0 it is made once
// per (device, record) and shared by every context on that device (the reference's one-time
// pooled upload, pt_v21_cuda.cu:96-235); wtab < 0 gives a per-call copy owned by `tmp`.
int weights_get(Ctx *x, cudaStream_t st, uint64_t kind, int wtab, int btab, const float *wp,
                const float *bias, int rows4, int ntap, int cin, int cout, int cphase,
                WEntry *out, Scratch *tmp, pt_ctx *c) {
  const uint64_t key = (kind << 56) ^ ((uint64_t)(uint32_t)wtab << 24) ^ (uint64_t)(uint32_t)(btab + 1);
  DevWeights &dw = g_dw[x->device];
  std::unique_lock<std::mutex> lk(dw.mu, std::defer_lock);
  if (wtab >= 0) {
    lk.lock();
    auto it = dw.map.find(key);
    if (it != dw.map.end()) {
      const WEntry &e = it->second;
      if (e.rows4 == rows4 && e.ntap == ntap && e.cin == cin) {
        *out = e;
        return 0;
      }
    }
  }
  WEntry e;
  e.rows4 = rows4;
  e.ntap = ntap;
  e.cin = cin;
  e.cin32 = (int)round_up(cin, kBK);
  if (pick_bn(rows4, &e.bn, &e.n_pad)) return -1;
  const size_t wbytes = (size_t)e.n_pad * ntap * e.cin32 * 4;
  const size_t bbytes = (size_t)round_up(e.n_pad, 32) * 4;
  const size_t pbytes = (size_t)rows4 * ntap * cin * 4;
  float *dpacked = nullptr;
  if (wtab >= 0) {
    PTB_CUDA(cudaMalloc(&e.w, wbytes));
    PTB_CUDA(cudaMalloc(&e.bias, bbytes));
  } else {
    e.w = static_cast<float *>(tmp->get(c, wbytes));
    e.bias = static_cast<float *>(tmp->get(c, bbytes));
    PTB_REQUIRE(e.w && e.bias, "pt_b200: out of device memory for per-call weights");
  }
  PTB_CUDA(cudaMalloc(&dpacked, pbytes));
  PTB_CUDA(cudaMemcpyAsync(dpacked, wp, pbytes, cudaMemcpyHostToDevice, st));
  int r = stage_packed_w(dpacked, rows4, ntap, cin, e.w, e.n_pad, e.cin32, st);
  std::vector<float> hb((size_t)round_up(e.n_pad, 32), 0.0f);
  if (bias)
    for (int n = 0; n < rows4; ++n) {
      const int co = n % cphase;
      if (co < cout) hb[n] = bias[co];
    }
  if (!r) r = cudaMemcpyAsync(e.bias, hb.data(), bbytes, cudaMemcpyHostToDevice, st) == cudaSuccess ? 0 : -1;
  const cudaError_t se = cudaStreamSynchronize(st);
  cudaFree(dpacked);
  PTB_REQUIRE(!r && se == cudaSuccess, "pt_b200: weight upload failed (%s)", cudaGetErrorString(se));
  e.host = wp;
  e.bytes = wbytes + bbytes;
  if (wtab >= 0) {
    dw.map[key] = e;
    dw.bytes += e.bytes;
  }
  *out = e;
  return 0;
}

int finish_sync(Ctx *x, cudaStream_t st) {
  if (cudaMemcpyAsync(x->gerr_host, x->gerr, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess) {
    set_error("pt_b200: error-word copy failed");
    return -1;
  }
  if (wait_stream(st)) return -1;
  return check_gerr(x);
}

}  // namespace

// =============================================================================== C ABI
extern "C" {

const char *pt_b200_last_error(void) { return last_error(); }
long pt_b200_kernel_launches(int reset) { return launches(reset); }

int pt_v21_cuda_prewarm(void) {
  const char *e = getenv("PT_V21_DEVICE");
  const int dev = e ? atoi(e) : 0;
  if (cudaSetDevice(dev) != cudaSuccess || cudaFree(0) != cudaSuccess) {
    cudaGetLastError();
    return 0;  // the reference's prewarm never fails the caller either
  }
  return 0;
}

int pt_v21_cuda_init_dev(pt_ctx *c, int device, int verbose) {
  PTB_REQUIRE(c, "pt_b200: NULL context");
  PTB_REQUIRE(device >= 0 && device < kMaxDev, "pt_b200: device %d out of range", device);
  PTB_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop;
  PTB_CUDA(cudaGetDeviceProperties(&prop, device));
  PTB_REQUIRE(prop.major == 10 && prop.minor == 0,
              "pt_b200: device %d is sm_%d%d; this library is built for sm_100a (B200) only",
              device, prop.major, prop.minor);
  Ctx *x = new Ctx();
  x->device = device;
  cudaStream_t st;
  PTB_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  PTB_CUDA(cudaMalloc(&x->gerr, 4));
  PTB_CUDA(cudaMemset(x->gerr, 0, 4));
  PTB_CUDA(cudaMallocHost(&x->gerr_host, 4));
  *x->gerr_host = 0;
  const size_t mb = getenv("PT_V21_ARENA_MB") ? (size_t)atol(getenv("PT_V21_ARENA_MB")) : 64u;
  void *arena = nullptr;
  PTB_CUDA(cudaMalloc(&arena, mb << 20));
  c->g_weights = x;
  c->g_stream = st;
  c->g_arena = arena;
  c->g_arena_bytes = mb << 20;
  c->g_arena_used = 0;
  c->dev_bytes_arena = (double)(mb << 20);
  c->conv_in_dev = nullptr;
  c->conv_out_dev = nullptr;
  c->chain_mark = nullptr;
  c->use_cuda = 1;
  __sync_add_and_fetch(&g_active, 1);
  if (verbose)
    fprintf(stderr, "pt_b200: device %d (%s, %d SMs), %zu MiB arena\n", device, prop.name,
            prop.multiProcessorCount, mb);
  return 0;
}

int pt_v21_cuda_init(pt_ctx *c, int verbose) {
  const char *e = getenv("PT_V21_DEVICE");
  return pt_v21_cuda_init_dev(c, e ? atoi(e) : 0, verbose);
}

void pt_v21_cuda_shutdown(pt_ctx *c) {
  if (!c || !c->g_weights) return;
  Ctx *x = static_cast<Ctx *>(c->g_weights);
  cudaSetDevice(x->device);
  if (c->g_stream) {
    cudaStreamSynchronize((cudaStream_t)c->g_stream);
    cudaStreamDestroy((cudaStream_t)c->g_stream);
  }
  for (void *p : x->dev_blocks) cudaFree(p);
  if (c->g_arena) cudaFree(c->g_arena);
  cudaFree(x->gerr);
  cudaFreeHost(x->gerr_host);
  delete x;
  c->g_weights = nullptr;
  c->g_stream = nullptr;
  c->g_arena = nullptr;
  c->g_arena_bytes = c->g_arena_used = 0;
  c->use_cuda = 0;
  __sync_sub_and_fetch(&g_active, 1);
}

int pt_v21_conv_pads_in_kernel(pt_ctx *c) {
  (void)c;
  return 1;
}

int pt_v21_conv(pt_ctx *c, const float *X, int64_t ldx, int64_t cin, float *Y, int64_t ldy,
                int64_t n, int cout, int K, int stride, int pad, int dil, const float *wp,
                const float *bias, int64_t batch, int wtab, int btab, int epi0, int epi1, float a0,
                float a1) {
  (void)ldy;
  Ctx *x = ctx_of(c);
  if (!x) return -1;
  PTB_REQUIRE(stride == 1, "pt_b200: conv stride %d unsupported (the v2.1 graph only uses 1)", stride);
  PTB_REQUIRE(cin > 0 && cout > 0 && K > 0 && n > 0 && batch > 0 && ldx > 0 && dil > 0,
              "pt_b200: bad conv arguments");
  PTB_CUDA(cudaSetDevice(x->device));
  cudaStream_t st = (cudaStream_t)c->g_stream;
  c->n_conv++;
  const int cout4 = (cout + 3) / 4 * 4;
  const int64_t Tout = n;
  const int64_t pad_in = c->conv_pad_in >= 0 ? c->conv_pad_in : 0;
  (void)pad;
  void *mark = arena_mark(c);
  const float *din = c->conv_in_dev;
  const int keep = c->conv_keep;
  c->conv_out_dev = nullptr;
  Scratch tmp;
  bool stray = false;
  WEntry w;
  if (weights_get(x, st, WK_CONV, wtab, btab, wp, bias, cout4, K, (int)cin, cout, 1 << 30, &w,
                  &tmp, c))
    return -1;
  const size_t xb = (size_t)batch * cin * ldx * 4;
  const float *dx = din;
  if (!dx) {
    float *p = static_cast<float *>(tmp.get(c, xb, &stray));
    PTB_REQUIRE(p, "pt_b200: out of device memory (conv input)");
    PTB_CUDA(cudaMemcpyAsync(p, X, xb, cudaMemcpyHostToDevice, st));
    dx = p;
  }
  float *dxc = static_cast<float *>(tmp.get(c, (size_t)batch * ldx * w.cin32 * 4, &stray));
  float *dy = static_cast<float *>(tmp.get(c, (size_t)batch * cout4 * Tout * 4, &stray));
  PTB_REQUIRE(dxc && dy, "pt_b200: out of device memory (conv scratch)");
  if (stage_act(dx, ldx, (int)cin, ldx, (int)batch, dxc, w.cin32, st)) return -1;
  ConvLaunch L{};
  L.act = dxc;
  L.act_rows = ldx;
  L.batch = (int)batch;
  L.w = w.w;
  L.bn = w.bn;
  L.g.m_rows = (int)Tout;
  L.g.n_cols = w.n_pad;
  L.g.cin32 = w.cin32;
  L.g.ntap = K;
  L.g.row_off0 = -(int)pad_in;
  L.g.row_step = dil;
  L.g.nkb = K * (w.cin32 / kBK);
  L.e.mode = EPI_PLAIN_CONV;
  L.e.bias = bias ? w.bias : nullptr;
  L.e.y = dy;
  L.e.ybatch = (long long)cout4 * Tout;
  L.e.ldy = Tout;
  L.e.nstore = cout4;
  L.e.tout = Tout;
  L.e.epi0 = epi0;
  L.e.epi1 = epi1;
  L.e.a0 = a0;
  L.e.a1 = a1;
  if (launch_conv(L, x->gerr, st)) return -1;
  if (keep && !stray && tmp.owned.empty()) {
    // chain link (pt_v21_cuda.cu:1924-1931): the next conv reads dy from the arena
    if (!c->chain_mark) c->chain_mark = mark;
    c->conv_out_dev = dy;
    return 0;
  }
  PTB_CUDA(cudaMemcpyAsync(Y, dy, (size_t)batch * cout4 * Tout * 4, cudaMemcpyDeviceToHost, st));
  const int r = finish_sync(x, st);
  if (c->chain_mark) {
    arena_release(c, c->chain_mark);
    c->chain_mark = nullptr;
  } else {
    arena_release(c, mark);
  }
  return r;
}

static int convT_impl(pt_ctx *c, const float *X, int64_t ldx, int64_t cin, int64_t tin, float *Y,
                      int cout, int s, int pad, int K, const float *wp, const float *bias,
                      int64_t batch, int wtab, int btab, int epi0, float a0) {
  Ctx *x = ctx_of(c);
  if (!x) return -1;
  PTB_REQUIRE(cin > 0 && cout > 0 && K > 0 && s > 0 && tin > 0 && batch > 0 && ldx >= tin,
              "pt_b200: bad convT arguments");
  PTB_CUDA(cudaSetDevice(x->device));
  cudaStream_t st = (cudaStream_t)c->g_stream;
  c->n_convT++;
  const int nt = (K + s - 1) / s;
  const int cout4 = (cout + 3) / 4 * 4;
  const int64_t Lout = (tin - 1) * s - 2 * (int64_t)pad + K;
  PTB_REQUIRE(Lout > 0, "pt_b200: convT output length %lld", (long long)Lout);
  // delay-line steps whose output lands in [0, Lout) for some phase (pt_v21_cuda.cu:2411-2416)
  int64_t qlo = pad - (s - 1) <= 0 ? 0 : (pad - (s - 1) + s - 1) / s;
  const int64_t qhi = (Lout - 1 + pad) / s;
  const int64_t nq = qhi - qlo + 1;
  void *mark = arena_mark(c);
  Scratch tmp;
  WEntry w;
  if (weights_get(x, st, WK_CONVT, wtab, btab, wp, bias, s * cout4, nt, (int)cin, cout, cout4, &w,
                  &tmp, c))
    return -1;
  const size_t xb = (size_t)batch * cin * ldx * 4;
  float *dx = static_cast<float *>(tmp.get(c, xb));
  float *dxc = static_cast<float *>(tmp.get(c, (size_t)batch * tin * w.cin32 * 4));
  float *dy = static_cast<float *>(tmp.get(c, (size_t)batch * cout4 * Lout * 4));
  PTB_REQUIRE(dx && dxc && dy, "pt_b200: out of device memory (convT scratch)");
  PTB_CUDA(cudaMemcpyAsync(dx, X, xb, cudaMemcpyHostToDevice, st));
  if (stage_act(dx, ldx, (int)cin, tin, (int)batch, dxc, w.cin32, st)) return -1;
  ConvLaunch L{};
  L.act = dxc;
  L.act_rows = tin;
  L.batch = (int)batch;
  L.w = w.w;
  L.bn = w.bn;
  L.g.m_rows = (int)nq;
  L.g.n_cols = w.n_pad;
  L.g.cin32 = w.cin32;
  L.g.ntap = nt;
  L.g.row_off0 = (int)qlo;
  L.g.row_step = -1;
  L.g.nkb = nt * (w.cin32 / kBK);
  L.e.mode = EPI_PLAIN_CONVT;
  L.e.bias = bias ? w.bias : nullptr;
  L.e.y = dy;
  L.e.ybatch = (long long)cout4 * Lout;
  L.e.ldy = Lout;
  L.e.nstore = s * cout4;
  L.e.tout = Lout;
  L.e.epi0 = epi0;
  L.e.a0 = a0;
  L.e.s = s;
  L.e.pad = pad;
  L.e.cphase = cout4;
  L.e.q0 = qlo;
  if (launch_conv(L, x->gerr, st)) return -1;
  PTB_CUDA(cudaMemcpyAsync(Y, dy, (size_t)batch * cout4 * Lout * 4, cudaMemcpyDeviceToHost, st));
  const int r = finish_sync(x, st);
  arena_release(c, mark);
  return r;
}

int pt_v21_convT(pt_ctx *c, const float *X, int64_t ldx, int64_t cin, int64_t tin, float *Y,
                 int64_t ldy, int cout, int s, int pad, int K, const float *wp, const float *bias,
                 int64_t batch, int wtab, int btab) {
  (void)ldy;
  return convT_impl(c, X, ldx, cin, tin, Y, cout, s, pad, K, wp, bias, batch, wtab, btab, 0, 0.0f);
}

int pt_v21_convT_epi(pt_ctx *c, const float *X, int64_t ldx, int64_t cin, int64_t tin, float *Y,
                     int64_t ldy, int cout, int s, int pad, int K, const float *wp,
                     const float *bias, int64_t batch, int wtab, int btab, int epi0, float a0) {
  (void)ldy;
  return convT_impl(c, X, ldx, cin, tin, Y, cout, s, pad, K, wp, bias, batch, wtab, btab, epi0, a0);
}

int pt_v21_matmul(pt_ctx *c, const float *A, int64_t m, int64_t k, int64_t lda, const float *B,
                  int64_t ldb, int64_t nn, float *Cm, int64_t ldc) {
  Ctx *x = ctx_of(c);
  if (!x) return -1;
  PTB_REQUIRE(m > 0 && k > 0 && nn > 0 && lda >= k && ldb >= nn && ldc >= nn,
              "pt_b200: bad matmul arguments");
  PTB_CUDA(cudaSetDevice(x->device));
  cudaStream_t st = (cudaStream_t)c->g_stream;
  c->n_matmul++;
  void *mark = arena_mark(c);
  Scratch tmp;
  const int k32 = (int)round_up(k, kBK);
  int bn, n_pad;
  if (pick_bn((int)nn, &bn, &n_pad)) return -1;
  float *dA = static_cast<float *>(tmp.get(c, (size_t)m * lda * 4));
  float *dB = static_cast<float *>(tmp.get(c, (size_t)k * ldb * 4));
  float *dAc = static_cast<float *>(tmp.get(c, (size_t)m * k32 * 4));
  float *dBw = static_cast<float *>(tmp.get(c, (size_t)n_pad * k32 * 4));
  float *dC = static_cast<float *>(tmp.get(c, (size_t)m * nn * 4));
  PTB_REQUIRE(dA && dB && dAc && dBw && dC, "pt_b200: out of device memory (matmul scratch)");
  PTB_CUDA(cudaMemcpyAsync(dA, A, (size_t)m * lda * 4, cudaMemcpyHostToDevice, st));
  PTB_CUDA(cudaMemcpyAsync(dB, B, (size_t)k * ldb * 4, cudaMemcpyHostToDevice, st));
  if (stage_rows(dA, lda, m, (int)k, dAc, k32, st)) return -1;
  if (stage_matmul_b(dB, ldb, (int)k, (int)nn, dBw, n_pad, k32, st)) return -1;
  ConvLaunch L{};
  L.act = dAc;
  L.act_rows = m;
  L.batch = 1;
  L.w = dBw;
  L.bn = bn;
  L.g.m_rows = (int)m;
  L.g.n_cols = n_pad;
  L.g.cin32 = k32;
  L.g.ntap = 1;
  L.g.row_off0 = 0;
  L.g.row_step = 0;
  L.g.nkb = k32 / kBK;
  L.e.mode = EPI_PLAIN_CONV;
  L.e.rowmajor = 1;
  L.e.y = dC;
  L.e.ybatch = 0;
  L.e.ldy = nn;
  L.e.nstore = (int)nn;
  L.e.tout = m;
  if (launch_conv(L, x->gerr, st)) return -1;
  PTB_CUDA(cudaMemcpy2DAsync(Cm, (size_t)ldc * 4, dC, (size_t)nn * 4, (size_t)nn * 4, (size_t)m,
                             cudaMemcpyDeviceToHost, st));
  const int r = finish_sync(x, st);
  arena_release(c, mark);
  return r;
}

// ---- device residency helpers (used by the interpreter only with PT_V21_DEVADD=1)
void *pt_v21_dev_alloc(pt_ctx *c, size_t bytes) {
  if (!c || !c->g_weights) return nullptr;
  Ctx *x = static_cast<Ctx *>(c->g_weights);
  void *p = nullptr;
  if (cudaSetDevice(x->device) != cudaSuccess || cudaMalloc(&p, bytes ? bytes : 256) != cudaSuccess) {
    cudaGetLastError();
    c->devres_oom = 1;
    return nullptr;
  }
  x->dev_blocks.push_back(p);
  c->dev_bytes_res += (double)bytes;
  return p;
}

void pt_v21_dev_free(pt_ctx *c, void *p) {
  if (!c || !c->g_weights || !p) return;
  Ctx *x = static_cast<Ctx *>(c->g_weights);
  for (size_t i = 0; i < x->dev_blocks.size(); ++i)
    if (x->dev_blocks[i] == p) {  // pointers this helper did not hand out are ignored
      cudaStreamSynchronize((cudaStream_t)c->g_stream);
      cudaFree(p);
      x->dev_blocks[i] = x->dev_blocks.back();
      x->dev_blocks.pop_back();
      return;
    }
}

void pt_v21_dev_reclaim(pt_ctx *c) { (void)c; }

float *pt_v21_dev_upload(pt_ctx *c, const void *h, int64_t n) {
  float *d = static_cast<float *>(pt_v21_dev_alloc(c, (size_t)n * 4));
  if (!d) return nullptr;
  if (cudaMemcpyAsync(d, h, (size_t)n * 4, cudaMemcpyHostToDevice, (cudaStream_t)c->g_stream) !=
      cudaSuccess) {
    pt_v21_dev_free(c, d);
    return nullptr;
  }
  return d;
}

void pt_v21_dev_sync_host(pt_ctx *c, void *host, const void *dev, int64_t n) {
  if (!c || !c->g_stream) return;
  cudaStream_t st = (cudaStream_t)c->g_stream;
  if (cudaMemcpyAsync(host, dev, (size_t)n * 4, cudaMemcpyDeviceToHost, st) == cudaSuccess)
    wait_stream(st);
}

int pt_v21_devadd_run(pt_ctx *c, const float *a, const float *b, float *y, int64_t n, int epi,
                      float alpha) {
  Ctx *x = ctx_of(c);
  if (!x) return -1;
  return launch_devadd(a, b, y, n, epi, alpha, (cudaStream_t)c->g_stream);
}

int pt_v21_devleaky_run(pt_ctx *c, const float *a, float *y, int64_t n, float alpha) {
  Ctx *x = ctx_of(c);
  if (!x) return -1;
  return launch_devadd(a, nullptr, y, n, 1, alpha, (cudaStream_t)c->g_stream);
}

void pt_v21_cuda_active(int delta) { (void)delta; }

double pt_v21_cuda_weights_mib(pt_ctx *c) {
  if (!c || !c->g_weights) return 0.0;
  const Ctx *x = static_cast<Ctx *>(c->g_weights);
  return (double)g_dw[x->device].bytes / 1048576.0;
}

int pt_v21_cuda_keepwarm(int iters) {
  (void)iters;
  return 0;
}

long pt_v21_gpu_cur_freq(void) { return -1; }

long pt_v21_gpu_max_freq(void) {
  int dev = 0, khz = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, dev) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  return (long)khz * 1000L;
}

int pt_v21_istft_pqmf(pt_ctx *c, const float *post, int64_t Tp, const float *pqmf, float *wav) {
  Ctx *x = ctx_of(c);
  if (!x) return -1;
  PTB_REQUIRE(post && pqmf && wav && Tp >= 2, "pt_b200: bad tail arguments");
  PTB_CUDA(cudaSetDevice(x->device));
  cudaStream_t st = (cudaStream_t)c->g_stream;
  void *mark = arena_mark(c);
  Scratch tmp;
  const int64_t nwav = 16 * (Tp - 1);
  float *dp = static_cast<float *>(tmp.get(c, (size_t)72 * Tp * 4));
  float *dq = static_cast<float *>(tmp.get(c, 4 * 63 * 4));
  float *dw = static_cast<float *>(tmp.get(c, (size_t)nwav * 4));
  PTB_REQUIRE(dp && dq && dw, "pt_b200: out of device memory (tail scratch)");
  PTB_CUDA(cudaMemcpyAsync(dp, post, (size_t)72 * Tp * 4, cudaMemcpyHostToDevice, st));
  PTB_CUDA(cudaMemcpyAsync(dq, pqmf, 4 * 63 * 4, cudaMemcpyHostToDevice, st));
  if (tail_run(dp, Tp, dq, dw, st)) return -1;
  PTB_CUDA(cudaMemcpyAsync(wav, dw, (size_t)nwav * 4, cudaMemcpyDeviceToHost, st));
  const int r = finish_sync(x, st);
  arena_release(c, mark);
  return r;
}

}  // extern "C"
