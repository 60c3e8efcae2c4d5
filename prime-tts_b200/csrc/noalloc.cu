// noalloc.cu -- pt_b200_conv_noalloc: the tensor-core Conv1d with no device allocation at all.
//
// Who needs it: callers that must not call cudaMalloc / cudaFree -- e.g. a host that owns every
// device allocation itself (a pooled allocator or framework that forbids foreign allocations), a
// real-time audio thread that must never take the allocator's locks, or a process that has to
// keep its device footprint fixed after start-up.  pt_v21_conv needs scratch for the
// channels-last copy of the input and for the re-laid-out weights and pads it from its arena
// (or cudaMalloc when that is full); this entry point takes the same scratch from one fixed
// array compiled into the library instead.
//
// The array is a file-scope __device__ variable, so every GPU that loads the library holds
// kScratchBytes of it until the process exits.  Host code cannot use the variable's name as a
// device address; the entry point asks the runtime for that address (cudaGetSymbolAddress) once
// per device, the first time it runs on that device, with the device made current.
#include <climits>
#include <mutex>

#include "../../include/pt_b200.h"
#include "common.cuh"

using namespace ptb;

namespace {

constexpr size_t kScratchBytes = 16u << 20;   // 16 MiB per device
constexpr size_t kHeader = 256;               // device error word lives here

__device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_addr_mu;
void *g_addr[64];   // device address of g_noalloc_scratch, per device (host-side cache)

__global__ void pad_bias_kernel(const float *__restrict__ bias, int cout, float *__restrict__ dst,
                                int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = (bias && i < cout) ? bias[i] : 0.0f;
}

size_t up256(size_t b) { return (b + 255) & ~(size_t)255; }

}  // namespace

extern "C" int pt_b200_conv_noalloc(int device, void *stream, const float *x, int64_t ldx,
                                    int64_t cin, int64_t T, float *y, int cout, int K, int pad,
                                    int dil, const float *wp, const float *bias, int epi0,
                                    float a0) {
  PTB_REQUIRE(device >= 0 && device < 64, "pt_b200_conv_noalloc: device %d out of range", device);
  PTB_REQUIRE(x && y && wp && cin > 0 && T > 0 && ldx >= T && cout > 0 && K > 0 && dil > 0 &&
                  pad >= 0,
              "pt_b200_conv_noalloc: bad arguments");
  // sizes are checked in 64-bit arithmetic before anything is narrowed to int: whatever does not
  // fit the scratch array is rejected here, which also keeps every later int in range
  const int64_t Tout = T + 2 * (int64_t)pad - (int64_t)(K - 1) * dil;
  PTB_REQUIRE(Tout > 0, "pt_b200_conv_noalloc: empty output (T=%lld K=%d dil=%d pad=%d)",
              (long long)T, K, dil, pad);
  PTB_REQUIRE(cin <= (int64_t)kScratchBytes && T <= (int64_t)kScratchBytes &&
                  Tout <= (int64_t)INT_MAX && cout <= INT_MAX - 3,
              "pt_b200_conv_noalloc: cin=%lld / T=%lld / Tout=%lld exceed the fixed scratch array",
              (long long)cin, (long long)T, (long long)Tout);
  const int64_t cin32l = round_up(cin, kBK);
  const int64_t cout16 = round_up(cout, 16);
  const int64_t need_l = (int64_t)kHeader + (int64_t)up256((size_t)(T * cin32l * 4)) +
                         (int64_t)up256((size_t)(cout16 * K * cin32l * 4));
  PTB_REQUIRE(need_l <= (int64_t)kScratchBytes,
              "pt_b200_conv_noalloc: this conv needs at least %lld bytes of scratch, the fixed "
              "array holds %zu (T x round_up(cin,32) + round_up(cout,16) x K x round_up(cin,32) "
              "floats too large); use pt_v21_conv",
              (long long)need_l, kScratchBytes);
  const int cout4 = (cout + 3) / 4 * 4;
  const int cin32 = (int)cin32l;
  int bn = 0, n_pad = 0;
  if (pick_bn(cout4, &bn, &n_pad)) return -1;
  const size_t xbytes = up256((size_t)T * cin32 * 4);
  const size_t wbytes = up256((size_t)n_pad * K * cin32 * 4);
  const size_t bbytes = up256((size_t)round_up(n_pad, 32) * 4);
  const size_t need = kHeader + xbytes + wbytes + bbytes;
  PTB_REQUIRE(need <= kScratchBytes,
              "pt_b200_conv_noalloc: this conv needs %zu bytes of scratch, the fixed array holds "
              "%zu (T x round_up(cin,32) + round_up(cout,16) x K x round_up(cin,32) floats too "
              "large); use pt_v21_conv",
              need, kScratchBytes);

  int prev = -1;
  PTB_CUDA(cudaGetDevice(&prev));
  if (prev != device) PTB_CUDA(cudaSetDevice(device));
  struct Restore {
    int d;
    ~Restore() {
      if (d >= 0) cudaSetDevice(d);
    }
  } restore{prev != device ? prev : -1};

  void *base = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_addr_mu);
    if (!g_addr[device]) {
      // the device address of the static array on this (current) device
      void *p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      PTB_REQUIRE(e == cudaSuccess && p, "pt_b200_conv_noalloc: cudaGetSymbolAddress failed (%s)",
                  cudaGetErrorString(e));
      g_addr[device] = p;
    }
    base = g_addr[device];
  }
  char *b = static_cast<char *>(base);
  uint32_t *gerr = reinterpret_cast<uint32_t *>(b);
  float *xcl = reinterpret_cast<float *>(b + kHeader);
  float *w = reinterpret_cast<float *>(b + kHeader + xbytes);
  float *bpad = reinterpret_cast<float *>(b + kHeader + xbytes + wbytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // The array keeps the previous call's contents: the error word is the only thing that must
  // start at zero; every staged element the conv reads is rewritten below.
  PTB_CUDA(cudaMemsetAsync(gerr, 0, 4, st));
  if (stage_act(x, ldx, (int)cin, T, 1, xcl, cin32, st)) return -1;
  if (stage_packed_w(wp, cout4, K, (int)cin, w, n_pad, cin32, st)) return -1;
  const int nb = (int)round_up(n_pad, 32);
  pad_bias_kernel<<<(nb + 127) / 128, 128, 0, st>>>(bias, cout, bpad, nb);
  PTB_CUDA(cudaGetLastError());
  count_launch();

  ConvLaunch L{};
  L.act = xcl;
  L.act_rows = T;
  L.batch = 1;
  L.w = w;
  L.bn = bn;
  L.g.m_rows = (int)Tout;
  L.g.n_cols = n_pad;
  L.g.cin32 = cin32;
  L.g.ntap = K;
  L.g.row_off0 = -pad;
  L.g.row_step = dil;
  L.g.nkb = K * (cin32 / kBK);
  L.e.mode = EPI_PLAIN_CONV;
  L.e.bias = bias ? bpad : nullptr;
  L.e.y = y;
  L.e.ybatch = (long long)cout4 * Tout;
  L.e.ldy = Tout;
  L.e.nstore = cout4;
  L.e.tout = Tout;
  L.e.epi0 = epi0;
  L.e.a0 = a0;
  if (launch_conv(L, gerr, st)) return -1;

  // synchronous: the error word is read back once the stream has finished (a bounded wait, like
  // every other host wait of this library)
  uint32_t herr = 0;
  PTB_CUDA(cudaMemcpyAsync(&herr, gerr, 4, cudaMemcpyDeviceToHost, st));
  if (wait_stream(st)) return -1;
  PTB_REQUIRE(herr == 0, "pt_b200_conv_noalloc: device error word 0x%x", herr);
  return 0;
}
