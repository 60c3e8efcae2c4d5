// mma_probe.cu -- the tensor core's kind::tf32 rate on this GPU, measured live.
//
// The conv stack's roofline is the rate at which the 5th-generation tensor core retires
// tcgen05.mma kind::tf32 instructions, and that rate is only known by measuring it: one CTA per
// SM issues a long run of M128 x N256 x K8 MMAs whose operands sit in shared memory (written once,
// pseudo-random TF32 values, so the datapath toggles as it does on real data) into one TMEM
// accumulator, and times the run with the SM clock counter and the global timer.  The result is
// FLOP per SM clock (the clock-independent figure) and the aggregate FLOP/s at the clock the run
// held.  No global memory is read in the loop, so the figure is the tensor pipe's alone.
#include <vector>

#include "../../include/pt_b200.h"
#include "common.cuh"

using namespace ptb;

namespace {

constexpr int kProbeM = 128, kProbeN = 256;
constexpr int kProbeA = kProbeM * kBK * 4;   // 16 KiB: A tile, 128 rows x 32 fp32 (K-major)
constexpr int kProbeB = kProbeN * kBK * 4;   // 32 KiB: B tile, 256 rows x 32 fp32
// more dynamic shared memory than two CTAs can share on one SM (228 KB), so every SM runs
// exactly one probe CTA and no two CTAs compete for one tensor pipe
constexpr int kProbeSmem = 120 * 1024;
static_assert(kProbeA + kProbeB + 1024 + 64 <= kProbeSmem, "probe operands exceed its shared memory");
constexpr int kProbeThreads = 128;

__device__ __forceinline__ float probe_value(uint32_t i) {
  uint32_t h = i * 0x9E3779B1u;
  h ^= h >> 15;
  h *= 0x85EBCA77u;
  h ^= h >> 13;
  // a TF32 value in [-1, 1): 10 mantissa bits, exponent of 2^-1 .. 2^0
  const float f = static_cast<float>(static_cast<int32_t>(h >> 1) - (1 << 30)) * (1.0f / (1 << 30));
  return tf32_rna(f);
}

__global__ void __launch_bounds__(kProbeThreads, 1)
    mma_rate_kernel(int iters, unsigned long long *cycles, unsigned long long *nanos,
                    uint32_t *gerr) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t *gbase = smem_raw + (base - raw);
  const uint32_t a0 = base, b0 = base + kProbeA, bar = base + kProbeA + kProbeB;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(gbase + kProbeA + kProbeB + 8);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  // operands: the layout does not matter for the rate, only that the values are varied
  float *ops = reinterpret_cast<float *>(gbase);
  for (int i = threadIdx.x; i < (kProbeA + kProbeB) / 4; i += kProbeThreads)
    ops[i] = probe_value(static_cast<uint32_t>(i + 7919 * blockIdx.x));
  fence_proxy_async_smem();   // generic-proxy writes before the tensor core reads them
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (threadIdx.x < 32) {
    tmem_alloc(smem_u32(tmem_slot), kProbeN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) {
    const uint32_t idesc = idesc_tf32(kProbeM, kProbeN);
    const uint64_t dA = sdesc_kmajor_sw128(a0), dB = sdesc_kmajor_sw128(b0);
    uint64_t g0, g1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g0));
    const long long c0 = clock64();
    for (int it = 0; it < iters; ++it) {
      mma_tf32(tmem, dA, dB, idesc, it > 0 ? 1u : 0u);
      mma_tf32(tmem, dA + 2u, dB + 2u, idesc, 1u);
      mma_tf32(tmem, dA + 4u, dB + 4u, idesc, 1u);
      mma_tf32(tmem, dA + 6u, dB + 6u, idesc, 1u);
    }
    mma_commit(bar);
    const bool ok = mbar_wait(bar, 0, abort_flag, gerr, ERR_WAIT_ACC);
    const long long c1 = clock64();
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g1));
    cycles[blockIdx.x] = ok ? static_cast<unsigned long long>(c1 - c0) : 0ull;
    nanos[blockIdx.x] = ok ? g1 - g0 : 0ull;
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x < 32) {
    tc_fence_after();
    tmem_dealloc(tmem, kProbeN);
  }
}

}  // namespace

extern "C" int pt_b200_mma_rate(int device, int iters, double *flop_per_clk_sm, double *tflops,
                                double *sm_mhz) {
  PTB_REQUIRE(iters > 0 && iters <= (1 << 22) && flop_per_clk_sm && tflops && sm_mhz,
              "pt_b200_mma_rate: bad arguments");
  PTB_CUDA(cudaSetDevice(device));
  int sms = 0;
  PTB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  unsigned long long *buf = nullptr;
  uint32_t *gerr = nullptr;
  PTB_CUDA(cudaMalloc(&buf, (size_t)2 * sms * sizeof(unsigned long long) + 16));
  gerr = reinterpret_cast<uint32_t *>(buf + 2 * sms);
  int rc = -1;
  do {
    if (cudaMemset(buf, 0, (size_t)2 * sms * sizeof(unsigned long long) + 16) != cudaSuccess ||
        cudaFuncSetAttribute(mma_rate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kProbeSmem) != cudaSuccess) {
      set_error("pt_b200_mma_rate: set-up failed");
      break;
    }
    // one CTA per SM (its shared memory keeps a second one off any SM)
    mma_rate_kernel<<<sms, kProbeThreads, kProbeSmem>>>(iters, buf, buf + sms, gerr);
    count_launch();
    if (cudaGetLastError() != cudaSuccess || wait_stream(nullptr)) {
      set_error("pt_b200_mma_rate: probe launch failed");
      break;
    }
    std::vector<unsigned long long> h((size_t)2 * sms);
    uint32_t herr = 0;
    if (cudaMemcpy(h.data(), buf, h.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost) !=
            cudaSuccess ||
        cudaMemcpy(&herr, gerr, 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
      set_error("pt_b200_mma_rate: read-back failed");
      break;
    }
    if (herr) {
      set_error("pt_b200_mma_rate: a bounded wait gave up (error word 0x%x)", herr);
      break;
    }
    const double flop_cta = 4.0 * iters * 2.0 * kProbeM * kProbeN * 8;
    double cyc = 0.0, ns_max = 0.0;
    for (int i = 0; i < sms; ++i) {
      cyc += (double)h[i];
      ns_max = (double)h[sms + i] > ns_max ? (double)h[sms + i] : ns_max;
    }
    cyc /= sms;
    *flop_per_clk_sm = flop_cta / cyc;
    *tflops = flop_cta * sms / (ns_max * 1e-9) / 1e12;
    *sm_mhz = cyc / ns_max * 1e3;
    rc = 0;
  } while (false);
  cudaFree(buf);
  return rc;
}
