// conv_tc.cu -- instances of the tensor-core conv kernel, TMA map encoding, error plumbing.
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "common.cuh"

namespace ptb {

static thread_local char g_err[1024];
static thread_local long g_launches;

void set_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  fprintf(stderr, "%s\n", g_err);
}
const char *last_error() { return g_err; }
void count_launch(long n) { g_launches += n; }
long launches(int reset) {
  const long v = g_launches;
  if (reset) g_launches = 0;
  return v;
}

// ---------------------------------------------------------------------------- tensor maps
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

static int encoder(PFN_cuTensorMapEncodeTiled_v12000 *fn) {
  std::call_once(g_encode_once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  PTB_REQUIRE(g_encode, "pt_b200: cuTensorMapEncodeTiled unavailable from the driver");
  *fn = g_encode;
  return 0;
}

int make_map_act(CUtensorMap *m, const float *base, int cin32, int64_t rows, int batch) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  if (encoder(&enc)) return -1;
  PTB_REQUIRE((reinterpret_cast<uintptr_t>(base) & 15) == 0 && cin32 % kBK == 0 && rows > 0 &&
                  batch > 0,
              "pt_b200: activation map needs a 16-byte aligned base and 32-channel rows");
  cuuint64_t dims[3] = {(cuuint64_t)cin32, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)cin32 * 4, (cuuint64_t)cin32 * 4 * (cuuint64_t)rows};
  cuuint32_t box[3] = {(cuuint32_t)kBK, (cuuint32_t)kBM, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(base), dims, strides,
                   box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  PTB_REQUIRE(r == CUDA_SUCCESS, "pt_b200: activation tensor map encode failed (%d)", (int)r);
  return 0;
}

int make_map_w(CUtensorMap *m, const float *base, int64_t krow, int64_t nrows, int box_n) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  if (encoder(&enc)) return -1;
  PTB_REQUIRE((reinterpret_cast<uintptr_t>(base) & 15) == 0 && krow % kBK == 0 && box_n <= 256,
              "pt_b200: weight map needs a 16-byte aligned base and 32-element rows");
  cuuint64_t dims[2] = {(cuuint64_t)krow, (cuuint64_t)nrows};
  cuuint64_t strides[1] = {(cuuint64_t)krow * 4};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_n};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides,
                   box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  PTB_REQUIRE(r == CUDA_SUCCESS, "pt_b200: weight tensor map encode failed (%d)", (int)r);
  return 0;
}

// ---------------------------------------------------------------------------- instances
// N tiles compiled: the decoder needs 256 (256/512-channel layers, upsamplers), 128 (128-channel
// layers) and 80 (conv_post, 72 channels); 16/32/64 serve the small tail convs and generic calls.
template <int BN>
struct StagesFor {
  static constexpr int value = BN >= 256 ? 4 : BN >= 128 ? 6 : 8;
};

template <int BN>
static int launch_bn(const ConvLaunch &L, uint32_t *gerr, cudaStream_t st) {
  constexpr int S = StagesFor<BN>::value;
  constexpr int smem = ConvSmem<BN, S>::kBytes;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(conv_tc_kernel<BN, S>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  });
  PTB_CUDA(attr_err);
  CUtensorMap ta, tb;
  if (make_map_act(&ta, L.act, L.g.cin32, L.act_rows, L.batch)) return -1;
  if (make_map_w(&tb, L.w, (int64_t)L.g.ntap * L.g.cin32, L.g.n_cols, BN)) return -1;
  dim3 grid((unsigned)((L.g.m_rows + kBM - 1) / kBM), (unsigned)(L.g.n_cols / BN),
            (unsigned)L.batch);
  conv_tc_kernel<BN, S><<<grid, kThreads, smem, st>>>(ta, tb, L.g, L.e, gerr);
  PTB_CUDA(cudaGetLastError());
  count_launch();
  return 0;
}

static const int kTiles[] = {16, 32, 64, 80, 128, 256};

int pick_bn(int ncols, int *bn, int *n_pad) {
  PTB_REQUIRE(ncols > 0, "pt_b200: empty N extent");
  const int n16 = (int)round_up(ncols, 16);
  for (int t : kTiles)
    if (t >= n16) {
      *bn = t;
      *n_pad = t;
      return 0;
    }
  *bn = 256;
  *n_pad = (int)round_up(ncols, 256);
  return 0;
}

int launch_conv(const ConvLaunch &L, uint32_t *gerr, cudaStream_t st) {
  PTB_REQUIRE(L.g.m_rows > 0 && L.g.nkb > 0 && L.g.n_cols % L.bn == 0,
              "pt_b200: bad conv geometry (m=%d nkb=%d n=%d bn=%d)", L.g.m_rows, L.g.nkb,
              L.g.n_cols, L.bn);
  switch (L.bn) {
    case 16: return launch_bn<16>(L, gerr, st);
    case 32: return launch_bn<32>(L, gerr, st);
    case 64: return launch_bn<64>(L, gerr, st);
    case 80: return launch_bn<80>(L, gerr, st);
    case 128: return launch_bn<128>(L, gerr, st);
    case 256: return launch_bn<256>(L, gerr, st);
    default: set_error("pt_b200: no conv instance for N tile %d", L.bn); return -1;
  }
}

}  // namespace ptb
