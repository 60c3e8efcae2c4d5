// conv_tc.cu -- instances of the tensor-core conv kernel, TMA map encoding, error plumbing.
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <set>
#include <utility>

#define PTB_CONV_KERNELS
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

int make_map_act(CUtensorMap *m, const float *base, int cin32, int64_t rows, int batch,
                 int box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  if (encoder(&enc)) return -1;
  PTB_REQUIRE((reinterpret_cast<uintptr_t>(base) & 15) == 0 && cin32 % kBK == 0 && rows > 0 &&
                  batch > 0,
              "pt_b200: activation map needs a 16-byte aligned base and 32-channel rows");
  cuuint64_t dims[3] = {(cuuint64_t)cin32, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)cin32 * 4, (cuuint64_t)cin32 * 4 * (cuuint64_t)rows};
  cuuint32_t box[3] = {(cuuint32_t)kBK, (cuuint32_t)box_rows, 1};
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

// Output map of a rows-mode epilogue: [rows][ld] fp32, tiles of 16 rows x 32 channels, no swizzle
// (the staging tile is row-major, 128 bytes a row).
int make_map_out(CUtensorMap *m, const float *base, int ld, int64_t rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  if (encoder(&enc)) return -1;
  PTB_REQUIRE(base && (reinterpret_cast<uintptr_t>(base) & 15) == 0 && ld % 4 == 0 && rows > 0,
              "pt_b200: output map needs a 16-byte aligned base and rows of 4k floats");
  cuuint64_t dims[2] = {(cuuint64_t)ld, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {(cuuint32_t)kBK, 16};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides,
                   box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  PTB_REQUIRE(r == CUDA_SUCCESS, "pt_b200: output tensor map encode failed (%d)", (int)r);
  return 0;
}

// Output map of conv_post's frames epilogue: [rows][ld] fp32, the frame's 64 samples in two boxes
// of 32 floats (128 bytes) x box_rows rows, 128-byte swizzle (the staging layout).
static int make_map_frames(CUtensorMap *m, const float *base, int ld, int64_t rows, int box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  if (encoder(&enc)) return -1;
  PTB_REQUIRE(base && (reinterpret_cast<uintptr_t>(base) & 15) == 0 && ld % 4 == 0 && ld >= 64 &&
                  rows > 0,
              "pt_b200: frames map needs a 16-byte aligned base and rows of at least 64 floats");
  cuuint64_t dims[2] = {(cuuint64_t)ld, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides,
                   box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  PTB_REQUIRE(r == CUDA_SUCCESS, "pt_b200: frames tensor map encode failed (%d)", (int)r);
  return 0;
}

// Output map of the upsampler epilogue: [rows][ld] fp32 viewed as (ld, 4, rows / 4), so that
// rows 4q + p for 16 consecutive q (one phase p) are one 32-channel x 1 x 16 box.
static int make_map_out_convt(CUtensorMap *m, const float *base, int ld, int64_t rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  if (encoder(&enc)) return -1;
  PTB_REQUIRE(base && (reinterpret_cast<uintptr_t>(base) & 15) == 0 && ld % kBK == 0 && rows > 0 &&
                  rows % 4 == 0,
              "pt_b200: upsampler output map needs a 16-byte aligned base, 32-channel rows and "
              "a multiple of 4 rows");
  cuuint64_t dims[3] = {(cuuint64_t)ld, 4, (cuuint64_t)(rows / 4)};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 4, (cuuint64_t)ld * 16};
  cuuint32_t box[3] = {(cuuint32_t)kBK, 1, 16};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(base), dims, strides,
                   box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  PTB_REQUIRE(r == CUDA_SUCCESS, "pt_b200: upsampler output map encode failed (%d)", (int)r);
  return 0;
}

// ---------------------------------------------------------------------------- instances
// N tiles compiled: the decoder needs 256 (256/512-channel layers, upsamplers), 128 (128-channel
// layers) and 80 (conv_post, 72 channels); 16/32/64 serve the small tail convs and generic calls.
template <int BN>
struct StagesFor {
  static constexpr int value = BN >= 256 ? 4 : BN >= 128 ? 6 : 8;
};

// A kernel's opt-in to more than 48 KB of dynamic shared memory belongs to the device it was
// made on: make it once per (kernel, device), on the calling thread's current device.
static int smem_optin(const void *kernel, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void *, int>> done;
  int dev = 0;
  PTB_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(mu);
  if (done.count({kernel, dev})) return 0;
  PTB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done.insert({kernel, dev});
  return 0;
}

template <int BN>
static int launch_bn(const ConvLaunch &L, uint32_t *gerr, cudaStream_t st) {
  constexpr int S = StagesFor<BN>::value;
  constexpr int smem = ConvSmem<BN, S>::kBytes;
  if (smem_optin(reinterpret_cast<const void *>(conv_tc_kernel<BN, S>), smem)) return -1;
  CUtensorMap ta, tb;
  if (make_map_act(&ta, L.act, L.g.cin32, L.act_rows, L.batch, kBM)) return -1;
  if (make_map_w(&tb, L.w, (int64_t)L.g.ntap * L.g.cin32, L.g.n_cols, BN)) return -1;
  dim3 grid((unsigned)((L.g.m_rows + kBM - 1) / kBM), (unsigned)(L.g.n_cols / BN),
            (unsigned)L.batch);
  conv_tc_kernel<BN, S><<<grid, kThreads, smem, st>>>(ta, tb, L.g, L.e, gerr);
  PTB_CUDA(cudaGetLastError());
  count_launch();
  return 0;
}

template <int BN, int MSUB>
static int launch_win(const ConvLaunch &L, uint32_t *gerr, cudaStream_t st) {
  using W = WinCfg<BN, MSUB>;
  if (smem_optin(reinterpret_cast<const void *>(conv_tc_win_kernel<BN, MSUB>), W::kBytes))
    return -1;
  CUtensorMap ta, tb;
  if (make_map_act(&ta, L.act, L.g.cin32, L.act_rows, L.batch, kWinBox)) return -1;
  if (make_map_w(&tb, L.w, (int64_t)L.g.ntap * L.g.cin32, L.g.n_cols, BN)) return -1;
  dim3 grid((unsigned)((L.g.m_rows + MSUB * kBM - 1) / (MSUB * kBM)), (unsigned)(L.g.n_cols / BN),
            (unsigned)L.batch);
  conv_tc_win_kernel<BN, MSUB><<<grid, kThreads, W::kBytes, st>>>(ta, tb, L.g, L.e, gerr);
  PTB_CUDA(cudaGetLastError());
  count_launch();
  return 0;
}

template <int MODE, int F>
static int launch_tn_mode(const ConvLaunch &L, uint32_t *gerr, cudaStream_t st) {
  if (smem_optin(reinterpret_cast<const void *>(conv_tc_tn_kernel<MODE, F>), TNCfg<F>::kBytes))
    return -1;
  int dev = 0;
  PTB_CUDA(cudaGetDevice(&dev));
  static int sms = 0;
  if (!sms) {
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  CUtensorMap tx, tw, to0, to1;
  std::memset(&to0, 0, sizeof(to0));
  std::memset(&to1, 0, sizeof(to1));
  if (make_map_act(&tx, L.act, L.g.cin32, L.act_rows, L.batch, kWinBox)) return -1;
  if (make_map_w(&tw, L.w, (int64_t)L.g.ntap * L.g.cin32, L.g.n_cols, kBM)) return -1;
  if constexpr (TNCfg<F>::kFrames) {
    PTB_REQUIRE(L.g.n_cols == 128 && L.e.nstore >= 72, "pt_b200: the frames epilogue is conv_post's");
    if (make_map_frames(&to0, L.e.out0, L.e.ldc, L.g.m_rows, 32) ||
        make_map_frames(&to1, L.e.out0, L.e.ldc, L.g.m_rows, 16))
      return -1;
  } else if constexpr (TNTmaStore<MODE, F>::value) {
    if ((F & EF_OUT0) && make_map_out(&to0, L.e.out0, L.e.ldc, L.g.m_rows)) return -1;
    if ((F & EF_OUT1) && make_map_out(&to1, L.e.out1, L.e.ldc1, L.g.m_rows)) return -1;
  }
  if constexpr (TNConvTStore<MODE, F>::value) {
    if (make_map_out_convt(&to0, L.e.out0, L.e.ldc, L.e.out_rows) ||
        make_map_out_convt(&to1, L.e.out1, L.e.ldc1, L.e.out_rows))
      return -1;
  }
  PTB_REQUIRE(!L.g.tiles || (L.batch == 1 && L.g.ntiles > 0),
              "pt_b200: a conv tile list needs batch 1 and at least one tile");
  ConvGeom g = L.g;
  const long long mtl = (L.g.n_cols + kBM - 1) / kBM;
  g.tile_rows = kTNRows;
  // three activation windows for kernel-3 convs (a window lasts three taps), else two windows
  // and a third weight stage; residual instances always run two windows
  g.win_slots = TNCfg<F>::kRes || L.g.ntap > 3 ? 2 : 3;
  if (!L.g.tiles) {
    // The tile height whose last wave is fullest: waves x (rows + a per-tile cost of 16 rows,
    // the weight stream and pipeline fill) over heights 256 .. 160.
    long long best = -1;
    for (int h = kTNRows; h >= 160; h -= 16) {
      const long long n = mtl * ((L.g.m_rows + h - 1) / h) * L.batch;
      const long long cost = ((n + sms - 1) / sms) * (h + 16);
      if (best < 0 || cost < best) {
        best = cost;
        g.tile_rows = h;
      }
    }
  }
  const long long tiles =
      mtl * (L.g.tiles ? L.g.ntiles : ((L.g.m_rows + g.tile_rows - 1) / g.tile_rows) * L.batch);
  g.nbatch = L.batch;
  const unsigned grid = (unsigned)(tiles < sms ? tiles : sms);
  conv_tc_tn_kernel<MODE, F><<<grid, TNCfg<F>::kThreads, TNCfg<F>::kBytes, st>>>(tx, tw, to0, to1, g, L.e, gerr);
  PTB_CUDA(cudaGetLastError());
  count_launch();
  return 0;
}

// The decoder's epilogue combinations get their own instances; anything else runs the generic
// instance, which reads the same choices from EpiParams at run time.
static int launch_tn(const ConvLaunch &L, uint32_t *gerr, cudaStream_t st) {
  const EpiParams &e = L.e;
  if (e.mode == EPI_PLAIN_CONV) return launch_tn_mode<EPI_PLAIN_CONV, 0>(L, gerr, st);
  if (e.mode == EPI_PLAIN_CONVT) return launch_tn_mode<EPI_PLAIN_CONVT, 0>(L, gerr, st);
  const int f = (e.res ? EF_RES : 0) | (e.acc_mode == 2 ? EF_ACC2 : 0) |
                (e.acc_mode == 3 ? EF_ACC3 : 0) | (e.out0 ? EF_OUT0 : 0) |
                (e.out1 ? EF_OUT1 : 0) | (e.refl ? EF_REFL : 0) | (e.frames ? EF_FRAMES : 0);
  if (e.mode == EPI_ROWS_CONVT) {
    if (f == (EF_OUT0 | EF_OUT1)) return launch_tn_mode<EPI_ROWS_CONVT, EF_OUT0 | EF_OUT1>(L, gerr, st);
    return launch_tn_mode<EPI_ROWS_CONVT, EF_GENERIC>(L, gerr, st);
  }
  if (e.mode != EPI_ROWS) {
    set_error("pt_b200: unknown epilogue mode %d", e.mode);
    return -1;
  }
  switch (f) {
    case EF_OUT1: return launch_tn_mode<EPI_ROWS, EF_OUT1>(L, gerr, st);
    case EF_OUT0: return launch_tn_mode<EPI_ROWS, EF_OUT0>(L, gerr, st);
    case EF_OUT0 | EF_FRAMES: return launch_tn_mode<EPI_ROWS, EF_OUT0 | EF_FRAMES>(L, gerr, st);
    case EF_RES | EF_OUT0 | EF_OUT1: return launch_tn_mode<EPI_ROWS, EF_RES | EF_OUT0 | EF_OUT1>(L, gerr, st);
    case EF_RES | EF_OUT0: return launch_tn_mode<EPI_ROWS, EF_RES | EF_OUT0>(L, gerr, st);
    case EF_RES | EF_ACC2 | EF_OUT0: return launch_tn_mode<EPI_ROWS, EF_RES | EF_ACC2 | EF_OUT0>(L, gerr, st);
    case EF_RES | EF_ACC3 | EF_OUT1: return launch_tn_mode<EPI_ROWS, EF_RES | EF_ACC3 | EF_OUT1>(L, gerr, st);
    case EF_RES | EF_ACC3 | EF_OUT1 | EF_REFL:
      return launch_tn_mode<EPI_ROWS, EF_RES | EF_ACC3 | EF_OUT1 | EF_REFL>(L, gerr, st);
    default:
      PTB_REQUIRE(!e.frames, "pt_b200: the frames epilogue takes out0 alone");
      return launch_tn_mode<EPI_ROWS, EF_GENERIC>(L, gerr, st);
  }
}

// Weight rows (output channels, or phases x channels) per tile.  Up to 64 rows: one N tile of
// the time-on-M kernels; more: 128-row M tiles of the channels-on-M kernel (weights padded to a
// multiple of 128 rows).
static const int kTiles[] = {16, 32, 64};

int pick_bn(int ncols, int *bn, int *n_pad) {
  PTB_REQUIRE(ncols > 0, "pt_b200: empty N extent");
  const int n16 = (int)round_up(ncols, 16);
  for (int t : kTiles)
    if (t >= n16) {
      *bn = t;
      *n_pad = t;
      return 0;
    }
  *bn = 128;
  *n_pad = (int)round_up(ncols, 128);
  return 0;
}

int launch_conv(const ConvLaunch &L, uint32_t *gerr, cudaStream_t st) {
  PTB_REQUIRE(L.g.m_rows > 0 && L.g.nkb > 0 && L.g.n_cols % L.bn == 0,
              "pt_b200: bad conv geometry (m=%d nkb=%d n=%d bn=%d)", L.g.m_rows, L.g.nkb,
              L.g.n_cols, L.bn);
  const int halo = std::abs((L.g.ntap - 1) * L.g.row_step);
  if (L.g.tiles) {   // tile lists exist only in the channels-on-M kernel
    PTB_REQUIRE(L.bn == 128 && halo <= kWinHalo, "pt_b200: a conv tile list needs the channels-on-M kernel");
    return launch_tn(L, gerr, st);
  }
  // Convs whose taps reach at most kWinHalo rows run on one activation window per 32-channel
  // chunk: more than 64 output columns on the channels-on-M kernel, 16/32/64 on the time-on-M
  // window kernel.  Wider reaches (only generic C-ABI calls) run the per-tap kernel.
  if (halo <= kWinHalo) {
    if (L.bn == 128) return launch_tn(L, gerr, st);
    switch (L.bn) {
      case 64: return launch_win<64, 2>(L, gerr, st);
      case 32: return launch_win<32, 2>(L, gerr, st);
      case 16: return launch_win<16, 2>(L, gerr, st);
      default: break;
    }
  }
  switch (L.bn) {
    case 16: return launch_bn<16>(L, gerr, st);
    case 32: return launch_bn<32>(L, gerr, st);
    case 64: return launch_bn<64>(L, gerr, st);
    case 128: return launch_bn<128>(L, gerr, st);
    default: set_error("pt_b200: no conv instance for N tile %d", L.bn); return -1;
  }
}

}  // namespace ptb
