// conv_tc.cuh -- the implicit-GEMM Conv1d / ConvTranspose1d kernel on tcgen05 tensor cores.
//
// Problem (per batch item z): Y[m][n] = sum_{tap, ci} X[row(m, tap)][ci] * W[n][tap][ci]
//   M = output time rows (128 per CTA tile, TMEM lanes), N = output channels (<= 256 per tile,
//   TMEM columns), K = taps x input channels in 32-channel blocks (128-byte rows).
//   row(m, tap) = m + row_off0 + tap * row_step:  conv -> row_off0 = -pad, row_step = dilation;
//   convT phase decomposition -> rows are delay-line steps q, row_step = -1 (tap j reads q - j),
//   and N = stride * cout4 covers every phase at once, so no zero-stuffed MACs are issued.
//
// Operands: activations channels-last [z][rows][cin32] and weights [n][tap][cin32], both fp32
// values already rounded to tf32, TMA-loaded in 128-byte-swizzled K-major tiles.  Rows outside
// the activation tensor are zero-filled by TMA, which is the convolution's zero padding (and the
// convT head / tail flush).  The accumulator lives in TMEM; the epilogue warps read it back with
// tcgen05.ld and apply bias, the fused elementwise ops and the stores.
//
// Warp roles (192 threads): warps 0-3 epilogue (TMEM lanes 32w..32w+31), warp 4 TMA producer,
// warp 5 TMEM allocator + MMA issuer.  Every mbarrier wait is bounded (ptx.cuh).
#pragma once
#include <climits>
#include <cstdint>

#include "ptx.cuh"
#include "tail_math.cuh"

namespace ptb {

constexpr int kBM = 128;       // rows per tile
constexpr int kBK = 32;        // fp32 per k-block row (one 128 B swizzle row)
constexpr int kThreads = 192;

enum EpiMode : int {
  EPI_PLAIN_CONV = 0,   // channel-major output [z][n][t] (the pt_v21_conv C-ABI layout)
  EPI_PLAIN_CONVT = 1,  // channel-major convT output [z][co][oi], oi = q*s + r - pad
  EPI_ROWS = 2,         // channels-last ragged rows (decoder conv)
  EPI_ROWS_CONVT = 3,   // channels-last ragged rows (decoder upsampler)
};

struct ConvGeom {
  int m_rows;     // output rows per batch item
  int n_cols;     // N extent of the weight matrix (multiple of the N tile)
  int cin32;      // activation row length = weight row length per tap
  int ntap;
  int row_off0;   // activation row of output row 0, tap 0
  int row_step;   // activation row increment per tap
  int nkb;        // ntap * cin32 / 32
  int nbatch;     // batch items (the persistent kernel walks them in its tile list)
  // Channels-on-M kernel only: an explicit tile list {first row, rows} (rows a multiple of 16,
  // at most 256; batch 1), used instead of 256-row tiles over [0, m_rows) -- the streaming
  // executor computes only each stream's newly computable rows of a layer.
  const int2 *tiles;
  int ntiles;
  // Channels-on-M kernel only: walk the tiles last to first, so that a layer starts on the rows
  // its producer wrote last (still in L2); the decoder alternates it between layers.
  int reverse;
  // Channels-on-M kernel only: rows per tile of the uniform schedule (a multiple of 16, <= 256;
  // 0 = 256), chosen by the launcher so that the last wave of tiles is nearly full.
  int tile_rows;
  int win_slots;   // channels-on-M kernel: activation windows in its shared-memory ring (2 or 3)
};

struct EpiParams {
  int mode;
  const float *bias;       // [n_cols] zero-padded; may be null
  // channel-major outputs
  float *y;
  long long ybatch, ldy;
  int nstore;              // columns that are stored (cout4, or s * cout4 for convT)
  int rowmajor;            // EPI_PLAIN_CONV only: store y[z][t][n] (matmul) instead of y[z][n][t]
  long long tout;          // conv: rows stored; convT: output length Lout
  int epi0, epi1;
  float a0, a1;
  int s, pad, cphase;      // convT: column n = r * cphase + co
  long long q0;            // convT: delay-line step of tile row 0
  // channels-last ragged outputs (decoder)
  const unsigned char *mask;  // per output row: bit0 valid, bit1 duplicate into row - 2
  const int *obase;           // convT: per input row g -> output row obase[g] + s*g + r
  const float *res;           // residual input
  const float *accin;         // branch-sum accumulator input
  float *out0;                // fp32 output
  float *out1;                // tf32-rounded leaky output (next conv's input)
  int ldc, ldc1;
  int acc_mode;               // 0 none, 2: v = accin + v, 3: v = (accin + v) / 3
  float alpha1;
  int refl;                   // rows marked bit1 in mask are also written to row - 2
  int out_rows;               // convT: rows of out0 / out1 (a multiple of 4; the TMA-store view)
  int frames;                 // conv_post only: out0 rows get the 64 windowed iSTFT frame samples
};

// Compile-time shape of a decoder epilogue (the TN kernel is instantiated per combination, so
// each instance carries only the straight-line code it needs).
enum EpiFlags : int {
  EF_RES = 1, EF_ACC2 = 2, EF_ACC3 = 4, EF_OUT0 = 8, EF_OUT1 = 16, EF_REFL = 32,
  EF_FRAMES = 64,    // conv_post: the epilogue computes the tail's windowed frames (below)
  EF_GENERIC = -1,   // decide everything at run time from EpiParams
};

__device__ __forceinline__ float epi_op(float v, int op, float a) {
  switch (op) {
    case 1: return v >= 0.0f ? v : a * v;
    case 2: return v > 0.0f ? v : 0.0f;
    case 3: return v * a;
    case 4: return v + a;
    default: return v;
  }
}

__device__ __forceinline__ float leaky(float v, float a) { return v >= 0.0f ? v : a * v; }

template <int BN>
struct TmemCols {
  static constexpr uint32_t value = BN <= 32 ? 32u : BN <= 64 ? 64u : BN <= 128 ? 128u : 256u;
};

template <int BN, int STAGES>
struct ConvSmem {
  static constexpr int kA = kBM * kBK * 4;        // 16 KiB
  static constexpr int kB = BN * kBK * 4;
  static constexpr int kStage = kA + kB;
  static constexpr int kBytes = STAGES * kStage + 1024 /*align*/ + 256 /*barriers*/;
};

#ifdef PTB_CONV_KERNELS   // kernel bodies: compiled in conv_tc.cu only
// Epilogue for one 32-column chunk held by this thread (its TMEM lane = tile row).
template <int BN>
__device__ __forceinline__ void epilogue_chunk(const EpiParams &e, const float (&acc)[32], int z,
                                               int row, int m_rows, int n_base) {
  if (e.mode == EPI_PLAIN_CONV) {
    if (row >= e.tout) return;
    float *yz = e.y + (long long)z * e.ybatch + (e.rowmajor ? (long long)row * e.ldy : row);
    const long long nstride = e.rowmajor ? 1 : e.ldy;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int n = n_base + i;
      if (n < e.nstore) {
        float v = acc[i] + (e.bias ? __ldg(e.bias + n) : 0.0f);
        if (e.epi0) v = epi_op(v, e.epi0, e.a0);
        if (e.epi1) v = epi_op(v, e.epi1, e.a1);
        yz[(long long)n * nstride] = v;
      }
    }
    return;
  }
  if (e.mode == EPI_PLAIN_CONVT) {
    if (row >= m_rows) return;
    const long long q = e.q0 + row;
    float *yz = e.y + (long long)z * e.ybatch;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int n = n_base + i;
      if (n < e.nstore) {
        const int r = n / e.cphase, co = n - r * e.cphase;
        const long long oi = q * e.s + r - e.pad;
        if (oi >= 0 && oi < e.tout) {
          float v = acc[i] + (e.bias ? __ldg(e.bias + n) : 0.0f);
          if (e.epi0) v = epi_op(v, e.epi0, e.a0);
          yz[(long long)co * e.ldy + oi] = v;
        }
      }
    }
    return;
  }
  // channels-last ragged rows
  long long orow;
  int col0;
  if (e.mode == EPI_ROWS) {
    if (row >= m_rows) return;
    orow = row;
    col0 = n_base;
  } else {
    if (row >= m_rows) return;
    const int base = __ldg(e.obase + row);
    if (base == INT_MIN) return;
    const int r = n_base / e.cphase;
    orow = (long long)base + (long long)e.s * row + r;
    col0 = n_base - r * e.cphase;
  }
  const unsigned char mk = __ldg(e.mask + orow);
  if (!(mk & 1)) return;
  // columns of this chunk that exist in the output rows (conv_post: 80-wide tile, 72 real);
  // nstore counts columns of one output row (one phase for the upsampler)
  const int lim = e.nstore - col0 < 32 ? e.nstore - col0 : 32;
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    const float4 b = (e.bias && i < lim) ? __ldg(reinterpret_cast<const float4 *>(e.bias + n_base + i))
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
    v[i + 0] = acc[i + 0] + b.x;
    v[i + 1] = acc[i + 1] + b.y;
    v[i + 2] = acc[i + 2] + b.z;
    v[i + 3] = acc[i + 3] + b.w;
  }
  const long long off = orow * e.ldc + col0;
  if (e.res) {
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      if (i >= lim) break;
      const float4 r4 = *reinterpret_cast<const float4 *>(e.res + off + i);
      v[i + 0] += r4.x;
      v[i + 1] += r4.y;
      v[i + 2] += r4.z;
      v[i + 3] += r4.w;
    }
  }
  if (e.acc_mode) {
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      if (i >= lim) break;
      const float4 a4 = *reinterpret_cast<const float4 *>(e.accin + off + i);
      if (e.acc_mode == 2) {
        v[i + 0] = a4.x + v[i + 0];
        v[i + 1] = a4.y + v[i + 1];
        v[i + 2] = a4.z + v[i + 2];
        v[i + 3] = a4.w + v[i + 3];
      } else {
        v[i + 0] = div3_rn(a4.x + v[i + 0]);
        v[i + 1] = div3_rn(a4.y + v[i + 1]);
        v[i + 2] = div3_rn(a4.z + v[i + 2]);
        v[i + 3] = div3_rn(a4.w + v[i + 3]);
      }
    }
  }
  if (e.out0) {
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      if (i >= lim) break;
      *reinterpret_cast<float4 *>(e.out0 + off + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    }
  }
  if (e.out1) {
    const long long off1 = orow * e.ldc1 + col0;
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      if (i >= lim) break;
      const float4 w = make_float4(tf32_rna(leaky(v[i], e.alpha1)), tf32_rna(leaky(v[i + 1], e.alpha1)),
                                   tf32_rna(leaky(v[i + 2], e.alpha1)), tf32_rna(leaky(v[i + 3], e.alpha1)));
      *reinterpret_cast<float4 *>(e.out1 + off1 + i) = w;
      if (mk & 2) *reinterpret_cast<float4 *>(e.out1 + off1 - 2LL * e.ldc1 + i) = w;
    }
  }
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const ConvGeom g, const EpiParams e, uint32_t *gerr) {
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "tcgen05 M=128 needs N % 16 == 0, <= 256");
  using S = ConvSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;            // 1024 B: swizzle-atom aligned
  uint8_t *gbase = smem_raw + (base - raw);
  const uint32_t bar0 = base + STAGES * S::kStage;         // full[S], empty[S], acc, drain
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (STAGES + s); };
  const uint32_t accbar = bar0 + 8u * (2 * STAGES);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(gbase + STAGES * S::kStage + 8 * (2 * STAGES + 2));
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kBM, n0 = blockIdx.y * BN, z = blockIdx.z;
  constexpr uint32_t kCols = TmemCols<BN>::value;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    mbar_init(accbar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(tmem_slot), kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    if (lane == 0) {
      // ---------------- TMA producer
      const int kc = g.cin32 / kBK;
      int issued[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) issued[s] = 0;
      bool ok = true;
      for (int kb = 0; kb < g.nkb && ok; ++kb) {
        const int s = kb % STAGES;
        const uint32_t par = ((kb / STAGES) & 1) ^ 1;
        if (!mbar_wait(empty(s), par, abort_flag, gerr, ERR_WAIT_EMPTY)) {
          ok = false;
          break;
        }
        const int tap = kb / kc, c = kb - tap * kc;
        const uint32_t sa = base + s * S::kStage, sb = sa + S::kA;
        mbar_expect_tx(full(s), S::kStage);
        tma_load_3d(sa, &tmA, full(s), c * kBK, m0 + g.row_off0 + tap * g.row_step, z);
        tma_load_2d(sb, &tmB, full(s), tap * g.cin32 + c * kBK, n0);
        ++issued[s];
      }
      if (!ok) {
        // drain: every issued load must land before this CTA's shared memory is released
        for (int s = 0; s < STAGES; ++s) {
          if (!issued[s]) continue;
          const uint32_t par = (issued[s] - 1) & 1;
          uint32_t it = 0;
          while (!mbar_try_wait(full(s), par) && ++it < kWaitLimit) {
          }
          if (it >= kWaitLimit) atomicOr(gerr, ERR_WAIT_DRAIN);
        }
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      // ---------------- MMA issuer
      const uint32_t idesc = idesc_tf32(kBM, BN);
      bool ok = true;
      for (int kb = 0; kb < g.nkb; ++kb) {
        const int s = kb % STAGES;
        if (!mbar_wait(full(s), (kb / STAGES) & 1, abort_flag, gerr, ERR_WAIT_FULL)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = base + s * S::kStage, sb = sa + S::kA;
        const uint64_t da = sdesc_kmajor_sw128(sa), db = sdesc_kmajor_sw128(sb);
#pragma unroll
        for (int k = 0; k < kBK / 8; ++k)  // K = 8 tf32 (32 bytes) per instruction
          mma_tf32(tmem, da + 2u * k, db + 2u * k, idesc, (kb | k) != 0);
        mma_commit(empty(s));  // frees the stage once these MMAs have read it
      }
      mma_commit(accbar);
      if (!ok) {
        // MMAs already issued must finish before TMEM is released
        uint32_t it = 0;
        while (!mbar_try_wait(accbar, 0) && ++it < kWaitLimit) {
        }
        if (it >= kWaitLimit) atomicOr(gerr, ERR_WAIT_DRAIN);
      }
    }
  } else {
    // ---------------- epilogue warps 0..3
    if (mbar_wait(accbar, 0, abort_flag, gerr, ERR_WAIT_ACC)) {
      tc_fence_after();
      const int row = m0 + warp * 32 + lane;
      const uint32_t tl = tmem + (static_cast<uint32_t>(warp * 32) << 16);
#pragma unroll 1
      for (int j = 0; j < (BN + 31) / 32; ++j) {
        float acc[32];
        tmem_ld32(tl + 32u * j, acc);
        epilogue_chunk<BN>(e, acc, z, row, g.m_rows, n0 + 32 * j);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
}


// ---------------------------------------------------------------------------------------------
// Window variant: one activation window per 32-channel block serves every tap.
//
// The CTA owns MSUB x 128 output rows.  For input-channel block c it loads the activation rows
// [m0 + row_off0 + min(0, (ntap-1)*row_step), ... + MSUB*128 + (ntap-1)*|row_step|) once (64-row
// TMA boxes) and, for each tap, points the MMA's A descriptor at the tap's first row inside that
// window: a K-major 128B-swizzled operand may start at any 128-byte row (the tensor core applies
// the swizzle on absolute shared-memory address bits, base offset 0).  Only the weight tile is
// fetched per (tap, block), and it is shared by the MSUB accumulators, so operand traffic per
// output row drops by ~ntap for A and by MSUB for B compared with conv_tc_kernel.
constexpr int kWinBox = 64;     // rows per window TMA box
constexpr int kWinHalo = 64;    // max (ntap-1)*|row_step| supported by the window variant

template <int BN, int MSUB>
struct WinCfg {
  static constexpr int kColStride = BN <= 128 ? 128 : 256;        // TMEM columns per accumulator
  static constexpr uint32_t kCols = MSUB * kColStride <= 32 ? 32u : (uint32_t)(MSUB * kColStride);
  static constexpr int kWinRows = MSUB * kBM + kWinHalo;           // multiple of 64
  static constexpr int kWinBytes = kWinRows * kBK * 4;             // multiple of 1024
  static constexpr int kB = BN * kBK * 4;
  static constexpr int kBStagesRaw = (224 * 1024 - 2 * kWinBytes) / kB;
  static constexpr int kBStages = kBStagesRaw > 8 ? 8 : kBStagesRaw;
  static constexpr int kBytes = 2 * kWinBytes + kBStages * kB + 1024 + 256;
  static_assert(kBStages >= 2, "window variant needs at least two weight stages");
  static_assert(kCols <= 512, "TMEM holds 512 columns");
};

template <int BN, int MSUB>
__global__ void __launch_bounds__(kThreads, 1)
    conv_tc_win_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const ConvGeom g, const EpiParams e, uint32_t *gerr) {
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "tcgen05 M=128 needs N % 16 == 0, <= 256");
  using W = WinCfg<BN, MSUB>;
  constexpr int BS = W::kBStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t *gbase = smem_raw + (base - raw);
  const uint32_t win0 = base, bst0 = base + 2 * W::kWinBytes;
  const uint32_t bar0 = bst0 + BS * W::kB;
  auto wfull = [&](int s) { return bar0 + 8u * s; };
  auto wempty = [&](int s) { return bar0 + 8u * (2 + s); };
  auto bfull = [&](int s) { return bar0 + 8u * (4 + s); };
  auto bempty = [&](int s) { return bar0 + 8u * (4 + BS + s); };
  const uint32_t accbar = bar0 + 8u * (4 + 2 * BS);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(gbase + (bar0 - base) + 8 * (5 + 2 * BS) + 8);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * (MSUB * kBM), n0 = blockIdx.y * BN, z = blockIdx.z;
  const int kc = g.cin32 / kBK;
  const int span = (g.ntap - 1) * g.row_step;             // row offset of the last tap
  const int lo_off = span < 0 ? span : 0;                 // window starts at the lowest tap row
  const int wrows = MSUB * kBM + (span < 0 ? -span : span);
  const int nbox = (wrows + kWinBox - 1) / kWinBox;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(wfull(s), 1);
      mbar_init(wempty(s), 1);
    }
    for (int s = 0; s < BS; ++s) {
      mbar_init(bfull(s), 1);
      mbar_init(bempty(s), 1);
    }
    mbar_init(accbar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(tmem_slot), W::kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    if (lane == 0) {
      // ---------------- TMA producer: window per channel block, weight tile per (tap, block)
      int wiss[2] = {0, 0}, biss[BS];
#pragma unroll
      for (int s = 0; s < BS; ++s) biss[s] = 0;
      bool ok = true;
      const int wlo = m0 + g.row_off0 + lo_off;
      for (int c = 0; c < kc && ok; ++c) {
        const int ws = c & 1;
        if (!mbar_wait(wempty(ws), ((c >> 1) & 1) ^ 1, abort_flag, gerr, ERR_WAIT_EMPTY)) {
          ok = false;
          break;
        }
        const uint32_t wb = win0 + ws * W::kWinBytes;
        mbar_expect_tx(wfull(ws), nbox * kWinBox * kBK * 4);
        for (int b = 0; b < nbox; ++b)
          tma_load_3d(wb + b * kWinBox * kBK * 4, &tmA, wfull(ws), c * kBK, wlo + b * kWinBox, z);
        ++wiss[ws];
        for (int k = 0; k < g.ntap; ++k) {
          const int idx = c * g.ntap + k, bs = idx % BS;
          if (!mbar_wait(bempty(bs), ((idx / BS) & 1) ^ 1, abort_flag, gerr, ERR_WAIT_EMPTY)) {
            ok = false;
            break;
          }
          mbar_expect_tx(bfull(bs), W::kB);
          tma_load_2d(bst0 + bs * W::kB, &tmB, bfull(bs), k * g.cin32 + c * kBK, n0);
          ++biss[bs];
        }
      }
      if (!ok) {
        for (int s = 0; s < 2; ++s)
          if (wiss[s]) {
            uint32_t it = 0;
            while (!mbar_try_wait(wfull(s), (wiss[s] - 1) & 1) && ++it < kWaitLimit) {
            }
            if (it >= kWaitLimit) atomicOr(gerr, ERR_WAIT_DRAIN);
          }
        for (int s = 0; s < BS; ++s)
          if (biss[s]) {
            uint32_t it = 0;
            while (!mbar_try_wait(bfull(s), (biss[s] - 1) & 1) && ++it < kWaitLimit) {
            }
            if (it >= kWaitLimit) atomicOr(gerr, ERR_WAIT_DRAIN);
          }
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      // ---------------- MMA issuer
      const uint32_t idesc = idesc_tf32(kBM, BN);
      bool ok = true;
      for (int c = 0; c < kc && ok; ++c) {
        const int ws = c & 1;
        if (!mbar_wait(wfull(ws), (c >> 1) & 1, abort_flag, gerr, ERR_WAIT_FULL)) {
          ok = false;
          break;
        }
        const uint32_t wb = win0 + ws * W::kWinBytes;
        for (int k = 0; k < g.ntap; ++k) {
          const int idx = c * g.ntap + k, bs = idx % BS;
          if (!mbar_wait(bfull(bs), (idx / BS) & 1, abort_flag, gerr, ERR_WAIT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t db = sdesc_kmajor_sw128(bst0 + bs * W::kB);
          const uint32_t arow = wb + (uint32_t)(k * g.row_step - lo_off) * (kBK * 4);
#pragma unroll
          for (int s = 0; s < MSUB; ++s) {
            const uint64_t da = sdesc_kmajor_sw128(arow + s * kBM * kBK * 4);
#pragma unroll
            for (int kk = 0; kk < kBK / 8; ++kk)
              mma_tf32(tmem + s * W::kColStride, da + 2u * kk, db + 2u * kk, idesc, (c | k | kk) != 0);
          }
          mma_commit(bempty(bs));
        }
        if (ok) mma_commit(wempty(ws));
      }
      mma_commit(accbar);
      if (!ok) {
        uint32_t it = 0;
        while (!mbar_try_wait(accbar, 0) && ++it < kWaitLimit) {
        }
        if (it >= kWaitLimit) atomicOr(gerr, ERR_WAIT_DRAIN);
      }
    }
  } else {
    // ---------------- epilogue warps 0..3: TMEM lanes 32w..32w+31 of every accumulator
    if (mbar_wait(accbar, 0, abort_flag, gerr, ERR_WAIT_ACC)) {
      tc_fence_after();
      const uint32_t tl = tmem + (static_cast<uint32_t>(warp * 32) << 16);
#pragma unroll 1
      for (int s = 0; s < MSUB; ++s) {
        const int row = m0 + s * kBM + warp * 32 + lane;
#pragma unroll 1
        for (int j = 0; j < (BN + 31) / 32; ++j) {
          float acc[32];
          tmem_ld32(tl + s * W::kColStride + 32u * j, acc);
          epilogue_chunk<BN>(e, acc, z, row, g.m_rows, n0 + 32 * j);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, W::kCols);
  }
}


// ---------------------------------------------------------------------------------------------
// Channels-on-M variant ("TN"): D[co][t] = W[co][k] . X[t][k].
//
// The MMA is M = 128 output channels (weights, A operand) x N = 256 time rows (the activation
// window, B operand) x K = 8.  With 4-byte operands, M128 x N128 MMAs need ~122 B/clk of shared
// memory per SM at the tensor core's TF32 rate -- all of it -- while N = 256 needs ~92 B/clk, so
// this orientation reaches the tensor core's rate on the 128-channel layers that dominate the
// decoder.  TMEM lanes are output channels: an epilogue warp holds 32 channels x 32 time rows,
// and for each time row its 32 lanes store 32 consecutive channels (one full 128-byte line per
// warp instruction).  Persistent CTAs walk (128 channels x 256 rows) tiles with two TMEM
// accumulator sets (2 x 256 columns), channel blocks fastest so consecutive tiles reuse the same
// activation window from L2.
constexpr int kTNRows = 256;    // time rows per tile (MMA N)
// Warps 0 .. E-1 epilogue (E = TNCfg<F>::kEpiWarps), E activation-window producer, E+1 TMEM
// allocator + MMA issuer, E+2 weight producer.

// Pipeline shape.  Windows and weight stages come from two producer warps, so each ring runs
// ahead of the MMAs by its own depth.  Weight stages hold PTB_TN_GROUP consecutive (chunk, tap)
// steps of 16 KiB each, so the MMA issuer waits on one barrier and commits one release per
// 4 x PTB_TN_GROUP MMAs: the tensor pipe runs at most about one M128 x N256 MMA (~128 cycles)
// ahead of its issuing thread, and with the epilogue warps sharing the SM sub-partitions every
// handshake between two MMAs risks an idle pipe (32 KiB stages: 4,829 -> 4,722 us per config-4
// decode, mostly on the residual-reading k = 7 / 11 layers).  One shared-memory ring holds the
// activation windows and the weight stages, split per launch: kernel-3 layers consume a
// 32-channel window in 3 taps (~1.3 us of MMA, less than a window's load) and take three windows
// and two weight stages; wider kernels hold a window for 7-11 taps and take two windows and
// three weight stages (k = 3 convs1 61.6 vs 63.5 us, k = 11 convs1 139.5 vs 148.4 us, either way
// round losing).
#ifndef PTB_TN_GROUP
#define PTB_TN_GROUP 2
#endif
// Residual-reading instances (two staged outputs, 4 KB of staging per warp) run 12 epilogue warps
// and keep two windows and three weight stages whatever the kernel size.
#ifndef PTB_RES_EW
#define PTB_RES_EW 12
#endif
// The frames instance (conv_post, 72 channels, k = 7) also keeps two windows and three stages and
// gives the rest to its epilogue's per-part staging.
template <int F>
struct TNCfg {
  static constexpr bool kRes = F != EF_GENERIC && (F & EF_RES);
  static constexpr bool kFrames = F != EF_GENERIC && (F & EF_FRAMES);
  static constexpr bool kTwoWin = kRes || kFrames;
  static constexpr int kWinRows = kTNRows + kWinHalo;             // 320
  static constexpr int kWinBytes = kWinRows * kBK * 4;            // 40 KiB
  static constexpr int kA = kBM * kBK * 4;                        // 16 KiB weight tile
  static constexpr int kGroup = PTB_TN_GROUP;                     // weight tiles per stage
  static constexpr int kAS = kA * kGroup;                         // bytes per weight stage
  // ring of windows + weight stages: (3 windows, 2 stages) or (2, 3); residual instances (2, 3)
  static constexpr int kWinMax = kTwoWin ? 2 : 3;                 // barrier slots
  static constexpr int kStageMax = 3;
  static constexpr int kRing = kTwoWin ? 2 * kWinBytes + 3 * kAS
                                    : (3 * kWinBytes + 2 * kAS > 2 * kWinBytes + 3 * kAS
                                           ? 3 * kWinBytes + 2 * kAS
                                           : 2 * kWinBytes + 3 * kAS);
  // weight stages that fit beside `ws` windows
  __host__ __device__ static constexpr int stages(int ws) {
    return (kRing - ws * kWinBytes) / kAS < kStageMax ? (kRing - ws * kWinBytes) / kAS : kStageMax;
  }
  // Single-output instances without residual or branch-sum inputs (conv_pre, convs1, conv_post)
  // run 16 epilogue warps of one staging slot each: their epilogue is a chain of short dependent
  // steps per 16-row pass, and on the 128-channel k = 3 layers it, not the MMA, sets the pace;
  // twice the warps hide twice the latency in the same registers and shared memory.
  static constexpr int kEpiWarps =
      (F == EF_OUT1 || F == EF_OUT0 || kFrames) ? 16 : kRes ? PTB_RES_EW : 8;
  static constexpr int kThreads = 32 * (kEpiWarps + 3);
  static constexpr int kSlots = kEpiWarps == 16 ? 1 : 2;          // staging slots per warp
  static constexpr int kStageWarp = kSlots * 16 * kBK * 4;        // slots x (16 rows x 32 channels)
  // frames instance: per part (4 warps, 32 rows a pass) the raw 32 x 72 conv_post tile in rows of
  // kRawLd floats, aliased at offset 0 by the two 32-row x 128-byte frame boxes (1 KiB aligned)
  static constexpr int kRawLd = 73;
  static constexpr int kFrPart = 10 * 1024;
  static_assert(32 * kRawLd * 4 <= kFrPart, "frames staging: raw tile over the part's region");
  static constexpr int kStage = kFrames ? 4 * kFrPart : kEpiWarps * kStageWarp;   // 32 / 40 / 48 KiB
  static constexpr int kBytes = kRing + kStage + 1024 + 256;
  static_assert(kBytes <= 227 * 1024, "TN kernel shared memory over the per-CTA limit");
};

// Instances whose outputs leave through TMA tile stores staged in shared memory: the rows-mode
// decoder epilogues.  The reflection-row instance stages the mirrored value into the target gap
// row (mask bit 2), which the decoder layout keeps in the same 16-row pass as its source.
// Tile t of a channels-on-M launch: channel tile mi (fastest) of time tile t / mt -- a 256-row
// slice of [0, m_rows) of batch item z, or entry t / mt of the launch's tile list.
struct TNTile {
  int z, mi, r0, nr;
};
__device__ __forceinline__ TNTile tn_tile(const ConvGeom &g, int t, int mt, int tt, int ntiles) {
  TNTile x;
  if (g.reverse) t = ntiles - 1 - t;
  if (g.tiles) {
    const int entry = t / mt;
    const int2 v = g.tiles[entry];
    x.z = 0;
    x.mi = t - entry * mt;
    x.r0 = v.x;
    x.nr = v.y;
  } else {
    const int h = g.tile_rows ? g.tile_rows : kTNRows;
    x.z = t / (mt * tt);
    const int r = t - x.z * mt * tt, ti = r / mt;
    x.mi = r - ti * mt;
    x.r0 = ti * h;
    x.nr = h;
  }
  return x;
}

template <int MODE, int F>
struct TNTmaStore {
  static constexpr bool value = MODE == EPI_ROWS && F != EF_GENERIC;
};
// The upsampler instance (out0 + out1) stores a pass whose 16 delay-line steps all map into one
// request -- output rows 4 apart, one phase per warp -- as one TMA tile through a (C, 4, rows/4)
// view of each output; other passes (a request boundary inside) store directly.
template <int MODE, int F>
struct TNConvTStore {
  static constexpr bool value = MODE == EPI_ROWS_CONVT && F == (EF_OUT0 | EF_OUT1);
};

// Plain-mode (interpreter ABI) epilogue of one 32-channel x 32-row block: this thread's channel
// n, time rows t0..t0+31, read from TMEM at `taddr` (D[n][t0 + i] -> column i).  Rows at or past
// `tend` (the tile's end, at most m_rows) are not stored.
template <int MODE, int F>
__device__ __forceinline__ void tn_epi(const EpiParams &e, uint32_t taddr, int z, int n, int t0,
                                       int tend) {
  if constexpr (MODE == EPI_PLAIN_CONV || MODE == EPI_PLAIN_CONVT) {
    float v[32];
    tmem_ld32(taddr, v);
    const float bias = e.bias ? __ldg(e.bias + n) : 0.0f;
    if constexpr (MODE == EPI_PLAIN_CONV) {
      if (n >= e.nstore) return;
      float *y = e.y + (long long)z * e.ybatch;
      const long long rstride = e.rowmajor ? e.ldy : 1, cstride = e.rowmajor ? 1 : e.ldy;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int t = t0 + i;
        if (t < e.tout && t < tend) {
          float x = v[i] + bias;
          if (e.epi0) x = epi_op(x, e.epi0, e.a0);
          if (e.epi1) x = epi_op(x, e.epi1, e.a1);
          y[(long long)n * cstride + (long long)t * rstride] = x;
        }
      }
    } else {  // EPI_PLAIN_CONVT
      if (n >= e.nstore) return;
      const int r = n / e.cphase, co = n - r * e.cphase;
      float *y = e.y + (long long)z * e.ybatch + (long long)co * e.ldy;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int t = t0 + i;
        if (t < tend) {
          const long long oi = (e.q0 + t) * e.s + r - e.pad;
          if (oi >= 0 && oi < e.tout) {
            float x = v[i] + bias;
            if (e.epi0) x = epi_op(x, e.epi0, e.a0);
            y[oi] = x;
          }
        }
      }
    }
  }
}

// Rows-mode (decoder) epilogue.  An epilogue warp owns 32 channels (its TMEM lane quarter) x 128
// time rows of a tile: four 32-row blocks of two 16-row passes.  Everything that does not depend on
// the accumulator -- the per-row output map and masks of all four blocks, the bias, and the first
// pass's residual / branch-sum inputs -- is loaded before the accumulator wait, and each pass's
// inputs are requested one pass ahead of their use, so a warp keeps loads in flight instead of
// waiting on one dependent round trip per block.  Residual and branch-sum rows below m_rows are
// always inside their (m_rows x ldc) buffers, so these loads need no mask.
template <int MODE, int F>
struct TNRowsFlags {
  __device__ __forceinline__ static bool res(const EpiParams &e) {
    return F == EF_GENERIC ? e.res != nullptr : (F & EF_RES) != 0;
  }
  __device__ __forceinline__ static int acc(const EpiParams &e) {
    return F == EF_GENERIC ? e.acc_mode : (F & EF_ACC2) ? 2 : (F & EF_ACC3) ? 3 : 0;
  }
  __device__ __forceinline__ static bool out0(const EpiParams &e) {
    return F == EF_GENERIC ? e.out0 != nullptr : (F & EF_OUT0) != 0;
  }
  __device__ __forceinline__ static bool out1(const EpiParams &e) {
    return F == EF_GENERIC ? e.out1 != nullptr : (F & EF_OUT1) != 0;
  }
  __device__ __forceinline__ static bool refl(const EpiParams &e) {
    return F == EF_GENERIC ? e.refl != 0 : (F & EF_REFL) != 0;
  }
};

// residual / branch-sum inputs of rows th .. th+15 for this lane's output column
template <int MODE, int F>
__device__ __forceinline__ void tn_rows_load(const EpiParams &e, int th, int col, bool colok,
                                             int m_rows, float (&rs)[16], float (&ac)[16]) {
  using FL = TNRowsFlags<MODE, F>;
  if constexpr (MODE == EPI_ROWS) {
    const bool hr = FL::res(e);
    const int am = FL::acc(e);
    if (!hr && !am) return;
    const int ldc = e.ldc, base = th * ldc + col;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const bool ok = colok && th + i < m_rows;
      if (hr) rs[i] = ok ? e.res[base + i * ldc] : 0.0f;
      if (am) ac[i] = ok ? e.accin[base + i * ldc] : 0.0f;
    }
  }
}

// One 16-row pass: rows th .. th+15 are TMEM columns taddr .. taddr+15.  `mk` is this lane's row
// mask in the pass's 32-row block (bit 0 store, bit 1 also store the reflected row) and
// `orow_blk` its output row (row-map mode).
// With TMA stores (TNTmaStore) the pass writes its 16 rows x 32 channels into this warp's
// staging slots (row-major 16 x 128 B, conflict-free) and one lane issues the tile stores; masked
// rows are written as zeros, which keeps gap rows zero.  One output tensor alternates between the
// two slots (its previous store may still be reading the other); two tensors take one slot each.
template <int MODE, int F>
__device__ __forceinline__ void tn_rows_pass(const EpiParams &e, uint32_t taddr, int th, int h,
                                             int col, bool colok, float bias, unsigned mk,
                                             int orow_blk, const float (&rs)[16],
                                             const float (&ac)[16], const CUtensorMap *tm0,
                                             const CUtensorMap *tm1, uint32_t stage, int &slot,
                                             int lane) {
  using FL = TNRowsFlags<MODE, F>;
  const bool hr = FL::res(e), o0 = FL::out0(e), o1 = FL::out1(e), hrefl = FL::refl(e);
  const int am = FL::acc(e);
  const unsigned valid = __ballot_sync(0xffffffffu, mk & 1u);
  const unsigned vh = (valid >> (16 * h)) & 0xffffu;
  if (!vh) return;   // uniform over the warp: nothing of this pass is stored
  if constexpr (TNTmaStore<MODE, F>::value) {
    constexpr bool two = (F & EF_OUT0) && (F & EF_OUT1);
    constexpr bool one_slot = TNCfg<F>::kSlots == 1;
    const int col0 = col - lane;
    float v[16];
    tmem_ld16(taddr, v);
    if (lane == 0) {
      if (two || one_slot) bulk_wait_read<0>();
      else bulk_wait_read<1>();
    }
    __syncwarp();
    const uint32_t s0 =
        stage + (two || one_slot ? 0u : static_cast<uint32_t>(slot) * (16 * kBK * 4));
    const uint32_t s1 = two ? stage + 16 * kBK * 4 : s0;
    if constexpr ((F & EF_REFL) != 0) {
      // out1 only: rows whose mask has bit 2 take the value of the row two below (same pass)
      const unsigned tg = (__ballot_sync(0xffffffffu, (mk >> 2) & 1u) >> (16 * h)) & 0xffffu;
      float wv[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float x = v[i] + bias;
        if (hr) x += rs[i];
        if (am == 2) x = ac[i] + x;
        else if (am == 3) x = div3_rn(ac[i] + x);
        wv[i] = tf32_rna(leaky(x, e.alpha1));
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float val = 0.0f;
        if (colok) {
          if ((vh >> i) & 1) val = wv[i];
          else if (i + 2 < 16 && ((tg >> i) & 1)) val = wv[i + 2 < 16 ? i + 2 : i];
        }
        st_shared_f32(s1 + static_cast<uint32_t>(i * kBK * 4 + lane * 4), val);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const bool ok = ((vh >> i) & 1) && colok;
        float x = v[i] + bias;
        if (hr) x += rs[i];
        if (am == 2) x = ac[i] + x;
        else if (am == 3) x = div3_rn(ac[i] + x);
        const uint32_t at = static_cast<uint32_t>(i * kBK * 4 + lane * 4);
        if (o0) st_shared_f32(s0 + at, ok ? x : 0.0f);
        if (o1) st_shared_f32(s1 + at, ok ? tf32_rna(leaky(x, e.alpha1)) : 0.0f);
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0 && col0 < e.nstore) {
      if (o0) tma_store_2d(tm0, s0, col0, th);
      if (o1) tma_store_2d(tm1, s1, col0, th);
      bulk_commit();
    }
    slot ^= 1;
    return;
  }
  if constexpr (TNConvTStore<MODE, F>::value) {
    const int li = lane & 15;
    const int myrow = __shfl_sync(0xffffffffu, orow_blk, 16 * h + li);
    const int row0 = __shfl_sync(0xffffffffu, orow_blk, 16 * h);
    if (__all_sync(0xffffffffu, myrow >= 0 && myrow == row0 + 4 * li)) {
      const int col0 = col - lane;
      float v[16];
      tmem_ld16(taddr, v);
      if (lane == 0) bulk_wait_read<0>();
      __syncwarp();
      const uint32_t s0 = stage, s1 = stage + 16 * kBK * 4;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const bool ok = ((vh >> i) & 1) && colok;
        const float x = v[i] + bias;
        const uint32_t at = static_cast<uint32_t>(i * kBK * 4 + lane * 4);
        st_shared_f32(s0 + at, ok ? x : 0.0f);
        st_shared_f32(s1 + at, ok ? tf32_rna(leaky(x, e.alpha1)) : 0.0f);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && col0 < e.nstore) {
        tma_store_3d(tm0, s0, col0, row0 & 3, row0 >> 2);
        tma_store_3d(tm1, s1, col0, row0 & 3, row0 >> 2);
        bulk_commit();
      }
      return;
    }
  }
  const unsigned rh =
      hrefl ? (__ballot_sync(0xffffffffu, (mk >> 1) & 1u) >> (16 * h)) & 0xffffu : 0u;
  const int ldc = e.ldc, ldc1 = e.ldc1;
  float v[16];
  tmem_ld16(taddr, v);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    int orow;
    if constexpr (MODE == EPI_ROWS) orow = th + i;
    else orow = __shfl_sync(0xffffffffu, orow_blk, 16 * h + i);
    if (!((vh >> i) & 1) || !colok) continue;
    float x = v[i] + bias;
    if constexpr (MODE == EPI_ROWS) {
      if (hr) x += rs[i];
      if (am == 2) x = ac[i] + x;
      else if (am == 3) x = div3_rn(ac[i] + x);
    }
    if (o0) e.out0[orow * ldc + col] = x;
    if (o1) {
      const float w = tf32_rna(leaky(x, e.alpha1));
      e.out1[orow * ldc1 + col] = w;
      if (hrefl && ((rh >> i) & 1)) e.out1[(orow - 2) * ldc1 + col] = w;
    }
  }
}

template <int MODE, int F>
__global__ void __launch_bounds__(TNCfg<F>::kThreads, 1)
    conv_tc_tn_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                      const __grid_constant__ CUtensorMap tmO0,
                      const __grid_constant__ CUtensorMap tmO1, const ConvGeom g, const EpiParams e,
                      uint32_t *gerr) {
  using P = TNCfg<F>;
  constexpr int WSM = P::kWinMax, ASM = P::kStageMax;   // barrier slots
  const int WS = g.win_slots, AS = P::stages(g.win_slots);   // this launch's ring split
  constexpr int EW = P::kEpiWarps;   // epilogue warps; then the window producer, MMA, weights
  if (WS < 2 || WS > WSM || AS < 1) {   // uniform over the grid: nothing has started yet
    if (threadIdx.x == 0) atomicOr(gerr, ERR_BAD_ARGS);
    return;
  }
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t *gbase = smem_raw + (base - raw);
  const uint32_t win0 = base, ast0 = base + WS * P::kWinBytes;
  const uint32_t stg0 = base + P::kRing;   // epilogue output staging, kStageWarp per warp
  const uint32_t bar0 = stg0 + P::kStage;
  auto wfull = [&](int s) { return bar0 + 8u * s; };
  auto wempty = [&](int s) { return bar0 + 8u * (WSM + s); };
  auto afull = [&](int s) { return bar0 + 8u * (2 * WSM + s); };       // accumulator ready
  auto aempty = [&](int s) { return bar0 + 8u * (2 * WSM + 2 + s); };  // accumulator drained
  auto sfull = [&](int s) { return bar0 + 8u * (2 * WSM + 4 + s); };   // weight stage loaded
  auto sempty = [&](int s) { return bar0 + 8u * (2 * WSM + 4 + ASM + s); };
  const uint32_t dbar = bar0 + 8u * (2 * WSM + 4 + 2 * ASM);
  uint32_t *tmem_slot =
      reinterpret_cast<uint32_t *>(gbase + (bar0 - base) + 8 * (2 * WSM + 5 + 2 * ASM));
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  // frames instance: one barrier per part of four epilogue warps (after the TMEM slot)
  auto pbar = [&](int p) { return bar0 + 8u * (2 * WSM + 6 + 2 * ASM + p); };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kc = g.cin32 / kBK;
  const int span = (g.ntap - 1) * g.row_step;
  const int lo_off = span < 0 ? span : 0;
  const int wspan = span < 0 ? -span : span;
  const int mt = (g.n_cols + kBM - 1) / kBM;              // channel tiles (fastest)
  const int th = g.tile_rows ? g.tile_rows : kTNRows;
  const int tt = (g.m_rows + th - 1) / th;                 // time tiles
  const int ntiles = g.tiles ? g.ntiles * mt : mt * tt * g.nbatch;

  if (threadIdx.x == 0) {
    for (int s = 0; s < WS; ++s) {
      mbar_init(wfull(s), 1);
      mbar_init(wempty(s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(afull(s), 1);
      mbar_init(aempty(s), EW);
    }
    for (int s = 0; s < AS; ++s) {
      mbar_init(sfull(s), 1);
      mbar_init(sempty(s), 1);
    }
    mbar_init(dbar, 1);
    if constexpr (P::kFrames)
      for (int p = 0; p < 4; ++p) mbar_init(pbar(p), 4);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == EW && lane == 0) {
    prefetch_tmap(&tmX);
    prefetch_tmap(&tmW);
  }
  if (warp == EW + 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == EW) {
    if (lane == 0) {
      // ---------------- TMA producer: activation windows (one per 32-channel chunk)
      int wiss[WSM] = {};
      bool ok = true;
      int cw = 0;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const TNTile tl = tn_tile(g, t, mt, tt, ntiles);
        const int z = tl.z;
        const int wlo = tl.r0 + g.row_off0 + lo_off;
        const int nbox = (tl.nr + wspan + kWinBox - 1) / kWinBox;
        for (int c = 0; c < kc; ++c, ++cw) {
          const int ws = cw % WS;
          if (!mbar_wait(wempty(ws), ((cw / WS) & 1) ^ 1, abort_flag, gerr, ERR_WAIT_EMPTY)) {
            ok = false;
            break;
          }
          const uint32_t wb = win0 + ws * P::kWinBytes;
          mbar_expect_tx(wfull(ws), nbox * kWinBox * kBK * 4);
          for (int b = 0; b < nbox; ++b)
            tma_load_3d(wb + b * kWinBox * kBK * 4, &tmX, wfull(ws), c * kBK, wlo + b * kWinBox, z);
          ++wiss[ws];
        }
      }
      if (!ok)
        for (int s = 0; s < WS; ++s)
          if (wiss[s]) {
            uint32_t it = 0;
            while (!mbar_try_wait(wfull(s), (wiss[s] - 1) & 1) && ++it < kWaitLimit) {
            }
            if (it >= kWaitLimit) atomicOr(gerr, ERR_WAIT_DRAIN);
          }
    }
  } else if (warp == EW + 2) {
    if (lane == 0) {
      // ---------------- TMA producer: weight stages, kGroup (chunk, tap) steps each; a tile's
      // steps run chunk-major, taps fastest, and a stage never spans two tiles
      constexpr int GR = P::kGroup;
      int aiss[ASM];
#pragma unroll
      for (int s = 0; s < ASM; ++s) aiss[s] = 0;
      bool ok = true;
      int ca = 0;
      const int steps = kc * g.ntap;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const int mi = tn_tile(g, t, mt, tt, ntiles).mi;
        int c = 0, k = 0;
        for (int j = 0; j < steps; j += GR, ++ca) {
          const int as = ca % AS;
          if (!mbar_wait(sempty(as), ((ca / AS) & 1) ^ 1, abort_flag, gerr, ERR_WAIT_EMPTY)) {
            ok = false;
            break;
          }
          const int nb = steps - j < GR ? steps - j : GR;
          mbar_expect_tx(sfull(as), nb * P::kA);
          for (int b = 0; b < nb; ++b) {
            tma_load_2d(ast0 + as * P::kAS + b * P::kA, &tmW, sfull(as), k * g.cin32 + c * kBK,
                        mi * kBM);
            if (++k == g.ntap) {
              k = 0;
              ++c;
            }
          }
          ++aiss[as];
        }
      }
      if (!ok)
        for (int s = 0; s < AS; ++s)
          if (aiss[s]) {
            uint32_t it = 0;
            while (!mbar_try_wait(sfull(s), (aiss[s] - 1) & 1) && ++it < kWaitLimit) {
            }
            if (it >= kWaitLimit) atomicOr(gerr, ERR_WAIT_DRAIN);
          }
    }
  } else if (warp == EW + 1) {
    if (lane == 0) {
      // ---------------- MMA issuer: M = 128 channels, N = the tile's time rows (<= 256)
      // The tensor pipe queues few MMAs, so every instruction this thread spends between two
      // MMAs beyond one MMA's duration idles it: descriptors advance by adds (the address field
      // is the shared-memory byte address / 16), ring slots and phases are counters, and the
      // next tile's height is read while this tile's MMAs run.
      bool ok = true;
      int it = 0, ws = 0, as = 0;
      uint32_t wph = 0, aph = 0;
      const uint64_t dA0 = sdesc_kmajor_sw128(ast0);
      const uint64_t dW0 = sdesc_kmajor_sw128(win0 + static_cast<uint32_t>(-lo_off) * (kBK * 4));
      const int64_t dtap = static_cast<int64_t>(g.row_step) * (kBK * 4 / 16);
      const int ntap = g.ntap;
      int nr = blockIdx.x < ntiles ? tn_tile(g, blockIdx.x, mt, tt, ntiles).nr : 0;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++it) {
        const uint32_t idesc = idesc_tf32(kBM, nr);
        if (t + static_cast<int>(gridDim.x) < ntiles)
          nr = tn_tile(g, t + gridDim.x, mt, tt, ntiles).nr;
        const int ab = it & 1;
        if (!mbar_wait(aempty(ab), ((it >> 1) & 1) ^ 1, abort_flag, gerr, ERR_WAIT_EMPTY)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + ab * kTNRows;
        uint32_t accum = 0;
        int sub = 0;   // weight tile within the current stage
        uint64_t dA = dA0 + static_cast<uint64_t>(as * (P::kAS / 16));
        for (int c = 0; c < kc && ok; ++c) {
          if (!mbar_wait(wfull(ws), wph, abort_flag, gerr, ERR_WAIT_FULL)) {
            ok = false;
            break;
          }
          uint64_t dB = dW0 + static_cast<uint64_t>(ws * (P::kWinBytes / 16));
          for (int k = 0; k < ntap; ++k) {
            if (sub == 0) {
              if (!mbar_wait(sfull(as), aph, abort_flag, gerr, ERR_WAIT_FULL)) {
                ok = false;
                break;
              }
              tc_fence_after();
            }
            mma_tf32(acc, dA, dB, idesc, accum);
            mma_tf32(acc, dA + 2u, dB + 2u, idesc, 1u);
            mma_tf32(acc, dA + 4u, dB + 4u, idesc, 1u);
            mma_tf32(acc, dA + 6u, dB + 6u, idesc, 1u);
            accum = 1u;
            dA += static_cast<uint64_t>(P::kA / 16);
            if (++sub == P::kGroup || (c == kc - 1 && k == ntap - 1)) {
              // the stage's last weight tile (or the tile's last step): release it
              mma_commit(sempty(as));
              sub = 0;
              if (++as == AS) {
                as = 0;
                aph ^= 1u;
              }
              dA = dA0 + static_cast<uint64_t>(as * (P::kAS / 16));
            }
            dB += static_cast<uint64_t>(dtap);
          }
          if (ok) mma_commit(wempty(ws));
          if (++ws == WS) {
            ws = 0;
            wph ^= 1u;
          }
        }
        if (ok) mma_commit(afull(ab));
      }
      if (!ok) {
        mma_commit(dbar);
        uint32_t n = 0;
        while (!mbar_try_wait(dbar, 0) && ++n < kWaitLimit) {
        }
        if (n >= kWaitLimit) atomicOr(gerr, ERR_WAIT_DRAIN);
      }
    }
  } else if constexpr (P::kFrames) {
    // ---------------- frames epilogue (conv_post): the tail's per-frame work on the SM that holds
    // the frame.  A part (warps 4p .. 4p+3, one per TMEM lane quarter) owns 32-row blocks of the
    // tile as in the rows epilogue and runs each block in four steps, its warps meeting on the
    // part's mbarrier (bounded waits) between them:
    //   (a) quarters 0-2 load their channels' 32 accumulator columns, add the bias and store
    //       the 32 x 72 conv_post values row-major (rows of kRawLd floats: conflict-free);
    //   (b) thread (row = lane, band = quarter) loads its row's 9 log-magnitudes and 9 phase
    //       logits;
    //   (c) it computes the band's 16 windowed frame samples (frame_band: the tail kernel's
    //       phases 1a-1b, same operations and order) and stores them, zeros for rows outside the
    //       tile or the mask, into two 32-row x 128-byte boxes with the 128-byte swizzle
    //       (conflict-free 16-byte stores), aliasing the raw tile;
    //   (d) quarter 3's lane 0 stores the boxes by TMA (a 16-row box when only 16 rows remain)
    //       and, before the next block's step (a), waits until they have been read.
    // Quarter 3 holds no conv_post channel, so it releases the accumulator at once; quarters 0-2
    // release it after their last block's TMEM loads.
    const int q = warp & 3, part = warp >> 2;
    const uint32_t reg = stg0 + static_cast<uint32_t>(part) * P::kFrPart;
    constexpr int RL = P::kRawLd;
    const uint32_t pb = pbar(part);
    uint32_t pph = 0;
    bool ok = true;
    auto psync = [&]() {
      __syncwarp();
      if (lane == 0) mbar_arrive(pb);
      ok = mbar_wait(pb, pph, abort_flag, gerr, ERR_WAIT_PART);
      pph ^= 1u;
      return ok;
    };
    const int ch = q * 32 + lane;   // this lane's conv_post channel (TMEM lane)
    const bool chok = q < 3 && ch < 72;
    const float bias = (chok && e.bias) ? __ldg(e.bias + ch) : 0.0f;
    const uint32_t raw_w = reg + static_cast<uint32_t>(ch) * 4u;                  // (a): column ch
    const uint32_t raw_r = reg + static_cast<uint32_t>(lane * RL + 18 * q) * 4u;  // (b): row lane
    int it = 0;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++it) {
      const int ab = it & 1;
      const TNTile tile = tn_tile(g, t, mt, tt, ntiles);
      const int r0 = tile.r0;
      const int nblk = (tile.nr + 31) / 32, bh = (nblk + 3) / 4;
      const int b0 = part * bh;
      const int nb = b0 >= nblk ? 0 : (nblk - b0 < bh ? nblk - b0 : bh);
      const int te = r0 + tile.nr < g.m_rows ? r0 + tile.nr : g.m_rows;
      const int rb = r0 + 32 * b0;
      unsigned vm = 0;   // bit j: this lane's row of block j is a stored frame
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int tr = rb + 32 * j + lane;
        if (j < nb && tr < te && (__ldg(e.mask + tr) & 1u)) vm |= 1u << j;
      }
      if (!mbar_wait(afull(ab), (it >> 1) & 1, abort_flag, gerr, ERR_WAIT_ACC)) break;
      tc_fence_after();
      const uint32_t tl = tmem + ab * kTNRows + (static_cast<uint32_t>(q * 32) << 16) + 32u * b0;
      if (q == 3 || nb == 0) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(aempty(ab));
      }
#pragma unroll 1
      for (int j = 0; j < nb; ++j) {
        const int th = rb + 32 * j;
        if (q == 3 && lane == 0) bulk_wait_read<0>();
        if (!psync()) break;
        if (q < 3) {   // (a)
          float v0[16], v1[16];
          tmem_ld16(tl + 32u * j, v0);
          tmem_ld16(tl + 32u * j + 16u, v1);
          if (j == nb - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(aempty(ab));
          }
          if (chok) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              st_shared_f32(raw_w + static_cast<uint32_t>(i * RL * 4), v0[i] + bias);
              st_shared_f32(raw_w + static_cast<uint32_t>((16 + i) * RL * 4), v1[i] + bias);
            }
          }
        }
        if (!psync()) break;
        float la[9], lb[9];   // (b)
#pragma unroll
        for (int k = 0; k < 9; ++k) {
          la[k] = ld_shared_f32(raw_r + static_cast<uint32_t>(k * 4));
          lb[k] = ld_shared_f32(raw_r + static_cast<uint32_t>((9 + k) * 4));
        }
        if (!psync()) break;
        float w[16];   // (c)
        frame_band(la, lb, w);
        const bool rv = (vm >> j) & 1u;
        const uint32_t sb =
            reg + static_cast<uint32_t>(q >> 1) * 4096u + static_cast<uint32_t>(lane) * 128u;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t u = static_cast<uint32_t>(((q & 1) * 4 + i) ^ (lane & 7));
          st_shared_v4(sb + u * 16u, rv ? w[4 * i] : 0.0f, rv ? w[4 * i + 1] : 0.0f,
                       rv ? w[4 * i + 2] : 0.0f, rv ? w[4 * i + 3] : 0.0f);
        }
        fence_proxy_async_smem();
        if (!psync()) break;
        if (q == 3 && lane == 0 && th < te) {   // (d)
          const CUtensorMap *m = te - th > 16 ? &tmO0 : &tmO1;
          tma_store_2d(m, reg, 0, th);
          tma_store_2d(m, reg + 4096u, 32, th);
          bulk_commit();
        }
      }
    }
    if (lane == 0) bulk_wait_all();   // staged stores done before the CTA's memory goes
    __syncwarp();
  } else {
    // ---------------- epilogue warps 0 .. EW-1: lane quarter (channels) x part of the time rows
    const int q = warp & 3, part = warp >> 2;
    constexpr int kParts = EW / 4;
    const uint32_t stg = stg0 + static_cast<uint32_t>(warp) * P::kStageWarp;
    int slot = 0;
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const int ab = it & 1;
      const TNTile tile = tn_tile(g, t, mt, tt, ntiles);
      const int z = tile.z, mi = tile.mi, r0 = tile.r0;
      // this warp's 32-row blocks of the tile: part p takes blocks [p * bh, (p + 1) * bh)
      const int nblk = (tile.nr + 31) / 32, bh = (nblk + kParts - 1) / kParts;
      const int b0 = part * bh;
      const int nb = b0 >= nblk ? 0 : (nblk - b0 < bh ? nblk - b0 : bh);
      const int te = r0 + tile.nr < g.m_rows ? r0 + tile.nr : g.m_rows;   // rows this tile stores
      const int co_row = mi * kBM + q * 32 + lane;
      const uint32_t tl = tmem + ab * kTNRows + (static_cast<uint32_t>(q * 32) << 16);
      if constexpr (MODE == EPI_ROWS || MODE == EPI_ROWS_CONVT) {
        int col = co_row, ph = 0;
        if constexpr (MODE == EPI_ROWS_CONVT) {
          ph = co_row / e.cphase;   // uniform over the warp: 32 lanes never straddle a phase
          col = co_row - ph * e.cphase;
        }
        const bool colok = col < e.nstore;
        const float bias = (e.bias && colok) ? __ldg(e.bias + co_row) : 0.0f;
        const int rb = r0 + 32 * b0;   // this warp's first time row
        // output row map and masks of its (up to four) blocks (lane = row within the block)
        int orow[4];
        unsigned mk = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int tr = rb + 32 * j + lane;
          orow[j] = -1;
          if (j < nb && tr < te) {
            if constexpr (MODE == EPI_ROWS) {
              orow[j] = tr;
            } else {
              const int b = __ldg(e.obase + tr);
              if (b != INT_MIN) orow[j] = b + e.s * tr + ph;
            }
          }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (orow[j] >= 0) mk |= static_cast<unsigned>(__ldg(e.mask + orow[j])) << (8 * j);
        float rsA[16], acA[16];
        if (nb > 0) tn_rows_load<MODE, F>(e, rb, col, colok, g.m_rows, rsA, acA);
        if (!mbar_wait(afull(ab), (it >> 1) & 1, abort_flag, gerr, ERR_WAIT_ACC)) break;
        tc_fence_after();
        const uint32_t tw = tl + static_cast<uint32_t>(32 * b0);
#pragma unroll 1
        for (int j = 0; j < nb; ++j) {
          const int th = rb + 32 * j;
          const unsigned mj = (mk >> (8 * j)) & 0xffu;
          const int oj = j == 0 ? orow[0] : j == 1 ? orow[1] : j == 2 ? orow[2] : orow[3];
          float rsB[16], acB[16];
          tn_rows_load<MODE, F>(e, th + 16, col, colok, g.m_rows, rsB, acB);
          tn_rows_pass<MODE, F>(e, tw + 32u * j, th, 0, col, colok, bias, mj, oj, rsA, acA, &tmO0,
                                &tmO1, stg, slot, lane);
          if (j + 1 < nb) tn_rows_load<MODE, F>(e, th + 32, col, colok, g.m_rows, rsA, acA);
          tn_rows_pass<MODE, F>(e, tw + 32u * j + 16u, th + 16, 1, col, colok, bias, mj, oj, rsB,
                                acB, &tmO0, &tmO1, stg, slot, lane);
        }
      } else {
        if (!mbar_wait(afull(ab), (it >> 1) & 1, abort_flag, gerr, ERR_WAIT_ACC)) break;
        tc_fence_after();
#pragma unroll 1
        for (int j = b0; j < b0 + nb; ++j)
          tn_epi<MODE, F>(e, tl + 32u * j, z, co_row, r0 + 32 * j, te);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(aempty(ab));
    }
    if constexpr (TNTmaStore<MODE, F>::value || TNConvTStore<MODE, F>::value) {
      if (lane == 0) bulk_wait_all();   // staged stores done before the CTA's memory goes
      __syncwarp();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == EW + 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

#endif  // PTB_CONV_KERNELS

}  // namespace ptb
