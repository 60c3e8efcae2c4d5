// decoder.cu -- the whole MB-iSTFT decoder device-resident, for a batch of independent requests.
//
// Ragged batch layout.  At each time resolution (level 0: latent frames T, level 1: 4T after
// ups.0, level 2: 16T after ups.1) the requests are stacked along time in one channels-last
// tensor [rows][C], each request's rows preceded and followed by zero gap rows: 16 at level 0
// (conv_pre reaches 3 rows, ups.0 reads 2 before and 1 after a request; 16 so that a 16-row
// epilogue slab rounded outward from one request never reaches the next), 28 at level 1 and 32
// at level 2 (the widest conv reaches dilation 5 x (11-1)/2 = 25 rows; conv_post reads 3 + 1
// reflection row).  So one launch per layer computes every request exactly as if it ran
// alone: the zero gap rows are the convolutions' zero padding, and the epilogue never writes them
// (a per-row mask), so they stay zero.
//
// A request is a window (pt_b200_window): a column slice of a latent (offset, channel stride),
// the output samples it keeps and where they go.  Whole utterances keep everything; streaming
// windows keep their interiors, which the tail kernel writes straight into the stitched output.
//
// Graph wiring (ref/v21_graph_trace.txt 3819-4065), with every elementwise node fused:
//   conv_pre(+LeakyRelu) -> ups.0 (writes u and leaky(u)) ->
//   per resblock r, stage j: convs1 (+LeakyRelu) -> convs2 (+ residual add, + leaky for the next
//   stage; the last stage of the last resblock also does /dec/Add, /dec/Add_1, /3, LeakyRelu) ->
//   ups.1 -> the same MRF at 128 channels (final LeakyRelu 0.01 and the (1,0) reflection pad row)
//   -> subband_conv_post -> the iSTFT/PQMF tail kernel.
#include "decoder.cuh"

using namespace ptb;
using namespace ptb::dec;

namespace {

constexpr int64_t kStreamBatchFrames = 65536;   // default latent frames per streaming batch

// Stage packed weights into the kernel layout on the device (once per decoder).
int make_layer(DLayer *L, const float *wp, const float *bias, int rows4, int ntap, int cin,
               int cout, int cphase, cudaStream_t st) {
  L->ntap = ntap;
  L->cin32 = (int)round_up(cin, kBK);
  if (pick_bn(rows4, &L->bn, &L->n_pad)) return -1;
  const size_t pbytes = (size_t)rows4 * ntap * cin * 4;
  float *dp = nullptr;
  PTB_CUDA(cudaMalloc(&L->w, (size_t)L->n_pad * ntap * L->cin32 * 4));
  PTB_CUDA(cudaMalloc(&L->b, (size_t)round_up(L->n_pad, 32) * 4));
  PTB_CUDA(cudaMalloc(&dp, pbytes));
  PTB_CUDA(cudaMemcpyAsync(dp, wp, pbytes, cudaMemcpyHostToDevice, st));
  if (stage_packed_w(dp, rows4, ntap, cin, L->w, L->n_pad, L->cin32, st)) return -1;
  std::vector<float> hb((size_t)round_up(L->n_pad, 32), 0.0f);
  for (int n = 0; n < rows4; ++n)
    if (n % cphase < cout) hb[n] = bias[n % cphase];
  PTB_CUDA(cudaMemcpyAsync(L->b, hb.data(), hb.size() * 4, cudaMemcpyHostToDevice, st));
  PTB_CUDA(cudaStreamSynchronize(st));
  cudaFree(dp);
  return 0;
}

}  // namespace

// scatter each request's channel-major latent columns (z[zoff + c*zld + t], f0 <= t < T) into the
// level-0 rows, tf32-rounded.  One 32 x 8 block moves 32 frames x all 192 channels: every thread
// issues its 24 loads before the barrier, and each frame row leaves as six 128-byte lines.
__global__ void ptb::dec::stage_z_kernel(const float *__restrict__ z, const long long *__restrict__ zoff,
                               const long long *__restrict__ zld, const long long *__restrict__ T,
                               const long long *__restrict__ a0, const long long *__restrict__ f0,
                               float *__restrict__ Z) {
  __shared__ float tile[192][33];
  const int r = blockIdx.z;
  const long long Tr = T[r];   // frames [f0, T) of request r (f0 null: from 0)
  const long long t0 = (f0 ? f0[r] : 0) + (long long)blockIdx.x * 32;
  if (t0 >= Tr) return;
  const float *zr = z + zoff[r];
  const long long ld = zld[r];
  const long long t = t0 + threadIdx.x;
  const bool tv = t < Tr;
#pragma unroll 8
  for (int c = threadIdx.y; c < 192; c += 8) tile[c][threadIdx.x] = tv ? zr[(long long)c * ld + t] : 0.0f;
  __syncthreads();
  const long long a = a0[r];
  for (int i = threadIdx.y; i < 32; i += 8) {
    const long long tt = t0 + i;
    if (tt >= Tr) break;
    float *dst = Z + (a + tt) * 192;
#pragma unroll
    for (int c = threadIdx.x; c < 192; c += 32) dst[c] = tf32_rna(tile[c][i]);
  }
}

namespace {

bool same_windows(const std::vector<pt_b200_window> &a, int n, const pt_b200_window *w) {
  if ((int)a.size() != n) return false;
  for (int i = 0; i < n; ++i)
    if (a[i].frames != w[i].frames || a[i].z_off != w[i].z_off || a[i].z_ld != w[i].z_ld ||
        a[i].keep_lo != w[i].keep_lo || a[i].keep_hi != w[i].keep_hi || a[i].dst != w[i].dst)
      return false;
  return true;
}

int check_windows(int n, const pt_b200_window *w) {
  PTB_REQUIRE(n > 0 && w, "pt_b200: no requests");
  for (int i = 0; i < n; ++i) {
    const pt_b200_window &x = w[i];
    PTB_REQUIRE(x.frames >= 2, "pt_b200: request %d has %lld frames (need >= 2)", i,
                (long long)x.frames);
    PTB_REQUIRE(x.z_off >= 0 && x.z_ld >= x.frames, "pt_b200: request %d: bad latent slice", i);
    PTB_REQUIRE(x.keep_lo >= 0 && x.keep_lo < x.keep_hi && x.keep_hi <= 256 * x.frames && x.dst >= 0,
                "pt_b200: request %d: kept samples [%lld, %lld) outside [0, %lld)", i,
                (long long)x.keep_lo, (long long)x.keep_hi, (long long)(256 * x.frames));
  }
  return 0;
}

}  // namespace

int ptb::dec::build_layout(Plan &p, cudaStream_t st, int nreq, const pt_b200_window *w) {
  if (check_windows(nreq, w)) return -1;
  p.W.assign(w, w + nreq);
  for (int i = 0; i < nreq; ++i) p.T.push_back(w[i].frames);
  const int64_t *T = p.T.data();
  const int64_t scale[3] = {1, 4, 16};
  std::vector<int64_t> *a = p.a;
  layout_rows(T, nreq, a, p.R);
  for (int i = 0; i < nreq; ++i)
    PTB_REQUIRE(a[2][i] % 16 == 4, "pt_b200: level-2 layout broke the reflection-row alignment");
  for (int i = 0; i < nreq; ++i) {
    p.max_T = T[i] > p.max_T ? T[i] : p.max_T;
    p.total_z += 192 * T[i];
    p.total_wav += 256 * T[i];
  }
  // epilogue offsets are 32-bit: every activation tensor must stay below 2^31 elements
  PTB_REQUIRE(p.R[2] * 128 < (int64_t)INT_MAX && p.R[0] * 512 < (int64_t)INT_MAX &&
                  p.R[1] * 256 < (int64_t)INT_MAX,
              "pt_b200: batch too large (%lld level-2 rows); split it into smaller batches",
              (long long)p.R[2]);
  // host tables in one block
  std::vector<unsigned char> m[3], mr, mp;
  for (int l = 0; l < 3; ++l) m[l].assign((size_t)p.R[l], 0);
  for (int l = 0; l < 3; ++l)
    for (int i = 0; i < nreq; ++i)
      std::memset(m[l].data() + a[l][i], 1, (size_t)(scale[l] * T[i]));
  mr = m[2];
  mp.assign((size_t)p.R[2], 0);
  for (int i = 0; i < nreq; ++i) {
    // reflection pad (1,0): local row 1 (bit 1 on the source) is mirrored into row -1 (bit 2 on
    // the target, a gap row)
    mr[(size_t)a[2][i] + 1] |= 2;
    mr[(size_t)a[2][i] - 1] |= 4;
    std::memset(mp.data() + a[2][i] - 1, 1, (size_t)(16 * T[i] + 1));
  }
  std::vector<int> ob01((size_t)p.R[0], INT_MIN), ob12((size_t)p.R[1], INT_MIN);
  for (int i = 0; i < nreq; ++i) {
    // delay-line steps q = 1 .. T+1 of request i produce its outputs o = 4q + r - 6
    for (int64_t q = 1; q <= T[i] + 1; ++q) {
      ob01[(size_t)(a[0][i] + q)] = (int)(a[1][i] - 4 * a[0][i] - 6);
    }
    for (int64_t q = 1; q <= 4 * T[i] + 1; ++q) {
      ob12[(size_t)(a[1][i] + q)] = (int)(a[2][i] - 4 * a[1][i] - 6);
    }
  }
  // per-request tables: z offset, z channel stride, frames, level-0 row, conv_post first row,
  // tail frames, wav offset (dst - keep_lo), kept sample range
  constexpr int kTab = 9;
  std::vector<long long> tab((size_t)kTab * nreq);
  for (int i = 0; i < nreq; ++i) {
    long long *t = tab.data();
    t[0 * nreq + i] = w[i].z_off;
    t[1 * nreq + i] = w[i].z_ld;
    t[2 * nreq + i] = T[i];
    t[3 * nreq + i] = a[0][i];
    t[4 * nreq + i] = a[2][i] - 1;
    t[5 * nreq + i] = 16 * T[i] + 1;
    t[6 * nreq + i] = w[i].dst - w[i].keep_lo;
    t[7 * nreq + i] = w[i].keep_lo;
    t[8 * nreq + i] = w[i].keep_hi;
  }
  // gap-row ranges of every level: before the first request, between requests, after the last
  std::vector<long long> gap((size_t)3 * (nreq + 1) * 2);
  for (int l = 0; l < 3; ++l) {
    long long *g = gap.data() + (size_t)l * (nreq + 1) * 2;
    int64_t prev = 0;
    for (int i = 0; i <= nreq; ++i) {
      const int64_t next = i < nreq ? a[l][i] : p.R[l];
      g[2 * i] = prev;
      g[2 * i + 1] = next - prev;
      if (i < nreq) prev = a[l][i] + scale[l] * T[i];
    }
  }
  // one device block: masks, convT row maps, per-request tables, gap ranges
  auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
  size_t off[9], tot = 0;
  const size_t sz[9] = {(size_t)p.R[0], (size_t)p.R[1], (size_t)p.R[2], (size_t)p.R[2],
                        (size_t)p.R[2], ob01.size() * 4, ob12.size() * 4, tab.size() * 8,
                        gap.size() * 8};
  for (int k = 0; k < 9; ++k) {
    off[k] = tot;
    tot += al(sz[k]);
  }
  if (tot > p.table_cap) {
    // grow with headroom (half again), so that later plans of similar batches reuse the buffers
    if (p.table_block) cudaFree(p.table_block);
    if (p.host_stage) cudaFreeHost(p.host_stage);
    p.table_block = p.host_stage = nullptr;
    p.table_cap = 0;
    const size_t cap = al(tot + tot / 2);
    PTB_CUDA(cudaMalloc(&p.table_block, cap));
    PTB_CUDA(cudaMallocHost(&p.host_stage, cap));
    p.table_cap = cap;
  }
  char *base = static_cast<char *>(p.table_block);
  char *host = static_cast<char *>(p.host_stage);
  std::memcpy(host + off[0], m[0].data(), sz[0]);
  std::memcpy(host + off[1], m[1].data(), sz[1]);
  std::memcpy(host + off[2], m[2].data(), sz[2]);
  std::memcpy(host + off[3], mr.data(), sz[3]);
  std::memcpy(host + off[4], mp.data(), sz[4]);
  std::memcpy(host + off[5], ob01.data(), sz[5]);
  std::memcpy(host + off[6], ob12.data(), sz[6]);
  std::memcpy(host + off[7], tab.data(), sz[7]);
  std::memcpy(host + off[8], gap.data(), sz[8]);
  // from pinned memory: asynchronous, ordered before every later launch on `st`
  PTB_CUDA(cudaMemcpyAsync(base, host, tot, cudaMemcpyHostToDevice, st));
  p.gap = reinterpret_cast<long long *>(base + off[8]);
  for (int l = 0; l < 3; ++l) p.mask[l] = reinterpret_cast<unsigned char *>(base + off[l]);
  p.mask_refl = reinterpret_cast<unsigned char *>(base + off[3]);
  p.mask_post = reinterpret_cast<unsigned char *>(base + off[4]);
  p.ob01 = reinterpret_cast<int *>(base + off[5]);
  p.ob12 = reinterpret_cast<int *>(base + off[6]);
  long long *tb = reinterpret_cast<long long *>(base + off[7]);
  p.zoff = tb;
  p.zld = tb + nreq;
  p.Td = tb + 2 * nreq;
  p.a0 = tb + 3 * nreq;
  p.row0 = tb + 4 * nreq;
  p.tp = tb + 5 * nreq;
  p.wav0 = tb + 6 * nreq;
  p.klo = tb + 7 * nreq;
  p.khi = tb + 8 * nreq;
  p.table_bytes = tot;
  return 0;
}

void ptb::dec::free_plan(Plan &p) {
  if (p.table_block) cudaFree(p.table_block);
  if (p.host_stage) cudaFreeHost(p.host_stage);
  if (p.used) cudaEventDestroy(p.used);
  p = Plan();
}

namespace {

// Zero every gap row of the activation tensors: one block per (gap range, tensor); a gap range of
// a channels-last tensor is one contiguous run of rows x C floats (C a multiple of 4).
struct GapTargets {
  float *t[3][8];
  int c[3][8];
  int nt[3];
};

__global__ void zero_gaps_kernel(const long long *__restrict__ gap, int nrange, GapTargets tg) {
  const int l = blockIdx.x / nrange, r = blockIdx.x - l * nrange;
  if (blockIdx.y >= (unsigned)tg.nt[l]) return;
  const long long *g = gap + ((long long)l * nrange + r) * 2;
  const int C = tg.c[l][blockIdx.y];
  float4 *dst = reinterpret_cast<float4 *>(tg.t[l][blockIdx.y] + g[0] * C);
  const long long n4 = g[1] * C / 4;
  for (long long i = threadIdx.x; i < n4; i += blockDim.x) dst[i] = make_float4(0.f, 0.f, 0.f, 0.f);
}

// The activation tensors of the current plan, carved out of the decoder's buffer.
void carve(pt_b200_decoder *d) {
  const Plan &p = d->plan;
  const size_t r0 = (size_t)p.R[0], r1 = (size_t)p.R[1], r2 = (size_t)p.R[2];
  float *q = static_cast<float *>(d->act);
  auto take = [&](size_t n) {
    float *r = q;
    q += (n + 63) & ~(size_t)63;
    return r;
  };
  d->Z = take(r0 * 192);
  d->X0 = take(r0 * 512);
  d->U[0] = take(r1 * 256); d->LU[0] = take(r1 * 256); d->XB[0] = take(r1 * 256);
  d->XT[0] = take(r1 * 256); d->H[0] = take(r1 * 256); d->ACC[0] = take(r1 * 256);
  d->OUT1 = take(r1 * 256);
  d->U[1] = take(r2 * 128); d->LU[1] = take(r2 * 128); d->XB[1] = take(r2 * 128);
  d->XT[1] = take(r2 * 128); d->H[1] = take(r2 * 128); d->ACC[1] = take(r2 * 128);
  d->P = take(r2 * 128);
  d->POST = take(r2 * 80);
}

size_t act_floats(const Plan &p) {
  const size_t r0 = (size_t)p.R[0], r1 = (size_t)p.R[1], r2 = (size_t)p.R[2];
  return r0 * 192 + r0 * 512 + 7 * r1 * 256 + 7 * r2 * 128 + r2 * 80 + 64 * 24;
}

// Forget every captured decode graph (they hold the activation buffers' old addresses).
void drop_graphs(pt_b200_decoder *d) {
  for (int i = 0; i < pt_b200_decoder::kGraphs; ++i) {
    if (d->gexec[i]) cudaGraphExecDestroy(d->gexec[i]);
    d->gexec[i] = nullptr;
    d->g_key[i] = pt_b200_decoder::GKey{};
    d->g_seen[i] = pt_b200_decoder::GKey{};
  }
}

// Make the layout of these requests the current plan: the current one if it matches, a spare
// one that matches (no rebuild), or a new one built into the buffers of the least recently used
// spare plan once that plan's last decode has finished.  Then make sure the activation buffers
// hold this plan's tensors and read zeros in its gap rows (rows another layout used for data are
// cleared on every switch).  Everything is enqueued on `st`, so later work there is ordered
// after it.
int build_plan(pt_b200_decoder *d, cudaStream_t st, int nreq, const pt_b200_window *w) {
  if (!(d->have_plan && same_windows(d->plan.W, nreq, w))) {
    if (check_windows(nreq, w)) return -1;
    int hit = -1;
    for (int i = 0; i < (int)d->spare.size() && hit < 0; ++i)
      if (same_windows(d->spare[i].W, nreq, w)) hit = i;
    Plan next;
    if (hit >= 0) {
      next = std::move(d->spare[(size_t)hit]);
      d->spare.erase(d->spare.begin() + hit);
    } else {
      if ((int)d->spare.size() >= pt_b200_decoder::kSparePlans) {
        Plan old = std::move(d->spare.back());
        d->spare.pop_back();
        if (old.used) PTB_CUDA(cudaEventSynchronize(old.used));
        next.table_block = old.table_block;
        next.host_stage = old.host_stage;
        next.table_cap = old.table_cap;
        next.used = old.used;
      } else if (!d->free_tabs.empty()) {
        Plan t = std::move(d->free_tabs.back());
        d->free_tabs.pop_back();
        next.table_block = t.table_block;
        next.host_stage = t.host_stage;
        next.table_cap = t.table_cap;
      }
      if (!next.used) PTB_CUDA(cudaEventCreateWithFlags(&next.used, cudaEventDisableTiming));
      next.id = ++d->plan_id;
      if (build_layout(next, st, nreq, w)) {
        free_plan(next);
        return -1;
      }
      if (next.id == 1) {
        // the first plan: the buffers of the plans that can be cached beside it, at its size
        for (int k = 0; k < pt_b200_decoder::kSparePlans; ++k) {
          d->free_tabs.emplace_back();
          Plan &t = d->free_tabs.back();
          PTB_CUDA(cudaMalloc(&t.table_block, next.table_cap));
          PTB_CUDA(cudaMallocHost(&t.host_stage, next.table_cap));
          t.table_cap = next.table_cap;
        }
      }
    }
    if (d->have_plan) d->spare.insert(d->spare.begin(), std::move(d->plan));
    d->plan = std::move(next);
    d->have_plan = true;
    const size_t need = act_floats(d->plan) * 4;
    if (need > d->act_bytes) {
      // grow (with headroom) once every decode that used the old buffers has finished
      if (d->done) PTB_CUDA(cudaEventSynchronize(d->done));
      PTB_CUDA(cudaDeviceSynchronize());
      drop_graphs(d);
      if (d->act) cudaFree(d->act);
      d->act = nullptr;
      d->act_bytes = 0;
      // half again as much: batches of the same workload vary by tens of percent, and each
      // growth waits for the device and drops the captured graphs
      const size_t cap = need + need / 2;
      PTB_CUDA(cudaMalloc(&d->act, cap));
      PTB_CUDA(cudaMemsetAsync(d->act, 0, cap, st));
      d->act_bytes = cap;
      d->act_plan = d->plan.id;
    }
    carve(d);
  }
  if (d->act_plan != d->plan.id) {
    const Plan &p = d->plan;
    GapTargets tg{};
    float *l0[] = {d->Z, d->X0};
    const int c0[] = {192, 512};
    float *l1[] = {d->U[0], d->LU[0], d->XB[0], d->XT[0], d->H[0], d->ACC[0], d->OUT1};
    float *l2[] = {d->U[1], d->LU[1], d->XB[1], d->XT[1], d->H[1], d->ACC[1], d->P, d->POST};
    tg.nt[0] = 2;
    tg.nt[1] = 7;
    tg.nt[2] = 8;
    for (int i = 0; i < 2; ++i) tg.t[0][i] = l0[i], tg.c[0][i] = c0[i];
    for (int i = 0; i < 7; ++i) tg.t[1][i] = l1[i], tg.c[1][i] = 256;
    for (int i = 0; i < 8; ++i) tg.t[2][i] = l2[i], tg.c[2][i] = i == 7 ? 80 : 128;
    const int nrange = (int)p.T.size() + 1;
    zero_gaps_kernel<<<dim3((unsigned)(3 * nrange), 8), 256, 0, st>>>(p.gap, nrange, tg);
    PTB_CUDA(cudaGetLastError());
    count_launch();
    d->act_plan = p.id;
  }
  return 0;
}

}  // namespace

int ptb::dec::run_conv(pt_b200_decoder *d, cudaStream_t st, const DLayer &L, const float *act,
                       int64_t rows, int row_off0, int row_step, const EpiParams &e,
                       const int2 *tiles, int ntiles, int reverse) {
  ConvLaunch c{};
  c.act = act;
  c.act_rows = rows;
  c.batch = 1;
  c.w = L.w;
  c.bn = L.bn;
  c.g.m_rows = (int)rows;
  c.g.n_cols = L.n_pad;
  c.g.cin32 = L.cin32;
  c.g.ntap = L.ntap;
  c.g.row_off0 = row_off0;
  c.g.row_step = row_step;
  c.g.nkb = L.ntap * (L.cin32 / kBK);
  c.g.tiles = tiles;
  c.g.ntiles = ntiles;
  c.g.reverse = reverse;
  c.e = e;
  c.e.bias = L.b;
  return launch_conv(c, d->gerr, st);
}

EpiParams ptb::dec::rows_epi(const unsigned char *mask, int ldc) {
  EpiParams e{};
  e.mode = EPI_ROWS;
  e.mask = mask;
  e.nstore = ldc;
  e.ldc = ldc;
  e.ldc1 = ldc;
  e.alpha1 = kLr;
  return e;
}

namespace {

// launch kinds reported by pt_b200_decoder_launch_times
enum { LK_STAGE = 0, LK_CONV = 1, LK_CONVT = 2, LK_POST = 3, LK_TAIL = 4 };

// channels-last rows [r0, r0 + L) x C of a [rows][ld] tensor -> channel-major [C][L]
__global__ void unstage_rows_kernel(const float *__restrict__ src, int ld, long long r0,
                                    long long L, int C, float *__restrict__ dst) {
  __shared__ float tile[32][33];
  const long long t0 = (long long)blockIdx.x * 32;
  const int c0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const long long t = t0 + i;
    const int c = c0 + threadIdx.x;
    tile[i][threadIdx.x] = (t < L && c < C) ? src[(r0 + t) * ld + c] : 0.0f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int c = c0 + i;
    const long long t = t0 + threadIdx.x;
    if (c < C && t < L) dst[(long long)c * L + t] = tile[threadIdx.x][i];
  }
}

// checkpoint `layer` (pt_b200_decoder_checkpoints): rows [r0, r0 + L) x C of a [rows][ld] tensor
int ckpt(pt_b200_decoder *d, cudaStream_t st, int layer, const float *src, int ld, int C,
         int64_t r0, int64_t L) {
  if (!d->ck_dev) return 0;
  dim3 grid((unsigned)((L + 31) / 32), (unsigned)((C + 31) / 32));
  unstage_rows_kernel<<<grid, dim3(32, 8), 0, st>>>(src, ld, r0, L, C, d->ck_dev + d->ck_off[layer]);
  PTB_CUDA(cudaGetLastError());
  count_launch();
  return 0;
}

// kind | (N tile << 8): the N tile names the conv kernel instance the launch used
void rec(pt_b200_decoder *d, cudaStream_t st, int kind, double flops, double bytes, int bn = 0) {
  if (!d->prof || d->nrec >= pt_b200_decoder::kMaxRec) return;
  cudaEventRecord(d->ev[d->nrec], st);
  d->rkind[d->nrec] = kind | (bn << 8);
  d->rflops[d->nrec] = flops;
  d->rbytes[d->nrec] = bytes;
  ++d->nrec;
}

int run_decoder(pt_b200_decoder *d, cudaStream_t st, const float *z_dev, float *wav_dev) {
  const Plan &p = d->plan;
  const int nreq = (int)p.T.size();
  d->nrec = 0;
  double frames = 0;  // sum of latent frames over the batch
  for (int64_t t : p.T) frames += (double)t;
  // algorithmic work of one conv layer over every request's valid rows (2 x MACs)
  auto cflops = [&](double rows, int cin, int cout, int K) { return 2.0 * rows * cin * cout * K; };
  // every other conv launch walks its tiles last to first, starting on the rows its producer
  // wrote last, which are still in L2
  int nconv = 0;
  auto rev = [&]() { return nconv++ & 1; };
  // latents -> level-0 rows
  rec(d, st, LK_STAGE, 0.0, frames * 192 * 8);
  {
    dim3 grid((unsigned)((p.max_T + 31) / 32), 1, (unsigned)nreq);
    stage_z_kernel<<<grid, dim3(32, 8), 0, st>>>(z_dev, p.zoff, p.zld, p.Td, p.a0, nullptr, d->Z);
    PTB_CUDA(cudaGetLastError());
    count_launch();
  }
  // conv_pre 192 -> 512, k7 p3, + LeakyRelu
  rec(d, st, LK_CONV, cflops(frames, 192, 512, 7), frames * (192 + 512) * 4, d->pre.bn);
  {
    EpiParams e = rows_epi(p.mask[0], 512);
    e.out1 = d->X0;
    if (run_conv(d, st, d->pre, d->Z, p.R[0], -3, 1, e, nullptr, 0, rev())) return -1;
    if (ckpt(d, st, 0, d->X0, 512, 512, p.a[0][0], p.T[0])) return -1;
  }
  const float *lvl_in = d->X0;
  for (int s = 0; s < 2; ++s) {
    const int C = s == 0 ? 256 : 128;
    const int64_t rin = p.R[s], rout = p.R[s + 1];
    const unsigned char *mk = p.mask[s + 1];
    const int64_t lo_rows = (s == 0 ? 4 : 16) * p.T[0];   // rows of request 0 (checkpoints)
    // ups.s: phase-decomposed convT, taps read delay-line rows g - j
    const double fin = frames * (s == 0 ? 1 : 4), fout = 4 * fin;
    rec(d, st, LK_CONVT, cflops(fin, 2 * C, C, 16), fin * 2 * C * 4 + fout * 2 * C * 4, d->ups[s].bn);
    {
      EpiParams e = rows_epi(mk, C);
      e.mode = EPI_ROWS_CONVT;
      e.obase = s == 0 ? p.ob01 : p.ob12;
      e.s = 4;
      e.cphase = C;
      e.out_rows = (int)rout;
      e.out0 = d->U[s];
      e.out1 = d->LU[s];
      if (run_conv(d, st, d->ups[s], lvl_in, rin, 0, -1, e, nullptr, 0, rev())) return -1;
      if (ckpt(d, st, 1 + 19 * s, d->U[s], C, C, p.a[s + 1][0], (s == 0 ? 4 : 16) * p.T[0]))
        return -1;
    }
    for (int rb = 0; rb < 3; ++rb) {
      const int r = 3 * s + rb, K = kK[rb];
      for (int j = 0; j < 3; ++j) {
        rec(d, st, LK_CONV, cflops(fout, C, C, K), fout * 2 * C * 4, d->rb1[r][j].bn);
        {  // convs1.j (+ LeakyRelu)
          EpiParams e = rows_epi(mk, C);
          e.out1 = d->H[s];
          const float *in = j == 0 ? d->LU[s] : d->XT[s];
          if (run_conv(d, st, d->rb1[r][j], in, rout, -kD[j] * (K - 1) / 2, kD[j], e, nullptr, 0,
                       rev()))
            return -1;
          if (ckpt(d, st, 2 + 19 * s + 6 * rb + 2 * j, d->H[s], C, C, p.a[s + 1][0], lo_rows))
            return -1;
        }
        // convs2 bytes: input + residual + outputs (+ the branch sum read by resblocks 1, 2)
        const int nio = j < 2 ? 4 : rb == 0 ? 3 : 4;
        rec(d, st, LK_CONV, cflops(fout, C, C, K), fout * nio * C * 4, d->rb2[r][j].bn);
        {  // convs2.j + residual (+ leaky for the next stage / branch sum)
          EpiParams e = rows_epi(mk, C);
          e.res = j == 0 ? d->U[s] : d->XB[s];
          if (j < 2) {
            e.out0 = d->XB[s];
            e.out1 = d->XT[s];
          } else if (rb == 0) {
            e.out0 = d->ACC[s];
          } else if (rb == 1) {
            e.accin = d->ACC[s];
            e.acc_mode = 2;
            e.out0 = d->ACC[s];
          } else {
            e.accin = d->ACC[s];
            e.acc_mode = 3;
            if (s == 0) {
              e.out1 = d->OUT1;
            } else {
              e.out1 = d->P;
              e.alpha1 = kLrFinal;
              e.mask = p.mask_refl;
              e.refl = 1;
            }
          }
          if (run_conv(d, st, d->rb2[r][j], d->H[s], rout, -(K - 1) / 2, 1, e, nullptr, 0, rev()))
            return -1;
          if (d->ck_dev) {
            const int li = 3 + 19 * s + 6 * rb + 2 * j;
            const float *o = e.out0 ? e.out0 : e.out1;
            const bool refl = j == 2 && rb == 2 && s == 1;   // the reflection-pad row in front
            if (ckpt(d, st, li, o, C, C, p.a[s + 1][0] - (refl ? 1 : 0), lo_rows + (refl ? 1 : 0)))
              return -1;
          }
        }
      }
    }
    lvl_in = d->OUT1;
  }
  // subband_conv_post 128 -> 72 (N tile 80), k7 p3, over the reflection-padded rows.  Its
  // epilogue computes each frame's 64 windowed iSTFT samples into POST (the tail's per-frame
  // phases), except in a checkpoint decode, which keeps conv_post's own output and runs the
  // whole tail after it.
  const double fpost = 16 * frames + nreq;
  const int fused = d->ck_dev ? 0 : 1;
  // (its FLOPs are the convolution's, the tensor-core work; the epilogue's per-frame arithmetic
  // is about 0.03 % on top)
  rec(d, st, LK_POST, cflops(fpost, 128, 72, 7), fpost * (128 + (fused ? 64 : 80)) * 4, d->post.bn);
  {
    EpiParams e = rows_epi(p.mask_post, 80);
    e.out0 = d->POST;
    e.frames = fused;
    if (run_conv(d, st, d->post, d->P, p.R[2], -3, 1, e, nullptr, 0, rev())) return -1;
    if (ckpt(d, st, 39, d->POST, 80, 72, p.a[2][0] - 1, 16 * p.T[0] + 1)) return -1;
  }
  // tail: algorithmic bytes = read the 72 conv_post channels (or the 64 frame samples) + write
  // the waveform
  rec(d, st, LK_TAIL,
      2.0 * ((fused ? 0 : 4 * 9 * 16 * 2) + 4 * 16 + 4 * 63 * 16) * fpost,
      fpost * (fused ? 64 : 72) * 4 + frames * 256 * 4);
  if (tail_run_rows(d->POST, 80, p.row0, p.tp, p.wav0, p.klo, p.khi, nullptr, 0, nreq,
                    16 * p.max_T + 1, d->pqmf, wav_dev, st, fused))
    return -1;
  if (d->prof) cudaEventRecord(d->ev[d->nrec], st);
  return 0;
}

}  // namespace

extern "C" {

pt_b200_decoder *pt_b200_decoder_create(int device, const pt_b200_dec_weights *w) {
  if (!w) {
    set_error("pt_b200: NULL decoder weights");
    return nullptr;
  }
  if (cudaSetDevice(device) != cudaSuccess) {
    set_error("pt_b200: cannot select device %d", device);
    return nullptr;
  }
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10 || prop.minor != 0) {
    set_error("pt_b200: device %d is not sm_100 (B200); this library has no other path", device);
    return nullptr;
  }
  auto *d = new pt_b200_decoder();
  d->device = device;
  auto fail = [&](const char *what) {
    fprintf(stderr, "pt_b200: decoder create failed at %s\n", what);
    pt_b200_decoder_destroy(d);
    return static_cast<pt_b200_decoder *>(nullptr);
  };
  if (cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&d->done, cudaEventDisableTiming) != cudaSuccess)
    return fail("stream");
  if (cudaMalloc(&d->gerr, 4) != cudaSuccess || cudaMemset(d->gerr, 0, 4) != cudaSuccess ||
      cudaMallocHost(&d->gerr_host, 4) != cudaSuccess)
    return fail("error word");
  *d->gerr_host = 0;
  cudaStream_t st = d->stream;
  if (make_layer(&d->pre, w->pre_w, w->pre_b, 512, 7, 192, 512, 1 << 30, st)) return fail("conv_pre");
  for (int s = 0; s < 2; ++s) {
    const int Cin = s == 0 ? 512 : 256, C = Cin / 2;
    if (make_layer(&d->ups[s], w->ups_w[s], w->ups_b[s], 4 * C, 4, Cin, C, C, st)) return fail("ups");
    for (int rb = 0; rb < 3; ++rb)
      for (int j = 0; j < 3; ++j) {
        const int r = 3 * s + rb;
        if (make_layer(&d->rb1[r][j], w->rb_w1[r][j], w->rb_b1[r][j], C, kK[rb], C, C, 1 << 30, st) ||
            make_layer(&d->rb2[r][j], w->rb_w2[r][j], w->rb_b2[r][j], C, kK[rb], C, C, 1 << 30, st))
          return fail("resblock");
      }
  }
  if (make_layer(&d->post, w->post_w, w->post_b, 72, 7, 128, 72, 1 << 30, st)) return fail("conv_post");
  if (cudaMalloc(&d->pqmf, 4 * 63 * 4) != cudaSuccess ||
      cudaMemcpy(d->pqmf, w->pqmf, 4 * 63 * 4, cudaMemcpyHostToDevice) != cudaSuccess)
    return fail("pqmf");
  // the iSTFT constants conv_post's frames epilogue and the tail read, on this device
  if (tail_prepare()) return fail("tail constants");
  return d;
}

void pt_b200_decoder_destroy(pt_b200_decoder *d) {
  if (!d) return;
  cudaSetDevice(d->device);
  if (d->stream) cudaStreamSynchronize(d->stream);
  auto fl = [](DLayer &L) {
    if (L.w) cudaFree(L.w);
    if (L.b) cudaFree(L.b);
  };
  fl(d->pre);
  fl(d->ups[0]);
  fl(d->ups[1]);
  for (int r = 0; r < 6; ++r)
    for (int j = 0; j < 3; ++j) {
      fl(d->rb1[r][j]);
      fl(d->rb2[r][j]);
    }
  fl(d->post);
  if (d->pqmf) cudaFree(d->pqmf);
  if (d->act) cudaFree(d->act);
  free_plan(d->plan);
  for (auto &p : d->spare) free_plan(p);
  for (auto &p : d->free_tabs) free_plan(p);
  if (d->zbuf) cudaFree(d->zbuf);
  if (d->wavbuf) cudaFree(d->wavbuf);
  if (d->gerr) cudaFree(d->gerr);
  if (d->gerr_host) cudaFreeHost(d->gerr_host);
  for (auto &e : d->ev)
    if (e) cudaEventDestroy(e);
  if (d->done) cudaEventDestroy(d->done);
  for (auto &g : d->gexec)
    if (g) cudaGraphExecDestroy(g);
  if (d->h2d) {
    cudaStreamSynchronize(d->h2d);
    cudaStreamDestroy(d->h2d);
  }
  if (d->d2h) {
    cudaStreamSynchronize(d->d2h);
    cudaStreamDestroy(d->d2h);
  }
  for (int s = 0; s < 2; ++s) {
    if (d->ev_up[s]) cudaEventDestroy(d->ev_up[s]);
    if (d->ev_dec[s]) cudaEventDestroy(d->ev_dec[s]);
    if (d->ev_down[s]) cudaEventDestroy(d->ev_down[s]);
    if (d->az[s]) cudaFree(d->az[s]);
    if (d->aw[s]) cudaFree(d->aw[s]);
  }
  if (d->stream) cudaStreamDestroy(d->stream);
  delete d;
}

int pt_b200_decode_windows(pt_b200_decoder *d, void *stream, int n, const pt_b200_window *w,
                           const float *z_dev, float *wav_dev) {
  PTB_REQUIRE(d && w && z_dev && wav_dev && n > 0, "pt_b200: bad decode arguments");
  std::lock_guard<std::mutex> lk(d->mu);
  PTB_CUDA(cudaSetDevice(d->device));
  cudaStream_t st = stream ? (cudaStream_t)stream : d->stream;
  if (build_plan(d, st, n, w)) return -1;
  if (d->graph_on < 0) d->graph_on = getenv("PT_B200_GRAPH") ? atoi(getenv("PT_B200_GRAPH")) : 1;
  const pt_b200_decoder::GKey key{d->plan.id, z_dev, wav_dev, st, d->prof};
  constexpr int NG = pt_b200_decoder::kGraphs;
  int hit = -1;
  bool seen = false;
  for (int i = 0; i < NG; ++i) {
    if (d->gexec[i] && key == d->g_key[i]) hit = i;
    if (key == d->g_seen[i]) seen = true;
  }
  // profiled decodes stay eager: events recorded by graph nodes cannot be timed
  if (d->graph_on && !d->prof && (hit >= 0 || seen)) {
    if (hit < 0) {
      // second identical call: capture the decode once (into the older slot), then replay it
      hit = d->g_next;
      d->g_next = (d->g_next + 1) % NG;
      if (d->gexec[hit]) cudaGraphExecDestroy(d->gexec[hit]);
      d->gexec[hit] = nullptr;
      d->g_key[hit] = pt_b200_decoder::GKey{};
      if (tail_prepare()) return -1;   // one-time constant uploads happen outside the capture
      const long before = launches(0);
      PTB_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
      const int rc = run_decoder(d, st, z_dev, wav_dev);
      cudaGraph_t g = nullptr;
      const cudaError_t ec = cudaStreamEndCapture(st, &g);
      const long captured = launches(0) - before;
      count_launch(-captured);   // capturing launches nothing
      if (rc || ec != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        PTB_REQUIRE(false, "pt_b200: decode graph capture failed (%s)", cudaGetErrorString(ec));
      }
      const cudaError_t ei = cudaGraphInstantiate(&d->gexec[hit], g, 0);
      cudaGraphDestroy(g);
      PTB_CUDA(ei);
      d->g_kernels[hit] = captured;
      d->g_key[hit] = key;
    }
    PTB_CUDA(cudaGraphLaunch(d->gexec[hit], st));
    count_launch(d->g_kernels[hit]);
  } else {
    d->g_seen[d->g_seen_next] = key;
    d->g_seen_next = (d->g_seen_next + 1) % NG;
    if (run_decoder(d, st, z_dev, wav_dev)) return -1;
  }
  PTB_CUDA(cudaEventRecord(d->plan.used, st));
  PTB_CUDA(cudaEventRecord(d->done, st));
  return 0;
}

int pt_b200_decode_batch_device(pt_b200_decoder *d, void *stream, int nreq, const int64_t *T,
                                const float *z_dev, float *wav_dev) {
  PTB_REQUIRE(d && T && z_dev && wav_dev && nreq > 0, "pt_b200: bad decode arguments");
  // whole utterances: request i reads its own [192][T_i] block and keeps every sample
  std::vector<pt_b200_window> w((size_t)nreq);
  int64_t zo = 0, wo = 0;
  for (int i = 0; i < nreq; ++i) {
    w[i].frames = T[i];
    w[i].z_off = zo;
    w[i].z_ld = T[i];
    w[i].keep_lo = 0;
    w[i].keep_hi = 256 * T[i];
    w[i].dst = wo;
    zo += 192 * T[i];
    wo += 256 * T[i];
  }
  return pt_b200_decode_windows(d, stream, nreq, w.data(), z_dev, wav_dev);
}

int64_t pt_b200_stream_plan(int nstreams, const int64_t *T, int win, int ctx, int exact,
                            pt_b200_window *out, int64_t cap) {
  PTB_REQUIRE(nstreams > 0 && T && win > 0 && ctx >= 0 && (cap == 0 || out),
              "pt_b200: bad stream plan arguments");
  const int64_t step = win - 2 * ctx > 1 ? win - 2 * ctx : 1;
  int64_t nw = 0, zo = 0, wo = 0;
  auto put = [&](int64_t a, int64_t frames, int64_t lo, int64_t hi, int64_t dst, int64_t Ts) {
    if (nw < cap) out[nw] = pt_b200_window{frames, zo + a, Ts, lo, hi, dst};
    ++nw;
  };
  for (int s = 0; s < nstreams; ++s) {
    const int64_t Ts = T[s];
    PTB_REQUIRE(Ts >= 2, "pt_b200: stream %d has %lld frames (need >= 2)", s, (long long)Ts);
    if (!exact) {
      // the reference's overlap-save loop (runtime/v21/src/main_v21.c:342-364)
      int64_t olen = 0;
      for (int64_t a = 0;; a += step) {
        const int64_t we = a + win > Ts ? Ts - a : win;
        const bool first = a == 0, last = a + we >= Ts;
        const int64_t n = 256 * we;
        const int64_t lo = first ? 0 : 256 * (int64_t)ctx;
        int64_t hi = last ? n : 256 * (we - ctx);
        if (hi > n) hi = n;
        if (hi > lo) {
          put(a, we, lo, hi, wo + olen, Ts);
          olen += hi - lo;
        }
        if (last) break;
      }
    } else {
      // same emission schedule, context widened to the receptive radius
      const int64_t cl = ctx > kReachLeft ? ctx : kReachLeft, cr = ctx > kReachRight ? ctx : kReachRight;
      for (int64_t e = 0; e < Ts; e += step) {
        const int64_t e1 = e + step < Ts ? e + step : Ts;
        const int64_t a = e - cl > 0 ? e - cl : 0, b = e1 + cr < Ts ? e1 + cr : Ts;
        put(a, b - a, 256 * (e - a), 256 * (e1 - a), wo + 256 * e, Ts);
      }
    }
    zo += 192 * Ts;
    wo += 256 * Ts;
  }
  return nw;
}

int pt_b200_stream_decode(pt_b200_decoder *d, void *stream, int nstreams, const int64_t *T,
                          const float *z_dev, int win, int ctx, int exact, int64_t max_frames,
                          float *wav_dev) {
  PTB_REQUIRE(d && T && z_dev && wav_dev && nstreams > 0, "pt_b200: bad stream arguments");
  const int64_t nw = pt_b200_stream_plan(nstreams, T, win, ctx, exact, nullptr, 0);
  if (nw < 0) return -1;
  std::vector<pt_b200_window> w((size_t)nw);
  pt_b200_stream_plan(nstreams, T, win, ctx, exact, w.data(), nw);
  if (max_frames <= 0) max_frames = kStreamBatchFrames;
  // windows in plan order, batched up to max_frames latent frames
  for (int64_t i = 0; i < nw;) {
    int64_t j = i, fr = 0;
    while (j < nw && (j == i || fr + w[j].frames <= max_frames) && j - i < INT_MAX) fr += w[j++].frames;
    if (pt_b200_decode_windows(d, stream, (int)(j - i), w.data() + i, z_dev, wav_dev)) return -1;
    i = j;
  }
  return 0;
}

int pt_b200_decoder_sync(pt_b200_decoder *d, void *stream) {
  PTB_REQUIRE(d, "pt_b200: NULL decoder");
  PTB_CUDA(cudaSetDevice(d->device));
  cudaStream_t st = stream ? (cudaStream_t)stream : d->stream;
  PTB_CUDA(cudaMemcpyAsync(d->gerr_host, d->gerr, 4, cudaMemcpyDeviceToHost, st));
  PTB_CUDA(cudaStreamSynchronize(st));
  if (*d->gerr_host) {
    set_error("pt_b200: decoder device error word 0x%x", *d->gerr_host);
    *d->gerr_host = 0;
    cudaMemset(d->gerr, 0, 4);
    return -1;
  }
  return 0;
}

int pt_b200_decode_batch(pt_b200_decoder *d, void *stream, int nreq, const int64_t *T,
                         const float *z_host, float *wav_host) {
  PTB_REQUIRE(d && T && z_host && wav_host && nreq > 0, "pt_b200: bad decode arguments");
  int64_t nz = 0, nw = 0;
  for (int i = 0; i < nreq; ++i) {
    nz += 192 * T[i];
    nw += 256 * T[i];
  }
  {
    std::lock_guard<std::mutex> lk(d->mu);
    PTB_CUDA(cudaSetDevice(d->device));
    if ((size_t)nz * 4 > d->zbuf_bytes) {
      if (d->zbuf) cudaFree(d->zbuf);
      d->zbuf = nullptr;
      d->zbuf_bytes = 0;
      PTB_CUDA(cudaMalloc(&d->zbuf, (size_t)nz * 4));
      d->zbuf_bytes = (size_t)nz * 4;
    }
    if ((size_t)nw * 4 > d->wavbuf_bytes) {
      if (d->wavbuf) cudaFree(d->wavbuf);
      d->wavbuf = nullptr;
      d->wavbuf_bytes = 0;
      PTB_CUDA(cudaMalloc(&d->wavbuf, (size_t)nw * 4));
      d->wavbuf_bytes = (size_t)nw * 4;
    }
  }
  cudaStream_t st = stream ? (cudaStream_t)stream : d->stream;
  PTB_CUDA(cudaMemcpyAsync(d->zbuf, z_host, (size_t)nz * 4, cudaMemcpyHostToDevice, st));
  if (pt_b200_decode_batch_device(d, st, nreq, T, d->zbuf, d->wavbuf)) return -1;
  PTB_CUDA(cudaMemcpyAsync(wav_host, d->wavbuf, (size_t)nw * 4, cudaMemcpyDeviceToHost, st));
  return pt_b200_decoder_sync(d, st);
}

namespace {

// the upload / download streams and the per-slot events of the pipelined entry point
int async_setup(pt_b200_decoder *d) {
  if (d->h2d) return 0;
  PTB_CUDA(cudaStreamCreateWithFlags(&d->h2d, cudaStreamNonBlocking));
  PTB_CUDA(cudaStreamCreateWithFlags(&d->d2h, cudaStreamNonBlocking));
  for (int s = 0; s < 2; ++s) {
    PTB_CUDA(cudaEventCreateWithFlags(&d->ev_up[s], cudaEventDisableTiming));
    PTB_CUDA(cudaEventCreateWithFlags(&d->ev_dec[s], cudaEventDisableTiming));
    PTB_CUDA(cudaEventCreateWithFlags(&d->ev_down[s], cudaEventDisableTiming));
  }
  return 0;
}

}  // namespace

int pt_b200_decode_batch_async(pt_b200_decoder *d, int nreq, const int64_t *T, const float *z_host,
                               float *wav_host) {
  PTB_REQUIRE(d && T && z_host && wav_host && nreq > 0, "pt_b200: bad decode arguments");
  int64_t nz = 0, nw = 0;
  for (int i = 0; i < nreq; ++i) {
    nz += 192 * T[i];
    nw += 256 * T[i];
  }
  int s = 0;
  {
    std::lock_guard<std::mutex> lk(d->mu);
    PTB_CUDA(cudaSetDevice(d->device));
    if (async_setup(d)) return -1;
    if ((size_t)nz * 4 > d->az_bytes || (size_t)nw * 4 > d->aw_bytes) {
      // grow both slots once nothing in flight uses them, by half again so that a stream of
      // ragged batches does not stop the pipeline at every new largest batch
      PTB_CUDA(cudaStreamSynchronize(d->h2d));
      PTB_CUDA(cudaStreamSynchronize(d->stream));
      PTB_CUDA(cudaStreamSynchronize(d->d2h));
      for (int k = 0; k < 2; ++k) {
        if (d->az[k]) cudaFree(d->az[k]);
        if (d->aw[k]) cudaFree(d->aw[k]);
        d->az[k] = d->aw[k] = nullptr;
        d->slot_used[k] = false;
      }
      d->az_bytes = d->aw_bytes = 0;
      const size_t zb = (size_t)(nz + nz / 2) * 4, wb = (size_t)(nw + nw / 2) * 4;
      for (int k = 0; k < 2; ++k) {
        PTB_CUDA(cudaMalloc(&d->az[k], zb));
        PTB_CUDA(cudaMalloc(&d->aw[k], wb));
      }
      d->az_bytes = zb;
      d->aw_bytes = wb;
    }
    s = d->async_next;
    d->async_next ^= 1;
    // upload into slot s once the decode that read it last has finished
    if (d->slot_used[s]) PTB_CUDA(cudaStreamWaitEvent(d->h2d, d->ev_dec[s], 0));
    PTB_CUDA(cudaMemcpyAsync(d->az[s], z_host, (size_t)nz * 4, cudaMemcpyHostToDevice, d->h2d));
    PTB_CUDA(cudaEventRecord(d->ev_up[s], d->h2d));
    // the decode waits for its upload and for the download that last read its output slot
    PTB_CUDA(cudaStreamWaitEvent(d->stream, d->ev_up[s], 0));
    if (d->slot_used[s]) PTB_CUDA(cudaStreamWaitEvent(d->stream, d->ev_down[s], 0));
  }
  if (pt_b200_decode_batch_device(d, d->stream, nreq, T, d->az[s], d->aw[s])) return -1;
  std::lock_guard<std::mutex> lk(d->mu);
  PTB_CUDA(cudaEventRecord(d->ev_dec[s], d->stream));
  PTB_CUDA(cudaStreamWaitEvent(d->d2h, d->ev_dec[s], 0));
  PTB_CUDA(cudaMemcpyAsync(wav_host, d->aw[s], (size_t)nw * 4, cudaMemcpyDeviceToHost, d->d2h));
  PTB_CUDA(cudaEventRecord(d->ev_down[s], d->d2h));
  d->slot_used[s] = true;
  return 0;
}

int pt_b200_decode_async_wait(pt_b200_decoder *d) {
  PTB_REQUIRE(d, "pt_b200: NULL decoder");
  PTB_CUDA(cudaSetDevice(d->device));
  if (d->d2h) PTB_CUDA(cudaStreamSynchronize(d->d2h));   // downloads follow every decode
  return pt_b200_decoder_sync(d, d->stream);
}

int pt_b200_decode_async_streams(pt_b200_decoder *d, void **upload, void **decode, void **download) {
  PTB_REQUIRE(d, "pt_b200: NULL decoder");
  std::lock_guard<std::mutex> lk(d->mu);
  PTB_CUDA(cudaSetDevice(d->device));
  if (async_setup(d)) return -1;
  if (upload) *upload = d->h2d;
  if (decode) *decode = d->stream;
  if (download) *download = d->d2h;
  return 0;
}

int pt_b200_decoder_profile(pt_b200_decoder *d, int enable) {
  PTB_REQUIRE(d, "pt_b200: NULL decoder");
  std::lock_guard<std::mutex> lk(d->mu);
  PTB_CUDA(cudaSetDevice(d->device));
  if (enable && !d->ev[0])
    for (int i = 0; i <= pt_b200_decoder::kMaxRec; ++i) PTB_CUDA(cudaEventCreate(&d->ev[i]));
  d->prof = enable != 0;
  d->nrec = 0;
  return 0;
}

int pt_b200_decoder_launch_times(pt_b200_decoder *d, int max, double *ms, double *flops,
                                 double *bytes, int *kind) {
  PTB_REQUIRE(d && d->prof, "pt_b200: decoder profiling is off");
  std::lock_guard<std::mutex> lk(d->mu);
  PTB_CUDA(cudaSetDevice(d->device));
  const int n = d->nrec < max ? d->nrec : max;
  for (int i = 0; i < n; ++i) {
    float t = 0.0f;
    PTB_CUDA(cudaEventElapsedTime(&t, d->ev[i], d->ev[i + 1]));
    ms[i] = t;
    flops[i] = d->rflops[i];
    bytes[i] = d->rbytes[i];
    kind[i] = d->rkind[i];
  }
  return n;
}

int pt_b200_decoder_checkpoints(pt_b200_decoder *d, const float *z_host, int64_t T,
                                float *const *ckpt_host, float *wav_host) {
  PTB_REQUIRE(d && z_host && ckpt_host && wav_host && T >= 2, "pt_b200: bad checkpoint arguments");
  // element counts of the 40 layer outputs (include/pt_b200.h)
  int64_t n[PT_B200_NCKPT];
  n[0] = 512 * T;
  for (int s = 0; s < 2; ++s) {
    const int64_t C = s == 0 ? 256 : 128, L = (s == 0 ? 4 : 16) * T;
    for (int i = 0; i < 19; ++i) n[1 + 19 * s + i] = C * L;
  }
  n[38] = 128 * (16 * T + 1);
  n[39] = 72 * (16 * T + 1);
  int64_t tot = 0;
  for (int i = 0; i < PT_B200_NCKPT; ++i) {
    d->ck_off[i] = tot;
    tot += (n[i] + 63) & ~(int64_t)63;
  }
  std::lock_guard<std::mutex> lk(d->mu);
  PTB_CUDA(cudaSetDevice(d->device));
  cudaStream_t st = d->stream;
  float *zd = nullptr, *wd = nullptr, *ck = nullptr;
  auto release = [&]() {
    d->ck_dev = nullptr;
    cudaStreamSynchronize(st);
    if (zd) cudaFree(zd);
    if (wd) cudaFree(wd);
    if (ck) cudaFree(ck);
  };
  int rc = -1;
  do {
    if (cudaMalloc(&zd, (size_t)T * 192 * 4) != cudaSuccess ||
        cudaMalloc(&wd, (size_t)T * 256 * 4) != cudaSuccess ||
        cudaMalloc(&ck, (size_t)tot * 4) != cudaSuccess) {
      set_error("pt_b200: checkpoint buffers: out of device memory");
      break;
    }
    if (cudaMemcpyAsync(zd, z_host, (size_t)T * 192 * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
      break;
    pt_b200_window w{T, 0, T, 0, 256 * T, 0};
    if (build_plan(d, st, 1, &w)) break;
    d->ck_dev = ck;
    if (run_decoder(d, st, zd, wd)) break;
    d->ck_dev = nullptr;
    if (cudaEventRecord(d->plan.used, st) != cudaSuccess || cudaEventRecord(d->done, st) != cudaSuccess)
      break;
    if (cudaMemcpyAsync(wav_host, wd, (size_t)T * 256 * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
      break;
    bool ok = true;
    for (int i = 0; i < PT_B200_NCKPT && ok; ++i)
      if (ckpt_host[i])
        ok = cudaMemcpyAsync(ckpt_host[i], ck + d->ck_off[i], (size_t)n[i] * 4,
                             cudaMemcpyDeviceToHost, st) == cudaSuccess;
    if (!ok) break;
    rc = 0;
  } while (false);
  if (rc) {
    release();
    return -1;
  }
  release();
  // device errors of the decode (the error word) -- the lock is still held, so check here
  PTB_CUDA(cudaMemcpy(d->gerr_host, d->gerr, 4, cudaMemcpyDeviceToHost));
  if (*d->gerr_host) {
    set_error("pt_b200: decoder device error word 0x%x", *d->gerr_host);
    *d->gerr_host = 0;
    cudaMemset(d->gerr, 0, 4);
    return -1;
  }
  return 0;
}

int pt_v21_decode(pt_ctx *c, const pt_b200_decoder *d, const float *z, int64_t T, float *wav) {
  PTB_REQUIRE(c && c->use_cuda && c->g_stream, "pt_b200: context is not initialised for the GPU");
  return pt_b200_decode_batch(const_cast<pt_b200_decoder *>(d), c->g_stream, 1, &T, z, wav);
}

}  // extern "C"
