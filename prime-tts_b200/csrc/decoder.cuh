// decoder.cuh -- internals shared by the batched decoder (decoder.cu) and the carried-state
// streaming executor (carry.cu): the layer table, the ragged row layout and the decoder object.
#pragma once
#include <climits>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/pt_b200.h"
#include "common.cuh"

namespace ptb {
int tail_prepare();
int tail_run_rows(const float *post_dev, long long ld, const long long *row0, const long long *tp,
                  const long long *wav0, const long long *klo, const long long *khi,
                  const long long *jbase, long long chunks, int nreq, long long max_tp,
                  const float *pqmf_dev, float *wav_dev, cudaStream_t st, int frames);

namespace dec {

// Zero rows between requests at each level (level 0: latent frames, 1: 4x, 2: 16x), at least 16
// so that a 16-row epilogue pass rounded outward from one request never reaches the next one:
// conv_pre reaches 3 rows, ups.0 reads 2 before / 1 after a request, the widest level-1/2 conv
// reaches dilation 5 x (11-1)/2 = 25 rows, conv_post reads 3 + 1 reflection row.
constexpr int64_t kGap[3] = {16, 28, 32};
// rows before the first request; level 2 starts every request at a row = 4 (mod 16) (a lead of
// 36, gaps of 32, request lengths 16T), so a request's reflection row (-1) and its source (+1)
// fall in the same 16-row epilogue pass
constexpr int64_t kLead[3] = {16, 28, 36};
// receptive radius of one output sample, in latent frames before / after its own frame
// (PQMF 63 taps, overlap-add, conv_post k7, two MRF blocks reaching 60 rows, two k16/s4 convT,
// conv_pre k7, propagated back to the latent)
constexpr int64_t kReachLeft = 25, kReachRight = 24;
constexpr int kK[3] = {3, 7, 11};
constexpr int kD[3] = {1, 3, 5};
constexpr float kLr = 0.10000000149011612f;
constexpr float kLrFinal = 0.009999999776482582f;

struct DLayer {
  float *w = nullptr, *b = nullptr;  // [n_pad][ntap][cin32] tf32, bias [round_up(n_pad, 32)]
  int n_pad = 0, bn = 0, cin32 = 0, ntap = 0;
};

// First row of every request at each level, and the rows of each level: a lead, then per request
// its rows (T, 4T, 16T) and a zero gap.
inline void layout_rows(const int64_t *T, int n, std::vector<int64_t> a[3], int64_t R[3]) {
  const int64_t scale[3] = {1, 4, 16};
  for (int l = 0; l < 3; ++l) {
    a[l].clear();
    int64_t off = kLead[l];
    for (int i = 0; i < n; ++i) {
      a[l].push_back(off);
      off += scale[l] * T[i] + kGap[l];
    }
    R[l] = off;
  }
}

// The ragged row layout of a set of requests and its device tables.
struct Plan {
  std::vector<pt_b200_window> W;   // the requests this plan lays out
  std::vector<int64_t> T;
  std::vector<int64_t> a[3];       // first row of every request at each level
  int64_t R[3] = {0, 0, 0};
  int64_t max_T = 0, total_z = 0, total_wav = 0;
  // device tables
  unsigned char *mask[3] = {nullptr, nullptr, nullptr};
  unsigned char *mask_refl = nullptr, *mask_post = nullptr;
  int *ob01 = nullptr, *ob12 = nullptr;
  long long *zoff = nullptr, *zld = nullptr, *Td = nullptr, *a0 = nullptr;
  long long *row0 = nullptr, *tp = nullptr, *wav0 = nullptr, *klo = nullptr, *khi = nullptr;
  long long *gap = nullptr;        // per level l: nreq + 1 gap-row ranges {first row, rows}
  void *table_block = nullptr;     // device tables (reused by later plans: table_cap bytes)
  void *host_stage = nullptr;      // pinned host copy the tables are uploaded from (table_cap)
  size_t table_bytes = 0, table_cap = 0;
  uint64_t id = 0;                 // unique per layout (graph keys, gap-row bookkeeping)
  cudaEvent_t used = nullptr;      // recorded after each decode that read the device tables
};

// Lay the requests out and upload the tables (masks, convT row maps, per-request tables, gap
// ranges) on `st`, asynchronously from p.host_stage.  Reuses p.table_block / p.host_stage when
// they are large enough (the caller makes sure no earlier upload or decode still uses them).
int build_layout(Plan &p, cudaStream_t st, int nreq, const pt_b200_window *w);
// Free a plan's device tables, staging buffer and event.
void free_plan(Plan &p);

// one conv layer over the rows of a level (all of them, or the tile list {first row, rows})
int run_conv(pt_b200_decoder *d, cudaStream_t st, const DLayer &L, const float *act, int64_t rows,
             int row_off0, int row_step, const EpiParams &e, const int2 *tiles = nullptr,
             int ntiles = 0, int reverse = 0);
EpiParams rows_epi(const unsigned char *mask, int ldc);

// latents -> level-0 rows: frames [f0, T) of every request (f0 null: from 0), tf32-rounded
__global__ void stage_z_kernel(const float *__restrict__ z, const long long *__restrict__ zoff,
                               const long long *__restrict__ zld, const long long *__restrict__ T,
                               const long long *__restrict__ a0, const long long *__restrict__ f0,
                               float *__restrict__ Z);

}  // namespace dec
}  // namespace ptb

struct pt_b200_decoder {
  int device = 0;
  cudaStream_t stream = nullptr;
  uint32_t *gerr = nullptr, *gerr_host = nullptr;
  ptb::dec::DLayer pre, ups[2], rb1[6][3], rb2[6][3], post;
  float *pqmf = nullptr;
  std::mutex mu;
  ptb::dec::Plan plan;
  bool have_plan = false;
  // recently used layouts with their device tables, most recent first: a batch seen again (or
  // pipelined batches that alternate) switches back without rebuilding, and a new batch reuses the
  // least recently used plan's buffers instead of allocating
  static constexpr int kSparePlans = 4;
  std::vector<ptb::dec::Plan> spare;
  // table buffers (device block + pinned staging) made beside the first plan's, one for each plan
  // that can be cached, so that the first new batches after it allocate nothing (pinned
  // allocations take milliseconds, more on a loaded host)
  std::vector<ptb::dec::Plan> free_tabs;
  uint64_t act_plan = ~0ull;    // plan whose gap rows are zero in the activation buffers
  cudaEvent_t done = nullptr;   // recorded after every decode: plan changes wait for it
  uint64_t plan_id = 0;         // bumped whenever the plan (tables, buffers) changes
  // CUDA graphs of the whole decode: captured on the second identical call (same plan, latents,
  // output and stream), replayed after that; two are kept, so the two staging slots of the
  // pipelined host entry point both replay; PT_B200_GRAPH=0 keeps every decode eager
  static constexpr int kGraphs = 2;
  int graph_on = -1;
  cudaGraphExec_t gexec[kGraphs] = {};
  long g_kernels[kGraphs] = {};  // kernels per replay (for pt_b200_kernel_launches)
  int g_next = 0, g_seen_next = 0;
  struct GKey {
    uint64_t plan = ~0ull;
    const void *z = nullptr;
    void *wav = nullptr;
    cudaStream_t st = nullptr;
    bool prof = false;
    bool operator==(const GKey &o) const {
      return plan == o.plan && z == o.z && wav == o.wav && st == o.st && prof == o.prof;
    }
  } g_key[kGraphs], g_seen[kGraphs];
  // activation buffers (grown on demand, zeroed when the plan changes)
  void *act = nullptr;
  size_t act_bytes = 0;
  float *Z = nullptr, *X0 = nullptr;
  float *U[2], *LU[2], *XB[2], *XT[2], *H[2], *ACC[2], *OUT1 = nullptr, *P = nullptr, *POST = nullptr;
  float *zbuf = nullptr, *wavbuf = nullptr;  // staging for the host-buffer entry point
  size_t zbuf_bytes = 0, wavbuf_bytes = 0;
  // pipelined host-buffer decodes (pt_b200_decode_batch_async): two staging slots, an upload and
  // a download stream beside the decode stream
  cudaStream_t h2d = nullptr, d2h = nullptr;
  cudaEvent_t ev_up[2] = {}, ev_dec[2] = {}, ev_down[2] = {};
  bool slot_used[2] = {false, false};
  float *az[2] = {}, *aw[2] = {};
  size_t az_bytes = 0, aw_bytes = 0;
  int async_next = 0;
  // per-layer checkpoints (pt_b200_decoder_checkpoints): when ck_dev is set, a one-request decode
  // copies each conv launch's output, channel-major, to ck_dev + ck_off[layer]
  float *ck_dev = nullptr;
  int64_t ck_off[PT_B200_NCKPT] = {};
  // live per-launch timing (pt_b200_decoder_profile): one event before each launch, one at the end
  static constexpr int kMaxRec = 64;
  bool prof = false;
  cudaEvent_t ev[kMaxRec + 1] = {};
  int nrec = 0;
  int rkind[kMaxRec] = {};
  double rflops[kMaxRec] = {}, rbytes[kMaxRec] = {};
};
