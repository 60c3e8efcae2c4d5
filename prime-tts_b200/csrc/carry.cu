// carry.cu -- streaming with carried state: the decoder run chunk by chunk, every row once.
//
// A session lays its streams out as whole requests of the batched decoder (decoder.cuh: the
// ragged row layout, zero gap rows) and keeps every activation tensor for the session's life.
// Pass k stages latent frames [k*chunk, (k+1)*chunk) of each stream; then, layer by layer in
// the decoder's order, each layer computes the rows of each stream whose inputs are complete:
// a conv with right reach b over an input complete below row F completes its rows below F - b,
// a transposed conv completes the delay-line steps below F (outputs below 4 F - 6), a residual
// or branch-sum input caps its consumer at its own frontier.  Frontiers are rounded down to 16
// rows in absolute row numbers (the epilogue's pass height, so no two passes ever write one
// 16-row slab) for the MRF convs and conv_post, whose outputs are updated in place or shared by
// stages.  conv_pre and the upsamplers write tensors nobody updates in place, so they stop at the
// exact frontier: their last tile rounds up to 16 rows (the MMA's N step), computing up to 15 rows
// past it from incomplete inputs; nothing reads those rows before the next pass, whose tiles
// start at that frontier, rewrites them.  This keeps level 0, where 16 rows are 16 latent frames,
// from adding to the emission delay.  In a stream's last pass every layer runs to the end of the
// stream rounded up into its zero gap (every gap is >= 16 rows, so that never reaches another
// stream).
// The tail then emits the samples whose frames are all complete.  Rows are computed once, by
// the same kernels with the same operand order as the whole-utterance decode, and read back from
// where earlier passes left them, so the output is bit-identical to it.
//
// Buffers.  A tensor a later pass still reads must not be overwritten by another layer in
// between.  Per level the session keeps u, leaky(u), the branch sum and the level's output, and
// per resblock h (the convs1 output, shared by its three stages), xb (the residual chain,
// updated in place) and xt for stages 0 and 1 separately.  Sharing h is safe because stage j+1's
// convs1 frontier trails stage j's convs2 reads by its own reach (>= 3 x (K-1)/2 rows); one xt
// could not be shared: stage j+1's convs1 reads xt d x (K-1)/2 rows back (d = 3, 5), further back
// than stage j+1's convs2 has already overwritten it.  The planner checks these orders.
#include <algorithm>

#include <vector>

#include "decoder.cuh"

using namespace ptb;
using namespace ptb::dec;

namespace {

constexpr int kNL = 40;   // conv launches per pass: conv_pre, 2 x (ups + 18 MRF convs), conv_post

inline int64_t floor16(int64_t x) { return x >= 0 ? x / 16 * 16 : -((-x + 15) / 16 * 16); }
inline int64_t ceil16(int64_t x) { return -floor16(-x); }

// The pass plan: per pass, per conv launch, the tiles {first row, rows} of every stream's new
// rows; the latent frames each pass stages and the samples it emits.
struct CarryPlan {
  int n = 0, chunk = 0, npass = 0;
  std::vector<int64_t> T, a[3];
  int64_t R[3] = {0, 0, 0};
  std::vector<int2> tiles;
  std::vector<int> toff, tcnt;              // [npass][kNL] into tiles
  std::vector<long long> f0, f1;            // [npass][n] staged frames [f0, f1)
  std::vector<long long> klo, khi, jb;      // [npass][n] emitted samples, first tail chunk
  std::vector<long long> zchunks, tchunks;  // [npass] stage / tail grid widths
};

// tiles of at most 256 rows from lo to hi, the last one rounded up to a multiple of 16 rows
void add_tiles(std::vector<int2> &t, int64_t lo, int64_t hi) {
  for (int64_t r = lo; r < hi; r += 256)
    t.push_back(make_int2((int)r, (int)ceil16(std::min<int64_t>(256, hi - r))));
}

int plan_carry(CarryPlan &P, int n, const int64_t *T, int chunk) {
  PTB_REQUIRE(n > 0 && T && chunk > 0, "pt_b200: bad carried-stream arguments");
  for (int s = 0; s < n; ++s)
    PTB_REQUIRE(T[s] >= 2, "pt_b200: stream %d has %lld frames (need >= 2)", s, (long long)T[s]);
  P = CarryPlan();
  P.n = n;
  P.chunk = chunk;
  P.T.assign(T, T + n);
  layout_rows(T, n, P.a, P.R);
  PTB_REQUIRE(P.R[2] * 128 < (int64_t)INT_MAX && P.R[0] * 512 < (int64_t)INT_MAX &&
                  P.R[1] * 256 < (int64_t)INT_MAX,
              "pt_b200: carried session too large (%lld level-2 rows); open fewer streams",
              (long long)P.R[2]);
  int64_t maxT = 0;
  for (int s = 0; s < n; ++s) maxT = std::max(maxT, T[s]);
  P.npass = (int)((maxT + chunk - 1) / chunk);

  // per stream, per launch: the absolute end of the rows computed so far (a multiple of 16)
  std::vector<int64_t> hi((size_t)kNL * n);
  std::vector<int64_t> fz(n, 0), S(n, 0);
  // where each launch's output rows start, relative to its stream's first row at that level
  auto start_local = [](int L) { return L == kNL - 1 ? -1 : 0; };
  auto level_of = [](int L) {   // level whose row numbers the launch's tiles use
    if (L == 0 || L == 1) return 0;     // conv_pre; ups.0 walks level-0 delay-line steps
    if (L <= 19) return 1;              // level-1 MRF
    if (L == 20) return 1;              // ups.1 walks level-1 steps
    return 2;                           // level-2 MRF, conv_post
  };
  for (int L = 0; L < kNL; ++L)
    for (int s = 0; s < n; ++s) hi[(size_t)L * n + s] = floor16(P.a[level_of(L)][s] + start_local(L));

  std::vector<std::vector<int2>> lt(kNL);
  for (int k = 0; k < P.npass; ++k) {
    for (auto &v : lt) v.clear();
    long long zmax = 0, tmax = 0;
    for (int s = 0; s < n; ++s) {
      const int64_t Ts = T[s];
      const int64_t fz1 = std::min<int64_t>(Ts, (int64_t)(k + 1) * chunk);
      const bool done = fz1 == Ts;
      P.f0.push_back(fz[s]);
      P.f1.push_back(fz1);
      zmax = std::max<long long>(zmax, (fz1 - fz[s] + 31) / 32);
      // advance launch L of stream s toward local row `target` (rows of [start, end) at `base`);
      // returns the local frontier (rows below it are complete)
      auto adv = [&](int L, int64_t base, int64_t end, int64_t target) -> int64_t {
        int64_t &h = hi[(size_t)L * n + s];
        const bool exact = L == 0 || L == 1 || L == 20;   // conv_pre, ups.0, ups.1
        const int64_t nh = done ? ceil16(base + end)
                                : std::max(h, exact ? base + target : floor16(base + target));
        // a stream's last tiles start on a 16-row boundary so that they end exactly at nh (the
        // rows they redo below h are complete: recomputed to the same bits)
        if (nh > h) add_tiles(lt[L], exact && done ? floor16(h) : h, nh);
        h = nh;
        return done ? end : nh - base;
      };
      const int64_t b0 = P.a[0][s], b1 = P.a[1][s], b2 = P.a[2][s];
      int L = 0;
      const int64_t fX0 = adv(L++, b0, Ts, fz1 - 3);                   // conv_pre (k7, p3)
      int64_t lvl_out = fX0, lvl_base = b0, lvl_T = Ts;
      int64_t fP = 0;
      for (int lv = 0; lv < 2; ++lv) {
        const int64_t base = lv == 0 ? b1 : b2, len = 4 * lvl_T;
        // ups: steps q (local rows of the level below) complete below the input frontier;
        // step q writes outputs 4q + r - 6, so outputs below 4Q - 6 are complete
        const int64_t Q = adv(L++, lvl_base, lvl_T + 2, lvl_out);
        const int64_t fU = done ? len : 4 * Q - 6;
        int64_t fAcc = 0;
        for (int rb = 0; rb < 3; ++rb) {
          const int64_t r = (kK[rb] - 1) / 2;
          int64_t fin = fU, fres = fU, fX = 0;
          for (int j = 0; j < 3; ++j) {
            const int64_t fH = adv(L++, base, len, fin - kD[j] * r);     // convs1.j
            int64_t tgt = std::min(fH - r, fres);                          // convs2.j
            if (j == 2 && rb > 0) tgt = std::min(tgt, fAcc);               // branch sum
            fX = adv(L++, base, len, tgt);
            // the shared h: stage j+1 writes below its frontier, which must stay under the
            // rows stage j's convs2 still reads (from fX - r on)
            if (j < 2 && !done) {
              const int64_t next = floor16(base + fX - kD[j + 1] * r) - base;
              PTB_REQUIRE(next <= fX - r, "pt_b200: carried plan: shared h would be overwritten");
            }
            fin = fX;
            fres = fX;
          }
          fAcc = fX;
        }
        lvl_out = fAcc;
        lvl_base = base;
        lvl_T = len;
        fP = fAcc;
      }
      // conv_post over the reflection-padded rows [-1, 16T): row -1 is written with row 1, in the
      // stream's first 16-row slab, so the padded input is complete below fP once fP > 1
      const int64_t fPost = adv(L++, b2, 16 * Ts, fP > 1 ? fP - 3 : -1);
      PTB_REQUIRE(L == kNL, "pt_b200: carried plan walked %d launches", L);
      // tail: sample j reads conv_post frames up to ((((j + 31) >> 2) + 8) >> 2) (PQMF reach 31
      // stuffed samples, overlap-add of 4 frames); frames are conv_post rows -1, 0, ...
      const int64_t nwav = 256 * Ts;
      int64_t s1 = done ? nwav : std::min(nwav, std::max<int64_t>(0, 16 * (fPost + 1) - 63));
      s1 = std::max(s1, S[s]);
      const int64_t base_j = S[s] / 1024 * 1024;
      P.klo.push_back(S[s]);
      P.khi.push_back(s1);
      P.jb.push_back(base_j);
      if (s1 > S[s]) tmax = std::max<long long>(tmax, (s1 - base_j + 1023) / 1024);
      S[s] = s1;
      fz[s] = fz1;
    }
    P.zchunks.push_back(zmax);
    P.tchunks.push_back(tmax);
    for (int L = 0; L < kNL; ++L) {
      P.toff.push_back((int)P.tiles.size());
      P.tcnt.push_back((int)lt[L].size());
      P.tiles.insert(P.tiles.end(), lt[L].begin(), lt[L].end());
    }
  }
  // every launch ends at its stream's end and every sample is emitted
  for (int s = 0; s < n; ++s) {
    PTB_REQUIRE(S[s] == 256 * T[s] && fz[s] == T[s], "pt_b200: carried plan left stream %d unfinished", s);
    for (int L = 0; L < kNL; ++L) {
      const int lv = level_of(L);
      const int64_t end = L == 0 ? T[s] : L == 1 ? T[s] + 2 : L == 20 ? 4 * T[s] + 2
                        : L == kNL - 1 ? 16 * T[s] : (lv == 1 ? 4 : 16) * T[s];
      PTB_REQUIRE(hi[(size_t)L * n + s] == ceil16(P.a[lv][s] + end),
                  "pt_b200: carried plan: launch %d of stream %d stops short", L, s);
    }
  }
  return 0;
}

}  // namespace

struct pt_b200_carry {
  pt_b200_decoder *d = nullptr;
  CarryPlan P;
  Plan lay;              // the whole-stream layout and its device tables
  int next = 0;          // the next pass to run
  void *block = nullptr; // activations + pass tables, one allocation
  float *Z = nullptr, *X0 = nullptr, *POST = nullptr;
  float *U[2], *LU[2], *ACC[2], *OUT[2], *H[2][3], *XB[2][3], *XT[2][3][2];
  int2 *tiles = nullptr;
  long long *f0 = nullptr, *f1 = nullptr, *klo = nullptr, *khi = nullptr, *jb = nullptr;
  // One CUDA graph per pass: a pass's launches depend only on the session's plan and on the
  // latent / waveform buffers and stream it ran with, so the second identical run of a pass
  // captures it and later runs replay it (PT_B200_GRAPH=0: always eager).
  struct PassGraph {
    cudaGraphExec_t exec = nullptr;
    const float *z = nullptr;
    float *wav = nullptr;
    cudaStream_t st = nullptr;
    bool seen = false;
    long kernels = 0;
  };
  std::vector<PassGraph> graphs;
};

namespace {

int run_pass(pt_b200_carry *c, cudaStream_t st, int k, const float *z_dev, float *wav_dev) {
  pt_b200_decoder *d = c->d;
  const CarryPlan &P = c->P;
  const Plan &p = c->lay;
  const int n = P.n;
  const size_t o = (size_t)k * n;
  int L = 0;
  // conv launch L of this pass over level rows `rows` (skipped when it has no new rows)
  auto conv = [&](const DLayer &W, const float *act, int64_t rows, int off0, int step,
                  const EpiParams &e) -> int {
    const int cnt = P.tcnt[(size_t)k * kNL + L], off = P.toff[(size_t)k * kNL + L];
    ++L;
    if (!cnt) return 0;
    return run_conv(d, st, W, act, rows, off0, step, e, c->tiles + off, cnt);
  };
  if (P.zchunks[k] > 0) {
    dim3 grid((unsigned)P.zchunks[k], 1, (unsigned)n);
    stage_z_kernel<<<grid, dim3(32, 8), 0, st>>>(z_dev, p.zoff, p.zld, c->f1 + o, p.a0, c->f0 + o, c->Z);
    PTB_CUDA(cudaGetLastError());
    count_launch();
  }
  {
    EpiParams e = rows_epi(p.mask[0], 512);
    e.out1 = c->X0;
    if (conv(d->pre, c->Z, p.R[0], -3, 1, e)) return -1;
  }
  const float *lvl_in = c->X0;
  for (int s = 0; s < 2; ++s) {
    const int C = s == 0 ? 256 : 128;
    const unsigned char *mk = p.mask[s + 1];
    const int64_t rin = p.R[s], rout = p.R[s + 1];
    {
      EpiParams e = rows_epi(mk, C);
      e.mode = EPI_ROWS_CONVT;
      e.obase = s == 0 ? p.ob01 : p.ob12;
      e.s = 4;
      e.cphase = C;
      e.out_rows = (int)rout;
      e.out0 = c->U[s];
      e.out1 = c->LU[s];
      if (conv(d->ups[s], lvl_in, rin, 0, -1, e)) return -1;
    }
    for (int rb = 0; rb < 3; ++rb) {
      const int r = 3 * s + rb, K = kK[rb];
      for (int j = 0; j < 3; ++j) {
        {  // convs1.j (+ LeakyRelu)
          EpiParams e = rows_epi(mk, C);
          e.out1 = c->H[s][rb];
          const float *in = j == 0 ? c->LU[s] : c->XT[s][rb][j - 1];
          if (conv(d->rb1[r][j], in, rout, -kD[j] * (K - 1) / 2, kD[j], e)) return -1;
        }
        {  // convs2.j + residual (+ leaky for the next stage / branch sum)
          EpiParams e = rows_epi(mk, C);
          e.res = j == 0 ? c->U[s] : c->XB[s][rb];
          if (j < 2) {
            e.out0 = c->XB[s][rb];
            e.out1 = c->XT[s][rb][j];
          } else if (rb == 0) {
            e.out0 = c->ACC[s];
          } else if (rb == 1) {
            e.accin = c->ACC[s];
            e.acc_mode = 2;
            e.out0 = c->ACC[s];
          } else {
            e.accin = c->ACC[s];
            e.acc_mode = 3;
            e.out1 = c->OUT[s];
            if (s == 1) {
              e.alpha1 = kLrFinal;
              e.mask = p.mask_refl;
              e.refl = 1;
            }
          }
          if (conv(d->rb2[r][j], c->H[s][rb], rout, -(K - 1) / 2, 1, e)) return -1;
        }
      }
    }
    lvl_in = c->OUT[s];
  }
  {
    EpiParams e = rows_epi(p.mask_post, 80);
    e.out0 = c->POST;
    if (conv(d->post, c->OUT[1], p.R[2], -3, 1, e)) return -1;
  }
  if (P.tchunks[k] > 0 &&
      tail_run_rows(c->POST, 80, p.row0, p.tp, p.wav0, c->klo + o, c->khi + o, c->jb + o,
                    P.tchunks[k], n, 16 * p.max_T + 1, d->pqmf, wav_dev, st))
    return -1;
  return 0;
}

}  // namespace

extern "C" {

int64_t pt_b200_carry_plan(int nstreams, const int64_t *T, int chunk, int64_t *lo, int64_t *hi,
                           int64_t cap) {
  CarryPlan P;
  if (plan_carry(P, nstreams, T, chunk)) return -1;
  const int64_t need = (int64_t)P.npass * nstreams;
  if (lo && hi && cap >= need)
    for (int64_t i = 0; i < need; ++i) {
      lo[i] = P.klo[(size_t)i];
      hi[i] = P.khi[(size_t)i];
    }
  return P.npass;
}

pt_b200_carry *pt_b200_carry_open(pt_b200_decoder *d, int nstreams, const int64_t *T, int chunk) {
  if (!d) {
    set_error("pt_b200: NULL decoder");
    return nullptr;
  }
  auto *c = new pt_b200_carry();
  c->d = d;
  auto fail = [&]() {
    pt_b200_carry_close(c);
    return static_cast<pt_b200_carry *>(nullptr);
  };
  if (plan_carry(c->P, nstreams, T, chunk)) return fail();
  if (cudaSetDevice(d->device) != cudaSuccess) {
    set_error("pt_b200: cannot select device %d", d->device);
    return fail();
  }
  const CarryPlan &P = c->P;
  // whole streams as requests: latents [192][T] back to back, every sample kept in place
  std::vector<pt_b200_window> w((size_t)nstreams);
  int64_t zo = 0, wo = 0;
  for (int i = 0; i < nstreams; ++i) {
    w[i] = pt_b200_window{T[i], zo, T[i], 0, 256 * T[i], wo};
    zo += 192 * T[i];
    wo += 256 * T[i];
  }
  cudaStream_t st = d->stream;
  if (build_layout(c->lay, st, nstreams, w.data())) return fail();
  const size_t r0 = (size_t)P.R[0], r1 = (size_t)P.R[1], r2 = (size_t)P.R[2];
  const size_t na = (size_t)nstreams * P.npass;
  auto al = [](size_t x) { return (x + 63) & ~(size_t)63; };   // floats, 256-byte aligned
  const size_t nfl = al(r0 * 192) + al(r0 * 512) + 16 * al(r1 * 256) + 16 * al(r2 * 128) + al(r2 * 80);
  const size_t tbytes = al(P.tiles.size() * 2) * 4 + 5 * al(na * 2) * 4;
  if (cudaMalloc(&c->block, nfl * 4 + tbytes) != cudaSuccess) {
    cudaGetLastError();
    set_error("pt_b200: carried session needs %.2f GB of device memory", (nfl * 4 + tbytes) / 1e9);
    c->block = nullptr;
    return fail();
  }
  float *q = static_cast<float *>(c->block);
  auto take = [&](size_t nf) {
    float *r = q;
    q += al(nf);
    return r;
  };
  c->Z = take(r0 * 192);
  c->X0 = take(r0 * 512);
  for (int s = 0; s < 2; ++s) {
    const size_t rows = s == 0 ? r1 : r2, C = s == 0 ? 256 : 128;
    c->U[s] = take(rows * C);
    c->LU[s] = take(rows * C);
    c->ACC[s] = take(rows * C);
    c->OUT[s] = take(rows * C);
    for (int rb = 0; rb < 3; ++rb) {
      c->H[s][rb] = take(rows * C);
      c->XB[s][rb] = take(rows * C);
      c->XT[s][rb][0] = take(rows * C);
      c->XT[s][rb][1] = take(rows * C);
    }
  }
  c->POST = take(r2 * 80);
  const size_t act_bytes = (size_t)(reinterpret_cast<char *>(q) - static_cast<char *>(c->block));
  // pass tables after the activations
  char *tb = reinterpret_cast<char *>(q);
  std::vector<char> host(tbytes, 0);
  size_t off = 0;
  auto put = [&](const void *src, size_t bytes) {
    std::memcpy(host.data() + off, src, bytes);
    char *dst = tb + off;
    off += al((bytes + 3) / 4) * 4;
    return dst;
  };
  c->tiles = reinterpret_cast<int2 *>(put(P.tiles.data(), P.tiles.size() * sizeof(int2)));
  c->f0 = reinterpret_cast<long long *>(put(P.f0.data(), na * 8));
  c->f1 = reinterpret_cast<long long *>(put(P.f1.data(), na * 8));
  c->klo = reinterpret_cast<long long *>(put(P.klo.data(), na * 8));
  c->khi = reinterpret_cast<long long *>(put(P.khi.data(), na * 8));
  c->jb = reinterpret_cast<long long *>(put(P.jb.data(), na * 8));
  if (cudaMemsetAsync(c->block, 0, act_bytes, st) != cudaSuccess ||
      cudaMemcpyAsync(tb, host.data(), off, cudaMemcpyHostToDevice, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess) {
    set_error("pt_b200: carried session set-up failed (%s)", cudaGetErrorString(cudaGetLastError()));
    return fail();
  }
  if (tail_prepare()) return fail();
  return c;
}

int pt_b200_carry_passes(const pt_b200_carry *c) { return c ? c->P.npass : -1; }

int pt_b200_carry_run(pt_b200_carry *c, void *stream, int pass, const float *z_dev, float *wav_dev) {
  PTB_REQUIRE(c && z_dev && wav_dev, "pt_b200: bad carried-stream arguments");
  PTB_REQUIRE(pass == c->next && pass < c->P.npass,
              "pt_b200: carried pass %d out of order (next is %d of %d)", pass, c->next, c->P.npass);
  pt_b200_decoder *d = c->d;
  std::lock_guard<std::mutex> lk(d->mu);
  PTB_CUDA(cudaSetDevice(d->device));
  cudaStream_t st = stream ? (cudaStream_t)stream : d->stream;
  if (d->graph_on < 0) d->graph_on = getenv("PT_B200_GRAPH") ? atoi(getenv("PT_B200_GRAPH")) : 1;
  if (c->graphs.size() != (size_t)c->P.npass) c->graphs.assign((size_t)c->P.npass, {});
  pt_b200_carry::PassGraph &G = c->graphs[(size_t)pass];
  const bool same = G.z == z_dev && G.wav == wav_dev && G.st == st;
  if (!d->graph_on || !same || !G.seen) {
    // first run with these buffers: eager (one-time uploads and attribute settings happen here)
    if (G.exec && !same) {
      cudaGraphExecDestroy(G.exec);
      G.exec = nullptr;
    }
    G.z = z_dev;
    G.wav = wav_dev;
    G.st = st;
    G.seen = true;
    if (run_pass(c, st, pass, z_dev, wav_dev)) return -1;
  } else {
    if (!G.exec) {
      const long before = launches(0);
      PTB_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
      const int rc = run_pass(c, st, pass, z_dev, wav_dev);
      cudaGraph_t g = nullptr;
      const cudaError_t ec = cudaStreamEndCapture(st, &g);
      const long captured = launches(0) - before;
      count_launch(-captured);   // capturing launches nothing
      if (rc || ec != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        PTB_REQUIRE(false, "pt_b200: carried pass %d graph capture failed (%s)", pass,
                    cudaGetErrorString(ec));
      }
      const cudaError_t ei = cudaGraphInstantiate(&G.exec, g, 0);
      cudaGraphDestroy(g);
      PTB_CUDA(ei);
      G.kernels = captured;
    }
    PTB_CUDA(cudaGraphLaunch(G.exec, st));
    count_launch(G.kernels);
  }
  ++c->next;
  return 0;
}

int pt_b200_carry_reset(pt_b200_carry *c) {
  PTB_REQUIRE(c, "pt_b200: NULL carried session");
  std::lock_guard<std::mutex> lk(c->d->mu);
  c->next = 0;
  return 0;
}

void pt_b200_carry_close(pt_b200_carry *c) {
  if (!c) return;
  if (c->d) {
    cudaSetDevice(c->d->device);
    cudaDeviceSynchronize();
  }
  for (auto &G : c->graphs)
    if (G.exec) cudaGraphExecDestroy(G.exec);
  if (c->block) cudaFree(c->block);
  free_plan(c->lay);
  delete c;
}

int pt_b200_stream_decode_carry(pt_b200_decoder *d, void *stream, int nstreams, const int64_t *T,
                                const float *z_dev, int chunk, float *wav_dev) {
  pt_b200_carry *c = pt_b200_carry_open(d, nstreams, T, chunk);
  if (!c) return -1;
  int rc = 0;
  for (int k = 0; k < c->P.npass && !rc; ++k) rc = pt_b200_carry_run(c, stream, k, z_dev, wav_dev);
  if (!rc) rc = pt_b200_decoder_sync(d, stream);
  pt_b200_carry_close(c);
  return rc;
}

}  // extern "C"
