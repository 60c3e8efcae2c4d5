// carry.cu -- streaming with carried state: the decoder run chunk by chunk, every row once, in a
// bounded amount of device memory per stream.
//
// Frontiers.  Pass k stages latent frames [k*chunk, (k+1)*chunk) of each stream; then, layer by
// layer in the decoder's order, each layer computes the rows of each stream whose inputs are
// complete: a conv with right reach b over an input complete below row F completes its rows
// below F - b, a transposed conv completes the delay-line steps below F (outputs below 4 F - 6), a
// residual or branch-sum input caps its consumer at its own frontier.  Frontiers are rounded down
// to 16 rows (the epilogue's pass height, so no two passes ever write one 16-row slab) for the
// MRF convs and conv_post, whose outputs are updated in place or shared by stages.  conv_pre and
// the upsamplers write tensors nobody updates in place, so they stop at the exact frontier: their
// last tile rounds up to 16 rows (the MMA's N step), computing up to 15 rows past it from
// incomplete inputs; nothing reads those rows before the next pass, whose tiles start at that
// frontier, rewrites them.  This keeps level 0, where 16 rows are 16 latent frames, from adding to
// the emission delay.  The pass after the one that brings a stream's last frames flushes it:
// every layer runs to the end of the stream rounded up into the zero rows after it.  The tail
// then emits the samples whose frames are all complete.
// Rows are computed once, by the same kernels with the same operand order as the
// whole-utterance decode, and read back from where earlier passes left them, so the output is
// bit-identical to it.  The planner does this bookkeeping in virtual rows: each stream laid out
// whole, as the batched decoder lays out requests (decoder.cuh).
//
// Bounded memory.  Physically each stream owns, at each level, a window of a fixed number of rows
// (cap, the same for all streams), with zero gap rows between windows.  Pass k maps the stream's
// local row r to window row r - off_k.  Before a pass the planner moves the window up (off_k >
// off_{k-1}, a multiple of 16) when the pass would not fit the window otherwise: the rows every
// later pass may still touch -- the lowest row any launch reads (its tile start minus its reach,
// minus a 16-row slack) or writes, and the lowest conv_post row the tail reads -- are moved to
// the front of the window by a block copy, for every tensor of that level.  A stream's flush pass
// first clears the 48 rows after its end (its padding: the whole-stream layout's zero gap), since
// the window reuses rows that held earlier frames.  So a session holds about (chunk + receptive
// lag) rows per stream and level instead of the whole stream: at 32-frame chunks windows of 112
// / 288 / 800 rows at levels 0 / 1 / 2.  Tile rows, row masks, the upsamplers' row maps and the
// per-stream staging / tail offsets are tabulated per pass.
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

constexpr int kNL = 40;      // conv launches per pass: conv_pre, 2 x (ups + 18 MRF convs), conv_post
constexpr int kPad = 48;     // rows after a stream's end cleared in its last pass (>= reach + 16)
constexpr int kSlack = 16;   // rows kept below the lowest row a launch touches

inline int64_t floor16(int64_t x) { return x >= 0 ? x / 16 * 16 : -((-x + 15) / 16 * 16); }
inline int64_t ceil16(int64_t x) { return -floor16(-x); }

// level whose row numbers launch L's tiles use
int level_of(int L) {
  if (L == 0 || L == 1) return 0;     // conv_pre; ups.0 walks level-0 delay-line steps
  if (L <= 20) return 1;              // level-1 MRF; ups.1 walks level-1 steps
  return 2;                           // level-2 MRF, conv_post
}
bool is_ups(int L) { return L == 1 || L == 20; }
// input rows launch L reads below / above each output row (tile rows for the upsamplers)
int reach_lo(int L) {
  if (L == 0 || is_ups(L)) return 3;           // conv_pre k7 p3; convT taps q - 0 .. q - 3
  if (L == kNL - 1) return 4;                  // conv_post k7 p3 over the reflection-padded rows
  const int m = L <= 19 ? L - 2 : L - 21;      // MRF conv m: resblock m / 6, stage (m % 6) / 2
  const int rb = m / 6, j = (m % 6) / 2, r = (kK[rb] - 1) / 2;
  return (m & 1) ? r : kD[j] * r;
}
int reach_hi(int L) { return is_ups(L) ? 0 : reach_lo(L); }

// rows of level l a stream of T frames occupies (the tensors' valid rows)
int64_t level_len(int l, int64_t T) { return l == 0 ? T : l == 1 ? 4 * T : 16 * T; }

// The pass plan: per pass, per conv launch, the tiles {first row, rows} of every stream's new
// rows (window rows); the latent frames each pass stages and the samples it emits; the window
// offsets and moves.
struct CarryPlan {
  int n = 0, chunk = 0, npass = 0;
  std::vector<int64_t> T, a[3];             // virtual whole-stream layout
  int64_t R[3] = {0, 0, 0};
  std::vector<int> done;                    // [n] the stream's last pass
  // physical layout: windows of cap[l] rows with zero gaps between them
  int64_t cap[3] = {0, 0, 0}, RP[3] = {0, 0, 0};
  std::vector<int64_t> A[3];                // [n] window start rows
  std::vector<int64_t> off[3];              // [npass][n] local row at the window start
  std::vector<int64_t> mv[3];               // [npass][n] rows moved to the window start (0: none)
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
  PTB_REQUIRE(P.R[2] < (int64_t)INT_MAX / 2, "pt_b200: carried session too large (%lld level-2 "
              "rows of stream data); open fewer streams", (long long)P.R[2]);
  int64_t maxT = 0;
  for (int s = 0; s < n; ++s) maxT = std::max(maxT, T[s]);
  // a stream's frames arrive in passes 0 .. ceil(T / chunk) - 1, each run like any other; the
  // pass after them flushes it (every layer to the stream's end).  Flushing in the pass that
  // brings the last frames would make that pass span the receptive lag, the last chunk and the
  // flush at once, and the windows are sized by the largest pass: level-2 windows of 1,312 rows
  // instead of 768 at 32-frame chunks.
  P.npass = (int)((maxT + chunk - 1) / chunk) + 1;
  const int np = P.npass;
  P.done.resize(n);
  for (int s = 0; s < n; ++s) P.done[s] = (int)((T[s] + chunk - 1) / chunk);

  // ---- 1. frontiers in virtual rows; per pass and stream, the local rows each level's tensors
  // are touched over [lo, hi) and written up to (wr)
  constexpr int64_t kBig = INT64_MAX / 4;
  std::vector<int64_t> tlo[3], thi[3], twr[3];
  for (int l = 0; l < 3; ++l) {
    tlo[l].assign((size_t)np * n, kBig);
    thi[l].assign((size_t)np * n, -kBig);
    twr[l].assign((size_t)np * n, -kBig);
  }
  std::vector<int64_t> hi((size_t)kNL * n);
  std::vector<int64_t> fz(n, 0), S(n, 0);
  auto start_local = [](int L) { return L == kNL - 1 ? -1 : 0; };
  for (int L = 0; L < kNL; ++L)
    for (int s = 0; s < n; ++s) hi[(size_t)L * n + s] = floor16(P.a[level_of(L)][s] + start_local(L));

  // virtual tiles with their stream, per launch of a pass
  struct VT {
    int2 t;
    int s;
  };
  std::vector<std::vector<VT>> lt(kNL);
  std::vector<VT> vtiles;
  std::vector<int> vtoff, vtcnt;
  for (int k = 0; k < np; ++k) {
    for (auto &v : lt) v.clear();
    long long zmax = 0, tmax = 0;
    for (int s = 0; s < n; ++s) {
      const int64_t Ts = T[s];
      const size_t ks = (size_t)k * n + s;
      const int64_t fz1 = std::min<int64_t>(Ts, (int64_t)(k + 1) * chunk);
      const bool done = k >= P.done[s];
      P.f0.push_back(fz[s]);
      P.f1.push_back(fz1);
      zmax = std::max<long long>(zmax, (fz1 - fz[s] + 31) / 32);
      auto touch = [&](int l, int64_t lo, int64_t hi_, bool wr) {
        tlo[l][ks] = std::min(tlo[l][ks], lo);
        thi[l][ks] = std::max(thi[l][ks], hi_);
        if (wr) twr[l][ks] = std::max(twr[l][ks], hi_);
      };
      if (fz1 > fz[s]) touch(0, fz[s], fz1, true);   // staged latent frames
      // advance launch L of stream s toward local row `target` (rows of [start, end) at `base`);
      // returns the local frontier (rows below it are complete)
      auto adv = [&](int L, int64_t base, int64_t end, int64_t target) -> int64_t {
        int64_t &h = hi[(size_t)L * n + s];
        const bool exact = L == 0 || is_ups(L);   // conv_pre, ups.0, ups.1
        const int64_t nh = done ? ceil16(base + end)
                                : std::max(h, exact ? base + target : floor16(base + target));
        // a stream's last tiles start on a 16-row boundary so that they end exactly at nh (the
        // rows they redo below h are complete: recomputed to the same bits)
        if (nh > h) {
          const int64_t lo = exact && done ? floor16(h) : h;
          std::vector<int2> tt;
          add_tiles(tt, lo, nh);
          for (const int2 &x : tt) lt[L].push_back({x, s});
          const int l = level_of(L);
          const int64_t b = P.a[l][s];
          const int64_t tend = lo + ceil16(nh - lo);   // the last tile's end
          touch(l, lo - b - reach_lo(L), tend - b + reach_hi(L), false);
          if (is_ups(L)) {   // outputs 4q + r - 6 of the level above, steps q >= 1 only
            touch(l + 1, std::max<int64_t>(4 * (lo - b) - 6, -2), 4 * (tend - b) - 2, true);
          } else {
            touch(l, lo - b, tend - b, true);
          }
        }
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
      if (s1 > S[s]) {
        tmax = std::max<long long>(tmax, (s1 - base_j + 1023) / 1024);
        // the tail CTAs of chunks base_j .. the chunk of sample s1 - 1 read conv_post frames
        // ((m + 8) >> 2) - 3 .. ((m' + 8) >> 2), m .. m' the overlap-add samples their 1024
        // outputs need (clipped to the signal); frame f is conv_post row f - 1
        const int64_t Ls = 4 * 16 * Ts;
        const int64_t m = std::max<int64_t>(0, (base_j - 28) >> 2);
        const int64_t jl = (s1 - 1) / 1024 * 1024;
        const int64_t m2 = std::min<int64_t>((jl + 1023 + 31) >> 2, Ls - 1);
        const int64_t f2 = std::min<int64_t>((m2 + 8) >> 2, 16 * Ts);
        touch(2, ((m + 8) >> 2) - 4, f2, false);
      }
      S[s] = s1;
      fz[s] = fz1;
    }
    P.zchunks.push_back(zmax);
    P.tchunks.push_back(tmax);
    for (int L = 0; L < kNL; ++L) {
      vtoff.push_back((int)vtiles.size());
      vtcnt.push_back((int)lt[L].size());
      vtiles.insert(vtiles.end(), lt[L].begin(), lt[L].end());
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

  // ---- 2. window offsets.  Per level and stream, the highest offset a pass may use is the
  // lowest row it or any later pass touches, less the slack (rounded down to 16); the window
  // capacity is the largest span a pass touches from that offset (the last pass's flush and
  // padding included).  Then the windows move lazily: before a pass, only when its span from the
  // current offset would not fit, and then to that highest offset -- every window move copies
  // the live rows of all the level's tensors, so fewer moves are less traffic.
  for (int l = 0; l < 3; ++l) {
    P.off[l].assign((size_t)np * n, 0);
    P.mv[l].assign((size_t)np * n, 0);
    std::vector<int64_t> hiw((size_t)np * n, 0), top((size_t)np * n, 0);
    int64_t cap = 16;
    for (int s = 0; s < n; ++s) {
      const int last = P.done[s];
      int64_t need = kBig, prev = 0;
      for (int k = last; k >= 0; --k) {
        const size_t ks = (size_t)k * n + s;
        need = std::min(need, tlo[l][ks] - kSlack);
        hiw[ks] = floor16(std::max<int64_t>(need, 0));
        int64_t t = thi[l][ks] == -kBig ? 0 : thi[l][ks];
        if (k == last) t = std::max(t, level_len(l, T[s]) + kPad + (l == 0 ? 2 : 0));
        top[ks] = t;
      }
      for (int k = 0; k <= last; ++k) {   // offsets never go down
        const size_t ks = (size_t)k * n + s;
        hiw[ks] = std::max(hiw[ks], prev);
        prev = hiw[ks];
        cap = std::max(cap, ceil16(top[ks] - hiw[ks]));
      }
    }
    P.cap[l] = cap;
    for (int s = 0; s < n; ++s) {
      const int last = P.done[s];
      int64_t off = 0, wr = 0;
      for (int k = 0; k < np; ++k) {
        const size_t ks = (size_t)k * n + s;
        if (k > 0 && k <= last && top[ks] - off > cap) {
          const int64_t cand = hiw[ks];
          P.mv[l][ks] = std::max<int64_t>(wr - cand, 0);
          off = cand;
        }
        P.off[l][ks] = off;
        if (k <= last) {
          // rows below the window are read only while it starts at local row 0: the gap in
          // front of the stream, as in the whole-stream layout (zeros wherever a valid output
          // row reaches; tiles rounded down to 16 rows also read further, for outputs that are
          // masked off)
          PTB_REQUIRE(off == 0 || tlo[l][ks] >= off || tlo[l][ks] == kBig,
                      "pt_b200: carried plan: level %d row %lld below the window of stream %d",
                      l, (long long)tlo[l][ks], s);
          PTB_REQUIRE(top[ks] - off <= cap, "pt_b200: carried plan: level %d pass %d of stream %d "
                      "does not fit its window", l, k, s);
          if (twr[l][ks] != -kBig) wr = std::max(wr, twr[l][ks]);
        }
      }
    }
  }
  // physical windows: a lead, then per stream its window and a zero gap; a window starts at the
  // same row mod 16 as the stream's virtual rows (offsets move by multiples of 16), so every
  // 16-row slab and the level-2 reflection-row alignment stay where the virtual layout has them
  for (int l = 0; l < 3; ++l) {
    P.A[l].resize(n);
    int64_t r = kLead[l];
    for (int s = 0; s < n; ++s) {
      const int64_t A = r + (((P.a[l][s] - r) % 16) + 16) % 16;
      P.A[l][s] = A;
      r = A + P.cap[l] + kGap[l];
    }
    P.RP[l] = r;
  }
  PTB_REQUIRE(P.RP[2] * 128 < (int64_t)INT_MAX && P.RP[0] * 512 < (int64_t)INT_MAX &&
                  P.RP[1] * 256 < (int64_t)INT_MAX,
              "pt_b200: carried session too large (%lld level-2 rows); open fewer streams",
              (long long)P.RP[2]);
  // ---- 3. virtual tiles -> window rows
  for (int k = 0; k < np; ++k)
    for (int L = 0; L < kNL; ++L) {
      const int l = level_of(L);
      const int vo = vtoff[(size_t)k * kNL + L], vc = vtcnt[(size_t)k * kNL + L];
      P.toff.push_back((int)P.tiles.size());
      P.tcnt.push_back(vc);
      for (int i = 0; i < vc; ++i) {
        const VT &v = vtiles[(size_t)vo + i];
        const int64_t shift = P.a[l][v.s] + P.off[l][(size_t)k * n + v.s] - P.A[l][v.s];
        const int64_t r0 = v.t.x - shift;
        PTB_REQUIRE(shift % 16 == 0 && r0 >= P.A[l][v.s] - 16 &&
                        r0 + v.t.y <= P.A[l][v.s] + P.cap[l],
                    "pt_b200: carried plan: a tile leaves the window of stream %d", v.s);
        P.tiles.push_back(make_int2((int)r0, v.t.y));
      }
    }
  return 0;
}

// Per-pass device tables of a session: row masks and upsampler row maps for the pass's window
// offsets, the staging and tail rows, the window moves.
struct PassTab {
  unsigned char *mask[3], *mask_refl, *mask_post;
  int *ob01, *ob12;
  long long *a0, *row0;
  long long *cp;   // window moves and clears: {src element (-1: clear), dst element, floats}
  int ncp_move, ncp_clear;
};

// One block per descriptor {src element (-1: clear), dst element, floats}: a window move copies
// rows down by src - dst elements within one tensor, so source and destination may overlap; the
// block copies in steps of src - dst elements with a barrier between steps -- step c writes the
// run step c - 1 read, and reads the run step c + 1 writes -- which makes the move exact.
// Every offset and length is a whole number of rows of 80 / 128 / 192 / 256 / 512 floats in a
// 256-byte aligned block, so the copy moves float4s.
__global__ void carry_move_kernel(const long long *__restrict__ d, float *base) {
  const long long *q = d + 3 * blockIdx.x;
  const long long src = q[0], dst = q[1], n4 = q[2] / 4;
  float4 *o = reinterpret_cast<float4 *>(base + dst);
  if (src < 0) {
    for (long long i = threadIdx.x; i < n4; i += blockDim.x) o[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    return;
  }
  const float4 *in = reinterpret_cast<const float4 *>(base + src);
  const long long step = (src - dst) / 4;   // > 0: rows move to the window start
  for (long long b0 = 0; b0 < n4; b0 += step) {
    const long long e = b0 + step < n4 ? b0 + step : n4;
    for (long long i = b0 + threadIdx.x; i < e; i += blockDim.x) o[i] = in[i];
    __syncthreads();
  }
}

size_t al64(size_t x) { return (x + 63) & ~(size_t)63; }   // floats, 256-byte aligned
size_t alb(size_t b) { return (b + 255) & ~(size_t)255; }  // bytes, 256-byte aligned

// floats of the session's activation tensors
size_t act_floats(const CarryPlan &P) {
  const size_t r0 = (size_t)P.RP[0], r1 = (size_t)P.RP[1], r2 = (size_t)P.RP[2];
  return al64(r0 * 192) + al64(r0 * 512) + 16 * al64(r1 * 256) + 16 * al64(r2 * 128) + al64(r2 * 80);
}

// bytes of one pass's tables (masks, row maps, per-stream rows, moves), and its move / clear counts
size_t pass_table_bytes(const CarryPlan &P, int k, int *nmove, int *nclear) {
  const int n = P.n;
  int mvc = 0, clr = 0;
  for (int s = 0; s < n; ++s) {
    const size_t ks = (size_t)k * n + s;
    if (P.mv[0][ks] > 0) mvc += 2;     // Z, X0
    if (P.mv[1][ks] > 0) mvc += 16;    // the 16 level-1 tensors
    if (P.mv[2][ks] > 0) mvc += 17;    // the 16 level-2 tensors and conv_post's output
    if (P.done[s] == k) clr += 2 + 16 + 17;
  }
  *nmove = mvc;
  *nclear = clr;
  return alb((size_t)P.RP[0]) + alb((size_t)P.RP[1]) + 3 * alb((size_t)P.RP[2]) +
         alb((size_t)P.RP[0] * 4) + alb((size_t)P.RP[1] * 4) + 2 * alb((size_t)n * 8) +
         alb((size_t)(mvc + clr) * 24);
}

size_t plan_bytes(const CarryPlan &P) {
  const size_t na = (size_t)P.n * P.npass;
  return alb(P.tiles.size() * sizeof(int2)) + 5 * alb(na * 8);
}

}  // namespace

struct pt_b200_carry {
  pt_b200_decoder *d = nullptr;
  CarryPlan P;
  Plan lay;              // per-stream constant tables (latent offsets, frames, output offsets)
  int next = 0;          // the next pass to run
  void *block = nullptr; // activations + pass tables, one allocation
  size_t bytes = 0;
  float *Z = nullptr, *X0 = nullptr, *POST = nullptr;
  float *U[2], *LU[2], *ACC[2], *OUT[2], *H[2][3], *XB[2][3], *XT[2][3][2];
  int2 *tiles = nullptr;
  long long *f0 = nullptr, *f1 = nullptr, *klo = nullptr, *khi = nullptr, *jb = nullptr;
  std::vector<PassTab> tab;
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
  const PassTab &t = c->tab[(size_t)k];
  const int n = P.n;
  const size_t o = (size_t)k * n;
  // window moves first, then the clears of the streams ending in this pass
  if (t.ncp_move > 0) {
    carry_move_kernel<<<(unsigned)t.ncp_move, 512, 0, st>>>(t.cp, static_cast<float *>(c->block));
    PTB_CUDA(cudaGetLastError());
    count_launch();
  }
  if (t.ncp_clear > 0) {
    carry_move_kernel<<<(unsigned)t.ncp_clear, 512, 0, st>>>(t.cp + 3 * (size_t)t.ncp_move,
                                                            static_cast<float *>(c->block));
    PTB_CUDA(cudaGetLastError());
    count_launch();
  }
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
    stage_z_kernel<<<grid, dim3(32, 8), 0, st>>>(z_dev, p.zoff, p.zld, c->f1 + o, t.a0, c->f0 + o, c->Z);
    PTB_CUDA(cudaGetLastError());
    count_launch();
  }
  {
    EpiParams e = rows_epi(t.mask[0], 512);
    e.out1 = c->X0;
    if (conv(d->pre, c->Z, P.RP[0], -3, 1, e)) return -1;
  }
  const float *lvl_in = c->X0;
  for (int s = 0; s < 2; ++s) {
    const int C = s == 0 ? 256 : 128;
    const unsigned char *mk = t.mask[s + 1];
    const int64_t rin = P.RP[s], rout = P.RP[s + 1];
    {
      EpiParams e = rows_epi(mk, C);
      e.mode = EPI_ROWS_CONVT;
      e.obase = s == 0 ? t.ob01 : t.ob12;
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
              e.mask = t.mask_refl;
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
    EpiParams e = rows_epi(t.mask_post, 80);
    e.out0 = c->POST;
    e.frames = 1;   // POST rows hold the windowed iSTFT frames (conv_post's frames epilogue)
    if (conv(d->post, c->OUT[1], P.RP[2], -3, 1, e)) return -1;
  }
  if (P.tchunks[k] > 0 &&
      tail_run_rows(c->POST, 80, t.row0, p.tp, p.wav0, c->klo + o, c->khi + o, c->jb + o,
                    P.tchunks[k], n, 16 * p.max_T + 1, d->pqmf, wav_dev, st, 1))
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

int64_t pt_b200_carry_device_bytes(int nstreams, const int64_t *T, int chunk) {
  CarryPlan P;
  if (plan_carry(P, nstreams, T, chunk)) return -1;
  size_t b = act_floats(P) * 4 + plan_bytes(P);
  for (int k = 0; k < P.npass; ++k) {
    int nm, nc;
    b += pass_table_bytes(P, k, &nm, &nc);
  }
  return (int64_t)b;
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
  const int n = nstreams, np = P.npass;
  // per-stream constant tables (latent offsets and channel strides, frames, tail frames and
  // output offsets): the batched decoder's layout of whole streams
  std::vector<pt_b200_window> w((size_t)n);
  int64_t zo = 0, wo = 0;
  for (int i = 0; i < n; ++i) {
    w[i] = pt_b200_window{T[i], zo, T[i], 0, 256 * T[i], wo};
    zo += 192 * T[i];
    wo += 256 * T[i];
  }
  cudaStream_t st = d->stream;
  if (build_layout(c->lay, st, n, w.data())) return fail();

  // one allocation: activations, then the per-pass tables, then the pass plan
  const size_t r0 = (size_t)P.RP[0], r1 = (size_t)P.RP[1], r2 = (size_t)P.RP[2];
  const size_t act_b = act_floats(P) * 4;
  std::vector<size_t> pt_off((size_t)np + 1, 0);
  std::vector<int> nmove((size_t)np), nclear((size_t)np);
  for (int k = 0; k < np; ++k)
    pt_off[(size_t)k + 1] = pt_off[(size_t)k] + pass_table_bytes(P, k, &nmove[(size_t)k], &nclear[(size_t)k]);
  const size_t na = (size_t)n * np;
  const size_t plan_b = plan_bytes(P);
  c->bytes = act_b + pt_off[(size_t)np] + plan_b;
  if (cudaMalloc(&c->block, c->bytes) != cudaSuccess) {
    cudaGetLastError();
    set_error("pt_b200: carried session needs %.2f GB of device memory", c->bytes / 1e9);
    c->block = nullptr;
    return fail();
  }
  float *q = static_cast<float *>(c->block);
  auto take = [&](size_t nf) {
    float *r = q;
    q += al64(nf);
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
  // the tensors of each level (element offset in the block, channels), for the window moves
  float *blk = static_cast<float *>(c->block);
  std::vector<std::pair<size_t, int>> tens[3];
  tens[0] = {{(size_t)(c->Z - blk), 192}, {(size_t)(c->X0 - blk), 512}};
  for (int s = 0; s < 2; ++s) {
    const int C = s == 0 ? 256 : 128;
    auto &v = tens[s + 1];
    for (float *x : {c->U[s], c->LU[s], c->ACC[s], c->OUT[s]}) v.push_back({(size_t)(x - blk), C});
    for (int rb = 0; rb < 3; ++rb)
      for (float *x : {c->H[s][rb], c->XB[s][rb], c->XT[s][rb][0], c->XT[s][rb][1]})
        v.push_back({(size_t)(x - blk), C});
  }
  tens[2].push_back({(size_t)(c->POST - blk), 80});

  // host copies of every pass table, uploaded in one copy
  const size_t tab_b = pt_off[(size_t)np] + plan_b;
  std::vector<char> host(tab_b, 0);
  char *dev_tab = reinterpret_cast<char *>(c->block) + act_b;
  c->tab.resize((size_t)np);
  for (int k = 0; k < np; ++k) {
    char *h = host.data() + pt_off[(size_t)k];
    char *dv = dev_tab + pt_off[(size_t)k];
    size_t o = 0;
    auto place = [&](size_t bytes) {
      const size_t at = o;
      o += alb(bytes);
      return at;
    };
    PassTab &t = c->tab[(size_t)k];
    const size_t om0 = place(r0), om1 = place(r1), om2 = place(r2), omr = place(r2), omp = place(r2);
    const size_t oo1 = place(r0 * 4), oo2 = place(r1 * 4), oa0 = place((size_t)n * 8),
                 orw = place((size_t)n * 8);
    const size_t ocp = place((size_t)(nmove[(size_t)k] + nclear[(size_t)k]) * 24);
    unsigned char *m[3] = {reinterpret_cast<unsigned char *>(h + om0),
                           reinterpret_cast<unsigned char *>(h + om1),
                           reinterpret_cast<unsigned char *>(h + om2)};
    unsigned char *mr = reinterpret_cast<unsigned char *>(h + omr);
    unsigned char *mp = reinterpret_cast<unsigned char *>(h + omp);
    int *ob[2] = {reinterpret_cast<int *>(h + oo1), reinterpret_cast<int *>(h + oo2)};
    for (size_t i = 0; i < r0; ++i) ob[0][i] = INT_MIN;
    for (size_t i = 0; i < r1; ++i) ob[1][i] = INT_MIN;
    long long *a0 = reinterpret_cast<long long *>(h + oa0);
    long long *rw = reinterpret_cast<long long *>(h + orw);
    long long *cp = reinterpret_cast<long long *>(h + ocp);
    int ncp = 0;
    for (int s = 0; s < n; ++s) {
      const size_t ks = (size_t)k * n + s;
      int64_t A[3], off[3];
      for (int l = 0; l < 3; ++l) {
        A[l] = P.A[l][s];
        off[l] = P.off[l][ks];
        // valid rows: local [0, len) inside the window
        const int64_t len = level_len(l, T[s]);
        for (int64_t r = std::max<int64_t>(off[l], 0); r < len && r - off[l] < P.cap[l]; ++r)
          m[l][A[l] + r - off[l]] = 1;
      }
      // level 2: the reflection pad (1, 0) -- local row 1 mirrored into row -1, the gap row in
      // front of the window -- and conv_post's rows [-1, 16T); the row in front only while the
      // window starts at local row 0 (the window moves past it only once conv_post has read it)
      std::memcpy(mr + A[2], m[2] + A[2], (size_t)P.cap[2]);
      std::memcpy(mp + A[2], m[2] + A[2], (size_t)P.cap[2]);
      if (off[2] == 0) {
        mr[A[2] + 1] |= 2;
        mr[A[2] - 1] |= 4;
        mp[A[2] - 1] = 1;
      }
      // upsampler row maps: delay-line step q (local, 1 .. T'+1) at window row A + q - off
      // writes outputs 4q + r - 6 (local) at window row A' + 4q + r - 6 - off'
      for (int u = 0; u < 2; ++u) {
        const int64_t Tin = level_len(u, T[s]);
        const int64_t base = A[u + 1] - off[u + 1] - 4 * (A[u] - off[u]) - 6;
        for (int64_t qq = std::max<int64_t>(1, off[u]); qq <= Tin + 1 && qq - off[u] < P.cap[u]; ++qq)
          if (4 * qq - 6 >= off[u + 1] - 16 && 4 * qq - 3 - off[u + 1] <= P.cap[u + 1])
            ob[u][A[u] + qq - off[u]] = (int)base;   // outputs inside the window (and its gap)
      }
      a0[s] = A[0] - off[0];
      rw[s] = A[2] - off[2] - 1;
      // window moves: rows [off, off + mv) of every tensor to the window start
      for (int l = 0; l < 3; ++l) {
        const int64_t mvr = P.mv[l][ks];
        if (mvr <= 0) continue;
        const int64_t d = off[l] - P.off[l][(size_t)(k - 1) * n + s];
        for (const auto &tc : tens[l]) {
          cp[3 * ncp + 0] = (long long)(tc.first + (size_t)(A[l] + d) * tc.second);
          cp[3 * ncp + 1] = (long long)(tc.first + (size_t)A[l] * tc.second);
          cp[3 * ncp + 2] = (long long)(mvr * tc.second);
          ++ncp;
        }
      }
    }
    const int nm = ncp;
    for (int s = 0; s < n; ++s) {
      if (P.done[s] != k) continue;
      // the stream's last pass: clear the rows after its end (the zero padding its convs read)
      const size_t ks = (size_t)k * n + s;
      for (int l = 0; l < 3; ++l) {
        const int64_t from = level_len(l, T[s]) - P.off[l][ks];
        const int64_t rows = std::min<int64_t>(kPad, P.cap[l] - from);
        if (rows <= 0) continue;
        for (const auto &tc : tens[l]) {
          cp[3 * ncp + 0] = -1;
          cp[3 * ncp + 1] = (long long)(tc.first + (size_t)(P.A[l][s] + from) * tc.second);
          cp[3 * ncp + 2] = (long long)(rows * tc.second);
          ++ncp;
        }
      }
    }
    if (nm != nmove[(size_t)k] || ncp - nm > nclear[(size_t)k]) {
      set_error("pt_b200: carried session: pass %d move table mismatch", k);
      return fail();
    }
    t.mask[0] = reinterpret_cast<unsigned char *>(dv + om0);
    t.mask[1] = reinterpret_cast<unsigned char *>(dv + om1);
    t.mask[2] = reinterpret_cast<unsigned char *>(dv + om2);
    t.mask_refl = reinterpret_cast<unsigned char *>(dv + omr);
    t.mask_post = reinterpret_cast<unsigned char *>(dv + omp);
    t.ob01 = reinterpret_cast<int *>(dv + oo1);
    t.ob12 = reinterpret_cast<int *>(dv + oo2);
    t.a0 = reinterpret_cast<long long *>(dv + oa0);
    t.row0 = reinterpret_cast<long long *>(dv + orw);
    t.cp = reinterpret_cast<long long *>(dv + ocp);
    t.ncp_move = nm;
    t.ncp_clear = ncp - nm;
  }
  // the pass plan after the pass tables
  {
    char *h = host.data() + pt_off[(size_t)np];
    char *dv = dev_tab + pt_off[(size_t)np];
    size_t o = 0;
    auto put = [&](const void *src, size_t bytes) {
      std::memcpy(h + o, src, bytes);
      char *dst = dv + o;
      o += alb(bytes);
      return dst;
    };
    c->tiles = reinterpret_cast<int2 *>(put(P.tiles.data(), P.tiles.size() * sizeof(int2)));
    c->f0 = reinterpret_cast<long long *>(put(P.f0.data(), na * 8));
    c->f1 = reinterpret_cast<long long *>(put(P.f1.data(), na * 8));
    c->klo = reinterpret_cast<long long *>(put(P.klo.data(), na * 8));
    c->khi = reinterpret_cast<long long *>(put(P.khi.data(), na * 8));
    c->jb = reinterpret_cast<long long *>(put(P.jb.data(), na * 8));
  }
  if (cudaMemsetAsync(c->block, 0, act_b, st) != cudaSuccess ||
      cudaMemcpyAsync(dev_tab, host.data(), tab_b, cudaMemcpyHostToDevice, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess) {
    set_error("pt_b200: carried session set-up failed (%s)", cudaGetErrorString(cudaGetLastError()));
    return fail();
  }
  if (tail_prepare()) return fail();
  return c;
}

int pt_b200_carry_passes(const pt_b200_carry *c) { return c ? c->P.npass : -1; }

int64_t pt_b200_carry_bytes(const pt_b200_carry *c) { return c ? (int64_t)c->bytes : -1; }

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
