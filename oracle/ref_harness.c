/* ref_harness.c -- drives the reference's OWN CPU code for the decoder hot path (TEST
 * INFRASTRUCTURE, built only by oracle/Makefile into oracle/_ref/libptref.so).
 *
 * The reference interpreter source is compiled where it lies (read-only, never copied): this
 * translation unit #includes runtime/v21/src/pt_v21_host.c so that its file-static ops (un_op,
 * bin_op, op_einsum, op_pad, op_slice) can be called, and links runtime/v21/gen/pt_graph.c for
 * the tables that file references.  The functions below only wire those ops together in the
 * order of ref/v21_graph_trace.txt nodes 3819-4065; every arithmetic step is the reference's.
 *
 * Used to (1) pin the restatement in oracle/pt_oracle.c, (2) generate tests/golden fixtures and
 * (3) time the reference CPU path in bench.py (the reference arm and the cpu_baseline).
 */
#include "pt_v21_host.c"
#include "pt_oracle.h" /* only for the or_dec_weights layout shared with the restatement */

#define REF_EXPORT __attribute__((visibility("default")))

static pt_ctx *ref_ctx(void) {
  static __thread pt_ctx *c;
  if (!c) c = (pt_ctx *) calloc(1, sizeof(pt_ctx));
  return c;
}

REF_EXPORT int ref_conv(const float *X, int64_t ldx, int64_t cin, float *Y, int64_t ldy, int64_t n,
                        int cout, int K, int stride, int pad, int dil, const float *wp,
                        const float *bias, int64_t batch, int epi0, int epi1, float a0, float a1) {
  return pt_v21_conv_cpu(ref_ctx(), X, ldx, cin, Y, ldy, n, cout, K, stride, pad, dil, wp, bias,
                         batch, -1, -1, epi0, epi1, a0, a1);
}

REF_EXPORT int ref_convT(const float *X, int64_t ldx, int64_t cin, int64_t tin, float *Y,
                         int64_t ldy, int cout, int s, int pad, int K, const float *wp,
                         const float *bias, int64_t batch) {
  return pt_v21_convT_cpu(ref_ctx(), X, ldx, cin, tin, Y, ldy, cout, s, pad, K, wp, bias, batch,
                          -1, -1);
}

/* ---------------------------------------------------------------- tensor plumbing */
static int t_new(pt_ctx *c, pt_tv *t, int nd, int64_t d0, int64_t d1, int64_t d2, int64_t d3) {
  int64_t d[4] = {d0, d1, d2, d3};
  memset(t, 0, sizeof(*t));
  return tv_alloc_nz(c, t, DT_F32, d, nd, 0);
}
/* a same-buffer view with another shape (Reshape / Squeeze are views in the graph) */
static pt_tv t_view(const pt_tv *s, int nd, int64_t d0, int64_t d1, int64_t d2, int64_t d3) {
  pt_tv v = *s;
  int64_t d[4] = {d0, d1, d2, d3};
  v.ndim = nd;
  for (int i = 0; i < PT_V21_MAX_RANK; i++) v.d[i] = i < nd ? d[i] : 1;
  return v;
}
static pt_tv t_scalar(float *v) {
  pt_tv t;
  memset(&t, 0, sizeof(t));
  t.dt = DT_F32;
  t.ndim = 0;
  t.n = 1;
  for (int i = 0; i < PT_V21_MAX_RANK; i++) t.d[i] = 1;
  t.p = v;
  t.alive = 1;
  return t;
}
static pt_tv t_wrap(float *p, int nd, int64_t d0, int64_t d1, int64_t d2) {
  pt_tv t;
  memset(&t, 0, sizeof(t));
  int64_t d[3] = {d0, d1, d2};
  t.dt = DT_F32;
  t.ndim = nd;
  t.n = 1;
  for (int i = 0; i < PT_V21_MAX_RANK; i++) {
    t.d[i] = i < nd ? d[i] : 1;
    if (i < nd) t.n *= d[i];
  }
  t.p = p;
  t.alive = 1;
  return t;
}

/* PT_CONV node on the CPU path (runtime/v21/src/pt_v21_host.c:3243-3405): zero-padded scratch,
 * pt_v21_conv_cpu, cout4 trim.  X [N][cin][T] -> O [N][cout][Tout]. */
static int node_conv(pt_ctx *c, const pt_tv *X, int cin, int cout, int K, int pad, int dil,
                     const float *wp, const float *bias, int epi0, float a0, pt_tv *O) {
  const int64_t T = X->d[X->ndim - 1], N = X->ndim >= 3 ? X->d[0] : 1;
  const int cout4 = (cout + 3) / 4 * 4;
  const int64_t Tout = T + 2 * (int64_t) pad - (int64_t) (K - 1) * dil;
  if (t_new(c, O, 3, N, cout, Tout, 1)) return -1;
  const int64_t ldxp = T + 2 * (int64_t) pad;
  float *xp = (float *) calloc((size_t) (N * cin * ldxp), sizeof(float));
  float *yp = cout4 == cout ? (float *) O->p : (float *) malloc(sizeof(float) * N * cout4 * Tout);
  if (!xp || !yp) return -1;
  for (int64_t b = 0; b < N; b++)
    for (int ci = 0; ci < cin; ci++)
      memcpy(xp + (b * cin + ci) * ldxp + pad, (const float *) X->p + (b * cin + ci) * T,
             sizeof(float) * T);
  pt_v21_conv_cpu(c, xp, ldxp, cin, yp, Tout, Tout, cout, K, 1, pad, dil, wp, bias, N, -1, -1,
                  epi0, 0, a0, 0.0f);
  if (cout4 != cout) {
    for (int64_t b = 0; b < N; b++)
      memcpy((float *) O->p + b * cout * Tout, yp + b * cout4 * Tout, sizeof(float) * cout * Tout);
    free(yp);
  }
  free(xp);
  return 0;
}

/* PT_CONVT node (runtime/v21/src/pt_v21_host.c:3406-3435) */
static int node_convT(pt_ctx *c, const pt_tv *X, int cin, int cout, int K, int s, int pad,
                      const float *wp, const float *bias, pt_tv *O) {
  const int64_t Tin = X->d[X->ndim - 1], N = X->ndim >= 3 ? X->d[0] : 1;
  const int cout4 = (cout + 3) / 4 * 4;
  const int64_t Lout = (Tin - 1) * s - 2 * (int64_t) pad + K;
  if (t_new(c, O, 3, N, cout, Lout, 1)) return -1;
  if (cout4 == cout) {
    pt_v21_convT_cpu(c, (const float *) X->p, Tin, cin, Tin, (float *) O->p, Lout, cout, s, pad, K,
                     wp, bias, N, -1, -1);
  } else {
    float *sc = (float *) malloc(sizeof(float) * N * cout4 * Lout);
    if (!sc) return -1;
    pt_v21_convT_cpu(c, (const float *) X->p, Tin, cin, Tin, sc, Lout, cout, s, pad, K, wp, bias,
                     N, -1, -1);
    for (int64_t b = 0; b < N; b++)
      memcpy((float *) O->p + b * cout * Lout, sc + b * cout4 * Lout, sizeof(float) * cout * Lout);
    free(sc);
  }
  return 0;
}

/* ---------------------------------------------------------------- tail constants (inputs) */
/* spec/v21_layers.json constants 4009 (Hann window) and 3617 (Hann^2 window-sum kernel) */
static const float h_win16[16] = {
    0.0f,        0.03806024789810181f, 0.1464466154575348f, 0.30865830183029175f,
    0.5f,        0.691341757774353f,   0.8535534143447876f, 0.961939811706543f,
    1.0f,        0.9619397521018982f,  0.853553295135498f,  0.6913415789604187f,
    0.5f,        0.3086581826210022f,  0.14644649624824524f, 0.03806021809577942f};
static const float h_win2_16[16] = {
    0.0f,  0.0014485825086012483f, 0.02144661173224449f, 0.09526994824409485f,
    0.25f, 0.4779534339904785f,    0.7285534143447876f,  0.9253281950950623f,
    1.0f,  0.9253280758857727f,    0.7285532355308533f,  0.477953165769577f,
    0.25f, 0.09526987373828888f,   0.021446576341986656f, 0.0014485801802948117f};

REF_EXPORT int ref_tail(const float *post, int64_t Tp, const float *pqmf, float *wav) {
  pt_ctx *c = ref_ctx();
  if (Tp < 2) return -1;
  /* irfft bases, nodes 3530-3615: w = ScatterND([9,1] of 2, ends -> 1); Bc = (w*C24)/16,
   * Bs = (Neg(w)*C26)/16, with the [9,16] cos / sin tables as fp32-rounded constants */
  float w9[9], c24[144], c26[144], sixteen = 16.0f;
  for (int k = 0; k < 9; k++) w9[k] = (k == 0 || k == 8) ? 1.0f : 2.0f;
  for (int k = 0; k < 9; k++)
    for (int n = 0; n < 16; n++) {
      const double ang = 2.0 * M_PI * (double) k * (double) n / 16.0;
      c24[k * 16 + n] = (float) cos(ang);
      c26[k * 16 + n] = (float) sin(ang);
    }
  pt_tv tw = t_wrap(w9, 2, 9, 1, 1), tc24 = t_wrap(c24, 2, 9, 16, 1), tc26 = t_wrap(c26, 2, 9, 16, 1);
  pt_tv t16 = t_scalar(&sixteen), m6, bc, nw, m7, bs;
  if (bin_op(c, PT_MUL, &tw, &tc24, &m6) || bin_op(c, PT_DIV, &m6, &t16, &bc)) return -1;
  if (un_op(c, PT_NEG, &tw, NULL, &nw, 0.0f) || bin_op(c, PT_MUL, &nw, &tc26, &m7) ||
      bin_op(c, PT_DIV, &m7, &t16, &bs))
    return -1;

  pt_tv P = t_wrap((float *) post, 3, 1, 72, Tp);
  pt_tv R6 = t_view(&P, 4, 1, 4, 18, Tp);                                  /* Reshape_6 */
  int64_t st0[1] = {0}, en9[1] = {9}, st9[1] = {9}, enmax[1] = {INT64_MAX}, ax2[1] = {2};
  pt_tv S4, E, S5, Sn, M24, Cs, M27, Sn1, M28, E0, E1, A4, M29;
  if (op_slice(c, &R6, st0, en9, ax2, 1, 1, &S4) || un_op(c, PT_EXP, &S4, NULL, &E, 0.0f)) return -1;
  float pi = 3.1415927410125732f;
  pt_tv tpi = t_scalar(&pi);
  if (op_slice(c, &R6, st9, enmax, ax2, 1, 1, &S5) || un_op(c, PT_SIN, &S5, NULL, &Sn, 0.0f) ||
      bin_op(c, PT_MUL, &Sn, &tpi, &M24))
    return -1;
  pt_tv R7 = t_view(&E, 3, 4, 9, Tp, 1), R8 = t_view(&M24, 3, 4, 9, Tp, 1);  /* Reshape_7/8 */
  if (un_op(c, PT_COS, &R8, NULL, &Cs, 0.0f) || bin_op(c, PT_MUL, &R7, &Cs, &M27)) return -1;
  if (un_op(c, PT_SIN, &R8, NULL, &Sn1, 0.0f) || bin_op(c, PT_MUL, &R7, &Sn1, &M28)) return -1;
  memset(&E0, 0, sizeof(E0));
  memset(&E1, 0, sizeof(E1));
  if (op_einsum(c, "bkt,kn->bnt", &M27, &bc, &E0) || op_einsum(c, "bkt,kn->bnt", &M28, &bs, &E1))
    return -1;
  float win[16];
  memcpy(win, h_win16, sizeof(win));
  pt_tv twin = t_wrap(win, 3, 1, 16, 1);
  if (bin_op(c, PT_ADD, &E0, &E1, &A4) || bin_op(c, PT_MUL, &A4, &twin, &M29)) return -1;

  /* ConvTranspose with the eye(16) kernel [16][1][16], packed [4 phases][4 taps][16][4] */
  float wola[4 * 4 * 16 * 4], wenv[4 * 4 * 1 * 4], wup[4 * 1 * 4 * 4], wpq[63 * 4 * 4];
  memset(wola, 0, sizeof(wola));
  memset(wenv, 0, sizeof(wenv));
  memset(wup, 0, sizeof(wup));
  memset(wpq, 0, sizeof(wpq));
  for (int r = 0; r < 4; r++)
    for (int j = 0; j < 4; j++) {
      const int k = r + 4 * j;                       /* ONNX tap of phase r, tap j */
      wola[((r * 4 + j) * 16 + k) * 4 + 0] = 1.0f;   /* input channel ci == k feeds cout 0 */
      wenv[((r * 4 + j) * 1 + 0) * 4 + 0] = h_win2_16[k];
    }
  /* ConvTranspose_2 kernel 4*delta(i==j, tap 0): phase 0 / tap 0 only, packed rows r*4+c */
  for (int i = 0; i < 4; i++) wup[((0 * 1 + 0) * 4 + i) * 4 + i] = 4.0f;
  /* the 63-tap PQMF conv 4 -> 1, ONNX [1][4][63] packed as [1][63][4][4] (lane 0 real) */
  for (int k = 0; k < 63; k++)
    for (int ci = 0; ci < 4; ci++) wpq[(k * 4 + ci) * 4 + 0] = pqmf[ci * 63 + k];
  float zb[4] = {0.0f, 0.0f, 0.0f, 0.0f};

  pt_tv OL, S6, ENV, CL, D5, S7, U, PD, WV;
  if (node_convT(c, &M29, 16, 1, 16, 4, 0, wola, zb, &OL)) return -1;
  int64_t en1[1] = {1}, ax1[1] = {1};
  if (op_slice(c, &M29, st0, en1, ax1, 1, 1, &S6)) return -1;                /* Slice_6 */
  for (int64_t i = 0; i < S6.n; i++) ((float *) S6.p)[i] = 1.0f;           /* ConstantOfShape_22 */
  if (node_convT(c, &S6, 1, 1, 16, 4, 0, wenv, zb, &ENV)) return -1;
  float lo = 1e-9f;
  pt_tv tlo = t_scalar(&lo);
  if (un_op(c, PT_CLIP, &ENV, &tlo, &CL, 0.0f) || bin_op(c, PT_DIV, &OL, &CL, &D5)) return -1;
  int64_t st8[1] = {8}, enm8[1] = {-8};
  if (op_slice(c, &D5, st8, enm8, ax2, 1, 1, &S7)) return -1;                /* Slice_7 */
  const int64_t Ls = S7.d[2];
  pt_tv SQ = t_view(&S7, 3, 1, 4, Ls, 1);                                    /* Reshape_9+Squeeze */
  if (node_convT(c, &SQ, 4, 4, 4, 4, 0, wup, zb, &U)) return -1;             /* ConvTranspose_2 */
  int64_t pads[6] = {0, 0, 31, 0, 0, 31};
  if (op_pad(c, &U, pads, 0.0, 0, &PD)) return -1;                           /* Pad */
  if (node_conv(c, &PD, 4, 1, 63, 0, 1, wpq, zb, 0, 0.0f, &WV)) return -1;   /* Conv -> wav */
  memcpy(wav, WV.p, sizeof(float) * WV.n);

  pt_tv *own[] = {&m6, &bc, &nw, &m7, &bs, &S4, &E, &S5, &Sn, &M24, &Cs, &M27, &Sn1, &M28,
                  &E0, &E1, &A4, &M29, &OL, &S6, &ENV, &CL, &D5, &S7, &U, &PD, &WV};
  for (size_t i = 0; i < sizeof(own) / sizeof(own[0]); i++) tv_free(c, own[i]);
  return 0;
}

/* ---------------------------------------------------------------- whole decoder */
REF_EXPORT int ref_decode(const or_dec_weights *w, const float *z, int64_t T, float *wav) {
  static const int kk[3] = {3, 7, 11}, dd[3] = {1, 3, 5};
  pt_ctx *c = ref_ctx();
  const float lr = 0.10000000149011612f, lr_final = 0.009999999776482582f;
  float three = 3.0f;
  pt_tv t3 = t_scalar(&three);
  pt_tv Z = t_wrap((float *) z, 3, 1, 192, T);
  pt_tv X;
  if (node_conv(c, &Z, 192, 512, 7, 3, 1, w->pre_w, w->pre_b, 1, lr, &X)) return -1;
  int C = 512;
  for (int stage = 0; stage < 2; stage++) {
    const int Co = C / 2;
    pt_tv U, LU, ACC;
    memset(&ACC, 0, sizeof(ACC));
    if (node_convT(c, &X, C, Co, 16, 4, 6, w->ups_w[stage], w->ups_b[stage], &U)) return -1;
    tv_free(c, &X);
    if (un_op(c, PT_LEAKYRELU, &U, NULL, &LU, lr)) return -1;
    for (int rb = 0; rb < 3; rb++) {
      const int r = stage * 3 + rb, K = kk[rb];
      pt_tv XR = U, XT;   /* running residual: starts as the ups output (not owned here) */
      int xr_own = 0, xt_own = 0;
      for (int j = 0; j < 3; j++) {
        pt_tv H, Y, NX;
        const pt_tv *in = j == 0 ? &LU : &XT;
        if (node_conv(c, in, Co, Co, K, dd[j] * (K - 1) / 2, dd[j], w->rb_w1[r][j], w->rb_b1[r][j],
                      1, lr, &H))
          return -1;
        if (node_conv(c, &H, Co, Co, K, (K - 1) / 2, 1, w->rb_w2[r][j], w->rb_b2[r][j], 0, 0.0f, &Y))
          return -1;
        tv_free(c, &H);
        if (bin_op(c, PT_ADD, &Y, &XR, &NX)) return -1;
        tv_free(c, &Y);
        if (xr_own) tv_free(c, &XR);
        XR = NX;
        xr_own = 1;
        if (xt_own) tv_free(c, &XT);
        xt_own = 0;
        if (j < 2) {
          if (un_op(c, PT_LEAKYRELU, &XR, NULL, &XT, lr)) return -1;
          xt_own = 1;
        }
      }
      if (rb == 0) {
        ACC = XR;
      } else {
        pt_tv NA;
        if (bin_op(c, PT_ADD, &ACC, &XR, &NA)) return -1;
        tv_free(c, &ACC);
        tv_free(c, &XR);
        ACC = NA;
      }
    }
    pt_tv DV;
    if (bin_op(c, PT_DIV, &ACC, &t3, &DV)) return -1;
    if (un_op(c, PT_LEAKYRELU, &DV, NULL, &X, stage == 0 ? lr : lr_final)) return -1;
    tv_free(c, &ACC);
    tv_free(c, &DV);
    tv_free(c, &U);
    tv_free(c, &LU);
    C = Co;
  }
  /* reflection_pad (1, 0) then subband_conv_post */
  pt_tv PADX, POST;
  int64_t pads[6] = {0, 0, 1, 0, 0, 0};
  if (op_pad(c, &X, pads, 0.0, 1, &PADX)) return -1;
  if (node_conv(c, &PADX, 128, 72, 7, 3, 1, w->post_w, w->post_b, 0, 0.0f, &POST)) return -1;
  const int r = ref_tail((const float *) POST.p, POST.d[2], w->pqmf, wav);
  tv_free(c, &X);
  tv_free(c, &PADX);
  tv_free(c, &POST);
  return r;
}
