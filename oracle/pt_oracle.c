/* pt_oracle.c -- CPU restatement of the PrimeTTS v2.1 decoder hot path (TEST INFRASTRUCTURE).
 *
 * This file is the checker, never the product: the shipped library (prime-tts_b200/csrc) does not
 * link it, and the product path fails loudly instead of falling back to it.
 *
 * Each routine follows the reference CPU code's fp32 operation order (cited per function), so a
 * build with the reference's own flags (gcc -O3 -std=gnu11, runtime/v21/Makefile:11) reproduces
 * the reference bit for bit.  tests/test_oracle.py pins that claim against oracle/_ref (the
 * reference's own sources compiled by oracle/Makefile) and against tests/golden/ fixtures.
 */
#include "pt_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

static int r4i(int n) { return (n + 3) / 4 * 4; }

/* ------------------------------------------------------------------------------------------ */
/* Fused conv epilogue codes: runtime/v21/src/pt_v21_host.c:2287-2297 */
static float epi_apply(float v, int op, float a) {
  switch (op) {
    case 1: return v >= 0.0f ? v : a * v;
    case 2: return v > 0.0f ? v : 0.0f;
    case 3: return v * a;
    case 4: return v + a;
    default: return v;
  }
}

/* runtime/v21/src/pt_v21_host.c:2299-2361.  Per output element the sum starts at the bias and
 * adds w*x for tap k ascending, then input channel ascending; zero inputs are skipped (they add
 * an exact +-0).  The loop nest below visits (k, ci) in that order for every output. */
void or_conv(const float *X, int64_t ldx, int64_t cin, float *Y, int64_t ldy, int64_t Tout,
             int cout, int K, int stride, int dil, const float *wp, const float *bias,
             int64_t batch, int epi0, int epi1, float a0, float a1) {
  const int c4 = r4i(cout);
  for (int64_t b = 0; b < batch; b++) {
    const float *xb = X + b * cin * ldx;
    float *yb = Y + b * (int64_t) c4 * ldy;
    for (int co = 0; co < c4; co++) {
      const float init = (bias != NULL && co < cout) ? bias[co] : 0.0f;
      float *row = yb + (int64_t) co * ldy;
      for (int64_t t = 0; t < Tout; t++) row[t] = init;
    }
    for (int k = 0; k < K; k++) {
      for (int g = 0; g < c4 / 4; g++) {
        const float *wg = wp + ((int64_t) g * K + k) * cin * 4;
        float *y0 = yb + (int64_t) (4 * g) * ldy;
        for (int64_t ci = 0; ci < cin; ci++) {
          const float *xr = xb + ci * ldx + (int64_t) k * dil;
          const float w0 = wg[4 * ci + 0], w1 = wg[4 * ci + 1];
          const float w2 = wg[4 * ci + 2], w3 = wg[4 * ci + 3];
          for (int64_t t = 0; t < Tout; t++) {
            const float xv = xr[t * stride];
            if (xv == 0.0f) continue;
            y0[t] += w0 * xv;
            y0[ldy + t] += w1 * xv;
            y0[2 * ldy + t] += w2 * xv;
            y0[3 * ldy + t] += w3 * xv;
          }
        }
      }
    }
    if (epi0 || epi1) {
      for (int co = 0; co < c4; co++)
        for (int64_t t = 0; t < Tout; t++) {
          float v = yb[(int64_t) co * ldy + t];
          if (epi0) v = epi_apply(v, epi0, a0);
          if (epi1) v = epi_apply(v, epi1, a1);
          yb[(int64_t) co * ldy + t] = v;
        }
    }
  }
}

/* runtime/v21/src/pt_v21_host.c:2547-2593.  Output index oi = q*s + r - pad for the delay-line
 * step q (0 .. tin+ntap-2, the last ntap-1 steps being the zero-input tail flush) and phase r;
 * tap j of phase r reads input column q - j.  Per output element: bias, then tap ascending,
 * then input channel ascending. */
void or_convT(const float *X, int64_t ldx, int64_t cin, int64_t tin, float *Y, int64_t ldy,
              int cout, int s, int pad, int K, const float *wp, const float *bias, int64_t batch) {
  const int nt = (K + s - 1) / s;
  const int c4 = r4i(cout);
  const int64_t Q = tin + nt - 1;
  const int64_t Lout = (tin - 1) * s - 2 * (int64_t) pad + K;
  for (int64_t b = 0; b < batch; b++) {
    const float *xb = X + b * cin * ldx;
    float *yb = Y + b * (int64_t) c4 * ldy;
    for (int co = 0; co < c4; co++) {
      const float init = (bias != NULL && co < cout) ? bias[co] : 0.0f;
      for (int64_t t = 0; t < Lout; t++) yb[(int64_t) co * ldy + t] = init;
    }
    for (int64_t q = 0; q < Q; q++) {
      for (int r = 0; r < s; r++) {
        const int64_t oi = q * s + r - pad;
        if (oi < 0 || oi >= Lout) continue;
        for (int g = 0; g < c4 / 4; g++) {
          const float *wg = wp + ((int64_t) (r * c4 / 4 + g) * nt) * cin * 4;
          for (int j = 0; j < nt && j <= q; j++) {
            const int64_t col = q - j;
            if (col >= tin) continue;
            for (int64_t ci = 0; ci < cin; ci++) {
              const float xv = xb[ci * ldx + col];
              if (xv == 0.0f) continue;
              const float *w = wg + ((int64_t) j * cin + ci) * 4;
              for (int p = 0; p < 4; p++) yb[(int64_t) (4 * g + p) * ldy + oi] += w[p] * xv;
            }
          }
        }
      }
    }
  }
}

/* tools/export_v21.py:88-95 */
void or_pack_conv(const float *W, int cout, int cin, int K, float *wp) {
  const int c4 = r4i(cout);
  for (int g = 0; g < c4 / 4; g++)
    for (int k = 0; k < K; k++)
      for (int ci = 0; ci < cin; ci++)
        for (int p = 0; p < 4; p++) {
          const int co = 4 * g + p;
          wp[(((int64_t) g * K + k) * cin + ci) * 4 + p] =
              co < cout ? W[((int64_t) co * cin + ci) * K + k] : 0.0f;
        }
}

/* tools/export_v21.py:107-121: phase r / channel c / tap j holds ONNX tap k = r + j*s */
void or_pack_convT(const float *W, int cin, int cout, int K, int s, float *wp) {
  const int c4 = r4i(cout), nt = (K + s - 1) / s;
  for (int r = 0; r < s; r++)
    for (int g = 0; g < c4 / 4; g++)
      for (int j = 0; j < nt; j++)
        for (int ci = 0; ci < cin; ci++)
          for (int p = 0; p < 4; p++) {
            const int c = 4 * g + p, k = r + j * s;
            const int64_t dst = ((((int64_t) (r * c4 / 4 + g)) * nt + j) * cin + ci) * 4 + p;
            wp[dst] = (c < cout && k < K) ? W[((int64_t) ci * cout + c) * K + k] : 0.0f;
          }
}

int64_t or_packed_conv_elems(int cout, int cin, int K) { return (int64_t) r4i(cout) * K * cin; }
int64_t or_packed_convT_elems(int cin, int cout, int K, int s) {
  return (int64_t) s * r4i(cout) * ((K + s - 1) / s) * cin;
}

/* ------------------------------------------------------------------------------------------ */
/* elementwise ops, x86 paths of runtime/v21/src/pt_v21_host.c */

/* un_op LEAKYRELU, :605-606 */
static void leaky(const float *a, float *o, int64_t n, float alpha) {
  for (int64_t i = 0; i < n; i++) o[i] = a[i] >= 0.0f ? a[i] : alpha * a[i];
}

/* un_op EXP/SIN/COS, :545-551 (fp32 libm for n >= 4096) and :627-645 (double path below) */
static void un_trans(int which, const float *a, float *o, int64_t n) {
  if (n >= 4096) {
    for (int64_t i = 0; i < n; i++)
      o[i] = which == 0 ? expf(a[i]) : which == 1 ? sinf(a[i]) : cosf(a[i]);
  } else {
    for (int64_t i = 0; i < n; i++) {
      const double v = (double) a[i];
      o[i] = (float) (which == 0 ? exp(v) : which == 1 ? sin(v) : cos(v));
    }
  }
}

/* ------------------------------------------------------------------------------------------ */
/* tail constants */

/* spec/v21_layers.json constant idx 4009 (/dec/Constant_109_output_0): the periodic Hann(16)
 * window exactly as the export recorded it (fp32 values, not symmetric in the last bit). */
static const float k_win16[16] = {
    0.0f,        0.03806024789810181f, 0.1464466154575348f, 0.30865830183029175f,
    0.5f,        0.691341757774353f,   0.8535534143447876f, 0.961939811706543f,
    1.0f,        0.9619397521018982f,  0.853553295135498f,  0.6913415789604187f,
    0.5f,        0.3086581826210022f,  0.14644649624824524f, 0.03806021809577942f};
/* constant idx 3617 (onnx::ConvTranspose_5159): the window-sum (Hann^2) kernel */
static const float k_win2_16[16] = {
    0.0f,  0.0014485825086012483f, 0.02144661173224449f, 0.09526994824409485f,
    0.25f, 0.4779534339904785f,    0.7285534143447876f,  0.9253281950950623f,
    1.0f,  0.9253280758857727f,    0.7285532355308533f,  0.477953165769577f,
    0.25f, 0.09526987373828888f,   0.021446576341986656f, 0.0014485801802948117f};

/* Nodes 3530-3615: w = [1,2,...,2,1] (ScatterND on a [9,1] tensor of 2s), then
 * Bc = (w * C24) / 16 and Bs = ((-w) * C26) / 16 in fp32, where C24 / C26 are the [9,16]
 * cos / sin tables (graph constants 3607 / 3612; their values are not recorded in the reference
 * spec, so they are taken as round_fp32(cos / sin(2*pi*k*n/16)) ). */
void or_tail_constants(float *win16, float *win2_16, float *bc, float *bs) {
  for (int n = 0; n < 16; n++) {
    if (win16) win16[n] = k_win16[n];
    if (win2_16) win2_16[n] = k_win2_16[n];
  }
  for (int k = 0; k < 9; k++) {
    const float wk = (k == 0 || k == 8) ? 1.0f : 2.0f;
    for (int n = 0; n < 16; n++) {
      const double ang = 2.0 * M_PI * (double) k * (double) n / 16.0;
      const float c = (float) cos(ang), sn = (float) sin(ang);
      if (bc) bc[k * 16 + n] = (wk * c) / 16.0f;
      if (bs) bs[k * 16 + n] = ((-wk) * sn) / 16.0f;
    }
  }
}

/* op_einsum 'bkt,kn->bnt' fast path, runtime/v21/src/pt_v21_host.c:1963-1995: the k-sum is
 * accumulated in double (k ascending, zero basis entries skipped) and rounded once. */
static void einsum_bkt_kn(const float *A, const float *B, float *O, int64_t nb, int K, int N,
                          int64_t T, double *acc) {
  for (int64_t b = 0; b < nb; b++) {
    for (int64_t i = 0; i < (int64_t) N * T; i++) acc[i] = 0.0;
    for (int k = 0; k < K; k++) {
      const float *arow = A + (b * K + k) * T;
      for (int n = 0; n < N; n++) {
        const double bv = (double) B[k * N + n];
        if (bv == 0.0) continue;
        double *an = acc + (int64_t) n * T;
        for (int64_t t = 0; t < T; t++) an[t] += bv * (double) arow[t];
      }
    }
    for (int64_t i = 0; i < (int64_t) N * T; i++) O[b * N * T + i] = (float) acc[i];
  }
}

/* ------------------------------------------------------------------------------------------ */
/* The iSTFT + PQMF tail, graph nodes 3957-4065 (see ref/v21_graph_trace.txt). */
int or_tail(const float *post, int64_t Tp, const float *pqmf, float *wav) {
  if (Tp < 2) return -1;
  const int64_t nb = 4;                   /* subbands (Reshape_6 [1,4,18,Tp]) */
  const int64_t nbin = 9, nfft = 16, hop = 4;
  const int64_t n9 = nb * nbin * Tp;
  float win[16], win2[16], bc[144], bs[144];
  or_tail_constants(win, win2, bc, bs);

  float *mag = malloc(sizeof(float) * n9), *ph = malloc(sizeof(float) * n9);
  float *tmp = malloc(sizeof(float) * n9), *re = malloc(sizeof(float) * n9);
  float *im = malloc(sizeof(float) * n9);
  float *ere = malloc(sizeof(float) * nb * nfft * Tp), *eim = malloc(sizeof(float) * nb * nfft * Tp);
  double *acc = malloc(sizeof(double) * nfft * Tp);
  const int64_t Lo = (Tp - 1) * hop + nfft;         /* ConvTranspose output length */
  const int64_t Ls = Lo - 16;                       /* Slice_7 [8:-8] */
  const int64_t Lu = Ls * 4;                        /* ConvTranspose_2 x4 */
  float *ola = malloc(sizeof(float) * nb * 4 * Lo), *env = malloc(sizeof(float) * nb * 4 * Lo);
  float *ones = malloc(sizeof(float) * nb * Tp);
  float *sl = malloc(sizeof(float) * nb * Ls);
  float *up = malloc(sizeof(float) * nb * Lu);
  float *upad = malloc(sizeof(float) * nb * (Lu + 62));
  float *w_ola = malloc(sizeof(float) * or_packed_convT_elems(16, 1, 16, 4));
  float *w_env = malloc(sizeof(float) * or_packed_convT_elems(1, 1, 16, 4));
  float *w_up = malloc(sizeof(float) * or_packed_convT_elems(4, 4, 4, 4));
  float *w_pq = malloc(sizeof(float) * or_packed_conv_elems(1, 4, 63));
  float *wav4 = malloc(sizeof(float) * 4 * Lu);
  if (!mag || !ph || !tmp || !re || !im || !ere || !eim || !acc || !ola || !env || !ones || !sl ||
      !up || !upad || !w_ola || !w_env || !w_up || !w_pq || !wav4)
    return -2;

  /* Slice_4 / Slice_5 of Reshape_6: bins 0..8 are log-magnitudes, 9..17 phases */
  for (int64_t b = 0; b < nb; b++)
    for (int64_t k = 0; k < nbin; k++) {
      memcpy(mag + (b * nbin + k) * Tp, post + (b * 18 + k) * Tp, sizeof(float) * Tp);
      memcpy(ph + (b * nbin + k) * Tp, post + (b * 18 + 9 + k) * Tp, sizeof(float) * Tp);
    }
  un_trans(0, mag, mag, n9);                               /* Exp */
  un_trans(1, ph, ph, n9);                                 /* Sin */
  for (int64_t i = 0; i < n9; i++) ph[i] = ph[i] * 3.1415927410125732f;   /* Mul_24 by pi */
  un_trans(2, ph, tmp, n9);                                /* Cos */
  for (int64_t i = 0; i < n9; i++) re[i] = mag[i] * tmp[i];              /* Mul_27 */
  un_trans(1, ph, tmp, n9);                                /* Sin_1 */
  for (int64_t i = 0; i < n9; i++) im[i] = mag[i] * tmp[i];              /* Mul_28 */
  einsum_bkt_kn(re, bc, ere, nb, 9, 16, Tp, acc);          /* Einsum */
  einsum_bkt_kn(im, bs, eim, nb, 9, 16, Tp, acc);          /* Einsum_1 */
  for (int64_t b = 0; b < nb; b++)                          /* Add_4, Mul_29 by the window */
    for (int64_t n = 0; n < nfft; n++)
      for (int64_t t = 0; t < Tp; t++) {
        const int64_t i = (b * nfft + n) * Tp + t;
        ere[i] = (ere[i] + eim[i]) * win[n];
      }

  /* ConvTranspose (eye(16) kernel = overlap-add), ConvTranspose_1 (ones * Hann^2 = window sum) */
  {
    float *W = calloc(16 * 1 * 16, sizeof(float));
    for (int i = 0; i < 16; i++) W[i * 16 + i] = 1.0f;      /* [cin=16][cout=1][K=16] */
    or_pack_convT(W, 16, 1, 16, 4, w_ola);
    free(W);
    or_pack_convT(win2, 1, 1, 16, 4, w_env);
    float zb[4] = {0, 0, 0, 0};
    or_convT(ere, Tp, 16, Tp, ola, Lo, 1, 4, 0, 16, w_ola, zb, nb);
    for (int64_t i = 0; i < nb * Tp; i++) ones[i] = 1.0f;
    or_convT(ones, Tp, 1, Tp, env, Lo, 1, 4, 0, 16, w_env, zb, nb);
  }
  /* Clip(min 1e-9) in double (un_op generic path), Div_5, Slice_7 [8:-8]; row 0 of each cout4 */
  for (int64_t b = 0; b < nb; b++)
    for (int64_t j = 0; j < Ls; j++) {
      const float e = env[b * 4 * Lo + 8 + j];
      const double ed = (double) e, lo = (double) 1e-9f;
      const float ec = (float) (ed > lo ? ed : lo);
      sl[b * Ls + j] = ola[b * 4 * Lo + 8 + j] / ec;
    }
  /* ConvTranspose_2: 4 -> 4, k4 s4, kernel 4*delta(i==j, tap 0) (zero-stuff x4, gain 4) */
  {
    float W[4 * 4 * 4];
    memset(W, 0, sizeof(W));
    for (int i = 0; i < 4; i++) W[(i * 4 + i) * 4 + 0] = 4.0f;   /* [cin][cout][K] */
    or_pack_convT(W, 4, 4, 4, 4, w_up);
    float zb[4] = {0, 0, 0, 0};
    or_convT(sl, Ls, 4, Ls, up, Lu, 4, 4, 0, 4, w_up, zb, 1);
  }
  /* Pad 31|31 (constant 0), Conv 4 -> 1 k63 (no bias in the graph: packed zeros) */
  memset(upad, 0, sizeof(float) * nb * (Lu + 62));
  for (int64_t b = 0; b < nb; b++) memcpy(upad + b * (Lu + 62) + 31, up + b * Lu, sizeof(float) * Lu);
  or_pack_conv(pqmf, 1, 4, 63, w_pq);
  {
    float zb[1] = {0};
    or_conv(upad, Lu + 62, 4, wav4, Lu, Lu, 1, 63, 1, 1, w_pq, zb, 1, 0, 0, 0.0f, 0.0f);
  }
  memcpy(wav, wav4, sizeof(float) * Lu);

  free(mag); free(ph); free(tmp); free(re); free(im); free(ere); free(eim); free(acc);
  free(ola); free(env); free(ones); free(sl); free(up); free(upad);
  free(w_ola); free(w_env); free(w_up); free(w_pq); free(wav4);
  return 0;
}

/* ------------------------------------------------------------------------------------------ */
/* one conv node as the interpreter runs it on the CPU path: zero-padded scratch rows
 * (runtime/v21/src/pt_v21_host.c:3274-3281), then pt_v21_conv_cpu, then the cout4 trim */
static int conv_node(const float *x, int64_t T, int cin, int cout, int K, int pad, int dil,
                     const float *wp, const float *bias, int epi0, float a0, float *y) {
  const int64_t ldxp = T + 2 * (int64_t) pad;
  const int64_t Tout = T + 2 * (int64_t) pad - (int64_t) (K - 1) * dil;
  float *xp = calloc((size_t) cin * ldxp, sizeof(float));
  if (!xp) return -1;
  for (int ci = 0; ci < cin; ci++) memcpy(xp + ci * ldxp + pad, x + (int64_t) ci * T, sizeof(float) * T);
  or_conv(xp, ldxp, cin, y, Tout, Tout, cout, K, 1, dil, wp, bias, 1, epi0, 0, a0, 0.0f);
  free(xp);
  return 0;
}

/* Decoder wiring: ref/v21_graph_trace.txt nodes 3819-4065 with the interpreter's epilogue fusion
 * (a LeakyRelu whose input has that single consumer folds into the conv, pt_v21_host.c:3290-3333;
 * bit-identical to running it separately). */
#define CK(i, src, count) \
  do { if (ck && ck[i]) memcpy(ck[i], (src), sizeof(float) * (size_t) (count)); } while (0)

int or_decode(const or_dec_weights *w, const float *z, int64_t T, float *wav) {
  return or_decode_ckpt(w, z, T, wav, NULL);
}

int or_decode_ckpt(const or_dec_weights *w, const float *z, int64_t T, float *wav,
                   float *const *ck) {
  static const int kk[3] = {3, 7, 11}, dd[3] = {1, 3, 5};
  const float lr = 0.10000000149011612f, lr_final = 0.009999999776482582f;
  int64_t L = T;
  float *x = malloc(sizeof(float) * 512 * T);
  if (!x) return -1;
  /* conv_pre + LeakyRelu (node 3819/3820) */
  if (conv_node(z, T, 192, 512, 7, 3, 1, w->pre_w, w->pre_b, 1, lr, x)) return -1;
  CK(0, x, 512 * T);
  int C = 512;
  for (int stage = 0; stage < 2; stage++) {
    const int Co = C / 2;
    const int64_t Lo = (L - 1) * 4 - 12 + 16;
    float *u = malloc(sizeof(float) * Co * Lo);
    float *lu = malloc(sizeof(float) * Co * Lo);
    float *xr = malloc(sizeof(float) * Co * Lo), *xt = malloc(sizeof(float) * Co * Lo);
    float *h = malloc(sizeof(float) * Co * Lo), *y = malloc(sizeof(float) * Co * Lo);
    float *acc = malloc(sizeof(float) * Co * Lo);
    if (!u || !lu || !xr || !xt || !h || !y || !acc) return -1;
    /* ups.i ConvTranspose (no epilogue in the convT ABI) then resblocks.(3i).LeakyRelu */
    or_convT(x, L, C, L, u, Lo, Co, 4, 6, 16, w->ups_w[stage], w->ups_b[stage], 1);
    leaky(u, lu, (int64_t) Co * Lo, lr);
    const int64_t n = (int64_t) Co * Lo;
    CK(1 + 19 * stage, u, n);
    for (int rb = 0; rb < 3; rb++) {
      const int r = stage * 3 + rb, K = kk[rb];
      memcpy(xr, u, sizeof(float) * n);          /* the running residual x starts at ups out */
      for (int j = 0; j < 3; j++) {
        const float *in = j == 0 ? lu : xt;      /* xt = leaky(x); stage 0 shares the ups leaky */
        /* convs1.j (dilation dd[j], pad d*(K-1)/2) + LeakyRelu */
        if (conv_node(in, Lo, Co, Co, K, dd[j] * (K - 1) / 2, dd[j], w->rb_w1[r][j], w->rb_b1[r][j],
                      1, lr, h))
          return -1;
        CK(2 + 19 * stage + 6 * rb + 2 * j, h, n);
        /* convs2.j (dilation 1) */
        if (conv_node(h, Lo, Co, Co, K, (K - 1) / 2, 1, w->rb_w2[r][j], w->rb_b2[r][j], 0, 0.0f, y))
          return -1;
        for (int64_t i = 0; i < n; i++) xr[i] = y[i] + xr[i];   /* resblocks.r/Add_j */
        if (j < 2) leaky(xr, xt, n, lr);                          /* LeakyRelu_(2j+2) */
        if (j < 2) CK(3 + 19 * stage + 6 * rb + 2 * j, xr, n);
      }
      /* /dec/Add, /dec/Add_1: ((rb0 + rb1) + rb2) */
      if (rb == 0) memcpy(acc, xr, sizeof(float) * n);
      else for (int64_t i = 0; i < n; i++) acc[i] = acc[i] + xr[i];
      if (rb < 2) CK(7 + 19 * stage + 6 * rb, acc, n);
    }
    free(x);
    x = malloc(sizeof(float) * n);
    if (!x) return -1;
    /* Div by 3 (node 3868/3917), then LeakyRelu 0.1 (3869) or 0.01 (3918) */
    for (int64_t i = 0; i < n; i++) acc[i] = acc[i] / 3.0f;
    leaky(acc, x, n, stage == 0 ? lr : lr_final);
    if (stage == 0) CK(19, x, n);
    free(u); free(lu); free(xr); free(xt); free(h); free(y); free(acc);
    C = Co;
    L = Lo;
  }
  /* reflection_pad (1, 0): column 0 mirrors column 1 (op_pad reflect, :1640-1690) */
  const int64_t Tp = L + 1;
  float *xp = malloc(sizeof(float) * 128 * Tp), *post = malloc(sizeof(float) * 72 * Tp);
  if (!xp || !post) return -1;
  for (int c = 0; c < 128; c++) {
    xp[c * Tp] = x[c * L + 1];
    memcpy(xp + c * Tp + 1, x + c * L, sizeof(float) * L);
  }
  CK(38, xp, 128 * Tp);
  /* subband_conv_post 128 -> 72 k7 p3 (node 3935; its consumer is a Reshape: no epilogue) */
  if (conv_node(xp, Tp, 128, 72, 7, 3, 1, w->post_w, w->post_b, 0, 0.0f, post)) return -1;
  CK(39, post, 72 * Tp);
  const int r = or_tail(post, Tp, w->pqmf, wav);
  free(x); free(xp); free(post);
  return r;
}
