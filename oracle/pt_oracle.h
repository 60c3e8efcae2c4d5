/* pt_oracle.h -- CPU restatement of the PrimeTTS v2.1 MB-iSTFT decoder hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the checker the CUDA path is compared against; nothing in
 * the shipped library links it.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline
 * leg may load it.
 *
 * Every function restates the arithmetic of the reference CPU path in its own code, in the same
 * fp32 operation order, so that on identical inputs it is bit-identical to the reference compiled
 * from its own sources (oracle/_ref, built by oracle/Makefile).  Citations are path:line inside the
 * reference project (vieenrose/prime-tts).
 *
 * Layouts (the reference container's packed layouts, tools/export_v21.py:88-121):
 *   conv   weight  [cout4/4][K][cin][4]          (lane p of block b is output channel 4b+p)
 *   convT  weight  [s*cout4/4][ntap][cin][4]     (row r*cout4+c is phase r / channel c, tap j is
 *                                                 ONNX kernel tap r + j*s)
 *   activations    [batch][channels][time]
 */
#ifndef PT_ORACLE_H_
#define PT_ORACLE_H_
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* conv1d over zero-padded input rows: Y[b][co][t] = bias[co] + sum_k sum_ci W * X[b][ci][t*stride
 * + k*dil] (X already holds `pad` zeros on the left), then the fused epilogue codes
 * (1 leaky a, 2 relu, 3 mul a, 4 add a).  Y rows are cout4 = round_up(cout, 4) long.
 * Restates pt_v21_conv_cpu, runtime/v21/src/pt_v21_host.c:2299-2361. */
void or_conv(const float *X, int64_t ldx, int64_t cin, float *Y, int64_t ldy, int64_t Tout,
             int cout, int K, int stride, int dil, const float *wp, const float *bias,
             int64_t batch, int epi0, int epi1, float a0, float a1);

/* conv_transpose1d through the phase layout including the tail flush.
 * Restates pt_v21_convT_cpu, runtime/v21/src/pt_v21_host.c:2547-2593. */
void or_convT(const float *X, int64_t ldx, int64_t cin, int64_t tin, float *Y, int64_t ldy,
              int cout, int s, int pad, int K, const float *wp, const float *bias, int64_t batch);

/* Pack helpers (tools/export_v21.py:88-121): ONNX conv W[cout][cin][K] and ONNX convT
 * W[cin][cout][K] into the packed layouts above. */
void or_pack_conv(const float *W, int cout, int cin, int K, float *wp);
void or_pack_convT(const float *W, int cin, int cout, int K, int s, float *wp);
int64_t or_packed_conv_elems(int cout, int cin, int K);
int64_t or_packed_convT_elems(int cin, int cout, int K, int s);

/* Decoder weights in the container's packed layouts.  Resblock r (0..5) uses kernel
 * (3,7,11)[r%3] and dilations (1,3,5) in convs1, 1 in convs2; r<3 works on 256 channels after
 * ups.0, r>=3 on 128 channels after ups.1. */
typedef struct {
  const float *pre_w, *pre_b;            /* conv_pre 192->512 k7 p3 */
  const float *ups_w[2], *ups_b[2];      /* ups.0 512->256, ups.1 256->128, k16 s4 p6 */
  const float *rb_w1[6][3], *rb_b1[6][3];
  const float *rb_w2[6][3], *rb_b2[6][3];
  const float *post_w, *post_b;          /* subband_conv_post 128->72 k7 p3 */
  const float *pqmf;                     /* PQMF synthesis filter, ONNX [1][4][63] */
} or_dec_weights;

/* Whole decoder for one request: z [192][T] -> wav [256*T].
 * Graph wiring: ref/v21_graph_trace.txt nodes 3819-4065. */
int or_decode(const or_dec_weights *w, const float *z, int64_t T, float *wav);

/* The same decode, also copying the output of every conv node (with its fused epilogue, residual
 * add, branch sum, /3 and LeakyRelu as the graph applies them) into ck[i] when ck and ck[i] are
 * non-NULL.  The 40 layers and their shapes are those of pt_b200_decoder_checkpoints
 * (include/pt_b200.h): 0 conv_pre+leaky [512][T]; 1 ups.0 [256][4T]; 2+6rb+2j convs1.j+leaky;
 * 3+6rb+2j convs2.j + residual (j = 2: branch, branch sum, leaky(sum/3)); 20..38 the same at 128
 * channels and 16T (38: the reflection-padded [128][16T+1]); 39 conv_post [72][16T+1]. */
int or_decode_ckpt(const or_dec_weights *w, const float *z, int64_t T, float *wav,
                   float *const *ck);

/* The iSTFT + PQMF tail alone: post [72][Tp] (Tp = 16T+1 frames) -> wav [256T] with
 * 256T = 16 * 4 * (Tp - 1). Graph nodes 3957-4065. */
int or_tail(const float *post, int64_t Tp, const float *pqmf, float *wav);

/* Tail constants (graph constants 4009 = periodic Hann(16), 3617 = Hann^2, and the irfft bases
 * built by nodes 3530-3615): exposed for the GPU library's tests. */
void or_tail_constants(float *win16, float *win2_16, float *bc_9x16, float *bs_9x16);

#ifdef __cplusplus
}
#endif
#endif
