/* pt_b200.h -- C ABI of libpt_b200.so, the B200 (sm_100a) implementation of the PrimeTTS v2.1
 * MB-iSTFT decoder hot path.
 *
 * Part 1 is the drop-in boundary: every symbol the reference graph interpreter
 * (runtime/v21/src/pt_v21_host.c) binds for its CUDA build, with the reference's names, argument
 * meaning, return codes and threading rules (runtime/v21/src/pt_v21.h:208-259).  A build of the
 * interpreter with -DPT_V21_CUDA links against this library instead of pt_v21_cuda.cu.
 * Part 2 adds entry points the reference does not have (multi-GPU device selection, fused
 * convT epilogue, the iSTFT+PQMF tail, and the batched device-resident decoder).
 *
 * All pointers are plain host or device pointers; sizes are element counts unless named *_bytes.
 * Return codes: 0 = success, -1 = failure (a message is printed to stderr and kept for
 * pt_b200_last_error()).  There is no CPU fallback: a context that was not initialised for the
 * GPU makes every compute entry point fail with -1.
 */
#ifndef PT_B200_H_
#define PT_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PT_B200_API __attribute__((visibility("default")))
#else
#define PT_B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------------------------------------
 * The interpreter's per-request context and tensor view.  The library reads and writes a handful
 * of these fields (use_cuda, g_stream, g_arena*, conv_pad_in, conv_in_dev, conv_keep*,
 * conv_out_dev, chain_mark, the counters), so the layout must be identical to the interpreter's
 * struct (runtime/v21/src/pt_v21.h:79-162).  tests/test_abi.py checks every offset against the
 * reference header.  When the reference header is already included, its definitions are used.
 * ------------------------------------------------------------------------------------------- */
#ifndef PT_V21_H_
#define PT_B200_RANK 6
typedef struct {
  int dt;
  int ndim;
  int64_t d[PT_B200_RANK];
  int64_t n;
  void *p;
  int dev;
  int dev_res;
  void *dev_p;
  int alive;
  void *base;
  int view;
} pt_tv;

struct pt_ctx {
  int use_cuda;                 /* 1 after pt_v21_cuda_init: conv/convT/matmul run on the GPU */
  void *map;
  size_t maplen;
  char *base;
  uint32_t n_tensor;
  const char **cont_names;
  float **cont_f32;
  int *cont_isz;
  int64_t *cont_n;
  int *cont_ndim;
  char *cont_path;
  int *cont_shared;
  int64_t *cont_dims;
  int n_cont;
  pt_tv *V;
  float *wav;
  int64_t wav_n;
  int ck_n;
  const int *ck_ids;
  char ck_dir[512];
  int dev_mode;
  long n_conv, n_convT, n_matmul, n_alloc_fail;
  double t_conv, t_convT, t_matmul, t_total;
  double g_alloc_ms, g_copy_ms, g_kernel_ms, g_free_ms;
  long g_calls;
  int prof;
  int prof_node_on;
  long host_bytes_live, host_bytes_peak;
  void *pool[64];
  long pool_bytes, pool_cap;
  long host_alloc_count;
  double dev_bytes_weights, dev_bytes_arena, dev_bytes_stray;
  double dev_bytes_res;
  int devres_oom;
  size_t arena_alloc_bytes;
  char *skip;
  int fuse;
  int run_from, run_to;
  int stream_inject_id;
  pt_tv *stream_inject;
  void *stream_seeds;
  int stream_nseeds;
  void *stream_state;
  double *prof_node;
  double t_ekind[96];
  long n_ekind[96];
  void *g_weights;              /* this library: its per-context state (device, arena, events) */
  void *g_arena;                /* device arena base (bump allocator, mark/release) */
  void *g_stream;               /* the context's own non-blocking cudaStream_t */
  size_t g_arena_bytes, g_arena_used;
  int64_t conv_pad_in;          /* >= 0: conv input rows are unpadded, the kernel pads by this */
  const float *conv_in_dev;     /* chained conv input already on the device, or NULL */
  int conv_keep;                /* 1: keep this conv's output on the device for the next conv */
  int conv_keep_res;
  int devadd_used;
  int dev_live;
  float *conv_out_dev;          /* set by pt_v21_conv when the output was kept */
  void *chain_mark;             /* arena mark held while a conv chain is in flight */
  void *devres;
};
typedef struct pt_ctx pt_ctx;
#endif /* PT_V21_H_ */

/* ============================================================================================
 * Part 1 -- the reference's CUDA-layer symbols (runtime/v21/src/pt_v21.h:208-259)
 * ========================================================================================== */

/* Replaces pt_v21_cuda_prewarm (pt_v21.h:213; pt_v21_cuda.cu:719-751): creates the CUDA context
 * of the selected device early.  The Nano clock ramp has no B200 counterpart. */
PT_B200_API int pt_v21_cuda_prewarm(void);

/* Replaces pt_v21_cuda_init (pt_v21.h:209; pt_v21_cuda.cu:753-798): binds the context to device
 * $PT_V21_DEVICE (default 0), creates its non-blocking stream and device arena
 * ($PT_V21_ARENA_MB MiB, default 64) and sets c->use_cuda = 1.  Weights become resident on first
 * use and are shared by every context on the same device. */
PT_B200_API int pt_v21_cuda_init(pt_ctx *c, int verbose);

/* Replaces pt_v21_cuda_shutdown (pt_v21.h:214; pt_v21_cuda.cu:800-813). */
PT_B200_API void pt_v21_cuda_shutdown(pt_ctx *c);

/* Replaces pt_v21_conv (pt_v21.h:253-255; pt_v21_cuda.cu:1756-1957).
 * Y[b][co][t] = bias[co] + sum_k sum_ci W[co][ci][k] X[b][ci][t*stride + k*dil - pad_in], then
 * the fused epilogue codes epi0/epi1 (1 LeakyReLU a, 2 ReLU, 3 x*a, 4 x+a).
 * X: host [batch][cin][ldx]; unpadded rows when c->conv_pad_in >= 0 (padding = conv_pad_in),
 * zero-padded rows otherwise.  When c->conv_in_dev is set, X is ignored and that device buffer
 * (a kept output of the previous conv) is read instead.  Y: host [batch][cout4][n] (padded rows,
 * cout4 = round_up(cout, 4); every element written; ldy is unused, as in the reference).
 * wp: packed weights [cout4/4][K][cin][4]; bias: [cout] or NULL.  wtab/btab >= 0 identify
 * container records: the device copy is made once per device and reused by all contexts.
 * c->conv_keep = 1 leaves the result on the device in c->conv_out_dev (Y untouched).
 * Only stride 1 is supported (every conv of the v2.1 graph has stride 1). */
PT_B200_API int pt_v21_conv(pt_ctx *c, const float *X, int64_t ldx, int64_t cin, float *Y, int64_t ldy,
                int64_t n, int cout, int K, int stride, int pad, int dil, const float *wp,
                const float *bias, int64_t batch, int wtab, int btab, int epi0, int epi1,
                float a0, float a1);

/* Replaces pt_v21_convT (pt_v21.h:257-259; pt_v21_cuda.cu:2351-2491): conv_transpose1d through
 * the packed phase layout [s*cout4/4][ntap][cin][4], including the tail flush.
 * X: host [batch][cin][ldx] (tin columns used); Y: host [batch][cout4][Lout],
 * Lout = (tin-1)*s - 2*pad + K. */
PT_B200_API int pt_v21_convT(pt_ctx *c, const float *X, int64_t ldx, int64_t cin, int64_t tin, float *Y,
                 int64_t ldy, int cout, int s, int pad, int K, const float *wp, const float *bias,
                 int64_t batch, int wtab, int btab);

/* Replaces pt_v21_matmul (pt_v21.h:260-261; pt_v21_cuda.cu:2493-2636): C[m][nn] = A[m][k] B[k][nn]
 * (row-major, leading dimensions lda/ldb/ldc), on the same tensor-core kernel. */
PT_B200_API int pt_v21_matmul(pt_ctx *c, const float *A, int64_t m, int64_t k, int64_t lda, const float *B,
                  int64_t ldb, int64_t nn, float *C, int64_t ldc);

/* Replaces pt_v21_conv_pads_in_kernel (pt_v21.h:224; pt_v21_cuda.cu:457-463): always 1, the
 * tensor-core conv pads with TMA out-of-bounds zero fill. */
PT_B200_API int pt_v21_conv_pads_in_kernel(pt_ctx *c);

/* Replace the device-residency helpers (pt_v21.h:229-247; pt_v21_cuda.cu:246-454): a residual
 * Add (epi=1 fuses a LeakyReLU), a LeakyReLU, and their buffers.  Allocation helpers return NULL
 * on failure so that the interpreter keeps the tensor on its host path. */
PT_B200_API int pt_v21_devadd_run(pt_ctx *c, const float *a, const float *b, float *y, int64_t n, int epi,
                      float alpha);
PT_B200_API int pt_v21_devleaky_run(pt_ctx *c, const float *a, float *y, int64_t n, float alpha);
PT_B200_API float *pt_v21_dev_upload(pt_ctx *c, const void *h, int64_t n);
PT_B200_API void pt_v21_dev_sync_host(pt_ctx *c, void *host, const void *dev, int64_t n);
PT_B200_API void *pt_v21_dev_alloc(pt_ctx *c, size_t bytes);
PT_B200_API void pt_v21_dev_free(pt_ctx *c, void *p);
PT_B200_API void pt_v21_dev_reclaim(pt_ctx *c);

/* Replace the bookkeeping symbols (pt_v21.h:215-221). */
PT_B200_API void pt_v21_cuda_active(int delta);
PT_B200_API double pt_v21_cuda_weights_mib(pt_ctx *c);
PT_B200_API int pt_v21_cuda_keepwarm(int iters);   /* no clock governor to ramp on B200: returns 0 */
PT_B200_API long pt_v21_gpu_cur_freq(void);        /* -1: not readable without NVML (as in the reference) */
PT_B200_API long pt_v21_gpu_max_freq(void);        /* max SM clock of the current device in Hz */

/* ============================================================================================
 * Part 2 -- extensions (no counterpart symbol in the reference)
 * ========================================================================================== */

/* pt_v21_cuda_init on an explicit device (request-parallel multi-GPU: one context per request
 * thread, weights resident once per device). */
PT_B200_API int pt_v21_cuda_init_dev(pt_ctx *c, int device, int verbose);

/* pt_v21_convT with one fused epilogue op (codes as pt_v21_conv), e.g. the LeakyReLU that
 * follows each upsampler in the graph (node /dec/resblocks.0/LeakyRelu). */
PT_B200_API int pt_v21_convT_epi(pt_ctx *c, const float *X, int64_t ldx, int64_t cin, int64_t tin, float *Y,
                     int64_t ldy, int cout, int s, int pad, int K, const float *wp,
                     const float *bias, int64_t batch, int wtab, int btab, int epi0, float a0);

/* The iSTFT + PQMF synthesis tail (graph nodes /dec/Reshape_6 ... /dec/Conv) for one request:
 * post [72][Tp] (subband_conv_post output, host) -> wav [256*(Tp-1)/16] (host).
 * pqmf: the [1][4][63] synthesis filter (ONNX layout, host). */
PT_B200_API int pt_v21_istft_pqmf(pt_ctx *c, const float *post, int64_t Tp, const float *pqmf, float *wav);

/* Decoder weights in the container's packed layouts (tools/export_v21.py:88-121): conv
 * [cout4/4][K][cin][4], convT [4*cout4/4][4][cin][4], biases [cout]; pqmf [1][4][63].
 * Resblock r (0..5): kernel (3,7,11)[r%3], convs1 dilations (1,3,5), convs2 dilation 1;
 * r < 3 follow ups.0 (256 channels), r >= 3 follow ups.1 (128 channels). */
typedef struct {
  const float *pre_w, *pre_b;
  const float *ups_w[2], *ups_b[2];
  const float *rb_w1[6][3], *rb_b1[6][3];
  const float *rb_w2[6][3], *rb_b2[6][3];
  const float *post_w, *post_b;
  const float *pqmf;
} pt_b200_dec_weights;

typedef struct pt_b200_decoder pt_b200_decoder;

/* Uploads and re-lays-out the decoder weights on `device` (once; the handle is shareable by
 * threads that serialise their calls).  NULL on failure. */
PT_B200_API pt_b200_decoder *pt_b200_decoder_create(int device, const pt_b200_dec_weights *w);
PT_B200_API void pt_b200_decoder_destroy(pt_b200_decoder *d);

/* Decode a batch of independent requests in one device-resident pass (all requests share each
 * layer's launches).  Request i has T[i] latent frames; z_host is the concatenation of the
 * requests' [192][T[i]] latents, wav_host receives the concatenation of their [256*T[i]]
 * waveforms.  Host buffers should be pinned for full copy speed.  stream: a cudaStream_t or NULL
 * for the decoder's own stream.  Synchronous: returns after wav_host is written. */
PT_B200_API int pt_b200_decode_batch(pt_b200_decoder *d, void *stream, int nreq, const int64_t *T,
                         const float *z_host, float *wav_host);

/* Same with device buffers (z_dev / wav_dev on the decoder's device, same concatenated layouts).
 * Asynchronous on `stream`; the returned status covers argument and launch errors only --
 * pt_b200_decoder_sync() waits and reports device-side errors. */
PT_B200_API int pt_b200_decode_batch_device(pt_b200_decoder *d, void *stream, int nreq, const int64_t *T,
                                const float *z_dev, float *wav_dev);
PT_B200_API int pt_b200_decoder_sync(pt_b200_decoder *d, void *stream);

/* Pipelined host-buffer decodes (a server's steady state): each call queues the upload of z_host
 * into one of two device staging slots, the decode, and the download of the waveform into
 * wav_host, and returns at once.  Uploads and downloads run on their own streams, so batch k+1's
 * upload and batch k's download overlap batch k's decode (host buffers must be pinned).  A call
 * reuses the slot of the call before the previous one only after that call's decode and download
 * are done.  One thread at a time; the host buffers of a call must stay valid until
 * pt_b200_decode_async_wait() returns (it waits for every queued call and reports device errors).
 * pt_b200_decode_async_streams() hands out the upload, decode and download streams (created on
 * first use) for callers that order their own work around the pipeline. */
PT_B200_API int pt_b200_decode_batch_async(pt_b200_decoder *d, int nreq, const int64_t *T,
                                           const float *z_host, float *wav_host);
PT_B200_API int pt_b200_decode_async_wait(pt_b200_decoder *d);
PT_B200_API int pt_b200_decode_async_streams(pt_b200_decoder *d, void **upload, void **decode,
                                             void **download);

/* Live per-launch timing of the decoder, for the benchmark's roofline: with profiling enabled
 * every decode records a CUDA event before each of its launches (and one after the last) on the
 * decode stream.  After the decode has been synchronised, pt_b200_decoder_launch_times fills, per
 * launch of that decode: its duration in ms, its algorithmic FLOPs and bytes, and its kind
 * (low byte: 0 latent staging, 1 conv, 2 upsampler convT, 3 conv_post, 4 iSTFT+PQMF tail; bits
 * 8..: the N tile of the tensor-core conv instance, 0 for other kernels); it returns the number
 * of launches. */
PT_B200_API int pt_b200_decoder_profile(pt_b200_decoder *d, int enable);
PT_B200_API int pt_b200_decoder_launch_times(pt_b200_decoder *d, int max, double *ms,
                                             double *flops, double *bytes, int *kind);

/* Per-layer checkpoints of one request, for parity against a CPU decode node by node (the
 * batched decoder's counterpart of the reference's pt_v21_checkpoints, runtime/v21/src/
 * pt_v21.h:204-206, which dumps graph-node outputs for the per-node gate of
 * tests/v21_reference.py:430-447).  Decodes z_host [192][T] (host) on the decoder's stream,
 * eagerly, and after each of the 40 conv launches copies that launch's output, without gap rows,
 * channel-major, into ckpt[i] (host; NULL entries are skipped); wav_host [256*T] receives the
 * waveform.  Layer i and the tensor it holds (L1 = 4T, L2 = 16T rows):
 *   0  conv_pre + LeakyRelu                 [512][T]     (TF32-rounded, as the next conv reads it)
 *   1  ups.0                                [256][L1]    (fp32)
 *   2 + 6*rb + 2*j      convs1.j of resblock rb + LeakyRelu   [256][L1] (TF32-rounded)
 *   3 + 6*rb + 2*j      convs2.j + residual: j < 2 the running x; j = 2: rb 0 the branch, rb 1
 *                       the branch sum, rb 2 LeakyRelu((sum)/3)  [256][L1] (fp32; the last TF32)
 *   20 ups.1                                [128][L2]
 *   21 .. 38 as 2 .. 19 for resblocks 3..5 at 128 channels; 38 is LeakyRelu_0.01((sum)/3) with
 *                       the reflection-pad row in front: [128][L2 + 1]
 *   39 subband_conv_post                    [72][L2 + 1]
 * A debugging entry point: it allocates its own device buffer and synchronises. */
#define PT_B200_NCKPT 40
PT_B200_API int pt_b200_decoder_checkpoints(pt_b200_decoder *d, const float *z_host, int64_t T,
                                            float *const *ckpt, float *wav_host);

/* One request, the reference's driver shape (an extension the survey lists as pt_v21_decode):
 * z [192][T] host -> wav [256*T] host. */
PT_B200_API int pt_v21_decode(pt_ctx *c, const pt_b200_decoder *d, const float *z, int64_t T, float *wav);

/* ---- Streaming (extension) ------------------------------------------------------------------
 * The reference streams the decoder on sliding windows of one utterance's frames
 * (pt_v21_stream_open / _chunk / _close, runtime/v21/src/pt_v21_host.c:2749-2912: each chunk
 * re-runs the decoder nodes on frames [a, a+win)) and its drivers stitch the window interiors
 * (main_v21.c:331-368, main_v21_serve.c:210-264).  Here a window is one request of the batched
 * decoder, and the tail kernel writes each window's interior straight into the stitched output.
 *
 * One window: decode latent frames z_dev[z_off + c*z_ld + t] (c < 192, t < frames: a column
 * slice of a [192][z_ld] latent) as one request, and write its output samples
 * [keep_lo, keep_hi) (0 <= keep_lo < keep_hi <= 256*frames) to wav_dev[dst + (j - keep_lo)]. */
typedef struct {
  int64_t frames, z_off, z_ld, keep_lo, keep_hi, dst;
} pt_b200_window;

/* Decode n windows in one device-resident pass (asynchronous on `stream`, like
 * pt_b200_decode_batch_device; pt_b200_decoder_sync reports device errors). */
PT_B200_API int pt_b200_decode_windows(pt_b200_decoder *d, void *stream, int n,
                                       const pt_b200_window *w, const float *z_dev, float *wav_dev);

/* The window plan for nstreams utterances of T[i] frames (latents concatenated as [192][T[i]]
 * blocks, stitched waveforms as [256*T[i]] blocks), step = max(1, win - 2*ctx):
 *  exact = 0  the reference's overlap-save (main_v21.c:342-364): windows [a, a+win) every `step`
 *             frames; the first emits from its start, the last to its end, the others frames
 *             [a+ctx, a+win-ctx).  Samples near a window edge see zero padding instead of the
 *             neighbouring frames, so the stitched waveform differs from a whole-utterance decode.
 *  exact = 1  the same emission schedule (frames [e, e+step) per window), each window decoded
 *             over [e - max(ctx,25), e + step + max(ctx,24)) clipped to the utterance: the
 *             decoder's receptive radius is 25 frames back and 24 ahead, so every emitted sample
 *             equals the whole-utterance decode.
 * Writes min(cap, count) windows to `out` and returns the window count (cap 0 sizes), -1 on
 * bad arguments. */
PT_B200_API int64_t pt_b200_stream_plan(int nstreams, const int64_t *T, int win, int ctx,
                                        int exact, pt_b200_window *out, int64_t cap);

/* Plan, decode and stitch every stream: windows in plan order, max_frames latent frames per
 * decode pass (<= 0: 65536).  Device buffers; asynchronous on `stream` except that each new
 * batch waits for the previous one (they share the decoder's activation buffers). */
PT_B200_API int pt_b200_stream_decode(pt_b200_decoder *d, void *stream, int nstreams,
                                      const int64_t *T, const float *z_dev, int win, int ctx,
                                      int exact, int64_t max_frames, float *wav_dev);

/* ---- Streaming with carried state (extension) --------------------------------------------
 * The same streams decoded chunk by chunk without recomputing any frame: pass k feeds latent
 * frames [k*chunk, (k+1)*chunk) of every stream still running, and every layer computes only
 * the rows whose inputs are now complete, reading the rows it needs from earlier passes out of
 * the session's activations (the carried state).  Each pass emits the output samples whose
 * receptive field is complete (24 latent frames of look-ahead), bit-identical to the
 * whole-utterance decode; the pass after the one that brings a stream's last frames (it brings
 * none of its own) flushes that stream, so a session runs ceil(max T / chunk) + 1 passes.  This
 * replaces the reference's re-run of the decoder on overlapping windows (pt_v21_stream_chunk,
 * runtime/v21/src/pt_v21_host.c:2749-2912) where the windows were meant to cover the receptive
 * field.
 *
 * A session's activations are bounded per stream, not per frame: each stream keeps, per
 * resolution, a fixed window of rows (the rows a pass computes and the receptive context later
 * passes still read; the flush, in a pass of its own, fits the same window), and before a pass
 * the rows still needed move to the front of the window; only the per-pass tables (a few KB per
 * stream and pass) grow with the stream length.  pt_b200_carry_device_bytes tells the size
 * before opening.  Latents are concatenated as for pt_b200_decode_batch_device ([192][T[i]] per
 * stream); pass k reads only its own frames, so z_dev may be filled as frames arrive.  Output
 * samples go to wav_dev at the stream's offset in the concatenated waveform (256*T[i] samples
 * per stream). */
typedef struct pt_b200_carry pt_b200_carry;
/* Plan the passes and allocate the session on the decoder's device; NULL on error. */
PT_B200_API pt_b200_carry *pt_b200_carry_open(pt_b200_decoder *d, int nstreams, const int64_t *T,
                                             int chunk);
PT_B200_API int pt_b200_carry_passes(const pt_b200_carry *c);
/* Device bytes the session holds (activation windows, pass tables). */
PT_B200_API int64_t pt_b200_carry_bytes(const pt_b200_carry *c);
/* Device bytes a session of these streams would hold (no GPU needed); -1 on bad arguments. */
PT_B200_API int64_t pt_b200_carry_device_bytes(int nstreams, const int64_t *T, int chunk);
/* Pass `pass` (0, 1, ... in order, each once) on `stream` (NULL: the decoder's stream),
 * asynchronous; the status covers argument and launch errors (pt_b200_decoder_sync reports
 * device errors). */
PT_B200_API int pt_b200_carry_run(pt_b200_carry *c, void *stream, int pass, const float *z_dev,
                                  float *wav_dev);
/* Rewind to pass 0 for a new run of the same streams (new latents).  Nothing is cleared: every
 * row a pass reads was written earlier in the same run, and gap rows only ever hold zeros. */
PT_B200_API int pt_b200_carry_reset(pt_b200_carry *c);
PT_B200_API void pt_b200_carry_close(pt_b200_carry *c);
/* Open, run every pass, close. */
PT_B200_API int pt_b200_stream_decode_carry(pt_b200_decoder *d, void *stream, int nstreams,
                                            const int64_t *T, const float *z_dev, int chunk,
                                            float *wav_dev);
/* The pass plan alone (no GPU): returns the pass count (-1 on bad arguments or a plan that
 * fails its own checks) and, when cap >= passes * nstreams, the samples [lo, hi) of each
 * stream that each pass emits (index pass * nstreams + stream). */
PT_B200_API int64_t pt_b200_carry_plan(int nstreams, const int64_t *T, int chunk, int64_t *lo,
                                       int64_t *hi, int64_t cap);

/* ---- Weight container (extension) ------------------------------------------------------
 * The reference ships its weights in one .ptk container (tools/export_v21.py:1-40: header
 * <IIIiq> "PTK1", 136-byte records <64si4x6qqq>, 64-byte aligned payloads, fp16 for names ending
 * in "#h"), read by its runtime at start-up.  These read the decoder's records
 * (dec.conv_pre, dec.ups.{0,1}, dec.resblocks.{0..5}.convs{1,2}.{0..2}, dec.subband_conv_post,
 * and the PQMF synthesis filter dec.Conv) into pt_b200_dec_weights, fp16 payloads widened to
 * fp32 (exact; fp16 values are exact in TF32 too).  No GPU is needed to read a container.
 * pt_b200_ptk_open returns NULL (message in pt_b200_last_error) on a missing file, bad magic,
 * missing tensor or wrong size.  The weight pointers stay valid until pt_b200_ptk_close. */
typedef struct pt_b200_ptk pt_b200_ptk;
PT_B200_API pt_b200_ptk *pt_b200_ptk_open(const char *path);
PT_B200_API int pt_b200_ptk_decoder_weights(const pt_b200_ptk *k, pt_b200_dec_weights *w);
PT_B200_API void pt_b200_ptk_close(pt_b200_ptk *k);
/* Open, create the decoder on `device`, close. */
PT_B200_API pt_b200_decoder *pt_b200_decoder_create_from_ptk(int device, const char *path);

/* Conv1d with no device allocation (no counterpart in the reference).  For callers that cannot
 * call cudaMalloc/cudaFree: hosts that own every device allocation (pooled or framework
 * allocators), real-time threads that must not take the allocator's locks, processes whose
 * device footprint is fixed after start-up.  Same arithmetic as pt_v21_conv (stride 1, batch 1),
 * but every pointer is a DEVICE pointer on `device`: x [cin][ldx] (T unpadded columns, the kernel
 * pads by `pad`), y [cout4][Tout] with Tout = T + 2*pad - (K-1)*dil, wp packed
 * [cout4/4][K][cin][4], bias [cout] or NULL.  Scratch (staged input, re-laid-out weights) comes
 * from one fixed 16 MiB array inside the library on each device: calls needing more (T *
 * round_up(cin,32) + round_up(cout,16) * K * round_up(cin,32) floats, plus padding) are rejected
 * with -1 and a message, before any device work.  The first call on a device looks up that
 * array's device address, so make it before any stream capture.  All calls on a device share the
 * array: calls that overlap on the GPU (other streams, other threads) race and must be serialised
 * by the caller.  The call is synchronous: it reads a device error word back into host memory
 * and waits (with the library's bounded wait, PT_B200_WAIT_S) for its work on `stream`
 * (NULL = the default stream) to finish before it returns. */
PT_B200_API int pt_b200_conv_noalloc(int device, void *stream, const float *x, int64_t ldx,
                                     int64_t cin, int64_t T, float *y, int cout, int K, int pad,
                                     int dil, const float *wp, const float *bias, int epi0,
                                     float a0);

/* The tensor core's kind::tf32 rate on `device`, measured live (the conv stack's roofline): one
 * CTA per SM issues `iters` x 4 MMAs of M128 x N256 x K8 from shared-memory operands into TMEM.
 * Returns FLOP per SM clock (averaged over the SMs), the aggregate TFLOP/s over the run, and the
 * SM clock the run held (MHz).  Synchronous; about 5 ms at iters = 20000. */
PT_B200_API int pt_b200_mma_rate(int device, int iters, double *flop_per_clk_sm, double *tflops,
                                 double *sm_mhz);

/* Diagnostics: the last error message of the calling thread, and the number of this library's
 * kernels launched by the calling thread since the last reset. */
PT_B200_API const char *pt_b200_last_error(void);
PT_B200_API long pt_b200_kernel_launches(int reset);

#ifdef __cplusplus
}
#endif
#endif /* PT_B200_H_ */
