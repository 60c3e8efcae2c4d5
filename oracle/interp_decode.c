/* interp_decode.c -- TEST INFRASTRUCTURE: the reference's own graph interpreter decoding one latent.
 *
 * Built only by oracle/Makefile, twice, from the reference's sources where they lie (this file
 * #includes runtime/v21/src/pt_v21_host.c, so the interpreter's file-static streaming helpers are
 * reachable; nothing is copied):
 *   _ref/interp_decode_cpu  the interpreter's host build: every conv / convT node runs
 *                           pt_v21_conv_cpu / pt_v21_convT_cpu (the reference CPU path);
 *   _ref/interp_decode_gpu  its CUDA build (-DPT_V21_CUDA) linked against libpt_b200.so: the same
 *                           interpreter code calls pt_v21_conv / pt_v21_convT / pt_v21_cuda_init of
 *                           this repository's library for every conv node (the drop-in boundary).
 *
 * It opens a container with pt_v21_open (runtime/v21/src/pt_v21_host.c:1086), then decodes the
 * way pt_v21_stream_chunk does (:2859-2900): the decoder's node range [conv_pre node, end) runs on
 * an injected latent (the tensor conv_pre reads, /Mul_7_output_0, [1][192][T]).  The tensors that
 * range reads from outside itself besides the latent -- the irfft bases and the zero-stuff kernel,
 * built from constants by nodes before conv_pre -- are made by running exactly the nodes they
 * depend on (every one of them reads only constants), one node per call through the interpreter's
 * own run loop (run_from / run_to / stream_seeds, :2921-2976), each node's outputs carried to the
 * next call as seeds.  So every value comes from the interpreter's own node code.
 *
 *   interp_decode_{cpu,gpu} <container.ptk> <z.f32> <T> <wav.f32> [reps]
 * reads z ([192][T] float32), writes the waveform (float32) and prints one JSON line with the
 * sample count and the wall time per decode over `reps` decodes (the first one untimed).
 */
#include <time.h>

#include "pt_v21_host.c"

static double wall_s(void) {
  struct timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (double) ts.tv_sec + 1e-9 * (double) ts.tv_nsec;
}

/* the nodes whose outputs the decoder range reads from before it (other than the latent), and
 * every node they depend on */
static int *closure_nodes(int *count) {
  static int prod[PT_N_TENSOR];
  static char need[PT_N_NODE];
  int *stack = (int *) malloc(sizeof(int) * PT_N_NODE), sp = 0;
  for (int i = 0; i < PT_N_TENSOR; i++) prod[i] = -1;
  for (int i = 0; i < PT_N_NODE; i++)
    for (int j = 0; j < PT_V21_MAX_OUT; j++)
      if (pt_ndefs[i].out[j] >= 0) prod[pt_ndefs[i].out[j]] = i;
  for (int idx = g_stream_tail; idx < PT_N_NODE; idx++)
    for (int k = 0; k < PT_V21_MAX_IN; k++) {
      const int t = pt_ndefs[idx].in[k];
      if (t < 0 || t == g_stream_src) continue;
      const int p = prod[t];
      if (p >= 0 && p < g_stream_tail && !need[p]) {
        need[p] = 1;
        stack[sp++] = p;
      }
    }
  while (sp) {
    const pt_node_def *nd = &pt_ndefs[stack[--sp]];
    for (int k = 0; k < PT_V21_MAX_IN; k++) {
      const int t = nd->in[k];
      if (t < 0) continue;
      const int p = prod[t];
      if (p >= 0 && !need[p]) {
        need[p] = 1;
        stack[sp++] = p;
      }
    }
  }
  int n = 0;
  for (int i = 0; i < PT_N_NODE; i++)
    if (need[i]) stack[n++] = i;
  *count = n;
  return stack;
}

int main(int argc, char **argv) {
  if (argc < 5) {
    fprintf(stderr, "usage: %s container.ptk z.f32 T wav.f32 [reps]\n", argv[0]);
    return 1;
  }
  const int64_t T = atoll(argv[3]);
  const int reps = argc > 5 ? atoi(argv[5]) : 1;
  float *z = (float *) malloc(sizeof(float) * 192 * (size_t) T);
  FILE *fz = fopen(argv[2], "rb");
  if (!fz || fread(z, sizeof(float), 192 * (size_t) T, fz) != 192 * (size_t) T) {
    fprintf(stderr, "interp_decode: cannot read %lld x 192 floats from %s\n", (long long) T, argv[2]);
    return 1;
  }
  fclose(fz);
  pt_ctx *c = pt_v21_open(argv[1]);
  if (!c) return 2;
#ifdef PT_V21_CUDA
  if (pt_v21_cuda_init(c, 0)) {
    fprintf(stderr, "interp_decode: pt_v21_cuda_init failed\n");
    return 3;
  }
#endif
  stream_locate();
  if (g_stream_tail >= PT_N_NODE || g_stream_src < 0) {
    fprintf(stderr, "interp_decode: decoder range not found\n");
    return 4;
  }

  /* constants-only prefix: one node per run, outputs carried as seeds */
  int nclos = 0;
  int *clos = closure_nodes(&nclos);
  pt_stream_seed *seeds = (pt_stream_seed *) calloc((size_t) nclos * PT_V21_MAX_OUT + 1, sizeof(*seeds));
  int nseeds = 0;
  pt_tv feeds[16];
  static float zero_feed[8];
  memset(feeds, 0, sizeof(feeds));
  for (int i = 0; i < 16; i++) {
    feeds[i].dt = DT_F32;
    feeds[i].ndim = 1;
    feeds[i].d[0] = 1;
    feeds[i].n = 1;
    feeds[i].p = zero_feed;   /* graph inputs: aliased only when a run starts at node 0, never read */
  }
  for (int q = 0; q < nclos; q++) {
    const int idx = clos[q];
    c->stream_seeds = seeds;
    c->stream_nseeds = nseeds;
    c->run_from = idx;
    c->run_to = idx + 1;
    float *w = NULL;
    int64_t wn = 0;
    if (pt_v21_run(c, feeds, &w, &wn)) {
      fprintf(stderr, "interp_decode: prefix node %d failed\n", idx);
      return 5;
    }
    for (int j = 0; j < PT_V21_MAX_OUT; j++) {
      const int t = pt_ndefs[idx].out[j];
      if (t < 0 || !c->V[t].p || c->V[t].n <= 0) continue;
      pt_stream_seed *sd = &seeds[nseeds++];
      sd->id = t;
      sd->dt = c->V[t].dt;
      sd->ndim = c->V[t].ndim;
      sd->n = c->V[t].n;
      for (int r = 0; r < PT_V21_MAX_RANK; r++) sd->d[r] = c->V[t].d[r];
      sd->bytes = sd->n * dt_sz(c->V[t].dt);
      sd->buf = (float *) malloc((size_t) sd->bytes);
      memcpy(sd->buf, c->V[t].p, (size_t) sd->bytes);
    }
  }
  c->run_from = c->run_to = 0;

  /* the decoder range on the injected latent, as pt_v21_stream_chunk runs a window */
  pt_tv inj;
  memset(&inj, 0, sizeof inj);
  inj.dt = DT_F32;
  inj.ndim = 3;
  inj.d[0] = 1;
  inj.d[1] = 192;
  inj.d[2] = T;
  for (int r = 3; r < PT_V21_MAX_RANK; r++) inj.d[r] = 1;
  inj.n = 192 * T;
  inj.p = z;
  float *wav = NULL;
  int64_t wn = 0;
  double total = 0.0;
  for (int r = 0; r < (reps > 1 ? reps + 1 : 1); r++) {
    c->stream_inject = &inj;
    c->stream_inject_id = g_stream_src;
    c->stream_seeds = seeds;
    c->stream_nseeds = nseeds;
    c->run_from = g_stream_tail;
    c->run_to = PT_N_NODE;
    const double t0 = wall_s();
    const int rc = pt_v21_run(c, NULL, &wav, &wn);
    const double dt = wall_s() - t0;
    c->run_from = c->run_to = 0;
    c->stream_inject = NULL;
    c->stream_inject_id = -1;
    c->stream_seeds = NULL;
    c->stream_nseeds = 0;
    if (rc || !wav || wn <= 0) {
      fprintf(stderr, "interp_decode: decoder run failed (rc %d)\n", rc);
      return 6;
    }
    if (r > 0 || reps <= 1) total += dt;
  }
  const int timed = reps > 1 ? reps : 1;
  FILE *fw = fopen(argv[4], "wb");
  if (!fw || fwrite(wav, sizeof(float), (size_t) wn, fw) != (size_t) wn) {
    fprintf(stderr, "interp_decode: cannot write %s\n", argv[4]);
    return 7;
  }
  fclose(fw);
  printf("{\"frames\": %lld, \"samples\": %lld, \"s_per_decode\": %.6f, \"audio_s_per_s\": %.3f, "
         "\"prefix_nodes\": %d, \"seeds\": %d, \"decodes_timed\": %d}\n",
         (long long) T, (long long) wn, total / timed, (double) wn / 16000.0 / (total / timed),
         nclos, nseeds, timed);
#ifdef PT_V21_CUDA
  pt_v21_cuda_shutdown(c);
#endif
  return 0;
}
