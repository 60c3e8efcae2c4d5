// common.cuh -- host-side plumbing shared by the library's translation units.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>

#include "conv_tc.cuh"

namespace ptb {

// ---- errors: printed to stderr (as the reference's PTCHK does) and kept per thread
void set_error(const char *fmt, ...);
const char *last_error();

#define PTB_CUDA(x)                                                                    \
  do {                                                                                 \
    cudaError_t e_ = (x);                                                              \
    if (e_ != cudaSuccess) {                                                           \
      ::ptb::set_error("pt_b200 cuda: %s at %s:%d (%s)", cudaGetErrorString(e_), __FILE__, \
                       __LINE__, #x);                                                  \
      return -1;                                                                       \
    }                                                                                  \
  } while (0)

#define PTB_REQUIRE(cond, ...)    \
  do {                            \
    if (!(cond)) {                \
      ::ptb::set_error(__VA_ARGS__); \
      return -1;                  \
    }                             \
  } while (0)

// counts this library's kernel launches on the calling thread (reported by
// pt_b200_kernel_launches and by bench.py as gpu_launches)
void count_launch(long n = 1);
long launches(int reset);

inline int64_t round_up(int64_t a, int64_t b) { return (a + b - 1) / b * b; }

// Wait for a stream by polling it with a deadline (PT_B200_WAIT_S seconds, default 120): a stream
// that does not finish in time is reported as an error instead of blocking the caller forever.
int wait_stream(cudaStream_t s);

// ---- TMA tensor maps (cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library does not link libcuda directly)
int make_map_act(CUtensorMap *m, const float *base, int cin32, int64_t rows, int batch,
                 int box_rows);
int make_map_w(CUtensorMap *m, const float *base, int64_t krow, int64_t nrows, int box_n);

// ---- the tensor-core conv: picks the N tile instance and launches
struct ConvLaunch {
  const float *act;   // channels-last [batch][rows][cin32], tf32 values
  int64_t act_rows;
  int batch;
  const float *w;     // [n_pad][ntap][cin32], tf32 values
  int bn;             // N tile (one of the compiled instances)
  ConvGeom g;
  EpiParams e;
};
int pick_bn(int ncols, int *bn, int *n_pad);
int launch_conv(const ConvLaunch &L, uint32_t *gerr, cudaStream_t st);

// ---- staging / relayout kernels (stage.cu)
// channel-major [batch][C][ld] (first L columns) -> channels-last [batch][L][C32], tf32
int stage_act(const float *src, int64_t ld, int C, int64_t L, int batch, float *dst, int C32,
              cudaStream_t st);
// row-major [M][ld] (first K columns) -> [M][K32], tf32 (matmul A)
int stage_rows(const float *src, int64_t ld, int64_t M, int K, float *dst, int K32, cudaStream_t st);
// packed conv/convT weights [rows4/4][ntap][cin][4] -> [n_pad][ntap][cin32], tf32
int stage_packed_w(const float *wp, int rows4, int ntap, int cin, float *dst, int n_pad, int cin32,
                   cudaStream_t st);
// matmul B [k][ldb] (first nn columns) -> [n_pad][k32], tf32
int stage_matmul_b(const float *b, int64_t ldb, int k, int nn, float *dst, int n_pad, int k32,
                   cudaStream_t st);
int launch_devadd(const float *a, const float *b, float *y, int64_t n, int epi, float alpha,
                  cudaStream_t st);

}  // namespace ptb
