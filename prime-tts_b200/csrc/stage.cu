// stage.cu -- layout kernels feeding the tensor-core conv, and the device residual ops.
//
// The tensor-core conv consumes channels-last activations and [n][tap][cin32] weights whose
// values are already rounded to tf32 (round-to-nearest); these kernels produce them from the
// reference's layouts (channel-major activations, packed [rows/4][tap][cin][4] weights).
#include "common.cuh"

namespace ptb {

// 32x32 tiles through shared memory: reads coalesced along time, writes along channels.
__global__ void stage_act_kernel(const float *__restrict__ src, int64_t ld, int C, int64_t L,
                                 float *__restrict__ dst, int C32) {
  __shared__ float tile[32][33];
  const int64_t t0 = (int64_t)blockIdx.x * 32;
  const int c0 = blockIdx.y * 32;
  const int b = blockIdx.z;
  const float *s = src + (int64_t)b * C * ld;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i;
    const int64_t t = t0 + threadIdx.x;
    tile[i][threadIdx.x] = (c < C && t < L) ? s[(int64_t)c * ld + t] : 0.0f;
  }
  __syncthreads();
  float *d = dst + (int64_t)b * L * C32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t t = t0 + i;
    if (t < L) d[t * C32 + c0 + threadIdx.x] = tf32_rna(tile[threadIdx.x][i]);
  }
}

int stage_act(const float *src, int64_t ld, int C, int64_t L, int batch, float *dst, int C32,
              cudaStream_t st) {
  dim3 grid((unsigned)((L + 31) / 32), (unsigned)(C32 / 32), (unsigned)batch);
  stage_act_kernel<<<grid, dim3(32, 8), 0, st>>>(src, ld, C, L, dst, C32);
  PTB_CUDA(cudaGetLastError());
  count_launch();
  return 0;
}

__global__ void stage_rows_kernel(const float *__restrict__ src, int64_t ld, int64_t M, int K,
                                  float *__restrict__ dst, int K32) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= M * K32) return;
  const int64_t m = i / K32;
  const int k = (int)(i - m * K32);
  dst[i] = k < K ? tf32_rna(src[m * ld + k]) : 0.0f;
}

int stage_rows(const float *src, int64_t ld, int64_t M, int K, float *dst, int K32,
               cudaStream_t st) {
  const int64_t n = M * K32;
  stage_rows_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(src, ld, M, K, dst, K32);
  PTB_CUDA(cudaGetLastError());
  count_launch();
  return 0;
}

__global__ void stage_packed_w_kernel(const float *__restrict__ wp, int rows4, int ntap, int cin,
                                      float *__restrict__ dst, int n_pad, int cin32) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)n_pad * ntap * cin32;
  if (i >= total) return;
  const int ci = (int)(i % cin32);
  const int64_t r = i / cin32;
  const int k = (int)(r % ntap);
  const int n = (int)(r / ntap);
  float v = 0.0f;
  if (n < rows4 && ci < cin) v = wp[(((int64_t)(n >> 2) * ntap + k) * cin + ci) * 4 + (n & 3)];
  dst[i] = tf32_rna(v);
}

int stage_packed_w(const float *wp, int rows4, int ntap, int cin, float *dst, int n_pad, int cin32,
                   cudaStream_t st) {
  const int64_t n = (int64_t)n_pad * ntap * cin32;
  stage_packed_w_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(wp, rows4, ntap, cin, dst,
                                                                     n_pad, cin32);
  PTB_CUDA(cudaGetLastError());
  count_launch();
  return 0;
}

__global__ void stage_matmul_b_kernel(const float *__restrict__ b, int64_t ldb, int k, int nn,
                                      float *__restrict__ dst, int n_pad, int k32) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)n_pad * k32) return;
  const int n = (int)(i / k32);
  const int kk = (int)(i - (int64_t)n * k32);
  dst[i] = (n < nn && kk < k) ? tf32_rna(b[(int64_t)kk * ldb + n]) : 0.0f;
}

int stage_matmul_b(const float *b, int64_t ldb, int k, int nn, float *dst, int n_pad, int k32,
                   cudaStream_t st) {
  const int64_t n = (int64_t)n_pad * k32;
  stage_matmul_b_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(b, ldb, k, nn, dst, n_pad, k32);
  PTB_CUDA(cudaGetLastError());
  count_launch();
  return 0;
}

// y = a + b, then LeakyReLU(alpha) when epi == 1 (the interpreter's fp32 Add / LeakyRelu);
// b == nullptr gives the LeakyReLU alone.
__global__ void devadd_kernel(const float *__restrict__ a, const float *__restrict__ b,
                              float *__restrict__ y, int64_t n, int epi, float alpha) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float v = b ? a[i] + b[i] : a[i];
    if (epi == 1) v = v >= 0.0f ? v : alpha * v;
    y[i] = v;
  }
}

int launch_devadd(const float *a, const float *b, float *y, int64_t n, int epi, float alpha,
                  cudaStream_t st) {
  if (n <= 0) return 0;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  devadd_kernel<<<(unsigned)blocks, 256, 0, st>>>(a, b, y, n, epi, alpha);
  PTB_CUDA(cudaGetLastError());
  count_launch();
  return 0;
}

}  // namespace ptb
