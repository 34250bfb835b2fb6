// Exact-fp32 kernels behind the reference's fp32 contracts:
//   * SIMT fp32 GEMM for the public fp32 matmul (reference: cublasSgemm in
//     CudaTensorF32::matmul, cuda/kernels.cu:488-493);
//   * single-head fp32 attention (reference cuda_attention_f32,
//     cuda/kernels.cu:147-188 — there O(T^2 F^2); here each score is computed
//     once per (query, key) in shared memory);
//   (conv2d forward / data-gradient / weight-gradient: conv_igemm.cu.)
// These serve the small fp32 API surface; the bf16 training path uses the
// tcgen05 GEMM and the flash-attention kernels.
#include <stdexcept>

#include "common.cuh"
#include "gemm.h"
#include "kernels.h"

namespace uhfs {

namespace {

constexpr int TS = 64;   // C tile
constexpr int TK = 16;

__global__ void __launch_bounds__(256) sgemm_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                                    float* __restrict__ C, int M, int N, int K, bool b_trans) {
  __shared__ float As[TK][TS + 1];
  __shared__ float Bs[TK][TS + 1];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int m0 = blockIdx.y * TS, n0 = blockIdx.x * TS;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += TK) {
    for (int i = threadIdx.x; i < TS * TK; i += 256) {
      int r = i / TK, c = i % TK;  // A tile: rows m, cols k
      int gm = m0 + r, gk = k0 + c;
      As[c][r] = (gm < M && gk < K) ? A[(long long)gm * K + gk] : 0.f;
      int gn = n0 + r;
      float bv = 0.f;
      if (gn < N && gk < K) bv = b_trans ? B[(long long)gn * K + gk] : B[(long long)gk * N + gn];
      Bs[c][r] = bv;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int gm = m0 + ty * 4 + i, gn = n0 + tx * 4 + j;
      if (gm < M && gn < N) C[(long long)gm * N + gn] = acc[i][j];
    }
}

// One CTA per query row; scores for the row live in shared memory.
__global__ void attention_f32_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                     const float* __restrict__ v, float* __restrict__ out, int T, int F, float scale,
                                     bool causal) {
  extern __shared__ float sc[];  // [T]
  __shared__ float red[32];
  __shared__ float stat;
  const int row = blockIdx.x;
  const int last = causal ? row : T - 1;
  for (int j = threadIdx.x; j < T; j += blockDim.x) {
    float d = -INFINITY;
    if (j <= last) {
      d = 0.f;
      for (int f = 0; f < F; ++f) d += q[(long long)row * F + f] * k[(long long)j * F + f];
      d *= scale;
    }
    sc[j] = d;
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int j = threadIdx.x; j < T; j += blockDim.x) mx = fmaxf(mx, sc[j]);
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x + 31) / 32 ? red[threadIdx.x] : -INFINITY;
    t = warp_max(t);
    if (threadIdx.x == 0) stat = t;
  }
  __syncthreads();
  mx = stat;
  float sum = 0.f;
  for (int j = threadIdx.x; j < T; j += blockDim.x) {
    float e = (j <= last) ? expf(sc[j] - mx) : 0.f;
    sc[j] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x + 31) / 32 ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) stat = t;
  }
  __syncthreads();
  const float inv = 1.0f / stat;
  for (int f = threadIdx.x; f < F; f += blockDim.x) {
    float acc = 0.f;
    for (int j = 0; j <= last; ++j) acc += sc[j] * v[(long long)j * F + f];
    out[(long long)row * F + f] = acc * inv;
  }
}


}  // namespace

void gemm_f32_simt(const float* A, const float* B, float* C, int M, int N, int K, bool b_trans, cudaStream_t s) {
  if (M <= 0 || N <= 0) return;
  dim3 grid((N + TS - 1) / TS, (M + TS - 1) / TS);
  sgemm_kernel<<<grid, 256, 0, s>>>(A, B, C, M, N, K, b_trans);
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

void attention_naive_f32(const float* q, const float* k, const float* v, float* out, int tokens, int features,
                         float scale, bool causal, cudaStream_t s) {
  if (tokens <= 0) return;
  if ((size_t)tokens * sizeof(float) > 200 * 1024) throw std::runtime_error("attention_f32: too many tokens");
  if (tokens * sizeof(float) > 48 * 1024)
    UHFS_CUDA_CHECK(cudaFuncSetAttribute(attention_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         tokens * (int)sizeof(float)));
  attention_f32_kernel<<<tokens, 128, tokens * sizeof(float), s>>>(q, k, v, out, tokens, features, scale, causal);
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

}  // namespace uhfs
