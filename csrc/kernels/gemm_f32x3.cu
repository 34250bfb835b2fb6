// fp32 GEMM on the tf32 tensor cores with three products per term (3xTF32).
//
// Each operand element x is split into hi = tf32(x) (round to nearest) and
// lo = x - hi (exact in fp32; the tensor core keeps its top 10 mantissa
// bits).  hi*hi + hi*lo + lo*hi leaves out only lo*lo (~2^-22 of the
// product) and the truncation of lo (~2^-22 again), while the math runs on
// tcgen05 kind::tf32 at several times the rate of fp32 FMA units.  The three
// products are one GEMM over K' = 3 Kp: the split kernels write
//   A' = [hi(A) | lo(A) | hi(A)]  (M x 3Kp, K-major)
//   B' = [lo(B) | hi(B) | hi(B)]  (N x 3Kp, K-major; transposed from B[K,N])
// with zero padding from K to Kp (a multiple of 32, one tf32 k-block).  The
// tensor core's accumulation is not round-to-nearest: each MMA step loses
// about one unit in the last place of the running sum, so the small cross
// terms come first, while the sum is still small, and only the hi*hi steps
// run at the full magnitude.
//
// Replaces the reference's fp32 cublasSgemm in CudaTensorF32::matmul
// (cuda/kernels.cu:470-500) for large products; small ones keep the exact
// SIMT kernel.
#include <stdexcept>

#include "common.cuh"
#include "gemm.h"

namespace uhfs {

namespace {

__device__ __forceinline__ float tf32_round(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Segment s of the 3 Kp columns holds lo(x) where bit s of `lo_mask` is set,
// hi(x) otherwise.
__device__ __forceinline__ float4 pick4(int lo_mask, int s, const float4& hi, const float4& lo) {
  return ((lo_mask >> s) & 1) ? lo : hi;
}

// Row-major X[rows, K] (row stride ld) -> out[rows, 3 Kp], segments per
// lo_mask.  One thread per 4 consecutive k.
__global__ void split3_rows_kernel(const float* __restrict__ X, long long ld, int rows, int K, int Kp,
                                   float* __restrict__ out, int lo_mask) {
  const long long groups = (long long)rows * (Kp / 4);
  for (long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x; g < groups;
       g += (long long)gridDim.x * blockDim.x) {
    const long long r = g / (Kp / 4);
    const int k = (int)(g - r * (Kp / 4)) * 4;
    float4 hi, lo;
    float* h = &hi.x;
    float* l = &lo.x;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float x = (k + e < K) ? X[r * ld + k + e] : 0.f;
      h[e] = tf32_round(x);
      l[e] = x - h[e];
    }
    float* o = out + r * 3LL * Kp + k;
    *reinterpret_cast<float4*>(o) = pick4(lo_mask, 0, hi, lo);
    *reinterpret_cast<float4*>(o + Kp) = pick4(lo_mask, 1, hi, lo);
    *reinterpret_cast<float4*>(o + 2 * Kp) = pick4(lo_mask, 2, hi, lo);
  }
}

// X[K, N] (row stride ld) -> out[N, 3 Kp] (transposed), segments as above.
// 32 x 32 tiles through shared memory: reads along N, writes along K.
__global__ void split3_transpose_kernel(const float* __restrict__ X, long long ld, int K, int N, int Kp,
                                        float* __restrict__ out, int lo_mask) {
  __shared__ float tile[32][33];
  const int k0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    const int k = k0 + ty + i, n = n0 + tx;
    tile[ty + i][tx] = (k < K && n < N) ? X[(long long)k * ld + n] : 0.f;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    const int n = n0 + ty + i, k = k0 + tx;
    if (n < N && k < Kp) {
      const float x = tile[tx][ty + i];
      const float hi = tf32_round(x), lo = x - hi;
      float* o = out + (long long)n * 3 * Kp + k;
      o[0] = (lo_mask & 1) ? lo : hi;
      o[Kp] = (lo_mask & 2) ? lo : hi;
      o[2 * Kp] = (lo_mask & 4) ? lo : hi;
    }
  }
}

int grid_for(long long work, int threads) {
  const long long b = (work + threads - 1) / threads;
  return (int)(b < 148LL * 16 ? (b > 0 ? b : 1) : 148LL * 16);
}

}  // namespace

void gemm_f32_3xtf32(const float* A, const float* B, float* C, int M, int N, int K, bool b_trans, float* ws_a,
                     float* ws_b, cudaStream_t s) {
  if (M <= 0 || N <= 0) return;
  if (K <= 0) throw std::runtime_error("gemm_f32_3xtf32: K must be positive");
  if (N % 4 != 0) throw std::runtime_error("gemm_f32_3xtf32: N must be a multiple of 4 (fp32 row alignment)");
  const int Kp = (K + 31) / 32 * 32;
  // A' = [hi | lo | hi], B' = [lo | hi | hi]: hi*lo, lo*hi, then hi*hi
  constexpr int kLoA = 2, kLoB = 1;
  split3_rows_kernel<<<grid_for((long long)M * (Kp / 4), 256), 256, 0, s>>>(A, K, M, K, Kp, ws_a, kLoA);
  note_launch();
  if (b_trans) {
    split3_rows_kernel<<<grid_for((long long)N * (Kp / 4), 256), 256, 0, s>>>(B, K, N, K, Kp, ws_b, kLoB);
  } else {
    dim3 grid((N + 31) / 32, (Kp + 31) / 32);
    split3_transpose_kernel<<<grid, dim3(32, 8), 0, s>>>(B, N, K, N, Kp, ws_b, kLoB);
  }
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
  gemm_tf32_tcgen05(ws_a, 3LL * Kp, ws_b, 3LL * Kp, C, N, M, N, 3 * Kp, s);
}

}  // namespace uhfs
