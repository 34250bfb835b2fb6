// Vectorized elementwise, cast, GELU, reduction and bias-gradient kernels.
//
// Replaces the reference's one-element-per-thread SIMT kernels
// (cuda/kernels.cu:20-119: add/mul for fp32/fp16/bf16, fp32<->fp16/bf16
// conversion) and its multi-pass host-looped sum (cuda/kernels.cu:36-59,
// :518).  Here every kernel moves 16 bytes per thread per iteration over a
// grid-stride loop sized to the 148 SMs, and the sum is a single launch with a
// deterministic last-block-finishes reduction.  fp16/bf16 math is done in fp32
// and rounded once, matching the reference's bf16 kernels (kernels.cu:105-119).
#include <stdexcept>

#include "common.cuh"
#include "kernels.h"

namespace uhfs {

namespace {

template <typename T>
struct Vec;  // 16-byte vector of T
template <>
struct Vec<float> {
  static constexpr int N = 4;
};
template <>
struct Vec<__half> {
  static constexpr int N = 8;
};
template <>
struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
};

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ float from_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

__device__ __forceinline__ float apply(int op, float a, float b) {
  switch (op) {
    case OP_ADD: return a + b;
    case OP_MUL: return a * b;
    case OP_SUB: return a - b;
    default: return a / b;
  }
}

int grid_for(long long n_vec, int block) {
  long long g = (n_vec + block - 1) / block;
  const long long cap = 148LL * 8;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (int)g;
}

template <typename T>
__global__ void binary_kernel(int op, const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ out,
                              long long n, bool vec) {
  constexpr int V = Vec<T>::N;
  const long long nvec = vec ? n / V : 0;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nvec; i += stride) {
    uint4 ra = reinterpret_cast<const uint4*>(a)[i];
    uint4 rb = reinterpret_cast<const uint4*>(b)[i];
    uint4 ro;
    const T* pa = reinterpret_cast<const T*>(&ra);
    const T* pb = reinterpret_cast<const T*>(&rb);
    T* po = reinterpret_cast<T*>(&ro);
#pragma unroll
    for (int j = 0; j < V; ++j) po[j] = from_f<T>(apply(op, to_f(pa[j]), to_f(pb[j])));
    reinterpret_cast<uint4*>(out)[i] = ro;
  }
  for (long long i = nvec * V + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = from_f<T>(apply(op, to_f(a[i]), to_f(b[i])));
}

template <typename T>
__global__ void scalar_kernel(int op, const T* __restrict__ a, float s, T* __restrict__ out, long long n,
                              bool vec) {
  constexpr int V = Vec<T>::N;
  const long long nvec = vec ? n / V : 0;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nvec; i += stride) {
    uint4 ra = reinterpret_cast<const uint4*>(a)[i];
    uint4 ro;
    const T* pa = reinterpret_cast<const T*>(&ra);
    T* po = reinterpret_cast<T*>(&ro);
#pragma unroll
    for (int j = 0; j < V; ++j) po[j] = from_f<T>(apply(op, to_f(pa[j]), s));
    reinterpret_cast<uint4*>(out)[i] = ro;
  }
  for (long long i = nvec * V + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = from_f<T>(apply(op, to_f(a[i]), s));
}

template <typename S, typename D>
__global__ void cast_kernel(const S* __restrict__ src, D* __restrict__ dst, long long n) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long n4 = n / 4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += stride) {
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[i * 4 + j] = from_f<D>(to_f(src[i * 4 + j]));
  }
  for (long long i = n4 * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride)
    dst[i] = from_f<D>(to_f(src[i]));
}

template <typename T>
__global__ void gelu_fwd_kernel(const T* __restrict__ x, T* __restrict__ y, long long n) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride)
    y[i] = from_f<T>(sizeof(T) == 4 ? gelu_tanh(to_f(x[i])) : gelu_tanh_fast(to_f(x[i])));
}

template <typename T>
__global__ void gelu_bwd_kernel(const T* __restrict__ x, const T* __restrict__ dy, T* __restrict__ dx, long long n) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride)
    dx[i] = from_f<T>(to_f(dy[i]) * (sizeof(T) == 4 ? gelu_tanh_grad(to_f(x[i])) : gelu_tanh_grad_fast(to_f(x[i]))));
}

constexpr int kReduceBlocks = 296;
constexpr int kReduceThreads = 512;

template <typename T>
__global__ void __launch_bounds__(kReduceThreads) reduce_sum_kernel(const T* __restrict__ x, long long n,
                                                                    float* __restrict__ out,
                                                                    float* __restrict__ partials,
                                                                    unsigned int* __restrict__ counter) {
  __shared__ float warp_part[kReduceThreads / 32];
  __shared__ bool is_last;
  float acc = 0.f;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride) acc += to_f(x[i]);
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) warp_part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < kReduceThreads / 32 ? warp_part[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) {
      partials[blockIdx.x] = v;
      __threadfence();
      unsigned int done = atomicAdd(counter, 1u);
      is_last = (done == gridDim.x - 1);
    }
  }
  __syncthreads();
  if (is_last) {
    // Fixed-order final pass: deterministic for a fixed grid.
    __threadfence();
    float v = 0.f;
    for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) v += partials[i];
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) warp_part[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
      float w = threadIdx.x < kReduceThreads / 32 ? warp_part[threadIdx.x] : 0.f;
      w = warp_sum(w);
      if (threadIdx.x == 0) {
        out[0] = w;
        *counter = 0u;  // re-arm for the next launch (graph replay safe)
      }
    }
  }
}

// out[c] += sum_r x[r, c] for bf16 x with cols % 8 == 0 and 16-byte rows.
// A warp owns 256 consecutive columns (8 per lane, one 16-byte load per row),
// the 8 warps of a block stride over the block's rows, partial sums are
// combined in shared memory and added to `out` with one atomic per column per
// block.  Every warp load is a contiguous 512-byte segment.
__global__ void __launch_bounds__(256) colsum_vec_kernel(const __nv_bfloat16* __restrict__ x, long long ld,
                                                         float* __restrict__ out, int rows, int cols,
                                                         int rows_per_block) {
  __shared__ float part[8][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c0 = blockIdx.x * 256 + lane * 8;
  const int r0 = blockIdx.y * rows_per_block;
  const int r1 = min(rows, r0 + rows_per_block);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (c0 < cols) {
#pragma unroll 8
    for (int r = r0 + warp; r < r1; r += 8) {
      uint4 raw = __ldg(reinterpret_cast<const uint4*>(x + (long long)r * ld + c0));
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __bfloat1622float2(h[j]);
        acc[2 * j] += f.x;
        acc[2 * j + 1] += f.y;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) part[warp][lane * 8 + j] = acc[j];
  __syncthreads();
  const int c = blockIdx.x * 256 + threadIdx.x;
  if (c < cols) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += part[w][threadIdx.x];
    atomicAdd(out + c, s);
  }
}

// db[c] += sum_r x[r, c]; 128 threads x 2 columns, 256 rows per block-row (any alignment).
__global__ void colsum_kernel(const __nv_bfloat16* __restrict__ x, long long ld, float* __restrict__ out, int rows,
                              int cols) {
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 2;
  if (c >= cols) return;
  const int r0 = blockIdx.y * 256;
  const int r1 = min(rows, r0 + 256);
  float a0 = 0.f, a1 = 0.f;
  if (c + 1 < cols) {
    for (int r = r0; r < r1; ++r) {
      float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(x + (long long)r * ld + c));
      a0 += f.x;
      a1 += f.y;
    }
    atomicAdd(out + c, a0);
    atomicAdd(out + c + 1, a1);
  } else {
    for (int r = r0; r < r1; ++r) a0 += __bfloat162float(x[(long long)r * ld + c]);
    atomicAdd(out + c, a0);
  }
}

__global__ void fill_kernel(float* x, float v, long long n) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride) x[i] = v;
}

__global__ void increment_kernel(int* c) { *c += 1; }

template <typename T>
bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

}  // namespace

void ew_binary(int op, int dtype, const void* a, const void* b, void* out, long long n, cudaStream_t s) {
  if (n <= 0) return;
  const int block = 256;
  const bool vec = aligned16<void>(a) && aligned16<void>(b) && aligned16<void>(out);
  switch (dtype) {
    case DT_F32:
      binary_kernel<float><<<grid_for(vec ? n / 4 + 1 : n, block), block, 0, s>>>(op, (const float*)a, (const float*)b,
                                                                                  (float*)out, n, vec);
      break;
    case DT_F16:
      binary_kernel<__half><<<grid_for(vec ? n / 8 + 1 : n, block), block, 0, s>>>(op, (const __half*)a,
                                                                                   (const __half*)b, (__half*)out, n, vec);
      break;
    case DT_BF16:
      binary_kernel<__nv_bfloat16><<<grid_for(vec ? n / 8 + 1 : n, block), block, 0, s>>>(
          op, (const __nv_bfloat16*)a, (const __nv_bfloat16*)b, (__nv_bfloat16*)out, n, vec);
      break;
    default:
      throw std::runtime_error("ew_binary: unsupported dtype");
  }
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

void ew_scalar(int op, int dtype, const void* a, float scalar, void* out, long long n, cudaStream_t s) {
  if (n <= 0) return;
  const int block = 256;
  const bool vec = aligned16<void>(a) && aligned16<void>(out);
  switch (dtype) {
    case DT_F32:
      scalar_kernel<float><<<grid_for(vec ? n / 4 + 1 : n, block), block, 0, s>>>(op, (const float*)a, scalar,
                                                                                  (float*)out, n, vec);
      break;
    case DT_F16:
      scalar_kernel<__half><<<grid_for(vec ? n / 8 + 1 : n, block), block, 0, s>>>(op, (const __half*)a, scalar,
                                                                                   (__half*)out, n, vec);
      break;
    case DT_BF16:
      scalar_kernel<__nv_bfloat16><<<grid_for(vec ? n / 8 + 1 : n, block), block, 0, s>>>(
          op, (const __nv_bfloat16*)a, scalar, (__nv_bfloat16*)out, n, vec);
      break;
    default:
      throw std::runtime_error("ew_scalar: unsupported dtype");
  }
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

template <typename S>
static void cast_from(int dst, const S* src, void* out, long long n, cudaStream_t s) {
  const int block = 256;
  const int g = grid_for(n / 4 + 1, block);
  switch (dst) {
    case DT_F32: cast_kernel<S, float><<<g, block, 0, s>>>(src, (float*)out, n); break;
    case DT_F16: cast_kernel<S, __half><<<g, block, 0, s>>>(src, (__half*)out, n); break;
    case DT_BF16: cast_kernel<S, __nv_bfloat16><<<g, block, 0, s>>>(src, (__nv_bfloat16*)out, n); break;
    default: throw std::runtime_error("cast: unsupported dtype");
  }
}

void cast(int src_dtype, int dst_dtype, const void* src, void* dst, long long n, cudaStream_t s) {
  if (n <= 0) return;
  switch (src_dtype) {
    case DT_F32: cast_from<float>(dst_dtype, (const float*)src, dst, n, s); break;
    case DT_F16: cast_from<__half>(dst_dtype, (const __half*)src, dst, n, s); break;
    case DT_BF16: cast_from<__nv_bfloat16>(dst_dtype, (const __nv_bfloat16*)src, dst, n, s); break;
    default: throw std::runtime_error("cast: unsupported dtype");
  }
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

int reduce_sum_partials() { return kReduceBlocks; }

void reduce_sum(int dtype, const void* x, long long n, float* out, float* partials, unsigned int* counter,
                cudaStream_t s) {
  long long want = (n + kReduceThreads * 4 - 1) / (kReduceThreads * 4);
  int g = (int)(want < 1 ? 1 : (want > kReduceBlocks ? kReduceBlocks : want));
  switch (dtype) {
    case DT_F32: reduce_sum_kernel<float><<<g, kReduceThreads, 0, s>>>((const float*)x, n, out, partials, counter); break;
    case DT_F16: reduce_sum_kernel<__half><<<g, kReduceThreads, 0, s>>>((const __half*)x, n, out, partials, counter); break;
    case DT_BF16:
      reduce_sum_kernel<__nv_bfloat16><<<g, kReduceThreads, 0, s>>>((const __nv_bfloat16*)x, n, out, partials, counter);
      break;
    default: throw std::runtime_error("reduce_sum: unsupported dtype");
  }
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

void gelu_fwd(int dtype, const void* x, void* y, long long n, cudaStream_t s) {
  if (n <= 0) return;
  const int g = grid_for(n, 256);
  switch (dtype) {
    case DT_F32: gelu_fwd_kernel<float><<<g, 256, 0, s>>>((const float*)x, (float*)y, n); break;
    case DT_F16: gelu_fwd_kernel<__half><<<g, 256, 0, s>>>((const __half*)x, (__half*)y, n); break;
    case DT_BF16: gelu_fwd_kernel<__nv_bfloat16><<<g, 256, 0, s>>>((const __nv_bfloat16*)x, (__nv_bfloat16*)y, n); break;
    default: throw std::runtime_error("gelu: unsupported dtype");
  }
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

void gelu_bwd(int dtype, const void* x, const void* dy, void* dx, long long n, cudaStream_t s) {
  if (n <= 0) return;
  const int g = grid_for(n, 256);
  switch (dtype) {
    case DT_F32: gelu_bwd_kernel<float><<<g, 256, 0, s>>>((const float*)x, (const float*)dy, (float*)dx, n); break;
    case DT_F16: gelu_bwd_kernel<__half><<<g, 256, 0, s>>>((const __half*)x, (const __half*)dy, (__half*)dx, n); break;
    case DT_BF16:
      gelu_bwd_kernel<__nv_bfloat16><<<g, 256, 0, s>>>((const __nv_bfloat16*)x, (const __nv_bfloat16*)dy,
                                                        (__nv_bfloat16*)dx, n);
      break;
    default: throw std::runtime_error("gelu_bwd: unsupported dtype");
  }
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

void colsum_accum(const __nv_bfloat16* x, long long ld, float* out, int rows, int cols, cudaStream_t s) {
  if (rows <= 0 || cols <= 0) return;
  if (cols % 8 == 0 && ld % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
    const int gx = (cols + 255) / 256;
    // ~8 blocks (64 warps) per SM keep enough loads in flight.  Wide
    // matrices cap the blocks per column range at 64 (the per-column atomics
    // then stay off the critical path: 16384 x 3072 in 15.6 us); narrow ones
    // (fewer than 8 column ranges) need up to 256 to fill the GPU at all
    // (a cap of 64 gives 192 blocks, 1.3 waves, for 768 columns).
    int gy = min(gx < 8 ? 256 : 64, (8 * 148 + gx - 1) / gx);
    int rpb = (rows + gy - 1) / gy;
    rpb = (rpb + 7) / 8 * 8;
    gy = (rows + rpb - 1) / rpb;
    colsum_vec_kernel<<<dim3(gx, gy), 256, 0, s>>>(x, ld, out, rows, cols, rpb);
  } else {
    dim3 grid((cols / 2 + 127) / 128 + 1, (rows + 255) / 256);
    colsum_kernel<<<grid, 128, 0, s>>>(x, ld, out, rows, cols);
  }
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

void fill_f32(float* x, float v, long long n, cudaStream_t s) {
  if (n <= 0) return;
  fill_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, v, n);
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

void increment_counter(int* counter, cudaStream_t s) {
  increment_kernel<<<1, 1, 0, s>>>(counter);
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

}  // namespace uhfs
