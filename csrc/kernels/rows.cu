// Row-wise kernels: RMSNorm fwd/bwd, token+position embedding gather /
// scatter-add, fused softmax cross-entropy, row softmax.
//
// The reference computes all of these in pure Python over list storage
// (RMSNorm nn.py:166-181, Embedding nn.py:184-217, cross_entropy
// functional.py:20-76, softmax tensor.py:966-1027).  Here one warp (RMSNorm,
// embedding) or one CTA (cross-entropy over a 32K vocabulary) owns a row; all
// loads are 16-byte vectors, statistics are fp32, and the cross-entropy kernel
// emits the logits gradient in the same pass that computes the loss.
#include <type_traits>
#include <stdexcept>

#include "common.cuh"
#include "kernels.h"
#include "vec.cuh"

namespace uhfs {

namespace {

bool al16(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 8 x 16-bit <-> 8 x fp32 on the register words (no address-taken temporaries).
template <typename T>
__device__ __forceinline__ void unpack2(uint32_t w, float& lo, float& hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    lo = __uint_as_float(w << 16);  // bf16 -> fp32 is exact: the high half of the word
    hi = __uint_as_float(w & 0xffff0000u);
  } else {
    lo = __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)));
    hi = __half2float(__ushort_as_half((unsigned short)(w >> 16)));
  }
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4 raw, float (&f)[8]) {
  unpack2<T>(raw.x, f[0], f[1]);
  unpack2<T>(raw.y, f[2], f[3]);
  unpack2<T>(raw.z, f[4], f[5]);
  unpack2<T>(raw.w, f[6], f[7]);
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(pack2<T>(f[0], f[1]), pack2<T>(f[2], f[3]), pack2<T>(f[4], f[5]), pack2<T>(f[6], f[7]));
}

// ------------------------------------------------------------------ RMSNorm
template <typename T>
__global__ void rmsnorm_fwd_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y,
                                   float* __restrict__ rstd, int rows, int cols, float eps, bool vec) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < rows; row += gridDim.x * warps) {
    const T* xr = x + (long long)row * cols;
    float ss = 0.f;
    for (int c = lane * 8; c < cols; c += 256) {
      float f[8];
      load8_guard<T>(xr + c, f, c, cols, vec);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / (float)cols + eps);
    if (lane == 0 && rstd != nullptr) rstd[row] = r;
    T* yr = y + (long long)row * cols;
    for (int c = lane * 8; c < cols; c += 256) {
      float f[8], g[8];
      load8_guard<T>(xr + c, f, c, cols, vec);
      load8_guard<T>(w + c, g, c, cols, vec);
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = f[i] * r * g[i];
      store8_guard<T>(yr + c, f, c, cols, vec);
    }
  }
}

// 16-bit rows of cols <= 256 * VPL (cols % 8 == 0): the warp keeps its row
// slice in registers, so x is read once.
template <typename T, int VPL>
__global__ void __launch_bounds__(256) rmsnorm_fwd_reg_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                              T* __restrict__ y, float* __restrict__ rstd, int rows,
                                                              int cols, float eps) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float wv[VPL][8];
#pragma unroll
  for (int v = 0; v < VPL; ++v) {
    const int c = (v * 32 + lane) * 8;
    if (c < cols) unpack8<T>(*reinterpret_cast<const uint4*>(w + c), wv[v]);
  }
  for (int row = blockIdx.x * 8 + warp; row < rows; row += gridDim.x * 8) {
    const long long off = (long long)row * cols;
    uint4 rx[VPL];
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int c = (v * 32 + lane) * 8;
      if (c < cols) rx[v] = __ldcs(reinterpret_cast<const uint4*>(x + off + c));
    }
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      if ((v * 32 + lane) * 8 < cols) {
        float f[8];
        unpack8<T>(rx[v], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
      }
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / (float)cols + eps);
    if (lane == 0 && rstd != nullptr) rstd[row] = r;
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int c = (v * 32 + lane) * 8;
      if (c < cols) {
        float f[8];
        unpack8<T>(rx[v], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = f[j] * r * wv[v][j];
        *reinterpret_cast<uint4*>(y + off + c) = pack8<T>(f);
      }
    }
  }
}

// dx_i = r * (g_i - x_i * r^2 * sum_j(g_j x_j) / n),   g = dy * w
template <typename T>
__global__ void rmsnorm_bwd_dx_kernel(const T* __restrict__ dy, const T* __restrict__ x, const T* __restrict__ w,
                                      const float* __restrict__ rstd, const T* __restrict__ dres, T* __restrict__ dx,
                                      int rows, int cols, bool vec) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < rows; row += gridDim.x * warps) {
    const long long off = (long long)row * cols;
    float dot = 0.f;
    for (int c = lane * 8; c < cols; c += 256) {
      float a[8], b[8], g[8];
      load8_guard<T>(dy + off + c, a, c, cols, vec);
      load8_guard<T>(x + off + c, b, c, cols, vec);
      load8_guard<T>(w + c, g, c, cols, vec);
#pragma unroll
      for (int i = 0; i < 8; ++i) dot += a[i] * g[i] * b[i];
    }
    dot = warp_sum(dot);
    const float r = rstd[row];
    const float coef = r * r * dot / (float)cols;
    for (int c = lane * 8; c < cols; c += 256) {
      float a[8], b[8], g[8], o[8];
      load8_guard<T>(dy + off + c, a, c, cols, vec);
      load8_guard<T>(x + off + c, b, c, cols, vec);
      load8_guard<T>(w + c, g, c, cols, vec);
      if (dres != nullptr) {
        load8_guard<T>(dres + off + c, o, c, cols, vec);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] += r * (a[i] * g[i] - b[i] * coef);
      store8_guard<T>(dx + off + c, o, c, cols, vec);
    }
  }
}

// One pass for the whole backward (16-bit, cols <= 256 * VPL, cols % 8 == 0):
// a warp owns a row at a time and keeps its dy / x / dres slices in registers
// (VPL 16-byte vectors per lane), writes dx, and accumulates the dgamma
// partials dy * x * r of its columns across all rows it visits; the block
// combines the 8 warps' partials in shared memory and adds them to dw with
// one atomic per column.  Reads dy, x, dres once and writes dx once.
template <typename T, int VPL>
__global__ void __launch_bounds__(256) rmsnorm_bwd_fused_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                                                const T* __restrict__ w,
                                                                const float* __restrict__ rstd,
                                                                const T* __restrict__ dres, T* __restrict__ dx,
                                                                float* __restrict__ dw, int rows, int cols) {
  __shared__ float part[8][VPL * 256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float wv[VPL][8], acc[VPL][8];
#pragma unroll
  for (int v = 0; v < VPL; ++v) {
    const int c = (v * 32 + lane) * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[v][j] = 0.f;
    if (c < cols) unpack8<T>(*reinterpret_cast<const uint4*>(w + c), wv[v]);
    else {
#pragma unroll
      for (int j = 0; j < 8; ++j) wv[v][j] = 0.f;
    }
  }
  const float inv_cols = 1.0f / (float)cols;
  for (int row = blockIdx.x * 8 + warp; row < rows; row += gridDim.x * 8) {
    const long long off = (long long)row * cols;
    uint4 rdy[VPL], rx[VPL], rres[VPL];
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int c = (v * 32 + lane) * 8;
      if (c < cols) {
        rdy[v] = __ldcs(reinterpret_cast<const uint4*>(dy + off + c));
        rx[v] = __ldcs(reinterpret_cast<const uint4*>(x + off + c));
        if (dres != nullptr) rres[v] = __ldcs(reinterpret_cast<const uint4*>(dres + off + c));
      }
    }
    float dot = 0.f;
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      if ((v * 32 + lane) * 8 < cols) {
        float a[8], b[8];
        unpack8<T>(rdy[v], a);
        unpack8<T>(rx[v], b);
#pragma unroll
        for (int j = 0; j < 8; ++j) dot = fmaf(a[j] * wv[v][j], b[j], dot);
      }
    }
    dot = warp_sum(dot);
    const float r = rstd[row];
    const float coef = r * r * dot * inv_cols;
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int c = (v * 32 + lane) * 8;
      if (c < cols) {
        float a[8], b[8], o[8];
        unpack8<T>(rdy[v], a);
        unpack8<T>(rx[v], b);
        if (dres != nullptr) unpack8<T>(rres[v], o);
        else {
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          o[j] += r * (a[j] * wv[v][j] - b[j] * coef);
          acc[v][j] = fmaf(a[j] * b[j], r, acc[v][j]);
        }
        __stcs(reinterpret_cast<uint4*>(dx + off + c), pack8<T>(o));
      }
    }
  }
  if (dw == nullptr) return;
#pragma unroll
  for (int v = 0; v < VPL; ++v)
#pragma unroll
    for (int j = 0; j < 8; ++j) part[warp][(v * 32 + lane) * 8 + j] = acc[v][j];
  __syncthreads();
  for (int c = threadIdx.x; c < cols; c += 256) {
    float sum = 0.f;
#pragma unroll
    for (int w8 = 0; w8 < 8; ++w8) sum += part[w8][c];
    atomicAdd(dw + c, sum);
  }
}

// dw_j += sum_rows dy_rj * x_rj * r_r, 16-byte vector form: a warp owns 256
// columns (8 per lane), 8 warps stride over the block's rows, shared-memory
// combine, one atomic per column per block.
template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_bwd_dw_vec_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                                                 const float* __restrict__ rstd,
                                                                 float* __restrict__ dw, int rows, int cols,
                                                                 int rows_per_block) {
  __shared__ float part[8][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c0 = blockIdx.x * 256 + lane * 8;
  const int r0 = blockIdx.y * rows_per_block;
  const int r1 = min(rows, r0 + rows_per_block);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (c0 < cols) {
#pragma unroll 2
    for (int r = r0 + warp; r < r1; r += 8) {
      float a[8], b[8];
      load8<T>(dy + (long long)r * cols + c0, a);
      load8<T>(x + (long long)r * cols + c0, b);
      const float rs = rstd[r];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += a[j] * b[j] * rs;
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
    atomicAdd(dw + c, s);
  }
}

// dw_j += sum_rows dy_rj * x_rj * r_r; one thread per column pair-of-4, 128 rows per block-row.
template <typename T>
__global__ void rmsnorm_bwd_dw_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                      const float* __restrict__ rstd, float* __restrict__ dw, int rows, int cols) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  const int r0 = blockIdx.y * 128;
  const int r1 = min(rows, r0 + 128);
  float acc = 0.f;
  for (int r = r0; r < r1; ++r) {
    const long long o = (long long)r * cols + c;
    acc += to_float<T>(dy[o]) * to_float<T>(x[o]) * rstd[r];
  }
  atomicAdd(dw + c, acc);
}

// ---------------------------------------------------------------- embedding
template <typename T>
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids, const T* __restrict__ tok,
                                     const T* __restrict__ pos, T* __restrict__ out, int rows, int dim, int seq_len,
                                     bool vec, long long vocab, DeviceStatus* status) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < rows; row += gridDim.x * warps) {
    const long long id = ids[row];
    T* orow_bad = out + (long long)row * dim;
    if (vocab > 0 && (id < 0 || id >= vocab)) {
      // an id outside the table: record it and emit zeros instead of reading outside it
      if (lane == 0) report_error(status, kErrBounds, 50);
      for (int c = lane; c < dim; c += 32) orow_bad[c] = from_float<T>(0.f);
      continue;
    }
    const T* tr = tok + id * dim;
    const T* pr = pos != nullptr ? pos + (long long)(row % seq_len) * dim : nullptr;
    T* orow = out + (long long)row * dim;
    for (int c = lane * 8; c < dim; c += 256) {
      float a[8];
      load8_guard<T>(tr + c, a, c, dim, vec);
      if (pr != nullptr) {
        float b[8];
        load8_guard<T>(pr + c, b, c, dim, vec);
#pragma unroll
        for (int i = 0; i < 8; ++i) a[i] += b[i];
      }
      store8_guard<T>(orow + c, a, c, dim, vec);
    }
  }
}

template <typename T>
__global__ void embedding_bwd_kernel(const int64_t* __restrict__ ids, const T* __restrict__ dout,
                                     float* __restrict__ dtok, float* __restrict__ dpos, int rows, int dim,
                                     int seq_len, bool vec, long long vocab, DeviceStatus* status) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < rows; row += gridDim.x * warps) {
    const long long id = ids[row];
    if (vocab > 0 && (id < 0 || id >= vocab)) {
      if (lane == 0) report_error(status, kErrBounds, 51);
      continue;
    }
    const T* dr = dout + (long long)row * dim;
    float* tr = dtok != nullptr ? dtok + id * dim : nullptr;
    float* pr = dpos != nullptr ? dpos + (long long)(row % seq_len) * dim : nullptr;
    for (int c = lane * 8; c < dim; c += 256) {
      float a[8];
      load8_guard<T>(dr + c, a, c, dim, vec);
      if (vec && c + 8 <= dim) {
        if (tr) {
          atomicAdd(reinterpret_cast<float4*>(tr + c), make_float4(a[0], a[1], a[2], a[3]));
          atomicAdd(reinterpret_cast<float4*>(tr + c + 4), make_float4(a[4], a[5], a[6], a[7]));
        }
        if (pr) {
          atomicAdd(reinterpret_cast<float4*>(pr + c), make_float4(a[0], a[1], a[2], a[3]));
          atomicAdd(reinterpret_cast<float4*>(pr + c + 4), make_float4(a[4], a[5], a[6], a[7]));
        }
      } else {
        for (int i = 0; i < 8 && c + i < dim; ++i) {
          if (tr) atomicAdd(tr + c + i, a[i]);
          if (pr) atomicAdd(pr + c + i, a[i]);
        }
      }
    }
  }
}

// ------------------------------------------------------------- softmax + CE
constexpr int kCeThreads = 512;

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;
  s = s * __expf(m - mn) + s2 * __expf(m2 - mn);
  m = mn;
}

// 16-bit logits, row held in registers: every thread loads its (up to)
// kCeVecs 16-byte vectors once, so each row is read from memory once and
// written once (dlogits) -- the minimum traffic.  Block max, then block sum.
constexpr int kCeVecs = 8;  // rows up to kCeThreads * 8 * kCeVecs = 32768 columns

__device__ __forceinline__ float block_reduce_max(float v, float* sm) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = v;
  __syncthreads();
  v = sm[0];
#pragma unroll
  for (int w = 1; w < kCeThreads / 32; ++w) v = fmaxf(v, sm[w]);
  __syncthreads();
  return v;
}

__device__ __forceinline__ float block_reduce_sum(float v, float* sm) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = v;
  __syncthreads();
  v = 0.f;
#pragma unroll
  for (int w = 0; w < kCeThreads / 32; ++w) v += sm[w];
  __syncthreads();
  return v;
}

template <typename T>
__global__ void __launch_bounds__(kCeThreads, 2) softmax_ce_reg_kernel(const T* __restrict__ logits, long long ld,
                                                                      const int64_t* __restrict__ targets,
                                                                      float* __restrict__ loss_rows, T* dlogits,
                                                                      int cols, float grad_scale,
                                                                      const float* grad_scale_ptr,
                                                                      DeviceStatus* status) {
  __shared__ float sm[kCeThreads / 32];
  const int row = blockIdx.x;
  const T* lr = logits + (long long)row * ld;
  const int nvec = cols / 8;
  uint4 raw[kCeVecs];
#pragma unroll
  for (int k = 0; k < kCeVecs; ++k) {
    const int v = threadIdx.x + k * kCeThreads;
    if (v < nvec) raw[k] = __ldcs(reinterpret_cast<const uint4*>(lr) + v);  // read once: streaming
  }
  float mx = -INFINITY;
#pragma unroll
  for (int k = 0; k < kCeVecs; ++k) {
    if (threadIdx.x + k * kCeThreads < nvec) {
      float f[8];
      unpack8<T>(raw[k], f);
#pragma unroll
      for (int i = 0; i < 8; ++i) mx = fmaxf(mx, f[i]);
    }
  }
  mx = block_reduce_max(mx, sm);
  // exp(x - mx) = 2^(x log2e - mx log2e): one FMA and one MUFU ex2 per
  // logit, computed once; the exponentials replace the logits in `raw`
  // (rounded to T, the gradient's own type) for the gradient pass
  const float l2e = 1.4426950408889634f, mxl = mx * l2e;
  float sum = 0.f;
#pragma unroll
  for (int k = 0; k < kCeVecs; ++k) {
    if (threadIdx.x + k * kCeThreads < nvec) {
      float f[8];
      unpack8<T>(raw[k], f);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        f[i] = ex2_approx(fmaf(f[i], l2e, -mxl));
        sum += f[i];
      }
      raw[k] = pack8<T>(f);
    }
  }
  const long long tgt = targets[row];
  const bool tgt_ok = tgt >= 0 && tgt < cols;  // an invalid target is reported, never read
  if (!tgt_ok && threadIdx.x == 0) report_error(status, kErrBounds, 52);
  // the target logit is read before the block barrier inside the sum
  // reduction, so an in-place dlogits (== logits) cannot overwrite it first
  const float xt = (threadIdx.x == 0 && tgt_ok) ? to_float<T>(lr[tgt]) : 0.f;
  sum = block_reduce_sum(sum, sm);
  if (threadIdx.x == 0) {
    // -log(max(p_t, 1e-30)) as in the reference, computed in log space.
    const float nll = logf(sum) + mx - xt;
    loss_rows[row] = tgt_ok ? fminf(nll, 69.07755279f) : __int_as_float(0x7fc00000);  // NaN marks the bad row
  }
  if (dlogits == nullptr) return;
  if (grad_scale_ptr != nullptr) grad_scale *= *grad_scale_ptr;
  const float inv = grad_scale / sum;
  T* dr = dlogits + (long long)row * ld;
#pragma unroll
  for (int k = 0; k < kCeVecs; ++k) {
    const int v = threadIdx.x + k * kCeThreads;
    if (v < nvec) {
      float f[8];
      unpack8<T>(raw[k], f);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        f[i] *= inv;
        if ((long long)v * 8 + i == tgt) f[i] -= grad_scale;
      }
      __stcs(reinterpret_cast<uint4*>(dr) + v, pack8<T>(f));
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kCeThreads) softmax_ce_kernel(const T* __restrict__ logits, long long ld,
                                                                const int64_t* __restrict__ targets,
                                                                float* __restrict__ loss_rows, T* dlogits, int cols,
                                                                float grad_scale, const float* grad_scale_ptr,
                                                                bool vec, DeviceStatus* status) {
  const int row = blockIdx.x;
  const T* lr = logits + (long long)row * ld;
  __shared__ float sm_m[kCeThreads / 32], sm_s[kCeThreads / 32];
  __shared__ float row_max, row_sum;
  float m = -INFINITY, s = 0.f;
  for (int c = threadIdx.x * 8; c < cols; c += kCeThreads * 8) {
    float f[8];
    load8_guard<T>(lr + c, f, c, cols, vec);
    float lm = -INFINITY;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (c + i < cols) lm = fmaxf(lm, f[i]);
    float ls = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (c + i < cols) ls += __expf(f[i] - lm);
    online_merge(m, s, lm, ls);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  if ((threadIdx.x & 31) == 0) {
    sm_m[threadIdx.x >> 5] = m;
    sm_s[threadIdx.x >> 5] = s;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < kCeThreads / 32 ? sm_m[threadIdx.x] : -INFINITY;
    s = threadIdx.x < kCeThreads / 32 ? sm_s[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      online_merge(m, s, m2, s2);
    }
    if (threadIdx.x == 0) {
      row_max = m;
      row_sum = s;
    }
  }
  __syncthreads();
  const float mx = row_max;
  const float inv = 1.0f / row_sum;
  const long long tgt = targets[row];
  const bool tgt_ok = tgt >= 0 && tgt < cols;
  if (threadIdx.x == 0) {
    if (!tgt_ok) {
      report_error(status, kErrBounds, 53);
      loss_rows[row] = __int_as_float(0x7fc00000);
    } else {
      const float xt = to_float<T>(lr[tgt]);
      // -log(max(p_t, 1e-30)) as in the reference, computed in log space.
      const float nll = logf(row_sum) + mx - xt;
      loss_rows[row] = fminf(nll, 69.07755279f);
    }
  }
  if (dlogits == nullptr) return;
  if (grad_scale_ptr != nullptr) grad_scale *= *grad_scale_ptr;
  // Every thread has read its slice of the row above; the block barrier makes
  // the in-place overwrite (dlogits == logits) safe for the target logit too.
  __syncthreads();
  T* dr = dlogits + (long long)row * ld;
  for (int c = threadIdx.x * 8; c < cols; c += kCeThreads * 8) {
    float f[8];
    load8_guard<T>(lr + c, f, c, cols, vec);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float p = __expf(f[i] - mx) * inv;
      if (c + i == tgt) p -= 1.0f;
      f[i] = p * grad_scale;
    }
    store8_guard<T>(dr + c, f, c, cols, vec);
  }
}

template <typename T>
__global__ void __launch_bounds__(kCeThreads) softmax_rows_kernel(const T* __restrict__ x, T* __restrict__ y,
                                                                  int cols) {
  const int row = blockIdx.x;
  const T* xr = x + (long long)row * cols;
  T* yr = y + (long long)row * cols;
  __shared__ float sm_m[kCeThreads / 32], sm_s[kCeThreads / 32];
  __shared__ float row_max, row_sum;
  float m = -INFINITY, s = 0.f;
  for (int c = threadIdx.x; c < cols; c += kCeThreads) online_merge(m, s, to_float<T>(xr[c]), 1.0f);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  if ((threadIdx.x & 31) == 0) {
    sm_m[threadIdx.x >> 5] = m;
    sm_s[threadIdx.x >> 5] = s;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < kCeThreads / 32 ? sm_m[threadIdx.x] : -INFINITY;
    s = threadIdx.x < kCeThreads / 32 ? sm_s[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      online_merge(m, s, m2, s2);
    }
    if (threadIdx.x == 0) {
      row_max = m;
      row_sum = s;
    }
  }
  __syncthreads();
  const float mx = row_max, inv = 1.0f / row_sum;
  for (int c = threadIdx.x; c < cols; c += kCeThreads) yr[c] = from_float<T>(__expf(to_float<T>(xr[c]) - mx) * inv);
}

template <typename T>
__global__ void __launch_bounds__(kCeThreads) softmax_rows_bwd_kernel(const T* __restrict__ y, const T* __restrict__ dy,
                                                                      T* __restrict__ dx, int cols) {
  const int row = blockIdx.x;
  const long long off = (long long)row * cols;
  __shared__ float part[kCeThreads / 32];
  __shared__ float dot_s;
  float d = 0.f;
  for (int c = threadIdx.x; c < cols; c += kCeThreads) d += to_float<T>(y[off + c]) * to_float<T>(dy[off + c]);
  d = warp_sum(d);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = d;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < kCeThreads / 32 ? part[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) dot_s = v;
  }
  __syncthreads();
  const float dot = dot_s;
  for (int c = threadIdx.x; c < cols; c += kCeThreads)
    dx[off + c] = from_float<T>(to_float<T>(y[off + c]) * (to_float<T>(dy[off + c]) - dot));
}

int row_grid(int rows, int warps_per_block) {
  long long g = (rows + warps_per_block - 1) / warps_per_block;
  if (g > 148LL * 16) g = 148LL * 16;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace

#define UHFS_DISPATCH_DTYPE(dtype, ...)                                  \
  switch (dtype) {                                                       \
    case DT_F32: { using T = float; __VA_ARGS__; break; }                \
    case DT_F16: { using T = __half; __VA_ARGS__; break; }               \
    case DT_BF16: { using T = __nv_bfloat16; __VA_ARGS__; break; }       \
    default: throw std::runtime_error("unsupported dtype");              \
  }

void rmsnorm_fwd(int dtype, const void* x, const void* w, void* y, float* rstd, int rows, int cols, float eps,
                 cudaStream_t s) {
  if (rows <= 0) return;
  const bool vec = al16(x) && al16(w) && al16(y) && (cols % 8 == 0);
  if (vec && dtype != DT_F32 && cols <= 4 * 256) {
    int grid = (rows + 7) / 8;
    if (grid > 8 * 148) grid = 8 * 148;
    const int vpl = (cols + 255) / 256;
#define UHFS_RMS_FWD(TT, V)                                                                                      \
  rmsnorm_fwd_reg_kernel<TT, V><<<grid, 256, 0, s>>>((const TT*)x, (const TT*)w, (TT*)y, rstd, rows, cols, eps)
    if (dtype == DT_BF16) {
      if (vpl == 1) UHFS_RMS_FWD(__nv_bfloat16, 1);
      else if (vpl == 2) UHFS_RMS_FWD(__nv_bfloat16, 2);
      else if (vpl == 3) UHFS_RMS_FWD(__nv_bfloat16, 3);
      else UHFS_RMS_FWD(__nv_bfloat16, 4);
    } else {
      if (vpl == 1) UHFS_RMS_FWD(__half, 1);
      else if (vpl == 2) UHFS_RMS_FWD(__half, 2);
      else if (vpl == 3) UHFS_RMS_FWD(__half, 3);
      else UHFS_RMS_FWD(__half, 4);
    }
#undef UHFS_RMS_FWD
    note_launch();
    UHFS_CUDA_CHECK(cudaGetLastError());
    return;
  }
  UHFS_DISPATCH_DTYPE(dtype, rmsnorm_fwd_kernel<T><<<row_grid(rows, 8), 256, 0, s>>>(
                                 (const T*)x, (const T*)w, (T*)y, rstd, rows, cols, eps, vec));
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

void rmsnorm_bwd(int dtype, const void* dy, const void* x, const void* w, const float* rstd, const void* dres,
                 void* dx, float* dw_accum, int rows, int cols, cudaStream_t s) {
  if (rows <= 0) return;
  const bool vec = al16(dy) && al16(x) && al16(w) && al16(dres) && al16(dx) && (cols % 8 == 0);
  if (vec && dtype != DT_F32 && cols <= 4 * 256) {
    // 2 blocks per SM: enough rows in flight, and at most 296 atomics per dgamma column
    int grid = (rows + 7) / 8;
    if (grid > 2 * 148) grid = 2 * 148;
    const int vpl = (cols + 255) / 256;
#define UHFS_RMS_FUSED(TT, V)                                                                                  \
  rmsnorm_bwd_fused_kernel<TT, V><<<grid, 256, 0, s>>>((const TT*)dy, (const TT*)x, (const TT*)w, rstd,         \
                                                      (const TT*)dres, (TT*)dx, dw_accum, rows, cols)
    if (dtype == DT_BF16) {
      if (vpl == 1) UHFS_RMS_FUSED(__nv_bfloat16, 1);
      else if (vpl == 2) UHFS_RMS_FUSED(__nv_bfloat16, 2);
      else if (vpl == 3) UHFS_RMS_FUSED(__nv_bfloat16, 3);
      else UHFS_RMS_FUSED(__nv_bfloat16, 4);
    } else {
      if (vpl == 1) UHFS_RMS_FUSED(__half, 1);
      else if (vpl == 2) UHFS_RMS_FUSED(__half, 2);
      else if (vpl == 3) UHFS_RMS_FUSED(__half, 3);
      else UHFS_RMS_FUSED(__half, 4);
    }
#undef UHFS_RMS_FUSED
    note_launch();
    UHFS_CUDA_CHECK(cudaGetLastError());
    return;
  }
  UHFS_DISPATCH_DTYPE(dtype, rmsnorm_bwd_dx_kernel<T><<<row_grid(rows, 8), 256, 0, s>>>(
                                 (const T*)dy, (const T*)x, (const T*)w, rstd, (const T*)dres, (T*)dx, rows, cols, vec));
  note_launch();
  if (dw_accum != nullptr) {
    if (vec) {
      const int gx = (cols + 255) / 256;
      int gy = (2 * 148 + gx - 1) / gx;
      int rpb = (rows + gy - 1) / gy;
      rpb = (rpb + 7) / 8 * 8;
      gy = (rows + rpb - 1) / rpb;
      UHFS_DISPATCH_DTYPE(dtype, rmsnorm_bwd_dw_vec_kernel<T><<<dim3(gx, gy), 256, 0, s>>>(
                                     (const T*)dy, (const T*)x, rstd, dw_accum, rows, cols, rpb));
    } else {
      dim3 grid((cols + 255) / 256, (rows + 127) / 128);
      UHFS_DISPATCH_DTYPE(dtype, rmsnorm_bwd_dw_kernel<T><<<grid, 256, 0, s>>>((const T*)dy, (const T*)x, rstd,
                                                                               dw_accum, rows, cols));
    }
    note_launch();
  }
  UHFS_CUDA_CHECK(cudaGetLastError());
}

void embedding_fwd(int dtype, const int64_t* ids, const void* tok, const void* pos, void* out, int rows, int dim,
                   int seq_len, long long vocab, cudaStream_t s) {
  if (rows <= 0) return;
  const bool vec = al16(tok) && al16(pos) && al16(out) && (dim % 8 == 0);
  DeviceStatus* st = device_status_ptr();
  UHFS_DISPATCH_DTYPE(dtype, embedding_fwd_kernel<T><<<row_grid(rows, 8), 256, 0, s>>>(
                                 ids, (const T*)tok, (const T*)pos, (T*)out, rows, dim, seq_len > 0 ? seq_len : 1, vec,
                                 vocab, st));
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

void embedding_bwd(int dtype, const int64_t* ids, const void* dout, float* dtok, float* dpos, int rows, int dim,
                   int seq_len, long long vocab, cudaStream_t s) {
  if (rows <= 0) return;
  const bool vec = al16(dout) && al16(dtok) && al16(dpos) && (dim % 8 == 0);
  DeviceStatus* st = device_status_ptr();
  UHFS_DISPATCH_DTYPE(dtype, embedding_bwd_kernel<T><<<row_grid(rows, 8), 256, 0, s>>>(
                                 ids, (const T*)dout, dtok, dpos, rows, dim, seq_len > 0 ? seq_len : 1, vec, vocab,
                                 st));
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

void softmax_ce_fwd_bwd(int dtype, const void* logits, long long ld, const int64_t* targets, float* loss_rows,
                        void* dlogits, int rows, int cols, float grad_scale, const float* grad_scale_ptr,
                        cudaStream_t s) {
  if (rows <= 0) return;
  const bool vec = al16(logits) && al16(dlogits) && (cols % 8 == 0) && (ld % 8 == 0);
  if (vec && dtype != DT_F32 && cols <= kCeThreads * 8 * kCeVecs) {
    if (dtype == DT_BF16)
      softmax_ce_reg_kernel<__nv_bfloat16><<<rows, kCeThreads, 0, s>>>(
          (const __nv_bfloat16*)logits, ld, targets, loss_rows, (__nv_bfloat16*)dlogits, cols, grad_scale,
          grad_scale_ptr, device_status_ptr());
    else
      softmax_ce_reg_kernel<__half><<<rows, kCeThreads, 0, s>>>((const __half*)logits, ld, targets, loss_rows,
                                                               (__half*)dlogits, cols, grad_scale, grad_scale_ptr,
                                                               device_status_ptr());
    note_launch();
    UHFS_CUDA_CHECK(cudaGetLastError());
    return;
  }
  DeviceStatus* st = device_status_ptr();
  UHFS_DISPATCH_DTYPE(dtype, softmax_ce_kernel<T><<<rows, kCeThreads, 0, s>>>(
                                 (const T*)logits, ld, targets, loss_rows, (T*)dlogits, cols, grad_scale, grad_scale_ptr,
                                 vec, st));
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

void softmax_rows(int dtype, const void* x, void* y, int rows, int cols, cudaStream_t s) {
  if (rows <= 0) return;
  UHFS_DISPATCH_DTYPE(dtype, softmax_rows_kernel<T><<<rows, kCeThreads, 0, s>>>((const T*)x, (T*)y, cols));
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

void softmax_rows_bwd(int dtype, const void* y, const void* dy, void* dx, int rows, int cols, cudaStream_t s) {
  if (rows <= 0) return;
  UHFS_DISPATCH_DTYPE(dtype, softmax_rows_bwd_kernel<T><<<rows, kCeThreads, 0, s>>>((const T*)y, (const T*)dy,
                                                                                     (T*)dx, cols));
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

}  // namespace uhfs
