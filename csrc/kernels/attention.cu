// Multi-head flash attention forward / backward, bf16 in, fp32 softmax
// statistics, causal or full, head dim 64 or 128.
//
// Reference: the single-head O(T^2 F^2) fp32 kernel at cuda/kernels.cu:147-188
// (inference only; training attention is Python autograd, nn.py:229-271).
// This file is the first sm_100a implementation: FlashAttention-2 style
// tiling (online softmax, LSE saved, recompute in backward) on the warp-level
// mma.sync m16n8k16 tensor-core path, cp.async double-buffered tiles, XOR
// swizzled shared memory, memory O(T).  Q/K/V/O are addressed as [B, T, H, D]
// rows with arbitrary batch/token strides, so the fused QKV projection output
// [B*T, 3*H*D] is consumed in place.
#include <cstdlib>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace uhfs {

namespace {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm4(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm4t(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Byte offset of element (row, col) in a swizzled [rows][D] bf16 tile; col % 8 == 0.
template <int D>
__device__ __forceinline__ uint32_t swz(int row, int col) {
  return row * (D * 2) + ((((col >> 3) ^ (row & 7))) << 4);
}

// Load `rows` rows of D bf16 (global row stride `stride` elements) into a swizzled tile.
template <int D, int NT>
__device__ __forceinline__ void load_tile(uint32_t sbase, const __nv_bfloat16* g, long long stride, int rows,
                                          int valid_rows) {
  constexpr int CH = D / 8;
  for (int idx = threadIdx.x; idx < rows * CH; idx += NT) {
    const int r = idx / CH, c = idx % CH;
    const bool ok = r < valid_rows;
    const __nv_bfloat16* src = g + (long long)(ok ? r : 0) * stride + c * 8;
    cp_async16(sbase + swz<D>(r, c * 8), src, ok);
  }
}

// ------------------------------------------------------------------ forward
template <int D>
__global__ void __launch_bounds__(256) fa_fwd_kernel(const AttnParams p) {
  constexpr int BM = 128, BN = 64, NT = 256;
  constexpr int TILE_Q = BM * D * 2, TILE_KV = BN * D * 2;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + TILE_Q;
  const uint32_t sV0 = sK0 + 2 * TILE_KV;

  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int m_block = gridDim.x - 1 - blockIdx.x;  // longest causal rows first
  const int m0 = m_block * BM;
  const int T = p.T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  const __nv_bfloat16* qg = p.q + b * p.q_stride_b + (long long)m0 * p.q_stride_t + h * D;
  const __nv_bfloat16* kg = p.k + b * p.k_stride_b + h * D;
  const __nv_bfloat16* vg = p.v + b * p.v_stride_b + h * D;

  const int n_end = p.causal ? min(T, m0 + BM) : T;
  const int n_blocks = (n_end + BN - 1) / BN;

  load_tile<D, NT>(sQ, qg, p.q_stride_t, BM, T - m0);
  cp_commit();
  load_tile<D, NT>(sK0, kg, p.k_stride_t, BN, T);
  load_tile<D, NT>(sV0, vg, p.v_stride_t, BN, T);
  cp_commit();

  cp_wait<1>();
  __syncthreads();
  uint32_t qf[D / 16][4];
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int row = warp * 16 + (lane & 15);
    const int col = kk * 16 + (lane >> 4) * 8;
    ldsm4(qf[kk], sQ + swz<D>(row, col));
  }

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const float sl2 = p.scale * kLog2e;
  const int q_row0 = m0 + warp * 16 + g;

  for (int j = 0; j < n_blocks; ++j) {
    const int buf = j & 1;
    if (j + 1 < n_blocks) {
      const int nb = (j + 1) * BN;
      load_tile<D, NT>(sK0 + (buf ^ 1) * TILE_KV, kg + (long long)nb * p.k_stride_t, p.k_stride_t, BN, T - nb);
      load_tile<D, NT>(sV0 + (buf ^ 1) * TILE_KV, vg + (long long)nb * p.v_stride_t, p.v_stride_t, BN, T - nb);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    const uint32_t sK = sK0 + buf * TILE_KV, sV = sV0 + buf * TILE_KV;
    const int n0 = j * BN;

    float s[BN / 8][4];
#pragma unroll
    for (int i = 0; i < BN / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int jj = 0; jj < BN / 16; ++jj) {
        uint32_t bf[4];
        const int key = jj * 16 + (lane >> 4) * 8 + (lane & 7);
        const int col = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm4(bf, sK + swz<D>(key, col));
        mma16816(s[2 * jj], qf[kk], bf[0], bf[1]);
        mma16816(s[2 * jj + 1], qf[kk], bf[2], bf[3]);
      }
    }
    // scale into log2 domain, mask
    const bool need_mask = (p.causal && n0 + BN - 1 > m0 + warp * 16) || (n0 + BN > T);
#pragma unroll
    for (int i = 0; i < BN / 8; ++i) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = s[i][e] * sl2;
        if (need_mask) {
          const int key = n0 + i * 8 + 2 * t + (e & 1);
          const int q = q_row0 + (e >> 1) * 8;
          if (key >= T || (p.causal && key > q)) v = -INFINITY;
        }
        s[i][e] = v;
      }
    }
    // online softmax for rows g (e=0,1) and g+8 (e=2,3)
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < BN / 8; ++i) mx = fmaxf(mx, fmaxf(s[i][2 * r], s[i][2 * r + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(mrow[r], mx);
      const float base = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = exp2f(mrow[r] - base);
      mrow[r] = m_new;
      float ls = 0.f;
#pragma unroll
      for (int i = 0; i < BN / 8; ++i) {
        s[i][2 * r] = exp2f(s[i][2 * r] - base);
        s[i][2 * r + 1] = exp2f(s[i][2 * r + 1] - base);
        ls += s[i][2 * r] + s[i][2 * r + 1];
      }
      lrow[r] = lrow[r] * alpha + ls;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        o[i][2 * r] *= alpha;
        o[i][2 * r + 1] *= alpha;
      }
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dj = 0; dj < D / 16; ++dj) {
        uint32_t bf[4];
        const int key = kk * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
        const int col = dj * 16 + (lane >> 4) * 8;
        ldsm4t(bf, sV + swz<D>(key, col));
        mma16816(o[2 * dj], pa, bf[0], bf[1]);
        mma16816(o[2 * dj + 1], pa, bf[2], bf[3]);
      }
    }
    __syncthreads();
  }

  // finalize: O / l, LSE (log2 domain)
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float l = lrow[r];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const float inv = l > 0.f ? 1.0f / l : 0.f;
    const int q = q_row0 + r * 8;
    if (q < T) {
      __nv_bfloat16* og = p.o + b * p.o_stride_b + (long long)q * p.o_stride_t + h * D;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        *reinterpret_cast<uint32_t*>(og + i * 8 + 2 * t) = pack_bf16(o[i][2 * r] * inv, o[i][2 * r + 1] * inv);
      }
      if (t == 0) p.lse[(long long)bh * T + q] = (l > 0.f) ? (mrow[r] + log2f(l)) : INFINITY;
    }
  }
}

// --------------------------------------------------------- backward helpers
// delta[b,h,t] = sum_d dO * O ; dq_accum zeroed.  Eight elements per thread
// (16-byte loads), D/8 threads per (b, t, h) row.
template <int D>
__global__ void __launch_bounds__(256) fa_bwd_prep_kernel(const AttnBwdParams p) {
  constexpr int TPR = D / 8;  // threads per row
  const long long rows = (long long)p.f.B * p.f.T * p.f.H;
  const int sub = threadIdx.x % TPR;
  const long long stride = (long long)gridDim.x * (blockDim.x / TPR);
  for (long long r = blockIdx.x * (long long)(blockDim.x / TPR) + threadIdx.x / TPR; r < rows; r += stride) {
    const int h = r % p.f.H;
    const int tt = (r / p.f.H) % p.f.T;
    const int b = r / ((long long)p.f.H * p.f.T);
    const uint4 ov = *reinterpret_cast<const uint4*>(p.f.o + b * p.f.o_stride_b + (long long)tt * p.f.o_stride_t +
                                                     h * D + sub * 8);
    const uint4 dv = *reinterpret_cast<const uint4*>(p.dout + b * p.do_stride_b + (long long)tt * p.do_stride_t +
                                                     h * D + sub * 8);
    const __nv_bfloat162* o2 = reinterpret_cast<const __nv_bfloat162*>(&ov);
    const __nv_bfloat162* d2 = reinterpret_cast<const __nv_bfloat162*>(&dv);
    float acc = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 a = __bfloat1622float2(o2[e]), c = __bfloat1622float2(d2[e]);
      acc = fmaf(a.x, c.x, fmaf(a.y, c.y, acc));
    }
#pragma unroll
    for (int o = TPR / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (sub == 0) p.delta[((long long)b * p.f.H + h) * p.f.T + tt] = acc;
    float4* dq = reinterpret_cast<float4*>(p.dq_accum + r * D + sub * 8);
    dq[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    dq[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// dq (bf16, strided into the fused gradient) = scale * dq_accum; 8 elements per thread.
template <int D>
__global__ void __launch_bounds__(256) fa_bwd_dq_convert_kernel(const AttnBwdParams p) {
  const long long total = (long long)p.f.B * p.f.T * p.f.H * (D / 8);
  const float sc = p.f.scale;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int d8 = (int)(i % (D / 8)) * 8;
    const long long r = i / (D / 8);
    const int h = r % p.f.H;
    const int tt = (r / p.f.H) % p.f.T;
    const int b = r / ((long long)p.f.H * p.f.T);
    const float4* src = reinterpret_cast<const float4*>(p.dq_accum + r * D + d8);
    const float4 x = src[0], y = src[1];
    uint4 out;
    out.x = pack_bf16(x.x * sc, x.y * sc);
    out.y = pack_bf16(x.z * sc, x.w * sc);
    out.z = pack_bf16(y.x * sc, y.y * sc);
    out.w = pack_bf16(y.z * sc, y.w * sc);
    *reinterpret_cast<uint4*>(p.dq + b * p.dq_stride_b + (long long)tt * p.dq_stride_t + h * D + d8) = out;
  }
}

// ----------------------------------------------------------------- backward
// One CTA per (64-key block, b, h); 4 warps own 16 keys each and loop over
// 64-query blocks.  dK, dV accumulate in registers; dQ is accumulated in fp32
// global memory with vector atomics.
template <int D>
__global__ void __launch_bounds__(128) fa_bwd_kernel(const AttnBwdParams p) {
  constexpr int BN = 64, BQ = 64, NT = 128;
  constexpr int TILE = 64 * D * 2;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + TILE;
  const uint32_t sQ0 = sV + TILE;           // 2 buffers
  const uint32_t sdO0 = sQ0 + 2 * TILE;     // 2 buffers
  const uint32_t sdS = sdO0 + 2 * TILE;     // [64 keys][64 q] bf16, swizzled with D=64 geometry
  float* sLse = reinterpret_cast<float*>(smem + 6 * TILE + 64 * 64 * 2);  // [2][64]
  float* sDel = sLse + 2 * BQ;                                           // [2][64]

  const AttnParams& f = p.f;
  const int bh = blockIdx.y;
  const int b = bh / f.H, h = bh % f.H;
  const int n0 = blockIdx.x * BN;
  const int T = f.T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const float sl2 = f.scale * kLog2e;

  const __nv_bfloat16* kg = f.k + b * f.k_stride_b + (long long)n0 * f.k_stride_t + h * D;
  const __nv_bfloat16* vg = f.v + b * f.v_stride_b + (long long)n0 * f.v_stride_t + h * D;
  const __nv_bfloat16* qg = f.q + b * f.q_stride_b + h * D;
  const __nv_bfloat16* dog = p.dout + b * p.do_stride_b + h * D;
  const float* lse_g = f.lse + (long long)bh * T;
  const float* del_g = p.delta + (long long)bh * T;

  load_tile<D, NT>(sK, kg, f.k_stride_t, BN, T - n0);
  load_tile<D, NT>(sV, vg, f.v_stride_t, BN, T - n0);
  cp_commit();

  const int i_start = f.causal ? (n0 / BQ) : 0;
  const int i_end = (T + BQ - 1) / BQ;

  auto prefetch = [&](int i, int buf) {
    const int q0 = i * BQ;
    load_tile<D, NT>(sQ0 + buf * TILE, qg + (long long)q0 * f.q_stride_t, f.q_stride_t, BQ, T - q0);
    load_tile<D, NT>(sdO0 + buf * TILE, dog + (long long)q0 * p.do_stride_t, p.do_stride_t, BQ, T - q0);
    for (int x = threadIdx.x; x < BQ; x += NT) {
      const int q = q0 + x;
      sLse[buf * BQ + x] = q < T ? lse_g[q] : INFINITY;
      sDel[buf * BQ + x] = q < T ? del_g[q] : 0.f;
    }
  };
  if (i_start < i_end) prefetch(i_start, 0);
  cp_commit();
  cp_wait<1>();
  __syncthreads();

  float dk[D / 8][4], dv[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;

  const int key_r0 = n0 + warp * 16 + g;  // keys of this thread: key_r0, key_r0 + 8

  for (int i = i_start; i < i_end; ++i) {
    const int buf = (i - i_start) & 1;
    if (i + 1 < i_end) prefetch(i + 1, buf ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    const uint32_t sQ = sQ0 + buf * TILE, sdO = sdO0 + buf * TILE;
    const float* lse = sLse + buf * BQ;
    const float* del = sDel + buf * BQ;
    const int q0 = i * BQ;

    // S^T = K_w Q^T and dP^T = V_w dO^T  (16 keys x 64 queries per warp)
    float st[BQ / 8][4], dpt[BQ / 8][4];
#pragma unroll
    for (int x = 0; x < BQ / 8; ++x)
#pragma unroll
      for (int e = 0; e < 4; ++e) st[x][e] = dpt[x][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t kf[4], vf[4];
      {
        const int row = warp * 16 + (lane & 15);
        const int col = kk * 16 + (lane >> 4) * 8;
        ldsm4(kf, sK + swz<D>(row, col));
        ldsm4(vf, sV + swz<D>(row, col));
      }
#pragma unroll
      for (int jj = 0; jj < BQ / 16; ++jj) {
        uint32_t bq[4], bo[4];
        const int q = jj * 16 + (lane >> 4) * 8 + (lane & 7);
        const int col = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm4(bq, sQ + swz<D>(q, col));
        ldsm4(bo, sdO + swz<D>(q, col));
        mma16816(st[2 * jj], kf, bq[0], bq[1]);
        mma16816(st[2 * jj + 1], kf, bq[2], bq[3]);
        mma16816(dpt[2 * jj], vf, bo[0], bo[1]);
        mma16816(dpt[2 * jj + 1], vf, bo[2], bo[3]);
      }
    }
    // P^T and dS^T
    const bool diag = f.causal && (q0 < n0 + BN);
#pragma unroll
    for (int x = 0; x < BQ / 8; ++x) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ql = x * 8 + 2 * t + (e & 1);
        const int key = key_r0 + (e >> 1) * 8;
        float pv = exp2f(st[x][e] * sl2 - lse[ql]);
        if (diag && key > q0 + ql) pv = 0.f;
        st[x][e] = pv;
        dpt[x][e] = pv * (dpt[x][e] - del[ql]);
      }
    }
    // dV += P^T dO ; dK += dS^T Q
#pragma unroll
    for (int kk = 0; kk < BQ / 16; ++kk) {
      uint32_t pa[4], da[4];
      pa[0] = pack_bf16(st[2 * kk][0], st[2 * kk][1]);
      pa[1] = pack_bf16(st[2 * kk][2], st[2 * kk][3]);
      pa[2] = pack_bf16(st[2 * kk + 1][0], st[2 * kk + 1][1]);
      pa[3] = pack_bf16(st[2 * kk + 1][2], st[2 * kk + 1][3]);
      da[0] = pack_bf16(dpt[2 * kk][0], dpt[2 * kk][1]);
      da[1] = pack_bf16(dpt[2 * kk][2], dpt[2 * kk][3]);
      da[2] = pack_bf16(dpt[2 * kk + 1][0], dpt[2 * kk + 1][1]);
      da[3] = pack_bf16(dpt[2 * kk + 1][2], dpt[2 * kk + 1][3]);
#pragma unroll
      for (int dj = 0; dj < D / 16; ++dj) {
        uint32_t bo[4], bq[4];
        const int q = kk * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
        const int col = dj * 16 + (lane >> 4) * 8;
        ldsm4t(bo, sdO + swz<D>(q, col));
        ldsm4t(bq, sQ + swz<D>(q, col));
        mma16816(dv[2 * dj], pa, bo[0], bo[1]);
        mma16816(dv[2 * dj + 1], pa, bo[2], bo[3]);
        mma16816(dk[2 * dj], da, bq[0], bq[1]);
        mma16816(dk[2 * dj + 1], da, bq[2], bq[3]);
      }
    }
    // stash dS^T (rows = keys, cols = queries) for the dQ product
#pragma unroll
    for (int x = 0; x < BQ / 8; ++x) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int krow = warp * 16 + g + r * 8;
        const int qc = x * 8 + 2 * t;
        const uint32_t addr = sdS + swz<64>(krow, x * 8) + (2 * t) * 2;
        asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(pack_bf16(dpt[x][2 * r], dpt[x][2 * r + 1])) : "memory");
        (void)qc;
      }
    }
    __syncthreads();
    // dQ[q, :] += dS[q, keys] K[keys, :]   (warp owns 16 queries)
    {
      float dq[D / 8][4];
#pragma unroll
      for (int x = 0; x < D / 8; ++x) dq[x][0] = dq[x][1] = dq[x][2] = dq[x][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk) {
        uint32_t a[4];
        {
          const int mi = lane >> 3;
          const int krow = kk * 16 + (mi >> 1) * 8 + (lane & 7);
          const int qcol = warp * 16 + (mi & 1) * 8;
          ldsm4t(a, sdS + swz<64>(krow, qcol));
        }
#pragma unroll
        for (int dj = 0; dj < D / 16; ++dj) {
          uint32_t bk[4];
          const int key = kk * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
          const int col = dj * 16 + (lane >> 4) * 8;
          ldsm4t(bk, sK + swz<D>(key, col));
          mma16816(dq[2 * dj], a, bk[0], bk[1]);
          mma16816(dq[2 * dj + 1], a, bk[2], bk[3]);
        }
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int q = q0 + warp * 16 + g + r * 8;
        if (q < T) {
          float* dst = p.dq_accum + (((long long)b * T + q) * f.H + h) * D;
#pragma unroll
          for (int x = 0; x < D / 8; ++x)
            atomicAdd(reinterpret_cast<float2*>(dst + x * 8 + 2 * t), make_float2(dq[x][2 * r], dq[x][2 * r + 1]));
        }
      }
    }
    __syncthreads();
  }

  // write dK (scaled) and dV
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int key = key_r0 + r * 8;
    if (key < T) {
      __nv_bfloat16* dkg = p.dk + b * p.dk_stride_b + (long long)key * p.dk_stride_t + h * D;
      __nv_bfloat16* dvg = p.dv + b * p.dv_stride_b + (long long)key * p.dv_stride_t + h * D;
#pragma unroll
      for (int x = 0; x < D / 8; ++x) {
        *reinterpret_cast<uint32_t*>(dkg + x * 8 + 2 * t) = pack_bf16(dk[x][2 * r] * f.scale, dk[x][2 * r + 1] * f.scale);
        *reinterpret_cast<uint32_t*>(dvg + x * 8 + 2 * t) = pack_bf16(dv[x][2 * r], dv[x][2 * r + 1]);
      }
    }
  }
}

template <int D>
void fwd_impl(const AttnParams& p, cudaStream_t s) {
  constexpr int smem = 128 * D * 2 + 4 * 64 * D * 2;
  static PerDeviceOnce once;
  once([] {
    UHFS_CUDA_CHECK(cudaFuncSetAttribute(fa_fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  });
  dim3 grid((p.T + 127) / 128, p.B * p.H);
  fa_fwd_kernel<D><<<grid, 256, smem, s>>>(p);
  note_launch();
}

template <int D>
void bwd_impl(const AttnBwdParams& p, cudaStream_t s) {
  constexpr int smem = 6 * 64 * D * 2 + 64 * 64 * 2 + 4 * 64 * 4;
  static PerDeviceOnce once;
  once([] {
    UHFS_CUDA_CHECK(cudaFuncSetAttribute(fa_bwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  });
  const long long rows = (long long)p.f.B * p.f.T * p.f.H;
  const long long rows_per_block = 256 / (D / 8);
  int g1 = (int)((rows + rows_per_block - 1) / rows_per_block);
  if (g1 > 148 * 16) g1 = 148 * 16;
  fa_bwd_prep_kernel<D><<<g1, 256, 0, s>>>(p);
  note_launch();
  static const bool legacy = [] {
    const char* e = getenv("UHFS_ATTN_BWD");
    return e != nullptr && std::string(e) == "mma_sync";
  }();
  if (!legacy && flash_attn_bwd_tc_supported(p)) {
    flash_attn_bwd_tc_main(p, s);
  } else {
    dim3 grid((p.f.T + 63) / 64, p.f.B * p.f.H);
    fa_bwd_kernel<D><<<grid, 128, smem, s>>>(p);
    note_launch();
  }
  long long tot = rows * (D / 8);
  int g2 = (int)((tot + 255) / 256);
  if (g2 > 148 * 16) g2 = 148 * 16;
  fa_bwd_dq_convert_kernel<D><<<g2, 256, 0, s>>>(p);
  note_launch();
}

}  // namespace

void flash_attn_fwd(const AttnParams& p, cudaStream_t s) {
  if (p.T <= 0 || p.B <= 0 || p.H <= 0) return;
  static const bool legacy = [] {
    const char* e = getenv("UHFS_ATTN_FWD");
    return e != nullptr && std::string(e) == "mma_sync";
  }();
  if (!legacy && flash_attn_fwd_tc_supported(p)) {
    flash_attn_fwd_tc(p, s);
    return;
  }
  if (p.D == 64) fwd_impl<64>(p, s);
  else if (p.D == 128) fwd_impl<128>(p, s);
  else throw std::runtime_error("flash attention supports head_dim 64 or 128");
  UHFS_CUDA_CHECK(cudaGetLastError());
}

void flash_attn_bwd(const AttnBwdParams& p, cudaStream_t s) {
  if (p.f.T <= 0 || p.f.B <= 0 || p.f.H <= 0) return;
  // the delta / dQ helper kernels move 8 elements per 16-byte access
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  if (!al16(p.f.o) || !al16(p.dout) || !al16(p.dq) || !al16(p.dq_accum) || p.f.o_stride_t % 8 != 0 ||
      p.f.o_stride_b % 8 != 0 || p.do_stride_t % 8 != 0 || p.do_stride_b % 8 != 0 || p.dq_stride_t % 8 != 0 ||
      p.dq_stride_b % 8 != 0)
    throw std::runtime_error("flash attention backward: o / dout / dq need 16-byte aligned rows");
  if (p.f.D == 64) bwd_impl<64>(p, s);
  else if (p.f.D == 128) bwd_impl<128>(p, s);
  else throw std::runtime_error("flash attention supports head_dim 64 or 128");
  UHFS_CUDA_CHECK(cudaGetLastError());
}

}  // namespace uhfs
