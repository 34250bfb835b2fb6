// conv2d forward / data-gradient / weight-gradient as implicit GEMMs in exact
// fp32 (NCHW activations, KCRS weights: the reference's Conv2d contract).
//
// Reference: cuDNN cudnnConvolutionForward (IMPLICIT_PRECOMP_GEMM),
// cudnnConvolutionBackwardData (ALGO_1) and cudnnConvolutionBackwardFilter
// (ALGO_1) at cuda/kernels.cu:1093-1115, 1252-1265, 1395-1408.
//
// Each pass is one GEMM C[M, Nc] = sum_k A(m, k) B(k, n) whose operands are
// gathered on the fly from the activation / weight tensors (nothing is
// materialised):
//
//   mode   M           Nc          reduction    A(m, k)              B(k, n)
//   fwd    N*P*Q       K           C*R*S        x at (n,c,p*sh-ph+r, q*sw-pw+s)   w[n][k]
//   dgrad  N*H*W       C           K*R*S        dy at (n,k,(h+ph-r)/sh,(w+pw-s)/sw)  w[k][n][r][s]
//   wgrad  K           C*R*S       N*P*Q        dy[n][m][p][q]       x at (n,c,p*sh-ph+r, q*sw-pw+s)
//
// (dgrad's A is zero where the division is not exact or out of range.)
// Tiles of 128 x 64 outputs per 256-thread block, 8 x 4 per thread, k in
// steps of 8 through double-buffered shared memory with the next step's
// gathers in registers while the current step's 256 FMAs per thread run.
// The weight gradient reduces over every output pixel: it is split over
// blockIdx.z and accumulated with fp32 atomics into a zeroed dw.
#include <stdexcept>

#include "common.cuh"
#include "kernels.h"

namespace uhfs {

namespace {

constexpr int CBM = 128, CBN = 64, CBK = 8;
constexpr int kConvThreads = 256;

struct ConvGeom {
  int N, C, H, W, K, R, S, sh, sw, ph, pw, P, Q;
};

enum ConvMode { kFwd = 0, kDgrad = 1, kWgrad = 2 };

struct ConvArgs {
  ConvGeom g;
  const float* a;  // fwd: x, dgrad: dy, wgrad: dy
  const float* b;  // fwd: w, dgrad: w,  wgrad: x
  const float* bias;
  float* out;
  long long M, Nc, Kred;
  long long k_per_split;  // wgrad split-K chunk (multiple of CBK)
};

// Gather of A(m, kr) for one row m that a thread keeps fixed (fwd, dgrad).
struct RowPix {
  int n, y, x;   // fwd: n, p*sh - ph, q*sw - pw;  dgrad: n, h + ph, w + pw
  bool ok;
};

__device__ __forceinline__ RowPix row_pixel(const ConvGeom& g, int mode, long long m, long long M) {
  RowPix r{0, 0, 0, m < M};
  if (!r.ok) return r;
  if (mode == kFwd) {
    const int pq = g.P * g.Q;
    r.n = (int)(m / pq);
    const int rem = (int)(m - (long long)r.n * pq);
    const int p = rem / g.Q, q = rem - p * g.Q;
    r.y = p * g.sh - g.ph;
    r.x = q * g.sw - g.pw;
  } else {
    const int hw = g.H * g.W;
    r.n = (int)(m / hw);
    const int rem = (int)(m - (long long)r.n * hw);
    const int h = rem / g.W, w = rem - h * g.W;
    r.y = h + g.ph;
    r.x = w + g.pw;
  }
  return r;
}

// A(m, kr) for fwd / dgrad given the row's pixel and kr = (c|k, r, s).
__device__ __forceinline__ float load_a_row(const ConvArgs& a, int mode, const RowPix& px, int ch, int r, int s,
                                            bool kr_ok) {
  const ConvGeom& g = a.g;
  if (!px.ok || !kr_ok) return 0.f;
  if (mode == kFwd) {
    const int h = px.y + r, w = px.x + s;
    if (h < 0 || h >= g.H || w < 0 || w >= g.W) return 0.f;
    return __ldg(a.a + (((long long)px.n * g.C + ch) * g.H + h) * g.W + w);
  }
  // dgrad: output pixel p = (h + ph - r) / sh when exact and in range
  const int ty = px.y - r, tx = px.x - s;
  if (ty < 0 || tx < 0) return 0.f;
  const int p = ty / g.sh, q = tx / g.sw;
  if (p * g.sh != ty || q * g.sw != tx || p >= g.P || q >= g.Q) return 0.f;
  return __ldg(a.a + (((long long)px.n * g.K + ch) * g.P + p) * g.Q + q);
}

template <int MODE>
__global__ void __launch_bounds__(kConvThreads) conv_igemm_kernel(const ConvArgs a) {
  __shared__ __align__(16) float As[2][CBK][CBM + 4];
  __shared__ __align__(16) float Bs[2][CBK][CBN + 4];
  const ConvGeom& g = a.g;
  const int t = threadIdx.x;
  const long long m0 = (long long)blockIdx.x * CBM;
  const long long n0 = (long long)blockIdx.y * CBN;
  long long k_lo = 0, k_hi = a.Kred;
  if (MODE == kWgrad) {
    k_lo = (long long)blockIdx.z * a.k_per_split;
    k_hi = min(a.Kred, k_lo + a.k_per_split);
  }
  const int RS = g.R * g.S;

  // ---- per-thread gather assignment
  // fwd / dgrad: A column of 4 consecutive k for a fixed row; B 2 k x 1 col.
  // wgrad: A 4 rows x 1 k (k fastest across threads: consecutive pixels);
  //        B 2 cols x 1 k (k fastest).
  float ra[4], rb[2];
  RowPix px{};
  if (MODE != kWgrad) px = row_pixel(g, MODE, m0 + (t & (CBM - 1)), a.M);

  auto gather = [&](long long kb) {
    if constexpr (MODE != kWgrad) {
      // A: row t % 128, k = kb + (t / 128) * 4 + j
      long long kr = kb + (t >> 7) * 4;
      int ch = (int)(kr / RS), rem = (int)(kr - (long long)ch * RS);
      int r = rem / g.S, s = rem - r * g.S;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        ra[j] = load_a_row(a, MODE, px, ch, r, s, kr + j < k_hi);
        if (++s == g.S) {
          s = 0;
          if (++r == g.R) {
            r = 0;
            ++ch;
          }
        }
      }
      // B: col t % 64, k = kb + (t / 64) * 2 + j
      const long long col = n0 + (t & (CBN - 1));
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const long long k = kb + (t >> 6) * 2 + j;
        float v = 0.f;
        if (col < a.Nc && k < k_hi) {
          if (MODE == kFwd) {
            v = __ldg(a.b + col * a.Kred + k);  // w[K][C*R*S]
          } else {
            const int kk = (int)(k / RS), rr = (int)(k - (long long)kk * RS);
            v = __ldg(a.b + ((long long)kk * g.C + col) * RS + rr);  // w[k][c][r][s]
          }
        }
        rb[j] = v;
      }
    } else {
      // A: k = kb + t % 8 (a pixel (n, p, q)), rows m0 + (t / 8) * 4 + j
      const long long k = kb + (t & 7);
      const int pq = g.P * g.Q;
      const bool k_ok = k < k_hi;
      const int n = k_ok ? (int)(k / pq) : 0;
      const int rem = k_ok ? (int)(k - (long long)n * pq) : 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const long long m = m0 + (t >> 3) * 4 + j;
        ra[j] = (k_ok && m < a.M) ? __ldg(a.a + ((long long)n * g.K + m) * pq + rem) : 0.f;
      }
      // B: x at (n, c, p*sh-ph+r, q*sw-pw+s) for cols n0 + (t / 8) * 2 + j
      const int p = rem / g.Q, q = rem - (rem / g.Q) * g.Q;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const long long col = n0 + (t >> 3) * 2 + j;
        float v = 0.f;
        if (k_ok && col < a.Nc) {
          const int c = (int)(col / RS), rr = (int)(col - (long long)c * RS);
          const int r = rr / g.S, s = rr - r * g.S;
          const int h = p * g.sh - g.ph + r, w = q * g.sw - g.pw + s;
          if (h >= 0 && h < g.H && w >= 0 && w < g.W) v = __ldg(a.b + (((long long)n * g.C + c) * g.H + h) * g.W + w);
        }
        rb[j] = v;
      }
    }
  };
  auto stash = [&](int buf) {
    if constexpr (MODE != kWgrad) {
#pragma unroll
      for (int j = 0; j < 4; ++j) As[buf][(t >> 7) * 4 + j][t & (CBM - 1)] = ra[j];
#pragma unroll
      for (int j = 0; j < 2; ++j) Bs[buf][(t >> 6) * 2 + j][t & (CBN - 1)] = rb[j];
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) As[buf][t & 7][(t >> 3) * 4 + j] = ra[j];
#pragma unroll
      for (int j = 0; j < 2; ++j) Bs[buf][t & 7][(t >> 3) * 2 + j] = rb[j];
    }
  };

  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  const int ty = t >> 4, tx = t & 15;

  int buf = 0;
  if (k_lo < k_hi) {
    gather(k_lo);
    stash(0);
  }
  __syncthreads();
  for (long long kb = k_lo; kb < k_hi; kb += CBK) {
    const bool more = kb + CBK < k_hi;
    if (more) gather(kb + CBK);  // next step's loads in flight during the FMAs
#pragma unroll
    for (int kk = 0; kk < CBK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 8]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 8 + 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[4] = {b0.x, b0.y, b0.z, b0.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (more) {
      stash(buf ^ 1);
      __syncthreads();
      buf ^= 1;
    }
  }

  // ---- epilogue
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const long long m = m0 + ty * 8 + i;
    if (m >= a.M) break;
    if constexpr (MODE == kFwd) {
      const int pq = g.P * g.Q;
      const long long n = m / pq, rem = m - n * pq;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const long long col = n0 + tx * 4 + j;
        if (col < a.Nc)
          a.out[(n * g.K + col) * pq + rem] = acc[i][j] + (a.bias != nullptr ? __ldg(a.bias + col) : 0.f);
      }
    } else if constexpr (MODE == kDgrad) {
      const int hw = g.H * g.W;
      const long long n = m / hw, rem = m - n * hw;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const long long col = n0 + tx * 4 + j;
        if (col < a.Nc) a.out[(n * g.C + col) * hw + rem] = acc[i][j];
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const long long col = n0 + tx * 4 + j;
        if (col < a.Nc) atomicAdd(a.out + m * a.Nc + col, acc[i][j]);
      }
    }
  }
}

// db[k] = sum over (n, p, q) of dy[n][k][p][q]: one block per output channel.
__global__ void __launch_bounds__(256) conv_bias_grad_kernel(const float* __restrict__ dy, float* __restrict__ db,
                                                             int N, int K, int PQ) {
  const int k = blockIdx.x;
  float s = 0.f;
  for (int n = 0; n < N; ++n) {
    const float* row = dy + ((long long)n * K + k) * PQ;
    for (int i = threadIdx.x; i < PQ; i += blockDim.x) s += row[i];
  }
  s = warp_sum(s);
  __shared__ float part[8];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < 8 ? part[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) db[k] = v;
  }
}

ConvGeom geom(int N, int C, int H, int W, int K, int R, int S, int sh, int sw, int ph, int pw, int P, int Q) {
  if (N <= 0 || C <= 0 || H <= 0 || W <= 0 || K <= 0 || R <= 0 || S <= 0 || sh <= 0 || sw <= 0 || ph < 0 ||
      pw < 0 || P <= 0 || Q <= 0)
    throw std::invalid_argument("conv2d: non-positive size, stride or output extent");
  return ConvGeom{N, C, H, W, K, R, S, sh, sw, ph, pw, P, Q};
}

template <int MODE>
void launch(const ConvArgs& a, int splits, cudaStream_t s) {
  const long long gx = (a.M + CBM - 1) / CBM, gy = (a.Nc + CBN - 1) / CBN;
  if (gy > 65535 || gx > 0x7fffffffLL) throw std::runtime_error("conv2d: problem too large for one launch");
  conv_igemm_kernel<MODE><<<dim3((unsigned)gx, (unsigned)gy, (unsigned)splits), kConvThreads, 0, s>>>(a);
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

}  // namespace

void conv2d_fwd_f32(const float* x, const float* w, const float* b, float* y, int N, int C, int H, int W, int K,
                    int R, int S, int sh, int sw, int ph, int pw, int P, int Q, cudaStream_t s) {
  ConvArgs a{};
  a.g = geom(N, C, H, W, K, R, S, sh, sw, ph, pw, P, Q);
  a.a = x;
  a.b = w;
  a.bias = b;
  a.out = y;
  a.M = (long long)N * P * Q;
  a.Nc = K;
  a.Kred = (long long)C * R * S;
  launch<kFwd>(a, 1, s);
}

void conv2d_dgrad_f32(const float* dy, const float* w, float* dx, int N, int C, int H, int W, int K, int R, int S,
                      int sh, int sw, int ph, int pw, int P, int Q, cudaStream_t s) {
  ConvArgs a{};
  a.g = geom(N, C, H, W, K, R, S, sh, sw, ph, pw, P, Q);
  a.a = dy;
  a.b = w;
  a.out = dx;
  a.M = (long long)N * H * W;
  a.Nc = C;
  a.Kred = (long long)K * R * S;
  launch<kDgrad>(a, 1, s);
}

void conv2d_wgrad_f32(const float* dy, const float* x, float* dw, float* db, int N, int C, int H, int W, int K,
                      int R, int S, int sh, int sw, int ph, int pw, int P, int Q, cudaStream_t s) {
  ConvArgs a{};
  a.g = geom(N, C, H, W, K, R, S, sh, sw, ph, pw, P, Q);
  a.a = dy;
  a.b = x;
  a.out = dw;
  a.M = K;
  a.Nc = (long long)C * R * S;
  a.Kred = (long long)N * P * Q;
  // split the pixel reduction so the grid covers the SMs about twice
  const long long tiles = ((a.Nc + CBN - 1) / CBN) * ((a.M + CBM - 1) / CBM);
  long long splits = (2 * 148 + tiles - 1) / tiles;
  const long long max_splits = (a.Kred + 4 * CBK - 1) / (4 * CBK);  // at least 4 k-steps per split
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  if (splits > 65535) splits = 65535;
  long long per = (a.Kred + splits - 1) / splits;
  per = (per + CBK - 1) / CBK * CBK;
  splits = (a.Kred + per - 1) / per;
  a.k_per_split = per;
  UHFS_CUDA_CHECK(cudaMemsetAsync(dw, 0, sizeof(float) * (size_t)(a.M * a.Nc), s));
  launch<kWgrad>(a, (int)splits, s);
  if (db != nullptr) {
    conv_bias_grad_kernel<<<K, 256, 0, s>>>(dy, db, N, K, P * Q);
    note_launch();
    UHFS_CUDA_CHECK(cudaGetLastError());
  }
}

}  // namespace uhfs
