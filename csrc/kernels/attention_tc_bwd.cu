// Flash-attention backward on the 5th-generation tensor core (tcgen05 + TMEM).
//
// One CTA owns a block of 128 keys of one (batch, head) and loops over the
// 128-query blocks that attend to it (causal: from the diagonal on).
//
//   warp 0      TMA producer: K, V once; Q_i, dO_i per query block (ring),
//               plus lse_i / delta_i into shared memory
//   warp 1      TMEM allocator + MMA issuer (one elected thread), per block i:
//                 S^T  = K Q_i^T           M=128 keys, N=128 queries, K=D
//                 dP^T = V dO_i^T          (same shape)
//                 dV  += P^T dO_i          M=128 keys, N=D, K=128 queries
//                 dK  += dS^T Q_i          (same)
//                 dQ_i = dS K              M=128 queries, N=D, K=128 keys
//               (dS is read MN-major from the dS^T tile; dO_i, Q_i and K are
//               read MN-major as the B operands of the last three products)
//   warps 2..9  two warpgroups; TMEM lane r (warp%4 picks the lane quarter)
//               is key row r and warpgroup g takes query columns
//               [64g, 64g+64): P^T = exp2(S^T*scale*log2e - lse),
//               dS^T = P^T (dP^T - delta), both written as bf16 into the
//               swizzled shared tiles (warpgroup g fills sub-tile g); then
//               lane r takes query row r, columns [gD/2, gD/2+D/2) of dQ_i
//               from TMEM and adds them into the fp32 dQ accumulator in
//               global memory (vector reductions); at the end the same split
//               stores dK (scaled) and dV.
//
// TMEM: S^T [0,128), dP^T [128,256), dV, dK, dQ after that (dQ reuses the
// S^T columns when D = 128).  Every wait is bounded.
#include <cudaTypedefs.h>

#include <stdexcept>

#include "common.cuh"
#include "kernels.h"

namespace uhfs {

CUtensorMap make_tmap_bf16_2d(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                              uint32_t box_inner, uint32_t box_outer);

namespace {

constexpr int BK = 128;  // keys per CTA
constexpr int BQ = 128;  // queries per step
constexpr int kCompute = 256;  // warps 2..9
constexpr int kThreads = 64 + kCompute;
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct BwdCfg {
  static constexpr int kTile = 128 * D * 2;          // one [128][D] bf16 tile (D/64 swizzled sub-tiles)
  static constexpr int kStages = (D == 64) ? 2 : 1;  // Q_i / dO_i ring depth
  static constexpr int kStageBytes = 2 * kTile;      // Q_i | dO_i
  static constexpr int kPT = BK * BQ * 2;            // P^T or dS^T tile (2 sub-tiles of 128 x 64)
  static constexpr int kVec = 2 * BQ * 4;            // lse_i | delta_i
  static constexpr int kSmem = 1024 + 2 * kTile + kStages * kStageBytes + 2 * kPT + kStages * kVec + 256;
  static constexpr uint32_t kST = 0, kDPT = 128, kDV = 256, kDK = 256 + D;
  static constexpr uint32_t kDQ = (D == 64) ? 256 + 2 * D : 0;  // D=128: reuse S^T columns
  static constexpr uint32_t kCols = 512;
};

struct BwdArgs {
  int B, H, T;
  long long F;
  float sl2, scale;
  int causal;
  const float* lse;     // [B, H, T] log2 domain
  const float* delta;   // [B, H, T]
  float* dq_accum;      // [B, T, H, D] fp32
  __nv_bfloat16* dqkv;  // [B*T, 3F]
  DeviceStatus* status;
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    fa_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
                     const BwdArgs a) {
  using Cfg = BwdCfg<D>;
  constexpr int KD = D / 64;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + Cfg::kTile;
  uint8_t* sQD = sV + Cfg::kTile;                 // [S][Q | dO]
  uint8_t* sPT = sQD + S * Cfg::kStageBytes;      // P^T
  uint8_t* sDST = sPT + Cfg::kPT;                 // dS^T
  float* sVec = reinterpret_cast<float*>(sDST + Cfg::kPT);  // [S][lse(128) | delta(128)]
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sVec) + S * Cfg::kVec);
  uint64_t* kv_full = bars;          // 1
  uint64_t* qd_full = bars + 1;      // [2]
  uint64_t* qd_empty = bars + 3;     // [2]
  uint64_t* s_full = bars + 5;       // S^T and dP^T ready
  uint64_t* s_free = bars + 6;       // S^T / dP^T read by all 128 threads
  uint64_t* p_full = bars + 7;       // P^T / dS^T written
  uint64_t* dq_full = bars + 8;      // dQ_i ready (all MMAs of step i done)
  uint64_t* dq_free = bars + 9;      // dQ_i read
  uint64_t* done = bars + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y;
  const int b = bh / a.H, h = bh % a.H;
  const int n_block = blockIdx.x;
  const int n0 = n_block * BK;
  const int T = a.T;
  const int i_start = a.causal ? n0 / BQ : 0;
  const int i_end = (T + BQ - 1) / BQ;
  const int steps = i_end - i_start;
  const int row0 = b * T;

  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_qkv);
    tma_prefetch_desc(&tm_do);
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, kCompute);
    mbar_init(p_full, kCompute);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, kCompute);
    mbar_init(done, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    bool issued[2] = {false, false};
    uint32_t iph[2] = {0, 0};
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 2 * Cfg::kTile);
      for (int kd = 0; kd < KD; ++kd) {
        tma_load_2d(sK + kd * (BK * 128), &tm_qkv, kv_full, (int)(a.F + h * D + kd * 64), row0 + n0);
        tma_load_2d(sV + kd * (BK * 128), &tm_qkv, kv_full, (int)(2 * a.F + h * D + kd * 64), row0 + n0);
      }
    }
    bool ok = true;
    for (int t = 0; t < steps && ok; ++t) {
      const int st = t % S;
      const uint32_t ph = (t / S) & 1;
      int good = 1;
      if (lane == 0) good = mbar_wait_bounded(&qd_empty[st], ph ^ 1u, a.status, kErrWaitTimeoutEmpty, 300);
      good = __shfl_sync(0xffffffffu, good, 0);
      if (!good) {
        ok = false;
        break;
      }
      const int q0 = (i_start + t) * BQ;
      // lse / delta of this query block (generic stores, ordered by the barrier arrive)
      float* vec = sVec + st * (2 * BQ);
      for (int x = lane; x < BQ; x += 32) {
        const int qq = q0 + x;
        vec[x] = qq < T ? a.lse[(long long)bh * T + qq] : INFINITY;
        vec[BQ + x] = qq < T ? a.delta[(long long)bh * T + qq] : 0.f;
      }
      __syncwarp();
      if (lane == 0) {
        uint8_t* sQ = sQD + st * Cfg::kStageBytes;
        uint8_t* sDO = sQ + Cfg::kTile;
        mbar_arrive_expect_tx(&qd_full[st], 2 * Cfg::kTile);
        for (int kd = 0; kd < KD; ++kd) {
          tma_load_2d(sQ + kd * (BQ * 128), &tm_qkv, &qd_full[st], (int)(h * D + kd * 64), row0 + q0);
          tma_load_2d(sDO + kd * (BQ * 128), &tm_do, &qd_full[st], (int)(h * D + kd * 64), row0 + q0);
        }
        issued[st] = true;
        iph[st] = ph;
      }
    }
    if (lane == 0) {
      mbar_wait_bounded(kv_full, 0, a.status, kErrWaitTimeoutFull, 301);
      for (int s2 = 0; s2 < S; ++s2)
        if (issued[s2]) mbar_wait_bounded(&qd_full[s2], iph[s2], a.status, kErrWaitTimeoutFull, 302);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one_sync()) {
      constexpr uint32_t id_s = make_idesc(1, 0, 0, BK, BQ);   // K / V K-major, Q / dO K-major
      constexpr uint32_t id_kv = make_idesc(1, 0, 1, BK, D);   // P^T / dS^T K-major, dO / Q MN-major
      constexpr uint32_t id_q = make_idesc(1, 1, 1, BQ, D);    // dS MN-major, K MN-major
      bool ok = mbar_wait_bounded(kv_full, 0, a.status, kErrWaitTimeoutFull, 310);
      const uint32_t k_base = smem_u32(sK), v_base = smem_u32(sV);
      const uint32_t pt_base = smem_u32(sPT), dst_base = smem_u32(sDST);
      for (int t = 0; t < steps && ok; ++t) {
        const int st = t % S;
        const uint32_t ph = (t / S) & 1;
        const uint32_t tp = t & 1;
        if (!mbar_wait_bounded(&qd_full[st], ph, a.status, kErrWaitTimeoutFull, 311) ||
            !mbar_wait_bounded(s_free, tp ^ 1u, a.status, kErrWaitTimeoutAccum, 312)) {
          ok = false;
          break;
        }
        if (D == 128 && t > 0 && !mbar_wait_bounded(dq_free, (t - 1) & 1, a.status, kErrWaitTimeoutAccum, 313)) {
          ok = false;  // dQ shares the S^T columns when D = 128
          break;
        }
        tc_fence_after();
        const uint32_t q_base = smem_u32(sQD + st * Cfg::kStageBytes);
        const uint32_t do_base = q_base + Cfg::kTile;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
          tc_mma_f16(tmem + Cfg::kST, make_smem_desc(k_base + off, 16, 1024, kSwizzle128B),
                     make_smem_desc(q_base + off, 16, 1024, kSwizzle128B), id_s, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
          tc_mma_f16(tmem + Cfg::kDPT, make_smem_desc(v_base + off, 16, 1024, kSwizzle128B),
                     make_smem_desc(do_base + off, 16, 1024, kSwizzle128B), id_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(s_full);
        if (!mbar_wait_bounded(p_full, tp, a.status, kErrWaitTimeoutAccum, 314)) {
          ok = false;
          break;
        }
        if (D == 64 && t > 0 && !mbar_wait_bounded(dq_free, (t - 1) & 1, a.status, kErrWaitTimeoutAccum, 315)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // dV += P^T dO ; dK += dS^T Q    (K = 128 queries: sub-tile kk>>2 of the P^T / dS^T tiles)
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {
          const uint32_t aoff = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
          const uint64_t bdo = make_smem_desc(do_base + kk * 16 * 128, BQ * 128, 1024, kSwizzle128B);
          const uint64_t bq = make_smem_desc(q_base + kk * 16 * 128, BQ * 128, 1024, kSwizzle128B);
          const uint32_t acc = (t > 0 || kk > 0) ? 1u : 0u;
          tc_mma_f16(tmem + Cfg::kDV, make_smem_desc(pt_base + aoff, 16, 1024, kSwizzle128B), bdo, id_kv, acc);
          tc_mma_f16(tmem + Cfg::kDK, make_smem_desc(dst_base + aoff, 16, 1024, kSwizzle128B), bq, id_kv, acc);
        }
        // dQ_i = dS K  (A = dS^T read MN-major: 64-query chunks are the two sub-tiles)
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t ad = make_smem_desc(dst_base + kk * 16 * 128, BK * 128, 1024, kSwizzle128B);
          const uint64_t bd = make_smem_desc(k_base + kk * 16 * 128, BK * 128, 1024, kSwizzle128B);
          tc_mma_f16(tmem + Cfg::kDQ, ad, bd, id_q, kk > 0 ? 1u : 0u);
        }
        tc_commit(dq_full);
        tc_commit(&qd_empty[st]);
      }
      tc_commit(done);
      mbar_wait_bounded(done, 0, a.status, kErrWaitTimeoutAccum, 316);
    }
  } else {
    // ------------------------------------------------------------ compute
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;   // warpgroup 0 or 1
    const int r = quarter * 32 + lane;  // key row (S^T, dP^T, dV, dK) and query row (dQ)
    const int key = n0 + r;
    const bool kvalid = key < T;
    const uint32_t lb = tmem + ((uint32_t)(quarter * 32) << 16);
    bool ok = true;
    for (int t = 0; t < steps && ok; ++t) {
      const int st = t % S;
      const uint32_t tp = t & 1;
      const int q0 = (i_start + t) * BQ;
      // qd_full orders the producer's lse / delta stores before our reads
      if (!mbar_wait_warp(&qd_full[st], (t / S) & 1, a.status, kErrWaitTimeoutFull, 320) ||
          !mbar_wait_warp(s_full, tp, a.status, kErrWaitTimeoutAccum, 321)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float* lse = sVec + st * (2 * BQ);
      const float* dlt = lse + BQ;
      const bool diag = a.causal && (q0 < n0 + BK);
#pragma unroll 1
      for (int cc = 0; cc < 2; ++cc) {
        const int c = half * 2 + cc;  // 32-query chunk 0..3
        float sv[32], pv[32];
        tmem_ld_32x32b_x32(lb + Cfg::kST + c * 32, sv);
        tmem_ld_32x32b_x32(lb + Cfg::kDPT + c * 32, pv);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int qi = c * 32 + i;
          float p = exp2f(sv[i] * a.sl2 - lse[qi]);
          if (!kvalid || (diag && key > q0 + qi)) p = 0.f;
          sv[i] = p;
          pv[i] = p * (pv[i] - dlt[qi]);
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int ch = cc * 4 + g;  // 8-query chunk within sub-tile `half`
          const uint32_t off = half * (128 * 128) + r * 128 + ((ch ^ (r & 7)) << 4);
          __align__(16) __nv_bfloat162 hp[4], hd[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            hp[e] = __floats2bfloat162_rn(sv[g * 8 + 2 * e], sv[g * 8 + 2 * e + 1]);
            hd[e] = __floats2bfloat162_rn(pv[g * 8 + 2 * e], pv[g * 8 + 2 * e + 1]);
          }
          *reinterpret_cast<uint4*>(sPT + off) = *reinterpret_cast<uint4*>(hp);
          *reinterpret_cast<uint4*>(sDST + off) = *reinterpret_cast<uint4*>(hd);
        }
      }
      tc_fence_before();
      mbar_arrive(s_free);
      fence_proxy_async_smem();
      mbar_arrive(p_full);
      // dQ_i (query row r, this warpgroup's half of the columns) -> fp32 accumulator
      if (!mbar_wait_warp(dq_full, tp, a.status, kErrWaitTimeoutAccum, 322)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int qrow = q0 + r;
      float* dst = a.dq_accum + (((long long)b * T + qrow) * a.H + h) * D + half * (D / 2);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        float v[32];
        tmem_ld_32x32b_x32(lb + Cfg::kDQ + half * (D / 2) + c * 32, v);
        if (qrow < T) {
#pragma unroll
          for (int e = 0; e < 8; ++e)
            atomicAdd(reinterpret_cast<float4*>(dst + c * 32 + e * 4),
                      make_float4(v[e * 4], v[e * 4 + 1], v[e * 4 + 2], v[e * 4 + 3]));
        }
      }
      tc_fence_before();
      mbar_arrive(dq_free);
    }
    // dK (scaled) and dV: key row r, this warpgroup's half of the columns.
    // `ok` is warp-uniform (mbar_wait_warp); the TMEM loads are warp-collective
    // and run in every lane, only the stores depend on the key being in range.
    if (ok) {
      __nv_bfloat16* dk = a.dqkv + (long long)(row0 + key) * 3 * a.F + a.F + h * D + half * (D / 2);
      __nv_bfloat16* dv = dk + a.F;
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        float kv[32], vv[32];
        tmem_ld_32x32b_x32(lb + Cfg::kDK + half * (D / 2) + c * 32, kv);
        tmem_ld_32x32b_x32(lb + Cfg::kDV + half * (D / 2) + c * 32, vv);
        if (!kvalid) continue;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          __align__(16) __nv_bfloat162 hk[4], hv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            hk[e] = __floats2bfloat162_rn(kv[g * 8 + 2 * e] * a.scale, kv[g * 8 + 2 * e + 1] * a.scale);
            hv[e] = __floats2bfloat162_rn(vv[g * 8 + 2 * e], vv[g * 8 + 2 * e + 1]);
          }
          *reinterpret_cast<uint4*>(dk + c * 32 + g * 8) = *reinterpret_cast<uint4*>(hk);
          *reinterpret_cast<uint4*>(dv + c * 32 + g * 8) = *reinterpret_cast<uint4*>(hv);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kCols);
  }
}

template <int D>
void launch_bwd(const AttnBwdParams& p, cudaStream_t s) {
  using Cfg = BwdCfg<D>;
  static bool attr = false;
  if (!attr) {
    UHFS_CUDA_CHECK(cudaFuncSetAttribute(fa_bwd_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem));
    attr = true;
  }
  const long long F = (long long)p.f.H * D;
  CUtensorMap tq = make_tmap_bf16_2d(p.f.q, (uint64_t)(3 * F), (uint64_t)p.f.B * p.f.T, (uint64_t)(3 * F), 64, 128);
  CUtensorMap td = make_tmap_bf16_2d(p.dout, (uint64_t)F, (uint64_t)p.f.B * p.f.T, (uint64_t)p.do_stride_t, 64, 128);
  BwdArgs a{};
  a.B = p.f.B;
  a.H = p.f.H;
  a.T = p.f.T;
  a.F = F;
  a.sl2 = p.f.scale * kLog2e;
  a.scale = p.f.scale;
  a.causal = p.f.causal;
  a.lse = p.f.lse;
  a.delta = p.delta;
  a.dq_accum = p.dq_accum;
  a.dqkv = p.dq;
  a.status = device_status_ptr();
  dim3 grid((p.f.T + BK - 1) / BK, p.f.B * p.f.H);
  fa_bwd_tc_kernel<D><<<grid, kThreads, Cfg::kSmem, s>>>(tq, td, a);
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

}  // namespace

bool flash_attn_bwd_tc_supported(const AttnBwdParams& p) {
  const long long F = (long long)p.f.H * p.f.D;
  const bool fused_in = p.f.k == p.f.q + F && p.f.v == p.f.q + 2 * F && p.f.q_stride_t == 3 * F &&
                        p.f.q_stride_b == (long long)p.f.T * 3 * F;
  const bool fused_out = p.dk == p.dq + F && p.dv == p.dq + 2 * F && p.dq_stride_t == 3 * F &&
                         p.dq_stride_b == (long long)p.f.T * 3 * F;
  const bool dout_ok = p.do_stride_b == (long long)p.f.T * p.do_stride_t && p.do_stride_t % 8 == 0 &&
                       (reinterpret_cast<uintptr_t>(p.dout) & 15u) == 0;
  return (p.f.D == 64 || p.f.D == 128) && fused_in && fused_out && dout_ok &&
         (reinterpret_cast<uintptr_t>(p.f.q) & 15u) == 0;
}

void flash_attn_bwd_tc_main(const AttnBwdParams& p, cudaStream_t s) {
  if (p.f.D == 64) launch_bwd<64>(p, s);
  else launch_bwd<128>(p, s);
}

}  // namespace uhfs
