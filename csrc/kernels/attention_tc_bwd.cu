// Flash-attention backward on the 5th-generation tensor core (tcgen05 + TMEM).
//
// One CTA owns a block of 128 keys of one (batch, head) and loops over the
// 128-query blocks that attend to it (causal: from the diagonal on).
//
//   warps 0..7  two compute warpgroups; TMEM lane r (warp%4 picks the lane
//               quarter) is key row r and warpgroup g takes query columns
//               [64g, 64g+64).  Each thread loads its 64 S^T and 64 dP^T
//               values with four TMEM loads and one wait, frees S^T / dP^T,
//               and computes P^T = exp2(S^T*scale*log2e - lse) and
//               dS^T = P^T (dP^T - delta), both as bf16: dS^T into the
//               swizzled shared tile (warpgroup g fills sub-tile g), P^T for
//               D = 64 into TMEM (the A operand of dV; shared memory for
//               D = 128); at the end the same split stores dK (scaled) and
//               dV.
//   warp 8      TMA producer: K, V once; Q_i, dO_i per query block (ring),
//               plus lse_i / delta_i into shared memory
//   warps 12-15 dQ read-out: lane r of warp 12+q takes query row 32q + r of
//               dQ_i from TMEM, stages it as swizzled fp32 boxes and adds
//               them into the fp32 dQ accumulator with TMA reduce-add, off
//               the compute warps' critical path (per-thread vector
//               reductions of 32 different rows per warp instruction were
//               measured to saturate the load/store pipe the compute warps
//               need)
//   warp 9      TMEM allocator + MMA issuer (one elected thread), per block i:
//                 S^T  = K Q_i^T           M=128 keys, N=128 queries, K=D
//                 dP^T = V dO_i^T          (same shape)
//                 dV  += P^T dO_i          M=128 keys, N=D, K=128 queries
//                 dK  += dS^T Q_i          (same)
//                 dQ_i = dS K              M=128 queries, N=D, K=128 keys
//               (dS is read MN-major from the dS^T tile; dO_i, Q_i and K are
//               read MN-major as the B operands of the last three products).
//               For D = 64, S^T / dP^T of block i+1 are issued as soon as the
//               compute warps hold block i in registers, so they overlap the
//               softmax of block i.
//
// TMEM: S^T [0,128), dP^T [128,256), dV, dK, then for D = 64 dQ [384,448)
// and P^T [448,512) (bf16 pairs); for D = 128 dQ reuses the S^T columns,
// which keeps that case in step order.
// Shared memory bandwidth bounds this kernel (every MMA operand but P^T is
// read from it at 128 B/clk): with P^T in TMEM a 128 x 128 step of D = 64
// moves about 300 KB through it.
// Registers: 512 threads launch with 128 each; warpgroups 2 and 3 give back
// down to 64 and the compute warpgroups take 192 (the host checks the launch
// count).
// Every wait is bounded.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace uhfs {

CUtensorMap make_tmap_bf16_2d(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                              uint32_t box_inner, uint32_t box_outer);
CUtensorMap make_tmap_f32_2d(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                             uint32_t box_inner, uint32_t box_outer);

namespace {

constexpr int BK = 128;  // keys per CTA
constexpr int BQ = 128;  // queries per step
constexpr int kCompute = 256;      // warps 0..7
constexpr int kReadout = 128;      // warps 12..15
constexpr int kThreads = 512;      // 4 warpgroups
constexpr int kLaunchRegs = 128;   // 65536 / 512
constexpr int kComputeRegs = 192;
constexpr int kServiceRegs = 64;
static_assert(2 * 128 * kComputeRegs + 2 * 128 * kServiceRegs <= kThreads * kLaunchRegs, "register split");
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct BwdCfg {
  static constexpr int kTile = 128 * D * 2;          // one [128][D] bf16 tile (D/64 swizzled sub-tiles)
  static constexpr int kStages = (D == 64) ? 4 : 1;  // Q_i / dO_i ring depth
  static constexpr bool kPtTmem = (D == 64);          // P^T in TMEM (A operand of dV)
  static constexpr int kStageBytes = 2 * kTile;      // Q_i | dO_i
  static constexpr int kPT = BK * BQ * 2;            // P^T or dS^T tile (2 sub-tiles of 128 x 64)
  static constexpr int kVec = 2 * BQ * 4;            // lse_i | delta_i
  static constexpr int kStage = 128 * 32 * 4;        // fp32 dQ staging box (128 rows x 32)
  static constexpr int kStageBoxes = (D == 64) ? 1 : 2;
  static constexpr int kSmem = 1024 + 2 * kTile + kStages * kStageBytes + (kPtTmem ? 1 : 2) * kPT + kStages * kVec +
                               kStageBoxes * kStage + 256;
  static_assert(kSmem <= 227 * 1024, "attention backward shared memory");
  static constexpr uint32_t kST = 0, kDPT = 128, kDV = 256, kDK = 256 + D;
  static constexpr uint32_t kDQ = (D == 64) ? 256 + 2 * D : 0;  // D=128: reuse S^T columns
  static constexpr uint32_t kPTT = 256 + 3 * D;                  // D=64: P^T (64 columns of bf16 pairs)
  static constexpr int kDQBufs = 1;
  static_assert(!kPtTmem || kPTT + 64 <= 512, "P^T columns");
  static constexpr uint32_t kCols = 512;
};

// Optional per-step clock stamps (clock64 of the SM) for the CTAs of head 0
// of batch 0: trace[(blockIdx.x * kTraceEvents + event) * kTraceSteps + step].
// Off (nullptr) unless a buffer is installed with set_attn_bwd_trace.
constexpr int kTraceEvents = 16, kTraceSteps = 64;
enum BwdTraceEvent {
  kTrStart = 0, kTrQdEmpty, kTrQdStored, kTrMmaS, kTrMmaGrads, kTrSFull, kTrSRegs, kTrMath, kTrPFull,
  kTrDqFull, kTrDqDone, kTrEpiStart, kTrEpiEnd, kTrKvFull
};
unsigned long long* g_bwd_trace = nullptr;

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
  unsigned long long* trace;
  int trace_bh;  // (batch, head) whose CTAs are traced (UHFS_ATTN_TRACE_BH, trace builds)
};

// Compiled in only with -DUHFS_ATTN_TRACE (UNDERHFS_ATTN_TRACE=1 at build
// time); the product build has no stamps and no trace pointer test.
#ifdef UHFS_ATTN_TRACE
#define BWD_TRACE(ev, step)                                                                              \
  do {                                                                                                   \
    if (a.trace != nullptr && (int)blockIdx.y == a.trace_bh && (step) < kTraceSteps)                       \
      a.trace[((long long)blockIdx.x * kTraceEvents + (ev)) * kTraceSteps + (step)] = (unsigned long long)clock64(); \
  } while (0)
#else
#define BWD_TRACE(ev, step) \
  do { \
  } while (0)
#endif

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    fa_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
                     const __grid_constant__ CUtensorMap tm_dq, const BwdArgs a) {
  using Cfg = BwdCfg<D>;
  constexpr int KD = D / 64;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align1024(smem_raw);
  uint8_t* sK = smem;
  uint8_t* sV = sK + Cfg::kTile;
  uint8_t* sQD = sV + Cfg::kTile;                 // [S][Q | dO]
  uint8_t* sDST = sQD + S * Cfg::kStageBytes;     // dS^T
  uint8_t* sPT = sDST + Cfg::kPT;                 // P^T (D = 128 only)
  float* sVec = reinterpret_cast<float*>(sDST + (Cfg::kPtTmem ? 1 : 2) * Cfg::kPT);  // [S][lse(128) | delta(128)]
  uint8_t* sStage = reinterpret_cast<uint8_t*>(sVec) + S * Cfg::kVec;  // [kStageBoxes] fp32 dQ boxes
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStage + Cfg::kStageBoxes * Cfg::kStage);
  uint64_t* kv_full = bars;          // 1
  uint64_t* qd_full = bars + 1;      // [S]
  uint64_t* qd_empty = bars + 1 + S; // [S]
  uint64_t* s_full = bars + 1 + 2 * S;   // S^T and dP^T ready
  uint64_t* s_free = s_full + 1;     // S^T / dP^T held in registers by all compute threads
  uint64_t* p_full = s_full + 2;     // P^T / dS^T written
  uint64_t* dq_full = s_full + 3;    // dQ of a step ready (dQ MMAs done)
  uint64_t* dq_free = s_full + 4;    // dQ of a step read out
  uint64_t* pt_free = s_full + 5;    // dV / dK MMAs of step i done: P^T / dS^T reusable
  uint64_t* done = s_full + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 7);

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
  constexpr int kProducerWarp = 8, kMmaWarp = 9;

  if (warp == kProducerWarp && lane == 0) {
    tma_prefetch_desc(&tm_qkv);
    tma_prefetch_desc(&tm_do);
    tma_prefetch_desc(&tm_dq);
    mbar_init(kv_full, 1);
    for (int i = 0; i < S; ++i) {
      mbar_init(&qd_full[i], 2);  // TMA bytes + the producer's lse / delta stores
      mbar_init(&qd_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, kCompute);
    mbar_init(p_full, kCompute);
    for (int i = 0; i < Cfg::kDQBufs; ++i) {
      mbar_init(&dq_full[i], 1);
      mbar_init(&dq_free[i], kReadout);
    }
    mbar_init(pt_free, 1);
    mbar_init(done, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, Cfg::kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 8) {
    // register counts are set at the top of each role's branch so the
    // compiler allocates every region with the count it runs under
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kServiceRegs));
  }
  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer
    uint32_t issued = 0, iph = 0;  // bit s: stage s has a load in flight / its phase
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 2 * Cfg::kTile);
      for (int kd = 0; kd < KD; ++kd) {
        tma_load_2d(sK + kd * (BK * 128), &tm_qkv, kv_full, (int)(a.F + h * D + kd * 64), row0 + n0);
        tma_load_2d(sV + kd * (BK * 128), &tm_qkv, kv_full, (int)(2 * a.F + h * D + kd * 64), row0 + n0);
      }
    }
    for (int t = 0; t < steps; ++t) {
      const int st = t % S;
      const uint32_t ph = (t / S) & 1;
      int good = 1;
      if (lane == 0) good = mbar_wait_bounded(&qd_empty[st], ph ^ 1u, a.status, kErrWaitTimeoutEmpty, 300);
      good = __shfl_sync(0xffffffffu, good, 0);
      if (!good) break;
      if (lane == 0) BWD_TRACE(kTrQdEmpty, t);
      const int q0 = (i_start + t) * BQ;
      if (!UHFS_CHECK(q0 < T && n0 < T, a.status, 303)) break;
      if (lane == 0) {
        uint8_t* sQ = sQD + st * Cfg::kStageBytes;
        uint8_t* sDO = sQ + Cfg::kTile;
        mbar_arrive_expect_tx(&qd_full[st], 2 * Cfg::kTile);
        for (int kd = 0; kd < KD; ++kd) {
          tma_load_2d(sQ + kd * (BQ * 128), &tm_qkv, &qd_full[st], (int)(h * D + kd * 64), row0 + q0);
          tma_load_2d(sDO + kd * (BQ * 128), &tm_do, &qd_full[st], (int)(h * D + kd * 64), row0 + q0);
        }
        issued |= 1u << st;
        iph = (iph & ~(1u << st)) | (ph << st);
      }
      // lse / delta of this query block: all loads in flight at once, then the
      // stores, ordered before the second arrival on qd_full
      float lv[BQ / 32], dv[BQ / 32];
#pragma unroll
      for (int k = 0; k < BQ / 32; ++k) {
        const int qq = q0 + k * 32 + lane;
        lv[k] = qq < T ? __ldg(a.lse + (long long)bh * T + qq) : INFINITY;
        dv[k] = qq < T ? __ldg(a.delta + (long long)bh * T + qq) : 0.f;
      }
      float* vec = sVec + st * (2 * BQ);
#pragma unroll
      for (int k = 0; k < BQ / 32; ++k) {
        vec[k * 32 + lane] = lv[k];
        vec[BQ + k * 32 + lane] = dv[k];
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&qd_full[st]);
        BWD_TRACE(kTrQdStored, t);
      }
    }
    if (lane == 0) {
      mbar_wait_bounded(kv_full, 0, a.status, kErrWaitTimeoutFull, 301);
      for (int s2 = 0; s2 < S; ++s2)
        if (issued & (1u << s2)) mbar_wait_bounded(&qd_full[s2], (iph >> s2) & 1u, a.status, kErrWaitTimeoutFull, 302);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one_sync()) {
      constexpr uint32_t id_s = make_idesc(1, 0, 0, BK, BQ);   // K / V K-major, Q / dO K-major
      constexpr uint32_t id_kv = make_idesc(1, 0, 1, BK, D);   // P^T / dS^T K-major, dO / Q MN-major
      constexpr uint32_t id_q = make_idesc(1, 1, 1, BQ, D);    // dS MN-major, K MN-major
      // descriptors with a zero start address; the start field (address >> 4)
      // is added per operand and stays below 2^14 (shared memory < 256 KB)
      const uint64_t kmaj = make_smem_desc(0, 16, 1024, kSwizzle128B);
      const uint64_t mnmaj = make_smem_desc(0, 128 * 128, 1024, kSwizzle128B);  // 128-row operand tiles
      const uint32_t k16 = smem_u32(sK) >> 4, v16 = smem_u32(sV) >> 4, qd16 = smem_u32(sQD) >> 4;
      const uint32_t pt16 = smem_u32(sPT) >> 4, dst16 = smem_u32(sDST) >> 4;
      auto issue_s = [&](int t) -> bool {
        const int st = t % S;
        if (!mbar_wait_bounded(&qd_full[st], (uint32_t)(t / S) & 1u, a.status, kErrWaitTimeoutFull, 311)) return false;
        BWD_TRACE(kTrMmaS, t);
        tc_fence_after();
        const uint32_t q16 = qd16 + st * (Cfg::kStageBytes >> 4), do16 = q16 + (Cfg::kTile >> 4);
#pragma unroll 1
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * (128 * 128) + (kk & 3) * 32) >> 4;
          tc_mma_f16(tmem + Cfg::kST, kmaj + k16 + off, kmaj + q16 + off, id_s, kk > 0 ? 1u : 0u);
        }
#pragma unroll 1
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * (128 * 128) + (kk & 3) * 32) >> 4;
          tc_mma_f16(tmem + Cfg::kDPT, kmaj + v16 + off, kmaj + do16 + off, id_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(s_full);
        return true;
      };
      auto issue_grads = [&](int t) {
        const int st = t % S;
        const uint32_t q16 = qd16 + st * (Cfg::kStageBytes >> 4), do16 = q16 + (Cfg::kTile >> 4);
        // dQ_i = dS K first (A = dS^T read MN-major: 64-query chunks are the
        // two sub-tiles), so its read-out overlaps the dV / dK products
#pragma unroll 1
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint32_t off = (kk * 16 * 128) >> 4;
          tc_mma_f16(tmem + Cfg::kDQ + (uint32_t)((t % Cfg::kDQBufs) * D), mnmaj + dst16 + off, mnmaj + k16 + off,
                     id_q, kk > 0 ? 1u : 0u);
        }
        tc_commit(&dq_full[t % Cfg::kDQBufs]);
        // dV += P^T dO ; dK += dS^T Q    (K = 128 queries: sub-tile kk>>2 of the P^T / dS^T tiles)
#pragma unroll 1
        for (int kk = 0; kk < BQ / 16; ++kk) {
          const uint32_t aoff = ((kk >> 2) * (128 * 128) + (kk & 3) * 32) >> 4;
          const uint32_t boff = (kk * 16 * 128) >> 4;
          const uint32_t acc = (t > 0 || kk > 0) ? 1u : 0u;
          if constexpr (Cfg::kPtTmem)
            tc_mma_f16_ts(tmem + Cfg::kDV, tmem + Cfg::kPTT + (uint32_t)(kk * 8), mnmaj + do16 + boff, id_kv, acc);
          else
            tc_mma_f16(tmem + Cfg::kDV, kmaj + pt16 + aoff, mnmaj + do16 + boff, id_kv, acc);
          tc_mma_f16(tmem + Cfg::kDK, kmaj + dst16 + aoff, mnmaj + q16 + boff, id_kv, acc);
        }
        tc_commit(pt_free);
        tc_commit(&qd_empty[st]);
      };
      bool ok = mbar_wait_bounded(kv_full, 0, a.status, kErrWaitTimeoutFull, 310);
      BWD_TRACE(kTrKvFull, 0);
      if (D == 64) {
        // S^T / dP^T of block t+1 are issued before the gradients of block t
        ok = ok && issue_s(0);
        for (int t = 0; t < steps && ok; ++t) {
          if (t + 1 < steps) {
            if (!mbar_wait_bounded(s_free, (uint32_t)t & 1u, a.status, kErrWaitTimeoutAccum, 312) ||
                !issue_s(t + 1)) {
              ok = false;
              break;
            }
          }
          if (!mbar_wait_bounded(p_full, (uint32_t)t & 1u, a.status, kErrWaitTimeoutAccum, 314) ||
              (t >= Cfg::kDQBufs &&
               !mbar_wait_bounded(&dq_free[t % Cfg::kDQBufs], (uint32_t)(t / Cfg::kDQBufs - 1) & 1u, a.status,
                                  kErrWaitTimeoutAccum, 315))) {
            ok = false;
            break;
          }
          BWD_TRACE(kTrMmaGrads, t);
          tc_fence_after();
          issue_grads(t);
        }
      } else {
        // dQ shares the S^T columns: strictly one block after the other
        for (int t = 0; t < steps && ok; ++t) {
          if (t > 0 && (!mbar_wait_bounded(s_free, (uint32_t)(t - 1) & 1u, a.status, kErrWaitTimeoutAccum, 312) ||
                        !mbar_wait_bounded(&dq_free[0], (uint32_t)(t - 1) & 1u, a.status, kErrWaitTimeoutAccum, 313))) {
            ok = false;
            break;
          }
          if (!issue_s(t) || !mbar_wait_bounded(p_full, (uint32_t)t & 1u, a.status, kErrWaitTimeoutAccum, 314)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_grads(t);
        }
      }
      tc_commit(done);
      mbar_wait_bounded(done, 0, a.status, kErrWaitTimeoutAccum, 316);
    }
  } else if (warp < 8) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kComputeRegs));
    // ------------------------------------------------------------ compute
    const int quarter = warp & 3;
    const int half = warp >> 2;         // warpgroup 0 or 1
    const int r = quarter * 32 + lane;  // key row (S^T, dP^T, dV, dK) and query row (dQ)
    const int key = n0 + r;
    const bool kvalid = key < T;
    const uint32_t lb = tmem + ((uint32_t)(quarter * 32) << 16);
    [[maybe_unused]] uint8_t* pt_row = sPT + half * (128 * 128) + r * 128;
    uint8_t* dst_row = sDST + half * (128 * 128) + r * 128;
    // Failures are warp-uniform (mbar_wait_warp); after a failed wait a warp
    // skips the work but keeps arriving where the others expect it.
    bool ok = true;
    const bool tracer = warp == 0 && lane == 0;
    if (tracer) BWD_TRACE(kTrStart, 0);
    for (int t = 0; t < steps; ++t) {
      const int st = t % S;
      const uint32_t tp = t & 1;
      const int q0 = (i_start + t) * BQ;
      // qd_full orders the producer's lse / delta stores before our reads
      if (ok && (!mbar_wait_warp(&qd_full[st], (t / S) & 1, a.status, kErrWaitTimeoutFull, 320) ||
                 !mbar_wait_warp(s_full, tp, a.status, kErrWaitTimeoutAccum, 321)))
        ok = false;
      if (tracer) BWD_TRACE(kTrSFull, t);
      if (ok) {
        tc_fence_after();
        uint32_t sv[64], pv[64];
        tmem_ld_32x32b_x32_async(lb + Cfg::kST + half * 64, sv);
        tmem_ld_32x32b_x32_async(lb + Cfg::kST + half * 64 + 32, sv + 32);
        tmem_ld_32x32b_x32_async(lb + Cfg::kDPT + half * 64, pv);
        tmem_ld_32x32b_x32_async(lb + Cfg::kDPT + half * 64 + 32, pv + 32);
        tmem_wait_ld_regs<64>(sv);
        tmem_wait_ld_regs<64>(pv);
        tc_fence_before();
        mbar_arrive(s_free);  // S^T / dP^T may be overwritten
        if (tracer) BWD_TRACE(kTrSRegs, t);
        const float4* lse4 = reinterpret_cast<const float4*>(sVec + st * (2 * BQ) + half * 64);
        const float4* dlt4 = reinterpret_cast<const float4*>(sVec + st * (2 * BQ) + BQ + half * 64);
        // causal diagonal block: query column qi is visible for this key when qi >= key - q0
        const int qmin = (!kvalid) ? BQ + 1 : ((a.causal && q0 < n0 + BK) ? key - q0 - half * 64 : 0);
        uint32_t hp[32], hd[32];
#pragma unroll
        for (int g = 0; g < 16; ++g) {
          const float4 l = lse4[g], d = dlt4[g];
          const float lv[4] = {l.x, l.y, l.z, l.w}, dv[4] = {d.x, d.y, d.z, d.w};
          float p[4], ds[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i = g * 4 + e;
            float x = ex2_approx(fmaf(__uint_as_float(sv[i]), a.sl2, -lv[e]));
            if (i < qmin) x = 0.f;
            p[e] = x;
            ds[e] = x * (__uint_as_float(pv[i]) - dv[e]);
          }
          hp[g * 2] = pack_bf16x2(p[0], p[1]);
          hp[g * 2 + 1] = pack_bf16x2(p[2], p[3]);
          hd[g * 2] = pack_bf16x2(ds[0], ds[1]);
          hd[g * 2 + 1] = pack_bf16x2(ds[2], ds[3]);
        }
        if (tracer) BWD_TRACE(kTrMath, t);
        // P^T / dS^T tiles are free once the gradient MMAs of block t-1 finished
        if (t > 0 && !mbar_wait_warp(pt_free, (uint32_t)(t - 1) & 1u, a.status, kErrWaitTimeoutAccum, 323))
          ok = false;
        if (ok) {
          if constexpr (Cfg::kPtTmem) {
            // key row r, queries [64 half, 64 half + 64): columns [32 half, 32 half + 32)
            tmem_st_32x32b_x32(lb + Cfg::kPTT + half * 32, hp);
          }
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            const uint32_t off = (uint32_t)((ch ^ (r & 7)) << 4);
            if constexpr (!Cfg::kPtTmem)
              *reinterpret_cast<uint4*>(pt_row + off) =
                  make_uint4(hp[ch * 4], hp[ch * 4 + 1], hp[ch * 4 + 2], hp[ch * 4 + 3]);
            *reinterpret_cast<uint4*>(dst_row + off) =
                make_uint4(hd[ch * 4], hd[ch * 4 + 1], hd[ch * 4 + 2], hd[ch * 4 + 3]);
          }
          if constexpr (Cfg::kPtTmem) {
            tmem_wait_st();
            tc_fence_before();
          }
          fence_proxy_async_smem();
          mbar_arrive(p_full);
          if (tracer) BWD_TRACE(kTrPFull, t);
        }
      }
    }
    // the last dV / dK products have retired
    if (ok && steps > 0 &&
        !mbar_wait_warp(pt_free, (uint32_t)(steps - 1) & 1u, a.status, kErrWaitTimeoutAccum, 324))
      ok = false;
    if (tracer) BWD_TRACE(kTrEpiStart, 0);
    // dK (scaled) and dV: key row r, this warpgroup's half of the columns.
    // `ok` is warp-uniform (mbar_wait_warp); the TMEM loads are warp-collective
    // and run in every lane, only the stores depend on the key being in range.
    if (ok) {
      tc_fence_after();
      __nv_bfloat16* dk = a.dqkv + (long long)(row0 + key) * 3 * a.F + a.F + h * D + half * (D / 2);
      __nv_bfloat16* dv = dk + a.F;
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        uint32_t kv[32], vv[32];
        tmem_ld_32x32b_x32_async(lb + Cfg::kDK + half * (D / 2) + c * 32, kv);
        tmem_ld_32x32b_x32_async(lb + Cfg::kDV + half * (D / 2) + c * 32, vv);
        tmem_wait_ld_regs<32>(kv);
        tmem_wait_ld_regs<32>(vv);
        if (!kvalid) continue;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          uint4 hk, hv;
          hk.x = pack_bf16x2(__uint_as_float(kv[g * 8 + 0]) * a.scale, __uint_as_float(kv[g * 8 + 1]) * a.scale);
          hk.y = pack_bf16x2(__uint_as_float(kv[g * 8 + 2]) * a.scale, __uint_as_float(kv[g * 8 + 3]) * a.scale);
          hk.z = pack_bf16x2(__uint_as_float(kv[g * 8 + 4]) * a.scale, __uint_as_float(kv[g * 8 + 5]) * a.scale);
          hk.w = pack_bf16x2(__uint_as_float(kv[g * 8 + 6]) * a.scale, __uint_as_float(kv[g * 8 + 7]) * a.scale);
          hv.x = pack_bf16x2(__uint_as_float(vv[g * 8 + 0]), __uint_as_float(vv[g * 8 + 1]));
          hv.y = pack_bf16x2(__uint_as_float(vv[g * 8 + 2]), __uint_as_float(vv[g * 8 + 3]));
          hv.z = pack_bf16x2(__uint_as_float(vv[g * 8 + 4]), __uint_as_float(vv[g * 8 + 5]));
          hv.w = pack_bf16x2(__uint_as_float(vv[g * 8 + 6]), __uint_as_float(vv[g * 8 + 7]));
          *reinterpret_cast<uint4*>(dk + c * 32 + g * 8) = hk;
          *reinterpret_cast<uint4*>(dv + c * 32 + g * 8) = hv;
        }
      }
    }
    if (tracer) BWD_TRACE(kTrEpiEnd, 0);
  } else if (warp >= 12) {
    // ------------------------------------------------------------ dQ read-out
    // dQ_t: TMEM -> registers -> swizzled fp32 box -> TMA reduce-add into the
    // fp32 accumulator.  Rows past T add zeros (P is 0 there).  With two boxes
    // chunks of 32 columns alternate, so staging chunk c only waits for the
    // reduction issued two chunks earlier; with one box, for the previous.
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the block
    const uint32_t lb = tmem + ((uint32_t)(quarter * 32) << 16);
    const bool leader = warp == 12 && lane == 0;  // issues the TMA reductions
    bool ok = true;
    int chunk = 0;
    for (int tt = 0; tt < steps; ++tt) {
      const int q0 = (i_start + tt) * BQ;
      const int bi = tt % Cfg::kDQBufs;
      const uint32_t buf = (uint32_t)(bi * D);
      if (ok && !mbar_wait_warp(&dq_full[bi], (uint32_t)(tt / Cfg::kDQBufs) & 1u, a.status, kErrWaitTimeoutAccum, 322))
        ok = false;
      if (leader) BWD_TRACE(kTrDqFull, tt);
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c, ++chunk) {
        uint32_t v[32];
        if (ok) {
          tc_fence_after();
          tmem_ld_32x32b_x32_async(lb + Cfg::kDQ + buf + c * 32, v);
          tmem_wait_ld_regs<32>(v);
          if (c == D / 32 - 1) {
            tc_fence_before();
            mbar_arrive(&dq_free[bi]);  // this dQ buffer may be overwritten
          }
        }
        uint8_t* box = sStage + (Cfg::kStageBoxes == 2 ? (chunk & 1) : 0) * Cfg::kStage;
        if (leader) {  // the reduction that last used this box has read it
          if constexpr (Cfg::kStageBoxes == 2)
            bulk_wait_group_read1();
          else
            bulk_wait_group_read0();
        }
        named_barrier_sync(1, kReadout);
        if (ok) {
#pragma unroll
          for (int ch = 0; ch < 8; ++ch)
            *reinterpret_cast<uint4*>(box + r * 128 + ((ch ^ (r & 7)) << 4)) =
                make_uint4(v[ch * 4], v[ch * 4 + 1], v[ch * 4 + 2], v[ch * 4 + 3]);
          fence_proxy_async_smem();
        }
        named_barrier_sync(1, kReadout);
        if (leader && ok) {
          tma_reduce_add_2d(&tm_dq, box, h * D + c * 32, row0 + q0);
          bulk_commit_group();
        }
      }
      if (leader) BWD_TRACE(kTrDqDone, tt);
    }
    if (leader) bulk_wait_group0();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kCols);
  }
}

template <int D>
void launch_bwd(const AttnBwdParams& p, cudaStream_t s) {
  using Cfg = BwdCfg<D>;
  static PerDeviceOnce once;
  once([] {
    UHFS_CUDA_CHECK(cudaFuncSetAttribute(fa_bwd_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem));
    // setmaxnreg redistributes the launch allocation; a different launch count
    // could make the increase wait for registers that never come
    cudaFuncAttributes fa{};
    UHFS_CUDA_CHECK(cudaFuncGetAttributes(&fa, fa_bwd_tc_kernel<D>));
    if (fa.numRegs != kLaunchRegs)
      throw std::runtime_error("fa_bwd_tc_kernel: compiled with " + std::to_string(fa.numRegs) +
                               " registers per thread, the register split needs " + std::to_string(kLaunchRegs));
  });
  const long long F = (long long)p.f.H * D;
  CUtensorMap tq = make_tmap_bf16_2d(p.f.q, (uint64_t)(3 * F), (uint64_t)p.f.B * p.f.T, (uint64_t)(3 * F), 64, 128);
  CUtensorMap td = make_tmap_bf16_2d(p.dout, (uint64_t)F, (uint64_t)p.f.B * p.f.T, (uint64_t)p.do_stride_t, 64, 128);
  // dQ accumulator [B*T, H*D] fp32, reduced into in boxes of 32 columns x 128 rows
  CUtensorMap tdq = make_tmap_f32_2d(p.dq_accum, (uint64_t)F, (uint64_t)p.f.B * p.f.T, (uint64_t)F, 32, 128);
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
  a.trace = g_bwd_trace;
#ifdef UHFS_ATTN_TRACE
  {
    const char* e = getenv("UHFS_ATTN_TRACE_BH");
    a.trace_bh = e != nullptr ? atoi(e) : 0;
  }
#endif
  dim3 grid((p.f.T + BK - 1) / BK, p.f.B * p.f.H);
  fa_bwd_tc_kernel<D><<<grid, kThreads, Cfg::kSmem, s>>>(tq, td, tdq, a);
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

void set_attn_bwd_trace(unsigned long long* buf) {
#ifdef UHFS_ATTN_TRACE
  g_bwd_trace = buf;
#else
  if (buf != nullptr)
    throw std::runtime_error("set_attn_bwd_trace: the extension was built without UHFS_ATTN_TRACE "
                             "(rebuild with UNDERHFS_ATTN_TRACE=1)");
#endif
}

void flash_attn_bwd_tc_main(const AttnBwdParams& p, cudaStream_t s) {
  if (p.f.D == 64) launch_bwd<64>(p, s);
  else launch_bwd<128>(p, s);
}

}  // namespace uhfs
