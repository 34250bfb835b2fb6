// Flash-attention backward on the 5th-generation tensor core (tcgen05 + TMEM).
//
// Persistent: one CTA per SM walks (key block, batch-head) items, longest
// first; for each it owns the block of 128 keys and loops over the 128-query
// blocks that attend to it (causal: from the diagonal on).  Across items the
// barrier phases run on per-CTA counters, the next item's K / V are loaded
// into a second buffer (D = 64) while the current item runs, its first
// S^T / dP^T products overlap the current item's last step and dK / dV
// epilogue, and the dK / dV accumulators are reused once the epilogue has
// read them out (dkv_free).
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
// Registers: 512 threads launch with 128 each; warpgroups 2 (producer, MMA)
// and 3 (dQ read-out) give back down to 56 and the compute warpgroups take
// 200 (the host checks the launch count).
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
constexpr int kComputeRegs = 200;
constexpr int kIssueRegs = 56;     // warpgroup 2: producer + MMA issuer (per-item state of the persistent loop)
constexpr int kReadoutRegs = 56;   // warpgroup 3: dQ read-out
static_assert(2 * 128 * kComputeRegs + 128 * kIssueRegs + 128 * kReadoutRegs <= kThreads * kLaunchRegs,
              "register split");
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct BwdCfg {
  static constexpr int kTile = 128 * D * 2;          // one [128][D] bf16 tile (D/64 swizzled sub-tiles)
  static constexpr int kStages = (D == 64) ? 3 : 1;  // Q_i / dO_i ring depth
  // K / V buffers: D = 64 prefetches the next item's K / V while the current
  // item runs (the persistent CTA's per-item load is off the critical path);
  // D = 128 has the shared memory for one
  static constexpr int kKVBufs = (D == 64) ? 2 : 1;
  static constexpr bool kPtTmem = (D == 64);          // P^T in TMEM (A operand of dV)
  static constexpr int kStageBytes = 2 * kTile;      // Q_i | dO_i
  static constexpr int kPT = BK * BQ * 2;            // P^T or dS^T tile (2 sub-tiles of 128 x 64)
  static constexpr int kVec = 2 * BQ * 4;            // lse_i | delta_i
  static constexpr int kStage = 128 * 32 * 4;        // fp32 dQ staging box (128 rows x 32)
  static constexpr int kStageBoxes = (D == 64) ? 1 : 2;
  static constexpr int kSmem = 1024 + kKVBufs * 2 * kTile + kStages * kStageBytes + (kPtTmem ? 1 : 2) * kPT +
                               kStages * kVec + kStageBoxes * kStage + 256;
  static_assert(kSmem <= 227 * 1024, "attention backward shared memory");
  static constexpr uint32_t kST = 0, kDPT = 128, kDV = 256, kDK = 256 + D;
  static constexpr uint32_t kDQ = (D == 64) ? 256 + 2 * D : 0;  // D=128: reuse S^T columns
  static constexpr uint32_t kPTT = 256 + 3 * D;                  // D=64: P^T (64 columns of bf16 pairs)
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
#define BWD_TRACE(cta, ev, step)                                                                         \
  do {                                                                                                   \
    if (tr_on && (step) < kTraceSteps)                                                                   \
      a.trace[((long long)(cta) * kTraceEvents + (ev)) * kTraceSteps + (step)] = (unsigned long long)clock64(); \
  } while (0)
#else
#define BWD_TRACE(cta, ev, step) \
  do {                           \
  } while (0)
#endif

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    fa_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
                     const __grid_constant__ CUtensorMap tm_dq, const BwdArgs a) {
  using Cfg = BwdCfg<D>;
  constexpr int KD = D / 64;
  constexpr int S = Cfg::kStages;
  constexpr int KV = Cfg::kKVBufs;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align1024(smem_raw);
  uint8_t* sKV = smem;                              // [KV][K | V]
  uint8_t* sQD = sKV + KV * 2 * Cfg::kTile;         // [S][Q | dO]
  uint8_t* sDST = sQD + S * Cfg::kStageBytes;       // dS^T
  uint8_t* sPT = sDST + Cfg::kPT;                   // P^T (D = 128 only)
  float* sVec = reinterpret_cast<float*>(sDST + (Cfg::kPtTmem ? 1 : 2) * Cfg::kPT);  // [S][lse(128) | delta(128)]
  uint8_t* sStage = reinterpret_cast<uint8_t*>(sVec) + S * Cfg::kVec;  // [kStageBoxes] fp32 dQ boxes
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStage + Cfg::kStageBoxes * Cfg::kStage);
  uint64_t* kv_full = bars;              // [KV]
  uint64_t* kv_empty = bars + KV;        // [KV] an item's MMAs are done with its K / V buffer
  uint64_t* qd_full = bars + 2 * KV;     // [S]
  uint64_t* qd_empty = qd_full + S;      // [S]
  uint64_t* s_full = qd_empty + S;       // S^T and dP^T ready
  uint64_t* s_free = s_full + 1;         // S^T / dP^T held in registers by all compute threads
  uint64_t* p_full = s_full + 2;         // P^T / dS^T written
  uint64_t* dq_full = s_full + 3;        // dQ of a step ready (dQ MMAs done)
  uint64_t* dq_free = s_full + 4;        // dQ of a step read out
  uint64_t* pt_free = s_full + 5;        // dV / dK MMAs of a step done: P^T / dS^T reusable
  uint64_t* dkv_free = s_full + 6;       // an item's dK / dV were read out of TMEM
  uint64_t* done = s_full + 7;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = a.T;
  const int i_end = (T + BQ - 1) / BQ;
  const int n_kblocks = (T + BK - 1) / BK;
  // Work units pair key blocks j and n-1-j of one (batch, head): under the
  // causal mask every unit has n+1 query steps, so units balance across
  // CTAs, and units run head-major so that the CTAs working at the same time
  // share each head's Q / dO tiles in L2.  CTA c takes units c, c+G, c+2G, ...
  // (G = gridDim.x) and runs both halves of a unit back to back; the virtual
  // index it = c + m G walks them (half = (it / G) & 1).
  const int pairs = (n_kblocks + 1) / 2;
  const int n_units = pairs * a.B * a.H;
  const int n_virt = 2 * (int)gridDim.x * ((n_units + (int)gridDim.x - 1) / (int)gridDim.x);
  struct Item {
    int bh, b, h, n_block, n0, i_start, steps, row0;
    bool valid;
  };
  auto decode = [&](int it) {
    Item w{};
    const int G = gridDim.x;
    const int u = (it / (2 * G)) * G + it % G;
    const int hf = (it / G) & 1;
    const int p = u % pairs;
    w.bh = u / pairs;
    w.n_block = hf ? n_kblocks - 1 - p : p;
    w.valid = u < n_units && !(hf && w.n_block == p);  // an odd count's middle block has no partner
    w.b = w.bh / a.H;
    w.h = w.bh % a.H;
    w.n0 = w.n_block * BK;
    w.i_start = a.causal ? w.n0 / BQ : 0;
    w.steps = i_end - w.i_start;
    w.row0 = w.b * T;
    return w;
  };
  constexpr int kProducerWarp = 8, kMmaWarp = 9;

  if (warp == kProducerWarp && lane == 0) {
    tma_prefetch_desc(&tm_qkv);
    tma_prefetch_desc(&tm_do);
    tma_prefetch_desc(&tm_dq);
    for (int i = 0; i < KV; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < S; ++i) {
      mbar_init(&qd_full[i], 2);  // TMA bytes + the producer's lse / delta stores
      mbar_init(&qd_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, kCompute);
    mbar_init(p_full, kCompute);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, kReadout);
    mbar_init(pt_free, 1);
    mbar_init(dkv_free, kCompute);
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

  // register counts are set at the top of each role's branch so the
  // compiler allocates every region with the count it runs under
  if (warp >= 8 && warp < 12) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kIssueRegs));
  if (warp >= 12) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kReadoutRegs));
  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer
    uint32_t g = 0;  // query steps of this CTA (all items): ring position
    uint32_t k = 0;  // items of this CTA
    bool ok = true;
    for (int it = blockIdx.x; it < n_virt && ok; it += gridDim.x) {
      const Item w = decode(it);
      if (!w.valid) continue;
      const bool tr_on = a.trace != nullptr && w.bh == a.trace_bh;
      (void)tr_on;
      const uint32_t kvb = k % KV;
      ++k;
      int good = 1;
      if (lane == 0) {
        // the MMAs of the item that last used this K / V buffer are done
        good = mbar_wait_bounded(&kv_empty[kvb], (((k - 1) / KV) & 1u) ^ 1u, a.status, kErrWaitTimeoutEmpty, 304);
        if (good) {
          BWD_TRACE(w.n_block, kTrStart, 0);
          uint8_t* sK = sKV + kvb * 2 * Cfg::kTile;
          uint8_t* sV = sK + Cfg::kTile;
          mbar_arrive_expect_tx(&kv_full[kvb], 2 * Cfg::kTile);
          for (int kd = 0; kd < KD; ++kd) {
            tma_load_2d(sK + kd * (BK * 128), &tm_qkv, &kv_full[kvb], (int)(a.F + w.h * D + kd * 64), w.row0 + w.n0);
            tma_load_2d(sV + kd * (BK * 128), &tm_qkv, &kv_full[kvb], (int)(2 * a.F + w.h * D + kd * 64),
                        w.row0 + w.n0);
          }
        }
      }
      good = __shfl_sync(0xffffffffu, good, 0);
      if (!good) break;
      for (int t = 0; t < w.steps; ++t, ++g) {
        const int st = g % S;
        const uint32_t ph = (g / S) & 1u;
        if (lane == 0) good = mbar_wait_bounded(&qd_empty[st], ph ^ 1u, a.status, kErrWaitTimeoutEmpty, 300);
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good) {
          ok = false;
          break;
        }
        if (lane == 0) BWD_TRACE(w.n_block, kTrQdEmpty, t);
        const int q0 = (w.i_start + t) * BQ;
        if (!UHFS_CHECK(q0 < T && w.n0 < T, a.status, 303)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          uint8_t* sQ = sQD + st * Cfg::kStageBytes;
          uint8_t* sDO = sQ + Cfg::kTile;
          mbar_arrive_expect_tx(&qd_full[st], 2 * Cfg::kTile);
          for (int kd = 0; kd < KD; ++kd) {
            tma_load_2d(sQ + kd * (BQ * 128), &tm_qkv, &qd_full[st], (int)(w.h * D + kd * 64), w.row0 + q0);
            tma_load_2d(sDO + kd * (BQ * 128), &tm_do, &qd_full[st], (int)(w.h * D + kd * 64), w.row0 + q0);
          }
        }
        // lse / delta of this query block: all loads in flight at once, then the
        // stores, ordered before the second arrival on qd_full
        float lv[BQ / 32], dv[BQ / 32];
#pragma unroll
        for (int kk = 0; kk < BQ / 32; ++kk) {
          const int qq = q0 + kk * 32 + lane;
          lv[kk] = qq < T ? __ldg(a.lse + (long long)w.bh * T + qq) : INFINITY;
          dv[kk] = qq < T ? __ldg(a.delta + (long long)w.bh * T + qq) : 0.f;
        }
        float* vec = sVec + st * (2 * BQ);
#pragma unroll
        for (int kk = 0; kk < BQ / 32; ++kk) {
          vec[kk * 32 + lane] = lv[kk];
          vec[BQ + kk * 32 + lane] = dv[kk];
        }
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&qd_full[st]);
          BWD_TRACE(w.n_block, kTrQdStored, t);
        }
      }
    }
    // drain: every issued copy lands before the CTA exits
    if (lane == 0) {
      for (uint32_t kk = (k > (uint32_t)KV ? k - KV : 0); kk < k; ++kk)
        mbar_wait_bounded(&kv_full[kk % KV], (kk / KV) & 1u, a.status, kErrWaitTimeoutFull, 301);
      for (uint32_t gg = (g > (uint32_t)S ? g - S : 0); gg < g; ++gg)
        mbar_wait_bounded(&qd_full[gg % S], (gg / S) & 1u, a.status, kErrWaitTimeoutFull, 302);
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
      const uint32_t qd16 = smem_u32(sQD) >> 4;
      const uint32_t pt16 = smem_u32(sPT) >> 4, dst16 = smem_u32(sDST) >> 4;
      uint32_t g0 = 0;  // query steps before the current item
      uint32_t k = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < n_virt && ok; it += gridDim.x) {
        const Item w = decode(it);
        if (!w.valid) continue;
        const bool tr_on = a.trace != nullptr && w.bh == a.trace_bh;
        (void)tr_on;
        const uint32_t kvb = k % KV;
        const uint32_t k16 = smem_u32(sKV + kvb * 2 * Cfg::kTile) >> 4, v16 = k16 + (Cfg::kTile >> 4);
        auto issue_s = [&](uint32_t gs) -> bool {
          const int st = gs % S;
          if (!mbar_wait_bounded(&qd_full[st], (gs / S) & 1u, a.status, kErrWaitTimeoutFull, 311)) return false;
          BWD_TRACE(w.n_block, kTrMmaS, (int)(gs - g0));
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
        auto issue_grads = [&](uint32_t gs, int t) {
          const int st = gs % S;
          const uint32_t q16 = qd16 + st * (Cfg::kStageBytes >> 4), do16 = q16 + (Cfg::kTile >> 4);
          // dQ_i = dS K first (A = dS^T read MN-major: 64-query chunks are the
          // two sub-tiles), so its read-out overlaps the dV / dK products
#pragma unroll 1
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint32_t off = (kk * 16 * 128) >> 4;
            tc_mma_f16(tmem + Cfg::kDQ, mnmaj + dst16 + off, mnmaj + k16 + off, id_q, kk > 0 ? 1u : 0u);
          }
          tc_commit(dq_full);
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
        // waits before the gradient products of step gs (item step t)
        auto grads_ready = [&](uint32_t gs, int t) -> bool {
          if (!mbar_wait_bounded(p_full, gs & 1u, a.status, kErrWaitTimeoutAccum, 314)) return false;
          // the single dQ buffer was read out for the previous step
          if (gs > 0 && !mbar_wait_bounded(dq_free, (gs - 1) & 1u, a.status, kErrWaitTimeoutAccum, 315)) return false;
          // the previous item's dK / dV were read out before this item's first
          // products overwrite them
          if (t == 0 && k > 0 && !mbar_wait_bounded(dkv_free, (k - 1) & 1u, a.status, kErrWaitTimeoutAccum, 317))
            return false;
          return true;
        };
        if (!mbar_wait_bounded(&kv_full[kvb], (k / KV) & 1u, a.status, kErrWaitTimeoutFull, 310)) break;
        BWD_TRACE(w.n_block, kTrKvFull, 0);
        if (D == 64) {
          // S^T / dP^T of block t+1 are issued before the gradients of block t;
          // the item's first S^T waits for the last step of the previous item
          // to be held in registers
          if (g0 > 0 && !mbar_wait_bounded(s_free, (g0 - 1) & 1u, a.status, kErrWaitTimeoutAccum, 312)) break;
          ok = issue_s(g0);
          for (int t = 0; t < w.steps && ok; ++t) {
            const uint32_t gs = g0 + t;
            if (t + 1 < w.steps) {
              if (!mbar_wait_bounded(s_free, gs & 1u, a.status, kErrWaitTimeoutAccum, 312) || !issue_s(gs + 1)) {
                ok = false;
                break;
              }
            }
            if (!grads_ready(gs, t)) {
              ok = false;
              break;
            }
            BWD_TRACE(w.n_block, kTrMmaGrads, t);
            tc_fence_after();
            issue_grads(gs, t);
          }
        } else {
          // dQ shares the S^T columns: strictly one block after the other
          for (int t = 0; t < w.steps && ok; ++t) {
            const uint32_t gs = g0 + t;
            if (gs > 0 && (!mbar_wait_bounded(s_free, (gs - 1) & 1u, a.status, kErrWaitTimeoutAccum, 312) ||
                           !mbar_wait_bounded(dq_free, (gs - 1) & 1u, a.status, kErrWaitTimeoutAccum, 313))) {
              ok = false;
              break;
            }
            if (!issue_s(gs) || !grads_ready(gs, t)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_grads(gs, t);
          }
        }
        if (!ok) break;
        tc_commit(&kv_empty[kvb]);  // this item's K / V buffer may be refilled
        g0 += w.steps;
        ++k;
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
    const uint32_t lb = tmem + ((uint32_t)(quarter * 32) << 16);
    [[maybe_unused]] uint8_t* pt_row = sPT + half * (128 * 128) + r * 128;
    uint8_t* dst_row = sDST + half * (128 * 128) + r * 128;
    // Failures are warp-uniform (mbar_wait_warp); after a failed wait a warp
    // skips the work but keeps arriving where the others expect it.
    bool ok = true;
    const bool tracer = warp == 0 && lane == 0;
    (void)tracer;
    uint32_t g = 0;  // query steps of this CTA (all items)
    for (int it = blockIdx.x; it < n_virt; it += gridDim.x) {
      const Item w = decode(it);
      if (!w.valid) continue;
      const bool tr_on = a.trace != nullptr && w.bh == a.trace_bh;
      (void)tr_on;
      const int key = w.n0 + r;
      const bool kvalid = key < T;
      for (int t = 0; t < w.steps; ++t, ++g) {
        const int st = g % S;
        const int q0 = (w.i_start + t) * BQ;
        // qd_full orders the producer's lse / delta stores before our reads
        if (ok && (!mbar_wait_warp(&qd_full[st], (g / S) & 1u, a.status, kErrWaitTimeoutFull, 320) ||
                   !mbar_wait_warp(s_full, g & 1u, a.status, kErrWaitTimeoutAccum, 321)))
          ok = false;
        if (tracer) BWD_TRACE(w.n_block, kTrSFull, t);
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
          if (tracer) BWD_TRACE(w.n_block, kTrSRegs, t);
          const float4* lse4 = reinterpret_cast<const float4*>(sVec + st * (2 * BQ) + half * 64);
          const float4* dlt4 = reinterpret_cast<const float4*>(sVec + st * (2 * BQ) + BQ + half * 64);
          // causal diagonal block: query column qi is visible for this key when qi >= key - q0
          const int qmin = (!kvalid) ? BQ + 1 : ((a.causal && q0 < w.n0 + BK) ? key - q0 - half * 64 : 0);
          uint32_t hp[32], hd[32];
#pragma unroll
          for (int gg = 0; gg < 16; ++gg) {
            const float4 l = lse4[gg], d = dlt4[gg];
            const float lv[4] = {l.x, l.y, l.z, l.w}, dv[4] = {d.x, d.y, d.z, d.w};
            float p[4], ds[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int i = gg * 4 + e;
              float x = ex2_approx(fmaf(__uint_as_float(sv[i]), a.sl2, -lv[e]));
              if (i < qmin) x = 0.f;
              p[e] = x;
              ds[e] = x * (__uint_as_float(pv[i]) - dv[e]);
            }
            hp[gg * 2] = pack_bf16x2(p[0], p[1]);
            hp[gg * 2 + 1] = pack_bf16x2(p[2], p[3]);
            hd[gg * 2] = pack_bf16x2(ds[0], ds[1]);
            hd[gg * 2 + 1] = pack_bf16x2(ds[2], ds[3]);
          }
          if (tracer) BWD_TRACE(w.n_block, kTrMath, t);
          // P^T / dS^T tiles are free once the gradient MMAs of the previous step finished
          if (g > 0 && !mbar_wait_warp(pt_free, (g - 1) & 1u, a.status, kErrWaitTimeoutAccum, 323)) ok = false;
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
            if (tracer) BWD_TRACE(w.n_block, kTrPFull, t);
          }
        }
      }
      // the last dV / dK products of this item have retired
      if (ok && w.steps > 0 && !mbar_wait_warp(pt_free, (g - 1) & 1u, a.status, kErrWaitTimeoutAccum, 324))
        ok = false;
      if (tracer) BWD_TRACE(w.n_block, kTrEpiStart, 0);
      // dK (scaled) and dV: key row r, this warpgroup's half of the columns.
      // `ok` is warp-uniform (mbar_wait_warp); the TMEM loads are warp-collective
      // and run in every lane, only the stores depend on the key being in range.
      // chunks of 32 columns of dK and dV; the accumulators are released for
      // the next item once the last chunk is in registers
      __nv_bfloat16* dk = a.dqkv + (long long)(w.row0 + key) * 3 * a.F + a.F + w.h * D + half * (D / 2);
      __nv_bfloat16* dv = dk + a.F;
      if (ok) tc_fence_after();
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        uint32_t kv[32], vv[32];
        if (ok) {
          tmem_ld_32x32b_x32_async(lb + Cfg::kDK + half * (D / 2) + c * 32, kv);
          tmem_ld_32x32b_x32_async(lb + Cfg::kDV + half * (D / 2) + c * 32, vv);
          tmem_wait_ld_regs<32>(kv);
          tmem_wait_ld_regs<32>(vv);
        }
        if (c == D / 64 - 1) {
          tc_fence_before();
          mbar_arrive(dkv_free);  // dK / dV may be overwritten by the next item
        }
        if (!ok || !kvalid) continue;
#pragma unroll
        for (int gg = 0; gg < 4; ++gg) {
          uint4 hk, hv;
          hk.x = pack_bf16x2(__uint_as_float(kv[gg * 8 + 0]) * a.scale, __uint_as_float(kv[gg * 8 + 1]) * a.scale);
          hk.y = pack_bf16x2(__uint_as_float(kv[gg * 8 + 2]) * a.scale, __uint_as_float(kv[gg * 8 + 3]) * a.scale);
          hk.z = pack_bf16x2(__uint_as_float(kv[gg * 8 + 4]) * a.scale, __uint_as_float(kv[gg * 8 + 5]) * a.scale);
          hk.w = pack_bf16x2(__uint_as_float(kv[gg * 8 + 6]) * a.scale, __uint_as_float(kv[gg * 8 + 7]) * a.scale);
          hv.x = pack_bf16x2(__uint_as_float(vv[gg * 8 + 0]), __uint_as_float(vv[gg * 8 + 1]));
          hv.y = pack_bf16x2(__uint_as_float(vv[gg * 8 + 2]), __uint_as_float(vv[gg * 8 + 3]));
          hv.z = pack_bf16x2(__uint_as_float(vv[gg * 8 + 4]), __uint_as_float(vv[gg * 8 + 5]));
          hv.w = pack_bf16x2(__uint_as_float(vv[gg * 8 + 6]), __uint_as_float(vv[gg * 8 + 7]));
          *reinterpret_cast<uint4*>(dk + c * 32 + gg * 8) = hk;
          *reinterpret_cast<uint4*>(dv + c * 32 + gg * 8) = hv;
        }
      }
      if (tracer) BWD_TRACE(w.n_block, kTrEpiEnd, 0);
    }
  } else if (warp >= 12) {
    // ------------------------------------------------------------ dQ read-out
    // dQ of a step: TMEM -> registers -> swizzled fp32 box -> TMA reduce-add
    // into the fp32 accumulator.  Rows past T add zeros (P is 0 there).  With
    // two boxes chunks of 32 columns alternate, so staging chunk c only waits
    // for the reduction issued two chunks earlier; with one box, for the
    // previous.
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the block
    const uint32_t lb = tmem + ((uint32_t)(quarter * 32) << 16);
    const bool leader = warp == 12 && lane == 0;  // issues the TMA reductions
    bool ok = true;
    int chunk = 0;
    uint32_t g = 0;
    for (int it = blockIdx.x; it < n_virt; it += gridDim.x) {
      const Item w = decode(it);
      if (!w.valid) continue;
      const bool tr_on = a.trace != nullptr && w.bh == a.trace_bh;
      (void)tr_on;
      for (int tt = 0; tt < w.steps; ++tt, ++g) {
        const int q0 = (w.i_start + tt) * BQ;
        if (ok && !mbar_wait_warp(dq_full, g & 1u, a.status, kErrWaitTimeoutAccum, 322)) ok = false;
        if (leader) BWD_TRACE(w.n_block, kTrDqFull, tt);
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c, ++chunk) {
          uint32_t v[32];
          if (ok) {
            tc_fence_after();
            tmem_ld_32x32b_x32_async(lb + Cfg::kDQ + c * 32, v);
            tmem_wait_ld_regs<32>(v);
          }
          if (c == D / 32 - 1) {
            tc_fence_before();
            mbar_arrive(dq_free);  // the dQ buffer may be overwritten
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
            tma_reduce_add_2d(&tm_dq, box, w.h * D + c * 32, w.row0 + q0);
            bulk_commit_group();
          }
        }
        if (leader) BWD_TRACE(w.n_block, kTrDqDone, tt);
      }
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
  // persistent: one CTA per SM walks the units (pairs of key blocks of one head)
  const long long items = (long long)(((p.f.T + BK - 1) / BK + 1) / 2) * p.f.B * p.f.H;
  static int sms_by_dev[64] = {0};
  int dev = 0;
  UHFS_CUDA_CHECK(cudaGetDevice(&dev));
  int& sms = sms_by_dev[dev & 63];
  if (sms == 0) UHFS_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int grid = (int)(items < sms ? items : sms);
  if (grid <= 0) return;
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
