// Flash-attention forward on the 5th-generation tensor core (tcgen05 + TMEM).
//
// One CTA owns 256 query rows of one (batch, head) as two 128-row tiles A and
// B, and walks the key / value sequence in blocks of 128 (causal: up to the
// diagonal; tile B has one block more than tile A).
//
//   warps 0..3  softmax of tile A, warps 4..7 softmax of tile B (below)
//   warp 8      TMA producer: Q_A, Q_B once; then K_0, V_0, K_1, V_1, ...
//               through a ring of 128 x D slots (128B-swizzled, no multicast)
//   warp 9      TMEM allocator + MMA issuer (one elected thread), ordering
//                 S_A(j) | S_B(j) | PV_A(j-1) | PV_B(j-1)
//               so the next S is computed while the softmax warpgroups still
//               work on the current block:
//                 S_t(j)  = Q_t K_j^T   (M=128, N=128, K=D)   -> TMEM S_t
//                 O_t    += P_t(j) V_j  (M=128, N=D,   K=128) -> TMEM O_t
//   softmax     thread r of a softmax warpgroup owns query row r of its
//               tile (= TMEM lane r; warp w reads lanes 32*(w%4)..+31).  It loads its whole S row
//               (128 columns) with four TMEM loads and one wait, frees S for
//               the next block, and computes P = exp2(S*scale*log2e - m) in
//               registers.  The running max m is only raised when the block
//               max exceeds it by more than kRescaleThreshold (log2 units);
//               then, and only then, O in TMEM is rescaled by that warp before
//               the next PV product.  P goes to a 128B-swizzled shared tile
//               (the A operand of PV).  At the end O / l and the log2-domain
//               LSE are written.
//
// Registers: 384 threads launch with 168 each; warpgroup 2 (producer, MMA,
// two idle warps) gives back down to 96 and the softmax warpgroups take 200,
// within the launch total (the host checks the launch count).
// Every mbarrier wait is bounded; waits that precede warp-collective TMEM
// instructions return a warp-uniform result.
// Reference: the single-head fp32 kernel cuda/kernels.cu:147-188 and the
// Python attention of nn.py:229-271.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <stdexcept>
#include <string>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace uhfs {

CUtensorMap make_tmap_bf16_2d(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                              uint32_t box_inner, uint32_t box_outer);

namespace {

constexpr int BQ = 128;   // query rows per tile (two tiles per CTA)
constexpr int BKV = 128;  // keys per block
constexpr int kThreads = 384;       // 3 warpgroups
constexpr int kLaunchRegs = 168;    // 65536 / 384, rounded down to 8
constexpr int kSoftmaxRegs = 200;
constexpr int kServiceRegs = 104;   // 2 * 128 * 200 + 128 * 104 == 384 * 168
static_assert(2 * 128 * kSoftmaxRegs + 128 * kServiceRegs <= kThreads * kLaunchRegs, "register split");
constexpr float kLog2e = 1.4426950408889634f;
// P = exp2(s - m) stays below 2^kRescaleThreshold when m is kept stale.
constexpr float kRescaleThreshold = 8.0f;
// default number of polynomial pairs per 8 in the forward softmax
constexpr int kDefaultPolyPairs = 0;

// P placement.  D = 64: P (bf16 pairs, 64 columns per tile) lives in TMEM
// next to S and O, and PV reads it there (tcgen05.mma with A from TMEM), so
// the only shared-memory operands are Q, K and V -- an S product of M=N=128,
// K=16 reads 8 KB of operands per 68 tensor cycles, close to the 128 B/clk
// of shared memory, which made the shared-memory P tile (written by the
// softmax, read by PV) the limit of the loop.  D = 128: TMEM is full with S
// and O, P stays a 128B-swizzled shared tile.
template <int D>
struct FwdCfg {
  static constexpr bool kPTmem = (D == 64);
  static constexpr int kTile = 128 * D * 2;            // one 128 x D bf16 tile (D/64 swizzled sub-tiles)
  static constexpr int kSlots = (D == 64) ? 6 : 3;      // K / V ring
  static constexpr int kPBytes = BQ * BKV * 2;          // P tile (2 sub-tiles of 128 x 64)
  static constexpr int kBars = 2 + 2 * kSlots + 2 * 5 + 1;
  static constexpr int kSmem = 1024 + 2 * kTile + kSlots * kTile + (kPTmem ? 0 : 2 * kPBytes) + kBars * 8 + 16;
  static constexpr uint32_t kSCol = 0;                  // S_A [0,128), S_B [128,256)
  static constexpr uint32_t kOCol = 2 * BKV;            // O_A, O_B: D columns each
  static constexpr uint32_t kPCol = 2 * BKV + 2 * D;    // D = 64: P_A, P_B: 64 columns each
  static constexpr uint32_t kTmemCols = 512;
  static_assert(!kPTmem || kPCol + 2 * (BKV / 2) <= kTmemCols, "P columns");
  static_assert(kSmem <= 227 * 1024, "attention forward shared memory");
};

// Optional per-block clock stamps (clock64) for the CTAs of head 0 of batch 0:
// trace[(cta * kTraceEvents + event) * kTraceSteps + block], cta = blockIdx.x.
// Off (nullptr) unless a buffer is installed with set_attn_fwd_trace.
constexpr int kTraceEvents = 16, kTraceSteps = 64;
enum FwdTraceEvent {
  kTrStart = 0, kTrQFull, kTrKFull, kTrIssueS, kTrIssuePv, kTrSFullA, kTrSRegsA, kTrExpA, kTrODoneA, kTrPFullA,
  kTrSFullB, kTrPFullB, kTrEpiStart, kTrEpiEnd
};
unsigned long long* g_fwd_trace = nullptr;

struct FwdArgs {
  int H, T, BH;           // heads, sequence length, batch * heads
  long long F;            // H * D (columns per q / k / v section)
  float sl2;              // softmax scale * log2(e)
  int causal;
  __nv_bfloat16* o;
  long long o_stride_t;   // elements between tokens of o (rows are [b*T + t])
  float* lse;             // [B, H, T] (log2 domain)
  DeviceStatus* status;
  unsigned long long* trace;
  int trace_bh;  // (batch, head) whose CTAs are traced (UHFS_ATTN_TRACE_BH, trace builds)
};

// Compiled in only with -DUHFS_ATTN_TRACE (UNDERHFS_ATTN_TRACE=1 at build
// time); the product build has no stamps and no trace pointer test.
#ifdef UHFS_ATTN_TRACE
#define FWD_TRACE(cta, ev, step)                                                                         \
  do {                                                                                                   \
    if (tr_on && (step) < kTraceSteps)                                                                   \
      a.trace[((long long)(cta) * kTraceEvents + (ev)) * kTraceSteps + (step)] = (unsigned long long)clock64(); \
  } while (0)
#else
#define FWD_TRACE(cta, ev, step) \
  do {                           \
  } while (0)
#endif

// kPoly: of every 8 consecutive score pairs of a row, the first kPoly use
// exp2_poly3_x2 (packed FMA-pipe polynomial) instead of ex2.approx (MUFU), so
// the exponentials of a block split between the two pipes
// (UHFS_ATTN_POLY=0|2|3|4 selects it; 0 = MUFU only).
template <int D, int kPoly>
__global__ void __launch_bounds__(kThreads, 1)
    fa_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, const FwdArgs a) {
  using Cfg = FwdCfg<D>;
  constexpr int KD = D / 64;  // 64-column sub-tiles along the head dim
  constexpr int NS = Cfg::kSlots;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align1024(smem_raw);
  uint8_t* sQ = smem;                               // [2 tiles]
  uint8_t* sRing = sQ + 2 * Cfg::kTile;             // [NS slots]
  uint8_t* sP = sRing + NS * Cfg::kTile;            // [2 tiles] (D = 128 only)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + (Cfg::kPTmem ? 0 : 2 * Cfg::kPBytes));
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 1;        // the S products of an item are done with Q
  uint64_t* slot_full = bars + 2;
  uint64_t* slot_empty = slot_full + NS;
  uint64_t* s_full = slot_empty + NS;  // [2]
  uint64_t* s_free = s_full + 2;       // [2]
  uint64_t* p_full = s_free + 2;       // [2]
  uint64_t* o_done = p_full + 2;       // [2]
  uint64_t* o_free = o_done + 2;       // [2] an item's O was read out: the next item's first PV may overwrite it
  uint64_t* done = o_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = a.T;
  const int kv_blocks = (T + BKV - 1) / BKV;
  const int n_mblocks = (T + 2 * BQ - 1) / (2 * BQ);
  const int n_items = n_mblocks * a.BH;
  // work item -> (batch, head, first query row, key blocks of tile A / B);
  // the longest (causal) query blocks come first in item order
  struct Item {
    int bh, b, h, m0, nA, nB, cta;
  };
  auto decode = [&](int it) {
    Item w;
    const int mb = n_mblocks - 1 - it / a.BH;
    w.bh = it % a.BH;
    w.b = w.bh / a.H;
    w.h = w.bh % a.H;
    w.m0 = mb * (2 * BQ);
    w.nA = a.causal ? min(kv_blocks, w.m0 / BKV + 1) : kv_blocks;
    w.nB = a.causal ? min(kv_blocks, w.m0 / BKV + 2) : kv_blocks;
    w.cta = n_mblocks - 1 - mb;  // trace index (query blocks from the last)
    return w;
  };

  constexpr int kProducerWarp = 8, kMmaWarp = 9;
  if (warp == kProducerWarp && lane == 0) {
    tma_prefetch_desc(&tm_qkv);
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&slot_full[i], 1);
      mbar_init(&slot_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
      mbar_init(&o_free[i], 128);
    }
    mbar_init(done, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
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
    if (elect_one_sync()) {
      uint32_t L = 0;  // K / V loads issued (ring position, continues across items)
      uint32_t k = 0;  // items of this CTA
      bool ok = true;
      for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x, ++k) {
        const Item w = decode(it);
        const bool tr_on = a.trace != nullptr && w.bh == a.trace_bh;
        (void)tr_on;
        // Q of the previous item is no longer read by the tensor core
        if (!mbar_wait_bounded(q_empty, (k & 1u) ^ 1u, a.status, kErrWaitTimeoutEmpty, 203)) break;
        FWD_TRACE(w.cta, kTrStart, 0);
        const int row0 = w.b * T;
        mbar_arrive_expect_tx(q_full, 2 * Cfg::kTile);
        for (int t = 0; t < 2; ++t)
          for (int kd = 0; kd < KD; ++kd)
            tma_load_2d(sQ + t * Cfg::kTile + kd * (BQ * 128), &tm_qkv, q_full, (int)(w.h * D + kd * 64),
                        row0 + w.m0 + t * BQ);
        for (int i = 0; i < 2 * w.nB; ++i, ++L) {  // K_0, V_0, K_1, V_1, ...
          const uint32_t slot = L % NS, use = L / NS;
          if (!mbar_wait_bounded(&slot_empty[slot], (use & 1u) ^ 1u, a.status, kErrWaitTimeoutEmpty, 200)) {
            ok = false;
            break;
          }
          uint8_t* dst = sRing + slot * Cfg::kTile;
          mbar_arrive_expect_tx(&slot_full[slot], Cfg::kTile);
          const int col = (int)((i & 1) ? 2 * a.F : a.F) + w.h * D;
          const int row = row0 + (i >> 1) * BKV;
          for (int kd = 0; kd < KD; ++kd)
            tma_load_2d(dst + kd * (BKV * 128), &tm_qkv, &slot_full[slot], col + kd * 64, row);
        }
      }
      // drain: every issued copy lands before the CTA exits
      if (k > 0) mbar_wait_bounded(q_full, (k - 1) & 1u, a.status, kErrWaitTimeoutFull, 201);
      for (uint32_t i = (L > (uint32_t)NS ? L - NS : 0); i < L; ++i)
        mbar_wait_bounded(&slot_full[i % NS], (i / NS) & 1u, a.status, kErrWaitTimeoutFull, 202);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one_sync()) {
      constexpr uint32_t idesc_s = make_idesc(1, 0, 0, BQ, BKV);  // Q K-major, K K-major
      constexpr uint32_t idesc_o = make_idesc(1, 0, 1, BQ, D);    // P K-major, V MN-major
      // descriptors with a zero start address; the start field (address >> 4)
      // is added per operand and stays below 2^14 (shared memory < 256 KB)
      const uint64_t kmaj = make_smem_desc(0, 16, 1024, kSwizzle128B);
      const uint64_t mnmaj = make_smem_desc(0, BKV * 128, 1024, kSwizzle128B);
      const uint32_t q16 = smem_u32(sQ) >> 4, ring16 = smem_u32(sRing) >> 4, p16 = smem_u32(sP) >> 4;
      uint32_t L = 0;                      // ring position of the current item's K_0
      uint32_t s_cnt[2] = {0u, 0u};        // S products issued per tile (all items)
      uint32_t pv_cnt[2] = {0u, 0u};       // PV products issued per tile (all items)
      uint32_t k = 0;
      bool ok = true;
      auto slot_of = [&](uint32_t pos) { return pos % NS; };
      auto phase_of = [&](uint32_t pos) { return (pos / NS) & 1u; };
      for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x, ++k) {
        const Item w = decode(it);
        const bool tr_on = a.trace != nullptr && w.bh == a.trace_bh;
        (void)tr_on;
        auto issue_s = [&](int t, int j) -> bool {
          if (s_cnt[t] > 0 &&
              !mbar_wait_bounded(&s_free[t], (s_cnt[t] - 1) & 1u, a.status, kErrWaitTimeoutAccum, 211))
            return false;
          tc_fence_after();
          const uint64_t ad = kmaj + q16 + t * (Cfg::kTile >> 4);
          const uint64_t bd = kmaj + ring16 + slot_of(L + 2 * j) * (Cfg::kTile >> 4);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = ((kk >> 2) * (128 * 128) + (kk & 3) * 32) >> 4;
            tc_mma_f16(tmem + Cfg::kSCol + t * BKV, ad + off, bd + off, idesc_s, kk > 0 ? 1u : 0u);
          }
          tc_commit(&s_full[t]);
          ++s_cnt[t];
          return true;
        };
        auto issue_pv = [&](int t, int j) -> bool {
          if (!mbar_wait_bounded(&p_full[t], pv_cnt[t] & 1u, a.status, kErrWaitTimeoutAccum, 212) ||
              !mbar_wait_bounded(&slot_full[slot_of(L + 2 * j + 1)], phase_of(L + 2 * j + 1), a.status,
                                 kErrWaitTimeoutFull, 213))
            return false;
          // the previous item's O_t must have been read out before this item's first PV overwrites it
          if (j == 0 && k > 0 && !mbar_wait_bounded(&o_free[t], (k - 1) & 1u, a.status, kErrWaitTimeoutAccum, 216))
            return false;
          tc_fence_after();
          const uint64_t ad = kmaj + p16 + t * (Cfg::kPBytes >> 4);
          const uint64_t bd = mnmaj + ring16 + slot_of(L + 2 * j + 1) * (Cfg::kTile >> 4);
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk) {
            const uint32_t acc = (j > 0 || kk > 0) ? 1u : 0u;
            if constexpr (Cfg::kPTmem) {
              // A = P_t from TMEM: keys [16 kk, 16 kk + 16) are columns [8 kk, 8 kk + 8)
              tc_mma_f16_ts(tmem + Cfg::kOCol + t * D, tmem + Cfg::kPCol + t * (BKV / 2) + (uint32_t)(kk * 8),
                            bd + ((kk * 16 * 128) >> 4), idesc_o, acc);
            } else {
              const uint32_t aoff = ((kk >> 2) * (BQ * 128) + (kk & 3) * 32) >> 4;
              tc_mma_f16(tmem + Cfg::kOCol + t * D, ad + aoff, bd + ((kk * 16 * 128) >> 4), idesc_o, acc);
            }
          }
          tc_commit(&o_done[t]);
          ++pv_cnt[t];
          return true;
        };
        if (!mbar_wait_bounded(q_full, k & 1u, a.status, kErrWaitTimeoutFull, 210)) break;
        FWD_TRACE(w.cta, kTrQFull, 0);
        // S of block j for both tiles goes ahead of PV of block j-1: a softmax
        // warpgroup frees S as soon as it holds the row in registers, so the
        // next S is ready when it finishes P, and the PV product overlaps the
        // next block's exponentials instead of sitting on the critical path.
        for (int j = 0; j < w.nB && ok; ++j) {
          if (!mbar_wait_bounded(&slot_full[slot_of(L + 2 * j)], phase_of(L + 2 * j), a.status, kErrWaitTimeoutFull,
                                 214)) {
            ok = false;
            break;
          }
          FWD_TRACE(w.cta, kTrKFull, j);
          if ((j < w.nA && !issue_s(0, j)) || !issue_s(1, j)) {
            ok = false;
            break;
          }
          tc_commit(&slot_empty[slot_of(L + 2 * j)]);  // K_j read by both tiles
          if (j == w.nB - 1) tc_commit(q_empty);        // the item's last S products: Q is free
          FWD_TRACE(w.cta, kTrIssueS, j);
          if (j >= 1) {
            if ((j - 1 < w.nA && !issue_pv(0, j - 1)) || !issue_pv(1, j - 1)) {
              ok = false;
              break;
            }
            tc_commit(&slot_empty[slot_of(L + 2 * (j - 1) + 1)]);  // V_{j-1} read by both tiles
            FWD_TRACE(w.cta, kTrIssuePv, j - 1);
          }
        }
        if (ok && w.nB > 0) {
          if ((w.nB - 1 < w.nA && !issue_pv(0, w.nB - 1)) || !issue_pv(1, w.nB - 1)) ok = false;
          else tc_commit(&slot_empty[slot_of(L + 2 * (w.nB - 1) + 1)]);
        }
        L += 2 * w.nB;
      }
      tc_commit(done);
      mbar_wait_bounded(done, 0, a.status, kErrWaitTimeoutAccum, 215);
    }
  } else if (warp < 8) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
    // ------------------------------------------------------------ softmax
    const int t = warp >> 2;             // tile 0 (A) or 1 (B)
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;   // query row within the tile == TMEM lane
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    const uint32_t s_col = lane_base + Cfg::kSCol + t * BKV;
    const uint32_t o_col = lane_base + Cfg::kOCol + t * D;
    const uint32_t p_col = lane_base + Cfg::kPCol + t * (BKV / 2);
    uint8_t* prow = sP + t * Cfg::kPBytes + r * 128;
    const bool tracer = quarter == 0 && lane == 0;  // warp 0 (tile A) and warp 4 (tile B)
    (void)tracer;
    uint32_t blk = 0;  // key blocks of this tile processed (all items)
    bool ok = true;
    for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
      const Item w = decode(it);
      const bool tr_on = a.trace != nullptr && w.bh == a.trace_bh;
      (void)tr_on;
      const int q = w.m0 + t * BQ + r;
      const int nblk = t ? w.nB : w.nA;
      const int key_limit = a.causal ? min(q + 1, T) : T;  // keys [0, key_limit) are visible
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < nblk && ok; ++j, ++blk) {
        if (!mbar_wait_warp(&s_full[t], blk & 1u, a.status, kErrWaitTimeoutAccum, 220)) {
          ok = false;
          break;
        }
        if (tracer) FWD_TRACE(w.cta, t == 0 ? kTrSFullA : kTrSFullB, j);
        tc_fence_after();
        uint32_t sr[BKV];
#pragma unroll
        for (int c = 0; c < BKV / 32; ++c) tmem_ld_32x32b_x32_async(s_col + c * 32, sr + c * 32);
        tmem_wait_ld_regs<BKV>(sr);
        tc_fence_before();
        mbar_arrive(&s_free[t]);  // S_t may be overwritten by the next block
        if (tracer && t == 0) FWD_TRACE(w.cta, kTrSRegsA, j);
        const int lim = key_limit - j * BKV;  // visible columns of this block: [0, lim)
        if (lim < BKV) {
#pragma unroll
          for (int i = 0; i < BKV; ++i)
            if (i >= lim) sr[i] = __float_as_uint(-INFINITY);
        }
        // row max: four independent chains of three-input max (two scores each)
        float mx4[4] = {__uint_as_float(sr[0]), __uint_as_float(sr[1]), __uint_as_float(sr[2]),
                        __uint_as_float(sr[3])};
#pragma unroll
        for (int i = 4; i < BKV; i += 8) {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            mx4[e] = max3f(mx4[e], __uint_as_float(sr[i + e]), __uint_as_float(sr[i + 4 + e < BKV ? i + 4 + e : i + e]));
        }
        const float mx = max3f(mx4[0], mx4[1], fmaxf(mx4[2], mx4[3]));
        const float m_blk = mx * a.sl2;
        const bool rescale = m_blk > m_run + kRescaleThreshold;
        const float m_new = rescale ? m_blk : m_run;
        const float alpha = rescale ? ex2_approx(m_run - m_new) : 1.f;  // 0 while m_run = -inf
        const float base = (m_new == -INFINITY) ? 0.f : m_new;
        // P = exp2(S * scale * log2e - m): the scale and offset as packed fp32x2
        // FMAs, the row sum as packed adds into two accumulator pairs
        float2 rs2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        const float2 sl2x2 = make_float2(a.sl2, a.sl2), nbase = make_float2(-base, -base);
        uint32_t pk[BKV / 2];
#pragma unroll
        for (int i = 0; i < BKV / 2; ++i) {
          const float2 x =
              f2_fma(make_float2(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1])), sl2x2, nbase);
          float2 pr;
          if ((i & 7) < kPoly) {
            pr = exp2_poly3_x2(x);
          } else {
            pr.x = ex2_approx(x.x);
            pr.y = ex2_approx(x.y);
          }
          rs2[i & 1] = f2_add(rs2[i & 1], pr);
          pk[i] = pack_bf16x2(pr.x, pr.y);
        }
        const float2 rs = f2_add(rs2[0], rs2[1]);
        l_run = l_run * alpha + (rs.x + rs.y);
        m_run = m_new;
        if (tracer && t == 0) FWD_TRACE(w.cta, kTrExpA, j);
        // PV(j-1) finished: the P tile is free and O_t holds blocks < j
        if (j > 0) {
          if (!mbar_wait_warp(&o_done[t], (blk - 1) & 1u, a.status, kErrWaitTimeoutAccum, 221)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (tracer && t == 0) FWD_TRACE(w.cta, kTrODoneA, j);
          if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
              uint32_t ov[32];
              tmem_ld_32x32b_x32_async(o_col + c * 32, ov);
              tmem_wait_ld_regs<32>(ov);
#pragma unroll
              for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
              tmem_st_32x32b_x32(o_col + c * 32, ov);
            }
            tmem_wait_st();
          }
        }
        if constexpr (Cfg::kPTmem) {
          // P row -> TMEM lane r: column c holds keys 2c, 2c + 1
          tmem_st_32x32b_x32(p_col, pk);
          tmem_st_32x32b_x32(p_col + 32, pk + 32);
          tmem_wait_st();
        } else {
          // P row -> swizzled A tile: 16 chunks of 8 keys, chunk ch of sub-tile ch / 8
#pragma unroll
          for (int ch = 0; ch < 16; ++ch) {
            const int sub = ch >> 3, c8 = ch & 7;
            const uint4 v = make_uint4(pk[ch * 4], pk[ch * 4 + 1], pk[ch * 4 + 2], pk[ch * 4 + 3]);
            *reinterpret_cast<uint4*>(prow + sub * (BQ * 128) + ((c8 ^ (r & 7)) << 4)) = v;
          }
          fence_proxy_async_smem();  // P stores visible to the tensor core
        }
        tc_fence_before();  // P / O rescale TMEM stores ordered before the next MMA
        mbar_arrive(&p_full[t]);
        if (tracer) FWD_TRACE(w.cta, t == 0 ? kTrPFullA : kTrPFullB, j);
      }
      if (!ok) break;
      // the item's last PV
      if (!mbar_wait_warp(&o_done[t], (blk - 1) & 1u, a.status, kErrWaitTimeoutAccum, 222)) break;
      // epilogue: O / l and LSE (TMEM loads in every lane, stores for rows < T)
      if (tracer && t == 0) FWD_TRACE(w.cta, kTrEpiStart, 0);
      tc_fence_after();
      uint32_t ov[D];
#pragma unroll
      for (int c = 0; c < D / 32; ++c) tmem_ld_32x32b_x32_async(o_col + c * 32, ov + c * 32);
      tmem_wait_ld_regs<D>(ov);
      tc_fence_before();
      mbar_arrive(&o_free[t]);  // O_t may be overwritten by the next item
      const float inv = l_run > 0.f ? 1.0f / l_run : 0.f;
      if (q < T) {
        __nv_bfloat16* orow = a.o + (long long)(w.b * T + q) * a.o_stride_t + w.h * D;
#pragma unroll
        for (int g = 0; g < D / 8; ++g) {
          uint4 v;
          v.x = pack_bf16x2(__uint_as_float(ov[g * 8 + 0]) * inv, __uint_as_float(ov[g * 8 + 1]) * inv);
          v.y = pack_bf16x2(__uint_as_float(ov[g * 8 + 2]) * inv, __uint_as_float(ov[g * 8 + 3]) * inv);
          v.z = pack_bf16x2(__uint_as_float(ov[g * 8 + 4]) * inv, __uint_as_float(ov[g * 8 + 5]) * inv);
          v.w = pack_bf16x2(__uint_as_float(ov[g * 8 + 6]) * inv, __uint_as_float(ov[g * 8 + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + g * 8) = v;
        }
        a.lse[(long long)w.bh * T + q] = l_run > 0.f ? m_run + log2f(l_run) : INFINITY;
      }
      if (tracer && t == 0) FWD_TRACE(w.cta, kTrEpiEnd, 0);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

template <int D, int kPoly>
void launch_fwd(const AttnParams& p, cudaStream_t s) {
  using Cfg = FwdCfg<D>;
  static PerDeviceOnce once;
  once([] {
    UHFS_CUDA_CHECK(cudaFuncSetAttribute(fa_fwd_tc_kernel<D, kPoly>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::kSmem));
    // setmaxnreg redistributes exactly the launch allocation; any other
    // launch count would make the increase wait for registers that never come
    cudaFuncAttributes fa{};
    UHFS_CUDA_CHECK(cudaFuncGetAttributes(&fa, fa_fwd_tc_kernel<D, kPoly>));
    if (fa.numRegs != kLaunchRegs)
      throw std::runtime_error("fa_fwd_tc_kernel: compiled with " + std::to_string(fa.numRegs) +
                               " registers per thread, the register split needs " + std::to_string(kLaunchRegs));
  });
  const long long F = (long long)p.H * D;
  // q, k, v are column blocks of one [B*T, 3F] matrix (the fused projection)
  CUtensorMap tm = make_tmap_bf16_2d(p.q, (uint64_t)(3 * F), (uint64_t)p.B * p.T, (uint64_t)p.q_stride_t, 64, 128);
  FwdArgs a{};
  a.H = p.H;
  a.T = p.T;
  a.F = F;
  a.sl2 = p.scale * kLog2e;
  a.causal = p.causal;
  a.o = p.o;
  a.o_stride_t = p.o_stride_t;
  a.lse = p.lse;
  a.status = device_status_ptr();
  a.trace = g_fwd_trace;
#ifdef UHFS_ATTN_TRACE
  {
    const char* e = getenv("UHFS_ATTN_TRACE_BH");
    a.trace_bh = e != nullptr ? atoi(e) : 0;
  }
#endif
  a.BH = p.B * p.H;
  // persistent: one CTA per SM walks the (query block, head) items
  const long long items = (long long)((p.T + 2 * BQ - 1) / (2 * BQ)) * p.B * p.H;
  static int sms_by_dev[64] = {0};
  int dev = 0;
  UHFS_CUDA_CHECK(cudaGetDevice(&dev));
  int& sms = sms_by_dev[dev & 63];
  if (sms == 0) UHFS_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int grid = (int)(items < sms ? items : sms);
  if (grid <= 0) return;
  fa_fwd_tc_kernel<D, kPoly><<<grid, kThreads, Cfg::kSmem, s>>>(tm, a);
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

}  // namespace

bool flash_attn_fwd_tc_supported(const AttnParams& p) {
  // fused [B*T, 3F] layout: k = q + F, v = q + 2F, equal token strides, contiguous batches
  const long long F = (long long)p.H * p.D;
  return (p.D == 64 || p.D == 128) && p.k == p.q + F && p.v == p.q + 2 * F && p.q_stride_t == 3 * F &&
         p.k_stride_t == 3 * F && p.v_stride_t == 3 * F && p.q_stride_b == (long long)p.T * 3 * F &&
         p.o_stride_b == (long long)p.T * p.o_stride_t && (reinterpret_cast<uintptr_t>(p.q) & 15u) == 0 &&
         (reinterpret_cast<uintptr_t>(p.o) & 15u) == 0 && (p.o_stride_t % 8) == 0;
}

void set_attn_fwd_trace(unsigned long long* buf) {
#ifdef UHFS_ATTN_TRACE
  g_fwd_trace = buf;
#else
  if (buf != nullptr)
    throw std::runtime_error("set_attn_fwd_trace: the extension was built without UHFS_ATTN_TRACE "
                             "(rebuild with UNDERHFS_ATTN_TRACE=1)");
#endif
}

void flash_attn_fwd_tc(const AttnParams& p, cudaStream_t s) {
  // UHFS_ATTN_POLY: score pairs (of every 8) whose exponentials use the
  // FMA-pipe polynomial instead of MUFU
  static const int poly = [] {
    const char* e = getenv("UHFS_ATTN_POLY");
    const int v = e != nullptr ? atoi(e) : kDefaultPolyPairs;
    return (v == 0 || v == 2 || v == 3 || v == 4) ? v : kDefaultPolyPairs;
  }();
  auto go = [&](auto dtag) {
    constexpr int D = decltype(dtag)::value;
    switch (poly) {
      case 2: return launch_fwd<D, 2>(p, s);
      case 3: return launch_fwd<D, 3>(p, s);
      case 4: return launch_fwd<D, 4>(p, s);
      default: return launch_fwd<D, 0>(p, s);
    }
  };
  if (p.D == 64) go(std::integral_constant<int, 64>{});
  else go(std::integral_constant<int, 128>{});
}

}  // namespace uhfs
