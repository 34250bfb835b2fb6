// Flash-attention forward on the 5th-generation tensor core (tcgen05 + TMEM).
//
// One CTA computes 128 query rows of one (batch, head) and walks the key /
// value sequence in blocks of 128 (causal: up to the diagonal).
//
//   warp 0      TMA producer: Q once, then K_j / V_j into a 2-stage ring
//               (128B-swizzled, no multicast)
//   warp 1      TMEM allocator + MMA issuer (one elected thread):
//                 S_j   = Q K_j^T   (M=128, N=128, K=D)      -> TMEM S[j%2]
//                 O_j   = P_j V_j   (M=128, N=D,   K=128)    -> TMEM O[j%2]
//   warps 2..5  softmax: thread r owns query row r (= TMEM lane r); it reads
//               its S row from TMEM, keeps the running max / sum and the
//               output accumulator in registers (exp2 domain), writes P_j as
//               bf16 into a swizzled shared tile (the A operand of the PV MMA)
//               and folds O_j into its accumulator with the online-softmax
//               rescale.  Finally O / l and the log2-domain LSE are stored.
//
// S and O are double-buffered in TMEM, P in shared memory, so the MMA of
// block j+1 overlaps the softmax of block j.  Every mbarrier wait is bounded.
// Reference: the single-head fp32 kernel cuda/kernels.cu:147-188 and the
// Python attention of nn.py:229-271.
#include <cudaTypedefs.h>

#include <stdexcept>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace uhfs {

CUtensorMap make_tmap_bf16_2d(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                              uint32_t box_inner, uint32_t box_outer);

namespace {

constexpr int BQ = 128;   // query rows per CTA
constexpr int BKV = 128;  // keys per block
constexpr int kThreads = 192;
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct FaCfg {
  static constexpr int kQBytes = BQ * D * 2;
  static constexpr int kKBytes = BKV * D * 2;
  static constexpr int kVBytes = BKV * D * 2;
  static constexpr int kPBytes = BQ * BKV * 2;
  static constexpr int kStageBytes = kKBytes + kVBytes;
  static constexpr int kPBuffers = (D == 64) ? 2 : 1;
  static constexpr int kSmem = 1024 + kQBytes + 2 * kStageBytes + kPBuffers * kPBytes + 256;
  static constexpr uint32_t kSCol = 0;            // S[2]: columns [0, 256)
  static constexpr uint32_t kOCol = 2 * BKV;      // O[2]: columns [256, 256 + 2D)
  static constexpr uint32_t kTmemCols = 512;
};

struct FaTcArgs {
  int B, H, T, D;
  long long F;            // H * D (columns per q / k / v section)
  float sl2;              // softmax scale * log2(e)
  int causal;
  __nv_bfloat16* o;
  long long o_stride_t;   // elements between tokens of o (rows are [b*T + t])
  float* lse;             // [B, H, T] (log2 domain)
  DeviceStatus* status;
};

// 32 TMEM columns of this thread's lane.
__device__ __forceinline__ void tld32(uint32_t taddr, float* v) { tmem_ld_32x32b_x32(taddr, v); }

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    fa_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, const FaTcArgs a) {
  using Cfg = FaCfg<D>;
  constexpr int KD = D / 64;  // 64-column sub-tiles along the head dim
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + Cfg::kQBytes;                      // [2 stages][K | V]
  uint8_t* sP = sKV + 2 * Cfg::kStageBytes;              // [kPBuffers][2 sub-tiles of 128 x 64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + Cfg::kPBuffers * Cfg::kPBytes);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* s_free = bars + 7;    // [2]
  uint64_t* p_full = bars + 9;    // [2]
  uint64_t* o_full = bars + 11;   // [2]
  uint64_t* o_free = bars + 13;   // [2]
  uint64_t* done = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y;
  const int b = bh / a.H, h = bh % a.H;
  const int m_block = gridDim.x - 1 - blockIdx.x;  // longest (causal) rows first
  const int m0 = m_block * BQ;
  const int T = a.T;
  const int n_end = a.causal ? min(T, m0 + BQ) : T;
  const int nblocks = (n_end + BKV - 1) / BKV;
  const int row0 = b * T;  // first row of this batch in the [B*T, 3F] matrix

  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_qkv);
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 128);
    }
    mbar_init(done, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one_sync()) {
      mbar_arrive_expect_tx(q_full, Cfg::kQBytes);
      for (int kd = 0; kd < KD; ++kd)
        tma_load_2d(sQ + kd * (BQ * 128), &tm_qkv, q_full, (int)(h * D + kd * 64), row0 + m0);
      uint32_t issued_phase[2] = {0, 0};
      bool issued[2] = {false, false};
      bool ok = true;
      for (int j = 0; j < nblocks && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait_bounded(&kv_empty[st], ph ^ 1u, a.status, kErrWaitTimeoutEmpty, 200)) {
          ok = false;
          break;
        }
        uint8_t* sK = sKV + st * Cfg::kStageBytes;
        uint8_t* sV = sK + Cfg::kKBytes;
        mbar_arrive_expect_tx(&kv_full[st], Cfg::kStageBytes);
        const int r = row0 + j * BKV;
        for (int kd = 0; kd < KD; ++kd) {
          tma_load_2d(sK + kd * (BKV * 128), &tm_qkv, &kv_full[st], (int)(a.F + h * D + kd * 64), r);
          tma_load_2d(sV + kd * (BKV * 128), &tm_qkv, &kv_full[st], (int)(2 * a.F + h * D + kd * 64), r);
        }
        issued[st] = true;
        issued_phase[st] = ph;
      }
      mbar_wait_bounded(q_full, 0, a.status, kErrWaitTimeoutFull, 201);
      for (int s = 0; s < 2; ++s)
        if (issued[s]) mbar_wait_bounded(&kv_full[s], issued_phase[s], a.status, kErrWaitTimeoutFull, 202);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one_sync()) {
      constexpr uint32_t idesc_s = make_idesc(1, 0, 0, BQ, BKV);  // Q K-major, K K-major
      constexpr uint32_t idesc_o = make_idesc(1, 0, 1, BQ, D);    // P K-major, V MN-major
      bool ok = mbar_wait_bounded(q_full, 0, a.status, kErrWaitTimeoutFull, 210);
      const uint32_t q_base = smem_u32(sQ);
      auto issue_pv = [&](int jj) -> bool {
        const int st = jj & 1;
        const int ob = jj & 1;
        const uint32_t ph = (jj >> 1) & 1;
        const int pb = jj % Cfg::kPBuffers;
        if (!mbar_wait_bounded(&p_full[jj & 1], ph, a.status, kErrWaitTimeoutAccum, 211)) return false;
        if (!mbar_wait_bounded(&o_free[ob], ph ^ 1u, a.status, kErrWaitTimeoutAccum, 212)) return false;
        tc_fence_after();
        const uint32_t p_base = smem_u32(sP + pb * Cfg::kPBytes);
        const uint32_t v_base = smem_u32(sKV + st * Cfg::kStageBytes + Cfg::kKBytes);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk) {
          const uint64_t ad = make_smem_desc(p_base + (kk >> 2) * (BQ * 128) + (kk & 3) * 32, 16, 1024, kSwizzle128B);
          const uint64_t bd = make_smem_desc(v_base + kk * 16 * 128, BKV * 128, 1024, kSwizzle128B);
          tc_mma_f16(tmem + Cfg::kOCol + ob * D, ad, bd, idesc_o, kk > 0 ? 1u : 0u);
        }
        tc_commit(&o_full[ob]);
        tc_commit(&kv_empty[st]);
        return true;
      };
      for (int j = 0; j < nblocks && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait_bounded(&kv_full[st], ph, a.status, kErrWaitTimeoutFull, 213) ||
            !mbar_wait_bounded(&s_free[st], ph ^ 1u, a.status, kErrWaitTimeoutAccum, 214)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_base = smem_u32(sKV + st * Cfg::kStageBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t sub = (kk >> 2) * (BQ * 128), off = (kk & 3) * 32;
          const uint64_t ad = make_smem_desc(q_base + sub + off, 16, 1024, kSwizzle128B);
          const uint64_t bd = make_smem_desc(k_base + (kk >> 2) * (BKV * 128) + off, 16, 1024, kSwizzle128B);
          tc_mma_f16(tmem + Cfg::kSCol + st * BKV, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[st]);
        if (j >= 1 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok && nblocks > 0) issue_pv(nblocks - 1);
      tc_commit(done);
      mbar_wait_bounded(done, 0, a.status, kErrWaitTimeoutAccum, 215);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;   // query row within the tile == TMEM lane
    const int q = m0 + r;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    float o_acc[D];
#pragma unroll
    for (int i = 0; i < D; ++i) o_acc[i] = 0.f;
    float m_run = -INFINITY, l_run = 0.f, alpha_pending = 1.f;
    bool ok = true;
    auto fold_o = [&](int jj, float alpha) -> bool {
      const int ob = jj & 1;
      const uint32_t ph = (jj >> 1) & 1;
      if (!mbar_wait_warp(&o_full[ob], ph, a.status, kErrWaitTimeoutAccum, 220)) return false;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float v[32];
        tld32(lane_base + Cfg::kOCol + ob * D + c * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) o_acc[c * 32 + i] = o_acc[c * 32 + i] * alpha + v[i];
      }
      tc_fence_before();
      mbar_arrive(&o_free[ob]);
      return true;
    };
    for (int j = 0; j < nblocks && ok; ++j) {
      const int st = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      const int n0 = j * BKV;
      if (!mbar_wait_warp(&s_full[st], ph, a.status, kErrWaitTimeoutAccum, 221)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool need_mask = (a.causal && n0 + BKV - 1 > m0) || (n0 + BKV > T);
      const uint32_t s_base = lane_base + Cfg::kSCol + st * BKV;
      // pass 1: row max
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < BKV / 32; ++c) {
        float v[32];
        tld32(s_base + c * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float x = v[i] * a.sl2;
          const int key = n0 + c * 32 + i;
          if (need_mask && (key >= T || (a.causal && key > q))) x = -INFINITY;
          mx = fmaxf(mx, x);
        }
      }
      const float m_new = fmaxf(m_run, mx);
      const float base = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = exp2f(m_run - base);
      // the P buffer of block j is free once the PV MMA of block j - kPBuffers retired
      if (j >= Cfg::kPBuffers) {
        const int prev = j - Cfg::kPBuffers;
        if (!mbar_wait_warp(&o_full[prev & 1], (prev >> 1) & 1, a.status, kErrWaitTimeoutAccum, 222)) {
          ok = false;
          break;
        }
      }
      // pass 2: p = exp2(s - m), row sum, bf16 P row into the swizzled A tile
      uint8_t* prow = sP + (j % Cfg::kPBuffers) * Cfg::kPBytes;
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < BKV / 32; ++c) {
        float v[32];
        tld32(s_base + c * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float x = v[i] * a.sl2;
          const int key = n0 + c * 32 + i;
          if (need_mask && (key >= T || (a.causal && key > q))) x = -INFINITY;
          v[i] = exp2f(x - base);
          rs += v[i];
        }
        // 32 keys = 4 chunks of 8 -> 16-byte stores at swizzled positions
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int chunk = c * 4 + g;          // 0..15 over the 128 keys
          const int sub = chunk >> 3, ch = chunk & 7;
          __align__(16) __nv_bfloat162 hv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) hv[e] = __floats2bfloat162_rn(v[g * 8 + 2 * e], v[g * 8 + 2 * e + 1]);
          uint8_t* dst = prow + sub * (BQ * 128) + r * 128 + ((ch ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<uint4*>(hv);
        }
      }
      tc_fence_before();
      mbar_arrive(&s_free[st]);  // S[st] fully read
      fence_proxy_async_smem();  // make the P stores visible to the tensor core
      mbar_arrive(&p_full[st]);
      l_run = l_run * alpha + rs;
      m_run = m_new;
      if (j >= 1 && !fold_o(j - 1, alpha_pending)) {
        ok = false;
        break;
      }
      alpha_pending = alpha;
    }
    if (ok && nblocks > 0) ok = fold_o(nblocks - 1, alpha_pending);
    // epilogue: O / l and LSE
    if (ok && q < T) {
      const float inv = l_run > 0.f ? 1.0f / l_run : 0.f;
      __nv_bfloat16* orow = a.o + (long long)(b * T + q) * a.o_stride_t + h * D;
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        __align__(16) __nv_bfloat162 hv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) hv[e] = __floats2bfloat162_rn(o_acc[c * 8 + 2 * e] * inv, o_acc[c * 8 + 2 * e + 1] * inv);
        *reinterpret_cast<uint4*>(orow + c * 8) = *reinterpret_cast<uint4*>(hv);
      }
      a.lse[(long long)bh * T + q] = l_run > 0.f ? m_run + log2f(l_run) : INFINITY;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

template <int D>
void launch_fwd(const AttnParams& p, cudaStream_t s) {
  using Cfg = FaCfg<D>;
  static bool attr = false;
  if (!attr) {
    UHFS_CUDA_CHECK(cudaFuncSetAttribute(fa_fwd_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem));
    attr = true;
  }
  const long long F = (long long)p.H * D;
  // q, k, v are column blocks of one [B*T, 3F] matrix (the fused projection)
  const long long row_stride = p.q_stride_t;
  CUtensorMap tm = make_tmap_bf16_2d(p.q, (uint64_t)(3 * F), (uint64_t)p.B * p.T, (uint64_t)row_stride, 64, 128);
  FaTcArgs a{};
  a.B = p.B;
  a.H = p.H;
  a.T = p.T;
  a.D = D;
  a.F = F;
  a.sl2 = p.scale * kLog2e;
  a.causal = p.causal;
  a.o = p.o;
  a.o_stride_t = p.o_stride_t;
  a.lse = p.lse;
  a.status = device_status_ptr();
  dim3 grid((p.T + BQ - 1) / BQ, p.B * p.H);
  fa_fwd_tc_kernel<D><<<grid, kThreads, Cfg::kSmem, s>>>(tm, a);
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
         (p.o_stride_t % 8) == 0;
}

void flash_attn_fwd_tc(const AttnParams& p, cudaStream_t s) {
  if (p.D == 64) launch_fwd<64>(p, s);
  else launch_fwd<128>(p, s);
}

}  // namespace uhfs
