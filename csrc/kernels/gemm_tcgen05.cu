// Persistent, warp-specialized bf16 GEMM on the sm_100a 5th-generation tensor
// core (tcgen05.mma kind::f16, fp32 accumulators in TMEM), fed by TMA.
//
//   C[M,N] = sum_k A(m,k) * B(n,k)      (+ fused epilogue)
//
// A and B are each either K-major (row-major with K contiguous) or MN-major
// (K rows, M/N contiguous).  This covers every Linear layout without a
// transpose copy:
//   forward  Y  = X  W^T   A=X  (K-major), B=W  (K-major)
//   dgrad    dX = dY W     A=dY (K-major), B=W  (MN-major)
//   wgrad    dW = dY^T X   A=dY (MN-major), B=X (MN-major)
//
// Replaces the reference's cublasSgemm call in CudaTensorF32::matmul
// (cuda/kernels.cu:488-493) and its Python matmul (tensor.py:609-675).
//
// CTA layout (352 threads, one CTA per SM, persistent over tiles):
//   warp 0      TMA producer (one elected lane), 128B-swizzled tiles, no
//               multicast (this kernel also runs inside multi-GPU jobs)
//   warp 1      TMEM allocator + MMA issuer (one elected lane)
//   warps 2..9  epilogue: tcgen05.ld 32 lanes each (warp % 4 selects the
//               lane quarter, (warp - 2) / 4 the half of the BN columns),
//               fused bias / GELU / residual / dGELU / fp32-accumulate,
//               TMA-store epilogue
//   warp 10     pusher of the fused all-gather (ZeRO-3 weights): copies this
//               rank's rows to every peer over NVLink (peer stores) while
//               the other warps compute; idle without a gather
// The TMEM accumulator is double-buffered (2 x BN columns) so the epilogue of
// tile i overlaps the main loop of tile i+1.  Every wait is bounded.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>

#include "common.cuh"
#include "gemm.h"

namespace uhfs {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;           // 64 bf16 = 128 bytes = one swizzle row
constexpr int kThreads = 352;   // producer, MMA, 8 epilogue warps, pusher (fused all-gather)
constexpr int kSmemBudget = 200 * 1024;
constexpr int kDefaultStreamKChunk = 0;  // stream-K order: tile-major unless UHFS_STREAMK_CHUNK is set

template <int BN>
struct GemmCfg {
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (kSmemBudget - 2048) / kStageBytes;
  static constexpr int kTmemCols = 2 * BN;  // double-buffered accumulator
  static constexpr int kSmemBytes = 1024 /*align slack*/ + kStages * kStageBytes + 256 /*barriers*/;
};

// bf16 epilogues stage each warp's 32 x 32 output box in shared memory (64-byte
// rows, 64-byte swizzle) and write it with one TMA store; fp32 epilogues
// store directly.
constexpr int kEpiWarps = 8;
constexpr int kEpiBox = 32 * 32 * 2;
__host__ __device__ constexpr int epi_boxes(int epi) {
  return epi == GEMM_EPI_BIAS_GELU ? 2 : ((epi == GEMM_EPI_F32_ACCUM || epi == GEMM_EPI_F32_STORE) ? 0 : 1);
}

struct GemmArgs {
  int M, N, K;
  int tiles_m, tiles_n, splits, kb_per_split, kb_total;
  int stream_k;  // fp32-accumulate only: CTAs take equal contiguous (tile, k-block) ranges
  int sk_chunk;  // stream-K order: 0 = tile-major; C > 0 = chunks of C k-blocks outermost
  int group;     // grouped raster: M-tiles walked down a column of N before moving right
  int k_chunk;   // > 0: each tile as consecutive units of k_chunk k-blocks on one CTA (pair)
  void* C;
  long long ldc;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* aux;
  long long ld_aux;
  __nv_bfloat16* aux_out;
  long long ld_aux_out;
  DeviceStatus* status;
  GemmGather ag;
  unsigned long long* trace;  // UHFS_GEMM_TRACE builds: clock stamps of CTA 0 (set_gemm_trace)
};

// Per-unit clock64 stamps of CTA 0 of the single-CTA kernel, compiled in only
// with -DUHFS_GEMM_TRACE (UNDERHFS_GEMM_TRACE=1 at build time):
// trace[event * kGemmTraceUnits + unit].
constexpr int kGemmTraceUnits = 16;
enum GemmTraceEvent {
  kGtProdStart = 0, kGtProdLast, kGtMmaAccFree, kGtMmaFirstFull, kGtMmaCommit, kGtEpiFull, kGtEpiRelease, kGtEpiDone,
  kGtChunkLd,                        // + j: chunk j's accumulator columns in registers
  kGtChunkMath = kGtChunkLd + 4,     // + j: chunk j's values final (bias, operand, activation)
  kGtChunkStore = kGtChunkMath + 4,  // + j: chunk j's TMA store issued
  kGtEvents = kGtChunkStore + 4
};
unsigned long long* g_gemm_trace = nullptr;
#ifdef UHFS_GEMM_TRACE
#define GEMM_TRACE(ev, u)                                                                                 \
  do {                                                                                                    \
    if (args.trace != nullptr && blockIdx.x == 0 && (u) < kGemmTraceUnits)                                \
      args.trace[(ev) * kGemmTraceUnits + (u)] = (unsigned long long)clock64();                           \
  } while (0)
#else
#define GEMM_TRACE(ev, u) \
  do {                    \
  } while (0)
#endif

__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until a flag reaches `epoch` (wrap-safe comparison).
__device__ __forceinline__ bool wait_epoch(const uint32_t* f, uint32_t epoch, DeviceStatus* st, int where) {
  if ((int32_t)(ld_acquire_sys_u32(f) - epoch) >= 0) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if ((int32_t)(ld_acquire_sys_u32(f) - epoch) >= 0) return true;
    if (((++spins) & 63u) == 0u && globaltimer_ns() - t0 > kWaitBoundNs) {
      report_error(st, kErrPeerTimeout, where);
      return false;
    }
  }
}

// Wait for the gathered B rows [r0, r1) (32-row flags of this rank), then
// order the remote generic-proxy stores before this thread's TMA loads.
__device__ __forceinline__ bool wait_gathered_rows(const GemmGather& g, int r0, int r1, DeviceStatus* st) {
  const uint32_t* flags = g.peer_flags[g.rank] + g.b_flag_base;
  for (int c = r0 / 32; c < (r1 + 31) / 32; ++c)
    if (!wait_epoch(flags + c, g.epoch, st, 40)) return false;
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

__device__ __forceinline__ void tile_coords(const GemmArgs& a, int t, int& tm, int& tn, int& split);

// Work units of one CTA (or CTA pair), identical in the producer, MMA and
// epilogue roles; `idx` / `cnt` are the CTA's (pair's) index and count.
//   tiled:    units idx, idx + cnt, ... of tiles_m * tiles_n * splits
//   stream-K: the k-block range [idx*W/cnt, (idx+1)*W/cnt) of the
//             W = tiles * kb_total linearised (tile, k-block) space, cut at
//             tile boundaries; each piece is accumulated into C by the fp32
//             epilogue.  With sk_chunk = C the space is ordered (k-chunk of
//             C k-blocks, tile, k-block): the CTAs running at the same time
//             then cover the same k-range of many tiles, so the A rows and
//             B columns of that range are shared in L2 instead of each CTA
//             streaming a different k-range of one tile.
struct UnitIter {
  long long pos, end;
  int stride;
  int chunk = 0;  // k_chunk mode: next chunk of tile `pos`
};

__device__ __forceinline__ UnitIter unit_begin(const GemmArgs& a, int idx, int cnt) {
  if (a.stream_k) {
    const long long total = (long long)a.tiles_m * a.tiles_n * a.kb_total;
    return {(long long)idx * total / cnt, (long long)(idx + 1) * total / cnt, cnt};
  }
  return {(long long)idx, (long long)a.tiles_m * a.tiles_n * a.splits, cnt};
}

__device__ __forceinline__ bool unit_next(const GemmArgs& a, UnitIter& it, int& tm, int& tn, int& kb0, int& kb1) {
  if (it.pos >= it.end) return false;
  int split;
  if (a.stream_k) {
    int tile;
    if (a.sk_chunk > 0) {
      const long long tiles = (long long)a.tiles_m * a.tiles_n;
      const long long per_chunk = tiles * a.sk_chunk;
      const long long c = it.pos / per_chunk;
      const int chunk_lo = (int)(c * a.sk_chunk);
      const int chunk_len = min(a.sk_chunk, a.kb_total - chunk_lo);
      const long long rem = it.pos - c * per_chunk;
      tile = (int)(rem / chunk_len);
      kb0 = chunk_lo + (int)(rem - (long long)tile * chunk_len);
      kb1 = (int)min((long long)(chunk_lo + chunk_len), kb0 + (it.end - it.pos));
    } else {
      tile = (int)(it.pos / a.kb_total);
      kb0 = (int)(it.pos - (long long)tile * a.kb_total);
      kb1 = (int)min((long long)a.kb_total, kb0 + (it.end - it.pos));
    }
    it.pos += kb1 - kb0;
    tile_coords(a, tile, tm, tn, split);
    return true;
  }
  if (a.k_chunk > 0) {
    // tiles idx, idx + cnt, ..., each as its k-chunks in order on this CTA
    tile_coords(a, (int)it.pos, tm, tn, split);
    kb0 = it.chunk * a.k_chunk;
    kb1 = min(kb0 + a.k_chunk, a.kb_total);
    if (kb1 >= a.kb_total) {
      it.chunk = 0;
      it.pos += it.stride;
    } else {
      ++it.chunk;
    }
    return true;
  }
  tile_coords(a, (int)it.pos, tm, tn, split);
  kb0 = split * a.kb_per_split;
  kb1 = min(kb0 + a.kb_per_split, a.kb_total);
  it.pos += it.stride;
  return true;
}

__device__ __forceinline__ void tile_coords(const GemmArgs& a, int t, int& tm, int& tn, int& split) {
  const int mn_tiles = a.tiles_m * a.tiles_n;
  split = t / mn_tiles;
  int mn = t - split * mn_tiles;
  // Grouped raster: walk `group` M-tiles down a column of N before moving
  // right, so concurrently running CTAs share B tiles in L2.
  const int G = a.group;
  const int group_span = G * a.tiles_n;
  const int g = mn / group_span;
  const int first_m = g * G;
  const int gm = min(a.tiles_m - first_m, G);
  const int r = mn - g * group_span;
  tm = first_m + r % gm;
  tn = r / gm;
}

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float* v, int valid_cols) {
  if (valid_cols >= 32) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      __align__(16) __nv_bfloat162 h[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(v[q * 8 + 2 * j], v[q * 8 + 2 * j + 1]);
      *reinterpret_cast<uint4*>(dst + q * 8) = *reinterpret_cast<uint4*>(h);
    }
  } else {
    for (int q = 0; q < 4; ++q) {
      if (q * 8 >= valid_cols) break;
      __align__(16) __nv_bfloat162 h[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(v[q * 8 + 2 * j], v[q * 8 + 2 * j + 1]);
      *reinterpret_cast<uint4*>(dst + q * 8) = *reinterpret_cast<uint4*>(h);
    }
  }
}

__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* src, float* v, int valid_cols) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (q * 8 < valid_cols) {
      uint4 raw = *reinterpret_cast<const uint4*>(src + q * 8);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __bfloat1622float2(h[j]);
        v[q * 8 + 2 * j] = f.x;
        v[q * 8 + 2 * j + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[q * 8 + j] = 0.f;
    }
  }
}

// Epilogue operands read per output element (the residual of GEMM_EPI_RESID,
// the GELU input of GEMM_EPI_DGELU): each lane needs 64 bytes of its row per
// 32-column chunk.  They are loaded coalesced (eight rows per instruction;
// one row per lane cost 32 L1 wavefronts per instruction and made these
// epilogues longer than their tiles' main loops, per the per-unit clock
// trace) and regrouped by row through the warp's store box.  Chunk 0 is
// loaded before the warp waits for the accumulator and chunk j + 1 while
// chunk j is processed.
template <int BN>
struct AuxRegs {
  uint4 r[BN / 64][4];
};

template <int EPI>
constexpr bool epi_reads_aux() {
  return EPI == GEMM_EPI_RESID || EPI == GEMM_EPI_DGELU;
}

__device__ __forceinline__ int epi_c_end(const GemmArgs& args, int BN, int n0, int ehalf) {
  return min((ehalf + 1) * (BN / 64), (args.N - n0 + 31) / 32);
}

// Load chunk j of this warp's columns (zeros outside the matrix), coalesced:
// piece q of lane l is row 8q + l/4 of the warp's 32 rows, 16-byte column
// group l % 4, so one load instruction covers eight whole 64-byte row
// segments.  epi_aux_to_rows() regroups the pieces by row through the
// warp's store box.
template <int BN, int EPI>
__device__ __forceinline__ void epi_load_aux(const GemmArgs& args, int m0, int n0, int quarter, int ehalf, int lane,
                                             int j, uint4* r) {
  if constexpr (epi_reads_aux<EPI>()) {
    const int c = ehalf * (BN / 64) + j;
    const int col = n0 + c * 32 + (lane & 3) * 8;
    const bool ok = c < epi_c_end(args, BN, n0, ehalf) && col < args.N;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int row = m0 + quarter * 32 + q * 8 + (lane >> 2);
      r[q] = (ok && row < args.M) ? *reinterpret_cast<const uint4*>(args.aux + (long long)row * args.ld_aux + col)
                                  : make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

// The coalesced pieces of epi_load_aux -> this lane's own row (64 bytes as
// four 16-byte groups), through the warp's 32 x 64-byte box in the layout
// of the output rows (16-byte group g of row r at (g ^ ((r >> 1) & 3)) << 4).
// The box must be free (its last TMA store has read it).
__device__ __forceinline__ void epi_aux_to_rows(uint8_t* box, int lane, uint4* r) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int rr = q * 8 + (lane >> 2), g = lane & 3;
    *reinterpret_cast<uint4*>(box + rr * 64 + ((g ^ ((rr >> 1) & 3)) << 4)) = r[q];
  }
  __syncwarp();
#pragma unroll
  for (int q = 0; q < 4; ++q) r[q] = *reinterpret_cast<const uint4*>(box + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4));
  __syncwarp();
}

__device__ __forceinline__ void unpack_bf16x32(const uint4* raw, float* v) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[q]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      v[q * 8 + 2 * j] = f.x;
      v[q * 8 + 2 * j + 1] = f.y;
    }
  }
}

// One accumulator tile, one epilogue warp: TMEM lanes quarter*32.. are rows
// m0 + quarter*32 + lane of C (m0: first row held in this CTA's TMEM), the
// warp takes columns [n0 + 32*c_begin, n0 + 32*c_end) of the BN-wide tile.
// `release` runs once the warp holds its last TMEM chunk in registers (the
// accumulator may then be reused).  With kBufs == 2 consecutive chunks
// alternate between two sets of store boxes (`seq` counts the warp's chunks),
// so a chunk waits only for the stores issued two chunks earlier.
template <int BN, int EPI, int kBufs, class Release>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& args, const CUtensorMap* tmC, const CUtensorMap* tmAuxOut,
                                              uint32_t tmem_acc, int m0, int n0, int quarter, int ehalf, int lane,
                                              uint8_t* box_base, uint32_t& seq, AuxRegs<BN>& aux,
                                              Release release, [[maybe_unused]] bool tracer = false,
                                              [[maybe_unused]] int unit = 0) {
  constexpr int kBoxes = epi_boxes(EPI);
  const int row = m0 + quarter * 32 + lane;
  const bool row_ok = row < args.M;
  const int c_begin = ehalf * (BN / 64), c_end = epi_c_end(args, BN, n0, ehalf);
#pragma unroll
  for (int j = 0; j < BN / 64; ++j) {
    const int c = c_begin + j;
    if (c >= c_end) break;
    const int col0 = n0 + c * 32;
    if (j + 1 < BN / 64) epi_load_aux<BN, EPI>(args, m0, n0, quarter, ehalf, lane, j + 1, aux.r[j + 1 < BN / 64 ? j + 1 : j]);
    float v[32];
    const uint32_t taddr = tmem_acc + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(c * 32);
    tmem_ld_32x32b_x32(taddr, v);
    tc_wait_ld();
    if (tracer && j < 4) GEMM_TRACE(kGtChunkLd + j, unit);
    if (c == c_end - 1) {
      release();  // the whole accumulator of this warp is in registers
    }
    const int valid = min(32, args.N - col0);
    if constexpr (EPI == GEMM_EPI_BF16 || EPI == GEMM_EPI_BIAS_GELU || EPI == GEMM_EPI_RESID) {
      if (args.bias != nullptr) {
        float b[32];
        load_bf16x32(args.bias + col0, b, valid);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += b[i];
      }
    }
    if constexpr (epi_reads_aux<EPI>()) {
      // the box this chunk will store from must be free before it regroups
      // the operand rows (the store wait below then returns at once)
      uint8_t* tb = box_base + (kBufs == 2 ? (int)(seq & 1u) * kBoxes * kEpiBox : 0);
      if (lane == 0) {
        if constexpr (kBufs == 2)
          bulk_wait_group_read1();
        else
          bulk_wait_group_read0();
      }
      __syncwarp();
      epi_aux_to_rows(tb, lane, aux.r[j]);
    }
    if constexpr (EPI == GEMM_EPI_RESID) {
      float r[32];
      unpack_bf16x32(aux.r[j], r);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += r[i];
    } else if constexpr (EPI == GEMM_EPI_DGELU) {
      float u[32];
      unpack_bf16x32(aux.r[j], u);
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const float2 g = f2_mul(make_float2(v[i], v[i + 1]), gelu_tanh_grad_fast_x2(make_float2(u[i], u[i + 1])));
        v[i] = g.x;
        v[i + 1] = g.y;
      }
    }
    if (tracer && j < 4) GEMM_TRACE(kGtChunkMath + j, unit);
    if constexpr (kBoxes > 0) {
      uint8_t* box = box_base + (kBufs == 2 ? (int)(seq & 1u) * kBoxes * kEpiBox : 0);
      ++seq;
      // row `lane` of the warp's box: 4 chunks of 16 B at chunk ^ ((lane >> 1) & 3)
      if (lane == 0) {
        if constexpr (kBufs == 2)
          bulk_wait_group_read1();  // the stores that last used this box set have read it
        else
          bulk_wait_group_read0();
      }
      __syncwarp();
      uint8_t* brow = box + lane * 64;
      const int sw = (lane >> 1) & 3;
      if constexpr (EPI == GEMM_EPI_BIAS_GELU) {
        uint8_t* arow = brow + kEpiBox;  // pre-activation box (kept for the backward pass)
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(arow + ((q ^ sw) << 4)) =
              make_uint4(pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]), pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]),
                         pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]), pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]));
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float2 g = gelu_tanh_fast_x2(make_float2(v[i], v[i + 1]));
          v[i] = g.x;
          v[i + 1] = g.y;
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint4*>(brow + ((q ^ sw) << 4)) =
            make_uint4(pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]), pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]),
                       pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]), pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]));
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        // rows >= M and columns >= N fall outside the tensor map and are not written
        tma_store_2d(tmC, box, col0, m0 + quarter * 32);
        if constexpr (EPI == GEMM_EPI_BIAS_GELU) tma_store_2d(tmAuxOut, box + kEpiBox, col0, m0 + quarter * 32);
        bulk_commit_group();
      }
      if (tracer && j < 4) GEMM_TRACE(kGtChunkStore + j, unit);
    } else if constexpr (EPI == GEMM_EPI_F32_ACCUM) {
      if (row_ok) {
        float* dst = reinterpret_cast<float*>(args.C) + (long long)row * args.ldc + col0;
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (q * 4 < valid) red_add_f32x4(dst + q * 4, v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      }
    } else {  // GEMM_EPI_F32_STORE
      if (row_ok) {
        float* dst = reinterpret_cast<float*>(args.C) + (long long)row * args.ldc + col0;
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (q * 4 < valid)
            *reinterpret_cast<float4*>(dst + q * 4) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      }
    }
  }
  if (c_begin >= c_end) release();  // this warp has no columns in a narrow last tile
}

template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmAuxOut,
                        const GemmArgs args) {
  using Cfg = GemmCfg<BN>;
  constexpr int S = Cfg::kStages;
  constexpr uint32_t kIdesc = make_idesc(1 /*bf16*/, A_MN ? 1 : 0, B_MN ? 1 : 0, BM, BN);

  constexpr int kBoxes = epi_boxes(EPI);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align1024(smem_raw);
  uint8_t* tiles = smem;
  uint8_t* epi_stage = smem + S * Cfg::kStageBytes;  // [kEpiWarps][kBoxes] boxes
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi_stage + kEpiWarps * kBoxes * kEpiBox);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* tfull = bars + 2 * S;
  uint64_t* tempty = bars + 2 * S + 2;
  uint64_t* done = bars + 2 * S + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if constexpr (kBoxes > 0) tma_prefetch_desc(&tmC);
    if constexpr (kBoxes > 1) tma_prefetch_desc(&tmAuxOut);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 256);
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
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one_sync()) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      UnitIter it = unit_begin(args, (int)blockIdx.x, (int)gridDim.x);
      int tm, tn, kb0, kb1;
      int pu = 0;  // units started (trace index)
      while (ok && unit_next(args, it, tm, tn, kb0, kb1)) {
        const int m0 = tm * BM, n0 = tn * BN;
        GEMM_TRACE(kGtProdStart, pu);
        if (!UHFS_CHECK(m0 < args.M && n0 < args.N && kb0 < kb1 && kb1 <= args.kb_total, args.status, 12)) {
          ok = false;
          break;
        }
        const bool gathered_b = args.ag.world > 0 && args.ag.b_flag_base >= 0;
        if (gathered_b && !B_MN && !wait_gathered_rows(args.ag, n0, min(args.N, n0 + BN), args.status)) {
          ok = false;
          break;
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (gathered_b && B_MN && !wait_gathered_rows(args.ag, kb * BK, min(args.K, kb * BK + BK), args.status)) {
            ok = false;
            break;
          }
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, args.status, kErrWaitTimeoutEmpty, 10)) {
            ok = false;
            break;
          }
          uint8_t* sA = tiles + stage * Cfg::kStageBytes;
          uint8_t* sB = sA + Cfg::kABytes;
          mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
          const int k0 = kb * BK;
          if constexpr (!A_MN) {
            tma_load_2d(sA, &tmA, &full[stage], k0, m0);
          } else {
#pragma unroll
            for (int c = 0; c < BM / 64; ++c) tma_load_2d(sA + c * (64 * BK * 2), &tmA, &full[stage], m0 + 64 * c, k0);
          }
          if constexpr (!B_MN) {
            tma_load_2d(sB, &tmB, &full[stage], k0, n0);
          } else {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c) tma_load_2d(sB + c * (64 * BK * 2), &tmB, &full[stage], n0 + 64 * c, k0);
          }
          issued_mask |= (1u << stage);
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        GEMM_TRACE(kGtProdLast, pu);
        ++pu;
      }
      // Never leave the CTA with bulk copies still landing in shared memory.
      for (int s = 0; s < S; ++s)
        if (issued_mask & (1u << s)) mbar_wait_bounded(&full[s], (issued_parity >> s) & 1u, args.status, kErrWaitTimeoutFull, 11);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one_sync()) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      UnitIter it = unit_begin(args, (int)blockIdx.x, (int)gridDim.x);
      int tm, tn, kb0, kb1;
      [[maybe_unused]] int mu = 0;  // units issued (trace index)
      while (ok && unit_next(args, it, tm, tn, kb0, kb1)) {
        if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1u, args.status, kErrWaitTimeoutAccum, 20)) break;
        GEMM_TRACE(kGtMmaAccFree, mu);
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, args.status, kErrWaitTimeoutFull, 21)) {
            ok = false;
            break;
          }
          if (kb == kb0) GEMM_TRACE(kGtMmaFirstFull, mu);
          tc_fence_after();
          const uint32_t a_base = smem_u32(tiles + stage * Cfg::kStageBytes);
          const uint32_t b_base = a_base + Cfg::kABytes;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            uint64_t adesc, bdesc;
            if constexpr (!A_MN)
              adesc = make_smem_desc(a_base + kk * 32, 16, 1024, kSwizzle128B);
            else
              adesc = make_smem_desc(a_base + kk * 16 * 128, 64 * BK * 2, 1024, kSwizzle128B);
            if constexpr (!B_MN)
              bdesc = make_smem_desc(b_base + kk * 32, 16, 1024, kSwizzle128B);
            else
              bdesc = make_smem_desc(b_base + kk * 16 * 128, 64 * BK * 2, 1024, kSwizzle128B);
            tc_mma_f16(d_tmem, adesc, bdesc, kIdesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&empty[stage]);  // frees this smem stage once the MMAs retire
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&tfull[acc]);  // accumulator ready for the epilogue
        GEMM_TRACE(kGtMmaCommit, mu);
        ++mu;
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // All MMAs issued by this thread retire before TMEM is released.
      tc_commit(done);
      mbar_wait_bounded(done, 0, args.status, kErrWaitTimeoutAccum, 22);
    }
  } else if (warp == kThreads / 32 - 1) {
    // ------------------------------------------------------------ pusher
    const GemmGather& g = args.ag;
    if (g.world > 0) {
      // this rank is ready to receive this gather (every earlier kernel that
      // read the slot has finished here): tell every peer
      if (blockIdx.x == 0 && lane < g.world)
        st_release_sys_u32(g.peer_flags[lane] + g.ready_base + g.rank, g.epoch);
      long long total = 0;
      for (int s2 = 0; s2 < g.nseg; ++s2) total += (g.seg[s2].rows + 31) / 32;
      uint32_t ready_mask = 0;
      bool ok = true;
      for (long long item = blockIdx.x; item < total && ok; item += gridDim.x) {
        int s2 = 0;
        long long c = item;
        while (c >= (g.seg[s2].rows + 31) / 32) {
          c -= (g.seg[s2].rows + 31) / 32;
          ++s2;
        }
        const GemmGatherSeg& sg = g.seg[s2];
        const long long r0 = c * 32, nrows = min(32ll, sg.rows - r0);
        const long long n16 = nrows * sg.row_bytes / 16;
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const char*>(sg.src) + r0 * sg.row_bytes);
        for (int k = 0; k < g.world && ok; ++k) {
          const int p = (g.rank + 1 + k) % g.world;  // spread the first pushes over the peers
          if (!(ready_mask & (1u << p))) {
            int good = 1;
            if (lane == 0) good = wait_epoch(g.peer_flags[g.rank] + g.ready_base + p, g.epoch, args.status, 41);
            good = __shfl_sync(0xffffffffu, good, 0);
            if (!good) {
              ok = false;
              break;
            }
            ready_mask |= 1u << p;
          }
          uint4* dst = reinterpret_cast<uint4*>(g.peer_data[p] + sg.dst_off_bytes + r0 * sg.row_bytes);
          for (long long i = lane; i < n16; i += 128) {
            uint4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
              if (i + u * 32 < n16) v[u] = __ldg(src + i + u * 32);
#pragma unroll
            for (int u = 0; u < 4; ++u)
              if (i + u * 32 < n16) __stcg(dst + i + u * 32, v[u]);
          }
        }
        __syncwarp();
        if (ok && lane < g.world) {
          __threadfence_system();
          st_release_sys_u32(g.peer_flags[lane] + sg.flag_base + c, g.epoch);
        }
        __syncwarp();
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;        // TMEM lane quarter this warp may access
    const int ehalf = (warp - 2) >> 2;   // which half of the BN columns
    uint8_t* box = epi_stage + (warp - 2) * kBoxes * kEpiBox;
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t seq = 0;
    UnitIter it = unit_begin(args, (int)blockIdx.x, (int)gridDim.x);
    int tm, tn, kb0, kb1;
    [[maybe_unused]] const bool tracer = warp == 2 && lane == 0;
    [[maybe_unused]] int eu = 0;  // units finished (trace index)
    while (unit_next(args, it, tm, tn, kb0, kb1)) {
      const int m0 = tm * BM, n0 = tn * BN;
      AuxRegs<BN> aux;
      epi_load_aux<BN, EPI>(args, m0, n0, quarter, ehalf, lane, 0, aux.r[0]);
      if (!mbar_wait_warp(&tfull[acc], acc_phase, args.status, kErrWaitTimeoutAccum, 30)) break;
      if (tracer) GEMM_TRACE(kGtEpiFull, eu);
      tc_fence_after();
      epilogue_tile<BN, EPI, 1>(args, &tmC, &tmAuxOut, tmem_base + (uint32_t)(acc * BN), m0, n0, quarter, ehalf,
                                lane, box, seq, aux, [&] {
                                  tc_fence_before();
                                  mbar_arrive(&tempty[acc]);
                                  if (tracer) GEMM_TRACE(kGtEpiRelease, eu);
                                }, tracer, eu);
      if (tracer) GEMM_TRACE(kGtEpiDone, eu);
      ++eu;
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if constexpr (kBoxes > 0) {
      if (lane == 0) bulk_wait_group0();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// ------------------------------------------------------------ CTA-pair GEMM
// 256 x 256 output tiles on a cluster of two CTAs (one TPC) with
// tcgen05 .cta_group::2: the leader (rank 0) issues M = 256, N = 256 MMAs
// whose A rows [0,128) and B rows [0,128) come from its own shared memory
// and A rows [128,256), B rows [128,256) from its peer's.  Per SM that is
// half the B bytes of the single-CTA 128 x 256 tile for the same MMA work,
// so shared-memory bandwidth and L2 reads per FLOP drop by a third and six
// 32 KB stages fit.  Each CTA's TMEM holds the 128 accumulator rows of its
// own A half; both CTAs run the same epilogue on their rows.
//   full[s]   leader only: both CTAs' TMA bytes (expect_tx by the leader)
//   empty[s]  per CTA: the leader's MMA commit, sent to both CTAs
//   tfull[a]  per CTA: the leader's commit after the last k-block
//   tempty[a] leader only: 16 epilogue warps (8 per CTA) arrive
// Used for every epilogue of problems with M > 128 and N > 128, one pass
// per tile or stream-K (fp32 accumulate); classic split-K and the fused
// all-gather stay on the single-CTA kernel.
constexpr int kPairThreads = 320;  // producer, MMA, 8 epilogue warps
constexpr int kPairHalf = 128;     // rows of A and of B staged by each CTA
constexpr int kPairStageBytes = 2 * kPairHalf * BK * 2;
constexpr int kPairTmemCols = 512;  // 2 accumulators x 256 columns
constexpr int kPairBoxBufs = 2;     // epilogue store boxes double-buffered

__host__ __device__ constexpr int pair_box_bytes(int epi) { return kPairBoxBufs * kEpiWarps * epi_boxes(epi) * kEpiBox; }

__host__ __device__ constexpr int pair_stages(int epi) {
  return (227 * 1024 - 1280 - pair_box_bytes(epi)) / kPairStageBytes < 6
             ? (227 * 1024 - 1280 - pair_box_bytes(epi)) / kPairStageBytes
             : 6;
}

__host__ __device__ constexpr int pair_smem_bytes(int epi) {
  return 1024 + pair_stages(epi) * kPairStageBytes + pair_box_bytes(epi) + 256;
}

// TF32: operands are fp32 (tf32 math, kind::tf32), K-major both, fp32 store
// epilogue; a k-block is then 32 elements (the same 128-byte rows), and an
// MMA of K = 8 covers the 32 bytes a bf16 MMA of K = 16 does.
template <bool A_MN, bool B_MN, int EPI, bool TF32 = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmAuxOut,
                     const GemmArgs args) {
  static_assert(!TF32 || (!A_MN && !B_MN && EPI == GEMM_EPI_F32_STORE), "tf32: K-major operands, fp32 store");
  constexpr int S = pair_stages(EPI);
  constexpr int kABytes = kPairHalf * BK * 2;
  constexpr int kKElems = TF32 ? BK / 2 : BK;  // elements of K per k-block (128 bytes)
  constexpr uint32_t kIdesc = make_idesc(TF32 ? 2 : 1, A_MN ? 1 : 0, B_MN ? 1 : 0, 2 * kPairHalf, 2 * kPairHalf);
  constexpr int kBoxes = epi_boxes(EPI);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align1024(smem_raw);  // same offsets in both CTAs
  uint8_t* tiles = smem;
  uint8_t* epi_stage = smem + S * kPairStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi_stage + pair_box_bytes(EPI));
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* tfull = bars + 2 * S;
  uint64_t* tempty = bars + 2 * S + 2;
  uint64_t* done = bars + 2 * S + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if constexpr (kBoxes > 0) tma_prefetch_desc(&tmC);
    if constexpr (kBoxes > 1) tma_prefetch_desc(&tmAuxOut);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 2 * kEpiWarps);
    }
    mbar_init(done, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  __syncwarp();
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kPairTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers exist before either signals the other
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (elect_one_sync()) {
      const uint32_t full_leader = smem_cluster_addr(full, 0);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      UnitIter it = unit_begin(args, (int)cluster_id_x(), (int)cluster_count_x());
      int tm, tn, kb0, kb1;
      while (ok && unit_next(args, it, tm, tn, kb0, kb1)) {
        const int m0 = tm * 2 * kPairHalf + (int)rank * kPairHalf;
        const int nb0 = tn * 2 * kPairHalf + (int)rank * kPairHalf;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded_cluster(&empty[stage], phase ^ 1u, args.status, kErrWaitTimeoutEmpty, 13)) {
            ok = false;
            break;
          }
          uint8_t* sA = tiles + stage * kPairStageBytes;
          uint8_t* sB = sA + kABytes;
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * kPairStageBytes);
          const uint32_t bar = full_leader + stage * 8;
          const int k0 = kb * kKElems;
          if constexpr (!A_MN) {
            tma_load_2d_pair(sA, &tmA, bar, k0, m0);
          } else {
#pragma unroll
            for (int c = 0; c < kPairHalf / 64; ++c) tma_load_2d_pair(sA + c * (64 * BK * 2), &tmA, bar, m0 + 64 * c, k0);
          }
          if constexpr (!B_MN) {
            tma_load_2d_pair(sB, &tmB, bar, k0, nb0);
          } else {
#pragma unroll
            for (int c = 0; c < kPairHalf / 64; ++c) tma_load_2d_pair(sB + c * (64 * BK * 2), &tmB, bar, nb0 + 64 * c, k0);
          }
          issued_mask |= (1u << stage);
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // The leader's full barriers count both CTAs' bytes: once they have
      // all flipped no copy of either CTA is still landing.
      if (leader)
        for (int s = 0; s < S; ++s)
          if (issued_mask & (1u << s))
            mbar_wait_bounded_cluster(&full[s], (issued_parity >> s) & 1u, args.status, kErrWaitTimeoutFull, 14);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (leader) {
      if (elect_one_sync()) {
        const uint32_t empty_l = smem_cluster_addr(empty, 0), empty_p = smem_cluster_addr(empty, 1);
        const uint32_t tfull_l = smem_cluster_addr(tfull, 0), tfull_p = smem_cluster_addr(tfull, 1);
        int stage = 0;
        uint32_t phase = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        UnitIter it = unit_begin(args, (int)cluster_id_x(), (int)cluster_count_x());
        int tm, tn, kb0, kb1;
        while (ok && unit_next(args, it, tm, tn, kb0, kb1)) {
          if (!mbar_wait_bounded_cluster(&tempty[acc], acc_phase ^ 1u, args.status, kErrWaitTimeoutAccum, 23)) break;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + acc * 2 * kPairHalf;
          for (int kb = kb0; kb < kb1; ++kb) {
            if (!mbar_wait_bounded_cluster(&full[stage], phase, args.status, kErrWaitTimeoutFull, 24)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = smem_u32(tiles + stage * kPairStageBytes);
            const uint32_t b_base = a_base + kABytes;
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              uint64_t adesc, bdesc;
              if constexpr (!A_MN)
                adesc = make_smem_desc(a_base + kk * 32, 16, 1024, kSwizzle128B);
              else
                adesc = make_smem_desc(a_base + kk * 16 * 128, 64 * BK * 2, 1024, kSwizzle128B);
              if constexpr (!B_MN)
                bdesc = make_smem_desc(b_base + kk * 32, 16, 1024, kSwizzle128B);
              else
                bdesc = make_smem_desc(b_base + kk * 16 * 128, 64 * BK * 2, 1024, kSwizzle128B);
              if constexpr (TF32)
                tc_mma_tf32_pair(d_tmem, adesc, bdesc, kIdesc, (kb > kb0 || kk > 0) ? 1u : 0u);
              else
                tc_mma_f16_pair(d_tmem, adesc, bdesc, kIdesc, (kb > kb0 || kk > 0) ? 1u : 0u);
            }
            // frees this stage in both CTAs once the MMAs retire
            tc_commit_pair(empty_l + stage * 8);
            tc_commit_pair(empty_p + stage * 8);
            if (++stage == S) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          tc_commit_pair(tfull_l + acc * 8);
          tc_commit_pair(tfull_p + acc * 8);
          if (TF32) {
            acc_phase ^= 1u;  // one partial accumulator; the other holds the running sum
          } else if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1u;
          }
        }
        tc_commit_pair(smem_cluster_addr(done, 0));
        tc_commit_pair(smem_cluster_addr(done, 1));
        mbar_wait_bounded_cluster(done, 0, args.status, kErrWaitTimeoutAccum, 25);
      }
    } else if (lane == 0) {
      // the peer's TMEM is written by the leader's MMAs: wait until they retired
      mbar_wait_bounded_cluster(done, 0, args.status, kErrWaitTimeoutAccum, 26);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quarter = warp & 3;
    const int ehalf = (warp - 2) >> 2;
    uint8_t* box = epi_stage + (warp - 2) * kPairBoxBufs * kBoxes * kEpiBox;
    const uint32_t tempty_leader = smem_cluster_addr(tempty, 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t seq = 0;
    UnitIter it = unit_begin(args, (int)cluster_id_x(), (int)cluster_count_x());
    int tm, tn, kb0, kb1;
    if constexpr (TF32) {
      // The tensor core's fp32 accumulation is not round-to-nearest, so its
      // error grows with the number of MMA steps summed in TMEM.  A tile is
      // therefore accumulated in chunks of k_chunk k-blocks into TMEM columns
      // [0, 256); the epilogue adds each chunk (round-to-nearest, CUDA cores)
      // into a running sum in columns [256, 512) and writes the tile after
      // its last chunk.
      const uint32_t lane_base = tmem_base + ((uint32_t)(quarter * 32) << 16);
      while (unit_next(args, it, tm, tn, kb0, kb1)) {
        const int m0 = tm * 2 * kPairHalf + (int)rank * kPairHalf, n0 = tn * 2 * kPairHalf;
        if (!mbar_wait_warp_cluster(&tfull[0], acc_phase, args.status, kErrWaitTimeoutAccum, 31)) break;
        tc_fence_after();
        const bool first = kb0 == 0, last = kb1 >= args.kb_total;
        const int r = m0 + quarter * 32 + lane;
        float* dst = reinterpret_cast<float*>(args.C) + (long long)r * args.ldc;
#pragma unroll 1
        for (int j = 0; j < kPairHalf / 32; ++j) {
          const uint32_t col = (uint32_t)((ehalf * (kPairHalf / 32) + j) * 32);
          float v[32];
          tmem_ld_32x32b_x32(lane_base + col, v);
          if (!first) {
            float sum[32];
            tmem_ld_32x32b_x32(lane_base + 2 * kPairHalf + col, sum);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] += sum[i];
          }
          if (!last) {
            uint32_t bits[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) bits[i] = __float_as_uint(v[i]);
            tmem_st_32x32b_x32(lane_base + 2 * kPairHalf + col, bits);
          } else if (r < args.M) {
            const int col0 = n0 + (int)col;
#pragma unroll
            for (int q = 0; q < 8; ++q)
              if (col0 + q * 4 < args.N)
                *reinterpret_cast<float4*>(dst + col0 + q * 4) =
                    make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(tempty_leader);  // the partial accumulator may be overwritten
        acc_phase ^= 1u;
      }
    } else
    while (unit_next(args, it, tm, tn, kb0, kb1)) {
      const int m0 = tm * 2 * kPairHalf + (int)rank * kPairHalf, n0 = tn * 2 * kPairHalf;
      AuxRegs<2 * kPairHalf> aux;
      epi_load_aux<2 * kPairHalf, EPI>(args, m0, n0, quarter, ehalf, lane, 0, aux.r[0]);
      if (!mbar_wait_warp_cluster(&tfull[acc], acc_phase, args.status, kErrWaitTimeoutAccum, 31)) break;
      tc_fence_after();
      const uint32_t tempty_addr = tempty_leader + acc * 8;
      epilogue_tile<2 * kPairHalf, EPI, kPairBoxBufs>(
          args, &tmC, &tmAuxOut, tmem_base + (uint32_t)(acc * 2 * kPairHalf), m0, n0, quarter, ehalf, lane, box, seq,
          aux, [&] {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty_addr);
          });
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if constexpr (kBoxes > 0) {
      if (lane == 0) bulk_wait_group0();
    }
  }

  tc_fence_before();
  __syncwarp();
  cluster_sync_all();  // no CTA leaves while the other may still signal or read it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kPairTmemCols);
  }
}

// --------------------------------------------------------------------- host

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr)
      throw std::runtime_error("cuTensorMapEncodeTiled entry point unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D bf16 tensor map, 128-byte swizzle, box {64, box_outer}.
CUtensorMap make_tmap(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                      uint32_t box_outer) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) throw std::runtime_error("gemm operand must be 16-byte aligned");
  if ((row_stride_elems * 2) % 16 != 0) throw std::runtime_error("gemm leading dimension must be a multiple of 8");
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {64, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return m;
}

// 2-D fp32 tensor map, 128-byte swizzle, box {32, box_outer} (128-byte rows).
CUtensorMap make_tmap_f32(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                          uint32_t box_outer) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) throw std::runtime_error("gemm operand must be 16-byte aligned");
  if ((row_stride_elems * 4) % 16 != 0) throw std::runtime_error("fp32 gemm leading dimension must be a multiple of 4");
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * 4};
  cuuint32_t box[2] = {32, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return m;
}

// UHFS_GEMM_GROUP: M-tiles per raster group.  8 measured best on the 125M
// step (1,059,248 tokens/s against 1,036,639 with 16; 4 and 32 slower at
// 8192^3).
constexpr int kDefaultRasterGroup = 8;
int raster_group() {
  static const int g = [] {
    const char* e = getenv("UHFS_GEMM_GROUP");
    const int v = e != nullptr ? atoi(e) : kDefaultRasterGroup;
    return v > 0 ? v : kDefaultRasterGroup;
  }();
  return g;
}

// UHFS_STREAMK_CHUNK: k-blocks per chunk of the chunk-major stream-K order
// (0 = tile-major).
int stream_k_chunk() {
  static const int c = [] {
    const char* e = getenv("UHFS_STREAMK_CHUNK");
    const int v = e != nullptr ? atoi(e) : kDefaultStreamKChunk;
    return v > 0 ? v : 0;
  }();
  return c;
}

int num_sms() {
  static int by_dev[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  int& n = by_dev[dev & 63];
  if (n == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    n = v > 0 ? v : 148;
  }
  return n;
}

// 2-D bf16 output map for the epilogue: box of 32 columns x 32 rows, 64-byte swizzle.
CUtensorMap make_out_tmap(const void* base, uint64_t cols, uint64_t rows, uint64_t row_stride_elems) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) throw std::runtime_error("gemm output must be 16-byte aligned");
  if ((row_stride_elems * 2) % 16 != 0) throw std::runtime_error("gemm output stride must be a multiple of 8");
  CUtensorMap m;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return m;
}

template <int BN, bool A_MN, bool B_MN, int EPI>
void launch(const GemmProblem& p, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  constexpr int kSmem = Cfg::kSmemBytes + kEpiWarps * epi_boxes(EPI) * kEpiBox;
  static_assert(kSmem <= 227 * 1024, "gemm shared memory");
  auto kern = gemm_tcgen05_kernel<BN, A_MN, B_MN, EPI>;
  static PerDeviceOnce once;
  once([&] { UHFS_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem)); });
  // A: K-major [M][lda] -> dims {K, M}; MN-major [K][lda] -> dims {M, K}
  CUtensorMap ta = A_MN ? make_tmap(p.A, p.M, p.K, p.lda, BK) : make_tmap(p.A, p.K, p.M, p.lda, BM);
  CUtensorMap tb = B_MN ? make_tmap(p.B, p.N, p.K, p.ldb, BK) : make_tmap(p.B, p.K, p.N, p.ldb, BN);
  GemmArgs a = {};
  a.M = p.M;
  a.N = p.N;
  a.K = p.K;
  a.tiles_m = (p.M + BM - 1) / BM;
  a.tiles_n = (p.N + BN - 1) / BN;
  a.kb_total = (p.K + BK - 1) / BK;
  // splits == 0 with the fp32-accumulate epilogue selects stream-K
  a.stream_k = (EPI == GEMM_EPI_F32_ACCUM && p.splits == 0) ? 1 : 0;
  a.sk_chunk = a.stream_k ? stream_k_chunk() : 0;
  a.group = raster_group();
  a.trace = g_gemm_trace;
  int splits = p.splits < 1 ? 1 : p.splits;
  if (splits > a.kb_total) splits = a.kb_total;
  a.kb_per_split = (a.kb_total + splits - 1) / splits;
  a.splits = (a.kb_total + a.kb_per_split - 1) / a.kb_per_split;  // no empty splits
  a.C = p.C;
  a.ldc = p.ldc;
  a.bias = p.bias;
  a.aux = p.aux;
  a.ld_aux = p.ld_aux;
  a.aux_out = p.aux_out;
  a.ld_aux_out = p.ld_aux_out;
  a.status = device_status_ptr();
  a.ag = p.ag;
  if (a.ag.world > 8 || a.ag.nseg > 8) throw std::runtime_error("gemm: fused gather supports 8 ranks / 8 segments");
  const long long units = a.stream_k ? (long long)a.tiles_m * a.tiles_n * a.kb_total
                                     : (long long)a.tiles_m * a.tiles_n * a.splits;
  int grid = units < num_sms() ? (int)units : num_sms();
  if (p.max_ctas > 0 && grid > p.max_ctas) grid = p.max_ctas;
  CUtensorMap tc{}, taux{};
  if constexpr (epi_boxes(EPI) > 0) tc = make_out_tmap(p.C, p.N, p.M, p.ldc);
  if constexpr (epi_boxes(EPI) > 1) taux = make_out_tmap(p.aux_out, p.N, p.M, p.ld_aux_out);
  kern<<<grid, kThreads, kSmem, stream>>>(ta, tb, tc, taux, a);
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

template <int BN>
void dispatch_bn(const GemmProblem& p, cudaStream_t s) {
  const bool am = p.a_mn, bm = p.b_mn;
  switch (p.epi) {
    case GEMM_EPI_BF16:
      if (!am && !bm) return launch<BN, false, false, GEMM_EPI_BF16>(p, s);
      if (!am && bm) return launch<BN, false, true, GEMM_EPI_BF16>(p, s);
      if (am && !bm) return launch<BN, true, false, GEMM_EPI_BF16>(p, s);
      return launch<BN, true, true, GEMM_EPI_BF16>(p, s);
    case GEMM_EPI_BIAS_GELU:
      if (!am && !bm) return launch<BN, false, false, GEMM_EPI_BIAS_GELU>(p, s);
      break;
    case GEMM_EPI_RESID:
      if (!am && !bm) return launch<BN, false, false, GEMM_EPI_RESID>(p, s);
      if (!am && bm) return launch<BN, false, true, GEMM_EPI_RESID>(p, s);
      break;
    case GEMM_EPI_DGELU:
      if (!am && bm) return launch<BN, false, true, GEMM_EPI_DGELU>(p, s);
      break;
    case GEMM_EPI_F32_ACCUM:
      if (am && bm) return launch<BN, true, true, GEMM_EPI_F32_ACCUM>(p, s);
      if (!am && bm) return launch<BN, false, true, GEMM_EPI_F32_ACCUM>(p, s);
      break;
    case GEMM_EPI_F32_STORE:
      if (!am && !bm) return launch<BN, false, false, GEMM_EPI_F32_STORE>(p, s);
      if (!am && bm) return launch<BN, false, true, GEMM_EPI_F32_STORE>(p, s);
      if (am && bm) return launch<BN, true, true, GEMM_EPI_F32_STORE>(p, s);
      break;
    default:
      break;
  }
  throw std::runtime_error("gemm: unsupported (layout, epilogue) combination");
}


// Clusters of two CTAs that fit on the device at once (one CTA per SM).
template <class K>
int max_pair_clusters(K kern, int smem) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * (num_sms() / 2), 1, 1);
  cfg.blockDim = dim3(kPairThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
    (void)cudaGetLastError();
    n = num_sms() / 2;
  }
  return n;
}

template <bool A_MN, bool B_MN, int EPI>
void launch_pair(const GemmProblem& p, cudaStream_t stream) {
  constexpr int kSmem = pair_smem_bytes(EPI);
  static_assert(kSmem <= 227 * 1024, "pair gemm shared memory");
  auto kern = gemm_pair_kernel<A_MN, B_MN, EPI>;
  static int clusters_by_dev[64] = {0};
  static PerDeviceOnce once;
  int dev = 0;
  UHFS_CUDA_CHECK(cudaGetDevice(&dev));
  once([&] {
    UHFS_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    clusters_by_dev[dev & 63] = max_pair_clusters(kern, kSmem);
  });
  const int clusters = clusters_by_dev[dev & 63];
  // Each CTA stages 128 rows of A and 128 rows of B per k-block.
  CUtensorMap ta = A_MN ? make_tmap(p.A, p.M, p.K, p.lda, BK) : make_tmap(p.A, p.K, p.M, p.lda, kPairHalf);
  CUtensorMap tb = B_MN ? make_tmap(p.B, p.N, p.K, p.ldb, BK) : make_tmap(p.B, p.K, p.N, p.ldb, kPairHalf);
  GemmArgs a = {};
  a.M = p.M;
  a.N = p.N;
  a.K = p.K;
  a.tiles_m = (p.M + 2 * kPairHalf - 1) / (2 * kPairHalf);
  a.tiles_n = (p.N + 2 * kPairHalf - 1) / (2 * kPairHalf);
  a.kb_total = (p.K + BK - 1) / BK;
  a.splits = 1;
  a.kb_per_split = a.kb_total;
  // splits == 0 with the fp32-accumulate epilogue selects stream-K over pairs
  a.stream_k = (EPI == GEMM_EPI_F32_ACCUM && p.splits == 0) ? 1 : 0;
  a.sk_chunk = a.stream_k ? stream_k_chunk() : 0;
  a.group = raster_group();
  a.C = p.C;
  a.ldc = p.ldc;
  a.bias = p.bias;
  a.aux = p.aux;
  a.ld_aux = p.ld_aux;
  a.aux_out = p.aux_out;
  a.ld_aux_out = p.ld_aux_out;
  a.status = device_status_ptr();
  const long long units = a.stream_k ? (long long)a.tiles_m * a.tiles_n * a.kb_total : (long long)a.tiles_m * a.tiles_n;
  int ncl = units < clusters ? (int)units : clusters;
  if (p.max_ctas > 0 && 2 * ncl > p.max_ctas) ncl = p.max_ctas / 2 > 0 ? p.max_ctas / 2 : 1;
  CUtensorMap tc{}, taux{};
  if constexpr (epi_boxes(EPI) > 0) tc = make_out_tmap(p.C, p.N, p.M, p.ldc);
  if constexpr (epi_boxes(EPI) > 1) taux = make_out_tmap(p.aux_out, p.N, p.M, p.ld_aux_out);
  kern<<<2 * ncl, kPairThreads, kSmem, stream>>>(ta, tb, tc, taux, a);
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

// k-blocks (32 tf32 elements each, 4 MMAs of K = 8) accumulated in TMEM
// before the epilogue folds them into the round-to-nearest running sum
constexpr int kTf32ChunkKb = 16;

// fp32 C[M, N] = A[M, K] B[N, K]^T on the tensor cores in tf32 (K-major fp32
// operands, CTA pairs, 256 x 256 tiles).  The 3xTF32 fp32 GEMM calls it on
// operands split into tf32 high and low parts.
void gemm_tf32_pair(const float* A, long long lda, const float* B, long long ldb, float* C, long long ldc, int M,
                    int N, int K, cudaStream_t stream) {
  constexpr int EPI = GEMM_EPI_F32_STORE;
  constexpr int kSmem = pair_smem_bytes(EPI);
  auto kern = gemm_pair_kernel<false, false, EPI, true>;
  static int clusters_by_dev[64] = {0};
  static PerDeviceOnce once;
  int dev = 0;
  UHFS_CUDA_CHECK(cudaGetDevice(&dev));
  once([&] {
    UHFS_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    clusters_by_dev[dev & 63] = max_pair_clusters(kern, kSmem);
  });
  if (ldc % 4 != 0) throw std::runtime_error("tf32 gemm: ldc must be a multiple of 4");
  const int clusters = clusters_by_dev[dev & 63];
  CUtensorMap ta = make_tmap_f32(A, K, M, lda, kPairHalf);
  CUtensorMap tb = make_tmap_f32(B, K, N, ldb, kPairHalf);
  GemmArgs a = {};
  a.M = M;
  a.N = N;
  a.K = K;
  a.tiles_m = (M + 2 * kPairHalf - 1) / (2 * kPairHalf);
  a.tiles_n = (N + 2 * kPairHalf - 1) / (2 * kPairHalf);
  a.kb_total = (K + BK / 2 - 1) / (BK / 2);
  a.group = raster_group();
  a.k_chunk = kTf32ChunkKb;
  a.splits = 1;
  a.kb_per_split = a.kb_total;
  a.C = C;
  a.ldc = ldc;
  a.status = device_status_ptr();
  const long long units = (long long)a.tiles_m * a.tiles_n;
  const int ncl = units < clusters ? (int)units : clusters;
  CUtensorMap unused{};
  kern<<<2 * ncl, kPairThreads, kSmem, stream>>>(ta, tb, unused, unused, a);
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

// true if the CTA-pair kernel took the problem
bool dispatch_pair(const GemmProblem& p, cudaStream_t s) {
  const bool am = p.a_mn, bm = p.b_mn;
  switch (p.epi) {
    case GEMM_EPI_BF16:
      if (!am && !bm) return launch_pair<false, false, GEMM_EPI_BF16>(p, s), true;
      if (!am && bm) return launch_pair<false, true, GEMM_EPI_BF16>(p, s), true;
      if (am && !bm) return launch_pair<true, false, GEMM_EPI_BF16>(p, s), true;
      return launch_pair<true, true, GEMM_EPI_BF16>(p, s), true;
    case GEMM_EPI_BIAS_GELU:
      if (!am && !bm) return launch_pair<false, false, GEMM_EPI_BIAS_GELU>(p, s), true;
      break;
    case GEMM_EPI_RESID:
      if (!am && !bm) return launch_pair<false, false, GEMM_EPI_RESID>(p, s), true;
      if (!am && bm) return launch_pair<false, true, GEMM_EPI_RESID>(p, s), true;
      break;
    case GEMM_EPI_DGELU:
      if (!am && bm) return launch_pair<false, true, GEMM_EPI_DGELU>(p, s), true;
      break;
    case GEMM_EPI_F32_ACCUM:
      if (am && bm) return launch_pair<true, true, GEMM_EPI_F32_ACCUM>(p, s), true;
      if (!am && bm) return launch_pair<false, true, GEMM_EPI_F32_ACCUM>(p, s), true;
      break;
    case GEMM_EPI_F32_STORE:
      if (!am && !bm) return launch_pair<false, false, GEMM_EPI_F32_STORE>(p, s), true;
      if (!am && bm) return launch_pair<false, true, GEMM_EPI_F32_STORE>(p, s), true;
      if (am && bm) return launch_pair<true, true, GEMM_EPI_F32_STORE>(p, s), true;
      break;
    default:
      break;
  }
  return false;
}

// UHFS_GEMM_PAIR=0 keeps every launch on the single-CTA kernel.
bool pair_enabled() {
  static const bool on = [] {
    const char* e = getenv("UHFS_GEMM_PAIR");
    return e == nullptr || std::string(e) != "0";
  }();
  return on;
}

// Measured on B200 (16384-row Linear layers, K = 768..3072, CUDA events):
// the pair kernel wins for bf16 / fp32 outputs at every K, for bias + GELU
// (78 vs 84 us at K = 768) and for the residual / dGELU epilogues once
// K >= 2048 (64 vs 70 us); with a short main loop the row-wise aux loads of
// the residual / dGELU epilogues bound the tile and the single-CTA kernel is
// 4-7 % faster.
// Residual epilogues go to CTA pairs from this K on (UHFS_GEMM_PAIR_EPI_K
// overrides); with coalesced operand loads the dGELU epilogue is faster on
// pairs at any K (fc2 dgrad, K = 768: 80.0 against 83.0 us) while the K = 768
// residual GEMM is not (27.7 against 25.9 us).
int pair_epi_min_k() {
  static const int k = [] {
    const char* e = getenv("UHFS_GEMM_PAIR_EPI_K");
    return e != nullptr ? atoi(e) : 2048;
  }();
  return k;
}

bool pair_preferred(const GemmProblem& p) {
  if (!pair_enabled()) return false;
  return p.epi == GEMM_EPI_BF16 || p.epi == GEMM_EPI_F32_STORE || p.epi == GEMM_EPI_F32_ACCUM ||
         p.epi == GEMM_EPI_BIAS_GELU || p.epi == GEMM_EPI_DGELU || p.K >= pair_epi_min_k();
}
}  // namespace

CUtensorMap make_tmap_bf16_2d(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                              uint32_t box_inner, uint32_t box_outer) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
  if ((row_stride_elems * 2) % 16 != 0) throw std::runtime_error("TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return m;
}

CUtensorMap make_tmap_f32_2d(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                             uint32_t box_inner, uint32_t box_outer) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
  if ((row_stride_elems * 4) % 16 != 0) throw std::runtime_error("TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * 4};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return m;
}

void set_gemm_trace(unsigned long long* buf) {
#ifdef UHFS_GEMM_TRACE
  g_gemm_trace = buf;
#else
  if (buf != nullptr)
    throw std::runtime_error("set_gemm_trace: the extension was built without UHFS_GEMM_TRACE "
                             "(rebuild with UNDERHFS_GEMM_TRACE=1)");
#endif
}

void gemm_tf32_tcgen05(const float* A, long long lda, const float* B, long long ldb, float* C, long long ldc, int M,
                       int N, int K, cudaStream_t stream) {
  if (M <= 0 || N <= 0) return;
  if (K <= 0) throw std::runtime_error("tf32 gemm: K must be positive");
  gemm_tf32_pair(A, lda, B, ldb, C, ldc, M, N, K, stream);
}

void gemm_bf16_tcgen05(const GemmProblem& p, cudaStream_t stream) {
  if (p.M <= 0 || p.N <= 0) return;
  if (p.K <= 0) throw std::runtime_error("gemm: K must be positive");
  if (p.N % 8 != 0) throw std::runtime_error("gemm: N must be a multiple of 8");
  if (p.ldc % 8 != 0 && p.epi != GEMM_EPI_F32_ACCUM && p.epi != GEMM_EPI_F32_STORE)
    throw std::runtime_error("gemm: ldc must be a multiple of 8");
  if ((p.epi == GEMM_EPI_F32_ACCUM || p.epi == GEMM_EPI_F32_STORE) && p.ldc % 4 != 0)
    throw std::runtime_error("gemm: fp32 ldc must be a multiple of 4");
  int bn = p.block_n;
  if (bn != 128 && bn != 256) bn = (p.N <= 128) ? 128 : 256;
  // CTA pairs: 256 x 256 tiles (one pass or stream-K; classic split-K stays
  // on single CTAs) without a fused gather, when both M and N exceed one
  // 128-row tile
  const bool pair_ok = (p.epi != GEMM_EPI_F32_ACCUM || p.splits <= 1) && p.ag.world == 0 && p.M > 128 &&
                       p.N > 128 && bn == 256;
  const bool want_pair = p.cta_pair == 1 || (p.cta_pair < 0 && pair_preferred(p));
  if (pair_ok && want_pair && dispatch_pair(p, stream)) return;
  if (bn == 256) dispatch_bn<256>(p, stream);
  else dispatch_bn<128>(p, stream);
}

}  // namespace uhfs
