// Shared device-side helpers for the sm_100a kernels of underhfs_b200.
//
// Everything here is written for Blackwell (sm_100a) only:
//   * bounded mbarrier waits on %globaltimer (no wait can spin forever: on
//     expiry the kernel records an error code in a device status word and the
//     caller unwinds, freeing TMEM on the way out);
//   * thin inline-PTX wrappers for mbarrier, TMA (cp.async.bulk.tensor, no
//     multicast form) and the 5th-generation tensor core
//     (tcgen05.alloc / mma / commit / ld).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace uhfs {

// ---------------------------------------------------------------------------
// Device error status.  Kernels never trap: a timed-out wait or a failed
// bounds check writes a code here and returns.  Host code reads it with
// read_device_status() (runtime/runtime.cu).
// ---------------------------------------------------------------------------
enum DeviceError : int {
  kErrNone = 0,
  kErrWaitTimeoutFull = 1,      // MMA waited too long for a TMA stage
  kErrWaitTimeoutEmpty = 2,     // producer waited too long for a free stage
  kErrWaitTimeoutAccum = 3,     // epilogue / MMA accumulator hand-off timed out
  kErrPeerTimeout = 4,          // a collective waited too long for a peer flag
  kErrBounds = 5,               // debug bounds check failed
};

struct DeviceStatus {
  int code;        // first error code recorded (0 = none)
  int where;       // kernel-specific site id
  int block;       // blockIdx.x of the reporting CTA
  int count;       // number of errors recorded
};

// The status word lives in device memory owned by the host runtime
// (device_status_ptr()); kernels that can time out receive it as an argument.
__device__ __forceinline__ void report_error(DeviceStatus* st, int code, int where) {
  if (st == nullptr) return;
  if (atomicCAS(&st->code, 0, code) == 0) {
    st->where = where;
    st->block = blockIdx.x;
  }
  atomicAdd(&st->count, 1);
}

// Debug index checks, compiled in with UNDERHFS_KERNEL_CHECKS=1 at build time
// (-DUHFS_KERNEL_CHECKS): a failed check records kErrBounds with a site id and
// evaluates to false so the caller skips the access.  Without the flag the
// check is the constant true and costs nothing.
#ifdef UHFS_KERNEL_CHECKS
#define UHFS_CHECK(cond, st, where) ((cond) ? true : (::uhfs::report_error((st), ::uhfs::kErrBounds, (where)), false))
#else
#define UHFS_CHECK(cond, st, where) true
#endif

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Default bound for every spin-wait in a kernel: 2 seconds of wall time.
constexpr uint64_t kWaitBoundNs = 2000000000ull;

// ---------------------------------------------------------------------------
// Shared-memory address helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool elect_one_sync() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and records `err`) if the phase did not flip
// within kWaitBoundNs.  Callers must then unwind without further waits that
// could block.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, DeviceStatus* st, int err,
                                                  int where) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (((++spins) & 255u) == 0u) {
      if (globaltimer_ns() - t0 > kWaitBoundNs) {
        report_error(st, err, where);
        return false;
      }
    }
  }
}

// Bounded wait called by all 32 lanes of a warp; the result is the same in
// every lane (false if the wait gave up in any lane).  Warps that go on to
// warp-collective tcgen05 instructions (.sync.aligned) use it so that a
// timeout in some lanes cannot leave a partial warp at such an instruction.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, DeviceStatus* st, int err,
                                               int where) {
  const bool ok = mbar_wait_bounded(bar, parity, st, err, where);
  return __all_sync(0xffffffffu, ok);
}

// ---------------------------------------------------------------------------
// TMA (tiled, non-multicast).  `coord0` is the innermost coordinate and must
// be a multiple of 16 bytes / element size; callers guarantee that by tiling
// in multiples of 64 bf16 elements along the contiguous dimension.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar, int coord0,
                                            int coord1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
          "r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(coord0), "r"(coord1)
      : "memory");
}

// Element-wise add of a shared tile into global memory through the tensor
// map (TMA reduce, fp32 add in L2).  Coordinates must be non-negative; the
// innermost one times the element size must be a multiple of 16 bytes.
// Completion is tracked with the issuing thread's bulk async-group.
__device__ __forceinline__ void tma_reduce_add_2d(const void* tmap, const void* smem_src, int coord0, int coord1) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(tmap)),
      "r"(smem_u32(smem_src)), "r"(coord0), "r"(coord1)
      : "memory");
}

// Shared tile -> global through the tensor map (TMA store); elements outside
// the tensor are not written.  Same coordinate rules as the reduce above.
__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* smem_src, int coord0, int coord1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tmap)),
               "r"(smem_u32(smem_src)), "r"(coord0), "r"(coord1)
               : "memory");
}

__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Wait until this thread's bulk operations have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Wait until this thread's bulk operations have completed.
// At most one bulk group (the most recent) may still be reading shared memory.
__device__ __forceinline__ void bulk_wait_group_read1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

__device__ __forceinline__ void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Named barrier over `count` threads (a multiple of 32); id 0 is __syncthreads.
__device__ __forceinline__ void named_barrier_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Vector fp32 reduction into global memory (no return value).
__device__ __forceinline__ void red_add_f32x4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (5th generation tensor core, accumulators in TMEM)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16/f16 in, f32 acc).
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16: A is read from TMEM (M
// lanes, K along the columns as packed 16-bit pairs, 8 columns per K = 16).
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// kind::tf32 (fp32 storage, tf32 math, f32 accumulate).
__device__ __forceinline__ void tc_mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once all tcgen05 ops previously issued by this thread
// have completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bit, 32 consecutive columns -> 32 registers per thread.  The
// wait::ld sits in the same asm statement so no consumer of the registers can
// be scheduled before the load has completed.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Same load without the wait, so several loads can be in flight; follow the
// batch with tmem_wait_ld_regs() over every destination register.
__device__ __forceinline__ void tmem_ld_32x32b_x32_async(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// tcgen05.wait::ld, then an empty volatile asm that redefines each register:
// consumers read the redefined values, which exist only after the wait.
template <int N>
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t* r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

// 32 lanes x 32 bit store of 32 consecutive columns; complete with tmem_wait_st().
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Hardware base-2 exponential (MUFU, approximate, flushes denormals);
// ex2(-inf) = +0.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x without the MUFU pipe (FMA and integer pipes only), for kernels whose
// exponentials saturate MUFU: Cody-Waite range reduction x = k + f with
// k = round(x) (the 1.5 * 2^23 addition trick) and |f| <= 1/2, a degree-3
// polynomial for 2^f whose coefficients were fitted here by relative least
// squares on [-1/2, 1/2] (max relative error 7.7e-5, ample for bf16
// probabilities), and k added to the exponent field.  x < -125 returns 0
// (masked scores are -inf).  tests/test_exp2_poly.py checks the same float32
// steps against exp2.
__device__ __forceinline__ float exp2_poly3(float x) {
  const float xc = fmaxf(x, -125.f);
  const float magic = 12582912.f;  // 1.5 * 2^23
  const float t = __fadd_rn(xc, magic);
  const int k = __float_as_int(t) - 0x4B400000;
  const float f = __fsub_rn(xc, __fsub_rn(t, magic));
  float p = fmaf(f, 0.05508868396282196f, 0.24260404706001282f);
  p = fmaf(p, f, 0.6932762265205383f);
  p = fmaf(p, f, 0.9999289512634277f);
  // k is added to the exponent field in unsigned (modular) arithmetic
  const float r = __uint_as_float(__float_as_uint(p) + ((unsigned)k << 23));
  return x < -125.f ? 0.f : r;
}

// Packed fp32 pairs (sm_100 f32x2 instructions: one issue slot computes both
// halves), used by the softmax loops whose issue rate bounds them.
__device__ __forceinline__ float2 f2_fma(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n.reg .b64 ra, rb, rc, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\nmov.b64 rc, {%6, %7};\n"
      "fma.rn.f32x2 rd, ra, rb, rc;\nmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

__device__ __forceinline__ float2 f2_add(float2 a, float2 b) {
  float2 d;
  asm("{\n.reg .b64 ra, rb, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\n"
      "add.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ __forceinline__ float2 f2_mul(float2 a, float2 b) {
  float2 d;
  asm("{\n.reg .b64 ra, rb, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\n"
      "mul.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ __forceinline__ float2 f2_sub(float2 a, float2 b) {
  float2 d;
  asm("{\n.reg .b64 ra, rb, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\n"
      "sub.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// max of three floats in one instruction (sm_100 three-input max.f32).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// exp2_poly3 for a pair, with the additions and the polynomial in packed
// f32x2 instructions (the same float32 steps per half).  Inputs below -125
// are clamped there and return 2^-125 (about 2.4e-38) instead of exactly 0,
// which adds nothing measurable to a softmax row sum; every other input gives
// exp2_poly3's result bit for bit.
__device__ __forceinline__ float2 exp2_poly3_x2(float2 x) {
  const float2 xc = make_float2(fmaxf(x.x, -125.f), fmaxf(x.y, -125.f));
  const float2 magic = make_float2(12582912.f, 12582912.f);  // 1.5 * 2^23
  const float2 t = f2_add(xc, magic);
  const float2 f = f2_sub(xc, f2_sub(t, magic));
  float2 p = f2_fma(f, make_float2(0.05508868396282196f, 0.05508868396282196f),
                    make_float2(0.24260404706001282f, 0.24260404706001282f));
  p = f2_fma(p, f, make_float2(0.6932762265205383f, 0.6932762265205383f));
  p = f2_fma(p, f, make_float2(0.9999289512634277f, 0.9999289512634277f));
  // k = bits(t) - 0x4B400000 and (bits(t) << 23) == (k << 23) mod 2^32
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Dynamic shared memory rounded up to a 1024-byte boundary (the 128-byte
// swizzle atom) by pointer arithmetic, so the compiler keeps the shared
// address space and emits shared (not generic) loads and stores.
__device__ __forceinline__ uint8_t* smem_align1024(uint8_t* raw) {
  return raw + ((1024u - (smem_u32(raw) & 1023u)) & 1023u);
}

// Shared-memory matrix descriptor (Blackwell "version 1" format).
//   start address, leading-dim byte offset and stride-dim byte offset are in
//   16-byte units; layout 2 = 128-byte swizzle.
__device__ __forceinline__ uint64_t make_smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                                   uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;  // descriptor version for sm_100
  d |= (uint64_t)(layout & 0x7u) << 61;
  return d;
}

constexpr uint32_t kSwizzle128B = 2;

// Instruction descriptor for kind::f16 / kind::tf32 with f32 accumulation.
//   fmt: 0 = f16, 1 = bf16, 2 = tf32; major: 0 = K-major, 1 = MN-major.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t fmt, uint32_t a_mn, uint32_t b_mn, uint32_t M,
                                                  uint32_t N) {
  return (1u << 4)              // D = f32
         | (fmt << 7)           // A format
         | (fmt << 10)          // B format
         | (a_mn << 15)         // A major
         | (b_mn << 16)         // B major
         | ((N >> 3) << 17)     // N / 8
         | ((M >> 4) << 24);    // M / 16
}

// ---------------------------------------------------------------------------
// CTA pairs: a cluster of two CTAs on one TPC driving the tensor cores of
// both SMs as one (tcgen05 .cta_group::2).  CTA rank 0 (the leader) issues
// the MMAs; each CTA stages half of A and half of B in its own shared memory
// at the same offsets, and each holds half of the accumulator rows in its
// own TMEM.  Barriers of the other CTA are addressed through `mapa`.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}

// shared::cluster address of the object at `p` in the CTA of rank `rank`.
__device__ __forceinline__ uint32_t smem_cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

// Every thread of both CTAs; orders shared-memory writes (barrier init, the
// TMEM address) before the other CTA's accesses.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier given by its shared::cluster address (either CTA).
// Default semantics (release at CTA scope): used after tcgen05.wait::ld +
// tcgen05.fence::before_thread_sync, which order the TMEM reads themselves.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// mbar_wait_bounded for barriers that the other CTA of the pair signals.
__device__ __forceinline__ bool mbar_wait_bounded_cluster(uint64_t* bar, uint32_t parity, DeviceStatus* st, int err,
                                                          int where) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (((++spins) & 255u) == 0u) {
      if (globaltimer_ns() - t0 > kWaitBoundNs) {
        report_error(st, err, where);
        return false;
      }
    }
  }
}

__device__ __forceinline__ bool mbar_wait_warp_cluster(uint64_t* bar, uint32_t parity, DeviceStatus* st, int err,
                                                       int where) {
  const bool ok = mbar_wait_bounded_cluster(bar, parity, st, err, where);
  return __all_sync(0xffffffffu, ok);
}

// TMA tile load into this CTA's shared memory whose completion is counted on
// the leader CTA's mbarrier (`bar_cluster`: its shared::cluster address).
// No multicast: each CTA loads its own half of the operands.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const void* tmap, uint32_t bar_cluster, int coord0,
                                                 int coord1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar_cluster), "r"(coord0), "r"(coord1)
      : "memory");
}

__device__ __forceinline__ void tc_mma_tf32_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Paired TMEM allocation: one warp of each CTA (the same warp index in both)
// executes it; both CTAs receive the same column range.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D (+)= A * B^T over the pair: M = 256 rows (128 per CTA), A and B halves
// read from each CTA's shared memory at the descriptors' (common) offsets.
__device__ __forceinline__ void tc_mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the mbarrier at `bar_cluster` (either CTA) once the pair MMAs
// issued so far by this thread have completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
               : "memory");
}

// ---------------------------------------------------------------------------
// Small numeric helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  const float k1 = 0.044715f;
  float u = k0 * (x + k1 * x * x * x);
  return 0.5f * x * (1.0f + tanhf(u));
}

__device__ __forceinline__ float gelu_tanh_grad(float x) {
  const float k0 = 0.7978845608028654f;
  const float k1 = 0.044715f;
  float x2 = x * x;
  float u = k0 * (x + k1 * x2 * x);
  float t = tanhf(u);
  float du = k0 * (1.0f + 3.0f * k1 * x2);
  return 0.5f * (1.0f + t) + 0.5f * x * (1.0f - t * t) * du;
}

// Hardware tanh (MUFU tanh.approx: relative error around 2^-11), for values
// that are rounded to a 16-bit float right after.
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The same GELU forms on the hardware tanh: used where the result is stored
// as bf16 / fp16 (GEMM epilogues, 16-bit element-wise kernels).
__device__ __forceinline__ float gelu_tanh_fast(float x) {
  const float k0 = 0.7978845608028654f;
  const float k1 = 0.044715f;
  const float u = k0 * fmaf(k1 * x, x * x, x);
  const float hx = 0.5f * x;
  return fmaf(hx, tanh_approx(u), hx);
}

__device__ __forceinline__ float gelu_tanh_grad_fast(float x) {
  const float k0 = 0.7978845608028654f;
  const float k1 = 0.044715f;
  const float x2 = x * x;
  const float u = k0 * fmaf(k1 * x2, x, x);
  const float t = tanh_approx(u);
  const float du = k0 * fmaf(3.0f * k1, x2, 1.0f);
  return 0.5f * (1.0f + t) + 0.5f * x * fmaf(-t, t, 1.0f) * du;
}

// The same tanh-form GELU and its derivative on a pair of values with packed
// f32x2 arithmetic (GEMM epilogues, where the per-element math bounds the
// epilogue's issue rate):
//   gelu(x)  = hx (1 + t),                  hx = x / 2
//   gelu'(x) = (1 + t) / 2 * (1 + x du (1 - t)),
//   t = tanh(x (k0 + k0 k1 x^2)),  du = k0 (1 + 3 k1 x^2)
// (1 - t^2 = (1 - t)(1 + t) folds the two terms of the derivative).
__device__ __forceinline__ float2 gelu_tanh_fast_x2(float2 x) {
  const float k0 = 0.7978845608028654f, k0k1 = 0.7978845608028654f * 0.044715f;
  const float2 x2 = f2_mul(x, x);
  const float2 u = f2_mul(x, f2_fma(x2, make_float2(k0k1, k0k1), make_float2(k0, k0)));
  const float2 t = make_float2(tanh_approx(u.x), tanh_approx(u.y));
  const float2 hx = f2_mul(x, make_float2(0.5f, 0.5f));
  return f2_fma(hx, t, hx);
}

__device__ __forceinline__ float2 gelu_tanh_grad_fast_x2(float2 x) {
  const float k0 = 0.7978845608028654f, k0k1 = 0.7978845608028654f * 0.044715f;
  const float2 x2 = f2_mul(x, x);
  const float2 u = f2_mul(x, f2_fma(x2, make_float2(k0k1, k0k1), make_float2(k0, k0)));
  const float2 t = make_float2(tanh_approx(u.x), tanh_approx(u.y));
  const float2 du = f2_fma(x2, make_float2(3.0f * k0k1, 3.0f * k0k1), make_float2(k0, k0));
  const float2 a = f2_mul(x, du);
  const float2 c = f2_fma(a, f2_sub(make_float2(1.0f, 1.0f), t), make_float2(1.0f, 1.0f));
  const float2 h = f2_fma(t, make_float2(0.5f, 0.5f), make_float2(0.5f, 0.5f));
  return f2_mul(h, c);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Launch accounting shared with the host runtime (stream stats contract).
void note_launch();
// Per-device status word for bounded waits: a static __device__ object of
// the runtime module, resolved per device with cudaGetSymbolAddress (never
// allocates).
DeviceStatus* device_status_ptr();

// Runs a set-up step (cudaFuncSetAttribute and the like) once per device.
// Function attributes are per device, so a flag shared by every device would
// skip the set-up on the second GPU a process launches on.  Concurrent first
// calls may both run the step, which must therefore be idempotent.
struct PerDeviceOnce {
  unsigned long long mask = 0;  // bit d: done on device d (ordinals 0..63)
  template <class F>
  void operator()(F&& f) {
    int dev = 0;
    cudaGetDevice(&dev);
    const unsigned long long bit = 1ull << (dev & 63);
    if (__atomic_load_n(&mask, __ATOMIC_ACQUIRE) & bit) return;
    f();
    __atomic_fetch_or(&mask, bit, __ATOMIC_ACQ_REL);
  }
};

}  // namespace uhfs

#define UHFS_CUDA_CHECK(expr)                                                                   \
  do {                                                                                          \
    cudaError_t _e = (expr);                                                                    \
    if (_e != cudaSuccess) {                                                                    \
      throw std::runtime_error(std::string("CUDA error: ") + cudaGetErrorString(_e) + " at " + \
                               __FILE__ + ":" + std::to_string(__LINE__));                     \
    }                                                                                           \
  } while (0)
