// Allocation-free entry point for the flash-attention backward pass.
//
// This entry point has no counterpart in the reference implementation.
//
// Why it exists: the regular backward (flash_attn_bwd, reached from Python
// through underhfs_b200.ops.kernels.flash_attn_qkv_backward) needs two scratch
// buffers -- the per-row softmax statistic `delta` and an fp32 accumulator for
// dQ -- and expects its caller to allocate them.  Some callers cannot do that:
// code that links this library from C or another language without a CUDA
// allocator of its own, callers with a fixed memory budget that forbids any
// allocation once set-up is finished, and code running where cudaMalloc is not
// permitted at all (for example inside an allocator callback).  For them,
// uhfs_flash_attn_bwd_noalloc() takes only inputs and outputs and uses a
// scratch region that lives in this library's own device memory.
//
// The scratch region is a file-scope __device__ array of kScratchBytes
// (16 MiB).  Every GPU on which this library is loaded reserves it until the
// process exits, whether or not the entry point is used.  A call fits when
//     4 * B*H*T            (delta)
//   + 4 * B*T*H*D          (dQ accumulator, placed at the next 256-byte boundary)
// is at most 16 MiB; larger problems are rejected with an error code and a
// message, never truncated.  Example: B=2, T=1024, H=8, D=128 uses 8.06 MiB.
//
// Use rules:
//   * The first call on a device looks up, with that device current, the
//     device addresses of the scratch array and of the library's device status
//     word (both static __device__ objects, resolved with cudaGetSymbolAddress;
//     neither lookup allocates), and sets the kernel's shared-memory attribute.
//     Make that first call before any CUDA stream capture begins.
//   * The kernels' waits are bounded: a wait that runs out records a code in
//     the device status word and the kernel returns early, so the call itself
//     still returns 0.  Read (and optionally clear) that word with
//     uhfs_flash_attn_bwd_noalloc_status() after the stream has finished.
//   * All calls on a device share the one array and nothing is cleared between
//     calls except what the kernels initialise themselves (the dQ accumulator
//     is zeroed by the first kernel of every call; delta is fully rewritten).
//     Two calls that overlap on the GPU -- on different streams, or from
//     different host threads without ordering -- race on the array and give
//     wrong results.  Serialise them (same stream, or events).
//   * The entry point calls no cudaMalloc, cudaFree or allocating library
//     routine.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <stdexcept>

#include "attention_noalloc.h"
#include "kernels.h"
#include "../runtime/runtime.h"

namespace uhfs {
namespace {

constexpr size_t kScratchBytes = size_t(16) << 20;

static __device__ __align__(256) unsigned char g_attn_bwd_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};
// One message per host thread, so calls from different threads (on the same or
// different devices) do not overwrite each other's message.
thread_local char g_last_error[256] = "";

void set_error(const char* msg) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s", msg);
}

// Device address of the scratch array for the current device (looked up once).
void* scratch_for_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_bwd_scratch);
    if (e != cudaSuccess) {
      set_error(cudaGetErrorString(e));
      return nullptr;
    }
    g_scratch_ptr[dev] = p;
  }
  return g_scratch_ptr[dev];
}

}  // namespace
}  // namespace uhfs

extern "C" {

// Maximum scratch bytes (delta + aligned dQ accumulator) a call may need.
__attribute__((visibility("default"))) unsigned long long uhfs_flash_attn_bwd_noalloc_capacity() {
  return (unsigned long long)uhfs::kScratchBytes;
}

// Message of the last failed call made by the calling host thread ("" after success).
__attribute__((visibility("default"))) const char* uhfs_flash_attn_bwd_noalloc_error() { return uhfs::g_last_error; }

// Backward of causal / full multi-head attention over a fused QKV projection.
//   qkv  [B*T, 3*H*D] bf16  (q | k | v column blocks, as produced by the fused QKV GEMM)
//   o    [B*T, H*D]   bf16  forward output
//   lse  [B, H, T]    fp32  forward log-sum-exp (base 2), from the forward kernel
//   dout [B*T, H*D]   bf16  gradient of o
//   dqkv [B*T, 3*H*D] bf16  output gradients (q | k | v blocks)
// head_dim D must be 64 or 128.  `stream` is a cudaStream_t (0 = legacy default).
// Returns 0 on success, 1 for invalid arguments, 2 when the problem needs more
// scratch than uhfs_flash_attn_bwd_noalloc_capacity(), 3 for a CUDA error.
// Device status word of the current device: returns the first error code a
// kernel of this library recorded there (0 = none; 1-3 a bounded wait on the
// GPU ran out, 4 a peer wait ran out, 5 a bounds check failed), and clears the
// word when `clear` is non-zero.  Reads with a synchronous cudaMemcpy, so call
// it after the work has finished (and outside stream capture); returns -1 if
// the word cannot be read.
__attribute__((visibility("default"))) int uhfs_flash_attn_bwd_noalloc_status(int clear) {
  try {
    const uhfs::DeviceStatusHost st = uhfs::read_device_status(clear != 0);
    return st.code;
  } catch (const std::exception& e) {
    uhfs::set_error(e.what());
    return -1;
  }
}

__attribute__((visibility("default"))) int uhfs_flash_attn_bwd_noalloc(const void* qkv, const void* o,
                                                                      const float* lse, const void* dout,
                                                                      void* dqkv, int B, int T, int H, int D,
                                                                      float scale, int causal, void* stream) {
  using namespace uhfs;
  set_error("");
  if (qkv == nullptr || o == nullptr || lse == nullptr || dout == nullptr || dqkv == nullptr || B <= 0 || T <= 0 ||
      H <= 0 || (D != 64 && D != 128)) {
    set_error("invalid argument: null pointer, non-positive size, or head_dim not in {64, 128}");
    return 1;
  }
  const unsigned long long rows = (unsigned long long)B * H * T;
  const unsigned long long delta_bytes = rows * 4ull;
  const unsigned long long dq_off = (delta_bytes + 255ull) & ~255ull;
  const unsigned long long need = dq_off + rows * (unsigned long long)D * 4ull;
  if (need > kScratchBytes) {
    char msg[256];
    std::snprintf(msg, sizeof(msg),
                  "problem needs %llu scratch bytes (B*H*T=%llu, D=%d) but the static scratch holds %llu bytes",
                  need, rows, D, (unsigned long long)kScratchBytes);
    set_error(msg);
    return 2;
  }
  unsigned char* scratch = static_cast<unsigned char*>(scratch_for_current_device());
  if (scratch == nullptr) {
    if (g_last_error[0] == '\0') set_error("could not resolve the scratch array on the current device");
    return 3;
  }
  const long long F = (long long)H * D;
  const __nv_bfloat16* base = static_cast<const __nv_bfloat16*>(qkv);
  __nv_bfloat16* dbase = static_cast<__nv_bfloat16*>(dqkv);
  AttnBwdParams p{};
  p.f.q = base;
  p.f.k = base + F;
  p.f.v = base + 2 * F;
  p.f.o = const_cast<__nv_bfloat16*>(static_cast<const __nv_bfloat16*>(o));
  p.f.lse = const_cast<float*>(lse);
  p.f.q_stride_b = p.f.k_stride_b = p.f.v_stride_b = (long long)T * 3 * F;
  p.f.q_stride_t = p.f.k_stride_t = p.f.v_stride_t = 3 * F;
  p.f.o_stride_b = (long long)T * F;
  p.f.o_stride_t = F;
  p.f.B = B;
  p.f.H = H;
  p.f.T = T;
  p.f.D = D;
  p.f.scale = scale;
  p.f.causal = causal ? 1 : 0;
  p.dout = static_cast<const __nv_bfloat16*>(dout);
  p.do_stride_b = (long long)T * F;
  p.do_stride_t = F;
  p.dq = dbase;
  p.dk = dbase + F;
  p.dv = dbase + 2 * F;
  p.dq_stride_b = p.dk_stride_b = p.dv_stride_b = (long long)T * 3 * F;
  p.dq_stride_t = p.dk_stride_t = p.dv_stride_t = 3 * F;
  p.delta = reinterpret_cast<float*>(scratch);
  p.dq_accum = reinterpret_cast<float*>(scratch + dq_off);
  try {
    flash_attn_bwd(p, static_cast<cudaStream_t>(stream));
  } catch (const std::exception& e) {
    set_error(e.what());
    return 3;
  }
  return 0;
}

}  // extern "C"
