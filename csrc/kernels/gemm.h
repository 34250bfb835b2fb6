// Host-side interface of the tcgen05 GEMM (gemm_tcgen05.cu) and of the
// fp32 SIMT GEMM (gemm_f32.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace uhfs {

enum GemmEpilogue : int {
  GEMM_EPI_BF16 = 0,       // C = acc (+ bias)                       bf16 out
  GEMM_EPI_BIAS_GELU = 1,  // aux_out = acc + bias; C = gelu(aux_out) bf16 out
  GEMM_EPI_RESID = 2,      // C = acc (+ bias) + aux                  bf16 out (C may alias aux)
  GEMM_EPI_DGELU = 3,      // C = acc * gelu'(aux)                    bf16 out
  GEMM_EPI_F32_ACCUM = 4,  // C += acc   (fp32, atomic: split-K safe)
  GEMM_EPI_F32_STORE = 5,  // C = acc    (fp32)
};

// Fused all-gather of B rows (ZeRO-3 weights).  The kernel's pusher warp
// copies this rank's rows of a unit's weight matrices into every rank's
// gather buffer and publishes one flag per 32 rows (release, system scope);
// the TMA producer waits for the flags covering a B tile (K-major B: the
// tile's N rows; MN-major B: the k-block's rows) before loading it from the
// local gather buffer.  Flags hold an epoch that grows with every gather, so
// they are never reset.  Before pushing into rank p a pusher waits for p's
// ready flag: p raises it when this kernel starts there, i.e. after p has
// finished every earlier kernel that read the same gather slot.
struct GemmGatherSeg {
  const void* src = nullptr;    // this rank's rows (local shard), row-contiguous
  long long dst_off_bytes = 0;  // where these rows go inside every rank's gather region
  long long rows = 0;
  long long row_bytes = 0;      // multiple of 16
  int flag_base = 0;            // flag index of the first 32-row chunk
};

struct GemmGather {
  int world = 0;  // 0 = no fused gather
  int rank = 0;
  unsigned epoch = 0;
  char* peer_data[8] = {};      // gather region base on every rank
  unsigned* peer_flags[8] = {};  // flag array on every rank
  int nseg = 0;                 // segments this kernel pushes (0 = only wait)
  GemmGatherSeg seg[8];
  int b_flag_base = -1;         // flag of B row 0; -1 = B is not gathered
  int ready_base = 0;           // per-rank ready flags start here
};

struct GemmProblem {
  int M = 0, N = 0, K = 0;
  const __nv_bfloat16* A = nullptr;  // K-major: A[m*lda + k]; MN-major: A[k*lda + m]
  long long lda = 0;
  bool a_mn = false;
  const __nv_bfloat16* B = nullptr;  // K-major: B[n*ldb + k]; MN-major: B[k*ldb + n]
  long long ldb = 0;
  bool b_mn = false;
  void* C = nullptr;
  long long ldc = 0;
  int epi = GEMM_EPI_BF16;
  const __nv_bfloat16* bias = nullptr;
  const __nv_bfloat16* aux = nullptr;
  long long ld_aux = 0;
  __nv_bfloat16* aux_out = nullptr;
  long long ld_aux_out = 0;
  int splits = 1;     // split-K factor (GEMM_EPI_F32_ACCUM only); 0 = stream-K (equal k-block
                      // ranges per CTA, partial tiles accumulated by the fp32 epilogue)
  int block_n = 0;    // 0 = choose, else 128 or 256
  int max_ctas = 0;   // 0 = one per SM
  int cta_pair = -1;  // 256 x 256 tiles on CTA pairs: -1 = choose, 0 = off, 1 = on where supported
  GemmGather ag;      // fused all-gather of B rows (ZeRO-3), off by default
};

void gemm_bf16_tcgen05(const GemmProblem& p, cudaStream_t stream);

// Trace builds (-DUHFS_GEMM_TRACE): per-unit clock stamps of CTA 0 of the
// single-CTA kernel into buf[event * 16 + unit] (20 events); nullptr turns it off.
void set_gemm_trace(unsigned long long* buf);

// fp32 C[M,N] (row stride ldc) = A[M,K] B[N,K]^T with tf32 tensor-core math
// (both operands K-major fp32, rows 16-byte aligned, strides multiples of 4).
void gemm_tf32_tcgen05(const float* A, long long lda, const float* B, long long ldb, float* C, long long ldc, int M,
                       int N, int K, cudaStream_t stream);

// fp32 C[M,N] = A[M,K] x B (b_trans=false -> B[K,N], true -> B[N,K]) as three
// tf32 tensor-core products per term (3xTF32): x = hi + lo with hi the tf32
// rounding of x, and C = hi(A) lo(B) + lo(A) hi(B) + hi(A) hi(B), accumulated
// in fp32 -- one GEMM over operands concatenated along K.  The workspaces hold
// the split operands: ws_a M x 3Kp floats, ws_b N x 3Kp floats, Kp = K rounded
// up to 32.
void gemm_f32_3xtf32(const float* A, const float* B, float* C, int M, int N, int K, bool b_trans, float* ws_a,
                     float* ws_b, cudaStream_t stream);

// C[M,N] (fp32) = A[M,K] (fp32, row-major) x B (fp32): b_trans=false -> B[K,N], true -> B[N,K].
// Exact fp32 FMA accumulation (the fp32 contract of the public matmul).
void gemm_f32_simt(const float* A, const float* B, float* C, int M, int N, int K, bool b_trans, cudaStream_t stream);

}  // namespace uhfs
