// Host launchers of the memory-bound sm_100a kernels.  Every launcher takes
// raw device pointers and the CUDA stream to launch on; none allocates.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace uhfs {

enum DType : int { DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2 };
enum BinOp : int { OP_ADD = 0, OP_MUL = 1, OP_SUB = 2, OP_DIV = 3 };

// ---- elementwise / cast / reduce (reference K1..K11, cuda/kernels.cu:20-119)
void ew_binary(int op, int dtype, const void* a, const void* b, void* out, long long n, cudaStream_t s);
void ew_scalar(int op, int dtype, const void* a, float scalar, void* out, long long n, cudaStream_t s);
void cast(int src_dtype, int dst_dtype, const void* src, void* dst, long long n, cudaStream_t s);
// out[0] = sum(x) in fp32; `partials` must hold reduce_sum_partials() floats, `counter` one zeroed int.
int reduce_sum_partials();
void reduce_sum(int dtype, const void* x, long long n, float* out, float* partials, unsigned int* counter,
                cudaStream_t s);

// ---- RMSNorm (reference nn.py:166-181; here with a real backward)
void rmsnorm_fwd(int dtype, const void* x, const void* w, void* y, float* rstd, int rows, int cols, float eps,
                 cudaStream_t s);
// dx = rmsnorm_bwd(dy) (+ dres if dres != null); dw_accum += sum_rows(dy * xhat) (fp32).
void rmsnorm_bwd(int dtype, const void* dy, const void* x, const void* w, const float* rstd, const void* dres,
                 void* dx, float* dw_accum, int rows, int cols, cudaStream_t s);

// ---- embedding (reference nn.py:184-217): token gather + optional learned position
void embedding_fwd(int dtype, const int64_t* ids, const void* tok, const void* pos, void* out, int rows, int dim,
                   int seq_len, long long vocab, cudaStream_t s);
// ids outside [0, vocab) (vocab > 0) are reported as kErrBounds and skipped
void embedding_bwd(int dtype, const int64_t* ids, const void* dout, float* dtok, float* dpos, int rows, int dim,
                   int seq_len, long long vocab, cudaStream_t s);

// ---- fused softmax cross-entropy (reference functional.py:20-76)
// loss_rows[r] = -log softmax(logits[r])[target[r]];  if dlogits != null:
// dlogits[r] = (softmax(logits[r]) - onehot) * grad_scale (* *grad_scale_ptr when given; may alias logits).
void softmax_ce_fwd_bwd(int dtype, const void* logits, long long ld, const int64_t* targets, float* loss_rows,
                        void* dlogits, int rows, int cols, float grad_scale, const float* grad_scale_ptr,
                        cudaStream_t s);
// Row softmax (reference tensor.py:966-1027): y = softmax(x) along the last dim.
void softmax_rows(int dtype, const void* x, void* y, int rows, int cols, cudaStream_t s);
void softmax_rows_bwd(int dtype, const void* y, const void* dy, void* dx, int rows, int cols, cudaStream_t s);

// ---- GELU (tanh form, reference functional.py:83-85) and bias-gradient column sums
void gelu_fwd(int dtype, const void* x, void* y, long long n, cudaStream_t s);
void gelu_bwd(int dtype, const void* x, const void* dy, void* dx, long long n, cudaStream_t s);
void colsum_accum(const __nv_bfloat16* x, long long ld, float* out, int rows, int cols, cudaStream_t s);

// ---- AdamW (reference optim.py:144-156 / kernels.cu:121-145)
struct AdamWArgs {
  float lr, beta1, beta2, eps, weight_decay;
  int decoupled;          // 0: reference L2-coupled (g += wd*p); 1: decoupled (p -= lr*wd*p)
  float grad_scale;       // gradient multiplier (1/world, loss scale) fused into the read
  const int* step_ptr;    // device step counter (read, 1-based) or null -> `step`
  int step;
  const float* lr_ptr;    // optional device learning-rate override
};
// Flat fp32 master/m/v/grad; optional bf16 model copy written with the update.
void adamw_step(const AdamWArgs& a, float* p32, const float* g, float* m, float* v, __nv_bfloat16* p16,
                long long n, cudaStream_t s);
void adamw_step_bf16grad(const AdamWArgs& a, float* p32, const __nv_bfloat16* g, float* m, float* v,
                         __nv_bfloat16* p16, long long n, cudaStream_t s);
// Plain fp32 in-place AdamW on a single tensor (param/grad/m/v all fp32).
void increment_counter(int* counter, cudaStream_t s);
void fill_f32(float* x, float v, long long n, cudaStream_t s);

// ---- reference-contract attention / conv (small, fp32)
void attention_naive_f32(const float* q, const float* k, const float* v, float* out, int tokens, int features,
                         float scale, bool causal, cudaStream_t s);
void conv2d_fwd_f32(const float* x, const float* w, const float* b, float* y, int N, int C, int H, int W, int K,
                    int R, int S, int sh, int sw, int ph, int pw, int P, int Q, cudaStream_t s);
void conv2d_dgrad_f32(const float* dy, const float* w, float* dx, int N, int C, int H, int W, int K, int R, int S,
                      int sh, int sw, int ph, int pw, int P, int Q, cudaStream_t s);
void conv2d_wgrad_f32(const float* dy, const float* x, float* dw, float* db, int N, int C, int H, int W, int K,
                      int R, int S, int sh, int sw, int ph, int pw, int P, int Q, cudaStream_t s);

// ---- flash attention (bf16, causal or full), [B, T, H, D] rows with strides
struct AttnParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  __nv_bfloat16* o;
  float* lse;                   // [B, H, T]
  long long q_stride_b, q_stride_t;  // element strides (head stride = D)
  long long k_stride_b, k_stride_t;
  long long v_stride_b, v_stride_t;
  long long o_stride_b, o_stride_t;
  int B, H, T, D;
  float scale;
  int causal;
};
struct AttnBwdParams {
  AttnParams f;
  const __nv_bfloat16* dout;
  long long do_stride_b, do_stride_t;
  __nv_bfloat16* dq;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  long long dq_stride_b, dq_stride_t;
  long long dk_stride_b, dk_stride_t;
  long long dv_stride_b, dv_stride_t;
  float* delta;      // [B, H, T] scratch
  float* dq_accum;   // [B, T, H, D] fp32 scratch (zeroed by the launcher's prologue kernel)
};
void flash_attn_fwd(const AttnParams& p, cudaStream_t s);
// Per-step clock stamps of the tcgen05 attention backward (head 0 of batch 0):
// a buffer of ceil(T/128) * 16 * 64 uint64 values, or nullptr (off).
void set_attn_bwd_trace(unsigned long long* buf);
// Per-key-block clock stamps of the tcgen05 attention forward (head 0 of
// batch 0): a buffer of ceil(T/256) * 16 * 64 uint64 values, or nullptr.
void set_attn_fwd_trace(unsigned long long* buf);
// tcgen05/TMEM forward for the fused-QKV layout (attention_tc.cu)
bool flash_attn_fwd_tc_supported(const AttnParams& p);
void flash_attn_fwd_tc(const AttnParams& p, cudaStream_t s);
void flash_attn_bwd(const AttnBwdParams& p, cudaStream_t s);
// tcgen05/TMEM main backward kernel (attention_tc_bwd.cu); flash_attn_bwd runs the
// delta / dQ-zeroing prologue and the dQ conversion around it
bool flash_attn_bwd_tc_supported(const AttnBwdParams& p);
void flash_attn_bwd_tc_main(const AttnBwdParams& p, cudaStream_t s);

// ---- headless isometric voxel rasteriser (liveSee): quads [n][8] float, colors RGBA8
void raster_iso(const float* quads, const unsigned int* colors, int nquads, unsigned int* order, unsigned int* rgba,
                int width, int height, cudaStream_t s);

}  // namespace uhfs
