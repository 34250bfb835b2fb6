// Fused AdamW over flat fp32 master / moment / gradient buffers.
//
// Reference: the fp32 per-tensor kernel at cuda/kernels.cu:121-145 (host
// round trip per parameter, bias corrections from the host) and the Python
// update in optim.py:144-156.  Here one launch updates every parameter of the
// model: all state lives in one flat buffer, the step counter and learning
// rate can be read from device memory (so the update can be captured in a
// CUDA graph and replayed), the gradient scale (1/world, loss scale) is
// folded into the gradient read, and the bf16 model copy is written in the
// same pass.  Semantics: weight decay is L2-coupled like the reference
// (g += wd * p) unless `decoupled` selects the AdamW-paper form.
#include <stdexcept>

#include "common.cuh"
#include "kernels.h"

namespace uhfs {

namespace {

template <typename G>
__device__ __forceinline__ float gload(const G* g, long long i);
template <>
__device__ __forceinline__ float gload<float>(const float* g, long long i) { return g[i]; }
template <>
__device__ __forceinline__ float gload<__nv_bfloat16>(const __nv_bfloat16* g, long long i) {
  return __bfloat162float(g[i]);
}

template <typename G>
__global__ void adamw_kernel(AdamWArgs a, float* __restrict__ p32, const G* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ p16, long long n) {
  const int step = a.step_ptr != nullptr ? *a.step_ptr : a.step;
  const float lr = a.lr_ptr != nullptr ? *a.lr_ptr : a.lr;
  const float bc1 = 1.0f - powf(a.beta1, (float)step);
  const float bc2 = 1.0f - powf(a.beta2, (float)step);
  const float step_size = lr / bc1;
  const float inv_sqrt_bc2 = rsqrtf(bc2);
  const float b1 = a.beta1, b2 = a.beta2, wd = a.weight_decay, eps = a.eps, gs = a.grad_scale;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride) {
    float p = p32[i];
    float gr = gload<G>(g, i) * gs;
    if (a.decoupled) {
      p -= lr * wd * p;
    } else {
      gr += wd * p;
    }
    float mi = b1 * m[i] + (1.0f - b1) * gr;
    float vi = b2 * v[i] + (1.0f - b2) * gr * gr;
    m[i] = mi;
    v[i] = vi;
    // p -= lr * m_hat / (sqrt(v_hat) + eps)
    p -= step_size * mi / (sqrtf(vi) * inv_sqrt_bc2 + eps);
    p32[i] = p;
    if (p16 != nullptr) p16[i] = __float2bfloat16_rn(p);
  }
}

int adam_grid(long long n) {
  long long g = (n + 255) / 256;
  if (g > 148LL * 16) g = 148LL * 16;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace

void adamw_step(const AdamWArgs& a, float* p32, const float* g, float* m, float* v, __nv_bfloat16* p16, long long n,
                cudaStream_t s) {
  if (n <= 0) return;
  adamw_kernel<float><<<adam_grid(n), 256, 0, s>>>(a, p32, g, m, v, p16, n);
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

void adamw_step_bf16grad(const AdamWArgs& a, float* p32, const __nv_bfloat16* g, float* m, float* v,
                         __nv_bfloat16* p16, long long n, cudaStream_t s) {
  if (n <= 0) return;
  adamw_kernel<__nv_bfloat16><<<adam_grid(n), 256, 0, s>>>(a, p32, g, m, v, p16, n);
  note_launch();
  UHFS_CUDA_CHECK(cudaGetLastError());
}

}  // namespace uhfs
