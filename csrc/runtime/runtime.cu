// Host runtime: stream stats, caching allocator, device status word,
// TensorCore, CudaTensor storage, one-shot host helpers and the NCCL process
// group.  See runtime.h for the reference contracts each piece keeps.
#ifndef UHFS_NO_NCCL
#include <nccl.h>
#endif

#include <atomic>
#include <cmath>
#include <cstring>
#include <sstream>
#include <stdexcept>

#include "../kernels/common.cuh"
#include "../kernels/gemm.h"
#include "../kernels/kernels.h"
#include "runtime.h"

namespace uhfs {


// ------------------------------------------------------------------- stats
namespace {
std::atomic<int64_t> g_launches{0}, g_copies{0}, g_syncs{0};
cudaStream_t g_stream = nullptr;
std::mutex g_stream_mu;
}  // namespace

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
void note_copy() { g_copies.fetch_add(1, std::memory_order_relaxed); }
void note_sync() { g_syncs.fetch_add(1, std::memory_order_relaxed); }
int64_t launch_count() { return g_launches.load(); }
void reset_launch_count() { g_launches.store(0); }

cudaStream_t runtime_stream() {
  std::lock_guard<std::mutex> lk(g_stream_mu);
  if (g_stream == nullptr) UHFS_CUDA_CHECK(cudaStreamCreateWithFlags(&g_stream, cudaStreamNonBlocking));
  return g_stream;
}

void runtime_synchronize() {
  UHFS_CUDA_CHECK(cudaStreamSynchronize(runtime_stream()));
  note_sync();
}

StreamStats stream_stats() {
  StreamStats s;
  s.non_blocking_streams = g_stream != nullptr ? 1 : 0;
  s.launches = g_launches.load();
  s.copies = g_copies.load();
  s.synchronizations = g_syncs.load();
  return s;
}

namespace {
// One status word per GPU, in this library's own static device memory: the
// word exists as soon as the module is loaded on a device (zero-initialised)
// and looking it up allocates nothing, so every entry point -- including the
// allocation-free ones -- can hand it to a kernel.
__device__ DeviceStatus g_device_status;
constexpr int kMaxStatusDevices = 64;
std::mutex g_status_mu;
DeviceStatus* g_status[kMaxStatusDevices] = {nullptr};
}  // namespace

DeviceStatus* device_status_ptr() {
  int dev = 0;
  UHFS_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxStatusDevices) throw std::runtime_error("device ordinal out of range for status word");
  std::lock_guard<std::mutex> lk(g_status_mu);
  if (g_status[dev] == nullptr) {
    void* p = nullptr;
    UHFS_CUDA_CHECK(cudaGetSymbolAddress(&p, g_device_status));
    g_status[dev] = static_cast<DeviceStatus*>(p);
  }
  return g_status[dev];
}

DeviceStatusHost read_device_status(bool clear) {
  DeviceStatus s;
  DeviceStatus* p = device_status_ptr();
  UHFS_CUDA_CHECK(cudaMemcpy(&s, p, sizeof(s), cudaMemcpyDeviceToHost));
  if (clear) UHFS_CUDA_CHECK(cudaMemset(p, 0, sizeof(DeviceStatus)));
  return DeviceStatusHost{s.code, s.where, s.block, s.count};
}

// --------------------------------------------------------------- allocator
namespace {
std::mutex g_alloc_mu;
std::unordered_map<size_t, std::vector<void*>> g_free;  // size class -> blocks
std::unordered_map<void*, size_t> g_live;
AllocatorStats g_astats;

size_t size_class(size_t bytes) {
  if (bytes == 0) bytes = 1;
  if (bytes <= (1u << 20)) return (bytes + 511) & ~size_t(511);
  const size_t two_mb = size_t(2) << 20;
  return (bytes + two_mb - 1) & ~(two_mb - 1);
}
}  // namespace

void* cached_malloc(size_t bytes) {
  const size_t cls = size_class(bytes);
  std::lock_guard<std::mutex> lk(g_alloc_mu);
  auto it = g_free.find(cls);
  void* p = nullptr;
  if (it != g_free.end() && !it->second.empty()) {
    p = it->second.back();
    it->second.pop_back();
    g_astats.cached_bytes -= (int64_t)cls;
    g_astats.reuses += 1;
  } else {
    UHFS_CUDA_CHECK(cudaMalloc(&p, cls));
    g_astats.allocated_bytes += (int64_t)cls;
    g_astats.allocations += 1;
  }
  g_live[p] = cls;
  g_astats.active_bytes += (int64_t)cls;
  return p;
}

void cached_free(void* p) {
  if (p == nullptr) return;
  std::lock_guard<std::mutex> lk(g_alloc_mu);
  auto it = g_live.find(p);
  if (it == g_live.end()) return;
  const size_t cls = it->second;
  g_live.erase(it);
  g_free[cls].push_back(p);
  g_astats.active_bytes -= (int64_t)cls;
  g_astats.cached_bytes += (int64_t)cls;
}

void empty_cache() {
  std::lock_guard<std::mutex> lk(g_alloc_mu);
  // Blocks may still be read by queued kernels on the runtime stream.
  if (g_stream != nullptr) cudaStreamSynchronize(g_stream);
  for (auto& kv : g_free) {
    for (void* p : kv.second) {
      cudaFree(p);
      g_astats.allocated_bytes -= (int64_t)kv.first;
    }
  }
  g_free.clear();
  g_astats.cached_bytes = 0;
}

AllocatorStats allocator_stats() {
  std::lock_guard<std::mutex> lk(g_alloc_mu);
  return g_astats;
}

// -------------------------------------------------------------- TensorCore
int64_t shape_numel(const std::vector<int64_t>& shape) {
  int64_t n = 1;
  for (int64_t d : shape) {
    if (d < 0) throw std::invalid_argument("shape dimensions must be non-negative");
    n *= d;
  }
  return n;
}

std::vector<int64_t> contiguous_strides(const std::vector<int64_t>& shape) {
  std::vector<int64_t> s(shape.size(), 1);
  int64_t stride = 1;
  for (int i = (int)shape.size() - 1; i >= 0; --i) {
    s[i] = stride;
    stride *= shape[i];
  }
  return s;
}

TensorCore::TensorCore(std::vector<double> storage, std::vector<int64_t> shape)
    : storage_(std::move(storage)), shape_(std::move(shape)) {
  if ((int64_t)storage_.size() != shape_numel(shape_))
    throw std::invalid_argument("storage size does not match shape");
}

std::vector<int64_t> TensorCore::strides() const { return contiguous_strides(shape_); }
int64_t TensorCore::numel() const { return (int64_t)storage_.size(); }

TensorCore TensorCore::add(const TensorCore& o) const {
  if (o.shape_ != shape_) throw std::invalid_argument("add requires equal shapes");
  std::vector<double> out(storage_.size());
  for (size_t i = 0; i < out.size(); ++i) out[i] = storage_[i] + o.storage_[i];
  return TensorCore(std::move(out), shape_);
}

TensorCore TensorCore::mul(const TensorCore& o) const {
  if (o.shape_ != shape_) throw std::invalid_argument("mul requires equal shapes");
  std::vector<double> out(storage_.size());
  for (size_t i = 0; i < out.size(); ++i) out[i] = storage_[i] * o.storage_[i];
  return TensorCore(std::move(out), shape_);
}

TensorCore TensorCore::matmul(const TensorCore& o) const {
  if (shape_.size() != 2 || o.shape_.size() != 2 || shape_[1] != o.shape_[0])
    throw std::invalid_argument("matmul requires [m,k] x [k,n]");
  const int64_t m = shape_[0], k = shape_[1], n = o.shape_[1];
  std::vector<double> out(m * n, 0.0);
  for (int64_t i = 0; i < m; ++i)
    for (int64_t p = 0; p < k; ++p) {
      const double a = storage_[i * k + p];
      for (int64_t j = 0; j < n; ++j) out[i * n + j] += a * o.storage_[p * n + j];
    }
  return TensorCore(std::move(out), {m, n});
}

TensorCore TensorCore::sum() const {
  double s = 0.0;
  for (double v : storage_) s += v;
  return TensorCore({s}, {});
}

std::string TensorCore::repr() const {
  std::ostringstream os;
  os << "TensorCore(shape=[";
  for (size_t i = 0; i < shape_.size(); ++i) os << (i ? ", " : "") << shape_[i];
  os << "], numel=" << storage_.size() << ")";
  return os.str();
}

// -------------------------------------------------------------- CudaTensor
namespace {
size_t dtype_size(int dt) { return dt == DT_F32 ? 4 : 2; }
}  // namespace

CudaTensor::CudaTensor(int dtype, std::vector<int64_t> shape) : dtype_(dtype), shape_(std::move(shape)) {
  ptr_ = cached_malloc(bytes() == 0 ? 16 : bytes());
}

CudaTensor::CudaTensor(int dtype, const std::vector<float>& host, std::vector<int64_t> shape)
    : dtype_(dtype), shape_(std::move(shape)) {
  if ((int64_t)host.size() != shape_numel(shape_)) throw std::invalid_argument("storage size does not match shape");
  ptr_ = cached_malloc(bytes() == 0 ? 16 : bytes());
  cudaStream_t s = runtime_stream();
  if (host.empty()) return;
  if (dtype_ == DT_F32) {
    UHFS_CUDA_CHECK(cudaMemcpyAsync(ptr_, host.data(), bytes(), cudaMemcpyHostToDevice, s));
    note_copy();
  } else {
    // stage fp32 on the device and convert there (reference kernels.cu:544-600)
    float* tmp = static_cast<float*>(cached_malloc(host.size() * 4));
    UHFS_CUDA_CHECK(cudaMemcpyAsync(tmp, host.data(), host.size() * 4, cudaMemcpyHostToDevice, s));
    note_copy();
    cast(DT_F32, dtype_, tmp, ptr_, (long long)host.size(), s);
    UHFS_CUDA_CHECK(cudaStreamSynchronize(s));  // host buffer and tmp lifetime
    note_sync();
    cached_free(tmp);
  }
}

CudaTensor::~CudaTensor() {
  if (ptr_ != nullptr) {
    // queued kernels may still read this block: order the free on the stream
    cudaStreamSynchronize(runtime_stream());
    cached_free(ptr_);
  }
}

int64_t CudaTensor::numel() const { return shape_numel(shape_); }
size_t CudaTensor::bytes() const { return (size_t)numel() * dtype_size(dtype_); }

std::vector<float> CudaTensor::to_host() const {
  const int64_t n = numel();
  std::vector<float> out(n);
  if (n == 0) return out;
  cudaStream_t s = runtime_stream();
  if (dtype_ == DT_F32) {
    UHFS_CUDA_CHECK(cudaMemcpyAsync(out.data(), ptr_, bytes(), cudaMemcpyDeviceToHost, s));
    note_copy();
    UHFS_CUDA_CHECK(cudaStreamSynchronize(s));
    note_sync();
  } else {
    float* tmp = static_cast<float*>(cached_malloc(n * 4));
    cast(dtype_, DT_F32, ptr_, tmp, n, s);
    UHFS_CUDA_CHECK(cudaMemcpyAsync(out.data(), tmp, n * 4, cudaMemcpyDeviceToHost, s));
    note_copy();
    UHFS_CUDA_CHECK(cudaStreamSynchronize(s));
    note_sync();
    cached_free(tmp);
  }
  return out;
}

CudaTensor* CudaTensor::add(const CudaTensor& o) const {
  if (o.shape_ != shape_ || o.dtype_ != dtype_) throw std::invalid_argument("add requires equal shapes and dtypes");
  auto* out = new CudaTensor(dtype_, shape_);
  ew_binary(OP_ADD, dtype_, ptr_, o.ptr_, out->ptr_, numel(), runtime_stream());
  return out;
}

CudaTensor* CudaTensor::mul(const CudaTensor& o) const {
  if (o.shape_ != shape_ || o.dtype_ != dtype_) throw std::invalid_argument("mul requires equal shapes and dtypes");
  auto* out = new CudaTensor(dtype_, shape_);
  ew_binary(OP_MUL, dtype_, ptr_, o.ptr_, out->ptr_, numel(), runtime_stream());
  return out;
}

CudaTensor* CudaTensor::matmul(const CudaTensor& o) const {
  if (dtype_ != DT_F32 || o.dtype_ != DT_F32) throw std::invalid_argument("CudaTensorF32 matmul requires fp32");
  if (shape_.size() != 2 || o.shape_.size() != 2 || shape_[1] != o.shape_[0])
    throw std::invalid_argument("matmul requires [m,k] x [k,n]");
  const int m = (int)shape_[0], k = (int)shape_[1], n = (int)o.shape_[1];
  auto* out = new CudaTensor(DT_F32, std::vector<int64_t>{m, n});
  gemm_f32_simt((const float*)ptr_, (const float*)o.ptr_, (float*)out->ptr_, m, n, k, false, runtime_stream());
  return out;
}

CudaTensor* CudaTensor::sum() const {
  if (dtype_ != DT_F32) throw std::invalid_argument("CudaTensorF32 sum requires fp32");
  auto* out = new CudaTensor(DT_F32, std::vector<int64_t>{1});
  float* partials = static_cast<float*>(cached_malloc(reduce_sum_partials() * 4 + 16));
  unsigned int* counter = reinterpret_cast<unsigned int*>(partials + reduce_sum_partials());
  UHFS_CUDA_CHECK(cudaMemsetAsync(counter, 0, 4, runtime_stream()));
  reduce_sum(DT_F32, ptr_, numel(), (float*)out->ptr_, partials, counter, runtime_stream());
  UHFS_CUDA_CHECK(cudaStreamSynchronize(runtime_stream()));
  note_sync();
  cached_free(partials);
  return out;
}

// ------------------------------------------------------ one-shot helpers
namespace {
struct DevBuf {
  void* p = nullptr;
  explicit DevBuf(size_t bytes) { p = cached_malloc(bytes == 0 ? 16 : bytes); }
  ~DevBuf() { cached_free(p); }
  float* f() { return static_cast<float*>(p); }
};
void h2d(void* dst, const std::vector<float>& src) {
  if (src.empty()) return;
  UHFS_CUDA_CHECK(cudaMemcpyAsync(dst, src.data(), src.size() * 4, cudaMemcpyHostToDevice, runtime_stream()));
  note_copy();
}
std::vector<float> d2h(const void* src, size_t n) {
  std::vector<float> out(n);
  if (n == 0) return out;
  UHFS_CUDA_CHECK(cudaMemcpyAsync(out.data(), src, n * 4, cudaMemcpyDeviceToHost, runtime_stream()));
  note_copy();
  UHFS_CUDA_CHECK(cudaStreamSynchronize(runtime_stream()));
  note_sync();
  return out;
}
}  // namespace

std::vector<float> cuda_add_f32_host(const std::vector<float>& a, const std::vector<float>& b) {
  if (a.size() != b.size()) throw std::invalid_argument("cuda_add_f32 requires equal sizes");
  DevBuf da(a.size() * 4), db(b.size() * 4), dc(a.size() * 4);
  h2d(da.p, a);
  h2d(db.p, b);
  ew_binary(OP_ADD, DT_F32, da.p, db.p, dc.p, (long long)a.size(), runtime_stream());
  return d2h(dc.p, a.size());
}

std::map<std::string, std::vector<float>> cuda_fused_adamw_f32_host(std::vector<float> p, std::vector<float> g,
                                                                    std::vector<float> m, std::vector<float> v,
                                                                    float lr, float b1, float b2, float eps,
                                                                    float wd, int step) {
  const size_t n = p.size();
  if (g.size() != n || m.size() != n || v.size() != n) throw std::invalid_argument("adamw buffers must match");
  DevBuf dp(n * 4), dg(n * 4), dm(n * 4), dv(n * 4);
  h2d(dp.p, p);
  h2d(dg.p, g);
  h2d(dm.p, m);
  h2d(dv.p, v);
  AdamWArgs a{};
  a.lr = lr;
  a.beta1 = b1;
  a.beta2 = b2;
  a.eps = eps;
  a.weight_decay = wd;
  a.decoupled = 0;
  a.grad_scale = 1.0f;
  a.step = step;
  a.step_ptr = nullptr;
  a.lr_ptr = nullptr;
  adamw_step(a, dp.f(), dg.f(), dm.f(), dv.f(), nullptr, (long long)n, runtime_stream());
  std::map<std::string, std::vector<float>> out;
  out["param"] = d2h(dp.p, n);
  out["m"] = d2h(dm.p, n);
  out["v"] = d2h(dv.p, n);
  return out;
}

std::vector<float> cuda_attention_f32_host(const std::vector<float>& q, const std::vector<float>& k,
                                           const std::vector<float>& v, int tokens, int features, float scale,
                                           bool causal) {
  const size_t n = (size_t)tokens * features;
  if (q.size() != n || k.size() != n || v.size() != n) throw std::invalid_argument("attention inputs must be [T,F]");
  DevBuf dq(n * 4), dk(n * 4), dv(n * 4), dout(n * 4);
  h2d(dq.p, q);
  h2d(dk.p, k);
  h2d(dv.p, v);
  attention_naive_f32(dq.f(), dk.f(), dv.f(), dout.f(), tokens, features, scale, causal, runtime_stream());
  return d2h(dout.p, n);
}

static int out_dim(int in, int pad, int k, int stride) { return (in + 2 * pad - k) / stride + 1; }

std::vector<float> conv2d_forward_f32_host(const std::vector<float>& x, const std::vector<float>& w,
                                           const std::vector<float>& b, int N, int C, int H, int W, int K, int R,
                                           int S, int sh, int sw, int ph, int pw) {
  const int P = out_dim(H, ph, R, sh), Q = out_dim(W, pw, S, sw);
  if (P <= 0 || Q <= 0) throw std::invalid_argument("conv2d produces empty output");
  DevBuf dx(x.size() * 4), dw(w.size() * 4), db(b.size() * 4 + 4), dy((size_t)N * K * P * Q * 4);
  h2d(dx.p, x);
  h2d(dw.p, w);
  h2d(db.p, b);
  conv2d_fwd_f32(dx.f(), dw.f(), b.empty() ? nullptr : db.f(), dy.f(), N, C, H, W, K, R, S, sh, sw, ph, pw, P, Q,
                 runtime_stream());
  return d2h(dy.p, (size_t)N * K * P * Q);
}

std::vector<float> conv2d_backward_input_f32_host(const std::vector<float>& dyv, const std::vector<float>& w, int N,
                                                  int C, int H, int W, int K, int R, int S, int sh, int sw, int ph,
                                                  int pw) {
  const int P = out_dim(H, ph, R, sh), Q = out_dim(W, pw, S, sw);
  DevBuf ddy(dyv.size() * 4), dw(w.size() * 4), ddx((size_t)N * C * H * W * 4);
  h2d(ddy.p, dyv);
  h2d(dw.p, w);
  conv2d_dgrad_f32(ddy.f(), dw.f(), ddx.f(), N, C, H, W, K, R, S, sh, sw, ph, pw, P, Q, runtime_stream());
  return d2h(ddx.p, (size_t)N * C * H * W);
}

std::vector<float> conv2d_backward_weight_f32_host(const std::vector<float>& dyv, const std::vector<float>& x, int N,
                                                   int C, int H, int W, int K, int R, int S, int sh, int sw, int ph,
                                                   int pw) {
  const int P = out_dim(H, ph, R, sh), Q = out_dim(W, pw, S, sw);
  DevBuf ddy(dyv.size() * 4), dx(x.size() * 4), ddw((size_t)K * C * R * S * 4);
  h2d(ddy.p, dyv);
  h2d(dx.p, x);
  conv2d_wgrad_f32(ddy.f(), dx.f(), ddw.f(), nullptr, N, C, H, W, K, R, S, sh, sw, ph, pw, P, Q, runtime_stream());
  return d2h(ddw.p, (size_t)K * C * R * S);
}

#ifndef UHFS_NO_NCCL
// ------------------------------------------------------------------- NCCL
namespace {
void nccl_check(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) throw std::runtime_error(std::string(what) + ": " + ncclGetErrorString(r));
}
ncclDataType_t nccl_dtype(int dt) {
  switch (dt) {
    case DT_F32: return ncclFloat32;
    case DT_F16: return ncclFloat16;
    case DT_BF16: return ncclBfloat16;
    default: throw std::invalid_argument("unsupported collective dtype");
  }
}
size_t dt_bytes(int dt) { return dt == DT_F32 ? 4 : 2; }
}  // namespace

std::string nccl_create_unique_id_hex() {
  ncclUniqueId id;
  nccl_check(ncclGetUniqueId(&id), "ncclGetUniqueId");
  static const char* hex = "0123456789abcdef";
  std::string s;
  s.reserve(sizeof(id.internal) * 2);
  for (size_t i = 0; i < sizeof(id.internal); ++i) {
    const unsigned char c = (unsigned char)id.internal[i];
    s.push_back(hex[c >> 4]);
    s.push_back(hex[c & 15]);
  }
  return s;
}

NcclProcessGroup::NcclProcessGroup(int rank, int world_size, const std::string& unique_id_hex, int device)
    : rank_(rank), world_(world_size), device_(device) {
  if (world_size <= 0 || rank < 0 || rank >= world_size) throw std::invalid_argument("invalid rank/world_size");
  if (device >= 0) UHFS_CUDA_CHECK(cudaSetDevice(device));
  ncclUniqueId id;
  if (unique_id_hex.empty()) {
    if (world_size != 1) throw std::invalid_argument("a unique id is required when world_size > 1");
    nccl_check(ncclGetUniqueId(&id), "ncclGetUniqueId");
  } else {
    if (unique_id_hex.size() != sizeof(id.internal) * 2) throw std::invalid_argument("malformed NCCL unique id");
    for (size_t i = 0; i < sizeof(id.internal); ++i) {
      unsigned int byte = 0;
      std::sscanf(unique_id_hex.c_str() + 2 * i, "%2x", &byte);
      id.internal[i] = (char)byte;
    }
  }
  ncclComm_t comm;
  nccl_check(ncclCommInitRank(&comm, world_size, id, rank), "ncclCommInitRank");
  comm_ = comm;
  UHFS_CUDA_CHECK(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
}

NcclProcessGroup::~NcclProcessGroup() {
  if (stream_ != nullptr) cudaStreamSynchronize(stream_);
  if (comm_ != nullptr) ncclCommDestroy(static_cast<ncclComm_t>(comm_));
  if (stream_ != nullptr) cudaStreamDestroy(stream_);
}

std::vector<float> NcclProcessGroup::staged(const std::vector<float>& in, size_t out_count, int kind, int src) {
  ncclComm_t comm = static_cast<ncclComm_t>(comm_);
  DevBuf din(in.size() * 4), dout(out_count * 4);
  if (!in.empty()) {
    UHFS_CUDA_CHECK(cudaMemcpyAsync(din.p, in.data(), in.size() * 4, cudaMemcpyHostToDevice, stream_));
    note_copy();
  }
  switch (kind) {
    case 0: nccl_check(ncclAllReduce(din.p, dout.p, in.size(), ncclFloat32, ncclSum, comm, stream_), "all_reduce"); break;
    case 1: nccl_check(ncclBroadcast(din.p, dout.p, in.size(), ncclFloat32, src, comm, stream_), "broadcast"); break;
    case 2:
      nccl_check(ncclReduceScatter(din.p, dout.p, out_count, ncclFloat32, ncclSum, comm, stream_), "reduce_scatter");
      break;
    default: nccl_check(ncclAllGather(din.p, dout.p, in.size(), ncclFloat32, comm, stream_), "all_gather"); break;
  }
  std::vector<float> out(out_count);
  if (out_count) {
    UHFS_CUDA_CHECK(cudaMemcpyAsync(out.data(), dout.p, out_count * 4, cudaMemcpyDeviceToHost, stream_));
    note_copy();
  }
  UHFS_CUDA_CHECK(cudaStreamSynchronize(stream_));
  note_sync();
  return out;
}

void NcclProcessGroup::barrier() {
  std::vector<float> one{1.0f};
  staged(one, 1, 0, 0);
}

std::vector<float> NcclProcessGroup::all_reduce_sum(const std::vector<float>& v) { return staged(v, v.size(), 0, 0); }
std::vector<float> NcclProcessGroup::broadcast(const std::vector<float>& v, int src) {
  return staged(v, v.size(), 1, src);
}
std::vector<float> NcclProcessGroup::reduce_scatter(const std::vector<float>& v) {
  if (v.size() % world_ != 0) throw std::invalid_argument("reduce_scatter input must divide by world_size");
  return staged(v, v.size() / world_, 2, 0);
}
std::vector<float> NcclProcessGroup::all_gather(const std::vector<float>& v) {
  return staged(v, v.size() * world_, 3, 0);
}

void NcclProcessGroup::all_reduce_ptr(uintptr_t buf, int64_t count, int dtype, uintptr_t stream) {
  nccl_check(ncclAllReduce((void*)buf, (void*)buf, count, nccl_dtype(dtype), ncclSum, static_cast<ncclComm_t>(comm_),
                           (cudaStream_t)stream),
             "all_reduce");
}
void NcclProcessGroup::broadcast_ptr(uintptr_t buf, int64_t count, int dtype, int src, uintptr_t stream) {
  nccl_check(ncclBroadcast((void*)buf, (void*)buf, count, nccl_dtype(dtype), src, static_cast<ncclComm_t>(comm_),
                           (cudaStream_t)stream),
             "broadcast");
}
void NcclProcessGroup::reduce_scatter_ptr(uintptr_t send, uintptr_t recv, int64_t recv_count, int dtype,
                                          uintptr_t stream) {
  nccl_check(ncclReduceScatter((void*)send, (void*)recv, recv_count, nccl_dtype(dtype), ncclSum,
                               static_cast<ncclComm_t>(comm_), (cudaStream_t)stream),
             "reduce_scatter");
}
void NcclProcessGroup::all_gather_ptr(uintptr_t send, uintptr_t recv, int64_t send_count, int dtype,
                                      uintptr_t stream) {
  nccl_check(ncclAllGather((void*)send, (void*)recv, send_count, nccl_dtype(dtype), static_cast<ncclComm_t>(comm_),
                           (cudaStream_t)stream),
             "all_gather");
  (void)dt_bytes;
}

#else  // UHFS_NO_NCCL: built with UNDERHFS_WITH_NCCL=OFF
namespace {
[[noreturn]] void no_nccl() {
  throw std::runtime_error("NCCL process groups need the native core built with UNDERHFS_WITH_NCCL=ON");
}
}  // namespace
std::string nccl_create_unique_id_hex() { no_nccl(); }
NcclProcessGroup::NcclProcessGroup(int rank, int world_size, const std::string&, int device)
    : rank_(rank), world_(world_size), device_(device) {
  no_nccl();
}
NcclProcessGroup::~NcclProcessGroup() {}
std::vector<float> NcclProcessGroup::staged(const std::vector<float>&, size_t, int, int) { no_nccl(); }
void NcclProcessGroup::barrier() { no_nccl(); }
std::vector<float> NcclProcessGroup::all_reduce_sum(const std::vector<float>&) { no_nccl(); }
std::vector<float> NcclProcessGroup::broadcast(const std::vector<float>&, int) { no_nccl(); }
std::vector<float> NcclProcessGroup::reduce_scatter(const std::vector<float>&) { no_nccl(); }
std::vector<float> NcclProcessGroup::all_gather(const std::vector<float>&) { no_nccl(); }
void NcclProcessGroup::all_reduce_ptr(uintptr_t, int64_t, int, uintptr_t) { no_nccl(); }
void NcclProcessGroup::broadcast_ptr(uintptr_t, int64_t, int, int, uintptr_t) { no_nccl(); }
void NcclProcessGroup::reduce_scatter_ptr(uintptr_t, uintptr_t, int64_t, int, uintptr_t) { no_nccl(); }
void NcclProcessGroup::all_gather_ptr(uintptr_t, uintptr_t, int64_t, int, uintptr_t) { no_nccl(); }
#endif  // UHFS_NO_NCCL

}  // namespace uhfs
