// Native runtime of underhfs_b200 (host side, C++17).
//
// Covers the reference's C++/CUDA runtime contracts:
//   * TensorCore            (cpp/tensor_core.{hpp,cpp})   contiguous fp64 CPU tensor
//   * CudaRuntime stats     (cuda/kernels.cu:238-289)     one non-blocking stream + counters
//   * CudaCachingAllocator  (cuda/kernels.cu:291-357)     cached device blocks + stats
//   * CudaTensor{F32,F16,BF16} (cuda/kernels.cu:361-804) device storage + add/mul/matmul/sum
//   * NcclProcessGroup      (cpp/nccl_runtime.{hpp,cpp}) NCCL communicator
// Differences that matter on B200: ops are stream-ordered and only
// synchronize when a result is copied to the host; the allocator rounds sizes
// into classes (2 MiB granularity above 1 MiB) so a training loop's buffers
// are reused; the process group binds its GPU with cudaSetDevice and runs on
// its own stream instead of the legacy default stream.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

namespace uhfs {

// ----------------------------------------------------------------- stats
struct StreamStats {
  int64_t non_blocking_streams = 0;
  int64_t launches = 0;
  int64_t copies = 0;
  int64_t synchronizations = 0;
};
StreamStats stream_stats();
void reset_launch_count();
int64_t launch_count();
void note_copy();
void note_sync();
cudaStream_t runtime_stream();  // the process-wide non-blocking stream
void runtime_synchronize();

// ------------------------------------------------------------- allocator
struct AllocatorStats {
  int64_t active_bytes = 0;
  int64_t cached_bytes = 0;
  int64_t allocated_bytes = 0;
  int64_t allocations = 0;
  int64_t reuses = 0;
};
void* cached_malloc(size_t bytes);
void cached_free(void* p);
void empty_cache();
AllocatorStats allocator_stats();

// -------------------------------------------------------- device status
struct DeviceStatusHost {
  int code, where, block, count;
};
DeviceStatusHost read_device_status(bool clear);

// ------------------------------------------------------------ TensorCore
class TensorCore {
 public:
  TensorCore(std::vector<double> storage, std::vector<int64_t> shape);
  const std::vector<double>& storage() const { return storage_; }
  const std::vector<int64_t>& shape() const { return shape_; }
  std::vector<int64_t> strides() const;
  int64_t numel() const;
  TensorCore add(const TensorCore& o) const;
  TensorCore mul(const TensorCore& o) const;
  TensorCore matmul(const TensorCore& o) const;
  TensorCore sum() const;
  std::string repr() const;

 private:
  std::vector<double> storage_;
  std::vector<int64_t> shape_;
};
int64_t shape_numel(const std::vector<int64_t>& shape);
std::vector<int64_t> contiguous_strides(const std::vector<int64_t>& shape);

// ------------------------------------------------------------ CudaTensor
class CudaTensor {
 public:
  CudaTensor(int dtype, const std::vector<float>& host, std::vector<int64_t> shape);
  CudaTensor(int dtype, std::vector<int64_t> shape);  // uninitialised
  ~CudaTensor();
  CudaTensor(const CudaTensor&) = delete;
  CudaTensor& operator=(const CudaTensor&) = delete;

  std::vector<float> to_host() const;
  CudaTensor* add(const CudaTensor& o) const;
  CudaTensor* mul(const CudaTensor& o) const;
  CudaTensor* matmul(const CudaTensor& o) const;  // fp32 only
  CudaTensor* sum() const;                        // fp32 only
  const std::vector<int64_t>& shape() const { return shape_; }
  int64_t numel() const;
  int dtype() const { return dtype_; }
  uintptr_t data_ptr() const { return reinterpret_cast<uintptr_t>(ptr_); }

 private:
  size_t bytes() const;
  int dtype_;
  std::vector<int64_t> shape_;
  void* ptr_ = nullptr;
};

// one-shot helpers with the reference's host-list signatures
std::vector<float> cuda_add_f32_host(const std::vector<float>& a, const std::vector<float>& b);
std::map<std::string, std::vector<float>> cuda_fused_adamw_f32_host(std::vector<float> p, std::vector<float> g,
                                                                    std::vector<float> m, std::vector<float> v,
                                                                    float lr, float b1, float b2, float eps,
                                                                    float wd, int step);
std::vector<float> cuda_attention_f32_host(const std::vector<float>& q, const std::vector<float>& k,
                                           const std::vector<float>& v, int tokens, int features, float scale,
                                           bool causal);
std::vector<float> conv2d_forward_f32_host(const std::vector<float>& x, const std::vector<float>& w,
                                           const std::vector<float>& b, int N, int C, int H, int W, int K, int R,
                                           int S, int sh, int sw, int ph, int pw);
std::vector<float> conv2d_backward_input_f32_host(const std::vector<float>& dy, const std::vector<float>& w, int N,
                                                  int C, int H, int W, int K, int R, int S, int sh, int sw, int ph,
                                                  int pw);
std::vector<float> conv2d_backward_weight_f32_host(const std::vector<float>& dy, const std::vector<float>& x, int N,
                                                   int C, int H, int W, int K, int R, int S, int sh, int sw, int ph,
                                                   int pw);

// ---------------------------------------------------------- NCCL group
std::string nccl_create_unique_id_hex();

class NcclProcessGroup {
 public:
  NcclProcessGroup(int rank, int world_size, const std::string& unique_id_hex, int device);
  ~NcclProcessGroup();
  int rank() const { return rank_; }
  int world_size() const { return world_; }
  void barrier();
  std::vector<float> all_reduce_sum(const std::vector<float>& v);
  std::vector<float> broadcast(const std::vector<float>& v, int src);
  std::vector<float> reduce_scatter(const std::vector<float>& v);
  std::vector<float> all_gather(const std::vector<float>& v);
  // device-pointer collectives on the caller's stream (dtype: 0 f32, 2 bf16)
  void all_reduce_ptr(uintptr_t buf, int64_t count, int dtype, uintptr_t stream);
  void broadcast_ptr(uintptr_t buf, int64_t count, int dtype, int src, uintptr_t stream);
  void reduce_scatter_ptr(uintptr_t send, uintptr_t recv, int64_t recv_count, int dtype, uintptr_t stream);
  void all_gather_ptr(uintptr_t send, uintptr_t recv, int64_t send_count, int dtype, uintptr_t stream);

 private:
  std::vector<float> staged(const std::vector<float>& in, size_t out_count, int kind, int src);
  int rank_, world_, device_;
  void* comm_ = nullptr;
  cudaStream_t stream_ = nullptr;
};

}  // namespace uhfs
