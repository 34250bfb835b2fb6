// Host interface of the symmetric heap and fused collectives (comm.cu).
#pragma once

#include <array>
#include <vector>

#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

namespace uhfs {

// One device allocation per rank: [64 KiB signal pad | data region], exported
// with cudaIpcGetMemHandle and mapped into every peer with
// cudaIpcOpenMemHandle, so kernels can address every rank's region directly.
class SymmetricHeap {
 public:
  SymmetricHeap(int rank, int world, size_t data_bytes);
  ~SymmetricHeap();
  SymmetricHeap(const SymmetricHeap&) = delete;
  SymmetricHeap& operator=(const SymmetricHeap&) = delete;

  std::string ipc_handle() const;
  void open(const std::vector<std::string>& handles);
  void close();
  int rank() const { return rank_; }
  int world() const { return world_; }
  int device() const { return device_; }
  size_t data_bytes() const { return data_bytes_; }
  uintptr_t data_ptr(int r) const;
  uintptr_t signal_ptr(int r) const;

 private:
  int rank_, world_, device_ = 0;
  size_t data_bytes_ = 0;
  char* base_ = nullptr;
  std::vector<char*> ptrs_;
  std::vector<bool> opened_;
};

void comm_allreduce_f32(const SymmetricHeap& h, long long off_bytes, long long n, float scale, int blocks,
                        cudaStream_t s);
// In-place fp32 all-reduce through an NVLink multicast object: `mc_base` is
// the multicast address of the data buffer (every rank's copy bound to it);
// `h` provides the signal pads of the barriers.
void comm_allreduce_f32_nvls(const SymmetricHeap& h, uintptr_t mc_base, long long off_bytes, long long n, float scale,
                             int blocks, cudaStream_t s);
void comm_rs_adamw_ag(const SymmetricHeap& grads, long long g_off_bytes, const SymmetricHeap& params,
                      long long p_off_bytes, long long shard_lo, long long shard_n, uintptr_t master, uintptr_t m,
                      uintptr_t v, float lr, float beta1, float beta2, float eps, float weight_decay,
                      float grad_scale, bool decoupled, uintptr_t step_ptr, int blocks, cudaStream_t s);
void comm_allgather(const SymmetricHeap& h, long long off_bytes, long long shard_bytes, int blocks, cudaStream_t s);
void comm_allreduce_bf16(const SymmetricHeap& h, long long off_bytes, long long n, float scale, int blocks,
                         cudaStream_t s);
// In-place fp32 all-reduce whose transfers are bf16 (cast and scale fused);
// `wire_off_bytes` is a bf16 staging span of n elements in every rank's heap.
// Every rank ends with the same bf16-rounded sum (widened to fp32).
void comm_allreduce_f32_wire_bf16(const SymmetricHeap& h, long long off_bytes, long long wire_off_bytes, long long n,
                                  float scale, int blocks, cudaStream_t s);
void comm_reduce_scatter(const SymmetricHeap& h, long long in_off_bytes, long long out_off_bytes, long long n,
                         bool bf16, float scale, int blocks, cudaStream_t s);
void comm_gather_segments(const SymmetricHeap& h, long long dst_off_bytes, uintptr_t shard,
                          const std::vector<std::array<long long, 3>>& segs, int blocks, cudaStream_t s);
void comm_rs_adamw_segments(const SymmetricHeap& grads, long long g_off_bytes,
                            const std::vector<std::array<long long, 3>>& segs, uintptr_t master, uintptr_t m,
                            uintptr_t v, uintptr_t shard16, float lr, float beta1, float beta2, float eps,
                            float weight_decay, float grad_scale, bool decoupled, uintptr_t step_ptr, int blocks,
                            cudaStream_t s);
void comm_barrier(const SymmetricHeap& h, cudaStream_t s);
void comm_wait_probe(const SymmetricHeap& h, unsigned int want, unsigned long long bound_ns, cudaStream_t s);

}  // namespace uhfs
