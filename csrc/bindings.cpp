// pybind11 module `underhfs_b200._core`.
//
// Keeps the reference's `_core` surface (cpp/bindings.cpp:14-95): version and
// feature flags, TensorCore, CudaTensor{F32,F16,BF16}, the one-shot host
// helpers, allocator / stream stats, NcclProcessGroup.  Adds the launchers of
// the sm_100a kernels; these take raw device pointers (Python ints from
// torch.Tensor.data_ptr()) and a CUDA stream handle, so the Python layer owns
// memory and streams while every hot op runs a kernel from this library.
#include <array>

#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "kernels/gemm.h"
#include "kernels/kernels.h"
#include "runtime/comm.h"
#include "runtime/runtime.h"

namespace py = pybind11;
using namespace uhfs;

namespace {

template <typename T>
T* P(uintptr_t p) {
  return reinterpret_cast<T*>(p);
}
cudaStream_t S(uintptr_t s) { return reinterpret_cast<cudaStream_t>(s); }

template <int DT>
void bind_cuda_tensor(py::module_& m, const char* name) {
  py::class_<CudaTensor>(m, name)
      .def(py::init([](const std::vector<float>& host, const std::vector<int64_t>& shape) {
             return new CudaTensor(DT, host, shape);
           }),
           py::arg("storage"), py::arg("shape"))
      .def("to_host", &CudaTensor::to_host)
      .def("add", &CudaTensor::add, py::return_value_policy::take_ownership)
      .def("mul", &CudaTensor::mul, py::return_value_policy::take_ownership)
      .def("matmul", &CudaTensor::matmul, py::return_value_policy::take_ownership)
      .def("sum", &CudaTensor::sum, py::return_value_policy::take_ownership)
      .def("numel", &CudaTensor::numel)
      .def("data_ptr", &CudaTensor::data_ptr)
      .def_property_readonly("shape", &CudaTensor::shape)
      .def_property_readonly("dtype", &CudaTensor::dtype);
}

}  // namespace

PYBIND11_MODULE(_core, m) {
  m.doc() = "underhfs_b200 native core: sm_100a kernels and C++ runtime";
  m.attr("__version__") = "0.2.0";
  m.attr("cuda_enabled") = true;
#ifdef UHFS_NO_CONV
  m.attr("cudnn_enabled") = false;  // built with UNDERHFS_WITH_CUDNN=OFF: no conv2d kernels
#else
  m.attr("cudnn_enabled") = true;  // conv2d kernels present (own implicit-GEMM kernels, no cuDNN)
#endif
#ifdef UHFS_NO_NCCL
  m.attr("nccl_enabled") = false;  // built with UNDERHFS_WITH_NCCL=OFF
#else
  m.attr("nccl_enabled") = true;
#endif
  m.attr("arch") = "sm_100a";

  // --------------------------------------------------------- CPU contract
  py::class_<TensorCore>(m, "TensorCore")
      .def(py::init<std::vector<double>, std::vector<int64_t>>(), py::arg("storage"), py::arg("shape"))
      .def_property_readonly("storage", &TensorCore::storage)
      .def_property_readonly("shape", &TensorCore::shape)
      .def_property_readonly("strides", &TensorCore::strides)
      .def("numel", &TensorCore::numel)
      .def("add", &TensorCore::add)
      .def("mul", &TensorCore::mul)
      .def("matmul", &TensorCore::matmul)
      .def("sum", &TensorCore::sum)
      .def("__repr__", &TensorCore::repr);
  m.def("shape_numel", &shape_numel);
  m.def("contiguous_strides", &contiguous_strides);

  bind_cuda_tensor<DT_F32>(m, "CudaTensorF32");
  // F16 / BF16 share the C++ class; separate Python names keep the contract.
  m.attr("CudaTensorF16") = py::cpp_function([](const std::vector<float>& host, const std::vector<int64_t>& shape) {
    return new CudaTensor(DT_F16, host, shape);
  }, py::return_value_policy::take_ownership);
  m.attr("CudaTensorBF16") = py::cpp_function([](const std::vector<float>& host, const std::vector<int64_t>& shape) {
    return new CudaTensor(DT_BF16, host, shape);
  }, py::return_value_policy::take_ownership);

  m.def("cuda_add_f32", &cuda_add_f32_host);
  m.def("cuda_fused_adamw_f32", &cuda_fused_adamw_f32_host, py::arg("param"), py::arg("grad"), py::arg("m"),
        py::arg("v"), py::arg("lr"), py::arg("beta1"), py::arg("beta2"), py::arg("eps"), py::arg("weight_decay"),
        py::arg("step"));
  m.def("cuda_attention_f32", &cuda_attention_f32_host);
#ifndef UHFS_NO_CONV
  m.def("cudnn_conv2d_forward_f32", &conv2d_forward_f32_host);
  m.def("cudnn_conv2d_backward_input_f32", &conv2d_backward_input_f32_host);
  m.def("cudnn_conv2d_backward_weight_f32", &conv2d_backward_weight_f32_host);
#endif

  m.def("cuda_allocator_stats", []() {
    AllocatorStats s = allocator_stats();
    py::dict d;
    d["active_bytes"] = s.active_bytes;
    d["cached_bytes"] = s.cached_bytes;
    d["allocated_bytes"] = s.allocated_bytes;
    d["allocations"] = s.allocations;
    d["reuses"] = s.reuses;
    return d;
  });
  m.def("cuda_empty_cache", &empty_cache);
  m.def("cuda_stream_stats", []() {
    StreamStats s = stream_stats();
    py::dict d;
    d["non_blocking_streams"] = s.non_blocking_streams;
    d["launches"] = s.launches;
    d["copies"] = s.copies;
    d["synchronizations"] = s.synchronizations;
    return d;
  });
  m.def("cuda_synchronize", &runtime_synchronize);
  m.def("launch_count", &launch_count);
  m.def("reset_launch_count", &reset_launch_count);
  m.def("device_status", [](bool clear) {
    DeviceStatusHost s = read_device_status(clear);
    py::dict d;
    d["code"] = s.code;
    d["where"] = s.where;
    d["block"] = s.block;
    d["count"] = s.count;
    return d;
  }, py::arg("clear") = false);

  py::class_<NcclProcessGroup>(m, "NcclProcessGroup")
      .def(py::init<int, int, const std::string&, int>(), py::arg("rank"), py::arg("world_size"),
           py::arg("unique_id_hex") = std::string(), py::arg("device") = -1)
      .def_property_readonly("rank", &NcclProcessGroup::rank)
      .def_property_readonly("world_size", &NcclProcessGroup::world_size)
      .def("barrier", &NcclProcessGroup::barrier)
      .def("all_reduce_sum", &NcclProcessGroup::all_reduce_sum)
      .def("broadcast", &NcclProcessGroup::broadcast)
      .def("reduce_scatter", &NcclProcessGroup::reduce_scatter)
      .def("all_gather", &NcclProcessGroup::all_gather)
      .def("all_reduce_ptr", &NcclProcessGroup::all_reduce_ptr)
      .def("broadcast_ptr", &NcclProcessGroup::broadcast_ptr)
      .def("reduce_scatter_ptr", &NcclProcessGroup::reduce_scatter_ptr)
      .def("all_gather_ptr", &NcclProcessGroup::all_gather_ptr);
  m.def("nccl_create_unique_id_hex", &nccl_create_unique_id_hex);

  // ---------------------------------------------------- kernel launchers
  m.def(
      "gemm",
      [](int M, int N, int K, uintptr_t A, long long lda, bool a_mn, uintptr_t B, long long ldb, bool b_mn,
         uintptr_t C, long long ldc, int epi, uintptr_t bias, uintptr_t aux, long long ld_aux, uintptr_t aux_out,
         long long ld_aux_out, int splits, int block_n, int cta_pair, uintptr_t stream) {
        GemmProblem p;
        p.M = M;
        p.N = N;
        p.K = K;
        p.A = P<const __nv_bfloat16>(A);
        p.lda = lda;
        p.a_mn = a_mn;
        p.B = P<const __nv_bfloat16>(B);
        p.ldb = ldb;
        p.b_mn = b_mn;
        p.C = P<void>(C);
        p.ldc = ldc;
        p.epi = epi;
        p.bias = P<const __nv_bfloat16>(bias);
        p.aux = P<const __nv_bfloat16>(aux);
        p.ld_aux = ld_aux;
        p.aux_out = P<__nv_bfloat16>(aux_out);
        p.ld_aux_out = ld_aux_out;
        p.splits = splits;
        p.block_n = block_n;
        p.cta_pair = cta_pair;
        gemm_bf16_tcgen05(p, S(stream));
      },
      py::arg("M"), py::arg("N"), py::arg("K"), py::arg("A"), py::arg("lda"), py::arg("a_mn"), py::arg("B"),
      py::arg("ldb"), py::arg("b_mn"), py::arg("C"), py::arg("ldc"), py::arg("epi"), py::arg("bias") = 0,
      py::arg("aux") = 0, py::arg("ld_aux") = 0, py::arg("aux_out") = 0, py::arg("ld_aux_out") = 0,
      py::arg("splits") = 1, py::arg("block_n") = 0, py::arg("cta_pair") = -1, py::arg("stream") = 0);
  // GEMM whose B rows are gathered by the kernel itself (ZeRO-3): `segs` are
  // (src, dst_off_bytes, rows, row_bytes, flag_base) rows this rank pushes.
  m.def(
      "gemm_ag",
      [](int M, int N, int K, uintptr_t A, long long lda, bool a_mn, uintptr_t B, long long ldb, bool b_mn,
         uintptr_t C, long long ldc, int epi, uintptr_t bias, uintptr_t aux, long long ld_aux, uintptr_t aux_out,
         long long ld_aux_out, int splits, int world, int rank, unsigned epoch, std::vector<uintptr_t> peer_data,
         std::vector<uintptr_t> peer_flags, std::vector<std::array<long long, 5>> segs, int b_flag_base,
         int ready_base, uintptr_t stream) {
        GemmProblem p;
        p.M = M;
        p.N = N;
        p.K = K;
        p.A = P<const __nv_bfloat16>(A);
        p.lda = lda;
        p.a_mn = a_mn;
        p.B = P<const __nv_bfloat16>(B);
        p.ldb = ldb;
        p.b_mn = b_mn;
        p.C = P<void>(C);
        p.ldc = ldc;
        p.epi = epi;
        p.bias = P<const __nv_bfloat16>(bias);
        p.aux = P<const __nv_bfloat16>(aux);
        p.ld_aux = ld_aux;
        p.aux_out = P<__nv_bfloat16>(aux_out);
        p.ld_aux_out = ld_aux_out;
        p.splits = splits;
        if (world < 1 || world > 8 || (int)peer_data.size() != world || (int)peer_flags.size() != world ||
            segs.size() > 8)
          throw std::invalid_argument("gemm_ag: bad gather description");
        p.ag.world = world;
        p.ag.rank = rank;
        p.ag.epoch = epoch;
        for (int r = 0; r < world; ++r) {
          p.ag.peer_data[r] = reinterpret_cast<char*>(peer_data[r]);
          p.ag.peer_flags[r] = reinterpret_cast<unsigned*>(peer_flags[r]);
        }
        p.ag.nseg = (int)segs.size();
        for (size_t i = 0; i < segs.size(); ++i) {
          if (segs[i][0] % 16 || segs[i][1] % 16 || segs[i][3] % 16)
            throw std::invalid_argument("gemm_ag: gathered rows must be 16-byte aligned");
          p.ag.seg[i].src = reinterpret_cast<const void*>(segs[i][0]);
          p.ag.seg[i].dst_off_bytes = segs[i][1];
          p.ag.seg[i].rows = segs[i][2];
          p.ag.seg[i].row_bytes = segs[i][3];
          p.ag.seg[i].flag_base = (int)segs[i][4];
        }
        p.ag.b_flag_base = b_flag_base;
        p.ag.ready_base = ready_base;
        gemm_bf16_tcgen05(p, S(stream));
      });
  m.def("gemm_f32", [](uintptr_t A, uintptr_t B, uintptr_t C, int M, int N, int K, bool b_trans, uintptr_t s) {
    gemm_f32_simt(P<const float>(A), P<const float>(B), P<float>(C), M, N, K, b_trans, S(s));
  });
  m.def("gemm_f32_3xtf32", [](uintptr_t A, uintptr_t B, uintptr_t C, int M, int N, int K, bool b_trans, uintptr_t ws_a,
                              uintptr_t ws_b, uintptr_t s) {
    gemm_f32_3xtf32(P<const float>(A), P<const float>(B), P<float>(C), M, N, K, b_trans, P<float>(ws_a), P<float>(ws_b),
                    S(s));
  });
  m.def("ew_binary", [](int op, int dt, uintptr_t a, uintptr_t b, uintptr_t out, long long n, uintptr_t s) {
    ew_binary(op, dt, P<const void>(a), P<const void>(b), P<void>(out), n, S(s));
  });
  m.def("ew_scalar", [](int op, int dt, uintptr_t a, float sc, uintptr_t out, long long n, uintptr_t s) {
    ew_scalar(op, dt, P<const void>(a), sc, P<void>(out), n, S(s));
  });
  m.def("cast", [](int sdt, int ddt, uintptr_t src, uintptr_t dst, long long n, uintptr_t s) {
    cast(sdt, ddt, P<const void>(src), P<void>(dst), n, S(s));
  });
  m.def("reduce_sum_partials", &reduce_sum_partials);
  m.def("reduce_sum", [](int dt, uintptr_t x, long long n, uintptr_t out, uintptr_t partials, uintptr_t counter,
                         uintptr_t s) {
    reduce_sum(dt, P<const void>(x), n, P<float>(out), P<float>(partials), P<unsigned int>(counter), S(s));
  });
  m.def("gelu_fwd", [](int dt, uintptr_t x, uintptr_t y, long long n, uintptr_t s) {
    gelu_fwd(dt, P<const void>(x), P<void>(y), n, S(s));
  });
  m.def("gelu_bwd", [](int dt, uintptr_t x, uintptr_t dy, uintptr_t dx, long long n, uintptr_t s) {
    gelu_bwd(dt, P<const void>(x), P<const void>(dy), P<void>(dx), n, S(s));
  });
  m.def("colsum_accum", [](uintptr_t x, long long ld, uintptr_t out, int rows, int cols, uintptr_t s) {
    colsum_accum(P<const __nv_bfloat16>(x), ld, P<float>(out), rows, cols, S(s));
  });
  m.def("rmsnorm_fwd", [](int dt, uintptr_t x, uintptr_t w, uintptr_t y, uintptr_t rstd, int rows, int cols,
                          float eps, uintptr_t s) {
    rmsnorm_fwd(dt, P<const void>(x), P<const void>(w), P<void>(y), P<float>(rstd), rows, cols, eps, S(s));
  });
  m.def("rmsnorm_bwd", [](int dt, uintptr_t dy, uintptr_t x, uintptr_t w, uintptr_t rstd, uintptr_t dres,
                          uintptr_t dx, uintptr_t dw, int rows, int cols, uintptr_t s) {
    rmsnorm_bwd(dt, P<const void>(dy), P<const void>(x), P<const void>(w), P<const float>(rstd), P<const void>(dres),
                P<void>(dx), P<float>(dw), rows, cols, S(s));
  });
  m.def(
      "embedding_fwd",
      [](int dt, uintptr_t ids, uintptr_t tok, uintptr_t pos, uintptr_t out, int rows, int dim, int seq_len,
         uintptr_t s, long long vocab) {
        embedding_fwd(dt, P<const int64_t>(ids), P<const void>(tok), P<const void>(pos), P<void>(out), rows, dim,
                      seq_len, vocab, S(s));
      },
      py::arg("dt"), py::arg("ids"), py::arg("tok"), py::arg("pos"), py::arg("out"), py::arg("rows"), py::arg("dim"),
      py::arg("seq_len"), py::arg("stream"), py::arg("vocab") = 0);
  m.def(
      "embedding_bwd",
      [](int dt, uintptr_t ids, uintptr_t dout, uintptr_t dtok, uintptr_t dpos, int rows, int dim, int seq_len,
         uintptr_t s, long long vocab) {
        embedding_bwd(dt, P<const int64_t>(ids), P<const void>(dout), P<float>(dtok), P<float>(dpos), rows, dim,
                      seq_len, vocab, S(s));
      },
      py::arg("dt"), py::arg("ids"), py::arg("dout"), py::arg("dtok"), py::arg("dpos"), py::arg("rows"),
      py::arg("dim"), py::arg("seq_len"), py::arg("stream"), py::arg("vocab") = 0);
  m.def("softmax_ce", [](int dt, uintptr_t logits, long long ld, uintptr_t targets, uintptr_t loss_rows,
                         uintptr_t dlogits, int rows, int cols, float grad_scale, uintptr_t grad_scale_ptr,
                         uintptr_t s) {
    softmax_ce_fwd_bwd(dt, P<const void>(logits), ld, P<const int64_t>(targets), P<float>(loss_rows), P<void>(dlogits),
                       rows, cols, grad_scale, P<const float>(grad_scale_ptr), S(s));
  });
  m.def("softmax_rows", [](int dt, uintptr_t x, uintptr_t y, int rows, int cols, uintptr_t s) {
    softmax_rows(dt, P<const void>(x), P<void>(y), rows, cols, S(s));
  });
  m.def("softmax_rows_bwd", [](int dt, uintptr_t y, uintptr_t dy, uintptr_t dx, int rows, int cols, uintptr_t s) {
    softmax_rows_bwd(dt, P<const void>(y), P<const void>(dy), P<void>(dx), rows, cols, S(s));
  });
  m.def(
      "adamw",
      [](uintptr_t p32, uintptr_t g, uintptr_t mm, uintptr_t vv, uintptr_t p16, long long n, float lr, float b1,
         float b2, float eps, float wd, bool decoupled, float grad_scale, int step, uintptr_t step_ptr,
         uintptr_t lr_ptr, bool bf16_grad, uintptr_t s) {
        AdamWArgs a{};
        a.lr = lr;
        a.beta1 = b1;
        a.beta2 = b2;
        a.eps = eps;
        a.weight_decay = wd;
        a.decoupled = decoupled ? 1 : 0;
        a.grad_scale = grad_scale;
        a.step = step;
        a.step_ptr = P<const int>(step_ptr);
        a.lr_ptr = P<const float>(lr_ptr);
        if (bf16_grad)
          adamw_step_bf16grad(a, P<float>(p32), P<const __nv_bfloat16>(g), P<float>(mm), P<float>(vv),
                              P<__nv_bfloat16>(p16), n, S(s));
        else
          adamw_step(a, P<float>(p32), P<const float>(g), P<float>(mm), P<float>(vv), P<__nv_bfloat16>(p16), n, S(s));
      },
      py::arg("p32"), py::arg("g"), py::arg("m"), py::arg("v"), py::arg("p16"), py::arg("n"), py::arg("lr"),
      py::arg("beta1"), py::arg("beta2"), py::arg("eps"), py::arg("weight_decay"), py::arg("decoupled"),
      py::arg("grad_scale"), py::arg("step"), py::arg("step_ptr") = 0, py::arg("lr_ptr") = 0,
      py::arg("bf16_grad") = false, py::arg("stream") = 0);
  m.def("increment_counter", [](uintptr_t c, uintptr_t s) { increment_counter(P<int>(c), S(s)); });
  m.def("fill_f32", [](uintptr_t x, float v, long long n, uintptr_t s) { fill_f32(P<float>(x), v, n, S(s)); });
  m.def("attention_f32", [](uintptr_t q, uintptr_t k, uintptr_t v, uintptr_t out, int T, int F, float scale,
                            bool causal, uintptr_t s) {
    attention_naive_f32(P<const float>(q), P<const float>(k), P<const float>(v), P<float>(out), T, F, scale, causal,
                        S(s));
  });
  m.def("conv2d_fwd", [](uintptr_t x, uintptr_t w, uintptr_t b, uintptr_t y, int N, int C, int H, int W, int K, int R,
                         int S_, int sh, int sw, int ph, int pw, int P_, int Q, uintptr_t s) {
    conv2d_fwd_f32(P<const float>(x), P<const float>(w), P<const float>(b), P<float>(y), N, C, H, W, K, R, S_, sh, sw,
                   ph, pw, P_, Q, S(s));
  });
  m.def("conv2d_dgrad", [](uintptr_t dy, uintptr_t w, uintptr_t dx, int N, int C, int H, int W, int K, int R, int S_,
                           int sh, int sw, int ph, int pw, int P_, int Q, uintptr_t s) {
    conv2d_dgrad_f32(P<const float>(dy), P<const float>(w), P<float>(dx), N, C, H, W, K, R, S_, sh, sw, ph, pw, P_, Q,
                     S(s));
  });
  m.def("conv2d_wgrad", [](uintptr_t dy, uintptr_t x, uintptr_t dw, uintptr_t db, int N, int C, int H, int W, int K,
                           int R, int S_, int sh, int sw, int ph, int pw, int P_, int Q, uintptr_t s) {
    conv2d_wgrad_f32(P<const float>(dy), P<const float>(x), P<float>(dw), P<float>(db), N, C, H, W, K, R, S_, sh, sw,
                     ph, pw, P_, Q, S(s));
  });
  m.def(
      "flash_attn_fwd",
      [](uintptr_t q, uintptr_t k, uintptr_t v, uintptr_t o, uintptr_t lse, long long qsb, long long qst,
         long long ksb, long long kst, long long vsb, long long vst, long long osb, long long ost, int B, int H, int T,
         int D, float scale, bool causal, uintptr_t s) {
        AttnParams p{};
        p.q = P<const __nv_bfloat16>(q);
        p.k = P<const __nv_bfloat16>(k);
        p.v = P<const __nv_bfloat16>(v);
        p.o = P<__nv_bfloat16>(o);
        p.lse = P<float>(lse);
        p.q_stride_b = qsb;
        p.q_stride_t = qst;
        p.k_stride_b = ksb;
        p.k_stride_t = kst;
        p.v_stride_b = vsb;
        p.v_stride_t = vst;
        p.o_stride_b = osb;
        p.o_stride_t = ost;
        p.B = B;
        p.H = H;
        p.T = T;
        p.D = D;
        p.scale = scale;
        p.causal = causal ? 1 : 0;
        flash_attn_fwd(p, S(s));
      });
  m.def(
      "flash_attn_bwd",
      [](uintptr_t q, uintptr_t k, uintptr_t v, uintptr_t o, uintptr_t lse, uintptr_t dout, uintptr_t dq, uintptr_t dk,
         uintptr_t dv, uintptr_t delta, uintptr_t dq_accum, long long qsb, long long qst, long long ksb, long long kst,
         long long vsb, long long vst, long long osb, long long ost, long long dosb, long long dost, long long dqsb,
         long long dqst, long long dksb, long long dkst, long long dvsb, long long dvst, int B, int H, int T, int D,
         float scale, bool causal, uintptr_t s) {
        AttnBwdParams p{};
        p.f.q = P<const __nv_bfloat16>(q);
        p.f.k = P<const __nv_bfloat16>(k);
        p.f.v = P<const __nv_bfloat16>(v);
        p.f.o = P<__nv_bfloat16>(o);
        p.f.lse = P<float>(lse);
        p.f.q_stride_b = qsb;
        p.f.q_stride_t = qst;
        p.f.k_stride_b = ksb;
        p.f.k_stride_t = kst;
        p.f.v_stride_b = vsb;
        p.f.v_stride_t = vst;
        p.f.o_stride_b = osb;
        p.f.o_stride_t = ost;
        p.f.B = B;
        p.f.H = H;
        p.f.T = T;
        p.f.D = D;
        p.f.scale = scale;
        p.f.causal = causal ? 1 : 0;
        p.dout = P<const __nv_bfloat16>(dout);
        p.do_stride_b = dosb;
        p.do_stride_t = dost;
        p.dq = P<__nv_bfloat16>(dq);
        p.dk = P<__nv_bfloat16>(dk);
        p.dv = P<__nv_bfloat16>(dv);
        p.dq_stride_b = dqsb;
        p.dq_stride_t = dqst;
        p.dk_stride_b = dksb;
        p.dk_stride_t = dkst;
        p.dv_stride_b = dvsb;
        p.dv_stride_t = dvst;
        p.delta = P<float>(delta);
        p.dq_accum = P<float>(dq_accum);
        flash_attn_bwd(p, S(s));
      });

  m.def("set_attn_bwd_trace", [](uintptr_t buf) { set_attn_bwd_trace(P<unsigned long long>(buf)); });
  m.def("set_attn_fwd_trace", [](uintptr_t buf) { set_attn_fwd_trace(P<unsigned long long>(buf)); });
  m.def("set_gemm_trace", [](uintptr_t buf) { set_gemm_trace(P<unsigned long long>(buf)); });

  m.def("raster_iso", [](uintptr_t quads, uintptr_t colors, int n, uintptr_t order, uintptr_t rgba, int w, int h,
                         uintptr_t s) {
    raster_iso(P<const float>(quads), P<const unsigned int>(colors), n, P<unsigned int>(order),
               P<unsigned int>(rgba), w, h, S(s));
  });

  bind_comm(m);
}
