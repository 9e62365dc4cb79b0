// fa_torch_binding.cpp -- the pybind11 module flash_attention._fa_torch.
//
// Same role as the reference's compiled module flash_attention._C
// (csrc/flash_api.cpp:9-72): take torch tensors, run the input checks of
// csrc/flash_api.cpp:14-29 with the same messages, allocate O with
// empty_like(q) (flash_api.cpp:31), fill the launch block and launch on the
// current stream of q's device (flash_api.cpp:64).  The launch itself goes
// through the C ABI of libfa_sm100.so (include/fa_sm100.h), which this module
// links against; nothing here computes.  Doing the per-call work in C++
// rather than in Python keeps the host cost of one call well under the
// kernel time of small problems.
#include <torch/extension.h>

#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <cmath>
#include <optional>
#include <string>

#include "fa_sm100.h"

namespace {

void check_status(int rc, const char* what) {
  TORCH_CHECK(rc == FA_OK, what, " failed: ", fa_sm100_status_string(rc), " (status ", rc, ")");
}

void validate(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v) {
  // Same checks and messages as csrc/flash_api.cpp:14-29 ...
  TORCH_CHECK(q.is_cuda(), "q must be on CUDA");
  const auto dt = q.scalar_type();
  TORCH_CHECK(dt == at::kHalf || dt == at::kBFloat16, "q must be fp16 or bf16");
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "q, k, v must be 4-D (batch, seqlen, heads, head_dim)");
  TORCH_CHECK(q.stride(3) == 1, "q must be contiguous in last dim");
  TORCH_CHECK(k.stride(3) == 1, "k must be contiguous in last dim");
  TORCH_CHECK(v.stride(3) == 1, "v must be contiguous in last dim");
  const int64_t d = q.size(3);
  TORCH_CHECK(d == 64 || d == 128, "head_dim must be 64 or 128");
  TORCH_CHECK(k.size(2) > 0 && q.size(2) % k.size(2) == 0, "heads must be divisible by heads_k (for GQA)");
  // ... plus the ones the reference leaves out (its kernel would read K/V of
  // the wrong type, device or head otherwise).
  TORCH_CHECK(k.scalar_type() == dt && v.scalar_type() == dt, "q, k and v must have the same dtype");
  TORCH_CHECK(k.device() == q.device() && v.device() == q.device(), "q, k and v must be on the same device");
  TORCH_CHECK(k.sizes() == v.sizes() && k.size(0) == q.size(0) && k.size(3) == d,
              "k and v must be (batch, seqlen_k, heads_k, head_dim) matching q");
}

// O (and LSE when wanted) for q, k, v; `out` / `lse_out` are optional
// caller-provided destinations (O may be fp32 for partial results).
std::tuple<at::Tensor, std::optional<at::Tensor>> forward_impl(
    const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, bool causal, std::optional<double> softmax_scale,
    int64_t q_pos_offset, int64_t k_pos_offset, bool want_lse, const std::optional<at::Tensor>& out,
    const std::optional<at::Tensor>& lse_out) {
  validate(q, k, v);
  const int64_t b = q.size(0), sq = q.size(1), h = q.size(2), d = q.size(3);
  at::Tensor o;
  if (out.has_value()) {
    o = *out;
    TORCH_CHECK(o.sizes() == q.sizes() && (o.scalar_type() == q.scalar_type() || o.scalar_type() == at::kFloat) &&
                    o.device() == q.device() && o.stride(3) == 1,
                "out must match q's shape and device, with q's dtype or fp32, contiguous in last dim");
  } else {
    o = at::empty_like(q);
  }
  std::optional<at::Tensor> lse;
  if (want_lse) {
    lse = lse_out.has_value() ? *lse_out : at::empty({b, h, sq}, q.options().dtype(at::kFloat));
  }

  FaParams p;
  p.q = q.data_ptr();
  p.k = k.data_ptr();
  p.v = v.data_ptr();
  p.o = o.data_ptr();
  p.lse = lse.has_value() ? lse->data_ptr<float>() : nullptr;
  p.batch = static_cast<int32_t>(b);
  p.seqlen_q = static_cast<int32_t>(sq);
  p.seqlen_k = static_cast<int32_t>(k.size(1));
  p.heads = static_cast<int32_t>(h);
  p.heads_k = static_cast<int32_t>(k.size(2));
  p.head_dim = static_cast<int32_t>(d);
  p.q_batch_stride = q.stride(0);
  p.q_row_stride = q.stride(1);
  p.q_head_stride = q.stride(2);
  p.k_batch_stride = k.stride(0);
  p.k_row_stride = k.stride(1);
  p.k_head_stride = k.stride(2);
  p.v_batch_stride = v.stride(0);
  p.v_row_stride = v.stride(1);
  p.v_head_stride = v.stride(2);
  p.o_batch_stride = o.stride(0);
  p.o_row_stride = o.stride(1);
  p.o_head_stride = o.stride(2);
  p.lse_batch_stride = lse.has_value() ? lse->stride(0) : 0;
  p.lse_head_stride = lse.has_value() ? lse->stride(1) : 0;
  p.softmax_scale =
      static_cast<float>(softmax_scale.has_value() ? *softmax_scale : 1.0 / std::sqrt(static_cast<double>(d)));
  p.is_causal = causal ? 1 : 0;
  p.is_bf16 = q.scalar_type() == at::kBFloat16 ? 1 : 0;
  p.q_pos_offset = q_pos_offset;
  p.k_pos_offset = k_pos_offset;
  p.error_flag = nullptr;
  p.out_f32 = o.scalar_type() == at::kFloat ? 1 : 0;

  const c10::cuda::CUDAGuard guard(q.device());
  const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(q.device().index()).stream();
  check_status(fa_sm100_fwd(&p, stream), "fa_sm100_fwd");
  return {o, lse};
}

// flash_attention._C.forward(q, k, v, causal) -> o  (csrc/flash_api.cpp:9-68)
at::Tensor forward(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, bool causal) {
  return std::get<0>(forward_impl(q, k, v, causal, std::nullopt, 0, 0, false, std::nullopt, std::nullopt));
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "pybind11 binding of libfa_sm100.so (attention forward on sm_100a)";
  m.def("forward", &forward, "attention forward, O only (reference _C.forward)", py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("causal"));
  m.def("forward_with_lse", &forward_impl, "attention forward with optional LSE and destinations", py::arg("q"),
        py::arg("k"), py::arg("v"), py::arg("causal"), py::arg("softmax_scale") = py::none(),
        py::arg("q_pos_offset") = 0, py::arg("k_pos_offset") = 0, py::arg("want_lse") = true,
        py::arg("out") = py::none(), py::arg("lse_out") = py::none());
  m.def("params_size", [] { return fa_sm100_params_size(); });
}
