// PyTorch operator library torch.ops.mrun_b200.* over the C ABI of libmrun_b200.so.
//
// A thin layer: each operator takes tensors, checks that they are CUDA tensors of the
// expected dtype and layout, and calls the matching mrb_* entry point on the current CUDA
// stream of the first tensor's device. Outputs are caller-allocated (`Tensor(a!)` in the
// schemas), so the operators allocate nothing and can be captured in CUDA graphs. The
// Python mirror (mrun_b200/dense_qstore_cuda.py, moe.py, qstore_build.py) validates
// arguments with the reference's messages and then calls these operators. A failed C call
// raises ValueError for a bad argument (MRB_ERR_ARG) and RuntimeError otherwise, with the
// library's message.
#include <ATen/cuda/CUDAContext.h>
#include <torch/library.h>

#include <optional>

#include "../../include/mrun_b200.h"

namespace {

void check_status(int rc, const char* what) {
  if (rc == MRB_OK) return;
  const char* msg = mrb_last_error();
  if (rc == MRB_ERR_ARG) TORCH_CHECK_VALUE(false, what, ": ", msg);
  TORCH_CHECK(false, what, ": ", msg);
}

void* stream_of(const at::Tensor& t) { return at::cuda::getCurrentCUDAStream(t.device().index()).stream(); }

void need(const at::Tensor& t, at::ScalarType dtype, const char* what) {
  TORCH_CHECK_VALUE(t.is_cuda(), what, " must be a CUDA tensor");
  TORCH_CHECK_VALUE(t.scalar_type() == dtype, what, " has dtype ", t.scalar_type(), ", expected ", dtype);
  TORCH_CHECK_VALUE(t.is_contiguous(), what, " must be contiguous");
}

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return MRB_F32;
    case at::kBFloat16: return MRB_BF16;
    case at::kHalf: return MRB_F16;
    default: TORCH_CHECK_VALUE(false, "unsupported activation dtype ", t);
  }
  return -1;
}

template <typename T>
T* opt_ptr(const std::optional<at::Tensor>& t) {
  return t.has_value() && t->defined() ? static_cast<T*>(t->data_ptr()) : nullptr;
}

// y = x @ (codes * scales[:, None]).T (+ bias): mrb_qrow_matmul
void qrow_linear(const at::Tensor& x, const at::Tensor& codes, const at::Tensor& scales,
                 const std::optional<at::Tensor>& bias, at::Tensor& out, const std::optional<at::Tensor>& workspace) {
  TORCH_CHECK_VALUE(x.dim() == 2 && codes.dim() == 2 && out.dim() == 2, "qrow_linear: 2-D tensors expected");
  need(x, x.scalar_type(), "activations");
  need(codes, at::kChar, "codes");
  need(scales, at::kFloat, "scales");
  need(out, x.scalar_type(), "out");
  const int64_t m = x.size(0), k = x.size(1), n = codes.size(0);
  TORCH_CHECK_VALUE(codes.size(1) == k && scales.numel() == n && out.size(0) == m && out.size(1) == n,
                    "qrow_linear: shapes do not match");
  if (bias.has_value() && bias->defined()) need(*bias, at::kFloat, "bias");
  if (workspace.has_value() && workspace->defined()) need(*workspace, at::kByte, "workspace");
  const int code = dtype_code(x.scalar_type());
  check_status(mrb_qrow_matmul(x.data_ptr(), code, m, k, codes.data_ptr<int8_t>(), scales.data_ptr<float>(), n,
                               opt_ptr<float>(bias), out.data_ptr(), code, opt_ptr<void>(workspace),
                               workspace.has_value() && workspace->defined() ? (size_t)workspace->numel() : 0,
                               stream_of(x)),
               "qrow_linear");
}

// y = bf16(silu(bf16(x.Wg)) * bf16(x.Wu)): mrb_qrow_swiglu
void qrow_swiglu(const at::Tensor& x, const at::Tensor& gate_codes, const at::Tensor& gate_scales,
                 const at::Tensor& up_codes, const at::Tensor& up_scales, at::Tensor& out,
                 const std::optional<at::Tensor>& workspace) {
  need(x, at::kBFloat16, "activations");
  need(gate_codes, at::kChar, "gate codes");
  need(up_codes, at::kChar, "up codes");
  need(gate_scales, at::kFloat, "gate scales");
  need(up_scales, at::kFloat, "up scales");
  need(out, at::kBFloat16, "out");
  const int64_t m = x.size(0), k = x.size(1), n = gate_codes.size(0);
  TORCH_CHECK_VALUE(gate_codes.sizes() == up_codes.sizes() && gate_codes.size(1) == k && out.size(0) == m &&
                        out.size(1) == n,
                    "qrow_swiglu: shapes do not match");
  if (workspace.has_value() && workspace->defined()) need(*workspace, at::kByte, "workspace");
  check_status(mrb_qrow_swiglu(x.data_ptr(), m, k, gate_codes.data_ptr<int8_t>(), gate_scales.data_ptr<float>(),
                               up_codes.data_ptr<int8_t>(), up_scales.data_ptr<float>(), n, out.data_ptr(),
                               opt_ptr<void>(workspace),
                               workspace.has_value() && workspace->defined() ? (size_t)workspace->numel() : 0,
                               stream_of(x)),
               "qrow_swiglu");
}

// per-output-channel symmetric int8: mrb_quant_row_int8
void quant_row_int8(const at::Tensor& weight, at::Tensor& codes, at::Tensor& scales) {
  need(weight, at::kFloat, "weight");
  need(codes, at::kChar, "codes");
  need(scales, at::kFloat, "scales");
  TORCH_CHECK_VALUE(weight.dim() == 2 && codes.sizes() == weight.sizes() && scales.numel() == weight.size(0),
                    "quant_row_int8: shapes do not match");
  check_status(mrb_quant_row_int8(weight.data_ptr<float>(), weight.size(0), weight.size(1), codes.data_ptr<int8_t>(),
                                  scales.data_ptr<float>(), stream_of(weight)),
               "quant_row_int8");
}

// softmax / top-k / renorm: mrb_router_topk
void router_topk(const at::Tensor& logits, int64_t k, bool renorm, at::Tensor& top_idx, at::Tensor& top_w_f32,
                 at::Tensor& top_w_bf16) {
  need(logits, logits.scalar_type(), "logits");
  TORCH_CHECK_VALUE(logits.dim() == 2, "router_topk: logits must be [tokens, experts]");
  need(top_idx, at::kLong, "top_idx");
  need(top_w_f32, at::kFloat, "top_w_f32");
  need(top_w_bf16, at::kBFloat16, "top_w_bf16");
  const int64_t t = logits.size(0), e = logits.size(1);
  TORCH_CHECK_VALUE(top_idx.numel() == t * k && top_w_f32.numel() == t * k && top_w_bf16.numel() == t * k,
                    "router_topk: outputs must hold tokens * k entries");
  check_status(mrb_router_topk(logits.data_ptr(), dtype_code(logits.scalar_type()), t, e, k, renorm ? 1 : 0,
                               top_idx.data_ptr<int64_t>(), top_w_f32.data_ptr<float>(), top_w_bf16.data_ptr(),
                               stream_of(logits)),
               "router_topk");
}

// stable expert-major route plan: mrb_route_compile
void route_compile(const at::Tensor& top_idx, const at::Tensor& top_w, int64_t experts, at::Tensor& counts,
                   at::Tensor& starts, at::Tensor& token_ids, at::Tensor& coef, at::Tensor& inverse) {
  need(top_idx, at::kLong, "top_idx");
  need(top_w, at::kFloat, "top_w");
  TORCH_CHECK_VALUE(top_idx.dim() == 2, "route_compile: top_idx must be [tokens, k]");
  need(counts, at::kInt, "counts");
  need(starts, at::kInt, "starts");
  need(token_ids, at::kLong, "token_ids");
  need(coef, at::kFloat, "coef");
  need(inverse, at::kLong, "inverse");
  const int64_t t = top_idx.size(0), k = top_idx.size(1), a = t * k;
  TORCH_CHECK_VALUE(top_w.numel() == a && counts.numel() == experts && starts.numel() == experts &&
                        token_ids.numel() == a && coef.numel() == a && inverse.numel() == a,
                    "route_compile: shapes do not match");
  check_status(mrb_route_compile(top_idx.data_ptr<int64_t>(), top_w.data_ptr<float>(), t, k, experts,
                                 counts.data_ptr<int32_t>(), starts.data_ptr<int32_t>(), token_ids.data_ptr<int64_t>(),
                                 coef.data_ptr<float>(), inverse.data_ptr<int64_t>(), nullptr, stream_of(top_idx)),
               "route_compile");
}

// fixed-rank combine: mrb_stable_route_reduce
void stable_route_reduce(const at::Tensor& expert_out, const at::Tensor& coef, const at::Tensor& inverse,
                         int64_t tokens, int64_t k, const std::optional<at::Tensor>& out_f32,
                         const std::optional<at::Tensor>& out_bf16) {
  need(expert_out, at::kBFloat16, "expert_out");
  need(coef, at::kFloat, "coef");
  need(inverse, at::kLong, "inverse");
  TORCH_CHECK_VALUE(expert_out.dim() == 2, "stable_route_reduce: expert_out must be [tokens * k, hidden]");
  const int64_t hidden = expert_out.size(1);
  TORCH_CHECK_VALUE(expert_out.size(0) == tokens * k && coef.numel() == tokens * k && inverse.numel() == tokens * k,
                    "stable_route_reduce: shapes do not match");
  const bool f32 = out_f32.has_value() && out_f32->defined(), bf16 = out_bf16.has_value() && out_bf16->defined();
  TORCH_CHECK_VALUE(f32 || bf16, "stable_route_reduce: give out_f32, out_bf16 or both");
  if (f32) {
    need(*out_f32, at::kFloat, "out_f32");
    TORCH_CHECK_VALUE(out_f32->numel() == tokens * hidden, "stable_route_reduce: out_f32 must be [tokens, hidden]");
  }
  if (bf16) {
    need(*out_bf16, at::kBFloat16, "out_bf16");
    TORCH_CHECK_VALUE(out_bf16->numel() == tokens * hidden, "stable_route_reduce: out_bf16 must be [tokens, hidden]");
  }
  check_status(mrb_stable_route_reduce(expert_out.data_ptr(), coef.data_ptr<float>(), inverse.data_ptr<int64_t>(),
                                       tokens, k, hidden, opt_ptr<float>(out_f32), opt_ptr<void>(out_bf16),
                                       stream_of(expert_out)),
               "stable_route_reduce");
}

// gate/up (SwiGLU) then down over expert pages, the down launch overlapping: mrb_grouped_expert_mlp
void grouped_expert_mlp(const at::Tensor& x, const at::Tensor& token_ids, const at::Tensor& starts,
                        const at::Tensor& counts, const at::Tensor& pages, int64_t page_stride,
                        int64_t gate_up_codes_offset, int64_t gate_up_scales_offset, int64_t down_codes_offset,
                        int64_t down_scales_offset, const std::optional<at::Tensor>& slot_of, at::Tensor& act,
                        at::Tensor& y, at::Tensor& sync) {
  need(x, at::kBFloat16, "activations");
  need(token_ids, at::kLong, "token_ids");
  need(starts, at::kInt, "starts");
  need(counts, at::kInt, "counts");
  need(pages, at::kByte, "pages");
  need(act, at::kBFloat16, "act");
  need(y, at::kBFloat16, "y");
  need(sync, at::kInt, "sync");
  if (slot_of.has_value() && slot_of->defined()) need(*slot_of, at::kInt, "slot_of");
  const int64_t experts = counts.numel(), a = token_ids.numel();
  TORCH_CHECK_VALUE(act.dim() == 2 && y.dim() == 2 && act.size(0) == a && y.size(0) == a,
                    "grouped_expert_mlp: act and y must be [assignments, ...]");
  TORCH_CHECK_VALUE(sync.numel() >= 2 * experts + 1, "grouped_expert_mlp: sync must be int32 [2 * experts + 1]");
  check_status(mrb_grouped_expert_mlp(x.data_ptr(), token_ids.data_ptr<int64_t>(), starts.data_ptr<int32_t>(),
                                      counts.data_ptr<int32_t>(), experts, pages.data_ptr(), page_stride,
                                      gate_up_codes_offset, gate_up_scales_offset, down_codes_offset,
                                      down_scales_offset, opt_ptr<int32_t>(slot_of), y.size(1), act.size(1), a,
                                      act.data_ptr(), y.data_ptr(), reinterpret_cast<uint32_t*>(sync.data_ptr<int32_t>()),
                                      stream_of(x)),
               "grouped_expert_mlp");
}

}  // namespace

TORCH_LIBRARY(mrun_b200, m) {
  m.def("qrow_linear(Tensor x, Tensor codes, Tensor scales, Tensor? bias, Tensor(a!) out, Tensor? workspace) -> ()");
  m.def("qrow_swiglu(Tensor x, Tensor gate_codes, Tensor gate_scales, Tensor up_codes, Tensor up_scales, "
        "Tensor(a!) out, Tensor? workspace) -> ()");
  m.def("quant_row_int8(Tensor weight, Tensor(a!) codes, Tensor(b!) scales) -> ()");
  m.def("router_topk(Tensor logits, int k, bool renorm, Tensor(a!) top_idx, Tensor(b!) top_w_f32, "
        "Tensor(c!) top_w_bf16) -> ()");
  m.def("route_compile(Tensor top_idx, Tensor top_w, int experts, Tensor(a!) counts, Tensor(b!) starts, "
        "Tensor(c!) token_ids, Tensor(d!) coef, Tensor(e!) inverse) -> ()");
  m.def("stable_route_reduce(Tensor expert_out, Tensor coef, Tensor inverse, int tokens, int k, "
        "Tensor(a!)? out_f32, Tensor(b!)? out_bf16) -> ()");
  m.def("grouped_expert_mlp(Tensor x, Tensor token_ids, Tensor starts, Tensor counts, Tensor pages, int page_stride, "
        "int gate_up_codes_offset, int gate_up_scales_offset, int down_codes_offset, int down_scales_offset, "
        "Tensor? slot_of, Tensor(a!) act, Tensor(b!) y, Tensor(c!) sync) -> ()");
}

TORCH_LIBRARY_IMPL(mrun_b200, CUDA, m) {
  m.impl("qrow_linear", &qrow_linear);
  m.impl("qrow_swiglu", &qrow_swiglu);
  m.impl("quant_row_int8", &quant_row_int8);
  m.impl("router_topk", &router_topk);
  m.impl("route_compile", &route_compile);
  m.impl("stable_route_reduce", &stable_route_reduce);
  m.impl("grouped_expert_mlp", &grouped_expert_mlp);
}
