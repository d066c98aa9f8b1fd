// torch_ops.cpp -- the MoE layer as PyTorch dispatcher operators over the C ABI.
//
// Registers torch.ops.gemms_b200.moe and torch.ops.gemms_b200.run (CUDA
// kernels plus Meta kernels for shape propagation).  Both call gemms_moe_fwd
// (include/gemms_moe.h) on the tensors' device and its current stream, with a
// workspace from PyTorch's caching allocator (stream-ordered, reused across
// calls); nothing here computes anything itself.
//
// run() is the reference operator's signature (flashinfer_baseline.py:5-16,
// with its fixed n_group / topk_group / top_k, :48-50, as defaulted
// arguments); moe() is the full layer surface moe(x, router_w, router_bias,
// w13, w13_scale, w2, w2_scale, ...).  Errors raise through TORCH_CHECK (a
// RuntimeError in Python), with the library's message for C-ABI codes.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include "gemms_moe.h"

namespace {

constexpr int64_t kBlock = 128;

void check_cuda(const at::Tensor& t, const char* name, at::ScalarType dt, c10::Device dev) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor (no CPU path)");
  TORCH_CHECK(t.device() == dev, name, " must be on ", dev);
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
  TORCH_CHECK(t.scalar_type() == dt, name, " must be ", c10::toString(dt), ", got ", c10::toString(t.scalar_type()));
}

at::Tensor call_fwd(GemmsMoeArgs& args, const at::Tensor& like) {
  const size_t nbytes = gemms_moe_workspace_size(&args.shape);
  TORCH_CHECK(nbytes > 0, "gemms_b200: unsupported MoE geometry (T=", args.shape.T, " H=", args.shape.H,
              " I=", args.shape.I, " E=", args.shape.E, " n_group=", args.shape.n_group, " topk_group=",
              args.shape.topk_group, " top_k=", args.shape.top_k, ")");
  at::Tensor ws = at::empty({static_cast<int64_t>(nbytes) + 256}, like.options().dtype(at::kByte));
  const uintptr_t base = reinterpret_cast<uintptr_t>(ws.data_ptr());
  void* aligned = reinterpret_cast<void*>((base + 255) & ~uintptr_t(255));
  auto stream = c10::cuda::getCurrentCUDAStream(like.device().index());
  const int rc = gemms_moe_fwd(&args, aligned, nbytes, reinterpret_cast<gemms_stream_t>(stream.stream()));
  TORCH_CHECK(rc == 0, "gemms_moe_fwd failed: ", gemms_strerror(rc), " (code ", rc, ")");
  return ws;
}

at::Tensor moe_cuda(const at::Tensor& x, const at::Tensor& router_w, const at::Tensor& router_bias,
                    const at::Tensor& w13, const at::Tensor& w13_scale, const at::Tensor& w2,
                    const at::Tensor& w2_scale, const c10::optional<at::Tensor>& shared_w13,
                    const c10::optional<at::Tensor>& shared_w13_scale, const c10::optional<at::Tensor>& shared_w2,
                    const c10::optional<at::Tensor>& shared_w2_scale, int64_t n_group, int64_t topk_group,
                    int64_t top_k, double routed_scaling_factor, int64_t inter_planes) {
  const c10::Device dev = x.device();
  c10::cuda::CUDAGuard guard(dev);
  TORCH_CHECK(x.dim() == 2, "x must be bf16 [T, H]");
  check_cuda(x, "x", at::kBFloat16, dev);
  const int64_t T = x.size(0), H = x.size(1);
  TORCH_CHECK(w13.dim() == 3 && w13.size(2) == H, "w13 must be [E, 2I, H]");
  const int64_t E = w13.size(0), I = w13.size(1) / 2;
  TORCH_CHECK(H % kBlock == 0 && I % kBlock == 0, "H and I must be multiples of 128");
  check_cuda(router_w, "router_w", at::kFloat, dev);
  TORCH_CHECK(router_w.dim() == 2 && router_w.size(0) == E && router_w.size(1) == H, "router_w must be [E, H]");
  TORCH_CHECK(router_bias.is_cuda() && router_bias.device() == dev && router_bias.is_contiguous() &&
                  (router_bias.scalar_type() == at::kFloat || router_bias.scalar_type() == at::kBFloat16) &&
                  router_bias.size(-1) == E,
              "router_bias must be fp32 or bf16 [E] on the device of x");
  check_cuda(w13, "w13", at::kFloat8_e4m3fn, dev);
  check_cuda(w2, "w2", at::kFloat8_e4m3fn, dev);
  check_cuda(w13_scale, "w13_scale", at::kFloat, dev);
  check_cuda(w2_scale, "w2_scale", at::kFloat, dev);
  TORCH_CHECK(w13_scale.sizes() == at::IntArrayRef({E, 2 * I / kBlock, H / kBlock}), "w13_scale must be [E, 2I/128, H/128]");
  TORCH_CHECK(w2.sizes() == at::IntArrayRef({E, H, I}), "w2 must be [E, H, I]");
  TORCH_CHECK(w2_scale.sizes() == at::IntArrayRef({E, H / kBlock, I / kBlock}), "w2_scale must be [E, H/128, I/128]");
  const bool has_shared = shared_w13.has_value();
  TORCH_CHECK(has_shared == shared_w13_scale.has_value() && has_shared == shared_w2.has_value() &&
                  has_shared == shared_w2_scale.has_value(),
              "pass all four shared-expert tensors or none");
  if (has_shared) {
    check_cuda(*shared_w13, "shared_w13", at::kFloat8_e4m3fn, dev);
    check_cuda(*shared_w2, "shared_w2", at::kFloat8_e4m3fn, dev);
    check_cuda(*shared_w13_scale, "shared_w13_scale", at::kFloat, dev);
    check_cuda(*shared_w2_scale, "shared_w2_scale", at::kFloat, dev);
    TORCH_CHECK(shared_w13->sizes() == at::IntArrayRef({2 * I, H}) && shared_w2->sizes() == at::IntArrayRef({H, I}),
                "shared expert shapes");
  }
  at::Tensor out = at::empty({T, H}, x.options());
  GemmsMoeArgs a{};
  GemmsMoeShape& s = a.shape;
  s.T = static_cast<int32_t>(T);
  s.H = static_cast<int32_t>(H);
  s.I = static_cast<int32_t>(I);
  s.E = static_cast<int32_t>(E);
  s.E_local = static_cast<int32_t>(E);
  s.n_group = static_cast<int32_t>(n_group);
  s.topk_group = static_cast<int32_t>(topk_group);
  s.top_k = static_cast<int32_t>(top_k);
  s.has_shared = has_shared ? 1 : 0;
  s.input_mode = GEMMS_INPUT_BF16;
  s.bias_bf16 = router_bias.scalar_type() == at::kBFloat16 ? 1 : 0;
  s.inter_planes = static_cast<int32_t>(inter_planes);
  s.routed_scaling_factor = static_cast<float>(routed_scaling_factor);
  a.router_w = router_w.data_ptr<float>();
  a.routing_bias = router_bias.data_ptr();
  a.hidden_bf16 = x.data_ptr();
  a.w13 = w13.data_ptr();
  a.w13_scale = w13_scale.data_ptr<float>();
  a.w2 = w2.data_ptr();
  a.w2_scale = w2_scale.data_ptr<float>();
  if (has_shared) {
    a.shared_w13 = shared_w13->data_ptr();
    a.shared_w13_scale = shared_w13_scale->data_ptr<float>();
    a.shared_w2 = shared_w2->data_ptr();
    a.shared_w2_scale = shared_w2_scale->data_ptr<float>();
  }
  a.out = out.data_ptr();
  call_fwd(a, x);
  return out;
}

at::Tensor run_cuda(const at::Tensor& routing_logits, const at::Tensor& routing_bias, const at::Tensor& hidden_states,
                    const at::Tensor& hidden_states_scale, const at::Tensor& gemm1_weights,
                    const at::Tensor& gemm1_weights_scale, const at::Tensor& gemm2_weights,
                    const at::Tensor& gemm2_weights_scale, int64_t local_expert_offset, double routed_scaling_factor,
                    int64_t n_group, int64_t topk_group, int64_t top_k, int64_t inter_planes) {
  const c10::Device dev = hidden_states.device();
  c10::cuda::CUDAGuard guard(dev);
  check_cuda(routing_logits, "routing_logits", at::kFloat, dev);
  TORCH_CHECK(routing_logits.dim() == 2, "routing_logits must be [T, E]");
  const int64_t T = routing_logits.size(0), E = routing_logits.size(1);
  check_cuda(hidden_states, "hidden_states", at::kFloat8_e4m3fn, dev);
  TORCH_CHECK(hidden_states.dim() == 2 && hidden_states.size(0) == T, "hidden_states must be [T, H]");
  const int64_t H = hidden_states.size(1);
  check_cuda(gemm1_weights, "gemm1_weights", at::kFloat8_e4m3fn, dev);
  TORCH_CHECK(gemm1_weights.dim() == 3 && gemm1_weights.size(2) == H, "gemm1_weights must be [E_local, 2I, H]");
  const int64_t El = gemm1_weights.size(0), I = gemm1_weights.size(1) / 2;
  TORCH_CHECK(H % kBlock == 0 && I % kBlock == 0, "H and I must be multiples of 128");
  check_cuda(hidden_states_scale, "hidden_states_scale", at::kFloat, dev);
  TORCH_CHECK(hidden_states_scale.sizes() == at::IntArrayRef({H / kBlock, T}), "hidden_states_scale must be [H/128, T]");
  check_cuda(gemm1_weights_scale, "gemm1_weights_scale", at::kFloat, dev);
  TORCH_CHECK(gemm1_weights_scale.sizes() == at::IntArrayRef({El, 2 * I / kBlock, H / kBlock}), "gemm1_weights_scale shape");
  check_cuda(gemm2_weights, "gemm2_weights", at::kFloat8_e4m3fn, dev);
  TORCH_CHECK(gemm2_weights.sizes() == at::IntArrayRef({El, H, I}), "gemm2_weights must be [E_local, H, I]");
  check_cuda(gemm2_weights_scale, "gemm2_weights_scale", at::kFloat, dev);
  TORCH_CHECK(gemm2_weights_scale.sizes() == at::IntArrayRef({El, H / kBlock, I / kBlock}), "gemm2_weights_scale shape");
  TORCH_CHECK(routing_bias.is_cuda() && routing_bias.device() == dev && routing_bias.is_contiguous() &&
                  (routing_bias.scalar_type() == at::kFloat || routing_bias.scalar_type() == at::kBFloat16) &&
                  routing_bias.size(-1) == E,
              "routing_bias must be fp32 or bf16 [E] on the device of hidden_states");
  at::Tensor out = at::empty({T, H}, hidden_states.options().dtype(at::kBFloat16));
  GemmsMoeArgs a{};
  GemmsMoeShape& s = a.shape;
  s.T = static_cast<int32_t>(T);
  s.H = static_cast<int32_t>(H);
  s.I = static_cast<int32_t>(I);
  s.E = static_cast<int32_t>(E);
  s.E_local = static_cast<int32_t>(El);
  s.local_expert_offset = static_cast<int32_t>(local_expert_offset);
  s.n_group = static_cast<int32_t>(n_group);
  s.topk_group = static_cast<int32_t>(topk_group);
  s.top_k = static_cast<int32_t>(top_k);
  s.has_shared = 0;
  s.input_mode = GEMMS_INPUT_FP8;
  s.bias_bf16 = routing_bias.scalar_type() == at::kBFloat16 ? 1 : 0;
  s.inter_planes = static_cast<int32_t>(inter_planes);
  s.routed_scaling_factor = static_cast<float>(routed_scaling_factor);
  a.routing_logits = routing_logits.data_ptr<float>();
  a.routing_bias = routing_bias.data_ptr();
  a.hidden_fp8 = hidden_states.data_ptr();
  a.hidden_scale = hidden_states_scale.data_ptr<float>();
  a.w13 = gemm1_weights.data_ptr();
  a.w13_scale = gemm1_weights_scale.data_ptr<float>();
  a.w2 = gemm2_weights.data_ptr();
  a.w2_scale = gemm2_weights_scale.data_ptr<float>();
  a.out = out.data_ptr();
  call_fwd(a, hidden_states);
  return out;
}

// Meta kernels: output shape and dtype only (torch.compile / fake tensors).
at::Tensor moe_meta(const at::Tensor& x, const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                    const at::Tensor&, const at::Tensor&, const c10::optional<at::Tensor>&,
                    const c10::optional<at::Tensor>&, const c10::optional<at::Tensor>&,
                    const c10::optional<at::Tensor>&, int64_t, int64_t, int64_t, double, int64_t) {
  return at::empty_like(x);
}

at::Tensor run_meta(const at::Tensor& routing_logits, const at::Tensor&, const at::Tensor& hidden_states,
                    const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                    int64_t, double, int64_t, int64_t, int64_t, int64_t) {
  return at::empty({routing_logits.size(0), hidden_states.size(1)}, hidden_states.options().dtype(at::kBFloat16));
}

}  // namespace

TORCH_LIBRARY(gemms_b200, m) {
  m.def(
      "moe(Tensor x, Tensor router_w, Tensor router_bias, Tensor w13, Tensor w13_scale, Tensor w2, "
      "Tensor w2_scale, Tensor? shared_w13=None, Tensor? shared_w13_scale=None, Tensor? shared_w2=None, "
      "Tensor? shared_w2_scale=None, int n_group=8, int topk_group=4, int top_k=8, "
      "float routed_scaling_factor=2.5, int inter_planes=2) -> Tensor");
  m.def(
      "run(Tensor routing_logits, Tensor routing_bias, Tensor hidden_states, Tensor hidden_states_scale, "
      "Tensor gemm1_weights, Tensor gemm1_weights_scale, Tensor gemm2_weights, Tensor gemm2_weights_scale, "
      "int local_expert_offset, float routed_scaling_factor, int n_group=8, int topk_group=4, int top_k=8, "
      "int inter_planes=2) -> Tensor");
}

TORCH_LIBRARY_IMPL(gemms_b200, CUDA, m) {
  m.impl("moe", &moe_cuda);
  m.impl("run", &run_cuda);
}

TORCH_LIBRARY_IMPL(gemms_b200, Meta, m) {
  m.impl("moe", &moe_meta);
  m.impl("run", &run_meta);
}
