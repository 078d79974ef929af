// Bindings of the flash-attention kernels (attention.cu).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "kernels.h"

int* vagus_device_error_ptr();   // bindings.cpp

namespace {

using torch::Tensor;

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check(int rc, const char* what) {
  TORCH_CHECK(rc == 0, "vagus_b200 kernel '", what, "' rejected the problem or failed to launch (code ", rc, ")");
}

vagus::AttnArgs make_args(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& o, const Tensor& lse,
                          bool causal, double scale) {
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "attention: (B, H, L, D) tensors");
  for (const Tensor* t : {&q, &k, &v, &o})
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->stride(3) == 1, "attention: bf16 with unit inner stride");
  vagus::AttnArgs a;
  a.q = q.data_ptr(); a.k = k.data_ptr(); a.v = v.data_ptr(); a.o = o.data_ptr();
  a.lse = lse.data_ptr<float>();
  a.B = q.size(0); a.H = static_cast<int>(q.size(1)); a.Hk = static_cast<int>(k.size(1));
  a.Lq = static_cast<int>(q.size(2)); a.Lk = static_cast<int>(k.size(2));
  a.D = static_cast<int>(q.size(3)); a.Dv = static_cast<int>(v.size(3));
  a.sq_b = q.stride(0); a.sq_h = q.stride(1); a.sq_l = q.stride(2);
  a.sk_b = k.stride(0); a.sk_h = k.stride(1); a.sk_l = k.stride(2);
  a.sv_b = v.stride(0); a.sv_h = v.stride(1); a.sv_l = v.stride(2);
  a.so_b = o.stride(0); a.so_h = o.stride(1); a.so_l = o.stride(2);
  a.causal = causal ? 1 : 0;
  a.scale = static_cast<float>(scale);
  a.err = vagus_device_error_ptr();
  return a;
}

// q (B, H, Lq, D), k (B, Hk, Lk, D), v (B, Hk, Lk, Dv) -> o (B, H, Lq, Dv), lse (B, H, Lq)
// o is token-major underneath, (B, Lq, H, Dv) viewed as (B, H, Lq, Dv): the
// head concat that follows (transpose + reshape to (B, Lq, H Dv)) is a view
std::vector<Tensor> attn_fwd(Tensor q, Tensor k, Tensor v, bool causal, double scale) {
  auto o = torch::empty({q.size(0), q.size(2), q.size(1), v.size(3)}, q.options()).transpose(1, 2);
  auto lse = torch::empty({q.size(0), q.size(1), q.size(2)}, q.options().dtype(at::kFloat));
  auto a = make_args(q, k, v, o, lse, causal, scale);
  check(vagus::attn_fwd(a, stream()), "attn_fwd");
  return {o, lse};
}

// A gradient in the layout of x where that layout is dense with 8-element
// strides (so the gradient flows back through x's views without a copy),
// else contiguous.
Tensor grad_like(const Tensor& x) {
  auto t = torch::empty_like(x);
  bool ok = t.stride(3) == 1;
  for (int d = 0; d < 3; ++d) ok = ok && t.stride(d) % 8 == 0;
  return ok ? t : torch::empty(x.sizes(), x.options());
}

// A caller-given gradient buffer (a slice of a packed projection's gradient,
// say) or a fresh one in the layout of x
Tensor grad_out(const c10::optional<Tensor>& given, const Tensor& x, const char* what) {
  if (!given.has_value() || !given->defined()) return grad_like(x);
  const Tensor& t = *given;
  TORCH_CHECK(t.sizes() == x.sizes() && t.scalar_type() == at::kBFloat16 && t.is_cuda(), "attn_bwd: ", what,
              " must be shaped like its input, bf16 on the GPU");
  return t;
}

// dO in o's layout (copied into it when the strides differ) -> dq, dk, dv in
// the layouts of q, k, v, or written into the given buffers (any strides that
// are multiples of 8 elements)
std::vector<Tensor> attn_bwd(Tensor q, Tensor k, Tensor v, Tensor o, Tensor lse, Tensor dO, bool causal,
                             double scale, c10::optional<Tensor> dq_out, c10::optional<Tensor> dk_out,
                             c10::optional<Tensor> dv_out, c10::optional<Tensor> rope_cos,
                             c10::optional<Tensor> rope_sin) {
  TORCH_CHECK(lse.is_contiguous() && dO.sizes() == o.sizes(), "attn_bwd: contiguous lse, dO shaped like o");
  if (dO.strides() != o.strides()) {
    auto t = torch::empty_like(o);
    t.copy_(dO);
    dO = t;
  }
  TORCH_CHECK(dO.strides() == o.strides(), "attn_bwd: o must be dense (dO takes its strides)");
  auto a = make_args(q, k, v, o, lse, causal, scale);
  vagus::AttnBwdArgs b;
  b.f = a;
  b.dO = dO.data_ptr();
  auto dq = grad_out(dq_out, q, "dq_out"), dk = grad_out(dk_out, k, "dk_out"), dv = grad_out(dv_out, v, "dv_out");
  b.sdq_b = dq.stride(0); b.sdq_h = dq.stride(1); b.sdq_l = dq.stride(2);
  b.sdk_b = dk.stride(0); b.sdk_h = dk.stride(1); b.sdk_l = dk.stride(2);
  b.sdv_b = dv.stride(0); b.sdv_h = dv.stride(1); b.sdv_l = dv.stride(2);
  auto dq_acc = torch::empty({q.size(0), q.size(1), q.size(2), q.size(3)}, q.options().dtype(at::kFloat));
  auto delta = torch::empty({q.size(0), q.size(1), q.size(2)}, q.options().dtype(at::kFloat));
  b.dq = dq.data_ptr(); b.dk = dk.data_ptr(); b.dv = dv.data_ptr();
  b.dq_acc = dq_acc.data_ptr<float>(); b.delta = delta.data_ptr<float>();
  if (rope_cos.has_value() && rope_cos->defined()) {
    TORCH_CHECK(rope_sin.has_value() && rope_sin->defined(), "attn_bwd: rope_cos needs rope_sin");
    for (const Tensor* t : {&*rope_cos, &*rope_sin})
      TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->dim() == 2 && t->size(0) == k.size(2) &&
                      t->size(1) == q.size(3) / 2,
                  "attn_bwd: RoPE tables (Lk, D / 2) fp32 contiguous");
    b.rope_cos = rope_cos->data_ptr<float>();
    b.rope_sin = rope_sin->data_ptr<float>();
  }
  check(vagus::attn_bwd(b, stream()), "attn_bwd");
  return {dq, dk, dv};
}

}  // namespace

void register_attn_ops(pybind11::module& m) {
  m.def("attn_fwd", &attn_fwd);
  m.def("attn_bwd", &attn_bwd, pybind11::arg("q"), pybind11::arg("k"), pybind11::arg("v"), pybind11::arg("o"),
        pybind11::arg("lse"), pybind11::arg("dO"), pybind11::arg("causal"), pybind11::arg("scale"),
        pybind11::arg("dq_out") = pybind11::none(), pybind11::arg("dk_out") = pybind11::none(),
        pybind11::arg("dv_out") = pybind11::none(), pybind11::arg("rope_cos") = pybind11::none(),
        pybind11::arg("rope_sin") = pybind11::none());
  // buf: int64 device tensor of 512 entries, or None
  m.def("attn_set_trace", [](c10::optional<Tensor> buf) {
    if (buf) TORCH_CHECK(buf->is_cuda() && buf->numel() >= 512 && buf->element_size() == 8, "attn_set_trace: 512 x u64");
    vagus::attn_set_trace(buf ? reinterpret_cast<unsigned long long*>(buf->data_ptr()) : nullptr);
  });
}
