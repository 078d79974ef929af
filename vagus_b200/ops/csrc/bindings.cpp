// Python bindings of the sm_100a kernels.  Tensor checks live here; the .cu
// files see raw pointers only.  Every op runs on the current CUDA stream.
#include <torch/extension.h>
#include <vector>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "gemm.h"
#include "kernels.h"

namespace {

using torch::Tensor;

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check(int rc, const char* what) {
  TORCH_CHECK(rc == 0, "vagus_b200 kernel '", what, "' failed to launch (code ", rc, ")");
}

bool is_f32(const Tensor& t) { return t.scalar_type() == at::kFloat; }
void need_cuda(const Tensor& t, const char* n) { TORCH_CHECK(t.is_cuda(), n, " must be a CUDA tensor"); }
void need_bf16_or_f32(const Tensor& t, const char* n) {
  TORCH_CHECK(t.scalar_type() == at::kBFloat16 || t.scalar_type() == at::kFloat, n, " must be bf16 or fp32");
}

// -------------------------------------------------------------- error word --
// One host-mapped int per device: kernels record bounded-wait timeouts there
// and the host reads it without a device synchronisation.
int* g_err_host[64] = {nullptr};
int* g_err_dev[64] = {nullptr};

}  // namespace

// Bounds-checked build: every CUDA translation unit registers a function
// that points its copy of the device-side error-word pointer at a device's
// error word; they run when that word is created (one context per device).
namespace {
std::vector<int (*)(int*)>& bounds_installers() {
  static std::vector<int (*)(int*)> v;
  return v;
}
}  // namespace

extern "C" __attribute__((visibility("default"))) void vagus_register_bounds_installer(int (*fn)(int*)) {
  bounds_installers().push_back(fn);
}

// Device pointer of this device's error word (shared with the other binding units).
int* vagus_device_error_ptr() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (!g_err_host[dev]) {
    int* h = nullptr;
    TORCH_CHECK(cudaHostAlloc(&h, sizeof(int), cudaHostAllocMapped) == cudaSuccess, "cudaHostAlloc failed");
    *h = 0;
    int* d = nullptr;
    TORCH_CHECK(cudaHostGetDevicePointer(&d, h, 0) == cudaSuccess, "cudaHostGetDevicePointer failed");
    g_err_host[dev] = h;
    g_err_dev[dev] = d;
    for (auto fn : bounds_installers()) TORCH_CHECK(fn(d) == 0, "installing the bounds-check word failed");
  }
  return g_err_dev[dev];
}

namespace {

int* err_ptr() { return vagus_device_error_ptr(); }

int error_word() {
  int dev = 0;
  cudaGetDevice(&dev);
  err_ptr();
  return *reinterpret_cast<volatile int*>(g_err_host[dev]);
}

void reset_error() {
  int dev = 0;
  cudaGetDevice(&dev);
  err_ptr();
  *reinterpret_cast<volatile int*>(g_err_host[dev]) = 0;
}

// ------------------------------------------------------------------- GEMM --
// C = alpha * op(A) @ op(B)^T + beta * S, operands given as 2-D or 3-D
// (batched) row-major tensors with a unit inner stride.  a_mn / b_mn say the
// operand is stored M- / N-contiguous ([K][M], [K][N]) instead of K-contiguous.
// Returns the launcher's status code (0 = launched) instead of throwing: the
// caller decides how to report a rejected shape.
int64_t gemm(Tensor A, bool a_mn, Tensor B, bool b_mn, Tensor C, c10::optional<Tensor> S, double alpha, double beta,
             bool atomic, int64_t split_k, int64_t block_n) {
  need_cuda(A, "A"); need_cuda(B, "B"); need_cuda(C, "C");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm operands must be bf16");
  TORCH_CHECK(A.dim() == B.dim() && A.dim() == C.dim() && (A.dim() == 2 || A.dim() == 3), "gemm: rank mismatch");
  TORCH_CHECK(A.stride(-1) == 1 && B.stride(-1) == 1 && C.stride(-1) == 1, "gemm: inner stride must be 1");
  need_bf16_or_f32(C, "C");
  TORCH_CHECK(!atomic || is_f32(C), "atomic gemm needs an fp32 output");
  const bool batched = A.dim() == 3;
  vagus::GemmArgs g;
  g.batch = batched ? static_cast<int>(A.size(0)) : 1;
  g.a_mn = a_mn; g.b_mn = b_mn;
  const int64_t ar = A.size(-2), ac = A.size(-1), br = B.size(-2), bc = B.size(-1);
  g.M = static_cast<int>(a_mn ? ac : ar);
  g.K = static_cast<int>(a_mn ? ar : ac);
  g.N = static_cast<int>(b_mn ? bc : br);
  const int64_t kb = b_mn ? br : bc;
  TORCH_CHECK(kb == g.K, "gemm: K mismatch (", g.K, " vs ", kb, ")");
  TORCH_CHECK(C.size(-2) == g.M && C.size(-1) == g.N, "gemm: C shape mismatch");
  g.A = A.data_ptr(); g.B = B.data_ptr();
  g.lda = A.stride(-2); g.ldb = B.stride(-2);
  g.strideA = batched ? A.stride(0) : 0; g.strideB = batched ? B.stride(0) : 0;
  g.C = C.data_ptr(); g.ldc = C.stride(-2); g.strideC = batched ? C.stride(0) : 0; g.c_f32 = is_f32(C);
  if (S.has_value() && S->defined()) {
    const Tensor& s = *S;
    need_bf16_or_f32(s, "S");
    TORCH_CHECK(s.size(-2) == g.M && s.size(-1) == g.N && s.stride(-1) == 1, "gemm: S shape mismatch");
    g.S = s.data_ptr(); g.lds = s.stride(-2); g.strideS = batched ? s.stride(0) : 0; g.s_f32 = is_f32(s);
  }
  g.alpha = static_cast<float>(alpha); g.beta = static_cast<float>(beta);
  g.atomic = atomic ? 1 : 0; g.split_k = static_cast<int>(split_k); g.block_n = static_cast<int>(block_n);
  g.err = err_ptr();
  return vagus::gemm_launch(g, stream());
}

// GEMM whose bf16 product is not written to a local C but scattered by row
// blocks (mode 1) or column blocks (mode 2) of `span` to the buffers at the
// addresses in `dst` (peer mappings of other GPUs' memory for a fused
// product + all-to-all over NVLink): block o goes to dst[o] at
// [batch0 + b][local row][local col] with row pitch dst_ld, batch stride
// dst_stride (elements).
int64_t gemm_scatter(Tensor A, bool a_mn, Tensor B, bool b_mn, c10::optional<Tensor> S, double alpha, double beta,
                     std::vector<int64_t> dst, int64_t mode, int64_t span, int64_t dst_ld, int64_t dst_stride,
                     int64_t batch0) {
  need_cuda(A, "A"); need_cuda(B, "B");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm operands must be bf16");
  TORCH_CHECK(A.dim() == B.dim() && (A.dim() == 2 || A.dim() == 3), "gemm_scatter: rank mismatch");
  TORCH_CHECK(A.stride(-1) == 1 && B.stride(-1) == 1, "gemm_scatter: inner stride must be 1");
  TORCH_CHECK(!dst.empty() && dst.size() <= 16, "gemm_scatter: 1..16 destinations");
  const bool batched = A.dim() == 3;
  vagus::GemmArgs g;
  g.batch = batched ? static_cast<int>(A.size(0)) : 1;
  g.a_mn = a_mn; g.b_mn = b_mn;
  const int64_t ar = A.size(-2), ac = A.size(-1), br = B.size(-2), bc = B.size(-1);
  g.M = static_cast<int>(a_mn ? ac : ar);
  g.K = static_cast<int>(a_mn ? ar : ac);
  g.N = static_cast<int>(b_mn ? bc : br);
  TORCH_CHECK((b_mn ? br : bc) == g.K, "gemm_scatter: K mismatch");
  g.A = A.data_ptr(); g.B = B.data_ptr();
  g.lda = A.stride(-2); g.ldb = B.stride(-2);
  g.strideA = batched ? A.stride(0) : 0; g.strideB = batched ? B.stride(0) : 0;
  g.C = nullptr; g.ldc = 0; g.strideC = 0; g.c_f32 = 0;
  if (S.has_value() && S->defined()) {
    const Tensor& s = *S;
    need_bf16_or_f32(s, "S");
    TORCH_CHECK(s.size(-2) == g.M && s.size(-1) == g.N && s.stride(-1) == 1, "gemm_scatter: S shape mismatch");
    g.S = s.data_ptr(); g.lds = s.stride(-2); g.strideS = batched ? s.stride(0) : 0; g.s_f32 = is_f32(s);
  }
  g.alpha = static_cast<float>(alpha); g.beta = static_cast<float>(beta);
  g.split_k = 1;
  g.scatter = static_cast<int>(mode);
  g.scatter_span = static_cast<int>(span);
  g.scatter_n = static_cast<int>(dst.size());
  for (size_t i = 0; i < dst.size(); ++i) g.scatter_dst[i] = reinterpret_cast<void*>(dst[i]);
  g.dst_ld = dst_ld; g.dst_stride = dst_stride; g.scatter_batch0 = static_cast<int>(batch0);
  g.err = err_ptr();
  return vagus::gemm_launch(g, stream());
}

// C (M x N) = A @ B^T with B's rows gathered from `srcs` (each `rows` x K,
// K contiguous, same row pitch) -- e.g. the row shards of a weight on the
// GPUs of a group through peer mappings (data pointers, as int64).
int64_t gemm_gather(Tensor A, bool a_mn, std::vector<int64_t> srcs, int64_t rows, int64_t ldb, Tensor C) {
  need_cuda(A, "A"); need_cuda(C, "C");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && A.dim() == 2 && A.stride(-1) == 1, "gemm_gather: A 2-D bf16");
  need_bf16_or_f32(C, "C");
  TORCH_CHECK(C.dim() == 2 && C.stride(-1) == 1, "gemm_gather: C 2-D, inner stride 1");
  TORCH_CHECK(!srcs.empty() && srcs.size() <= 8, "gemm_gather: 1..8 sources");
  vagus::GemmArgs g;
  g.a_mn = a_mn; g.b_mn = false;
  g.M = static_cast<int>(a_mn ? A.size(1) : A.size(0));
  g.K = static_cast<int>(a_mn ? A.size(0) : A.size(1));
  g.N = static_cast<int>(C.size(1));
  TORCH_CHECK(C.size(0) == g.M, "gemm_gather: C rows");
  g.A = A.data_ptr(); g.lda = A.stride(0);
  g.ldb = ldb;
  g.C = C.data_ptr(); g.ldc = C.stride(0); g.c_f32 = is_f32(C);
  g.split_k = 1;
  g.gather_n = static_cast<int>(srcs.size());
  g.gather_rows = static_cast<int>(rows);
  for (size_t i = 0; i < srcs.size(); ++i) g.gather_src[i] = reinterpret_cast<const void*>(srcs[i]);
  g.err = err_ptr();
  return vagus::gemm_launch(g, stream());
}

// ------------------------------------------------------------------ norms --
std::vector<Tensor> rmsnorm_fwd(Tensor x, Tensor gamma, double eps, bool out_f32) {
  need_cuda(x, "x"); need_bf16_or_f32(x, "x");
  TORCH_CHECK(x.is_contiguous() && gamma.is_contiguous() && is_f32(gamma), "rmsnorm: layout");
  const int D = static_cast<int>(x.size(-1));
  const int64_t rows = x.numel() / D;
  auto y = torch::empty(x.sizes(), x.options().dtype(out_f32 ? at::kFloat : at::kBFloat16));
  auto rstd = torch::empty({rows}, x.options().dtype(at::kFloat));
  check(vagus::rmsnorm_fwd(x.data_ptr(), is_f32(x), gamma.data_ptr<float>(), y.data_ptr(), out_f32,
                           rstd.data_ptr<float>(), rows, D, static_cast<float>(eps), stream()), "rmsnorm_fwd");
  return {y, rstd};
}

std::vector<Tensor> rmsnorm_bwd(Tensor dy, Tensor x, Tensor gamma, Tensor rstd, c10::optional<Tensor> dres,
                                bool dx_f32, bool want_bf16) {
  TORCH_CHECK(dy.is_contiguous() && x.is_contiguous(), "rmsnorm_bwd: layout");
  const int D = static_cast<int>(x.size(-1));
  const int64_t rows = x.numel() / D;
  auto dx = torch::empty(x.sizes(), x.options().dtype(dx_f32 ? at::kFloat : at::kBFloat16));
  auto dgamma = torch::zeros({D}, x.options().dtype(at::kFloat));
  const float* dr = nullptr;
  if (dres.has_value() && dres->defined()) {
    TORCH_CHECK(is_f32(*dres) && dres->is_contiguous(), "dres must be contiguous fp32");
    dr = dres->data_ptr<float>();
  }
  Tensor dx16;
  if (want_bf16) dx16 = torch::empty(x.sizes(), x.options().dtype(at::kBFloat16));
  check(vagus::rmsnorm_bwd(dy.data_ptr(), is_f32(dy), x.data_ptr(), is_f32(x), gamma.data_ptr<float>(),
                           rstd.data_ptr<float>(), dr, dx.data_ptr(), dx_f32, dgamma.data_ptr<float>(), rows, D,
                           stream(), want_bf16 ? dx16.data_ptr() : nullptr), "rmsnorm_bwd");
  if (want_bf16) return {dx, dgamma, dx16};
  return {dx, dgamma};
}

// o: (T, H, D) bf16 contiguous; g: (T, H*D) bf16 rows with unit inner stride
// (may be a column block of a wider matrix).
std::vector<Tensor> rmsnorm_gated_fwd(Tensor o, Tensor g, Tensor gamma, double eps, int64_t H) {
  TORCH_CHECK(o.is_contiguous() && o.scalar_type() == at::kBFloat16 && g.scalar_type() == at::kBFloat16 &&
              g.stride(-1) == 1 && g.dim() == 2, "rmsnorm_gated: bf16 inputs, g as (T, H*D) rows");
  const int D = static_cast<int>(o.size(-1));
  const int64_t rows = o.numel() / D;
  auto y = torch::empty_like(o);
  auto rstd = torch::empty({rows}, o.options().dtype(at::kFloat));
  check(vagus::rmsnorm_gated_fwd(o.data_ptr(), g.data_ptr(), g.stride(0), static_cast<int>(H),
                                 gamma.data_ptr<float>(), y.data_ptr(), 0, rstd.data_ptr<float>(), rows, D,
                                 static_cast<float>(eps), stream()), "rmsnorm_gated_fwd");
  return {y, rstd};
}

// dG is written into `dG` ((T, H*D) rows, possibly a column block).
std::vector<Tensor> rmsnorm_gated_bwd(Tensor dy, Tensor o, Tensor g, Tensor gamma, Tensor rstd, Tensor dG, int64_t H) {
  const int D = static_cast<int>(o.size(-1));
  const int64_t rows = o.numel() / D;
  auto dO = torch::empty_like(o);
  auto dgamma = torch::zeros({D}, o.options().dtype(at::kFloat));
  TORCH_CHECK(dG.stride(-1) == 1 && dG.dim() == 2, "dG layout");
  check(vagus::rmsnorm_gated_bwd(dy.contiguous().data_ptr(), o.data_ptr(), g.data_ptr(), g.stride(0),
                                 static_cast<int>(H), gamma.data_ptr<float>(), rstd.data_ptr<float>(), dO.data_ptr(),
                                 dG.data_ptr(), dG.stride(0), dgamma.data_ptr<float>(), rows, D, stream()),
        "rmsnorm_gated_bwd");
  return {dO, dgamma};
}

// Token pitch (elements) of a (B, L, H, D) tensor whose heads of one token are
// dense and whose tokens are evenly spaced (a column slice of a packed
// projection, for instance); -1 when the layout is not of that form.
int64_t token_pitch(const Tensor& t) {
  if (t.dim() != 4 || t.stride(3) != 1 || t.stride(2) != t.size(3)) return -1;
  if (t.size(0) > 1 && t.stride(0) != t.size(1) * t.stride(1)) return -1;
  return t.stride(1);
}

Tensor pitched(const Tensor& t) { return token_pitch(t) > 0 ? t : t.contiguous(); }

// x: (B, L, H, D) bf16 with a token pitch (dense or a column slice of a packed
// projection); cos/sin (L, D/2) fp32 or undefined.  y is dense.
std::vector<Tensor> qk_norm_rope_fwd(Tensor x, c10::optional<Tensor> gamma, c10::optional<Tensor> cosv,
                                     c10::optional<Tensor> sinv, double eps) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 4, "qk_norm_rope: (B,L,H,D) bf16");
  x = pitched(x);
  const int L = static_cast<int>(x.size(1)), H = static_cast<int>(x.size(2)), D = static_cast<int>(x.size(3));
  const int64_t rows = x.numel() / D;
  auto y = torch::empty(x.sizes(), x.options());
  auto rstd = torch::empty({rows}, x.options().dtype(at::kFloat));
  const bool hg = gamma.has_value() && gamma->defined(), hr = cosv.has_value() && cosv->defined();
  check(vagus::qk_norm_rope_fwd(x.data_ptr(), hg ? gamma->data_ptr<float>() : nullptr,
                                hr ? cosv->data_ptr<float>() : nullptr, hr ? sinv->data_ptr<float>() : nullptr,
                                y.data_ptr(), rstd.data_ptr<float>(), rows, L, H, D, static_cast<float>(eps),
                                token_pitch(x), 0, stream()),
        "qk_norm_rope_fwd");
  return {y, rstd};
}

// dy, x and dx_out may each carry a token pitch; dx is dense when dx_out is not given
std::vector<Tensor> qk_norm_rope_bwd(Tensor dy, Tensor x, c10::optional<Tensor> gamma, c10::optional<Tensor> cosv,
                                     c10::optional<Tensor> sinv, Tensor rstd, c10::optional<Tensor> dx_out) {
  dy = pitched(dy);
  x = pitched(x);
  TORCH_CHECK(dy.sizes() == x.sizes(), "qk_norm_rope_bwd: dy shaped like x");
  const int L = static_cast<int>(x.size(1)), H = static_cast<int>(x.size(2)), D = static_cast<int>(x.size(3));
  const int64_t rows = x.numel() / D;
  Tensor dx;
  if (dx_out.has_value() && dx_out->defined()) {
    dx = *dx_out;
    TORCH_CHECK(dx.sizes() == x.sizes() && dx.scalar_type() == at::kBFloat16 && token_pitch(dx) > 0,
                "qk_norm_rope_bwd: dx_out (B, L, H, D) bf16 with a token pitch");
  } else {
    dx = torch::empty(x.sizes(), x.options());
  }
  const bool hg = gamma.has_value() && gamma->defined(), hr = cosv.has_value() && cosv->defined();
  auto dgamma = torch::zeros({hg ? D : 0}, x.options().dtype(at::kFloat));
  check(vagus::qk_norm_rope_bwd(dy.data_ptr(), x.data_ptr(), hg ? gamma->data_ptr<float>() : nullptr,
                                hr ? cosv->data_ptr<float>() : nullptr, hr ? sinv->data_ptr<float>() : nullptr,
                                rstd.data_ptr<float>(), dx.data_ptr(), hg ? dgamma.data_ptr<float>() : nullptr, rows,
                                L, H, D, token_pitch(dy), token_pitch(x), token_pitch(dx), stream()),
        "qk_norm_rope_bwd");
  return {dx, dgamma};
}

// ------------------------------------------------------------ elementwise --
Tensor swiglu_fwd(Tensor u) {
  TORCH_CHECK(u.is_contiguous() && u.scalar_type() == at::kBFloat16, "swiglu: bf16 contiguous");
  const int F = static_cast<int>(u.size(-1) / 2);
  TORCH_CHECK(F % 2 == 0, "swiglu: hidden width must be even");
  auto sizes = u.sizes().vec();
  sizes.back() = F;
  auto s = torch::empty(sizes, u.options());
  check(vagus::swiglu_fwd(u.data_ptr(), s.data_ptr(), u.numel() / (2 * F), F, stream()), "swiglu_fwd");
  return s;
}

Tensor swiglu_bwd(Tensor ds, Tensor u) {
  ds = ds.contiguous();
  const int F = static_cast<int>(u.size(-1) / 2);
  auto du = torch::empty_like(u);
  check(vagus::swiglu_bwd(ds.data_ptr(), u.data_ptr(), du.data_ptr(), u.numel() / (2 * F), F, stream()),
        "swiglu_bwd");
  return du;
}

Tensor sigmoid_gate_fwd(Tensor x, Tensor g) {
  TORCH_CHECK(x.is_contiguous() && g.is_contiguous() && x.sizes() == g.sizes(), "sigmoid_gate: layout");
  auto y = torch::empty_like(x);
  check(vagus::sigmoid_gate_fwd(x.data_ptr(), g.data_ptr(), y.data_ptr(), x.numel(), stream()), "sigmoid_gate_fwd");
  return y;
}

std::vector<Tensor> sigmoid_gate_bwd(Tensor dy, Tensor x, Tensor g) {
  dy = dy.contiguous();
  auto dx = torch::empty_like(x), dg = torch::empty_like(g);
  check(vagus::sigmoid_gate_bwd(dy.data_ptr(), x.data_ptr(), g.data_ptr(), dx.data_ptr(), dg.data_ptr(), x.numel(),
                                stream()), "sigmoid_gate_bwd");
  return {dx, dg};
}

// logits (rows, V) bf16, overwritten with d(loss)/d(logits) * scale
std::vector<Tensor> softmax_ce(Tensor logits, Tensor targets, double scale, double z_coef) {
  TORCH_CHECK(logits.is_contiguous() && logits.scalar_type() == at::kBFloat16 && logits.dim() == 2, "softmax_ce");
  TORCH_CHECK(targets.scalar_type() == at::kLong && targets.is_contiguous(), "targets must be int64");
  const int64_t rows = logits.size(0);
  const int V = static_cast<int>(logits.size(1));
  auto loss = torch::empty({rows}, logits.options().dtype(at::kFloat));
  auto lse = torch::empty({rows}, logits.options().dtype(at::kFloat));
  check(vagus::softmax_ce(logits.data_ptr(), reinterpret_cast<const long long*>(targets.data_ptr<int64_t>()), loss.data_ptr<float>(),
                          lse.data_ptr<float>(), rows, V, static_cast<float>(scale), static_cast<float>(z_coef),
                          stream()), "softmax_ce");
  return {loss, lse};
}

Tensor embedding_fwd(Tensor W, Tensor tok, bool out_f32) {
  TORCH_CHECK(is_f32(W) && W.is_contiguous() && tok.scalar_type() == at::kLong, "embedding_fwd");
  tok = tok.contiguous();
  const int D = static_cast<int>(W.size(1));
  auto sizes = tok.sizes().vec();
  sizes.push_back(D);
  auto y = torch::empty(sizes, W.options().dtype(out_f32 ? at::kFloat : at::kBFloat16));
  check(vagus::embedding_fwd(W.data_ptr<float>(), reinterpret_cast<const long long*>(tok.data_ptr<int64_t>()), y.data_ptr(), out_f32, tok.numel(), D,
                             W.size(0), stream()), "embedding_fwd");
  return y;
}

void embedding_bwd(Tensor dy, Tensor tok, Tensor dW) {
  dy = dy.contiguous();
  tok = tok.contiguous();
  TORCH_CHECK(is_f32(dW) && dW.is_contiguous(), "embedding_bwd: fp32 dW");
  check(vagus::embedding_bwd(dy.data_ptr(), is_f32(dy), reinterpret_cast<const long long*>(tok.data_ptr<int64_t>()), dW.data_ptr<float>(), tok.numel(),
                             static_cast<int>(dW.size(1)), dW.size(0), stream()), "embedding_bwd");
}

void adamw_step(Tensor p, Tensor g, Tensor m, Tensor v, c10::optional<Tensor> shadow, double lr, double b1, double b2,
                double eps, double wd, int64_t step, double gscale) {
  TORCH_CHECK(is_f32(p) && is_f32(g) && is_f32(m) && is_f32(v) && p.is_contiguous() && g.is_contiguous(),
              "adamw: fp32 contiguous");
  const double bc1 = 1.0 - std::pow(b1, static_cast<double>(step));
  const double bc2 = 1.0 - std::pow(b2, static_cast<double>(step));
  void* sh = (shadow.has_value() && shadow->defined()) ? shadow->data_ptr() : nullptr;
  check(vagus::adamw_step(p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), sh,
                          p.numel(), static_cast<float>(lr), static_cast<float>(b1), static_cast<float>(b2),
                          static_cast<float>(eps), static_cast<float>(wd), static_cast<float>(bc1),
                          static_cast<float>(bc2), static_cast<float>(gscale), stream()), "adamw");
}

void muon_momentum(Tensor g, Tensor buf, Tensor upd, double mu, bool nesterov, double gscale) {
  TORCH_CHECK(is_f32(g) && is_f32(buf) && upd.scalar_type() == at::kBFloat16 && g.is_contiguous() &&
              buf.is_contiguous() && upd.is_contiguous(), "muon_momentum: layout");
  check(vagus::muon_momentum(g.data_ptr<float>(), buf.data_ptr<float>(), upd.data_ptr(), g.numel(),
                             static_cast<float>(mu), nesterov ? 1 : 0, static_cast<float>(gscale), stream()),
        "muon_momentum");
}

}  // namespace

void register_seq_ops(pybind11::module& m);   // bind_seq.cpp: conv, gates, gdr
void register_attn_ops(pybind11::module& m);  // bind_attn.cpp: flash attention
void register_comm_ops(pybind11::module& m);  // bind_comm.cpp: NVLink peer-to-peer collectives

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "vagus_b200 sm_100a kernels";
  m.def("error_word", &error_word, "device error word (bounded-wait timeouts); 0 = none");
  m.def("bounds_checked", []() { return !bounds_installers().empty(); },
        "True in the bounds-checked build (VAGUS_BOUNDS_CHECK=1)");
  m.def("reset_error", &reset_error);
  m.def("gemm_gather", &gemm_gather);
  m.def("gemm_scatter", &gemm_scatter);
  m.def("gemm", &gemm, "tcgen05 GEMM", py::arg("A"), py::arg("a_mn"), py::arg("B"), py::arg("b_mn"), py::arg("C"),
        py::arg("S") = py::none(), py::arg("alpha") = 1.0, py::arg("beta") = 0.0, py::arg("atomic") = false,
        py::arg("split_k") = 0, py::arg("block_n") = 0);
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("rmsnorm_gated_fwd", &rmsnorm_gated_fwd);
  m.def("rmsnorm_gated_bwd", &rmsnorm_gated_bwd);
  m.def("qk_norm_rope_fwd", &qk_norm_rope_fwd);
  m.def("qk_norm_rope_bwd", &qk_norm_rope_bwd, py::arg("dy"), py::arg("x"), py::arg("gamma"), py::arg("cosv"),
        py::arg("sinv"), py::arg("rstd"), py::arg("dx_out") = py::none());
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("sigmoid_gate_fwd", &sigmoid_gate_fwd);
  m.def("sigmoid_gate_bwd", &sigmoid_gate_bwd);
  m.def("softmax_ce", &softmax_ce);
  m.def("embedding_fwd", &embedding_fwd);
  m.def("embedding_bwd", &embedding_bwd);
  m.def("adamw_step", &adamw_step);
  m.def("muon_momentum", &muon_momentum);
  register_seq_ops(m);
  register_attn_ops(m);
  register_comm_ops(m);
}

// the error-word accessor shared with bind_seq.cpp
int* vagus_err_ptr() { return err_ptr(); }
