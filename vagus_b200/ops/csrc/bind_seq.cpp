// Bindings of the sequence-mixing kernels: short conv, gate activations,
// the gated delta-rule recurrence and its decode step.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "kernels.h"

int* vagus_device_error_ptr();   // bindings.cpp

namespace {

using torch::Tensor;

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check(int rc, const char* what) {
  TORCH_CHECK(rc == 0, "vagus_b200 kernel '", what, "' failed to launch (code ", rc, ")");
}

const float* fptr(const c10::optional<Tensor>& t) {
  return (t.has_value() && t->defined()) ? t->data_ptr<float>() : nullptr;
}

// x: (B, L, >=D) bf16 view with unit inner stride (row pitch x.stride(1));
// w: (D, 1, K) fp32.  Returns (y (B, L, D) bf16, rnorm (B, L, D/hd) fp32).
std::vector<Tensor> conv_silu_fwd(Tensor x, Tensor w, int64_t head_dim, bool l2norm) {
  TORCH_CHECK(x.dim() == 3 && x.stride(2) == 1 && x.scalar_type() == at::kBFloat16, "conv: (B,L,D) bf16 rows");
  TORCH_CHECK(x.stride(0) == x.size(1) * x.stride(1), "conv: batch stride must follow the row pitch");
  const int64_t B = x.size(0), L = x.size(1);
  const int D = static_cast<int>(w.size(0)), K = static_cast<int>(w.size(-1));
  auto y = torch::empty({B, L, D}, x.options());
  auto rn = torch::empty({B, L, l2norm ? D / head_dim : 0}, x.options().dtype(at::kFloat));
  auto wc = w.contiguous();
  check(vagus::conv_silu_fwd(x.data_ptr(), x.stride(1), wc.data_ptr<float>(), y.data_ptr(),
                             l2norm ? rn.data_ptr<float>() : nullptr, B, L, D, K, static_cast<int>(head_dim),
                             l2norm ? 1 : 0, stream()), "conv_silu_fwd");
  return {y, rn};
}

// dx is written into `dx` (a (B, L, >=D) view with its own row pitch); dw (D*K fp32) accumulated.
void conv_silu_bwd(Tensor dy, Tensor x, Tensor w, Tensor rnorm, Tensor dx, Tensor dw, int64_t head_dim, bool l2norm) {
  dy = dy.contiguous();
  TORCH_CHECK(dx.stride(2) == 1 && dx.stride(0) == dx.size(1) * dx.stride(1), "conv_bwd: dx layout");
  const int64_t B = x.size(0), L = x.size(1);
  const int D = static_cast<int>(w.size(0)), K = static_cast<int>(w.size(-1));
  auto wc = w.contiguous();
  check(vagus::conv_silu_bwd(dy.data_ptr(), x.data_ptr(), x.stride(1), wc.data_ptr<float>(),
                             l2norm ? rnorm.data_ptr<float>() : nullptr, dx.data_ptr(), dx.stride(1),
                             dw.data_ptr<float>(), B, L, D, K, static_cast<int>(head_dim), l2norm ? 1 : 0, stream()),
        "conv_silu_bwd");
}

// ab: (T, >=2H) bf16 rows -> g, beta (T, H) fp32
std::vector<Tensor> gdn_gates_fwd(Tensor ab, Tensor A_log, Tensor dt_bias, int64_t H) {
  TORCH_CHECK(ab.dim() == 2 && ab.stride(1) == 1, "gates: (T, 2H) rows");
  const int64_t T = ab.size(0);
  auto g = torch::empty({T, H}, ab.options().dtype(at::kFloat));
  auto beta = torch::empty({T, H}, ab.options().dtype(at::kFloat));
  check(vagus::gdn_gates_fwd(ab.data_ptr(), ab.stride(0), A_log.data_ptr<float>(), dt_bias.data_ptr<float>(),
                             g.data_ptr<float>(), beta.data_ptr<float>(), T, static_cast<int>(H), stream()),
        "gdn_gates_fwd");
  return {g, beta};
}

// dab: (T, 2H) output rows with the same row pitch as ab (e.g. the a|b
// columns of the packed projection gradient).
std::vector<Tensor> gdn_gates_bwd(Tensor dg, Tensor dbeta, Tensor ab, Tensor A_log, Tensor dt_bias, int64_t H,
                                  Tensor dab) {
  const int64_t T = ab.size(0);
  TORCH_CHECK(dab.stride(0) == ab.stride(0) && dab.stride(1) == 1, "gates_bwd: dab must share ab's row pitch");
  auto dA = torch::zeros({H}, ab.options().dtype(at::kFloat));
  auto ddt = torch::zeros({H}, ab.options().dtype(at::kFloat));
  dg = dg.contiguous();
  dbeta = dbeta.contiguous();
  check(vagus::gdn_gates_bwd(dg.data_ptr<float>(), dbeta.data_ptr<float>(), ab.data_ptr(), ab.stride(0),
                             A_log.data_ptr<float>(), dt_bias.data_ptr<float>(), dab.data_ptr(), dA.data_ptr<float>(),
                             ddt.data_ptr<float>(), T, static_cast<int>(H), stream()), "gdn_gates_bwd");
  return {dA, ddt};
}

// Recurrence forward: returns (O, V'^T, states, S_out).  The per-chunk entry
// states (bf16, stored transposed as S_n^T (BH, N, DV, DK)) are always
// produced: the output stage reads them.  V'^T is (BH, N, DV, 64).
std::vector<Tensor> gdr_rec_fwd(Tensor W, Tensor Qh, Tensor Kt, Tensor A, Tensor U, Tensor gC,
                                c10::optional<Tensor> S0, bool need_states, int64_t H) {
  (void)need_states;
  gC = gC.contiguous();
  const int64_t BH = W.size(0);
  TORCH_CHECK(H > 0 && BH % H == 0, "gdr_rec_fwd: heads must divide B*H");
  const int N = static_cast<int>(W.size(1)), DK = static_cast<int>(W.size(3)), DV = static_cast<int>(U.size(3));
  TORCH_CHECK(W.size(2) == 64, "gdr: chunk size 64");
  for (auto* t : {&W, &Qh, &Kt, &A, &U}) TORCH_CHECK(t->is_contiguous() && t->scalar_type() == at::kBFloat16, "gdr: bf16");
  auto O = torch::empty({BH / H, static_cast<int64_t>(N) * 64, H, DV}, U.options());   // token-major
  auto Vp = torch::empty({BH, N, DV, 64}, U.options());           // V'^T per chunk (value-major)
  auto states = torch::empty({BH, N, DV, DK}, W.options());       // S_n^T per chunk (value-major)
  auto S_out = torch::empty({BH, DK, DV}, W.options().dtype(at::kFloat));
  vagus::GdrRecArgs a{W.data_ptr(), Qh.data_ptr(), Kt.data_ptr(), A.data_ptr(), U.data_ptr(),
                      gC.data_ptr<float>(), fptr(S0), O.data_ptr(), Vp.data_ptr(),
                      states.data_ptr(), S_out.data_ptr<float>(), BH, N, DK, DV, static_cast<int>(H),
                      vagus_device_error_ptr()};
  a.gvec = gC.dim() == 3 ? 1 : 0;
  TORCH_CHECK(gC.scalar_type() == at::kFloat && gC.size(0) == BH && gC.size(1) == N &&
                  (gC.dim() == 2 || (gC.dim() == 3 && gC.size(2) == DK)),
              "gdr_rec_fwd: gC (BH, N) or (BH, N, DK) fp32");
  check(vagus::gdr_rec_fwd(a, stream()), "gdr_rec_fwd");
  return {O, Vp, states, S_out};
}

// Recurrence backward: returns (dW, dQh, dKt (bf16), dA (fp32), dU (bf16), dgC (gC's shape), dS0)
// dO: token-major (B, L, H, DV) bf16
std::vector<Tensor> gdr_rec_bwd(Tensor W, Tensor Qh, Tensor Kt, Tensor A, Tensor Vp, Tensor gC, Tensor states,
                                Tensor dO, c10::optional<Tensor> dS_final, bool need_dS0) {
  gC = gC.contiguous();
  const int64_t BH = W.size(0);
  const int N = static_cast<int>(W.size(1)), DK = static_cast<int>(W.size(3)), DV = static_cast<int>(Vp.size(2));
  TORCH_CHECK(Vp.size(3) == 64 && states.size(2) == DV && states.size(3) == DK, "gdr_rec_bwd: value-major V', states");
  TORCH_CHECK(states.scalar_type() == at::kBFloat16 && states.is_contiguous(), "gdr_rec_bwd: bf16 states");
  dO = dO.contiguous();
  TORCH_CHECK(dO.dim() == 4 && dO.size(3) == DV && dO.scalar_type() == at::kBFloat16, "gdr_rec_bwd: dO (B, L, H, DV) bf16");
  const int H = static_cast<int>(dO.size(2));
  auto f32 = W.options().dtype(at::kFloat);
  auto bf = W.options();
  auto dW = torch::empty({BH, N, 64, DK}, bf);
  auto dQh = torch::empty({BH, N, 64, DK}, bf);
  auto dKt = torch::empty({BH, N, 64, DK}, bf);
  auto dA = torch::empty({BH, N, 64, 64}, f32);
  auto dU = torch::empty({BH, N, 64, DV}, bf);
  auto dgC = torch::zeros(gC.sizes(), f32);
  auto dS0 = torch::empty({need_dS0 ? BH : 0, DK, DV}, f32);
  auto dstates = torch::empty({BH, N, DV, DK}, bf);            // value-major, like the forward snapshots
  vagus::GdrRecBwdArgs a;
  a.f = vagus::GdrRecArgs{W.data_ptr(), Qh.data_ptr(), Kt.data_ptr(), A.data_ptr(), nullptr,
                          gC.data_ptr<float>(), nullptr, nullptr, Vp.data_ptr(), states.data_ptr(),
                          nullptr, BH, N, DK, DV, H};
  a.dO = dO.data_ptr();
  a.dS_final = fptr(dS_final);
  a.dW = dW.data_ptr(); a.dQh = dQh.data_ptr(); a.dKt = dKt.data_ptr(); a.dA = dA.data_ptr<float>();
  a.dU = dU.data_ptr(); a.dgC = dgC.data_ptr<float>(); a.dS0 = need_dS0 ? dS0.data_ptr<float>() : nullptr;
  a.dstates = dstates.data_ptr();
  a.f.gvec = gC.dim() == 3 ? 1 : 0;
  a.f.err = vagus_device_error_ptr();
  TORCH_CHECK(gC.scalar_type() == at::kFloat && (gC.dim() == 2 || (gC.dim() == 3 && gC.size(2) == DK)),
              "gdr_rec_bwd: gC (BH, N) or (BH, N, DK) fp32");
  check(vagus::gdr_rec_bwd(a, stream()), "gdr_rec_bwd");
  return {dW, dQh, dKt, dA, dU, dgC, dS0};
}

// Intra-chunk stage.  q, k (B, L, H, DK), v (B, L, H, DV) bf16 contiguous;
// g, beta (B, L, H) fp32.  Returns W, Qh, Kt, A, U (chunk-major bf16), gC.
std::vector<Tensor> gdr_intra_fwd(Tensor q, Tensor k, Tensor v, Tensor g, Tensor beta, double scale) {
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous() && q.scalar_type() == at::kBFloat16,
              "gdr_intra: contiguous bf16 q/k/v");
  const int64_t B = q.size(0), L = q.size(1);
  const int H = static_cast<int>(q.size(2)), DK = static_cast<int>(q.size(3)), DV = static_cast<int>(v.size(3));
  TORCH_CHECK(L % 64 == 0, "gdr_intra: L must be a multiple of 64");
  const int64_t N = L / 64;
  auto bf = q.options();
  auto W = torch::empty({B * H, N, 64, DK}, bf), Qh = torch::empty({B * H, N, 64, DK}, bf);
  auto Kt = torch::empty({B * H, N, 64, DK}, bf), A = torch::empty({B * H, N, 64, 64}, bf);
  auto U = torch::empty({B * H, N, 64, DV}, bf);
  auto gC = torch::empty({B * H, N}, q.options().dtype(at::kFloat));
  auto gc = g.contiguous(), bc = beta.contiguous();
  vagus::GdrIntraArgs a{q.data_ptr(), k.data_ptr(), v.data_ptr(), gc.data_ptr<float>(), bc.data_ptr<float>(),
                        W.data_ptr(), Qh.data_ptr(), Kt.data_ptr(), A.data_ptr(), U.data_ptr(), gC.data_ptr<float>(),
                        B, L, H, DK, DV, static_cast<float>(scale)};
  check(vagus::gdr_intra_fwd(a, stream()), "gdr_intra_fwd");
  return {W, Qh, Kt, A, U, gC};
}

// Returns dq, dk, dv (token-major bf16), dg, dbeta (fp32).
std::vector<Tensor> gdr_intra_bwd(Tensor q, Tensor k, Tensor v, Tensor g, Tensor beta, Tensor dW, Tensor dQh,
                                  Tensor dKt, Tensor dA, Tensor dU, Tensor dgC, double scale) {
  const int64_t B = q.size(0), L = q.size(1);
  const int H = static_cast<int>(q.size(2)), DK = static_cast<int>(q.size(3)), DV = static_cast<int>(v.size(3));
  auto dq = torch::empty_like(q), dk = torch::empty_like(k), dv = torch::empty_like(v);
  auto dg = torch::empty({B, L, H}, q.options().dtype(at::kFloat));
  auto db = torch::empty({B, L, H}, q.options().dtype(at::kFloat));
  auto gc = g.contiguous(), bc = beta.contiguous();
  vagus::GdrIntraBwdArgs a;
  a.f = vagus::GdrIntraArgs{q.data_ptr(), k.data_ptr(), v.data_ptr(), gc.data_ptr<float>(), bc.data_ptr<float>(),
                            nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, B, L, H, DK, DV,
                            static_cast<float>(scale)};
  TORCH_CHECK(dW.scalar_type() == at::kBFloat16 && dQh.scalar_type() == at::kBFloat16 &&
              dKt.scalar_type() == at::kBFloat16, "gdr_intra_bwd: bf16 dW / dQh / dKt");
  a.dW = dW.data_ptr(); a.dQh = dQh.data_ptr(); a.dKt = dKt.data_ptr(); a.dA = dA.data_ptr<float>();
  a.dU = dU.data_ptr(); a.dgC = dgC.data_ptr<float>();
  a.dq = dq.data_ptr(); a.dk = dk.data_ptr(); a.dv = dv.data_ptr(); a.dg = dg.data_ptr<float>(); a.dbeta = db.data_ptr<float>();
  check(vagus::gdr_intra_bwd(a, stream()), "gdr_intra_bwd");
  return {dq, dk, dv, dg, db};
}

// q, k (BH, dk) bf16, v (BH, dv) bf16, g, beta (BH) fp32, S (BH, dk, dv) fp32 in place -> o (BH, dv)
Tensor gdr_decode(Tensor q, Tensor k, Tensor v, Tensor g, Tensor beta, Tensor S, double scale) {
  const int64_t BH = S.size(0);
  const int dk = static_cast<int>(S.size(1)), dv = static_cast<int>(S.size(2));
  TORCH_CHECK(S.is_contiguous() && S.scalar_type() == at::kFloat, "gdr_decode: fp32 contiguous state");
  auto qc = q.contiguous(), kc = k.contiguous(), vc = v.contiguous();
  auto gc = g.contiguous(), bc = beta.contiguous();
  auto o = torch::empty({BH, dv}, q.options());
  check(vagus::gdr_decode(qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), gc.data_ptr<float>(), bc.data_ptr<float>(),
                          S.data_ptr<float>(), o.data_ptr(), BH, dk, dv, static_cast<float>(scale), stream()),
        "gdr_decode");
  return o;
}

// Gated inner products of the per-channel-gate chunk form (kda.cu).
// Q, K, G: (..., 64, dk) fp32 contiguous -> (Aqk, Akk) (..., 64, 64) fp32.
std::vector<Tensor> kda_gated_fwd(Tensor Q, Tensor K, Tensor G) {
  for (auto* t : {&Q, &K, &G})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->sizes() == Q.sizes(),
                "kda_gated_fwd: Q, K, G (..., 64, dk) fp32 contiguous");
  TORCH_CHECK(Q.dim() >= 2 && Q.size(-2) == 64, "kda_gated_fwd: 64-token chunks");
  const int dk = static_cast<int>(Q.size(-1));
  const long long chunks = Q.numel() / (64LL * dk);
  auto shape = Q.sizes().vec();
  shape.back() = 64;
  auto Aqk = torch::empty(shape, Q.options()), Akk = torch::empty(shape, Q.options());
  check(vagus::kda_gated_fwd(Q.data_ptr<float>(), K.data_ptr<float>(), G.data_ptr<float>(), Aqk.data_ptr<float>(),
                             Akk.data_ptr<float>(), chunks, dk, stream()), "kda_gated_fwd");
  return {Aqk, Akk};
}

// -> (dQ, dK, dG) (..., 64, dk) fp32
std::vector<Tensor> kda_gated_bwd(Tensor Q, Tensor K, Tensor G, Tensor dAqk, Tensor dAkk) {
  dAqk = dAqk.contiguous().to(at::kFloat);
  dAkk = dAkk.contiguous().to(at::kFloat);
  const int dk = static_cast<int>(Q.size(-1));
  const long long chunks = Q.numel() / (64LL * dk);
  TORCH_CHECK(dAqk.numel() == chunks * 64 * 64 && dAkk.numel() == chunks * 64 * 64, "kda_gated_bwd: dA shapes");
  auto dQ = torch::empty_like(Q), dK = torch::empty_like(K), dG = torch::empty_like(G);
  check(vagus::kda_gated_bwd(Q.data_ptr<float>(), K.data_ptr<float>(), G.data_ptr<float>(), dAqk.data_ptr<float>(),
                             dAkk.data_ptr<float>(), dQ.data_ptr<float>(), dK.data_ptr<float>(), dG.data_ptr<float>(),
                             chunks, dk, stream()), "kda_gated_bwd");
  return {dQ, dK, dG};
}

// Per-channel-gate intra-chunk stage (kda_intra.cu).  q, k (B, L, H, DK), v
// (B, L, H, DV) bf16; g (B, L, H, DK), beta (B, L, H) fp32; L a multiple of 64.
// -> (W, Qh, Kt, A, U, gC), chunk-major (B * H, N, 64, .).
std::vector<Tensor> kda_intra_fwd(Tensor q, Tensor k, Tensor v, Tensor g, Tensor beta, double scale) {
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous() && g.is_contiguous() &&
                  beta.is_contiguous() && q.scalar_type() == at::kBFloat16 && g.scalar_type() == at::kFloat &&
                  beta.scalar_type() == at::kFloat,
              "kda_intra_fwd: contiguous bf16 q / k / v, fp32 g / beta");
  const int B = q.size(0), L = q.size(1), H = q.size(2), DK = q.size(3), DV = v.size(3);
  TORCH_CHECK(L % 64 == 0 && k.sizes() == q.sizes() && g.sizes() == q.sizes() && v.size(1) == L &&
                  beta.numel() == (long long)B * L * H,
              "kda_intra_fwd: q / k / g (B, L, H, dk), v (B, L, H, dv), beta (B, L, H), L a multiple of 64");
  const int N = L / 64;
  auto bf = q.options();
  auto W = torch::empty({B * H, N, 64, DK}, bf), Qh = torch::empty_like(W), Kt = torch::empty_like(W);
  auto A = torch::empty({B * H, N, 64, 64}, bf), U = torch::empty({B * H, N, 64, DV}, bf);
  auto gC = torch::empty({B * H, N, DK}, g.options());
  check(vagus::kda_intra_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr<float>(), beta.data_ptr<float>(),
                             W.data_ptr(), Qh.data_ptr(), Kt.data_ptr(), A.data_ptr(), U.data_ptr(),
                             gC.data_ptr<float>(), B, L, H, DK, DV, static_cast<float>(scale), stream()),
        "kda_intra_fwd");
  return {W, Qh, Kt, A, U, gC};
}

// KDA gates: f (T, H dk) bf16 view (inner stride 1), b (T, H) bf16 view -> (g (T, H dk), beta (T, H)) fp32
std::vector<Tensor> kda_gates_fwd(Tensor f, Tensor b, Tensor A_log, Tensor dt_bias, int64_t H, int64_t dk) {
  TORCH_CHECK(f.dim() == 2 && b.dim() == 2 && f.stride(1) == 1 && b.stride(1) == 1 && f.size(1) == H * dk &&
                  b.size(1) == H && f.size(0) == b.size(0) && f.scalar_type() == at::kBFloat16 &&
                  b.scalar_type() == at::kBFloat16,
              "kda_gates_fwd: f (T, H dk), b (T, H) bf16 row views");
  A_log = A_log.to(at::kFloat).contiguous();
  dt_bias = dt_bias.to(at::kFloat).contiguous();
  const long long T = f.size(0);
  auto g = torch::empty({T, H * dk}, f.options().dtype(at::kFloat));
  auto beta = torch::empty({T, H}, f.options().dtype(at::kFloat));
  check(vagus::kda_gates_fwd(f.data_ptr(), f.stride(0), b.data_ptr(), b.stride(0), A_log.data_ptr<float>(),
                             dt_bias.data_ptr<float>(), g.data_ptr<float>(), beta.data_ptr<float>(), T,
                             static_cast<int>(H), static_cast<int>(dk), stream()),
        "kda_gates_fwd");
  return {g, beta};
}

// -> (dA_log (H), ddt_bias (H dk)); df, db written into the given bf16 views
std::vector<Tensor> kda_gates_bwd(Tensor dg, Tensor dbeta, Tensor f, Tensor b, Tensor A_log, Tensor dt_bias, Tensor df,
                                  Tensor db, int64_t H, int64_t dk) {
  dg = dg.contiguous().to(at::kFloat);
  dbeta = dbeta.contiguous().to(at::kFloat);
  const long long T = f.size(0);
  TORCH_CHECK(dg.numel() == T * H * dk && dbeta.numel() == T * H && df.stride(1) == 1 && db.stride(1) == 1 &&
                  df.size(0) == T && df.size(1) == H * dk && db.size(1) == H,
              "kda_gates_bwd: shapes");
  A_log = A_log.to(at::kFloat).contiguous();
  dt_bias = dt_bias.to(at::kFloat).contiguous();
  auto dA = torch::zeros({H}, dg.options());
  auto ddt = torch::zeros({H * dk}, dg.options());
  check(vagus::kda_gates_bwd(dg.data_ptr<float>(), dbeta.data_ptr<float>(), f.data_ptr(), f.stride(0), b.data_ptr(),
                             b.stride(0), A_log.data_ptr<float>(), dt_bias.data_ptr<float>(), df.data_ptr(),
                             df.stride(0), db.data_ptr(), db.stride(0), dA.data_ptr<float>(), ddt.data_ptr<float>(), T,
                             static_cast<int>(H), static_cast<int>(dk), stream()),
        "kda_gates_bwd");
  return {dA, ddt};
}

// -> (dq, dk, dv, dg, dbeta), token-major like the inputs.
std::vector<Tensor> kda_intra_bwd(Tensor q, Tensor k, Tensor v, Tensor g, Tensor beta, Tensor dW, Tensor dQh,
                                  Tensor dKt, Tensor dA, Tensor dU, Tensor dgC, double scale) {
  dW = dW.contiguous(); dQh = dQh.contiguous(); dKt = dKt.contiguous(); dU = dU.contiguous();
  dA = dA.contiguous().to(at::kFloat);
  dgC = dgC.contiguous().to(at::kFloat);
  TORCH_CHECK(dW.scalar_type() == at::kBFloat16 && dQh.scalar_type() == at::kBFloat16 &&
                  dKt.scalar_type() == at::kBFloat16 && dU.scalar_type() == at::kBFloat16,
              "kda_intra_bwd: bf16 dW / dQh / dKt / dU");
  const int B = q.size(0), L = q.size(1), H = q.size(2), DK = q.size(3), DV = v.size(3);
  TORCH_CHECK(L % 64 == 0 && dW.numel() == q.numel() && dQh.numel() == q.numel() && dKt.numel() == q.numel() &&
                  dU.numel() == v.numel() && dA.numel() == (long long)B * H * L * 64 &&
                  dgC.numel() == (long long)B * H * (L / 64) * DK,
              "kda_intra_bwd: gradient shapes do not match the forward's outputs");
  auto dq = torch::empty_like(q), dk = torch::empty_like(k), dv = torch::empty_like(v);
  auto dg = torch::empty_like(g), dbeta = torch::empty_like(beta);
  vagus::KdaIntraBwdArgs a;
  a.q = q.data_ptr(); a.k = k.data_ptr(); a.v = v.data_ptr(); a.g = g.data_ptr<float>();
  a.beta = beta.data_ptr<float>(); a.dW = dW.data_ptr(); a.dQh = dQh.data_ptr(); a.dKt = dKt.data_ptr();
  a.dU = dU.data_ptr(); a.dA = dA.data_ptr<float>(); a.dgC = dgC.data_ptr<float>();
  a.dq = dq.data_ptr(); a.dk = dk.data_ptr(); a.dv = dv.data_ptr(); a.dg = dg.data_ptr<float>();
  a.dbeta = dbeta.data_ptr<float>();
  a.B = B; a.L = L; a.H = H; a.DK = DK; a.DV = DV; a.scale = static_cast<float>(scale);
  check(vagus::kda_intra_bwd(a, stream()), "kda_intra_bwd");
  return {dq, dk, dv, dg, dbeta};
}

// Mobius-map scan (mobius.cu).  A, B, C, D: (batch, L, R) fp32; x0: (batch, R).
Tensor mobius_fwd(Tensor A, Tensor B, Tensor C, Tensor D, Tensor x0) {
  for (auto* t : {&A, &B, &C, &D})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->dim() == 3 &&
                    t->sizes() == A.sizes(),
                "mobius_fwd: A, B, C, D (batch, L, R) fp32 contiguous");
  TORCH_CHECK(x0.is_cuda() && x0.scalar_type() == at::kFloat && x0.is_contiguous() && x0.dim() == 2 &&
                  x0.size(0) == A.size(0) && x0.size(1) == A.size(2),
              "mobius_fwd: x0 (batch, R) fp32 contiguous");
  TORCH_CHECK(A.size(0) <= 65535, "mobius_fwd: batch <= 65535");
  auto X = torch::empty_like(A);
  check(vagus::mobius_fwd(A.data_ptr<float>(), B.data_ptr<float>(), C.data_ptr<float>(), D.data_ptr<float>(),
                          x0.data_ptr<float>(), X.data_ptr<float>(), static_cast<int>(A.size(0)),
                          static_cast<int>(A.size(1)), static_cast<int>(A.size(2)), stream()),
        "mobius_fwd");
  return X;
}

// -> (gA, gB, gC, gD, gx0)
std::vector<Tensor> mobius_bwd(Tensor A, Tensor B, Tensor C, Tensor D, Tensor x0, Tensor X, Tensor gO) {
  gO = gO.contiguous().to(at::kFloat);
  TORCH_CHECK(X.sizes() == A.sizes() && gO.sizes() == A.sizes() && X.is_contiguous(), "mobius_bwd: shapes");
  auto gA = torch::empty_like(A), gB = torch::empty_like(A), gC = torch::empty_like(A), gD = torch::empty_like(A);
  auto gx0 = torch::empty_like(x0);
  check(vagus::mobius_bwd(A.data_ptr<float>(), B.data_ptr<float>(), C.data_ptr<float>(), D.data_ptr<float>(),
                          x0.data_ptr<float>(), X.data_ptr<float>(), gO.data_ptr<float>(), gA.data_ptr<float>(),
                          gB.data_ptr<float>(), gC.data_ptr<float>(), gD.data_ptr<float>(), gx0.data_ptr<float>(),
                          static_cast<int>(A.size(0)), static_cast<int>(A.size(1)), static_cast<int>(A.size(2)),
                          stream()),
        "mobius_bwd");
  return {gA, gB, gC, gD, gx0};
}

}  // namespace

void register_seq_ops(pybind11::module& m) {
  m.def("mobius_fwd", &mobius_fwd);
  m.def("mobius_bwd", &mobius_bwd);
  m.def("kda_gated_fwd", &kda_gated_fwd);
  m.def("kda_gated_bwd", &kda_gated_bwd);
  m.def("conv_silu_fwd", &conv_silu_fwd);
  m.def("conv_silu_bwd", &conv_silu_bwd);
  m.def("gdn_gates_fwd", &gdn_gates_fwd);
  m.def("gdn_gates_bwd", &gdn_gates_bwd);
  m.def("gdr_rec_fwd", &gdr_rec_fwd);
  m.def("gdr_rec_bwd", &gdr_rec_bwd);
  m.def("gdr_decode", &gdr_decode);
  m.def("gdr_intra_fwd", &gdr_intra_fwd);
  m.def("gdr_intra_bwd", &gdr_intra_bwd);
  m.def("kda_intra_fwd", &kda_intra_fwd);
  m.def("kda_gates_fwd", &kda_gates_fwd);
  m.def("kda_gates_bwd", &kda_gates_bwd);
  m.def("kda_intra_bwd", &kda_intra_bwd);
  m.def("gdr_intra_set_trace", [](c10::optional<Tensor> buf) {
    if (buf) TORCH_CHECK(buf->is_cuda() && buf->numel() >= 8 && buf->element_size() == 8, "gdr_intra_set_trace: 8 x u64");
    vagus::gdr_intra_set_trace(buf ? reinterpret_cast<unsigned long long*>(buf->data_ptr()) : nullptr);
  });
  // buf: int64 device tensor of 32 entries, or None
  m.def("kda_set_trace", [](c10::optional<Tensor> buf) {
    if (buf) TORCH_CHECK(buf->is_cuda() && buf->numel() >= 32 && buf->element_size() == 8, "kda_set_trace: 32 x u64");
    vagus::kda_set_trace(buf ? reinterpret_cast<unsigned long long*>(buf->data_ptr()) : nullptr);
  });
}
