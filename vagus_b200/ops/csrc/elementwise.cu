// Memory-bound element-wise kernels: SwiGLU, sigmoid output gate, the row-wise
// softmax cross-entropy of the fused linear-CE path, embedding gradient,
// fused AdamW and the Muon momentum update.  All vectorised over 16-byte
// accesses where the shapes allow.
#include "common.cuh"
#include "kernels.h"

namespace vagus {
namespace {

// ---------------------------------------------------------------- SwiGLU --
// u: (rows, 2F) bf16 = [x1 | gate];  s = silu(x1) * gate : (rows, F)

__global__ void swiglu_fwd_k(const __nv_bfloat16* __restrict__ u, __nv_bfloat16* __restrict__ s, long long rows,
                             int F) {
  const long long n2 = rows * (long long)(F / 2);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n2; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / (F / 2);
    const int c = static_cast<int>(i - r * (F / 2)) * 2;
    const uint32_t a = *reinterpret_cast<const uint32_t*>(u + r * 2 * F + c);
    const uint32_t g = *reinterpret_cast<const uint32_t*>(u + r * 2 * F + F + c);
    const float2 af = unpack_bf16x2(a), gf = unpack_bf16x2(g);
    *reinterpret_cast<uint32_t*>(s + r * F + c) = pack_bf16x2(silu_f(af.x) * gf.x, silu_f(af.y) * gf.y);
  }
}

__global__ void swiglu_bwd_k(const __nv_bfloat16* __restrict__ ds, const __nv_bfloat16* __restrict__ u,
                             __nv_bfloat16* __restrict__ du, long long rows, int F) {
  const long long n2 = rows * (long long)(F / 2);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n2; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / (F / 2);
    const int c = static_cast<int>(i - r * (F / 2)) * 2;
    const float2 a = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(u + r * 2 * F + c));
    const float2 g = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(u + r * 2 * F + F + c));
    const float2 d = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(ds + r * F + c));
    const float sa = sigmoid_f(a.x), sb = sigmoid_f(a.y);
    const float da0 = d.x * g.x * sa * (1.f + a.x * (1.f - sa));
    const float da1 = d.y * g.y * sb * (1.f + a.y * (1.f - sb));
    const float dg0 = d.x * a.x * sa, dg1 = d.y * a.y * sb;
    *reinterpret_cast<uint32_t*>(du + r * 2 * F + c) = pack_bf16x2(da0, da1);
    *reinterpret_cast<uint32_t*>(du + r * 2 * F + F + c) = pack_bf16x2(dg0, dg1);
  }
}

// 16-byte version (8 features per thread, 32-bit indexing) for F % 8 == 0
// and rows * F / 8 < 2^31: the element-pair kernels above spend most of their
// issue slots on 64-bit index division.
__global__ void swiglu_fwd_v8(const __nv_bfloat16* __restrict__ u, __nv_bfloat16* __restrict__ s, unsigned n8,
                              unsigned f8) {
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += gridDim.x * blockDim.x) {
    const unsigned r = i / f8, c = (i - r * f8) * 8;
    const size_t F = size_t(f8) * 8;
    const uint4 a = *reinterpret_cast<const uint4*>(u + r * 2 * F + c);
    const uint4 g = *reinterpret_cast<const uint4*>(u + r * 2 * F + F + c);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, gw[4] = {g.x, g.y, g.z, g.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 af = unpack_bf16x2(aw[j]), gf = unpack_bf16x2(gw[j]);
      o[j] = pack_bf16x2(silu_f(af.x) * gf.x, silu_f(af.y) * gf.y);
    }
    *reinterpret_cast<uint4*>(s + r * F + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void swiglu_bwd_v8(const __nv_bfloat16* __restrict__ ds, const __nv_bfloat16* __restrict__ u,
                              __nv_bfloat16* __restrict__ du, unsigned n8, unsigned f8) {
  for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += gridDim.x * blockDim.x) {
    const unsigned r = i / f8, c = (i - r * f8) * 8;
    const size_t F = size_t(f8) * 8;
    const uint4 a = *reinterpret_cast<const uint4*>(u + r * 2 * F + c);
    const uint4 g = *reinterpret_cast<const uint4*>(u + r * 2 * F + F + c);
    const uint4 d = *reinterpret_cast<const uint4*>(ds + r * F + c);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, gw[4] = {g.x, g.y, g.z, g.w}, dw[4] = {d.x, d.y, d.z, d.w};
    uint32_t oa[4], og[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 af = unpack_bf16x2(aw[j]), gf = unpack_bf16x2(gw[j]), df = unpack_bf16x2(dw[j]);
      const float sa = sigmoid_f(af.x), sb = sigmoid_f(af.y);
      oa[j] = pack_bf16x2(df.x * gf.x * sa * (1.f + af.x * (1.f - sa)), df.y * gf.y * sb * (1.f + af.y * (1.f - sb)));
      og[j] = pack_bf16x2(df.x * af.x * sa, df.y * af.y * sb);
    }
    *reinterpret_cast<uint4*>(du + r * 2 * F + c) = make_uint4(oa[0], oa[1], oa[2], oa[3]);
    *reinterpret_cast<uint4*>(du + r * 2 * F + F + c) = make_uint4(og[0], og[1], og[2], og[3]);
  }
}

bool swiglu_v8_ok(const void* a, const void* b, const void* c, long long rows, int F) {
  auto al = [](const void* p) { return p == nullptr || reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  return F % 8 == 0 && rows * (long long)(F / 8) < (1LL << 31) && al(a) && al(b) && al(c);
}

// ------------------------------------------------------- sigmoid gate --
// y = x * sigmoid(g), all (n) bf16

__global__ void sgate_fwd_k(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ g,
                            __nv_bfloat16* __restrict__ y, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    y[i] = f2bf(bf2f(x[i]) * sigmoid_f(bf2f(g[i])));
}

__global__ void sgate_bwd_k(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                            const __nv_bfloat16* __restrict__ g, __nv_bfloat16* __restrict__ dx,
                            __nv_bfloat16* __restrict__ dg, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float s = sigmoid_f(bf2f(g[i]));
    const float d = bf2f(dy[i]);
    dx[i] = f2bf(d * s);
    dg[i] = f2bf(d * bf2f(x[i]) * s * (1.f - s));
  }
}

// --------------------------------------------------------- softmax CE --
// One CTA per row of bf16 logits (rows, V).  Writes per-row lse and loss
// (lse - logit[target]) and overwrites the logits with
//     d = scale * (softmax - onehot) + scale * 2 z_coef lse * softmax.
// Rows whose target is < 0 are ignored (loss 0, gradient 0).  A target >= V
// is out of range: the row is ignored the same way (the logits row is never
// read past its end) and, when `status` is given, kErrBadTarget is recorded
// there.

constexpr int CE_THREADS = 512;

__global__ void __launch_bounds__(CE_THREADS) softmax_ce_k(__nv_bfloat16* __restrict__ logits,
                                                           const long long* __restrict__ targets,
                                                           float* __restrict__ loss, float* __restrict__ lse_out,
                                                           int V, float scale, float z_coef, int* status) {
  __shared__ float red_m[CE_THREADS / 32], red_s[CE_THREADS / 32];
  __shared__ float bc[2];
  const long long r = blockIdx.x;
  __nv_bfloat16* row = logits + r * V;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // online max / sum, 8 bf16 per 16-byte load
  float m = -INFINITY, s = 0.f;
  const int V8 = V / 8;
  for (int i = threadIdx.x; i < V8; i += CE_THREADS) {
    const uint4 t = reinterpret_cast<const uint4*>(row)[i];
    const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(w[j]);
      const float mx = fmaxf(f.x, f.y);
      if (mx > m) { s *= __expf(m - mx); m = mx; }
      s += __expf(f.x - m) + __expf(f.y - m);
    }
  }
  for (int i = V8 * 8 + threadIdx.x; i < V; i += CE_THREADS) {
    const float f = bf2f(row[i]);
    if (f > m) { s *= __expf(m - f); m = f; }
    s += __expf(f - m);
  }
  // combine across the CTA
  // threads (or whole warps) that saw no element carry m = -inf, s = 0
  float wm = warp_max(m);
  float ws = (m == -INFINITY) ? 0.f : s * __expf(m - wm);
  ws = warp_sum(ws);
  if (lane == 0) { red_m[warp] = wm; red_s[warp] = ws; }
  __syncthreads();
  if (warp == 0) {
    float mm = lane < CE_THREADS / 32 ? red_m[lane] : -INFINITY;
    float ss = lane < CE_THREADS / 32 ? red_s[lane] : 0.f;
    const float gm = warp_max(mm);
    ss = warp_sum((lane < CE_THREADS / 32 && mm != -INFINITY) ? ss * __expf(mm - gm) : 0.f);
    if (lane == 0) { bc[0] = gm; bc[1] = gm + logf(ss); }
  }
  __syncthreads();
  const float lse = bc[1];
  const long long tgt = targets[r];
  const bool valid = tgt >= 0 && tgt < V;
  if (tgt >= V && threadIdx.x == 0) record_error(status, kErrBadTarget);
  if (threadIdx.x == 0) {
    lse_out[r] = lse;
    loss[r] = valid ? lse - bf2f(row[tgt]) : 0.f;
  }
  __syncthreads();   // the target logit is read before being overwritten
  const float zfac = valid ? scale * (1.f + 2.f * z_coef * lse) : 0.f;
  for (int i = threadIdx.x; i < V8; i += CE_THREADS) {
    uint4 t = reinterpret_cast<uint4*>(row)[i];
    uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(w[j]);
      const int c = i * 8 + 2 * j;
      float p0 = __expf(f.x - lse) * zfac, p1 = __expf(f.y - lse) * zfac;
      if (valid && c == tgt) p0 -= scale;
      if (valid && c + 1 == tgt) p1 -= scale;
      w[j] = pack_bf16x2(p0, p1);
    }
    reinterpret_cast<uint4*>(row)[i] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  for (int i = V8 * 8 + threadIdx.x; i < V; i += CE_THREADS) {
    float p = __expf(bf2f(row[i]) - lse) * zfac;
    if (valid && i == tgt) p -= scale;
    row[i] = f2bf(p);
  }
}

// ---------------------------------------------------- embedding grad --
// dW[tok[i], :] += dy[i, :]   (fp32 accumulate)

template <typename T>
__global__ void embedding_bwd_k(const T* __restrict__ dy, const long long* __restrict__ tok,
                                float* __restrict__ dW, long long n, int D, long long V) {
  const long long i = blockIdx.x;
  if (i >= n) return;
  const long long t = tok[i];
  if (!VAGUS_CHECK(t, V)) return;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float v;
    if constexpr (sizeof(T) == 4) v = dy[i * D + c]; else v = bf2f(dy[i * D + c]);
    atomicAdd(&dW[t * D + c], v);
  }
}

template <typename T>
__global__ void embedding_fwd_k(const float* __restrict__ W, const long long* __restrict__ tok, T* __restrict__ y,
                                long long n, int D, long long V) {
  const long long i = blockIdx.x;
  if (i >= n) return;
  const long long t = tok[i];
  if (!VAGUS_CHECK(t, V)) return;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    if constexpr (sizeof(T) == 4) y[i * D + c] = W[t * D + c]; else y[i * D + c] = f2bf(W[t * D + c]);
  }
}

// ------------------------------------------------------------- AdamW --
// Flat fp32 param / grad / m / v; optional bf16 shadow copy written in the
// same pass (the compute copy the next forward reads).

__global__ void adamw_k(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                        float* __restrict__ v, __nv_bfloat16* __restrict__ shadow, long long n, float lr, float b1,
                        float b2, float eps, float wd, float bc1, float bc2, float gscale) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float gi = g[i] * gscale;
    float mi = m[i] = b1 * m[i] + (1.f - b1) * gi;
    float vi = v[i] = b2 * v[i] + (1.f - b2) * gi * gi;
    float pi = p[i] * (1.f - lr * wd);
    pi -= lr * (mi / bc1) / (sqrtf(vi / bc2) + eps);
    p[i] = pi;
    if (shadow) shadow[i] = f2bf(pi);
  }
}

// Muon momentum (Nesterov): buf = lerp(buf, g, 1 - mu); upd = lerp(g, buf, mu) -> bf16
__global__ void muon_momentum_k(const float* __restrict__ g, float* __restrict__ buf, __nv_bfloat16* __restrict__ upd,
                                long long n, float mu, int nesterov, float gscale) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float gi = g[i] * gscale;
    const float b = buf[i] + (1.f - mu) * (gi - buf[i]);
    buf[i] = b;
    upd[i] = f2bf(nesterov ? gi + mu * (b - gi) : b);
  }
}

inline int grid_for(long long n, int t = 256) {
  long long g = (n + t - 1) / t;
  return static_cast<int>(g > 148 * 32 ? 148 * 32 : (g < 1 ? 1 : g));
}

}  // namespace

int swiglu_fwd(const void* u, void* s, long long rows, int F, cudaStream_t st) {
  if (swiglu_v8_ok(u, s, nullptr, rows, F)) {
    const unsigned n8 = static_cast<unsigned>(rows * (F / 8));
    swiglu_fwd_v8<<<grid_for(n8), 256, 0, st>>>((const __nv_bfloat16*)u, (__nv_bfloat16*)s, n8, F / 8);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
  }
  swiglu_fwd_k<<<grid_for(rows * F / 2), 256, 0, st>>>((const __nv_bfloat16*)u, (__nv_bfloat16*)s, rows, F);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int swiglu_bwd(const void* ds, const void* u, void* du, long long rows, int F, cudaStream_t st) {
  if (swiglu_v8_ok(ds, u, du, rows, F)) {
    const unsigned n8 = static_cast<unsigned>(rows * (F / 8));
    swiglu_bwd_v8<<<grid_for(n8), 256, 0, st>>>((const __nv_bfloat16*)ds, (const __nv_bfloat16*)u,
                                                (__nv_bfloat16*)du, n8, F / 8);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
  }
  swiglu_bwd_k<<<grid_for(rows * F / 2), 256, 0, st>>>((const __nv_bfloat16*)ds, (const __nv_bfloat16*)u,
                                                        (__nv_bfloat16*)du, rows, F);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int sigmoid_gate_fwd(const void* x, const void* g, void* y, long long n, cudaStream_t st) {
  sgate_fwd_k<<<grid_for(n), 256, 0, st>>>((const __nv_bfloat16*)x, (const __nv_bfloat16*)g, (__nv_bfloat16*)y, n);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int sigmoid_gate_bwd(const void* dy, const void* x, const void* g, void* dx, void* dg, long long n, cudaStream_t st) {
  sgate_bwd_k<<<grid_for(n), 256, 0, st>>>((const __nv_bfloat16*)dy, (const __nv_bfloat16*)x, (const __nv_bfloat16*)g,
                                           (__nv_bfloat16*)dx, (__nv_bfloat16*)dg, n);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int softmax_ce(void* logits, const long long* targets, float* loss, float* lse, long long rows, int V, float scale,
               float z_coef, cudaStream_t st, int* status) {
  if (rows <= 0) return 0;
  softmax_ce_k<<<static_cast<unsigned>(rows), CE_THREADS, 0, st>>>((__nv_bfloat16*)logits, targets, loss, lse, V,
                                                                   scale, z_coef, status);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int embedding_fwd(const float* W, const long long* tok, void* y, int y_f32, long long n, int D, long long V,
                  cudaStream_t st) {
  if (n <= 0) return 0;
  if (y_f32) embedding_fwd_k<float><<<static_cast<unsigned>(n), 256, 0, st>>>(W, tok, (float*)y, n, D, V);
  else embedding_fwd_k<__nv_bfloat16><<<static_cast<unsigned>(n), 256, 0, st>>>(W, tok, (__nv_bfloat16*)y, n, D, V);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int embedding_bwd(const void* dy, int dy_f32, const long long* tok, float* dW, long long n, int D, long long V,
                  cudaStream_t st) {
  if (n <= 0) return 0;
  if (dy_f32) embedding_bwd_k<float><<<static_cast<unsigned>(n), 256, 0, st>>>((const float*)dy, tok, dW, n, D, V);
  else embedding_bwd_k<__nv_bfloat16><<<static_cast<unsigned>(n), 256, 0, st>>>((const __nv_bfloat16*)dy, tok, dW, n, D, V);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int adamw_step(float* p, const float* g, float* m, float* v, void* shadow, long long n, float lr, float b1, float b2,
               float eps, float wd, float bc1, float bc2, float gscale, cudaStream_t st) {
  if (n <= 0) return 0;
  adamw_k<<<grid_for(n), 256, 0, st>>>(p, g, m, v, (__nv_bfloat16*)shadow, n, lr, b1, b2, eps, wd, bc1, bc2, gscale);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int muon_momentum(const float* g, float* buf, void* upd, long long n, float mu, int nesterov, float gscale,
                  cudaStream_t st) {
  if (n <= 0) return 0;
  muon_momentum_k<<<grid_for(n), 256, 0, st>>>(g, buf, (__nv_bfloat16*)upd, n, mu, nesterov, gscale);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

}  // namespace vagus
