// Row-wise normalisation kernels (one warp per row, fp32 statistics):
//   rmsnorm        y = x * rsqrt(mean(x^2) + eps) * gamma          (fwd / bwd)
//   rmsnorm_gated  y = rmsnorm(o) * gamma * silu(g)                (fwd / bwd)
//   qk_norm_rope   per-head RMSNorm (optional) then interleaved-pair RoPE
//                  (optional), the prologue of softmax attention   (fwd / bwd)
// gamma gradients are reduced per CTA in shared memory and added to an fp32
// buffer with one atomic per column per CTA.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace vagus {
namespace {

template <typename T>
__device__ __forceinline__ float ld(const T* p, long long i);
template <>
__device__ __forceinline__ float ld<float>(const float* p, long long i) { return p[i]; }
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p, long long i) { return bf2f(p[i]); }

template <typename T>
__device__ __forceinline__ void st(T* p, long long i, float v);
template <>
__device__ __forceinline__ void st<float>(float* p, long long i, float v) { p[i] = v; }
template <>
__device__ __forceinline__ void st<__nv_bfloat16>(__nv_bfloat16* p, long long i, float v) { p[i] = f2bf(v); }

constexpr int ROWS_PER_CTA = 8;   // one warp per row, 8 warps
constexpr int MAXV = 32;          // up to 32 values per lane (D <= 1024 in registers; larger loops)

// ------------------------------------------------------------- rmsnorm --

template <typename TI, typename TO>
__global__ void rmsnorm_fwd_k(const TI* __restrict__ x, const float* __restrict__ gamma, TO* __restrict__ y,
                              float* __restrict__ rstd, int rows, int D, float eps) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const long long r = (long long)blockIdx.x * ROWS_PER_CTA + warp;
  if (r >= rows) return;
  const TI* xr = x + r * D;
  float ss = 0.f;
  for (int c = lane; c < D; c += 32) { float v = ld(xr, c); ss += v * v; }
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss / D + eps);
  if (lane == 0 && rstd) rstd[r] = rs;
  TO* yr = y + r * D;
  for (int c = lane; c < D; c += 32) st(yr, c, ld(xr, c) * rs * gamma[c]);
}

// dx = rs * (dy*g - xhat * mean(dy*g*xhat)) (+ dres);  dgamma += sum_rows dy * xhat
template <typename TI, typename TG, typename TO>
__global__ void rmsnorm_bwd_k(const TG* __restrict__ dy, const TI* __restrict__ x, const float* __restrict__ gamma,
                              const float* __restrict__ rstd, const float* __restrict__ dres, TO* __restrict__ dx,
                              float* __restrict__ dgamma, int rows, int D) {
  extern __shared__ float sg[];   // [D] partial dgamma of this CTA
  for (int c = threadIdx.x; c < D; c += blockDim.x) sg[c] = 0.f;
  __syncthreads();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const long long r = (long long)blockIdx.x * ROWS_PER_CTA + warp;
  if (r < rows) {
    const TI* xr = x + r * D;
    const TG* dr = dy + r * D;
    const float rs = rstd[r];
    float dot = 0.f;
    for (int c = lane; c < D; c += 32) dot += ld(dr, c) * gamma[c] * ld(xr, c) * rs;
    dot = warp_sum(dot) / D;
    TO* o = dx + r * D;
    for (int c = lane; c < D; c += 32) {
      const float xh = ld(xr, c) * rs;
      const float g = ld(dr, c);
      float v = rs * (g * gamma[c] - xh * dot);
      if (dres) v += dres[r * D + c];
      st(o, c, v);
      atomicAdd(&sg[c], g * xh);
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += blockDim.x) atomicAdd(&dgamma[c], sg[c]);
}

// Vectorised backward for the residual-stream case: x, dx (and dres) fp32,
// dy bf16 or fp32, D = 128 * NV.  A persistent grid of 8-warp CTAs walks the
// rows (one warp per row, lane l owns columns 4 l + 128 j); the gamma
// gradient stays in registers across all rows of a warp and is reduced once
// per CTA.  dx16, when given, receives a bf16 copy of dx (the operand the
// next GEMM backward consumes).
template <typename TG, int NV>
__global__ void __launch_bounds__(256, NV >= 8 ? 1 : 2)
rmsnorm_bwd_vec_k(const TG* __restrict__ dy, const float* __restrict__ x, const float* __restrict__ gamma,
                  const float* __restrict__ rstd, const float* __restrict__ dres, float* __restrict__ dx,
                  __nv_bfloat16* __restrict__ dx16, float* __restrict__ dgamma, long long rows) {
  constexpr int D = 128 * NV;
  // rows wider than 1024 keep the gamma-gradient partials in a per-warp
  // shared-memory row (each lane owns its columns: no atomics) instead of
  // registers, which would spill
  constexpr bool kSmemAcc = NV > 8;
  __shared__ __align__(16) float sgam[D];
  __shared__ float sg[D];
  extern __shared__ __align__(16) float sacc[];     // [8][D] when kSmemAcc
  for (int c = threadIdx.x; c < D; c += blockDim.x) { sgam[c] = gamma[c]; sg[c] = 0.f; }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  float* wacc = kSmemAcc ? sacc + warp * D : nullptr;
  if constexpr (kSmemAcc) {
    for (int c = lane * 4; c < D; c += 128) *reinterpret_cast<float4*>(wacc + c) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncthreads();
  float4 acc[kSmemAcc ? 1 : NV];
#pragma unroll
  for (int j = 0; j < (kSmemAcc ? 1 : NV); ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  // two passes over the row (the second re-reads x and dy, which are in L1
  // by then)
  auto load_row = [&](long long r, int j, float4& xv, float4& gv) {
    const int c = 4 * lane + 128 * j;
    xv = *reinterpret_cast<const float4*>(x + r * D + c);
    if constexpr (sizeof(TG) == 4) {
      gv = *reinterpret_cast<const float4*>(dy + r * D + c);
    } else {
      const uint2 u = *reinterpret_cast<const uint2*>(dy + r * D + c);
      const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y);
      gv = make_float4(a.x, a.y, b.x, b.y);
    }
  };
  for (long long r = (long long)blockIdx.x * 8 + warp; r < rows; r += (long long)gridDim.x * 8) {
    const float rs = rstd[r];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      float4 xv, gv;
      load_row(r, j, xv, gv);
      const float4 gm = *reinterpret_cast<const float4*>(sgam + 4 * lane + 128 * j);
      dot += gv.x * gm.x * xv.x + gv.y * gm.y * xv.y + gv.z * gm.z * xv.z + gv.w * gm.w * xv.w;
    }
    dot = warp_sum(dot) * rs / D;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = 4 * lane + 128 * j;
      float4 xv, gv;
      load_row(r, j, xv, gv);
      const float4 gm = *reinterpret_cast<const float4*>(sgam + c);
      const float4 h = make_float4(xv.x * rs, xv.y * rs, xv.z * rs, xv.w * rs);
      float4 o = make_float4(rs * (gv.x * gm.x - h.x * dot), rs * (gv.y * gm.y - h.y * dot),
                             rs * (gv.z * gm.z - h.z * dot), rs * (gv.w * gm.w - h.w * dot));
      if (dres) {
        const float4 d = *reinterpret_cast<const float4*>(dres + r * D + c);
        o.x += d.x; o.y += d.y; o.z += d.z; o.w += d.w;
      }
      *reinterpret_cast<float4*>(dx + r * D + c) = o;
      if (dx16) *reinterpret_cast<uint2*>(dx16 + r * D + c) = make_uint2(pack_bf16x2(o.x, o.y), pack_bf16x2(o.z, o.w));
      if constexpr (kSmemAcc) {
        float4 a4 = *reinterpret_cast<float4*>(wacc + c);
        a4.x += gv.x * h.x; a4.y += gv.y * h.y; a4.z += gv.z * h.z; a4.w += gv.w * h.w;
        *reinterpret_cast<float4*>(wacc + c) = a4;
      } else {
        acc[j].x += gv.x * h.x; acc[j].y += gv.y * h.y; acc[j].z += gv.z * h.z; acc[j].w += gv.w * h.w;
      }
    }
  }
  if constexpr (kSmemAcc) {
    __syncthreads();
    for (int c = threadIdx.x; c < D; c += blockDim.x) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) t += sacc[w * D + c];
      atomicAdd(&dgamma[c], t);
    }
  } else {
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = 4 * lane + 128 * j;
      atomicAdd(&sg[c], acc[j].x); atomicAdd(&sg[c + 1], acc[j].y);
      atomicAdd(&sg[c + 2], acc[j].z); atomicAdd(&sg[c + 3], acc[j].w);
    }
    __syncthreads();
    for (int c = threadIdx.x; c < D; c += blockDim.x) atomicAdd(&dgamma[c], sg[c]);
  }
}

// ------------------------------------------------------- rmsnorm_gated --
// o: (rows, Dh) with rows = tokens * heads; g: same layout; gamma (Dh)

// The gate may be a column block of a wider packed matrix: row r = (token
// t, head h) reads g[t * ldg + h * D + c] (ldg = H * D when contiguous).
template <typename TO_>
__global__ void rmsnorm_gated_fwd_k(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ g,
                                    long long ldg, int H, const float* __restrict__ gamma, TO_* __restrict__ y,
                                    float* __restrict__ rstd, long long rows, int D, float eps) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const long long r = (long long)blockIdx.x * ROWS_PER_CTA + warp;
  if (r >= rows) return;
  const __nv_bfloat16* orow = o + r * D;
  const __nv_bfloat16* grow = g + (r / H) * ldg + (r % H) * D;
  float ss = 0.f;
  for (int c = lane; c < D; c += 32) { float v = bf2f(orow[c]); ss += v * v; }
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss / D + eps);
  if (lane == 0) rstd[r] = rs;
  for (int c = lane; c < D; c += 32) st(y + r * D, c, bf2f(orow[c]) * rs * gamma[c] * silu_f(bf2f(grow[c])));
}

__global__ void rmsnorm_gated_bwd_k(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ o,
                                    const __nv_bfloat16* __restrict__ g, long long ldg, int H,
                                    const float* __restrict__ gamma, const float* __restrict__ rstd,
                                    __nv_bfloat16* __restrict__ dO, __nv_bfloat16* __restrict__ dG, long long lddg,
                                    float* __restrict__ dgamma, long long rows, int D) {
  extern __shared__ float sg[];
  for (int c = threadIdx.x; c < D; c += blockDim.x) sg[c] = 0.f;
  __syncthreads();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const long long r = (long long)blockIdx.x * ROWS_PER_CTA + warp;
  if (r < rows) {
    const float rs = rstd[r];
    const __nv_bfloat16* grow = g + (r / H) * ldg + (r % H) * D;
    __nv_bfloat16* dgrow = dG + (r / H) * lddg + (r % H) * D;
    float dot = 0.f;
    for (int c = lane; c < D; c += 32) {
      const float gv = bf2f(grow[c]);
      const float dyn = bf2f(dy[r * D + c]) * silu_f(gv);          // grad wrt normalised*gamma
      dot += dyn * gamma[c] * bf2f(o[r * D + c]) * rs;
    }
    dot = warp_sum(dot) / D;
    for (int c = lane; c < D; c += 32) {
      const float ov = bf2f(o[r * D + c]);
      const float gv = bf2f(grow[c]);
      const float dyv = bf2f(dy[r * D + c]);
      const float sgm = sigmoid_f(gv);
      const float silu = gv * sgm;
      const float xh = ov * rs;
      const float dyn = dyv * silu;
      dO[r * D + c] = f2bf(rs * (dyn * gamma[c] - xh * dot));
      // d silu(g) / dg = s (1 + g (1 - s))
      dgrow[c] = f2bf(dyv * xh * gamma[c] * sgm * (1.f + gv * (1.f - sgm)));
      atomicAdd(&sg[c], dyn * xh);
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += blockDim.x) atomicAdd(&dgamma[c], sg[c]);
}

// Vectorised gated RMSNorm for head dims 128 / 256 (NV = D / 32 elements per
// lane, one or two 8-byte / 16-byte loads per tensor): each lane keeps its
// slice of the row in registers between the two passes, warps stride over
// rows, and the backward's dgamma stays in registers until one shared-memory
// reduction and one global atomic per column per CTA (the scalar kernels
// above issue a shared atomic per element and a global atomic per column per
// 8 rows).
template <int NV>
__device__ __forceinline__ void ld_bf16v(const __nv_bfloat16* p, float (&f)[NV]) {
  if constexpr (NV == 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) { const float2 t = unpack_bf16x2(w[i]); f[2 * i] = t.x; f[2 * i + 1] = t.y; }
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  }
}
template <int NV>
__device__ __forceinline__ void st_bf16v(__nv_bfloat16* p, const float (&f)[NV]) {
  if constexpr (NV == 8) {
    *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                                              pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
  } else {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]));
  }
}

template <int NV>
__global__ void __launch_bounds__(256)
rmsnorm_gated_fwd_vec_k(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ g, long long ldg,
                        int H, const float* __restrict__ gamma, __nv_bfloat16* __restrict__ y,
                        float* __restrict__ rstd, long long rows, float eps) {
  constexpr int D = 32 * NV;
  const int lane = threadIdx.x & 31;
  const long long w0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const long long nw = (long long)gridDim.x * blockDim.x / 32;
  float gm[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) gm[i] = gamma[lane * NV + i];
  for (long long r = w0; r < rows; r += nw) {
    float ov[NV], gv[NV];
    ld_bf16v<NV>(o + r * D + lane * NV, ov);
    ld_bf16v<NV>(g + (r / H) * ldg + (r % H) * D + lane * NV, gv);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) ss += ov[i] * ov[i];
    const float rs = rsqrtf(warp_sum(ss) / D + eps);
    if (lane == 0) rstd[r] = rs;
#pragma unroll
    for (int i = 0; i < NV; ++i) ov[i] = ov[i] * rs * gm[i] * silu_f(gv[i]);
    st_bf16v<NV>(y + r * D + lane * NV, ov);
  }
}

template <int NV>
__global__ void __launch_bounds__(256)
rmsnorm_gated_bwd_vec_k(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ o,
                        const __nv_bfloat16* __restrict__ g, long long ldg, int H, const float* __restrict__ gamma,
                        const float* __restrict__ rstd, __nv_bfloat16* __restrict__ dO,
                        __nv_bfloat16* __restrict__ dG, long long lddg, float* __restrict__ dgamma, long long rows) {
  constexpr int D = 32 * NV;
  __shared__ float red[8][D];
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const long long w0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const long long nw = (long long)gridDim.x * blockDim.x / 32;
  float gm[NV], acc[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) { gm[i] = gamma[lane * NV + i]; acc[i] = 0.f; }
  for (long long r = w0; r < rows; r += nw) {
    float ov[NV], gv[NV], dv[NV];
    ld_bf16v<NV>(o + r * D + lane * NV, ov);
    ld_bf16v<NV>(g + (r / H) * ldg + (r % H) * D + lane * NV, gv);
    ld_bf16v<NV>(dy + r * D + lane * NV, dv);
    const float rs = rstd[r];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) dot += dv[i] * silu_f(gv[i]) * gm[i] * ov[i] * rs;
    dot = warp_sum(dot) / D;
    float dov[NV], dgv[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const float sgm = sigmoid_f(gv[i]);
      const float xh = ov[i] * rs;
      const float dyn = dv[i] * gv[i] * sgm;                      // grad wrt normalised * gamma
      dov[i] = rs * (dyn * gm[i] - xh * dot);
      // d silu(g) / dg = s (1 + g (1 - s))
      dgv[i] = dv[i] * xh * gm[i] * sgm * (1.f + gv[i] * (1.f - sgm));
      acc[i] += dyn * xh;
    }
    st_bf16v<NV>(dO + r * D + lane * NV, dov);
    st_bf16v<NV>(dG + (r / H) * lddg + (r % H) * D + lane * NV, dgv);
  }
#pragma unroll
  for (int i = 0; i < NV; ++i) red[warp][lane * NV + i] = acc[i];
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w][c];
    atomicAdd(&dgamma[c], t);
  }
}

// ------------------------------------------------------- qk_norm_rope --
// x: (B, L, H, Dh) bf16 contiguous; cos/sin: (L, Dh/2) fp32 (already offset).
// One warp per (b, l, h) row.

__global__ void qk_norm_rope_fwd_k(const __nv_bfloat16* __restrict__ x, const float* __restrict__ gamma,
                                   const float* __restrict__ cosv, const float* __restrict__ sinv,
                                   __nv_bfloat16* __restrict__ y, float* __restrict__ rstd, int rows, int L, int H,
                                   int D, float eps) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const long long r = (long long)blockIdx.x * ROWS_PER_CTA + warp;
  if (r >= rows) return;
  const int l = static_cast<int>((r / H) % L);
  const __nv_bfloat16* xr = x + r * D;
  float rs = 1.f;
  if (gamma) {
    float ss = 0.f;
    for (int c = lane; c < D; c += 32) { float v = bf2f(xr[c]); ss += v * v; }
    rs = rsqrtf(warp_sum(ss) / D + eps);
    if (lane == 0) rstd[r] = rs;
  }
  const int half = D / 2;
  for (int i = lane; i < half; i += 32) {
    float x0 = bf2f(xr[2 * i]) * rs, x1 = bf2f(xr[2 * i + 1]) * rs;
    if (gamma) {
      // the reference casts the normalised value back to the input dtype before gamma
      x0 = bf2f(f2bf(x0)) * gamma[2 * i];
      x1 = bf2f(f2bf(x1)) * gamma[2 * i + 1];
    }
    if (cosv) {
      const float c = cosv[(long long)l * half + i], s = sinv[(long long)l * half + i];
      const float y0 = x0 * c - x1 * s, y1 = x0 * s + x1 * c;
      x0 = y0; x1 = y1;
    }
    y[r * D + 2 * i] = f2bf(x0);
    y[r * D + 2 * i + 1] = f2bf(x1);
  }
}

__global__ void qk_norm_rope_bwd_k(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                   const float* __restrict__ gamma, const float* __restrict__ cosv,
                                   const float* __restrict__ sinv, const float* __restrict__ rstd,
                                   __nv_bfloat16* __restrict__ dx, float* __restrict__ dgamma, int rows, int L, int H,
                                   int D) {
  extern __shared__ float sg[];
  if (gamma) {
    for (int c = threadIdx.x; c < D; c += blockDim.x) sg[c] = 0.f;
    __syncthreads();
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const long long r = (long long)blockIdx.x * ROWS_PER_CTA + warp;
  const int half = D / 2;
  if (r < rows) {
    const int l = static_cast<int>((r / H) % L);
    const float rs = gamma ? rstd[r] : 1.f;
    float dot = 0.f;
    // pass 1: un-rotate dy -> dz (grad wrt the normalised*gamma value)
    for (int i = lane; i < half; i += 32) {
      float d0 = bf2f(dy[r * D + 2 * i]), d1 = bf2f(dy[r * D + 2 * i + 1]);
      if (cosv) {
        const float c = cosv[(long long)l * half + i], s = sinv[(long long)l * half + i];
        const float e0 = d0 * c + d1 * s, e1 = -d0 * s + d1 * c;
        d0 = e0; d1 = e1;
      }
      if (gamma) {
        const float xh0 = bf2f(x[r * D + 2 * i]) * rs, xh1 = bf2f(x[r * D + 2 * i + 1]) * rs;
        dot += d0 * gamma[2 * i] * xh0 + d1 * gamma[2 * i + 1] * xh1;
        atomicAdd(&sg[2 * i], d0 * xh0);
        atomicAdd(&sg[2 * i + 1], d1 * xh1);
      }
    }
    if (gamma) dot = warp_sum(dot) / D;
    for (int i = lane; i < half; i += 32) {
      float d0 = bf2f(dy[r * D + 2 * i]), d1 = bf2f(dy[r * D + 2 * i + 1]);
      if (cosv) {
        const float c = cosv[(long long)l * half + i], s = sinv[(long long)l * half + i];
        const float e0 = d0 * c + d1 * s, e1 = -d0 * s + d1 * c;
        d0 = e0; d1 = e1;
      }
      if (gamma) {
        const float xh0 = bf2f(x[r * D + 2 * i]) * rs, xh1 = bf2f(x[r * D + 2 * i + 1]) * rs;
        d0 = rs * (d0 * gamma[2 * i] - xh0 * dot);
        d1 = rs * (d1 * gamma[2 * i + 1] - xh1 * dot);
      }
      dx[r * D + 2 * i] = f2bf(d0);
      dx[r * D + 2 * i + 1] = f2bf(d1);
    }
  }
  if (gamma) {
    __syncthreads();
    for (int c = threadIdx.x; c < D; c += blockDim.x) atomicAdd(&dgamma[c], sg[c]);
  }
}

inline int blocks_for(long long rows) { return static_cast<int>((rows + ROWS_PER_CTA - 1) / ROWS_PER_CTA); }

// Vectorised qk-norm + RoPE for head dims 64 / 128: a thread owns 8 adjacent
// channels (one 16-byte load), D / 8 lanes share a row (the norm is a
// shuffle reduction over them), so a warp covers 256 / D rows per pass;
// CTAs stride over the rows.  The backward keeps its gamma-gradient partials
// in registers across all rows it visits and adds them once per CTA.
template <int D>
__global__ void __launch_bounds__(256)
qk_norm_rope_fwd_v(const __nv_bfloat16* __restrict__ x, const float* __restrict__ gamma,
                   const float* __restrict__ cosv, const float* __restrict__ sinv, __nv_bfloat16* __restrict__ y,
                   float* __restrict__ rstd, long long rows, int L, int H, float eps, long long ldx, long long ldy) {
  constexpr int TPR = D / 8, RPW = 32 / TPR, HALF = D / 2;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int sub = lane % TPR, rw = lane / TPR;
  const int c0 = 8 * sub;
  float gm[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) gm[j] = gamma ? gamma[c0 + j] : 1.f;
  const long long step = (long long)gridDim.x * 8 * RPW;
  for (long long base = ((long long)blockIdx.x * 8 + warp) * RPW; base < rows; base += step) {
    const long long r = base + rw;
    const bool valid = r < rows;
    const long long t = r / H, hd = (r - t * H) * D;    // token, channel offset of the head in the token
    float v[8];
    {
      const uint4 u = valid ? *reinterpret_cast<const uint4*>(x + t * ldx + hd + c0) : make_uint4(0u, 0u, 0u, 0u);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) { const float2 f = unpack_bf16x2(w[j]); v[2 * j] = f.x; v[2 * j + 1] = f.y; }
    }
    if (gamma) {
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[j] * v[j];
#pragma unroll
      for (int o = 1; o < TPR; o <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float rs = rsqrtf(ss / D + eps);
      if (valid && sub == 0) rstd[r] = rs;
      // the normalised value is rounded to the input dtype before gamma, as in the unfused form
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = bf2f(f2bf(v[j] * rs)) * gm[j];
    }
    if (cosv && valid) {
      const long long l = t % L;
      const float4 c4 = *reinterpret_cast<const float4*>(cosv + l * HALF + 4 * sub);
      const float4 s4 = *reinterpret_cast<const float4*>(sinv + l * HALF + 4 * sub);
      const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = v[2 * j], b = v[2 * j + 1];
        v[2 * j] = a * cc[j] - b * sn[j];
        v[2 * j + 1] = a * sn[j] + b * cc[j];
      }
    }
    if (valid)
      *reinterpret_cast<uint4*>(y + t * ldy + hd + c0) =
          make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
  }
}

template <int D>
__global__ void __launch_bounds__(256)
qk_norm_rope_bwd_v(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                   const float* __restrict__ gamma, const float* __restrict__ cosv, const float* __restrict__ sinv,
                   const float* __restrict__ rstd, __nv_bfloat16* __restrict__ dx, float* __restrict__ dgamma,
                   long long rows, int L, int H, long long lddy, long long ldx, long long lddx) {
  constexpr int TPR = D / 8, RPW = 32 / TPR, HALF = D / 2;
  __shared__ float sg[D];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int sub = lane % TPR, rw = lane / TPR;
  const int c0 = 8 * sub;
  if (gamma) {
    for (int c = threadIdx.x; c < D; c += blockDim.x) sg[c] = 0.f;
    __syncthreads();
  }
  float gm[8], acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) { gm[j] = gamma ? gamma[c0 + j] : 1.f; acc[j] = 0.f; }
  const long long step = (long long)gridDim.x * 8 * RPW;
  for (long long base = ((long long)blockIdx.x * 8 + warp) * RPW; base < rows; base += step) {
    const long long r = base + rw;
    const bool valid = r < rows;
    const long long t = r / H, hd = (r - t * H) * D;
    float d[8], xv[8];
    {
      const uint4 u = valid ? *reinterpret_cast<const uint4*>(dy + t * lddy + hd + c0) : make_uint4(0u, 0u, 0u, 0u);
      const uint4 q =
          valid && gamma ? *reinterpret_cast<const uint4*>(x + t * ldx + hd + c0) : make_uint4(0u, 0u, 0u, 0u);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w}, wq[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = unpack_bf16x2(w[j]); d[2 * j] = f.x; d[2 * j + 1] = f.y;
        f = unpack_bf16x2(wq[j]); xv[2 * j] = f.x; xv[2 * j + 1] = f.y;
      }
    }
    if (cosv && valid) {                                  // un-rotate: the transpose of the rotation
      const long long l = t % L;
      const float4 c4 = *reinterpret_cast<const float4*>(cosv + l * HALF + 4 * sub);
      const float4 s4 = *reinterpret_cast<const float4*>(sinv + l * HALF + 4 * sub);
      const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = d[2 * j], b = d[2 * j + 1];
        d[2 * j] = a * cc[j] + b * sn[j];
        d[2 * j + 1] = -a * sn[j] + b * cc[j];
      }
    }
    if (gamma) {
      const float rs = valid ? rstd[r] : 0.f;
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xh = xv[j] * rs;
        dot += d[j] * gm[j] * xh;
        acc[j] += d[j] * xh;
      }
#pragma unroll
      for (int o = 1; o < TPR; o <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      dot /= D;
#pragma unroll
      for (int j = 0; j < 8; ++j) d[j] = rs * (d[j] * gm[j] - xv[j] * rs * dot);
    }
    if (valid)
      *reinterpret_cast<uint4*>(dx + t * lddx + hd + c0) =
          make_uint4(pack_bf16x2(d[0], d[1]), pack_bf16x2(d[2], d[3]), pack_bf16x2(d[4], d[5]), pack_bf16x2(d[6], d[7]));
  }
  if (gamma) {
    // lanes with the same `sub` hold the same channels: reduce over the warp's rows, then the CTA's
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float v = acc[j];
#pragma unroll
      for (int o = TPR; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      acc[j] = v;
    }
    if (rw == 0) {
#pragma unroll
      for (int j = 0; j < 8; ++j) atomicAdd(&sg[c0 + j], acc[j]);
    }
    __syncthreads();
    for (int c = threadIdx.x; c < D; c += blockDim.x) atomicAdd(&dgamma[c], sg[c]);
  }
}

inline int vec_rope_grid(long long rows, int rpw) {
  const long long want = (rows + 8LL * rpw - 1) / (8LL * rpw);
  return static_cast<int>(std::min<long long>(std::max<long long>(want, 1), 148LL * 8));
}

}  // namespace

int rmsnorm_fwd(const void* x, int x_f32, const float* gamma, void* y, int y_f32, float* rstd, long long rows, int D,
                float eps, cudaStream_t s) {
  const int g = blocks_for(rows), t = 32 * ROWS_PER_CTA;
  if (x_f32 && y_f32) rmsnorm_fwd_k<float, float><<<g, t, 0, s>>>((const float*)x, gamma, (float*)y, rstd, rows, D, eps);
  else if (x_f32) rmsnorm_fwd_k<float, __nv_bfloat16><<<g, t, 0, s>>>((const float*)x, gamma, (__nv_bfloat16*)y, rstd, rows, D, eps);
  else if (y_f32) rmsnorm_fwd_k<__nv_bfloat16, float><<<g, t, 0, s>>>((const __nv_bfloat16*)x, gamma, (float*)y, rstd, rows, D, eps);
  else rmsnorm_fwd_k<__nv_bfloat16, __nv_bfloat16><<<g, t, 0, s>>>((const __nv_bfloat16*)x, gamma, (__nv_bfloat16*)y, rstd, rows, D, eps);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int rmsnorm_bwd(const void* dy, int dy_f32, const void* x, int x_f32, const float* gamma, const float* rstd,
                const float* dres, void* dx, int dx_f32, float* dgamma, long long rows, int D, cudaStream_t s,
                void* dx16) {
  if (x_f32 && dx_f32 && D % 128 == 0 && (D == 512 || D == 768 || D == 1024 || D == 1536 || D == 2048)) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long need = (rows + 7) / 8;
    const int per_sm = D >= 1024 ? 1 : 2;      // the wide rows keep their gamma partials in 255 registers
    const int grid = static_cast<int>(std::min<long long>(need, (long long)per_sm * sms));
#define RV(TG, NV)                                                                                       \
  do {                                                                                                   \
    const int dyn = NV > 8 ? 8 * 128 * NV * 4 : 0;                                                       \
    if (dyn && cudaFuncSetAttribute(rmsnorm_bwd_vec_k<TG, NV>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                    dyn) != cudaSuccess)                                                 \
      return 3;                                                                                          \
    rmsnorm_bwd_vec_k<TG, NV><<<grid, 256, dyn, s>>>((const TG*)dy, (const float*)x, gamma, rstd, dres,   \
                                                     (float*)dx, (__nv_bfloat16*)dx16, dgamma, rows);    \
  } while (0)
#define RVD(TG) switch (D) { case 512: RV(TG, 4); break; case 768: RV(TG, 6); break; case 1024: RV(TG, 8); break; \
                             case 1536: RV(TG, 12); break; default: RV(TG, 16); }
    if (dy_f32) { RVD(float) } else { RVD(__nv_bfloat16) }
#undef RVD
#undef RV
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
  }
  if (dx16) return 5;
  const int g = blocks_for(rows), t = 32 * ROWS_PER_CTA;
  const size_t sm = D * sizeof(float);
#define RB(TI, TG, TO) rmsnorm_bwd_k<TI, TG, TO><<<g, t, sm, s>>>((const TG*)dy, (const TI*)x, gamma, rstd, dres, (TO*)dx, dgamma, rows, D)
  if (x_f32) {
    if (dy_f32) { if (dx_f32) RB(float, float, float); else RB(float, float, __nv_bfloat16); }
    else { if (dx_f32) RB(float, __nv_bfloat16, float); else RB(float, __nv_bfloat16, __nv_bfloat16); }
  } else {
    if (dy_f32) { if (dx_f32) RB(__nv_bfloat16, float, float); else RB(__nv_bfloat16, float, __nv_bfloat16); }
    else { if (dx_f32) RB(__nv_bfloat16, __nv_bfloat16, float); else RB(__nv_bfloat16, __nv_bfloat16, __nv_bfloat16); }
  }
#undef RB
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

// grid for the row-striding vector kernels: a few waves of 8-warp CTAs
int vec_grid(long long rows) {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  const long long want = (rows + 7) / 8;
  return static_cast<int>(std::min<long long>(want, 8LL * sms));
}

bool gated_vec_ok(const void* a, const void* b, long long ldb, int D) {
  const int al = D == 256 ? 16 : 8;
  return (D == 256 || D == 128) && reinterpret_cast<uintptr_t>(a) % al == 0 &&
         reinterpret_cast<uintptr_t>(b) % al == 0 && (ldb * 2) % al == 0;
}

int rmsnorm_gated_fwd(const void* o, const void* g, long long ldg, int H, const float* gamma, void* y, int y_f32,
                      float* rstd, long long rows, int D, float eps, cudaStream_t s) {
  if (!y_f32 && gated_vec_ok(o, g, ldg, D) && gated_vec_ok(y, y, D, D)) {
    if (D == 256)
      rmsnorm_gated_fwd_vec_k<8><<<vec_grid(rows), 256, 0, s>>>((const __nv_bfloat16*)o, (const __nv_bfloat16*)g,
                                                                ldg, H, gamma, (__nv_bfloat16*)y, rstd, rows, eps);
    else
      rmsnorm_gated_fwd_vec_k<4><<<vec_grid(rows), 256, 0, s>>>((const __nv_bfloat16*)o, (const __nv_bfloat16*)g,
                                                                ldg, H, gamma, (__nv_bfloat16*)y, rstd, rows, eps);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
  }
  if (y_f32)
    rmsnorm_gated_fwd_k<float><<<blocks_for(rows), 32 * ROWS_PER_CTA, 0, s>>>(
        (const __nv_bfloat16*)o, (const __nv_bfloat16*)g, ldg, H, gamma, (float*)y, rstd, rows, D, eps);
  else
    rmsnorm_gated_fwd_k<__nv_bfloat16><<<blocks_for(rows), 32 * ROWS_PER_CTA, 0, s>>>(
        (const __nv_bfloat16*)o, (const __nv_bfloat16*)g, ldg, H, gamma, (__nv_bfloat16*)y, rstd, rows, D, eps);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int rmsnorm_gated_bwd(const void* dy, const void* o, const void* g, long long ldg, int H, const float* gamma,
                      const float* rstd, void* dO, void* dG, long long lddg, float* dgamma, long long rows, int D,
                      cudaStream_t s) {
  if (gated_vec_ok(o, g, ldg, D) && gated_vec_ok(dy, dG, lddg, D) && gated_vec_ok(dO, dO, D, D)) {
    if (D == 256)
      rmsnorm_gated_bwd_vec_k<8><<<vec_grid(rows), 256, 0, s>>>(
          (const __nv_bfloat16*)dy, (const __nv_bfloat16*)o, (const __nv_bfloat16*)g, ldg, H, gamma, rstd,
          (__nv_bfloat16*)dO, (__nv_bfloat16*)dG, lddg, dgamma, rows);
    else
      rmsnorm_gated_bwd_vec_k<4><<<vec_grid(rows), 256, 0, s>>>(
          (const __nv_bfloat16*)dy, (const __nv_bfloat16*)o, (const __nv_bfloat16*)g, ldg, H, gamma, rstd,
          (__nv_bfloat16*)dO, (__nv_bfloat16*)dG, lddg, dgamma, rows);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
  }
  rmsnorm_gated_bwd_k<<<blocks_for(rows), 32 * ROWS_PER_CTA, D * sizeof(float), s>>>(
      (const __nv_bfloat16*)dy, (const __nv_bfloat16*)o, (const __nv_bfloat16*)g, ldg, H, gamma, rstd,
      (__nv_bfloat16*)dO, (__nv_bfloat16*)dG, lddg, dgamma, rows, D);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int qk_norm_rope_fwd(const void* x, const float* gamma, const float* cosv, const float* sinv, void* y, float* rstd,
                     long long rows, int L, int H, int D, float eps, long long ldx, long long ldy, cudaStream_t s) {
  const long long dense = static_cast<long long>(H) * D;
  if (ldx <= 0) ldx = dense;
  if (ldy <= 0) ldy = dense;
  const bool al = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15u) == 0 && ldx % 8 == 0 &&
                  ldy % 8 == 0;
  if (al && D == 64) {
    qk_norm_rope_fwd_v<64><<<vec_rope_grid(rows, 4), 256, 0, s>>>((const __nv_bfloat16*)x, gamma, cosv, sinv,
                                                                  (__nv_bfloat16*)y, rstd, rows, L, H, eps, ldx, ldy);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
  }
  if (al && D == 128) {
    qk_norm_rope_fwd_v<128><<<vec_rope_grid(rows, 2), 256, 0, s>>>((const __nv_bfloat16*)x, gamma, cosv, sinv,
                                                                   (__nv_bfloat16*)y, rstd, rows, L, H, eps, ldx, ldy);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
  }
  if (ldx != dense || ldy != dense) return 5;          // the row-per-warp kernel reads dense rows only
  qk_norm_rope_fwd_k<<<blocks_for(rows), 32 * ROWS_PER_CTA, 0, s>>>((const __nv_bfloat16*)x, gamma, cosv, sinv,
                                                                     (__nv_bfloat16*)y, rstd, rows, L, H, D, eps);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int qk_norm_rope_bwd(const void* dy, const void* x, const float* gamma, const float* cosv, const float* sinv,
                     const float* rstd, void* dx, float* dgamma, long long rows, int L, int H, int D, long long lddy,
                     long long ldx, long long lddx, cudaStream_t s) {
  const long long dense = static_cast<long long>(H) * D;
  if (lddy <= 0) lddy = dense;
  if (ldx <= 0) ldx = dense;
  if (lddx <= 0) lddx = dense;
  const bool al = ((reinterpret_cast<uintptr_t>(dy) | reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dx)) &
                   15u) == 0 && lddy % 8 == 0 && ldx % 8 == 0 && lddx % 8 == 0;
  if (al && D == 64) {
    qk_norm_rope_bwd_v<64><<<vec_rope_grid(rows, 4), 256, 0, s>>>((const __nv_bfloat16*)dy, (const __nv_bfloat16*)x,
                                                                  gamma, cosv, sinv, rstd, (__nv_bfloat16*)dx, dgamma,
                                                                  rows, L, H, lddy, ldx, lddx);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
  }
  if (al && D == 128) {
    qk_norm_rope_bwd_v<128><<<vec_rope_grid(rows, 2), 256, 0, s>>>((const __nv_bfloat16*)dy, (const __nv_bfloat16*)x,
                                                                   gamma, cosv, sinv, rstd, (__nv_bfloat16*)dx, dgamma,
                                                                   rows, L, H, lddy, ldx, lddx);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
  }
  if (lddy != dense || ldx != dense || lddx != dense) return 5;
  qk_norm_rope_bwd_k<<<blocks_for(rows), 32 * ROWS_PER_CTA, gamma ? D * sizeof(float) : 0, s>>>(
      (const __nv_bfloat16*)dy, (const __nv_bfloat16*)x, gamma, cosv, sinv, rstd, (__nv_bfloat16*)dx, dgamma, rows, L,
      H, D);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

}  // namespace vagus
