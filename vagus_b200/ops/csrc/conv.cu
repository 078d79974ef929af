// Fused causal depthwise short convolution + SiLU (+ per-head L2 norm) for
// the q / k / v streams of a gated delta-rule layer, forward and backward.
//
//   u[t, c] = sum_{i<K} w[c, K-1-i] x[t-i, c]     (zeros before the start)
//   z = silu(u);   y = z * rsqrt(sum_head z^2 + 1e-6)   (l2norm) or y = z
//
// One warp owns a strip of TPW consecutive tokens of one head; each lane owns
// VEC = head_dim / 32 adjacent channels (16-byte vector loads for head_dim
// 256) and slides along the strip keeping the last K inputs in registers.
// The head norm is a warp reduction (shuffles only).  The input may be a
// column block of a wider packed matrix (row pitch ldx); dx is written with
// its own pitch into the packed gradient.  Weight gradients are reduced over
// the 8 warps of a CTA in shared memory, then one atomic per (channel, tap).
#include "common.cuh"
#include "kernels.h"

namespace vagus {
namespace {

constexpr int TPW = 16;      // tokens per warp strip
constexpr int WARPS = 8;
constexpr int MAXK = 4;      // taps supported by the register window

template <int VEC>
__device__ __forceinline__ void load_vec(const __nv_bfloat16* p, float (&v)[VEC]) {
  if constexpr (VEC == 8) {
    const uint4 t = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) { const float2 f = unpack_bf16x2(w[j]); v[2 * j] = f.x; v[2 * j + 1] = f.y; }
  } else if constexpr (VEC == 4) {
    const uint2 t = *reinterpret_cast<const uint2*>(p);
    float2 f = unpack_bf16x2(t.x); v[0] = f.x; v[1] = f.y;
    f = unpack_bf16x2(t.y); v[2] = f.x; v[3] = f.y;
  } else {
#pragma unroll
    for (int j = 0; j < VEC; ++j) v[j] = bf2f(p[j]);
  }
}

template <int VEC>
__device__ __forceinline__ void store_vec(__nv_bfloat16* p, const float (&v)[VEC]) {
  if constexpr (VEC == 8) {
    uint4 t;
    t.x = pack_bf16x2(v[0], v[1]); t.y = pack_bf16x2(v[2], v[3]);
    t.z = pack_bf16x2(v[4], v[5]); t.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(p) = t;
  } else if constexpr (VEC == 4) {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
  } else {
#pragma unroll
    for (int j = 0; j < VEC; ++j) p[j] = f2bf(v[j]);
  }
}

template <int VEC, int K>
__global__ void __launch_bounds__(WARPS * 32)
conv_fwd_k(const __nv_bfloat16* __restrict__ x, long long ldx, const float* __restrict__ w,
           __nv_bfloat16* __restrict__ y, float* __restrict__ rnorm, long long L, int D, int l2) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const long long b = blockIdx.z;
  const int head = blockIdx.y;
  const int hd = VEC * 32;
  const int c0 = head * hd + lane * VEC;
  const long long t0 = ((long long)blockIdx.x * WARPS + warp) * TPW;
  if (t0 >= L) return;
  float wr[K][VEC];
#pragma unroll
  for (int j = 0; j < VEC; ++j)
#pragma unroll
    for (int i = 0; i < K; ++i) wr[i][j] = w[(long long)(c0 + j) * K + i];
  float hist[K][VEC];            // before token t is shifted in: hist[i] = x[t - 1 - i]
#pragma unroll
  for (int i = 0; i < K; ++i) {
    const long long t = t0 - 1 - i;
    if (t >= 0) load_vec<VEC>(x + (b * L + t) * ldx + c0, hist[i]);
    else
#pragma unroll
      for (int j = 0; j < VEC; ++j) hist[i][j] = 0.f;
  }
  const int nH = D / hd;
  const long long t_end = min(L, t0 + TPW);
  for (long long t = t0; t < t_end; ++t) {
#pragma unroll
    for (int i = K - 1; i > 0; --i)
#pragma unroll
      for (int j = 0; j < VEC; ++j) hist[i][j] = hist[i - 1][j];
    load_vec<VEC>(x + (b * L + t) * ldx + c0, hist[0]);
    float z[VEC];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      float u = 0.f;
#pragma unroll
      for (int i = 0; i < K; ++i) u += wr[K - 1 - i][j] * hist[i][j];
      z[j] = silu_f(u);
      ss += z[j] * z[j];
    }
    if (l2) {
      const float r = rsqrtf(warp_sum(ss) + 1e-6f);
#pragma unroll
      for (int j = 0; j < VEC; ++j) z[j] *= r;
      if (lane == 0) rnorm[(b * L + t) * nH + head] = r;
    }
    store_vec<VEC>(y + (b * L + t) * D + c0, z);
  }
}

template <int VEC, int K>
__global__ void __launch_bounds__(WARPS * 32)
conv_bwd_k(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x, long long ldx,
           const float* __restrict__ w, const float* __restrict__ rnorm, __nv_bfloat16* __restrict__ dx,
           long long lddx, float* __restrict__ dw, long long L, int D, int l2) {
  __shared__ float sdw[WARPS][VEC * 32 * K];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const long long b = blockIdx.z;
  const int head = blockIdx.y;
  const int hd = VEC * 32;
  const int c0 = head * hd + lane * VEC;
  const long long t0 = ((long long)blockIdx.x * WARPS + warp) * TPW;
  const int nH = D / hd;
  float wr[K][VEC];
#pragma unroll
  for (int j = 0; j < VEC; ++j)
#pragma unroll
    for (int i = 0; i < K; ++i) wr[i][j] = w[(long long)(c0 + j) * K + i];
  float dwp[K][VEC];
#pragma unroll
  for (int i = 0; i < K; ++i)
#pragma unroll
    for (int j = 0; j < VEC; ++j) dwp[i][j] = 0.f;
  if (t0 < L) {
    float xh[K][VEC];            // before token t is shifted in: xh[i] = x[t - 1 - i]
#pragma unroll
    for (int i = 0; i < K; ++i) {
      const long long t = t0 - 1 - i;
      if (t >= 0) load_vec<VEC>(x + (b * L + t) * ldx + c0, xh[i]);
      else
#pragma unroll
        for (int j = 0; j < VEC; ++j) xh[i][j] = 0.f;
    }
    float acc[K][VEC];           // acc[i] = pending dx of token t - i
#pragma unroll
    for (int i = 0; i < K; ++i)
#pragma unroll
      for (int j = 0; j < VEC; ++j) acc[i][j] = 0.f;
    const long long t_stop = min(L, t0 + TPW + K - 1);   // extra tokens feed dx of the strip's tail
    for (long long t = t0; t < t_stop; ++t) {
#pragma unroll
      for (int i = K - 1; i > 0; --i)
#pragma unroll
        for (int j = 0; j < VEC; ++j) { xh[i][j] = xh[i - 1][j]; acc[i][j] = acc[i - 1][j]; }
      load_vec<VEC>(x + (b * L + t) * ldx + c0, xh[0]);
      float g[VEC], u[VEC], s[VEC], z[VEC];
      load_vec<VEC>(dy + (b * L + t) * D + c0, g);
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        u[j] = 0.f;
#pragma unroll
        for (int i = 0; i < K; ++i) u[j] += wr[K - 1 - i][j] * xh[i][j];
        s[j] = sigmoid_f(u[j]);
        z[j] = u[j] * s[j];
        dot += g[j] * z[j];
      }
      if (l2) {
        const float r = rnorm[(b * L + t) * nH + head];
        dot = warp_sum(dot);
#pragma unroll
        for (int j = 0; j < VEC; ++j) g[j] = r * g[j] - r * r * r * z[j] * dot;
      }
      const bool in_strip = t < t0 + TPW;
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const float du = g[j] * s[j] * (1.f + u[j] * (1.f - s[j]));
        acc[0][j] = 0.f;
#pragma unroll
        for (int i = 0; i < K; ++i) acc[i][j] += wr[K - 1 - i][j] * du;
        if (in_strip)
#pragma unroll
          for (int i = 0; i < K; ++i) dwp[K - 1 - i][j] += du * xh[i][j];
      }
      const long long td = t - (K - 1);
      if (td >= t0 && td < t0 + TPW) store_vec<VEC>(dx + (b * L + td) * lddx + c0, acc[K - 1]);
    }
    // the strip's last K-1 tokens when the sequence ends inside the window
#pragma unroll
    for (int i = 0; i < K - 1; ++i) {
      const long long td = t_stop - 1 - i;
      if (t_stop == L && td >= t0 && td < t0 + TPW && td > t_stop - K) store_vec<VEC>(dx + (b * L + td) * lddx + c0, acc[i]);
    }
  }
  // reduce dw over the CTA's warps, then one atomic per (channel, tap)
#pragma unroll
  for (int i = 0; i < K; ++i)
#pragma unroll
    for (int j = 0; j < VEC; ++j) sdw[warp][(lane * VEC + j) * K + i] = dwp[i][j];
  __syncthreads();
  for (int e = threadIdx.x; e < hd * K; e += WARPS * 32) {
    float s = 0.f;
#pragma unroll
    for (int wi = 0; wi < WARPS; ++wi) s += sdw[wi][e];
    atomicAdd(&dw[(long long)head * hd * K + e], s);
  }
}

template <int VEC, int K>
void launch_fwd(const void* xp, long long ldx, const float* w, void* y, float* rnorm, long long B, long long L, int D,
                int l2, cudaStream_t st) {
  const int hd = VEC * 32;
  dim3 grid(static_cast<unsigned>((L + WARPS * TPW - 1) / (WARPS * TPW)), D / hd, static_cast<unsigned>(B));
  conv_fwd_k<VEC, K><<<grid, WARPS * 32, 0, st>>>((const __nv_bfloat16*)xp, ldx, w, (__nv_bfloat16*)y, rnorm, L, D, l2);
}

template <int VEC, int K>
void launch_bwd(const void* dy, const void* xp, long long ldx, const float* w, const float* rnorm, void* dx,
                long long lddx, float* dw, long long B, long long L, int D, int l2, cudaStream_t st) {
  const int hd = VEC * 32;
  dim3 grid(static_cast<unsigned>((L + WARPS * TPW - 1) / (WARPS * TPW)), D / hd, static_cast<unsigned>(B));
  conv_bwd_k<VEC, K><<<grid, WARPS * 32, 0, st>>>((const __nv_bfloat16*)dy, (const __nv_bfloat16*)xp, ldx, w, rnorm,
                                                   (__nv_bfloat16*)dx, lddx, dw, L, D, l2);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int conv_silu_fwd(const void* xp, long long ldx, const float* w, void* y, float* rnorm, long long B, long long L,
                  int D, int K, int head_dim, int l2norm, cudaStream_t st) {
  if (K != MAXK || D % head_dim) return 5;
  if (head_dim == 256 && aligned16(xp) && ldx % 8 == 0) launch_fwd<8, 4>(xp, ldx, w, y, rnorm, B, L, D, l2norm, st);
  else if (head_dim == 128 && ldx % 4 == 0) launch_fwd<4, 4>(xp, ldx, w, y, rnorm, B, L, D, l2norm, st);
  else if (head_dim == 64) launch_fwd<2, 4>(xp, ldx, w, y, rnorm, B, L, D, l2norm, st);
  else if (head_dim == 32) launch_fwd<1, 4>(xp, ldx, w, y, rnorm, B, L, D, l2norm, st);
  else return 5;
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int conv_silu_bwd(const void* dy, const void* xp, long long ldx, const float* w, const float* rnorm, void* dx,
                  long long lddx, float* dw, long long B, long long L, int D, int K, int head_dim, int l2norm,
                  cudaStream_t st) {
  if (K != MAXK || D % head_dim) return 5;
  if (head_dim == 256 && aligned16(xp) && ldx % 8 == 0 && lddx % 8 == 0 && aligned16(dx))
    launch_bwd<8, 4>(dy, xp, ldx, w, rnorm, dx, lddx, dw, B, L, D, l2norm, st);
  else if (head_dim == 128 && ldx % 4 == 0 && lddx % 4 == 0)
    launch_bwd<4, 4>(dy, xp, ldx, w, rnorm, dx, lddx, dw, B, L, D, l2norm, st);
  else if (head_dim == 64) launch_bwd<2, 4>(dy, xp, ldx, w, rnorm, dx, lddx, dw, B, L, D, l2norm, st);
  else if (head_dim == 32) launch_bwd<1, 4>(dy, xp, ldx, w, rnorm, dx, lddx, dw, B, L, D, l2norm, st);
  else return 5;
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

}  // namespace vagus
