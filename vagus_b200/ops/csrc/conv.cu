// Fused causal depthwise short convolution + SiLU (+ per-head L2 norm) for
// the q / k / v streams of a gated delta-rule layer, forward and backward.
//
//   u[t, c] = sum_{i<K} w[c, K-1-i] x[t-i, c]     (zeros before the start)
//   z = silu(u);   y = z * rsqrt(sum_head z^2 + 1e-6)   (l2norm) or y = z
//
// Grid: (token tiles of TT, heads, batch); block: one thread per channel of
// the head.  Each thread slides along its channel keeping the last K inputs
// in registers.  The input may be a column slice of a wider packed matrix
// (row pitch `ldx` elements), e.g. the q columns of the packed q|k|v|g
// projection; dx is written with its own pitch into the packed gradient.
#include "common.cuh"
#include "kernels.h"

namespace vagus {
namespace {

constexpr int TT = 64;       // tokens per CTA
constexpr int MAXK = 8;

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nw = blockDim.x / 32;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  return warp_sum(t);
}

// x: element (b, t, c) at x[(b*L + t) * ldx + c]; y contiguous (B, L, D)
__global__ void conv_fwd_k(const __nv_bfloat16* __restrict__ x, long long ldx, const float* __restrict__ w,
                           __nv_bfloat16* __restrict__ y, float* __restrict__ rnorm, long long L, int D, int K,
                           int hd, int l2) {
  __shared__ float red[32];
  const long long b = blockIdx.z;
  const int c = blockIdx.y * hd + threadIdx.x;
  const long long t0 = (long long)blockIdx.x * TT;
  float wr[MAXK];
#pragma unroll
  for (int j = 0; j < MAXK; ++j) wr[j] = j < K ? w[(long long)c * K + j] : 0.f;
  float hist[MAXK];   // before token t is inserted: hist[i] = x[t - 1 - i]
#pragma unroll
  for (int i = 0; i < MAXK; ++i) {
    const long long t = t0 - 1 - i;
    hist[i] = (i < K - 1 && t >= 0) ? bf2f(x[(b * L + t) * ldx + c]) : 0.f;
  }
  const int nH = D / hd;
  for (int tt = 0; tt < TT; ++tt) {
    const long long t = t0 + tt;
    if (t >= L) break;   // uniform across the block
#pragma unroll
    for (int i = MAXK - 1; i > 0; --i) hist[i] = hist[i - 1];
    hist[0] = bf2f(x[(b * L + t) * ldx + c]);
    float u = 0.f;
#pragma unroll
    for (int i = 0; i < MAXK; ++i) if (i < K) u += wr[K - 1 - i] * hist[i];
    const float z = silu_f(u);
    float out = z;
    if (l2) {
      const float ss = block_sum(z * z, red);
      const float r = rsqrtf(ss + 1e-6f);
      out = z * r;
      if (threadIdx.x == 0) rnorm[(b * L + t) * nH + blockIdx.y] = r;
    }
    y[(b * L + t) * D + c] = f2bf(out);
  }
}

__global__ void conv_bwd_k(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x, long long ldx,
                           const float* __restrict__ w, const float* __restrict__ rnorm,
                           __nv_bfloat16* __restrict__ dx, long long lddx, float* __restrict__ dw, long long L, int D,
                           int K, int hd, int l2) {
  __shared__ float red[32];
  const long long b = blockIdx.z;
  const int c = blockIdx.y * hd + threadIdx.x;
  const long long t0 = (long long)blockIdx.x * TT;
  const int nH = D / hd;
  float wr[MAXK];
#pragma unroll
  for (int j = 0; j < MAXK; ++j) wr[j] = j < K ? w[(long long)c * K + j] : 0.f;
  // du[t] for t in [t0, t0 + TT + K - 1): the dx of token t needs du[t .. t+K-1]
  // Recompute u from x: keep a rolling window.  Process tokens in order and
  // accumulate dx contributions into a small ring: dx[t - i] += w[K-1-i] du[t].
  float xh[MAXK];      // before token t is inserted: xh[i] = x[t - 1 - i]
#pragma unroll
  for (int i = 0; i < MAXK; ++i) {
    const long long t = t0 - 1 - i;
    xh[i] = (i < K - 1 && t >= 0) ? bf2f(x[(b * L + t) * ldx + c]) : 0.f;
  }
  float acc[MAXK];     // acc[i] = pending dx for token (t - i), i < K
#pragma unroll
  for (int i = 0; i < MAXK; ++i) acc[i] = 0.f;
  float dwp[MAXK];
#pragma unroll
  for (int j = 0; j < MAXK; ++j) dwp[j] = 0.f;
  const long long t_end = min(L, t0 + TT + K - 1);
  for (long long t = t0; t < t_end; ++t) {
#pragma unroll
    for (int i = MAXK - 1; i > 0; --i) { xh[i] = xh[i - 1]; acc[i] = acc[i - 1]; }
    xh[0] = bf2f(x[(b * L + t) * ldx + c]);
    acc[0] = 0.f;
    float u = 0.f;
#pragma unroll
    for (int i = 0; i < MAXK; ++i) if (i < K) u += wr[K - 1 - i] * xh[i];
    const float s = sigmoid_f(u);
    const float z = u * s;
    float dz = bf2f(dy[(b * L + t) * D + c]);
    if (l2) {
      const float r = rnorm[(b * L + t) * nH + blockIdx.y];
      const float dot = block_sum(dz * z, red);
      dz = r * dz - r * r * r * z * dot;
    }
    const float du = dz * s * (1.f + u * (1.f - s));
    // tokens beyond this CTA's range only contribute to dx of in-range tokens
#pragma unroll
    for (int i = 0; i < MAXK; ++i) if (i < K) acc[i] += wr[K - 1 - i] * du;
    if (t < t0 + TT) {
#pragma unroll
      for (int i = 0; i < MAXK; ++i) if (i < K) dwp[K - 1 - i] += du * xh[i];
    }
    // token t - (K-1) has received all its contributions
    const long long td = t - (K - 1);
    if (td >= t0 && td < t0 + TT) dx[(b * L + td) * lddx + c] = f2bf(acc[K - 1]);
  }
  // flush the last K-1 tokens of the range (their later taps fall beyond L)
  for (int i = K - 2; i >= 0; --i) {
    const long long td = t_end - 1 - i;
    if (td >= t0 && td < t0 + TT && td > t_end - 1 - (K - 1)) dx[(b * L + td) * lddx + c] = f2bf(acc[i]);
  }
#pragma unroll
  for (int j = 0; j < MAXK; ++j) if (j < K) atomicAdd(&dw[(long long)c * K + j], dwp[j]);
}

}  // namespace

int conv_silu_fwd(const void* xp, long long ldx, const float* w, void* y, float* rnorm, long long B, long long L,
                  int D, int K, int head_dim, int l2norm, cudaStream_t st) {
  if (K > MAXK || head_dim > 1024 || head_dim % 32 || D % head_dim) return 5;
  dim3 grid(static_cast<unsigned>((L + TT - 1) / TT), D / head_dim, static_cast<unsigned>(B));
  conv_fwd_k<<<grid, head_dim, 0, st>>>((const __nv_bfloat16*)xp, ldx, w, (__nv_bfloat16*)y, rnorm, L, D, K, head_dim,
                                         l2norm);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int conv_silu_bwd(const void* dy, const void* xp, long long ldx, const float* w, const float* rnorm, void* dx,
                  long long lddx, float* dw, long long B, long long L, int D, int K, int head_dim, int l2norm,
                  cudaStream_t st) {
  if (K > MAXK || head_dim > 1024 || head_dim % 32 || D % head_dim) return 5;
  dim3 grid(static_cast<unsigned>((L + TT - 1) / TT), D / head_dim, static_cast<unsigned>(B));
  conv_bwd_k<<<grid, head_dim, 0, st>>>((const __nv_bfloat16*)dy, (const __nv_bfloat16*)xp, ldx, w, rnorm,
                                         (__nv_bfloat16*)dx, lddx, dw, L, D, K, head_dim, l2norm);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

}  // namespace vagus
