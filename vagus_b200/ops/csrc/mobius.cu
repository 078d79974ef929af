// Mobius-map scan  x_t = (A_t x_{t-1} + B_t) / (C_t x_{t-1} + D_t),  t = 0..L-1,
// forward and backward, fp32, inputs (batch, L, R) contiguous (R = every
// trailing dim: heads, or heads x key channels) and x0 (batch, R).
//
// One CTA of 256 threads per (batch, tile of RT <= 8 sequences): RT
// consecutive sequences (one 32-byte sector per load) times SEG = 256 / RT
// segments of the time axis.  Three phases:
//   1. each thread composes its segment's steps into one 2x2 matrix (the
//      maps compose as matrix products; rescaled by a power of two every
//      step, since a scalar multiple of the matrix is the same map);
//   2. one thread per sequence walks the SEG segment maps to find every
//      segment's entry value (SEG Mobius applications);
//   3. each thread replays its segment's exact recurrence from its entry
//      value and writes x_t.
// The backward is the same three phases on the adjoint, a first-order linear
// recurrence run from the end: with den_t = C_t x_{t-1} + D_t,
//   g_t = dL/dx_t = go_t + y_{t+1},   y_t = g_t (A_t - C_t x_t) / den_t
// (y_t is what step t passes back to x_{t-1}; y_L = 0, dL/dx0 = y_0), and
//   dA_t = g_t x_{t-1} / den_t   dB_t = g_t / den_t
//   dC_t = -g_t x_t x_{t-1} / den_t   dD_t = -g_t x_t / den_t.
// A segment's adjoint is affine in the y entering from its right: phase 1
// composes (P, Q) with y_lo = Q + P y_hi.
// Reference behaviour: infra/components/kalman_delta.py:79-128 (a log-depth
// prefix product in torch); the recurrence itself is the definition.
#include "common.cuh"
#include "kernels.h"

namespace vagus {
namespace {

constexpr int MT = 256;

// 2^(127 - E) for a float of biased exponent E: brings mx into [1, 2) by an
// exact power-of-two scale (no rounding); 1 for zero / subnormal / huge mx.
__device__ __forceinline__ float pow2_scale(float mx) {
  const int e = (__float_as_int(mx) >> 23) & 0xff;
  return (e >= 1 && e <= 253) ? __int_as_float((254 - e) << 23) : 1.f;
}

struct Tile {
  int rl, s, seg, r, lo, hi;
  long long base;     // offset of (b, t = 0, r)
};

__device__ __forceinline__ Tile tile_of(int L, int R, int RT) {
  Tile t;
  t.rl = threadIdx.x % RT;
  t.s = threadIdx.x / RT;
  t.seg = MT / RT;
  t.r = blockIdx.x * RT + t.rl;
  const int Ls = (L + t.seg - 1) / t.seg;
  t.lo = min(L, t.s * Ls);
  t.hi = min(L, t.lo + Ls);
  t.base = (long long)blockIdx.y * L * R + t.r;
  return t;
}

__global__ void __launch_bounds__(MT)
mobius_fwd_k(const float* __restrict__ A, const float* __restrict__ Bm, const float* __restrict__ C,
             const float* __restrict__ D, const float* __restrict__ x0, float* __restrict__ X, int L, int R, int RT) {
  __shared__ float4 ms[MT];
  __shared__ float xs[MT];
  const Tile T = tile_of(L, R, RT);
  const bool live = T.r < R;
  float m00 = 1.f, m01 = 0.f, m10 = 0.f, m11 = 1.f;
  if (live) {
#pragma unroll 4
    for (int t = T.lo; t < T.hi; ++t) {
      const long long o = T.base + (long long)t * R;
      const float a = A[o], b = Bm[o], c = C[o], d = D[o];
      const float n00 = fmaf(a, m00, b * m10), n01 = fmaf(a, m01, b * m11);
      const float n10 = fmaf(c, m00, d * m10), n11 = fmaf(c, m01, d * m11);
      const float sc = pow2_scale(fmaxf(fmaxf(fabsf(n00), fabsf(n01)), fmaxf(fabsf(n10), fabsf(n11))));
      m00 = n00 * sc; m01 = n01 * sc; m10 = n10 * sc; m11 = n11 * sc;
    }
  }
  ms[threadIdx.x] = make_float4(m00, m01, m10, m11);
  __syncthreads();
  if (T.s == 0 && live) {
    float x = x0[(long long)blockIdx.y * R + T.r];
    for (int s = 0; s < T.seg; ++s) {
      xs[s * RT + T.rl] = x;
      const float4 m = ms[s * RT + T.rl];
      x = fmaf(m.x, x, m.y) / fmaf(m.z, x, m.w);
    }
  }
  __syncthreads();
  if (!live) return;
  float x = xs[threadIdx.x];
#pragma unroll 4
  for (int t = T.lo; t < T.hi; ++t) {
    const long long o = T.base + (long long)t * R;
    x = fmaf(A[o], x, Bm[o]) / fmaf(C[o], x, D[o]);
    if (VAGUS_CHECK(o, (long long)gridDim.y * L * R)) X[o] = x;
  }
}

__global__ void __launch_bounds__(MT)
mobius_bwd_k(const float* __restrict__ A, const float* __restrict__ Bm, const float* __restrict__ C,
             const float* __restrict__ D, const float* __restrict__ x0, const float* __restrict__ X,
             const float* __restrict__ gO, float* __restrict__ gA, float* __restrict__ gB, float* __restrict__ gC,
             float* __restrict__ gD, float* __restrict__ gx0, int L, int R, int RT) {
  __shared__ float2 ps[MT];
  __shared__ float ys[MT];
  const Tile T = tile_of(L, R, RT);
  const bool live = T.r < R;
  const float xin = live ? x0[(long long)blockIdx.y * R + T.r] : 0.f;
  // phase 1: y_lo = Q + P * y_hi over the segment, from its right end
  float P = 1.f, Q = 0.f;
  if (live) {
#pragma unroll 4
    for (int t = T.hi - 1; t >= T.lo; --t) {
      const long long o = T.base + (long long)t * R;
      const float xp = t > 0 ? X[o - R] : xin, xt = X[o];
      const float lam = (A[o] - C[o] * xt) / fmaf(C[o], xp, D[o]);
      Q = lam * (gO[o] + Q);
      P = lam * P;
    }
  }
  ps[threadIdx.x] = make_float2(P, Q);
  __syncthreads();
  if (T.s == 0 && live) {
    float y = 0.f;
    for (int s = T.seg - 1; s >= 0; --s) {
      ys[s * RT + T.rl] = y;
      const float2 pq = ps[s * RT + T.rl];
      y = fmaf(pq.x, y, pq.y);
    }
    gx0[(long long)blockIdx.y * R + T.r] = y;
  }
  __syncthreads();
  if (!live) return;
  float y = ys[threadIdx.x];
#pragma unroll 4
  for (int t = T.hi - 1; t >= T.lo; --t) {
    const long long o = T.base + (long long)t * R;
    const float xp = t > 0 ? X[o - R] : xin, xt = X[o];
    const float a = A[o], c = C[o];
    const float inv = 1.f / fmaf(c, xp, D[o]);
    const float g = gO[o] + y;
    const float gi = g * inv;
    gA[o] = gi * xp;
    gB[o] = gi;
    gC[o] = -gi * xt * xp;
    gD[o] = -gi * xt;
    y = gi * (a - c * xt);
  }
}

// 8 sequences per tile: a warp's load covers 4 segments x one 32-byte sector,
// and a (batch 8, 512-sequence) problem gets 512 CTAs of 32 segments each
// (32 sequences per tile gave 128 CTAs of 512-step segments: latency-bound).
int rt_of(int R) {
  int rt = 1;
  while (rt < R && rt < 8) rt *= 2;
  return rt;
}

}  // namespace

int mobius_fwd(const float* A, const float* B, const float* C, const float* D, const float* x0, float* X, int batch,
               int L, int R, cudaStream_t st) {
  if (batch == 0 || R == 0 || L == 0) return 0;
  const int rt = rt_of(R);
  mobius_fwd_k<<<dim3((R + rt - 1) / rt, batch), MT, 0, st>>>(A, B, C, D, x0, X, L, R, rt);
  return (int)cudaGetLastError();
}

int mobius_bwd(const float* A, const float* B, const float* C, const float* D, const float* x0, const float* X,
               const float* gO, float* gA, float* gB, float* gC, float* gD, float* gx0, int batch, int L, int R,
               cudaStream_t st) {
  if (batch == 0 || R == 0) return 0;
  const int rt = rt_of(R);
  mobius_bwd_k<<<dim3((R + rt - 1) / rt, batch), MT, 0, st>>>(A, B, C, D, x0, X, gO, gA, gB, gC, gD, gx0, L, R,
                                                               rt);
  return (int)cudaGetLastError();
}

}  // namespace vagus
