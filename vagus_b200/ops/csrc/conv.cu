// Fused causal depthwise short convolution + SiLU (+ per-head L2 norm) for
// the q / k / v streams of a gated delta-rule layer, forward and backward.
//
//   u[t, c] = sum_{i<K} w[c, K-1-i] x[t-i, c]     (zeros before the start)
//   z = silu(u);   y = z * rsqrt(sum_head z^2 + 1e-6)   (l2norm) or y = z
//
// Tiling: a CTA (8 warps) owns a tile of T consecutive tokens of one head.
// The tile's input rows (plus K - 1 rows of left context, and in the backward
// K - 1 rows of right context) are staged in shared memory with cp.async, so
// every byte the tile needs is in flight at once without costing registers;
// then each warp takes whole token rows, one lane per VEC = head_dim / 32
// adjacent channels, and the head norm is a warp reduction.  The input may be
// a column block of a wider packed matrix (row pitch ldx); dx is written with
// its own pitch into the packed gradient.
//
// Backward, heads of 128 / 256: warp pairs walk runs of tokens in registers,
// four tokens per step (conv_bwd_step_k below).  Other head dims: phase 1
// recomputes u, z and forms du = dL/du for T + K - 1 rows into shared memory
// (fp32); phase 2 gives dx[t] = sum_i w[K-1-i] du[t+i] and accumulates dw in
// registers; CTAs are persistent over the tiles of their (batch, head), so dw
// is reduced over warps in shared memory and added with one atomic per
// (channel, tap) per CTA.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <cstdlib>

namespace vagus {
namespace {

constexpr int WARPS = 8;
constexpr int THREADS = WARPS * 32;
constexpr int MAXK = 4;       // taps supported by the register window
constexpr int TF = 64;        // forward tile (tokens)
constexpr int TB = 32;        // backward tile (tokens)

template <int VEC>
__device__ __forceinline__ void lds_vec(const __nv_bfloat16* p, float (&v)[VEC]) {
  if constexpr (VEC == 8) {
    const uint4 t = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) { const float2 f = unpack_bf16x2(w[j]); v[2 * j] = f.x; v[2 * j + 1] = f.y; }
  } else if constexpr (VEC == 4) {
    const uint2 t = *reinterpret_cast<const uint2*>(p);
    float2 f = unpack_bf16x2(t.x); v[0] = f.x; v[1] = f.y;
    f = unpack_bf16x2(t.y); v[2] = f.x; v[3] = f.y;
  } else if constexpr (VEC == 2) {
    const float2 f = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(p));
    v[0] = f.x; v[1] = f.y;
  } else {
    v[0] = bf2f(p[0]);
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
  } else if constexpr (VEC == 2) {
    *reinterpret_cast<uint32_t*>(p) = pack_bf16x2(v[0], v[1]);
  } else {
    p[0] = f2bf(v[0]);
  }
}

// 16-byte global -> shared copy; reads nothing and writes zeros when !ok.
__device__ __forceinline__ void cp16(void* s, const void* g, bool ok) {
  const uint32_t sa = static_cast<uint32_t>(__cvta_generic_to_shared(s));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sa), "l"(g), "r"(ok ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_commit_wait() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

// rows [t_first, t_first + rows) of one head (HD channels) into s[row][HD];
// rows outside [0, L) are zero.
template <int HD>
__device__ __forceinline__ void stage_rows(__nv_bfloat16* s, const __nv_bfloat16* g, long long pitch, long long b,
                                           long long L, long long t_first, int rows, int c_base) {
  constexpr int CPR = HD / 8;
  for (int i = threadIdx.x; i < rows * CPR; i += THREADS) {
    const int r = i / CPR, cc = i - r * CPR;
    const long long t = t_first + r;
    const bool ok = t >= 0 && t < L;
    cp16(s + r * HD + cc * 8, g + (b * L + (ok ? t : 0)) * pitch + c_base + cc * 8, ok);
  }
}

// The head's taps, transposed into shared memory as ws[tap][channel]: thread
// c loads channel c's K taps (one coalesced 16-byte load per thread) and a
// lane then reads its VEC channels of each tap as contiguous vectors.
// Loading them per lane straight from global memory costs one 32-sector
// request per tap per warp.
template <int HD, int K>
__device__ __forceinline__ void stage_weights(float* ws, const float* __restrict__ w, int c_base) {
  static_assert(K == 4 && HD <= THREADS, "one float4 of taps per channel");
  if (threadIdx.x < HD) {
    const float4 v = *reinterpret_cast<const float4*>(w + (long long)(c_base + threadIdx.x) * K);
    ws[0 * HD + threadIdx.x] = v.x;
    ws[1 * HD + threadIdx.x] = v.y;
    ws[2 * HD + threadIdx.x] = v.z;
    ws[3 * HD + threadIdx.x] = v.w;
  }
}

template <int VEC, int K>
__device__ __forceinline__ void read_weights(const float* ws, int cl, float (&wr)[K][VEC]) {
  constexpr int HD = VEC * 32;
#pragma unroll
  for (int i = 0; i < K; ++i)
#pragma unroll
    for (int j = 0; j < VEC; ++j) wr[i][j] = ws[i * HD + cl + j];
}

template <int VEC, int K, int MINB>
__global__ void __launch_bounds__(THREADS, MINB)
conv_fwd_k(const __nv_bfloat16* __restrict__ x, long long ldx, const float* __restrict__ w,
           __nv_bfloat16* __restrict__ y, float* __restrict__ rnorm, long long L, int D, int l2) {
  constexpr int HD = VEC * 32;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* ws = reinterpret_cast<float*>(smem_raw);                     // [HD][K]
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(ws + HD * K);  // [TF + K - 1][HD]
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const long long b = blockIdx.z;
  const int head = blockIdx.y;
  const int nH = D / HD;
  const long long t0 = (long long)blockIdx.x * TF;
  stage_weights<HD, K>(ws, w, head * HD);
  stage_rows<HD>(xs, x, ldx, b, L, t0 - (K - 1), TF + K - 1, head * HD);
  cp_commit_wait();
  __syncthreads();
  float wr[K][VEC];
  read_weights<VEC, K>(ws, lane * VEC, wr);
  // each warp walks RW consecutive tokens with the last K - 1 inputs kept
  // unpacked in registers: one shared load per token
  constexpr int RW = TF / WARPS;
  const int r0 = warp * RW;
  float win[K - 1][VEC];                    // win[i] = x[t - 1 - i]; token t0 + r is tile row r + K - 1
#pragma unroll
  for (int i = 0; i < K - 1; ++i) lds_vec<VEC>(xs + (r0 + K - 2 - i) * HD + lane * VEC, win[i]);
#pragma unroll
  for (int rr = 0; rr < RW; ++rr) {
    const int r = r0 + rr;
    float xc[VEC], u[VEC];
    lds_vec<VEC>(xs + (r + K - 1) * HD + lane * VEC, xc);
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      u[j] = wr[K - 1][j] * xc[j];
#pragma unroll
      for (int i = 0; i < K - 1; ++i) u[j] += wr[K - 2 - i][j] * win[i][j];
    }
#pragma unroll
    for (int i = K - 2; i > 0; --i)
#pragma unroll
      for (int j = 0; j < VEC; ++j) win[i][j] = win[i - 1][j];
#pragma unroll
    for (int j = 0; j < VEC; ++j) win[0][j] = xc[j];
    const long long t = t0 + r;
    if (t < L) {                            // warp-uniform
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < VEC; ++j) { u[j] = silu_f(u[j]); ss += u[j] * u[j]; }
      if (l2) {
        const float rn = rsqrtf(warp_sum(ss) + 1e-6f);
#pragma unroll
        for (int j = 0; j < VEC; ++j) u[j] *= rn;
        if (lane == 0 && VAGUS_CHECK((b * L + t) * nH + head, (long long)gridDim.z * L * nH))
          rnorm[(b * L + t) * nH + head] = rn;
      }
      if (VAGUS_CHECK((b * L + t) * D + head * HD + lane * VEC + VEC - 1, (long long)gridDim.z * L * D))
        store_vec<VEC>(y + (b * L + t) * D + head * HD + lane * VEC, u);
    }
  }
}

template <int VEC, int K>
constexpr int bwd_smem_bytes() {
  constexpr int HD = VEC * 32;
  return HD * K * 4 + (TB + 2 * (K - 1)) * HD * 2 + (TB + K - 1) * HD * 2 + (TB + K - 1) * HD * 4;
}

template <int VEC, int K>
__global__ void __launch_bounds__(THREADS, 2)
conv_bwd_k(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x, long long ldx,
           const float* __restrict__ w, const float* __restrict__ rnorm, __nv_bfloat16* __restrict__ dx,
           long long lddx, float* __restrict__ dw, long long L, int D, int l2) {
  constexpr int HD = VEC * 32;
  constexpr int XR = TB + 2 * (K - 1);      // x rows: tokens [t0 - K + 1, t0 + TB + K - 1)
  constexpr int GR = TB + K - 1;            // dy / du rows: tokens [t0, t0 + TB + K - 1)
  static_assert(WARPS * K <= GR, "dw reduction reuses the du buffer");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* ws = reinterpret_cast<float*>(smem_raw);
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(ws + HD * K);
  __nv_bfloat16* gs = xs + XR * HD;
  float* dus = reinterpret_cast<float*>(gs + GR * HD);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const long long b = blockIdx.z;
  const int head = blockIdx.y;
  const int nH = D / HD;
  const int cl = lane * VEC;                  // lane's first channel within the head
  stage_weights<HD, K>(ws, w, head * HD);
  cp_commit_wait();
  __syncthreads();
  float wr[K][VEC];
  read_weights<VEC, K>(ws, cl, wr);
  float dwa[K][VEC];
#pragma unroll
  for (int k = 0; k < K; ++k)
#pragma unroll
    for (int j = 0; j < VEC; ++j) dwa[k][j] = 0.f;
  constexpr int RW = TB / WARPS;
  static_assert(TB % WARPS == 0 && K - 1 <= WARPS, "tile split");
  const int r0 = warp * RW;
  float win[K - 1][VEC];
  // du rows in shared memory: float4 groups interleaved across lanes so a
  // warp's 16-byte accesses are conflict-free
  auto du_at = [&](int r, int j) -> float* {
    if constexpr (VEC >= 4) return dus + r * HD + (j / 4) * 128 + lane * 4 + (j % 4);
    else return dus + r * HD + cl + j;
  };
  auto du_load = [&](int r, float (&v)[VEC]) {
#pragma unroll
    for (int j = 0; j < VEC; ++j) v[j] = *du_at(r, j);
  };
  long long t0 = 0;
  auto du_row = [&](int r, float (&u)[VEC]) {
    const long long t = t0 + r;
    float g[VEC], s[VEC], z[VEC];
    lds_vec<VEC>(gs + r * HD + cl, g);
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      s[j] = sigmoid_f(u[j]);
      z[j] = u[j] * s[j];
      dot += g[j] * z[j];
    }
    if (l2) {
      const float rn = t < L ? rnorm[(b * L + t) * nH + head] : 0.f;
      dot = warp_sum(dot);
      const float c3 = rn * rn * rn * dot;
#pragma unroll
      for (int j = 0; j < VEC; ++j) g[j] = rn * g[j] - c3 * z[j];
    }
#pragma unroll
    for (int j = 0; j < VEC; ++j) *du_at(r, j) = g[j] * s[j] * (1.f + u[j] * (1.f - s[j]));
  };
  const long long tiles = (L + TB - 1) / TB;
  for (long long tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    t0 = tile * TB;
    stage_rows<HD>(xs, x, ldx, b, L, t0 - (K - 1), XR, head * HD);
    stage_rows<HD>(gs, dy, D, b, L, t0, GR, head * HD);
    cp_commit_wait();
    __syncthreads();
    // phase 1: du for tokens t0 + r, r < GR (zero past the end: dy is zero
    // there).  Rows 0 .. TB-1 in runs of RW per warp with a sliding input
    // window; the K - 1 right-context rows go to the first warps.
#pragma unroll
    for (int i = 0; i < K - 1; ++i) lds_vec<VEC>(xs + (r0 + K - 2 - i) * HD + cl, win[i]);
#pragma unroll
    for (int rr = 0; rr < RW; ++rr) {
      const int r = r0 + rr;
      float xc[VEC], u[VEC];
      lds_vec<VEC>(xs + (r + K - 1) * HD + cl, xc);
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        u[j] = wr[K - 1][j] * xc[j];
#pragma unroll
        for (int i = 0; i < K - 1; ++i) u[j] += wr[K - 2 - i][j] * win[i][j];
      }
#pragma unroll
      for (int i = K - 2; i > 0; --i)
#pragma unroll
        for (int j = 0; j < VEC; ++j) win[i][j] = win[i - 1][j];
#pragma unroll
      for (int j = 0; j < VEC; ++j) win[0][j] = xc[j];
      du_row(r, u);
    }
    if (warp < K - 1) {
      const int r = TB + warp;
      float u[VEC];
#pragma unroll
      for (int j = 0; j < VEC; ++j) u[j] = 0.f;
#pragma unroll
      for (int i = 0; i < K; ++i) {
        float xv[VEC];
        lds_vec<VEC>(xs + (r + K - 1 - i) * HD + cl, xv);
#pragma unroll
        for (int j = 0; j < VEC; ++j) u[j] += wr[K - 1 - i][j] * xv[j];
      }
      du_row(r, u);
    }
    __syncthreads();
    // phase 2: dx and dw for the tile's own tokens
#pragma unroll
    for (int rr = 0; rr < RW; ++rr) {
      const int r = r0 + rr;
      const long long t = t0 + r;
      if (t < L) {
        float acc[VEC], d0[VEC];
#pragma unroll
        for (int j = 0; j < VEC; ++j) acc[j] = 0.f;
#pragma unroll
        for (int i = 0; i < K; ++i) {           // du[t + i] weighted by w[K-1-i]
          float dv[VEC];
          du_load(r + i, dv);
          if (i == 0)
#pragma unroll
            for (int j = 0; j < VEC; ++j) d0[j] = dv[j];
#pragma unroll
          for (int j = 0; j < VEC; ++j) acc[j] += wr[K - 1 - i][j] * dv[j];
        }
        store_vec<VEC>(dx + (b * L + t) * lddx + head * HD + cl, acc);
#pragma unroll
        for (int k = 0; k < K; ++k) {           // x[t - (K-1-k)] sits at x row r + k
          float xv[VEC];
          lds_vec<VEC>(xs + (r + k) * HD + cl, xv);
#pragma unroll
          for (int j = 0; j < VEC; ++j) dwa[k][j] += d0[j] * xv[j];
        }
      }
    }
    __syncthreads();
  }
  // reduce dw over the warps (reusing the du buffer), one atomic per (channel, tap)
  float* red = dus;                           // [WARPS][K][HD]
#pragma unroll
  for (int k = 0; k < K; ++k)
#pragma unroll
    for (int j = 0; j < VEC; ++j) red[(warp * K + k) * HD + cl + j] = dwa[k][j];
  __syncthreads();
  for (int idx = threadIdx.x; idx < HD * K; idx += THREADS) {
    const int c = idx / K, k = idx - c * K;
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < WARPS; ++q) s += red[(q * K + k) * HD + c];
    atomicAdd(&dw[(long long)(head * HD + c) * K + k], s);
  }
}

// ------------------------------------------------- backward, token runs --
// For heads of 128 / 256 channels: a pair of warps (64 lanes, VEC = HD / 64
// channels each) walks a run of consecutive tokens once, U = 4 tokens per
// step, with the last K - 1 inputs and the last K - 1 values of du = dL/du in
// registers:
//   token t:  u(t) from x[t-3..t];  du(t) through the L2 norm (the head's dot
//             product is a warp sum plus one exchange between the pair's two
//             warps, once per step for the step's U tokens) and SiLU;
//             dw[k] += du(t) x[t-3+k] for the run's own tokens;
//             dx[t-3] = sum_i w[3-i] du(t-3+i) is then complete.
// The U tokens' chains interleave.  x and dy come straight from global memory
// (each warp pair's row is one contiguous 2 * HD-byte segment) two steps ahead,
// in two register sets that alternate between the steps, so the prefetch queue
// costs no register moves; the run's K - 1 right-context tokens are recomputed.
// Token offsets inside a run are 32-bit and the pointers advance per step.
// Per element only x, g f and z f stay live across the exchange, where
// z = silu(u) and f = silu'(u) = s (1 + u - z):  du = rn g f - c3 z f with
// c3 = rn^3 <g, z>_head under the L2 norm, du = g f without it.  dw is summed
// over the CTA's pairs in shared memory and added with one atomic per
// (channel, tap) per CTA.

template <int VEC>
__device__ __forceinline__ void ldg_row(const __nv_bfloat16* p, bool ok, uint32_t (&r)[VEC / 2]) {
  if constexpr (VEC == 4) {
    uint2 t = ok ? __ldg(reinterpret_cast<const uint2*>(p)) : make_uint2(0u, 0u);
    r[0] = t.x; r[1] = t.y;
  } else {
    r[0] = ok ? __ldg(reinterpret_cast<const unsigned int*>(p)) : 0u;
  }
}

template <int VEC>
__device__ __forceinline__ void unpack_row(const uint32_t (&r)[VEC / 2], float (&v)[VEC]) {
#pragma unroll
  for (int j = 0; j < VEC / 2; ++j) {
    const float2 f = unpack_bf16x2(r[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}

template <int VEC, int U, int NT, int MINB>
__global__ void __launch_bounds__(NT, MINB)
conv_bwd_step_k(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x, long long ldx,
                const float* __restrict__ w, const float* __restrict__ rnorm, __nv_bfloat16* __restrict__ dx,
                long long lddx, float* __restrict__ dw, long long L, int D, int l2, int run_len) {
  constexpr int K = 4;
  constexpr int HD = VEC * 64;
  constexpr int PAIRS = NT / 64;
  __shared__ float dot_x[PAIRS][2][2][U];     // [pair][warp of the pair][step parity][token]
  __shared__ float red[PAIRS][K][HD];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int pair = warp >> 1, half = warp & 1;
  const int ch = (half * 32 + lane) * VEC;   // first channel of this thread within the head
  const long long b = blockIdx.z;
  const int head = blockIdx.y;
  const int nH = D / HD;
  const int c0 = head * HD + ch;
  float wr[K][VEC];
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
    const float4 t = *reinterpret_cast<const float4*>(w + (long long)(c0 + j) * K);
    wr[0][j] = t.x; wr[1][j] = t.y; wr[2][j] = t.z; wr[3][j] = t.w;
  }
  float dwa[K][VEC];
#pragma unroll
  for (int k = 0; k < K; ++k)
#pragma unroll
    for (int j = 0; j < VEC; ++j) dwa[k][j] = 0.f;
  const long long runs = (L + run_len - 1) / run_len;
  const int bar = 1 + pair;                  // named barrier of this warp pair (0 is __syncthreads)
  const __nv_bfloat16* xb = x + b * L * ldx + c0;
  const __nv_bfloat16* gb = dy + b * L * D + c0;
  int par = 0;
  for (long long run = (long long)blockIdx.x * PAIRS + pair; run < runs; run += (long long)gridDim.x * PAIRS) {
    const long long t0 = run * run_len;
    // token offsets within the run are 32-bit: m = t - t0
    const int n_end = static_cast<int>(min(L, t0 + run_len) - t0);          // the run's own tokens
    const int n_load = static_cast<int>(min(L, t0 + run_len + K - 1) - t0); // du is needed below this
    const __nv_bfloat16* xr = xb + t0 * ldx;
    const __nv_bfloat16* gr = gb + t0 * D;
    const float* rr = l2 ? rnorm + (b * L + t0) * nH + head : nullptr;
    __nv_bfloat16* dxr = dx + (b * L + t0) * lddx + c0;
    float xw[K - 1][VEC], dw3[K - 1][VEC];             // x and du of the 1st .. 3rd token before the step
#pragma unroll
    for (int i = 0; i < K - 1; ++i) {
      uint32_t r[VEC / 2];
      ldg_row<VEC>(xr - (long long)(1 + i) * ldx, t0 - 1 - i >= 0, r);
      unpack_row<VEC>(r, xw[i]);
#pragma unroll
      for (int j = 0; j < VEC; ++j) dw3[i][j] = 0.f;
    }
    uint32_t ax[U][VEC / 2], ag[U][VEC / 2], bx[U][VEC / 2], bg[U][VEC / 2];
    auto load_step = [&](uint32_t (&qx)[U][VEC / 2], uint32_t (&qg)[U][VEC / 2], int ms) {
      const __nv_bfloat16* px = xr + (long long)ms * ldx;
      const __nv_bfloat16* pg = gr + (long long)ms * D;
#pragma unroll
      for (int i = 0; i < U; ++i) {
        const bool ok = ms + i < n_load;
        ldg_row<VEC>(px, ok, qx[i]);
        ldg_row<VEC>(pg, ok, qg[i]);
        px += ldx;
        pg += D;
      }
    };
    // one step: du of tokens ms .. ms + U - 1, dx of tokens ms - 3 .. ms + U - 4 (run offsets)
    auto step = [&](uint32_t (&qx)[U][VEC / 2], uint32_t (&qg)[U][VEC / 2], int ms) {
      float xc[U][VEC], gf[U][VEC], zf[U][VEC], dot[U], rn[U];
#pragma unroll
      for (int i = 0; i < U; ++i) {
        unpack_row<VEC>(qx[i], xc[i]);
        unpack_row<VEC>(qg[i], gf[i]);
        // past n_load du is never used: rn only has to be finite there
        rn[i] = l2 && ms + i < n_load ? __ldg(rr + (ms + i) * nH) : 0.f;
      }
      load_step(qx, qg, ms + 2 * U);                   // refill this set two steps ahead
      // x of token ms + m for m in [-3, U)
      auto X = [&](int m, int j) -> float { return m >= 0 ? xc[m][j] : xw[-1 - m][j]; };
#pragma unroll
      for (int i = 0; i < U; ++i) {
        dot[i] = 0.f;
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const float u = wr[3][j] * X(i, j) + wr[2][j] * X(i - 1, j) + wr[1][j] * X(i - 2, j) + wr[0][j] * X(i - 3, j);
          const float sg = sigmoid_f(u);
          const float z = u * sg;
          const float f = sg * (1.f + u - z);
          dot[i] += gf[i][j] * z;
          gf[i][j] *= f;
          zf[i][j] = z * f;
        }
      }
      if (l2) {
#pragma unroll
        for (int o = 1; o < 32; o <<= 1)
#pragma unroll
          for (int i = 0; i < U; ++i) dot[i] += __shfl_xor_sync(0xffffffffu, dot[i], o);
        if (lane == 0)
#pragma unroll
          for (int i = 0; i < U; ++i) dot_x[pair][half][par][i] = dot[i];
        asm volatile("bar.sync %0, 64;" ::"r"(bar) : "memory");
#pragma unroll
        for (int i = 0; i < U; ++i) {
          const float c3 = rn[i] * rn[i] * rn[i] * (dot[i] + dot_x[pair][half ^ 1][par][i]);
#pragma unroll
          for (int j = 0; j < VEC; ++j) gf[i][j] = rn[i] * gf[i][j] - c3 * zf[i][j];     // du
        }
        par ^= 1;
      }
#pragma unroll
      for (int i = 0; i < U; ++i) {
        if (ms + i < n_end) {                          // the run's own token: weight gradient
#pragma unroll
          for (int k = 0; k < K; ++k)
#pragma unroll
            for (int j = 0; j < VEC; ++j) dwa[k][j] += gf[i][j] * X(i - (K - 1) + k, j);
        }
      }
      // du of token ms + m for m in [-3, U)
      auto DU = [&](int m, int j) -> float { return m >= 0 ? gf[m][j] : dw3[-1 - m][j]; };
      __nv_bfloat16* pd = dxr + (long long)(ms - (K - 1)) * lddx;
#pragma unroll
      for (int i = 0; i < U; ++i, pd += lddx) {
        const int sm = ms - (K - 1) + i;               // dx[sm] needs du(sm .. sm + 3)
        if (sm >= 0 && sm < n_end) {
          float o[VEC];
#pragma unroll
          for (int j = 0; j < VEC; ++j)
            o[j] = wr[3][j] * DU(i - 3, j) + wr[2][j] * DU(i - 2, j) + wr[1][j] * DU(i - 1, j) + wr[0][j] * DU(i, j);
          if (VAGUS_CHECK((b * L + t0 + sm) * lddx + c0 + VEC - 1, (long long)gridDim.z * L * lddx)) {
            if constexpr (VEC == 4)
              *reinterpret_cast<uint2*>(pd) = make_uint2(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]));
            else
              *reinterpret_cast<uint32_t*>(pd) = pack_bf16x2(o[0], o[1]);
          }
        }
      }
      // slide the windows by U tokens (highest index first: it reads the lower, older entries)
#pragma unroll
      for (int k = K - 2; k >= 0; --k)
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          xw[k][j] = U - 1 - k >= 0 ? xc[U - 1 - k >= 0 ? U - 1 - k : 0][j] : xw[k - U >= 0 ? k - U : 0][j];
          dw3[k][j] = U - 1 - k >= 0 ? gf[U - 1 - k >= 0 ? U - 1 - k : 0][j] : dw3[k - U >= 0 ? k - U : 0][j];
        }
    };
    load_step(ax, ag, 0);
    load_step(bx, bg, U);
    for (int ms = 0;; ms += 2 * U) {
      if (ms - (K - 1) >= n_end) break;                // pair-uniform
      step(ax, ag, ms);
      if (ms + U - (K - 1) >= n_end) break;
      step(bx, bg, ms + U);
    }
  }
  // dw: sum over the CTA's pairs, one atomic per (channel, tap)
#pragma unroll
  for (int k = 0; k < K; ++k)
#pragma unroll
    for (int j = 0; j < VEC; ++j) red[pair][k][ch + j] = dwa[k][j];
  __syncthreads();
  for (int idx = threadIdx.x; idx < HD * K; idx += NT) {
    const int c = idx / K, k = idx - c * K;
    float sum = 0.f;
#pragma unroll
    for (int q = 0; q < PAIRS; ++q) sum += red[q][k][c];
    atomicAdd(&dw[(long long)(head * HD + c) * K + k], sum);
  }
}

// Grid of the step kernel: CTA c of sequence (b, head) takes tokens
// [c * PAIRS * run_len, (c + 1) * PAIRS * run_len), one run per warp pair.
// The CTAs per sequence fill one wave of resident CTAs (nb per SM) when the
// sequences allow it, so no CTA starts late and every pair's run has the same
// length.
struct RunGrid {
  dim3 grid;
  int run_len;
};

inline RunGrid run_grid(long long B, long long L, int D, int head_dim, int pairs, int nb, int sms) {
  const long long seqs = B * (D / head_dim);
  const long long resident = static_cast<long long>(std::max(nb, 1)) * sms;
  long long cps = std::max<long long>(1, resident / seqs);            // CTAs per sequence
  long long run_len = (L + cps * pairs - 1) / (cps * pairs);
  run_len = std::max<long long>(32, (run_len + 3) / 4 * 4);           // a whole number of 4-token steps
  cps = std::max<long long>(1, (L + run_len * pairs - 1) / (run_len * pairs));
  RunGrid g;
  g.grid = dim3(static_cast<unsigned>(cps), D / head_dim, static_cast<unsigned>(B));
  g.run_len = static_cast<int>(run_len);
  return g;
}

template <typename Kern>
int resident_ctas(Kern k, int threads) {
  int nb = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k, threads, 0) != cudaSuccess) nb = 1;
  return nb;
}

template <int VEC, int U, int NT, int MINB>
void launch_bwd_step(const void* dy, const void* xp, long long ldx, const float* w, const float* rnorm, void* dx,
                     long long lddx, float* dw, long long B, long long L, int D, int head_dim, int l2, int sms,
                     cudaStream_t st) {
  static const int nb = resident_ctas(conv_bwd_step_k<VEC, U, NT, MINB>, NT);
  const RunGrid g = run_grid(B, L, D, head_dim, NT / 64, nb, sms);
  conv_bwd_step_k<VEC, U, NT, MINB><<<g.grid, NT, 0, st>>>((const __nv_bfloat16*)dy, (const __nv_bfloat16*)xp, ldx, w,
                                                           rnorm, (__nv_bfloat16*)dx, lddx, dw, L, D, l2, g.run_len);
}

template <int VEC, int K>
int launch_fwd(const void* xp, long long ldx, const float* w, void* y, float* rnorm, long long B, long long L, int D,
               int l2, cudaStream_t st) {
  constexpr int HD = VEC * 32;
  const int smem = HD * K * 4 + (TF + K - 1) * HD * 2;
  dim3 grid(static_cast<unsigned>((L + TF - 1) / TF), D / HD, static_cast<unsigned>(B));
  // three CTAs per SM (registers capped at 80: a few spilled, measured 107 -> 101 us at B = 16): one
  // CTA's staging loads overlap the others' arithmetic
  conv_fwd_k<VEC, K, 3><<<grid, THREADS, smem, st>>>((const __nv_bfloat16*)xp, ldx, w, (__nv_bfloat16*)y, rnorm, L, D,
                                                     l2);
  return 0;
}

template <int VEC, int K>
int launch_bwd(const void* dy, const void* xp, long long ldx, const float* w, const float* rnorm, void* dx,
               long long lddx, float* dw, long long B, long long L, int D, int l2, cudaStream_t st) {
  constexpr int HD = VEC * 32;
  constexpr int smem = bwd_smem_bytes<VEC, K>();
  static bool attr_set[64] = {};   // the attribute is held per device context
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 3;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(conv_bwd_k<VEC, K>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return 3;
    attr_set[dev] = true;
  }
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long tiles = (L + TB - 1) / TB;
  const long long pairs = B * (D / HD);
  const long long want = 2LL * sms / pairs;    // one wave of 2 CTAs per SM (no tail)
  const long long bx = std::max<long long>(1, std::min<long long>(tiles, want));
  dim3 grid(static_cast<unsigned>(bx), D / HD, static_cast<unsigned>(B));
  conv_bwd_k<VEC, K><<<grid, THREADS, smem, st>>>((const __nv_bfloat16*)dy, (const __nv_bfloat16*)xp, ldx, w, rnorm,
                                                  (__nv_bfloat16*)dx, lddx, dw, L, D, l2);
  return 0;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int conv_silu_fwd(const void* xp, long long ldx, const float* w, void* y, float* rnorm, long long B, long long L,
                  int D, int K, int head_dim, int l2norm, cudaStream_t st) {
  if (K != MAXK || D % head_dim || !aligned16(xp) || !aligned16(y) || !aligned16(w) || ldx % 8) return 5;
  int rc = 5;
  if (head_dim == 256) rc = launch_fwd<8, 4>(xp, ldx, w, y, rnorm, B, L, D, l2norm, st);
  else if (head_dim == 128) rc = launch_fwd<4, 4>(xp, ldx, w, y, rnorm, B, L, D, l2norm, st);
  else if (head_dim == 64) rc = launch_fwd<2, 4>(xp, ldx, w, y, rnorm, B, L, D, l2norm, st);
  else if (head_dim == 32) rc = launch_fwd<1, 4>(xp, ldx, w, y, rnorm, B, L, D, l2norm, st);
  if (rc) return rc;
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int conv_silu_bwd(const void* dy, const void* xp, long long ldx, const float* w, const float* rnorm, void* dx,
                  long long lddx, float* dw, long long B, long long L, int D, int K, int head_dim, int l2norm,
                  cudaStream_t st) {
  if (K != MAXK || D % head_dim || !aligned16(xp) || !aligned16(dy) || !aligned16(dx) || !aligned16(w) || ldx % 8 ||
      lddx % 8)
    return 5;
  int rc = 5;
  static const bool staged = std::getenv("VAGUS_CONV_STAGED") != nullptr;
  if ((head_dim == 256 || head_dim == 128) && !staged) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // At B = 8 x 4096 tokens, D = 1024: heads of 256 (237 registers, two CTAs of two pairs per
    // SM) 86 us (174 us at B = 16), heads of 128 (128 registers, four CTAs per SM) 94 us; one
    // token per iteration on a persistent grid took 110 / 204 us (231 us at B = 16, heads of
    // 256), and the step kernel with 64-bit index products per access 95 us at heads of 256.
    if (head_dim == 256)
      launch_bwd_step<4, 4, 128, 2>(dy, xp, ldx, w, rnorm, dx, lddx, dw, B, L, D, head_dim, l2norm, sms, st);
    else
      launch_bwd_step<2, 4, 128, 4>(dy, xp, ldx, w, rnorm, dx, lddx, dw, B, L, D, head_dim, l2norm, sms, st);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
  }
  if (head_dim == 256) rc = launch_bwd<8, 4>(dy, xp, ldx, w, rnorm, dx, lddx, dw, B, L, D, l2norm, st);
  else if (head_dim == 128) rc = launch_bwd<4, 4>(dy, xp, ldx, w, rnorm, dx, lddx, dw, B, L, D, l2norm, st);
  else if (head_dim == 64) rc = launch_bwd<2, 4>(dy, xp, ldx, w, rnorm, dx, lddx, dw, B, L, D, l2norm, st);
  else if (head_dim == 32) rc = launch_bwd<1, 4>(dy, xp, ldx, w, rnorm, dx, lddx, dw, B, L, D, l2norm, st);
  if (rc) return rc;
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

}  // namespace vagus
