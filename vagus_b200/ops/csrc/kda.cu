// Gated inner products of the per-channel-gate (KDA) chunk form, forward and
// backward, one CTA per 64-token chunk:
//   Aqk[i][j] = sum_c Q[i][c] K[j][c] exp(g[i][c] - g[j][c])   (j <= i, else 0)
//   Akk[i][j] = sum_c K[i][c] K[j][c] exp(g[i][c] - g[j][c])   (j <  i, else 0)
// with g the in-chunk cumulative log decay (non-increasing in i, so every
// exponent is <= 0).  The decay is applied elementwise -- the pairwise form
// is exact for fast channels, where factorising it through exp(+-g) would
// overflow -- and one exponential serves both products.  The backward forms
// dQ, dK and dg from dAqk and dAkk the same way, one thread per (token,
// channel).  Inputs Q, K, g and the outputs are fp32, (chunks, 64, dk) and
// (chunks, 64, 64) contiguous.  Reference behaviour: fla chunk_kda's
// intra-chunk products (the oracle is models/scans.py _vec_chunk).
#include "common.cuh"
#include "kernels.h"

namespace vagus {
namespace {

constexpr int KC = 64;           // chunk
constexpr int KT = 512;          // threads: one CTA per SM (shared memory), so 16 warps hide the latency

__device__ __forceinline__ void load_rows(float* s, const float* g, int dk, int sp) {
  for (int i = threadIdx.x; i < KC * dk / 4; i += KT) {
    const int r = (4 * i) / dk, c = (4 * i) % dk;
    const float4 v = *reinterpret_cast<const float4*>(g + (long long)r * dk + c);
    float* d = s + r * sp + c;
    d[0] = v.x; d[1] = v.y; d[2] = v.z; d[3] = v.w;
  }
}

__global__ void __launch_bounds__(KT)
kda_gated_fwd_k(const float* __restrict__ Q, const float* __restrict__ K, const float* __restrict__ G,
                float* __restrict__ Aqk, float* __restrict__ Akk, int dk) {
  extern __shared__ float sm[];
  const int sp = dk + 1;                       // odd pitch: rows land on distinct banks
  float *qs = sm, *ks = qs + KC * sp, *gs = ks + KC * sp;
  const long long ch = blockIdx.x;
  load_rows(qs, Q + ch * KC * dk, dk, sp);
  load_rows(ks, K + ch * KC * dk, dk, sp);
  load_rows(gs, G + ch * KC * dk, dk, sp);
  __syncthreads();
  for (int e = threadIdx.x; e < KC * KC; e += KT) {
    const int i = e / KC, j = e % KC;          // a warp: one row i, 32 consecutive j
    float aq = 0.f, ak = 0.f;
    if (j <= i) {
      const float *qi = qs + i * sp, *ki = ks + i * sp, *kj = ks + j * sp, *gi = gs + i * sp, *gj = gs + j * sp;
#pragma unroll 8
      for (int c = 0; c < dk; ++c) {
        const float w = kj[c] * __expf(gi[c] - gj[c]);
        aq = fmaf(qi[c], w, aq);
        ak = fmaf(ki[c], w, ak);
      }
    }
    Aqk[ch * KC * KC + e] = aq;
    Akk[ch * KC * KC + e] = j < i ? ak : 0.f;
  }
}

__global__ void __launch_bounds__(KT)
kda_gated_bwd_k(const float* __restrict__ Q, const float* __restrict__ K, const float* __restrict__ G,
                const float* __restrict__ dAqk, const float* __restrict__ dAkk, float* __restrict__ dQ,
                float* __restrict__ dK, float* __restrict__ dG, int dk) {
  extern __shared__ float sm[];
  const int sp = dk + 1;
  constexpr int ap = KC + 1;
  float *qs = sm, *ks = qs + KC * sp, *gs = ks + KC * sp, *daq = gs + KC * sp, *dak = daq + KC * ap;
  const long long ch = blockIdx.x;
  load_rows(qs, Q + ch * KC * dk, dk, sp);
  load_rows(ks, K + ch * KC * dk, dk, sp);
  load_rows(gs, G + ch * KC * dk, dk, sp);
  for (int e = threadIdx.x; e < KC * KC; e += KT) {
    daq[(e / KC) * ap + e % KC] = dAqk[ch * KC * KC + e];
    dak[(e / KC) * ap + e % KC] = dAkk[ch * KC * KC + e];
  }
  __syncthreads();
  for (int it = threadIdx.x; it < KC * dk; it += KT) {
    const int t = it / dk, c = it % dk;        // a warp: one token t, 32 consecutive channels
    const float qt = qs[t * sp + c], kt = ks[t * sp + c], gt = gs[t * sp + c];
    float dq = 0.f, dkk = 0.f, dg = 0.f;
    // row side: pairs (t, j), j <= t (j < t for K K^T)
    for (int j = 0; j <= t; ++j) {
      const float kj = ks[j * sp + c];
      const float e = __expf(gt - gs[j * sp + c]);
      const float a = daq[t * ap + j] * e * kj;                 // dAqk[t][j] K_j E_tj
      const float b = j < t ? dak[t * ap + j] * e * kj : 0.f;   // dAkk[t][j] K_j E_tj
      dq += a;
      dkk += b;
      dg += a * qt + b * kt;
    }
    // column side: pairs (i, t), i >= t (i > t for K K^T)
    for (int i = t; i < KC; ++i) {
      const float e = __expf(gs[i * sp + c] - gt);
      const float a = daq[i * ap + t] * e * qs[i * sp + c];      // dAqk[i][t] Q_i E_it
      const float b = i > t ? dak[i * ap + t] * e * ks[i * sp + c] : 0.f;
      dkk += a + b;
      dg -= (a + b) * kt;
    }
    dQ[ch * KC * dk + it] = dq;
    dK[ch * KC * dk + it] = dkk;
    dG[ch * KC * dk + it] = dg;
  }
}

}  // namespace

int kda_gated_fwd(const float* Q, const float* K, const float* G, float* Aqk, float* Akk, long long chunks, int dk,
                  cudaStream_t st) {
  if (dk % 4 || dk > 256 || chunks <= 0) return 5;
  const size_t smem = 3 * KC * (dk + 1) * sizeof(float);
  if (cudaFuncSetAttribute(kda_gated_fwd_k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
      cudaSuccess)
    return 3;
  kda_gated_fwd_k<<<static_cast<unsigned>(chunks), KT, smem, st>>>(Q, K, G, Aqk, Akk, dk);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int kda_gated_bwd(const float* Q, const float* K, const float* G, const float* dAqk, const float* dAkk, float* dQ,
                  float* dK, float* dG, long long chunks, int dk, cudaStream_t st) {
  if (dk % 4 || dk > 256 || chunks <= 0) return 5;
  const size_t smem = (3 * KC * (dk + 1) + 2 * KC * (KC + 1)) * sizeof(float);
  if (cudaFuncSetAttribute(kda_gated_bwd_k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
      cudaSuccess)
    return 3;
  kda_gated_bwd_k<<<static_cast<unsigned>(chunks), KT, smem, st>>>(Q, K, G, dAqk, dAkk, dQ, dK, dG, dk);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

}  // namespace vagus

