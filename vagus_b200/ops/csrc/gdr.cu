// Inter-chunk state recurrence of the chunked gated delta rule (scalar gate),
// forward scan and reverse-scan backward, on the tensor cores (bf16 mma.sync
// m16n8k16, fp32 accumulate; the state itself stays fp32 in registers).
//
// Per (batch, head, 64-wide value tile) one CTA walks the chunks in order.
// With the per-chunk operands prepared by the intra-chunk stage
//     W  (C x dk)  = T diag(b G) K          U  (C x dv) = T diag(b) V
//     Qh (C x dk)  = scale * diag(G) Q      Kt (C x dk) = diag(G_C / G) K
//     A  (C x C)   = scale * (Q K^T o D)    causal,  gC = G_C
// the chunk step is
//     V' = U - W S;   O = Qh S + A V';   S <- gC S + Kt^T V'
// and the backward, walking the chunks in reverse with dS = dL/dS_{n+1},
//     dV' = A^T dO + Kt dS               (dU = dV')
//     dW  = -dV' S^T   dQh = dO S^T   dKt = V' dS^T   dA = dO V'^T
//     dgC = <S, dS>
//     dS <- gC dS + Qh^T dO - W^T dV'
// The products that reduce over the value dimension (dW, dQh, dKt, dA, dgC)
// are summed across the value tiles with fp32 atomics.
//
// Layouts (all chunk-major, contiguous):
//   W, Qh, Kt: (BH, N, C, DK) bf16   A: (BH, N, C, C) bf16   U, V', O, dO: (BH, N, C, DV) bf16
//   gC: (BH, N) fp32   states: (BH, N, DK, DV) fp32 (entry state of each chunk)
#include "common.cuh"
#include "kernels.h"
#include "mma.cuh"

namespace vagus {
namespace {

using namespace mma;

constexpr int C = 64;        // chunk length
constexpr int DVT = 64;      // value tile per CTA
constexpr int THREADS = 256;

template <int DK>
struct FwdSmem {
  __nv_bfloat16 W[C][DK + PAD];
  __nv_bfloat16 Q[C][DK + PAD];
  __nv_bfloat16 K[C][DK + PAD];
  __nv_bfloat16 A[C][C + PAD];
  __nv_bfloat16 U[C][DVT + PAD];
  __nv_bfloat16 S[DK][DVT + PAD];
  __nv_bfloat16 V[C][DVT + PAD];
};

template <int DK>
__global__ void __launch_bounds__(THREADS, 1)
gdr_fwd_kernel(const __nv_bfloat16* __restrict__ W, const __nv_bfloat16* __restrict__ Qh,
               const __nv_bfloat16* __restrict__ Kt, const __nv_bfloat16* __restrict__ A,
               const __nv_bfloat16* __restrict__ U, const float* __restrict__ gC, const float* __restrict__ S0,
               __nv_bfloat16* __restrict__ O, __nv_bfloat16* __restrict__ Vp, float* __restrict__ states,
               float* __restrict__ S_out, int N, int DV) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  FwdSmem<DK>& sm = *reinterpret_cast<FwdSmem<DK>*>(smem_raw);
  constexpr int SMT = DK / 8 / 16;          // state rows per warp / 16
  const int tiles_v = DV / DVT;
  const long long bh = blockIdx.x / tiles_v;
  const int vt = blockIdx.x % tiles_v;
  const int warp = threadIdx.x / 32;
  const int v0 = vt * DVT;

  // state fragment: warp owns rows [warp * DK/8, +DK/8), all DVT columns
  float S[SMT][8][4];
  const int srow0 = warp * (DK / 8);
#pragma unroll
  for (int mt = 0; mt < SMT; ++mt)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = srow0 + frag_row(mt, e), c = frag_col(nt, e);
        S[mt][nt][e] = S0 ? S0[(bh * DK + r) * DV + v0 + c] : 0.f;
      }

  const int wm0 = (warp & 3) * 16, wn0 = (warp >> 2) * 32;   // 64 x 64 products
  for (int n = 0; n < N; ++n) {
    const long long cidx = bh * N + n;
    load_tile(&sm.W[0][0], DK + PAD, W + cidx * C * DK, DK, C, DK);
    load_tile(&sm.Q[0][0], DK + PAD, Qh + cidx * C * DK, DK, C, DK);
    load_tile(&sm.K[0][0], DK + PAD, Kt + cidx * C * DK, DK, C, DK);
    load_tile(&sm.A[0][0], C + PAD, A + cidx * C * C, C, C, C);
    load_tile(&sm.U[0][0], DVT + PAD, U + cidx * C * DV + v0, DV, C, DVT);
    cp_commit();
    // entry state: fp32 to the states buffer, bf16 to shared memory
#pragma unroll
    for (int mt = 0; mt < SMT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = srow0 + frag_row(mt, e), c = frag_col(nt, e);
          if (states) states[(cidx * DK + r) * DV + v0 + c] = S[mt][nt][e];
          sm.S[r][c] = f2bf(S[mt][nt][e]);
        }
    cp_wait_all();
    __syncthreads();

    // V' = U - W S
    float acc[1][4][4];
    zero(acc);
    warp_mma<1, 4, false, true>(acc, &sm.W[0][0], DK + PAD, &sm.S[0][0], DVT + PAD, wm0, wn0, DK);
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = wm0 + frag_row(0, e), c = wn0 + frag_col(nt, e);
        const float v = bf2f(sm.U[r][c]) - acc[0][nt][e];
        const __nv_bfloat16 vb = f2bf(v);
        sm.V[r][c] = vb;
        Vp[(cidx * C + r) * DV + v0 + c] = vb;
      }
    __syncthreads();

    // O = Qh S + A V'
    zero(acc);
    warp_mma<1, 4, false, true>(acc, &sm.Q[0][0], DK + PAD, &sm.S[0][0], DVT + PAD, wm0, wn0, DK);
    warp_mma<1, 4, false, true>(acc, &sm.A[0][0], C + PAD, &sm.V[0][0], DVT + PAD, wm0, wn0, C);
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int r = wm0 + frag_row(0, e), c = wn0 + frag_col(nt, e);
        *reinterpret_cast<uint32_t*>(O + (cidx * C + r) * DV + v0 + c) = pack_bf16x2(acc[0][nt][e], acc[0][nt][e + 1]);
      }

    // S <- gC S + Kt^T V'
    const float g = gC[cidx];
#pragma unroll
    for (int mt = 0; mt < SMT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) S[mt][nt][e] *= g;
    warp_mma<SMT, 8, true, true>(S, &sm.K[0][0], DK + PAD, &sm.V[0][0], DVT + PAD, srow0, 0, C);
    __syncthreads();   // every warp is done with this chunk's tiles
  }
  if (S_out) {
#pragma unroll
    for (int mt = 0; mt < SMT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = srow0 + frag_row(mt, e), c = frag_col(nt, e);
          S_out[(bh * DK + r) * DV + v0 + c] = S[mt][nt][e];
        }
  }
}

template <int DK>
struct BwdSmem {
  __nv_bfloat16 W[C][DK + PAD];
  __nv_bfloat16 Q[C][DK + PAD];
  __nv_bfloat16 K[C][DK + PAD];
  __nv_bfloat16 A[C][C + PAD];
  __nv_bfloat16 Vp[C][DVT + PAD];
  __nv_bfloat16 dO[C][DVT + PAD];
  __nv_bfloat16 S[DK][DVT + PAD];
  __nv_bfloat16 dS[DK][DVT + PAD];
  __nv_bfloat16 dVn[C][DVT + PAD];   // -dV'
  float red[THREADS / 32];
};

__device__ __forceinline__ void red_add2(float* p, float a, float b) {
  atomicAdd(reinterpret_cast<float2*>(p), make_float2(a, b));
}

template <int DK>
__global__ void __launch_bounds__(THREADS, 1)
gdr_bwd_kernel(const __nv_bfloat16* __restrict__ W, const __nv_bfloat16* __restrict__ Qh,
               const __nv_bfloat16* __restrict__ Kt, const __nv_bfloat16* __restrict__ A,
               const __nv_bfloat16* __restrict__ Vp, const float* __restrict__ gC, const float* __restrict__ states,
               const __nv_bfloat16* __restrict__ dO, const float* __restrict__ dS_final,
               float* __restrict__ dW, float* __restrict__ dQh, float* __restrict__ dKt, float* __restrict__ dA,
               __nv_bfloat16* __restrict__ dU, float* __restrict__ dgC, float* __restrict__ dS0, int N, int DV) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  BwdSmem<DK>& sm = *reinterpret_cast<BwdSmem<DK>*>(smem_raw);
  constexpr int SMT = DK / 8 / 16;
  const int tiles_v = DV / DVT;
  const long long bh = blockIdx.x / tiles_v;
  const int vt = blockIdx.x % tiles_v;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int v0 = vt * DVT;
  const int srow0 = warp * (DK / 8);
  const int wm0 = (warp & 3) * 16, wn0 = (warp >> 2) * 32;

  float dS[SMT][8][4];
#pragma unroll
  for (int mt = 0; mt < SMT; ++mt)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = srow0 + frag_row(mt, e), c = frag_col(nt, e);
        dS[mt][nt][e] = dS_final ? dS_final[(bh * DK + r) * DV + v0 + c] : 0.f;
      }

  for (int n = N - 1; n >= 0; --n) {
    const long long cidx = bh * N + n;
    load_tile(&sm.W[0][0], DK + PAD, W + cidx * C * DK, DK, C, DK);
    load_tile(&sm.Q[0][0], DK + PAD, Qh + cidx * C * DK, DK, C, DK);
    load_tile(&sm.K[0][0], DK + PAD, Kt + cidx * C * DK, DK, C, DK);
    load_tile(&sm.A[0][0], C + PAD, A + cidx * C * C, C, C, C);
    load_tile(&sm.Vp[0][0], DVT + PAD, Vp + cidx * C * DV + v0, DV, C, DVT);
    load_tile(&sm.dO[0][0], DVT + PAD, dO + cidx * C * DV + v0, DV, C, DVT);
    cp_commit();
    // S_n to shared (bf16); dS to shared (bf16); dgC partial = <S_n, dS>
    float part = 0.f;
#pragma unroll
    for (int mt = 0; mt < SMT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = srow0 + frag_row(mt, e), c = frag_col(nt, e);
          const float s = states[(cidx * DK + r) * DV + v0 + c];
          sm.S[r][c] = f2bf(s);
          sm.dS[r][c] = f2bf(dS[mt][nt][e]);
          part += s * dS[mt][nt][e];
        }
    part = warp_sum(part);
    if (lane == 0) sm.red[warp] = part;
    cp_wait_all();
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
      for (int i = 0; i < THREADS / 32; ++i) t += sm.red[i];
      atomicAdd(&dgC[cidx], t);
    }

    // dV' = A^T dO + Kt dS  -> dU (global), -dV' (shared)
    {
      float acc[1][4][4];
      zero(acc);
      warp_mma<1, 4, true, true>(acc, &sm.A[0][0], C + PAD, &sm.dO[0][0], DVT + PAD, wm0, wn0, C);
      warp_mma<1, 4, false, true>(acc, &sm.K[0][0], DK + PAD, &sm.dS[0][0], DVT + PAD, wm0, wn0, DK);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int r = wm0 + frag_row(0, e), c = wn0 + frag_col(nt, e);
          *reinterpret_cast<uint32_t*>(dU + (cidx * C + r) * DV + v0 + c) = pack_bf16x2(acc[0][nt][e], acc[0][nt][e + 1]);
          *reinterpret_cast<uint32_t*>(&sm.dVn[r][c]) = pack_bf16x2(-acc[0][nt][e], -acc[0][nt][e + 1]);
        }
    }
    __syncthreads();

    // value-reduced products, 64 x DK each, in 64-column blocks
    for (int nb = 0; nb < DK; nb += 64) {
      const int on0 = nb + (warp >> 2) * 32;
      float a1[1][4][4], a2[1][4][4], a3[1][4][4];
      zero(a1); zero(a2); zero(a3);
      warp_mma<1, 4, false, false>(a1, &sm.dVn[0][0], DVT + PAD, &sm.S[0][0], DVT + PAD, wm0, on0, DVT);
      warp_mma<1, 4, false, false>(a2, &sm.dO[0][0], DVT + PAD, &sm.S[0][0], DVT + PAD, wm0, on0, DVT);
      warp_mma<1, 4, false, false>(a3, &sm.Vp[0][0], DVT + PAD, &sm.dS[0][0], DVT + PAD, wm0, on0, DVT);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int r = wm0 + frag_row(0, e), c = on0 + frag_col(nt, e);
          const long long off = (cidx * C + r) * DK + c;
          red_add2(dW + off, a1[0][nt][e], a1[0][nt][e + 1]);
          red_add2(dQh + off, a2[0][nt][e], a2[0][nt][e + 1]);
          red_add2(dKt + off, a3[0][nt][e], a3[0][nt][e + 1]);
        }
    }
    {
      float acc[1][4][4];
      zero(acc);
      warp_mma<1, 4, false, false>(acc, &sm.dO[0][0], DVT + PAD, &sm.Vp[0][0], DVT + PAD, wm0, wn0, DVT);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int r = wm0 + frag_row(0, e), c = wn0 + frag_col(nt, e);
          red_add2(dA + (cidx * C + r) * C + c, acc[0][nt][e], acc[0][nt][e + 1]);
        }
    }

    // dS <- gC dS + Qh^T dO - W^T dV'
    const float g = gC[cidx];
#pragma unroll
    for (int mt = 0; mt < SMT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) dS[mt][nt][e] *= g;
    warp_mma<SMT, 8, true, true>(dS, &sm.Q[0][0], DK + PAD, &sm.dO[0][0], DVT + PAD, srow0, 0, C);
    warp_mma<SMT, 8, true, true>(dS, &sm.W[0][0], DK + PAD, &sm.dVn[0][0], DVT + PAD, srow0, 0, C);
    __syncthreads();
  }
  if (dS0) {
#pragma unroll
    for (int mt = 0; mt < SMT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = srow0 + frag_row(mt, e), c = frag_col(nt, e);
          dS0[(bh * DK + r) * DV + v0 + c] = dS[mt][nt][e];
        }
  }
}

// ----------------------------------------------------- single-token decode --
// S (B, H, dk, dv) fp32 in place; q, k (B, H, dk), v (B, H, dv) bf16; g, beta (B, H)
// S <- a S;  r = v - S^T k;  S <- S + b k r^T;  o = scale * S^T q
__global__ void gdr_decode_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                                  const __nv_bfloat16* __restrict__ v, const float* __restrict__ g,
                                  const float* __restrict__ beta, float* __restrict__ S, __nv_bfloat16* __restrict__ o,
                                  int dk, int dv, float scale) {
  // one CTA per (b, h); thread j owns value column j
  extern __shared__ float sk[];   // k (dk) then q (dk)
  const long long bh = blockIdx.x;
  float* sq = sk + dk;
  for (int i = threadIdx.x; i < dk; i += blockDim.x) {
    sk[i] = bf2f(k[bh * dk + i]);
    sq[i] = bf2f(q[bh * dk + i]) * scale;
  }
  __syncthreads();
  const float a = __expf(g[bh]);
  const float b = beta[bh];
  for (int j = threadIdx.x; j < dv; j += blockDim.x) {
    float* col = S + bh * (long long)dk * dv + j;
    float kS = 0.f;
    for (int i = 0; i < dk; ++i) kS += sk[i] * col[(long long)i * dv] * a;
    const float r = bf2f(v[bh * dv + j]) - kS;
    float out = 0.f;
    for (int i = 0; i < dk; ++i) {
      const float s = col[(long long)i * dv] * a + b * sk[i] * r;
      col[(long long)i * dv] = s;
      out += sq[i] * s;
    }
    o[bh * dv + j] = f2bf(out);
  }
}

template <int DK>
int launch_fwd(const GdrRecArgs& a, cudaStream_t st) {
  const size_t sm = sizeof(FwdSmem<DK>);
  auto kern = gdr_fwd_kernel<DK>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm));
  const int grid = static_cast<int>(a.BH * (a.DV / DVT));
  kern<<<grid, THREADS, sm, st>>>((const __nv_bfloat16*)a.W, (const __nv_bfloat16*)a.Qh, (const __nv_bfloat16*)a.Kt,
                                  (const __nv_bfloat16*)a.A, (const __nv_bfloat16*)a.U, a.gC, a.S0,
                                  (__nv_bfloat16*)a.O, (__nv_bfloat16*)a.Vp, a.states, a.S_out, a.N, a.DV);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

template <int DK>
int launch_bwd(const GdrRecBwdArgs& a, cudaStream_t st) {
  const size_t sm = sizeof(BwdSmem<DK>);
  auto kern = gdr_bwd_kernel<DK>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm));
  const int grid = static_cast<int>(a.f.BH * (a.f.DV / DVT));
  kern<<<grid, THREADS, sm, st>>>((const __nv_bfloat16*)a.f.W, (const __nv_bfloat16*)a.f.Qh,
                                  (const __nv_bfloat16*)a.f.Kt, (const __nv_bfloat16*)a.f.A,
                                  (const __nv_bfloat16*)a.f.Vp, a.f.gC, a.f.states, (const __nv_bfloat16*)a.dO,
                                  a.dS_final, a.dW, a.dQh, a.dKt, a.dA, (__nv_bfloat16*)a.dU, a.dgC, a.dS0, a.f.N,
                                  a.f.DV);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

}  // namespace

int gdr_rec_fwd(const GdrRecArgs& a, cudaStream_t st) {
  if (a.DV % DVT) return 5;
  if (a.DK == 256) return launch_fwd<256>(a, st);
  if (a.DK == 128) return launch_fwd<128>(a, st);
  return 5;
}

int gdr_rec_bwd(const GdrRecBwdArgs& a, cudaStream_t st) {
  if (a.f.DV % DVT) return 5;
  if (a.f.DK == 256) return launch_bwd<256>(a, st);
  if (a.f.DK == 128) return launch_bwd<128>(a, st);
  return 5;
}

int gdr_decode(const void* q, const void* k, const void* v, const float* g, const float* beta, float* S, void* o,
               long long BH, int dk, int dv, float scale, cudaStream_t st) {
  gdr_decode_kernel<<<static_cast<unsigned>(BH), 256, 2 * dk * sizeof(float), st>>>(
      (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, g, beta, S, (__nv_bfloat16*)o, dk,
      dv, scale);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

}  // namespace vagus
