// Inter-chunk state recurrence of the chunked gated delta rule (scalar gate),
// forward scan and reverse-scan backward, on the tensor cores (bf16 mma.sync
// m16n8k16, fp32 accumulate; the running state stays fp32 in registers).
//
// With the per-chunk operands prepared by the intra-chunk stage
//     W  (C x dk)  = T diag(b G) K          U  (C x dv) = T diag(b) V
//     Qh (C x dk)  = scale * diag(G) Q      Kt (C x dk) = diag(G_C / G) K
//     A  (C x C)   = scale * (Q K^T o D)    causal,  gC = G_C
// the chunk step is
//     V' = U - W S_n;   O = Qh S_n + A V';   S_{n+1} = gC S_n + Kt^T V'
// and the backward, walking the chunks in reverse with dS = dL/dS_{n+1},
//     dV' = A^T dO + Kt dS               (dU = dV')
//     dW  = -dV' S_n^T   dQh = dO S_n^T   dKt = V' dS^T   dA = dO V'^T
//     dgC = <S_n, dS>
//     dS <- gC dS + Qh^T dO - W^T dV'
//
// Only the state chains are sequential, so each direction is split in two:
//   * a scan kernel per (batch*head, 64-wide value tile) that carries S (or
//     dS) through the chunks and writes a bf16 snapshot of it per chunk,
//     with the next chunk's operands prefetched (cp.async, double buffered)
//     while the current one computes;
//   * a chunk-parallel kernel (one CTA per chunk and 64-wide tile) for the
//     products that only need the snapshots: O in the forward; dW, dQh, dKt,
//     dA and dgC in the backward, which reduce over the whole value
//     dimension inside one CTA and so need no atomics.
// The snapshots are bf16, the precision the tensor-core products consume.
//
// Layouts (all chunk-major, contiguous):
//   W, Qh, Kt: (BH, N, C, DK) bf16   A: (BH, N, C, C) bf16   U, V', dU: (BH, N, C, DV) bf16
//   O, dO: token-major (B, N * C, H, DV) bf16 (BH = B * H), the layout of the model's activations
//   gC, dgC: (BH, N) fp32   states, dstates: (BH, N, DK, DV) bf16
//   dW, dQh, dKt: (BH, N, C, DK) bf16   dA: (BH, N, C, C) fp32
#include "common.cuh"
#include "kernels.h"
#include "mma.cuh"

namespace vagus {
namespace {

using namespace mma;

constexpr int C = 64;        // chunk length
constexpr int DVT = 64;      // value tile
constexpr int THREADS = 256;

// O and dO are token-major (B, L, H, DV): the first row of chunk n of
// sequence bh = b * H + h, and the pitch between its rows
__device__ __forceinline__ long long tok_row0(long long bh, int n, int N, int H, int DV) {
  const long long b = bh / H, h = bh - b * H;
  return ((b * N * C + (long long)n * C) * H + h) * DV;
}

__device__ __forceinline__ void cp_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_2() { asm volatile("cp.async.wait_group 2;" ::: "memory"); }

// copy a rows x cols bf16 tile from shared (pitch sp) to global (pitch gp), 16 bytes per access
__device__ __forceinline__ void store_tile(__nv_bfloat16* g, long long gp, const __nv_bfloat16* s, int sp, int rows,
                                           int cols) {
  const int per_row = cols / 8;
  for (int i = threadIdx.x; i < rows * per_row; i += blockDim.x) {
    const int r = i / per_row, c = (i - r * per_row) * 8;
    *reinterpret_cast<uint4*>(g + r * gp + c) = *reinterpret_cast<const uint4*>(s + r * sp + c);
  }
}

// ------------------------------------------------------------- forward scan --

template <int DK>
struct FwdScanSmem {
  __nv_bfloat16 W[2][C][DK + PAD];
  __nv_bfloat16 K[2][C][DK + PAD];
  __nv_bfloat16 U[2][C][DVT + PAD];
  __nv_bfloat16 S[DK][DVT + PAD];
  __nv_bfloat16 V[C][DVT + PAD];
};

template <int DK>
__global__ void __launch_bounds__(THREADS, 1)
gdr_fwd_scan(const __nv_bfloat16* __restrict__ W, const __nv_bfloat16* __restrict__ Kt,
             const __nv_bfloat16* __restrict__ U, const float* __restrict__ gC, const float* __restrict__ S0,
             __nv_bfloat16* __restrict__ Vp, __nv_bfloat16* __restrict__ states, float* __restrict__ S_out, int N,
             int DV) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  FwdScanSmem<DK>& sm = *reinterpret_cast<FwdScanSmem<DK>*>(smem_raw);
  constexpr int SMT = DK / 8 / 16;          // state rows per warp / 16
  const int tiles_v = DV / DVT;
  const long long bh = blockIdx.x / tiles_v;
  const int vt = blockIdx.x % tiles_v;
  const int warp = threadIdx.x / 32;
  const int v0 = vt * DVT;
  const int srow0 = warp * (DK / 8);
  const int wm0 = (warp & 3) * 16, wn0 = (warp >> 2) * 32;

  auto issue = [&](int n) {
    const long long cidx = bh * N + n;
    const int b = n & 1;
    load_tile(&sm.W[b][0][0], DK + PAD, W + cidx * C * DK, DK, C, DK);
    load_tile(&sm.K[b][0][0], DK + PAD, Kt + cidx * C * DK, DK, C, DK);
    load_tile(&sm.U[b][0][0], DVT + PAD, U + cidx * C * DV + v0, DV, C, DVT);
  };

  float S[SMT][8][4];
#pragma unroll
  for (int mt = 0; mt < SMT; ++mt)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = srow0 + frag_row(mt, e), c = frag_col(nt, e);
        S[mt][nt][e] = S0 ? S0[(bh * DK + r) * DV + v0 + c] : 0.f;
      }
  issue(0);
  cp_commit();
  for (int n = 0; n < N; ++n) {
    const long long cidx = bh * N + n;
    const int b = n & 1;
    if (n + 1 < N) issue(n + 1);
    cp_commit();
#pragma unroll
    for (int mt = 0; mt < SMT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int r = srow0 + frag_row(mt, e), c = frag_col(nt, e);
          *reinterpret_cast<uint32_t*>(&sm.S[r][c]) = pack_bf16x2(S[mt][nt][e], S[mt][nt][e + 1]);
        }
    cp_wait_1();
    __syncthreads();
    if (states) store_tile(states + cidx * DK * DV + v0, DV, &sm.S[0][0], DVT + PAD, DK, DVT);

    // V' = U - W S
    {
      float acc[1][4][4];
      zero(acc);
      warp_mma<1, 4, false, true>(acc, &sm.W[b][0][0], DK + PAD, &sm.S[0][0], DVT + PAD, wm0, wn0, DK);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int r = wm0 + frag_row(0, e), c = wn0 + frag_col(nt, e);
          const float2 u = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(&sm.U[b][r][c]));
          *reinterpret_cast<uint32_t*>(&sm.V[r][c]) = pack_bf16x2(u.x - acc[0][nt][e], u.y - acc[0][nt][e + 1]);
        }
    }
    __syncthreads();
    store_tile(Vp + cidx * C * DV + v0, DV, &sm.V[0][0], DVT + PAD, C, DVT);

    // S <- gC S + Kt^T V'
    const float g = gC[cidx];
#pragma unroll
    for (int mt = 0; mt < SMT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) S[mt][nt][e] *= g;
    warp_mma<SMT, 8, true, true>(S, &sm.K[b][0][0], DK + PAD, &sm.V[0][0], DVT + PAD, srow0, 0, C);
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

// ------------------------------------------------------------ forward output --
// O[:, tile] = Qh S_n[:, tile] + A V'[:, tile]; grid (BH * N, DV / 64)

template <int DK>
struct OutSmem {
  __nv_bfloat16 Q[C][DK + PAD];
  __nv_bfloat16 S[DK][DVT + PAD];
  __nv_bfloat16 A[C][C + PAD];
  __nv_bfloat16 V[C][DVT + PAD];
};

template <int DK>
__global__ void __launch_bounds__(THREADS, 2)
gdr_fwd_out(const __nv_bfloat16* __restrict__ Qh, const __nv_bfloat16* __restrict__ A,
            const __nv_bfloat16* __restrict__ Vp, const __nv_bfloat16* __restrict__ states,
            __nv_bfloat16* __restrict__ O, int DV, int N, int H) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  OutSmem<DK>& sm = *reinterpret_cast<OutSmem<DK>*>(smem_raw);
  const long long cidx = blockIdx.x;
  const int v0 = blockIdx.y * DVT;
  const int warp = threadIdx.x / 32;
  const int wm0 = (warp & 3) * 16, wn0 = (warp >> 2) * 32;
  load_tile(&sm.Q[0][0], DK + PAD, Qh + cidx * C * DK, DK, C, DK);
  load_tile(&sm.S[0][0], DVT + PAD, states + cidx * DK * DV + v0, DV, DK, DVT);
  load_tile(&sm.A[0][0], C + PAD, A + cidx * C * C, C, C, C);
  load_tile(&sm.V[0][0], DVT + PAD, Vp + cidx * C * DV + v0, DV, C, DVT);
  cp_commit();
  cp_wait_all();
  __syncthreads();
  float acc[1][4][4];
  zero(acc);
  warp_mma<1, 4, false, true>(acc, &sm.Q[0][0], DK + PAD, &sm.S[0][0], DVT + PAD, wm0, wn0, DK);
  warp_mma<1, 4, false, true>(acc, &sm.A[0][0], C + PAD, &sm.V[0][0], DVT + PAD, wm0, wn0, C);
  __syncthreads();                          // V tile reused for the bf16 output
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      const int r = wm0 + frag_row(0, e), c = wn0 + frag_col(nt, e);
      *reinterpret_cast<uint32_t*>(&sm.V[r][c]) = pack_bf16x2(acc[0][nt][e], acc[0][nt][e + 1]);
    }
  __syncthreads();
  store_tile(O + tok_row0(cidx / N, static_cast<int>(cidx % N), N, H, DV) + v0, (long long)H * DV, &sm.V[0][0],
             DVT + PAD, C, DVT);
}

// ------------------------------------------------------------ backward scan --

template <int DK>
struct BwdScanSmem {
  __nv_bfloat16 K[2][C][DK + PAD];
  __nv_bfloat16 A[2][C][C + PAD];
  __nv_bfloat16 dO[2][C][DVT + PAD];
  __nv_bfloat16 Q[C][DK + PAD];
  __nv_bfloat16 W[C][DK + PAD];
  __nv_bfloat16 dS[DK][DVT + PAD];
  __nv_bfloat16 dVn[C][DVT + PAD];   // -dV'
};

template <int DK>
__global__ void __launch_bounds__(THREADS, 1)
gdr_bwd_scan(const __nv_bfloat16* __restrict__ W, const __nv_bfloat16* __restrict__ Qh,
             const __nv_bfloat16* __restrict__ Kt, const __nv_bfloat16* __restrict__ A,
             const float* __restrict__ gC, const __nv_bfloat16* __restrict__ dO, const float* __restrict__ dS_final,
             __nv_bfloat16* __restrict__ dU, __nv_bfloat16* __restrict__ dstates, float* __restrict__ dS0, int N,
             int DV, int H) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  BwdScanSmem<DK>& sm = *reinterpret_cast<BwdScanSmem<DK>*>(smem_raw);
  constexpr int SMT = DK / 8 / 16;
  const int tiles_v = DV / DVT;
  const long long bh = blockIdx.x / tiles_v;
  const int vt = blockIdx.x % tiles_v;
  const int warp = threadIdx.x / 32;
  const int v0 = vt * DVT;
  const int srow0 = warp * (DK / 8);
  const int wm0 = (warp & 3) * 16, wn0 = (warp >> 2) * 32;

  // group 1 of chunk n: Kt, A, dO (double buffered); group 2: Qh, W (single)
  auto issue1 = [&](int n) {
    const long long cidx = bh * N + n;
    const int b = n & 1;
    load_tile(&sm.K[b][0][0], DK + PAD, Kt + cidx * C * DK, DK, C, DK);
    load_tile(&sm.A[b][0][0], C + PAD, A + cidx * C * C, C, C, C);
    load_tile(&sm.dO[b][0][0], DVT + PAD, dO + tok_row0(bh, n, N, H, DV) + v0, (long long)H * DV, C, DVT);
  };
  auto issue2 = [&](int n) {
    const long long cidx = bh * N + n;
    load_tile(&sm.Q[0][0], DK + PAD, Qh + cidx * C * DK, DK, C, DK);
    load_tile(&sm.W[0][0], DK + PAD, W + cidx * C * DK, DK, C, DK);
  };

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
  // commit order: G1(N-1), G2(N-1), then per chunk n: G1(n-1) ... G2(n-1)
  issue1(N - 1);
  cp_commit();
  issue2(N - 1);
  cp_commit();
  for (int n = N - 1; n >= 0; --n) {
    const long long cidx = bh * N + n;
    const int b = n & 1;
    if (n > 0) issue1(n - 1);
    cp_commit();
#pragma unroll
    for (int mt = 0; mt < SMT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int r = srow0 + frag_row(mt, e), c = frag_col(nt, e);
          *reinterpret_cast<uint32_t*>(&sm.dS[r][c]) = pack_bf16x2(dS[mt][nt][e], dS[mt][nt][e + 1]);
        }
    cp_wait_2();                              // G1(n) done (G2(n), G1(n-1) may be in flight)
    __syncthreads();
    store_tile(dstates + cidx * DK * DV + v0, DV, &sm.dS[0][0], DVT + PAD, DK, DVT);

    // dV' = A^T dO + Kt dS  -> dU (global, via the tile), -dV' (shared)
    {
      float acc[1][4][4];
      zero(acc);
      warp_mma<1, 4, true, true>(acc, &sm.A[b][0][0], C + PAD, &sm.dO[b][0][0], DVT + PAD, wm0, wn0, C);
      warp_mma<1, 4, false, true>(acc, &sm.K[b][0][0], DK + PAD, &sm.dS[0][0], DVT + PAD, wm0, wn0, DK);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int r = wm0 + frag_row(0, e), c = wn0 + frag_col(nt, e);
          *reinterpret_cast<uint32_t*>(&sm.dVn[r][c]) = pack_bf16x2(-acc[0][nt][e], -acc[0][nt][e + 1]);
          *reinterpret_cast<uint32_t*>(dU + (cidx * C + r) * DV + v0 + c) =
              pack_bf16x2(acc[0][nt][e], acc[0][nt][e + 1]);
        }
    }
    cp_wait_1();                              // G2(n) done
    __syncthreads();

    // dS <- gC dS + Qh^T dO - W^T dV'
    const float g = gC[cidx];
#pragma unroll
    for (int mt = 0; mt < SMT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) dS[mt][nt][e] *= g;
    warp_mma<SMT, 8, true, true>(dS, &sm.Q[0][0], DK + PAD, &sm.dO[b][0][0], DVT + PAD, srow0, 0, C);
    warp_mma<SMT, 8, true, true>(dS, &sm.W[0][0], DK + PAD, &sm.dVn[0][0], DVT + PAD, srow0, 0, C);
    __syncthreads();
    if (n > 0) issue2(n - 1);
    cp_commit();
  }
  cp_wait_all();
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

// --------------------------------------------------- backward, per chunk --
// grid (BH * N, DK / 64): dW, dQh, dKt for 64 state rows k0..k0+63, over the
// whole value dimension in 64-wide steps (double buffered); the k0 == 0 CTA
// also forms dA.  dgC accumulates <S_n, dS> over the CTAs of a chunk.

struct ParSmem {
  __nv_bfloat16 dV[2][C][DVT + PAD];     // dU = dV'
  __nv_bfloat16 dO[2][C][DVT + PAD];
  __nv_bfloat16 V[2][C][DVT + PAD];      // V'
  __nv_bfloat16 S[2][64][DVT + PAD];     // S_n rows k0..k0+63
  __nv_bfloat16 dS[2][64][DVT + PAD];
  float red[THREADS / 32];
};

__global__ void __launch_bounds__(THREADS, 2)
gdr_bwd_chunk(const __nv_bfloat16* __restrict__ dU, const __nv_bfloat16* __restrict__ dO,
              const __nv_bfloat16* __restrict__ Vp, const __nv_bfloat16* __restrict__ states,
              const __nv_bfloat16* __restrict__ dstates, __nv_bfloat16* __restrict__ dW,
              __nv_bfloat16* __restrict__ dQh, __nv_bfloat16* __restrict__ dKt, float* __restrict__ dA,
              float* __restrict__ dgC, int DK, int DV, int N, int H) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  ParSmem& sm = *reinterpret_cast<ParSmem*>(smem_raw);
  const long long cidx = blockIdx.x;
  const int k0 = blockIdx.y * 64;
  const bool do_dA = blockIdx.y == 0;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int wm0 = (warp & 3) * 16, wn0 = (warp >> 2) * 32;
  auto issue = [&](int vb) {
    const int b = vb & 1, v0 = vb * DVT;
    load_tile(&sm.dV[b][0][0], DVT + PAD, dU + cidx * C * DV + v0, DV, C, DVT);
    load_tile(&sm.dO[b][0][0], DVT + PAD, dO + tok_row0(cidx / N, static_cast<int>(cidx % N), N, H, DV) + v0,
              (long long)H * DV, C, DVT);
    load_tile(&sm.V[b][0][0], DVT + PAD, Vp + cidx * C * DV + v0, DV, C, DVT);
    load_tile(&sm.S[b][0][0], DVT + PAD, states + (cidx * DK + k0) * DV + v0, DV, 64, DVT);
    load_tile(&sm.dS[b][0][0], DVT + PAD, dstates + (cidx * DK + k0) * DV + v0, DV, 64, DVT);
  };
  float aw[1][4][4], aq[1][4][4], ak[1][4][4], aa[1][4][4];
  zero(aw); zero(aq); zero(ak); zero(aa);
  float dot = 0.f;
  const int nvb = DV / DVT;
  issue(0);
  cp_commit();
  for (int vb = 0; vb < nvb; ++vb) {
    const int b = vb & 1;
    if (vb + 1 < nvb) issue(vb + 1);
    cp_commit();
    cp_wait_1();
    __syncthreads();
    // dW = -dV' S^T, dQh = dO S^T, dKt = V' dS^T   (64 x 64 blocks, K = value)
    warp_mma<1, 4, false, false>(aw, &sm.dV[b][0][0], DVT + PAD, &sm.S[b][0][0], DVT + PAD, wm0, wn0, DVT);
    warp_mma<1, 4, false, false>(aq, &sm.dO[b][0][0], DVT + PAD, &sm.S[b][0][0], DVT + PAD, wm0, wn0, DVT);
    warp_mma<1, 4, false, false>(ak, &sm.V[b][0][0], DVT + PAD, &sm.dS[b][0][0], DVT + PAD, wm0, wn0, DVT);
    if (do_dA) warp_mma<1, 4, false, false>(aa, &sm.dO[b][0][0], DVT + PAD, &sm.V[b][0][0], DVT + PAD, wm0, wn0, DVT);
    for (int i = threadIdx.x; i < 64 * (DVT / 2); i += THREADS) {
      const int r = i / (DVT / 2), c = (i % (DVT / 2)) * 2;
      const float2 sv = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(&sm.S[b][r][c]));
      const float2 dv = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(&sm.dS[b][r][c]));
      dot += sv.x * dv.x + sv.y * dv.y;
    }
    __syncthreads();
  }
  dot = warp_sum(dot);
  if (lane == 0) sm.red[warp] = dot;
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      const int r = wm0 + frag_row(0, e), c = wn0 + frag_col(nt, e);
      const long long off = (cidx * C + r) * DK + k0 + c;
      *reinterpret_cast<uint32_t*>(dW + off) = pack_bf16x2(-aw[0][nt][e], -aw[0][nt][e + 1]);
      *reinterpret_cast<uint32_t*>(dQh + off) = pack_bf16x2(aq[0][nt][e], aq[0][nt][e + 1]);
      *reinterpret_cast<uint32_t*>(dKt + off) = pack_bf16x2(ak[0][nt][e], ak[0][nt][e + 1]);
      if (do_dA)
        *reinterpret_cast<float2*>(dA + (cidx * C + r) * C + c) = make_float2(aa[0][nt][e], aa[0][nt][e + 1]);
    }
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < THREADS / 32; ++i) t += sm.red[i];
    atomicAdd(&dgC[cidx], t);
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

template <typename Kern>
bool set_smem(Kern kern, size_t bytes) {
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)) ==
         cudaSuccess;
}

template <int DK>
int launch_fwd(const GdrRecArgs& a, cudaStream_t st) {
  const size_t s1 = sizeof(FwdScanSmem<DK>), s2 = sizeof(OutSmem<DK>);
  if (!set_smem(gdr_fwd_scan<DK>, s1) || !set_smem(gdr_fwd_out<DK>, s2)) return 3;
  const int grid = static_cast<int>(a.BH * (a.DV / DVT));
  gdr_fwd_scan<DK><<<grid, THREADS, s1, st>>>((const __nv_bfloat16*)a.W, (const __nv_bfloat16*)a.Kt,
                                              (const __nv_bfloat16*)a.U, a.gC, a.S0, (__nv_bfloat16*)a.Vp,
                                              (__nv_bfloat16*)a.states, a.S_out, a.N, a.DV);
  dim3 g2(static_cast<unsigned>(a.BH * a.N), a.DV / DVT);
  gdr_fwd_out<DK><<<g2, THREADS, s2, st>>>((const __nv_bfloat16*)a.Qh, (const __nv_bfloat16*)a.A,
                                           (const __nv_bfloat16*)a.Vp, (const __nv_bfloat16*)a.states,
                                           (__nv_bfloat16*)a.O, a.DV, a.N, a.H);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

template <int DK>
int launch_bwd(const GdrRecBwdArgs& a, cudaStream_t st) {
  const size_t s1 = sizeof(BwdScanSmem<DK>), s2 = sizeof(ParSmem);
  if (!set_smem(gdr_bwd_scan<DK>, s1) || !set_smem(gdr_bwd_chunk, s2)) return 3;
  const int grid = static_cast<int>(a.f.BH * (a.f.DV / DVT));
  gdr_bwd_scan<DK><<<grid, THREADS, s1, st>>>((const __nv_bfloat16*)a.f.W, (const __nv_bfloat16*)a.f.Qh,
                                              (const __nv_bfloat16*)a.f.Kt, (const __nv_bfloat16*)a.f.A, a.f.gC,
                                              (const __nv_bfloat16*)a.dO, a.dS_final, (__nv_bfloat16*)a.dU,
                                              (__nv_bfloat16*)a.dstates, a.dS0, a.f.N, a.f.DV, a.f.H);
  dim3 g2(static_cast<unsigned>(a.f.BH * a.f.N), DK / 64);
  gdr_bwd_chunk<<<g2, THREADS, s2, st>>>((const __nv_bfloat16*)a.dU, (const __nv_bfloat16*)a.dO,
                                         (const __nv_bfloat16*)a.f.Vp, (const __nv_bfloat16*)a.f.states,
                                         (const __nv_bfloat16*)a.dstates, (__nv_bfloat16*)a.dW,
                                         (__nv_bfloat16*)a.dQh, (__nv_bfloat16*)a.dKt, a.dA, a.dgC, DK, a.f.DV,
                                         a.f.N, a.f.H);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

}  // namespace

int gdr_rec_fwd(const GdrRecArgs& a, cudaStream_t st) {
  if (a.DV % DVT || a.H <= 0 || a.BH % a.H) return 5;
  if (a.DK == 256) return launch_fwd<256>(a, st);
  if (a.DK == 128) return launch_fwd<128>(a, st);
  return 5;
}

int gdr_rec_bwd(const GdrRecBwdArgs& a, cudaStream_t st) {
  if (a.f.DV % DVT || a.f.H <= 0 || a.f.BH % a.f.H) return 5;
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
