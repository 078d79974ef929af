// Intra-chunk stage of the chunked delta rule with a per-channel (Kimi-delta,
// KDA) gate, forward and backward, one CTA per (batch, head, 64-token chunk).
//
// With gamma the in-chunk cumulative log decay of every key channel
// (gamma_ic = sum_{t <= i} g_tc, non-increasing in i) and G = exp(gamma), the
// gated inner products
//     <X_i, Y_j>_g = sum_c X_ic Y_jc exp(gamma_ic - gamma_jc)        (j <= i)
// give  Akk = strict_lower(<K, K>_g),  Aqk = lower(<Q, K>_g),  and
//     M  = diag(b) Akk,   T = (I + M)^{-1}
//     W  = T diag(b) (K o G)          U  = T diag(b) V
//     Qh = s Q o G    Kt = K o exp(gamma_C - gamma)    A = s Aqk    gC = exp(gamma_C)
// which the recurrence kernels (gdr.cu, per-channel decay) consume.
//
// The gated products are formed without the overflow of exp(+gamma) that
// factorising exp(gamma_i - gamma_j) through the chunk start would hit for
// fast channels: the chunk is cut into four 16-token blocks;
//   * for a block pair I > J the decay factorises through r_J = gamma at the
//     last token of block J:  exp(gamma_i - gamma_j) = exp(gamma_i - r_J)
//     exp(r_J - gamma_j), both factors <= 1, so
//     <X, K>_g over (I, J) = (X_I o exp(gamma_I - r_J)) (K_J o exp(r_J - gamma_J))^T,
//     a 16 x 16 x dk product on the tensor cores (mma.sync, bf16 operands);
//   * inside a block the decay is taken elementwise (fp32).
// The backward uses the same split: for I > J with P = X_I o exp(gamma_I - r_J)
// and R = K_J o exp(r_J - gamma_J), dP = dA R and dR = dA^T P are tensor-core
// products, and the r_J terms of the chain rule cancel exactly (the product
// does not depend on r_J), so gamma receives dP o P on block I and -dR o R on
// block J; inside a block the elementwise terms.  The WY part is the scalar
// gate's (gdr_intra.cu) with G per channel.
//
// Token-major inputs: q, k (B, L, H, DK), v (B, L, H, DV) bf16; g (B, L, H, DK)
// and beta (B, L, H) fp32.  Chunk-major outputs (BH, N, C, .) as the
// recurrence kernels expect.  Reference behaviour: fla chunk_kda's intra-chunk
// stage (the oracle is models/scans.py chunk_scan_vec).
#include "common.cuh"
#include "kernels.h"
#include "mma.cuh"
#include "tri_inverse.cuh"

namespace vagus {
namespace {

using namespace mma;
using wy::tri_inverse_inplace;

constexpr int C = 64;
constexpr int BLK = 16;
constexpr int THREADS = 256;
constexpr int GP = 4;                    // fp32 padding of the gamma rows: rows 8 apart share a bank, not all

// Phase clock of CTA (0, 0, 0): clock64() at phase boundaries into
// trace[event] (forward events 0..15, backward 16..31); null: off.
#define KDA_TR(ev)                                                                                     \
  do {                                                                                                 \
    if (trace != nullptr && threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) \
      trace[ev] = clock64();                                                                           \
  } while (0)

template <int DK, int DV>
struct KdaFwdSmem {
  __nv_bfloat16 Q[C][DK + PAD];
  __nv_bfloat16 K[C][DK + PAD];          // K, then diag(b) (K o G)
  float gam[C][DK + GP];                 // cumulative log decay per channel
  __nv_bfloat16 R[BLK][DK + PAD];        // K_J o exp(r_J - gamma_J)
  __nv_bfloat16 P[6][BLK][DK + PAD];     // Q_I / K_I o exp(gamma_I - r_J), I = J+1..3
  float Aqk[C][C + 1];
  float M[C][C + 1];                     // Akk, then M = diag(b) Akk, then T (in place)
  __nv_bfloat16 Tb[C][C + PAD];
  __nv_bfloat16 V[C][DV + PAD];          // V, then diag(b) V
  float beta[C];
};

// g (token-major, this chunk's rows) -> gam = per-channel inclusive prefix sum
template <int DK>
__device__ __forceinline__ void load_cumsum(float (*gam)[DK + GP], const float* g, long long gld) {
  for (int idx = threadIdx.x; idx < C * DK / 4; idx += THREADS) {
    const int i = idx / (DK / 4), c = (idx % (DK / 4)) * 4;
    *reinterpret_cast<float4*>(&gam[i][c]) = *reinterpret_cast<const float4*>(g + i * gld + c);
  }
  __syncthreads();
  for (int c = threadIdx.x; c < DK; c += THREADS) {
    float s = 0.f;
    for (int i = 0; i < C; ++i) {
      s += gam[i][c];
      gam[i][c] = s;
    }
  }
  __syncthreads();
}

// Shared-memory operands of the gated products.
template <int DK>
struct GatedView {
  __nv_bfloat16 (*Q)[DK + PAD];
  __nv_bfloat16 (*K)[DK + PAD];
  float (*gam)[DK + GP];
  __nv_bfloat16 (*R)[DK + PAD];          // [BLK] rows
  __nv_bfloat16 (*P)[BLK][DK + PAD];     // [6] tiles
  float (*Aqk)[C + 1];
  float (*M)[C + 1];
};

// The gated products of the chunk into Aqk (lower, diagonal included) and
// Akk (strictly lower, into M), both zero above.
template <int DK>
__device__ __forceinline__ void gated_products(const GatedView<DK>& sm, unsigned long long* trace, int ev) {
  const int warp = threadIdx.x >> 5;
  for (int idx = threadIdx.x; idx < C * C; idx += THREADS) {
    sm.Aqk[idx / C][idx % C] = 0.f;
    sm.M[idx / C][idx % C] = 0.f;
  }
  __syncthreads();
  // inside the 16-token blocks: elementwise decay.  Work items are the
  // blocks' 4 x 136 pairs (j <= i) x two halves of the channels; the halves of
  // a pair sit on neighbouring lanes and meet through one shuffle
  constexpr int PAIRS = BLK * (BLK + 1) / 2;
  constexpr int ITEMS = 4 * PAIRS * 2;
  for (int base = 0; base < ITEMS; base += THREADS) {
    const int it = base + threadIdx.x;
    const bool active = it < ITEMS;
    const int pr = active ? it >> 1 : 0, hf = it & 1;
    const int blk = pr / PAIRS, p = pr % PAIRS;
    int i = static_cast<int>((sqrtf(8.f * p + 1.f) - 1.f) * 0.5f);   // triangular index -> (i, j)
    while ((i + 1) * (i + 2) / 2 <= p) ++i;
    while (i * (i + 1) / 2 > p) --i;
    const int j = p - i * (i + 1) / 2;
    const int ri = blk * BLK + i, rj = blk * BLK + j;
    float aq = 0.f, ak = 0.f;
    if (active) {
#pragma unroll 4
      for (int c = hf * (DK / 2); c < (hf + 1) * (DK / 2); c += 2) {
        const float2 qi = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(&sm.Q[ri][c]));
        const float2 ki = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(&sm.K[ri][c]));
        const float2 kj = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(&sm.K[rj][c]));
        const float2 gi = *reinterpret_cast<const float2*>(&sm.gam[ri][c]);
        const float2 gj = *reinterpret_cast<const float2*>(&sm.gam[rj][c]);
        const float e0 = __expf(gi.x - gj.x) * kj.x, e1 = __expf(gi.y - gj.y) * kj.y;
        aq = fmaf(qi.x, e0, fmaf(qi.y, e1, aq));
        ak = fmaf(ki.x, e0, fmaf(ki.y, e1, ak));
      }
    }
    aq += __shfl_xor_sync(0xffffffffu, aq, 1);
    ak += __shfl_xor_sync(0xffffffffu, ak, 1);
    if (active && hf == 0) {
      sm.Aqk[ri][rj] = aq;
      if (j < i) sm.M[ri][rj] = ak;
    }
  }
  // across blocks: factorised through r_J, on the tensor cores
  KDA_TR(ev);
  for (int J = 0; J < 3; ++J) {
    __syncthreads();                                   // P / R free
    const int rJ = J * BLK + BLK - 1;
    for (int idx = threadIdx.x; idx < BLK * DK; idx += THREADS) {
      const int j = idx / DK, c = idx % DK;
      sm.R[j][c] = f2bf(bf2f(sm.K[J * BLK + j][c]) * __expf(sm.gam[rJ][c] - sm.gam[J * BLK + j][c]));
    }
    const int nI = 3 - J;
    for (int idx = threadIdx.x; idx < nI * BLK * DK; idx += THREADS) {
      const int t = idx / (BLK * DK), i = (idx / DK) % BLK, c = idx % DK;
      const int row = (J + 1 + t) * BLK + i;
      const float a = __expf(sm.gam[row][c] - sm.gam[rJ][c]);
      sm.P[2 * t][i][c] = f2bf(bf2f(sm.Q[row][c]) * a);
      sm.P[2 * t + 1][i][c] = f2bf(bf2f(sm.K[row][c]) * a);
    }
    __syncthreads();
    if (warp < 2 * nI) {
      const int t = warp >> 1, isk = warp & 1;
      float acc[1][2][4];
      zero(acc);
      warp_mma<1, 2, false, false>(acc, &sm.P[warp][0][0], DK + PAD, &sm.R[0][0], DK + PAD, 0, 0, DK);
      float (*dst)[C + 1] = isk ? sm.M : sm.Aqk;
      const int I = J + 1 + t;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) dst[I * BLK + frag_row(0, e)][J * BLK + frag_col(nt, e)] = acc[0][nt][e];
    }
  }
  __syncthreads();
}

template <int DK, int DV>
__global__ void __launch_bounds__(THREADS, 1)
kda_intra_fwd_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                     const __nv_bfloat16* __restrict__ v, const float* __restrict__ g,
                     const float* __restrict__ beta, __nv_bfloat16* __restrict__ Wo, __nv_bfloat16* __restrict__ Qho,
                     __nv_bfloat16* __restrict__ Kto, __nv_bfloat16* __restrict__ Ao, __nv_bfloat16* __restrict__ Uo,
                     float* __restrict__ gCo, int L, int H, float scale, unsigned long long* trace) {
  using S = KdaFwdSmem<DK, DV>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  S& sm = *reinterpret_cast<S*>(smem_raw);
  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int N = gridDim.x;
  const long long cidx = ((long long)b * H + h) * N + n;
  const long long tok0 = (long long)b * L + (long long)n * C;
  KDA_TR(0);
  const int warp = threadIdx.x >> 5;
  load_tile(&sm.Q[0][0], DK + PAD, q + (tok0 * H + h) * DK, (long long)H * DK, C, DK);
  load_tile(&sm.K[0][0], DK + PAD, k + (tok0 * H + h) * DK, (long long)H * DK, C, DK);
  load_tile(&sm.V[0][0], DV + PAD, v + (tok0 * H + h) * DV, (long long)H * DV, C, DV);
  cp_commit();
  if (threadIdx.x < C) sm.beta[threadIdx.x] = beta[(tok0 + threadIdx.x) * H + h];
  load_cumsum<DK>(sm.gam, g + (tok0 * H + h) * DK, (long long)H * DK);
  cp_wait_all();
  __syncthreads();
  KDA_TR(1);
  gated_products<DK>(GatedView<DK>{sm.Q, sm.K, sm.gam, sm.R, sm.P, sm.Aqk, sm.M}, trace, 2);
  KDA_TR(3);

  // A = s Aqk; M = diag(b) Akk -> T
  for (int idx = threadIdx.x; idx < C * C / 2; idx += THREADS) {
    const int i = idx / (C / 2), j = (idx % (C / 2)) * 2;
    *reinterpret_cast<uint32_t*>(Ao + (cidx * C + i) * C + j) = pack_bf16x2(scale * sm.Aqk[i][j], scale * sm.Aqk[i][j + 1]);
    sm.M[i][j] *= sm.beta[i];
    sm.M[i][j + 1] *= sm.beta[i];
  }
  __syncthreads();
  tri_inverse_inplace(sm.M);
  KDA_TR(4);
  for (int idx = threadIdx.x; idx < C * C; idx += THREADS) sm.Tb[idx / C][idx % C] = f2bf(sm.M[idx / C][idx % C]);

  // Qh, Kt, gC out; K -> diag(b) (K o G); V -> diag(b) V
  for (int idx = threadIdx.x; idx < C * DK / 2; idx += THREADS) {
    const int i = idx / (DK / 2), c = (idx % (DK / 2)) * 2;
    const float2 gi = *reinterpret_cast<const float2*>(&sm.gam[i][c]);
    const float2 gl = *reinterpret_cast<const float2*>(&sm.gam[C - 1][c]);
    const float2 qv = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(&sm.Q[i][c]));
    const float2 kv = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(&sm.K[i][c]));
    const float G0 = __expf(gi.x), G1 = __expf(gi.y);
    *reinterpret_cast<uint32_t*>(Qho + (cidx * C + i) * DK + c) = pack_bf16x2(scale * qv.x * G0, scale * qv.y * G1);
    *reinterpret_cast<uint32_t*>(Kto + (cidx * C + i) * DK + c) =
        pack_bf16x2(kv.x * __expf(gl.x - gi.x), kv.y * __expf(gl.y - gi.y));
    const float bi = sm.beta[i];
    *reinterpret_cast<uint32_t*>(&sm.K[i][c]) = pack_bf16x2(bi * kv.x * G0, bi * kv.y * G1);
    if (i == C - 1) { gCo[cidx * DK + c] = G0; gCo[cidx * DK + c + 1] = G1; }
  }
  for (int idx = threadIdx.x; idx < C * DV / 2; idx += THREADS) {
    const int i = idx / (DV / 2), c = (idx % (DV / 2)) * 2;
    const float2 vv = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(&sm.V[i][c]));
    *reinterpret_cast<uint32_t*>(&sm.V[i][c]) = pack_bf16x2(sm.beta[i] * vv.x, sm.beta[i] * vv.y);
  }
  __syncthreads();

  KDA_TR(5);
  // W = T Xw, U = T Xu: warp tile 16 rows x half of the columns
  const int m0 = (warp & 3) * 16;
  {
    constexpr int NT = DK / 16;
    float acc[1][NT][4];
    zero(acc);
    const int c0 = (warp >> 2) * (DK / 2);
    warp_mma<1, NT, false, true>(acc, &sm.Tb[0][0], C + PAD, &sm.K[0][0], DK + PAD, m0, c0, C);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int i = m0 + frag_row(0, e), c = c0 + frag_col(nt, e);
        *reinterpret_cast<uint32_t*>(Wo + (cidx * C + i) * DK + c) = pack_bf16x2(acc[0][nt][e], acc[0][nt][e + 1]);
      }
  }
  {
    constexpr int NT = DV / 16;
    float acc[1][NT][4];
    zero(acc);
    const int c0 = (warp >> 2) * (DV / 2);
    warp_mma<1, NT, false, true>(acc, &sm.Tb[0][0], C + PAD, &sm.V[0][0], DV + PAD, m0, c0, C);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int i = m0 + frag_row(0, e), c = c0 + frag_col(nt, e);
        *reinterpret_cast<uint32_t*>(Uo + (cidx * C + i) * DV + c) = pack_bf16x2(acc[0][nt][e], acc[0][nt][e + 1]);
      }
  }
  __syncthreads();
  KDA_TR(6);
}

// ---------------------------------------------------------------- backward --
// One kernel per chunk (one CTA, eight warps):
//   1. recompute gamma, the gated products and T;
//   2. WY backward --
//        dXw = T^T dW, dXu = T^T dU, dT = dW Xw^T + dU Xu^T,
//        dM = -strict_lower(T^T dT T^T), dAkk = diag(b) dM, dAqk = s dA
//      -- giving dv and dbeta, and the elementwise parts of dq / dk / dgamma
//        dq_e = s dQh o G,  dk_e = dKt o E + b dXw o G,
//        dgamma_e = s dQh o Q o G - dKt o K o E + b dXw o K o G
//      (E = exp(gamma_C - gamma); the last row also takes the column sums of
//      dKt o K o E and dgC o G_C), held in registers in the mma fragment
//      layout (warp w: rows 16 (w & 3).., key channels 64 (w >> 2)..);
//   3. the gated products' backward, in the same fragment layout:
//        dQ[i]  = sum_j dAqk[i,j] K_j e^(gamma_i - gamma_j)        (row role)
//        dKr[i] = sum_j dAkk[i,j] K_j e^(gamma_i - gamma_j)        (row role)
//        dKc[j] = sum_i (dAqk[i,j] Q_i + dAkk[i,j] K_i) e^(gamma_i - gamma_j)
//      and dgamma_g = Q o dQ + K o (dKr - dKc).  Across 16-token blocks the
//      decay factorises through one reference row per block, both factors
//      <= 1: block I's row role through r = 16 I - 1 (the row just before
//      it) over all earlier keys at once,
//        dQ[I] += e^(gamma_I - gamma_r) o (dAqk[I, :16 I] (K[:16 I] o e^(gamma_r - gamma)))
//      and block J's column role through r = 16 J + 15 (its last row) over
//      all later rows; these are mma.sync products over bf16 operands built
//      once per chunk.  Inside a block the decay is taken elementwise (fp32);
//   4. dq, dk (bf16) and dg = reverse cumsum over the chunk of dgamma (fp32)
//      written token-major.
template <int DK, int DV>
struct KdaBwdSmem {
  static constexpr int RK = 96;          // rows of the factorised operands: 16 + 32 + 48
  __nv_bfloat16 Q[C][DK + PAD];
  __nv_bfloat16 K[C][DK + PAD];
  float gam[C][DK + GP];                 // cumulative log decay; dgamma at the end
  // scratch A: the products' R / P tiles; then XW = diag(b) (K o G) and the dW
  // tile (later T^T dT); then Kr = the row-role key operands
  static constexpr int PR_BYTES = (1 + 6) * BLK * (DK + PAD) * 2;
  static constexpr int XD_BYTES = 2 * C * (DK + PAD) * 2;
  static constexpr int KR_BYTES = RK * (DK + PAD) * 2;
  static constexpr int A_BYTES = PR_BYTES > XD_BYTES ? (PR_BYTES > KR_BYTES ? PR_BYTES : KR_BYTES)
                                                     : (XD_BYTES > KR_BYTES ? XD_BYTES : KR_BYTES);
  __align__(16) unsigned char scratch[A_BYTES];
  float Aqk[C][C + 1];                   // products, then Akk (for dbeta), then dAqk
  float M[C][C + 1];                     // Akk -> M -> T, then dAkk
  __nv_bfloat16 Tb[C][C + PAD];          // T, then dAqk (bf16)
  __nv_bfloat16 DT[C][C + PAD];          // dT, then dAkk (bf16)
  // scratch B: V and dU; then Qc, Kc = the column-role operands
  static constexpr int VU_BYTES = 2 * C * (DV + PAD) * 2;
  static constexpr int QK_BYTES = 2 * RK * (DK + PAD) * 2;
  __align__(16) unsigned char scratch2[VU_BYTES > QK_BYTES ? VU_BYTES : QK_BYTES];
  float beta[C];
  float rw[C], ru[C], rm[C];
  float colk[DK];                        // sum_i dKt o K o E per channel (+ dgC G_C)

  __device__ __nv_bfloat16 (*R())[DK + PAD] { return reinterpret_cast<__nv_bfloat16 (*)[DK + PAD]>(scratch); }
  __device__ __nv_bfloat16 (*P())[BLK][DK + PAD] {
    return reinterpret_cast<__nv_bfloat16 (*)[BLK][DK + PAD]>(scratch + BLK * (DK + PAD) * 2);
  }
  __device__ __nv_bfloat16 (*XW())[DK + PAD] { return reinterpret_cast<__nv_bfloat16 (*)[DK + PAD]>(scratch); }
  __device__ __nv_bfloat16 (*DW())[DK + PAD] {
    return reinterpret_cast<__nv_bfloat16 (*)[DK + PAD]>(scratch + C * (DK + PAD) * 2);
  }
  __device__ __nv_bfloat16 (*Kr())[DK + PAD] { return reinterpret_cast<__nv_bfloat16 (*)[DK + PAD]>(scratch); }
  __device__ __nv_bfloat16 (*V())[DV + PAD] { return reinterpret_cast<__nv_bfloat16 (*)[DV + PAD]>(scratch2); }
  __device__ __nv_bfloat16 (*DU())[DV + PAD] {
    return reinterpret_cast<__nv_bfloat16 (*)[DV + PAD]>(scratch2 + C * (DV + PAD) * 2);
  }
  __device__ __nv_bfloat16 (*Qc())[DK + PAD] { return reinterpret_cast<__nv_bfloat16 (*)[DK + PAD]>(scratch2); }
  __device__ __nv_bfloat16 (*Kc())[DK + PAD] {
    return reinterpret_cast<__nv_bfloat16 (*)[DK + PAD]>(scratch2 + RK * (DK + PAD) * 2);
  }
};

// row offset of block I's (I = 1..3) row-role operand in Kr, and of block J's
// (J = 0..2) column-role operands in Qc / Kc
__device__ __forceinline__ int kr_off(int I) { return (I - 1) * I * 8; }                   // 0, 16, 48
__device__ __forceinline__ int qc_off(int J) { return J == 0 ? 0 : (J == 1 ? 48 : 80); }

// out[i] += sum over this warp's fragment columns of acc[i][c] * X[i][c] (bf16 X)
template <int NT>
__device__ __forceinline__ void frag_row_dot(const float (&acc)[1][NT][4], const __nv_bfloat16* X, int ldx, int m0,
                                             int c0, float* out) {
  float part[2] = {0.f, 0.f};
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = m0 + frag_row(0, e), c = c0 + frag_col(nt, e);
      part[e >> 1] += acc[0][nt][e] * bf2f(X[i * ldx + c]);
    }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float sum = part[r];
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if ((threadIdx.x & 3) == 0) atomicAdd(&out[m0 + ((threadIdx.x & 31) >> 2) + 8 * r], sum);
  }
}

template <int DK, int DV>
__global__ void __launch_bounds__(THREADS, 1)
kda_intra_bwd_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                     const __nv_bfloat16* __restrict__ v, const float* __restrict__ g,
                     const float* __restrict__ beta, const __nv_bfloat16* __restrict__ dW,
                     const __nv_bfloat16* __restrict__ dQh, const __nv_bfloat16* __restrict__ dKt,
                     const float* __restrict__ dA, const __nv_bfloat16* __restrict__ dU,
                     const float* __restrict__ dgC, __nv_bfloat16* __restrict__ dq, __nv_bfloat16* __restrict__ dk,
                     __nv_bfloat16* __restrict__ dv, float* __restrict__ dg, float* __restrict__ dbeta, int L, int H,
                     float scale, unsigned long long* trace) {
  using S = KdaBwdSmem<DK, DV>;
  constexpr int NTK = DK / 16;           // fragment column tiles of a warp's DK / 2 channels
  extern __shared__ __align__(128) uint8_t smem_raw[];
  S& sm = *reinterpret_cast<S*>(smem_raw);
  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int N = gridDim.x;
  const long long cidx = ((long long)b * H + h) * N + n;
  const long long tok0 = (long long)b * L + (long long)n * C;
  KDA_TR(16);
  const int warp = threadIdx.x >> 5;
  const int tid = threadIdx.x;
  __nv_bfloat16 (*Vs)[DV + PAD] = sm.V();
  __nv_bfloat16 (*DUs)[DV + PAD] = sm.DU();
  load_tile(&sm.Q[0][0], DK + PAD, q + (tok0 * H + h) * DK, (long long)H * DK, C, DK);
  load_tile(&sm.K[0][0], DK + PAD, k + (tok0 * H + h) * DK, (long long)H * DK, C, DK);
  load_tile(&Vs[0][0], DV + PAD, v + (tok0 * H + h) * DV, (long long)H * DV, C, DV);
  load_tile(&DUs[0][0], DV + PAD, dU + cidx * C * DV, DV, C, DV);
  cp_commit();
  if (tid < C) {
    sm.beta[tid] = beta[(tok0 + tid) * H + h];
    sm.rw[tid] = sm.ru[tid] = sm.rm[tid] = 0.f;
  }
  for (int c = tid; c < DK; c += THREADS) sm.colk[c] = 0.f;
  load_cumsum<DK>(sm.gam, g + (tok0 * H + h) * DK, (long long)H * DK);
  cp_wait_all();
  __syncthreads();
  KDA_TR(17);
  gated_products<DK>(GatedView<DK>{sm.Q, sm.K, sm.gam, sm.R(), sm.P(), sm.Aqk, sm.M}, trace, 18);
  KDA_TR(19);
  __nv_bfloat16 (*XW)[DK + PAD] = sm.XW();
  __nv_bfloat16 (*DWt)[DK + PAD] = sm.DW();

  // keep Akk (for dbeta); M = diag(b) Akk -> T
  for (int idx = tid; idx < C * C; idx += THREADS) {
    const int i = idx / C, j = idx % C;
    const float akk = sm.M[i][j];
    sm.Aqk[i][j] = akk;
    sm.M[i][j] = sm.beta[i] * akk;
  }
  __syncthreads();
  tri_inverse_inplace(sm.M);
  KDA_TR(20);
  for (int idx = tid; idx < C * C; idx += THREADS) sm.Tb[idx / C][idx % C] = f2bf(sm.M[idx / C][idx % C]);
  // XW = diag(b) (K o G); dW tile
  const long long cbase = cidx * C * DK;
  for (int idx = tid; idx < C * DK / 2; idx += THREADS) {
    const int i = idx / (DK / 2), c = (idx % (DK / 2)) * 2;
    const float2 kv = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(&sm.K[i][c]));
    const float2 gi = *reinterpret_cast<const float2*>(&sm.gam[i][c]);
    const float bi = sm.beta[i];
    *reinterpret_cast<uint32_t*>(&XW[i][c]) = pack_bf16x2(bi * kv.x * __expf(gi.x), bi * kv.y * __expf(gi.y));
  }
  load_tile(&DWt[0][0], DK + PAD, dW + cbase, DK, C, DK);
  cp_commit();
  cp_wait_all();
  __syncthreads();

  const int m0 = (warp & 3) * 16;
  const int c0 = (warp >> 2) * (DK / 2);
  {
    // dXu = T^T dU  ->  dv = diag(b) dXu ; ru += dXu . V
    constexpr int NT = DV / 16;
    const int v0 = (warp >> 2) * (DV / 2);
    float acc[1][NT][4];
    zero(acc);
    warp_mma<1, NT, true, true>(acc, &sm.Tb[0][0], C + PAD, &DUs[0][0], DV + PAD, m0, v0, C);
    frag_row_dot<NT>(acc, &Vs[0][0], DV + PAD, m0, v0, sm.ru);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int i = m0 + frag_row(0, e), c = v0 + frag_col(nt, e);
        *reinterpret_cast<uint32_t*>(dv + ((tok0 + i) * H + h) * DV + c) =
            pack_bf16x2(sm.beta[i] * acc[0][nt][e], sm.beta[i] * acc[0][nt][e + 1]);
      }
  }
  // the running gradients of this warp's fragment: dq, dk, dgamma
  float Rq[NTK][4], Rk[NTK][4], Rg[NTK][4];
  {
    // dXw = T^T dW, and every elementwise term of (i, c) in the same pass;
    // dQh / dKt come in as bf16 pairs, all issued before the product
    uint32_t dqh2[NTK][2], dkt2[NTK][2];
#pragma unroll
    for (int nt = 0; nt < NTK; ++nt)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const long long o = cbase + (long long)(m0 + frag_row(0, 2 * r)) * DK + c0 + frag_col(nt, 0);
        dqh2[nt][r] = __ldg(reinterpret_cast<const unsigned int*>(dQh + o));
        dkt2[nt][r] = __ldg(reinterpret_cast<const unsigned int*>(dKt + o));
      }
    float acc[1][NTK][4];
    zero(acc);
    warp_mma<1, NTK, true, true>(acc, &sm.Tb[0][0], C + PAD, &DWt[0][0], DK + PAD, m0, c0, C);
    float part[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < NTK; ++nt) {
      float ck[2] = {0.f, 0.f};                        // this column pair's share of colk
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = m0 + frag_row(0, e), c = c0 + frag_col(nt, e);
        const float gi = sm.gam[i][c], G = __expf(gi), E = __expf(sm.gam[C - 1][c] - gi);
        const float qv = bf2f(sm.Q[i][c]), kv = bf2f(sm.K[i][c]);
        const float2 dq2 = unpack_bf16x2(dqh2[nt][e >> 1]), dk2 = unpack_bf16x2(dkt2[nt][e >> 1]);
        const float dqh = (e & 1) ? dq2.y : dq2.x, dkt = (e & 1) ? dk2.y : dk2.x;
        const float dxw = acc[0][nt][e], bi = sm.beta[i];
        part[e >> 1] += dxw * kv * G;
        const float kte = dkt * kv * E;
        ck[e & 1] += kte;
        Rq[nt][e] = scale * dqh * G;
        Rk[nt][e] = dkt * E + bi * dxw * G;
        Rg[nt][e] = scale * dqh * qv * G - kte + bi * dxw * kv * G;
      }
      // the warp's 16 rows of the two columns: lanes with equal (lane & 3) hold them
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        float v = ck[u];
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        if ((threadIdx.x & 31) < 4) atomicAdd(&sm.colk[c0 + frag_col(nt, u)], v);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float sum = part[r];
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      if ((threadIdx.x & 3) == 0) atomicAdd(&sm.rw[m0 + ((threadIdx.x & 31) >> 2) + 8 * r], sum);
    }
  }
  __syncthreads();
  KDA_TR(21);
  // dT = dW XW^T + (dU V^T) diag(b)  (bf16 into DT)
  {
    float a1[1][4][4], a2[1][4][4];
    zero(a1);
    zero(a2);
    const int n0 = (warp >> 2) * 32;
    warp_mma<1, 4, false, false>(a1, &DWt[0][0], DK + PAD, &XW[0][0], DK + PAD, m0, n0, DK);
    warp_mma<1, 4, false, false>(a2, &DUs[0][0], DV + PAD, &Vs[0][0], DV + PAD, m0, n0, DV);
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int i = m0 + frag_row(0, e), j = n0 + frag_col(nt, e);
        *reinterpret_cast<uint32_t*>(&sm.DT[i][j]) =
            pack_bf16x2(a1[0][nt][e] + sm.beta[j] * a2[0][nt][e], a1[0][nt][e + 1] + sm.beta[j + 1] * a2[0][nt][e + 1]);
      }
  }
  __syncthreads();
  KDA_TR(22);
  // P = T^T dT (bf16, over the dW tile), dM = -strict_lower(P T^T)
  __nv_bfloat16 (*Pb)[DK + PAD] = DWt;
  {
    float p[1][4][4];
    zero(p);
    const int n0 = (warp >> 2) * 32;
    warp_mma<1, 4, true, true>(p, &sm.Tb[0][0], C + PAD, &sm.DT[0][0], C + PAD, m0, n0, C);
    __syncthreads();                                       // dW tile consumed everywhere
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int i = m0 + frag_row(0, e), j = n0 + frag_col(nt, e);
        *reinterpret_cast<uint32_t*>(&Pb[i][j]) = pack_bf16x2(p[0][nt][e], p[0][nt][e + 1]);
      }
  }
  __syncthreads();
  {
    // dAkk = diag(b) dM into M (T is in Tb from here on); dAqk = s lower(dA)
    // into Aqk once this element's Akk has been used for dbeta
    float dm[1][4][4];
    zero(dm);
    const int n0 = (warp >> 2) * 32;
    warp_mma<1, 4, false, false>(dm, &Pb[0][0], DK + PAD, &sm.Tb[0][0], C + PAD, m0, n0, C);
    float part[2] = {0.f, 0.f};
    const float* dAc = dA + cidx * C * C;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = m0 + frag_row(0, e), j = n0 + frag_col(nt, e);
        const float dmv = j < i ? -dm[0][nt][e] : 0.f;
        part[e >> 1] += dmv * sm.Aqk[i][j];
        sm.M[i][j] = sm.beta[i] * dmv;
        sm.Aqk[i][j] = j <= i ? scale * dAc[i * C + j] : 0.f;
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float sum = part[r];
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      if ((threadIdx.x & 3) == 0) atomicAdd(&sm.rm[m0 + ((threadIdx.x & 31) >> 2) + 8 * r], sum);
    }
  }
  __syncthreads();
  KDA_TR(23);
  if (tid < C) dbeta[(tok0 + tid) * H + h] = sm.rw[tid] + sm.ru[tid] + sm.rm[tid];

  // ---- the gated products' backward
  // bf16 dAqk / dAkk over T / dT; factorised operands; the last row's extra
  // dgamma terms (column sums, dgC G_C) folded into colk
  for (int idx = tid; idx < C * C / 2; idx += THREADS) {
    const int i = idx / (C / 2), j = (idx % (C / 2)) * 2;
    *reinterpret_cast<uint32_t*>(&sm.Tb[i][j]) = pack_bf16x2(sm.Aqk[i][j], sm.Aqk[i][j + 1]);
    *reinterpret_cast<uint32_t*>(&sm.DT[i][j]) = pack_bf16x2(sm.M[i][j], sm.M[i][j + 1]);
  }
  for (int c = tid; c < DK; c += THREADS) sm.colk[c] += dgC[cidx * DK + c] * __expf(sm.gam[C - 1][c]);
  __nv_bfloat16 (*Kr)[DK + PAD] = sm.Kr();
  __nv_bfloat16 (*Qc)[DK + PAD] = sm.Qc();
  __nv_bfloat16 (*Kc)[DK + PAD] = sm.Kc();
  for (int idx = tid; idx < S::RK * DK / 2; idx += THREADS) {
    const int row = idx / (DK / 2), c = (idx % (DK / 2)) * 2;
    // Kr: block I (rows kr_off(I).. of 16 I) = K[t] o e^(gamma_r - gamma_t), r = 16 I - 1
    const int I = row < 16 ? 1 : (row < 48 ? 2 : 3);
    const int t = row - kr_off(I), r = 16 * I - 1;
    const float2 gr = *reinterpret_cast<const float2*>(&sm.gam[r][c]);
    const float2 gt = *reinterpret_cast<const float2*>(&sm.gam[t][c]);
    const float2 kt = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(&sm.K[t][c]));
    *reinterpret_cast<uint32_t*>(&Kr[row][c]) =
        pack_bf16x2(kt.x * __expf(gr.x - gt.x), kt.y * __expf(gr.y - gt.y));
    // Qc / Kc: block J (rows qc_off(J).. of 48 - 16 J) = X[u] o e^(gamma_u - gamma_r), u > r = 16 J + 15
    const int J = row < 48 ? 0 : (row < 80 ? 1 : 2);
    const int u = 16 * (J + 1) + row - qc_off(J), rj = 16 * J + 15;
    const float2 gj = *reinterpret_cast<const float2*>(&sm.gam[rj][c]);
    const float2 gu = *reinterpret_cast<const float2*>(&sm.gam[u][c]);
    const float2 qu = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(&sm.Q[u][c]));
    const float2 ku = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(&sm.K[u][c]));
    const float e0 = __expf(gu.x - gj.x), e1 = __expf(gu.y - gj.y);
    *reinterpret_cast<uint32_t*>(&Qc[row][c]) = pack_bf16x2(qu.x * e0, qu.y * e1);
    *reinterpret_cast<uint32_t*>(&Kc[row][c]) = pack_bf16x2(ku.x * e0, ku.y * e1);
  }
  __syncthreads();
  KDA_TR(24);
  const int blk = warp & 3;
  if (blk >= 1) {
    // row role of block blk over keys [0, 16 blk), through r = 16 blk - 1
    float x1[1][NTK][4], x2[1][NTK][4];
    zero(x1);
    zero(x2);
    warp_mma<1, NTK, false, true>(x1, &sm.Tb[0][0], C + PAD, &Kr[kr_off(blk)][0], DK + PAD, m0, c0, 16 * blk);
    warp_mma<1, NTK, false, true>(x2, &sm.DT[0][0], C + PAD, &Kr[kr_off(blk)][0], DK + PAD, m0, c0, 16 * blk);
    const int r = 16 * blk - 1;
#pragma unroll
    for (int nt = 0; nt < NTK; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = m0 + frag_row(0, e), c = c0 + frag_col(nt, e);
        const float f = __expf(sm.gam[i][c] - sm.gam[r][c]);
        const float a = x1[0][nt][e] * f, bk = x2[0][nt][e] * f;
        Rq[nt][e] += a;
        Rk[nt][e] += bk;
        Rg[nt][e] += bf2f(sm.Q[i][c]) * a + bf2f(sm.K[i][c]) * bk;
      }
  }
  if (blk <= 2) {
    // column role of block blk over rows [16 (blk + 1), 64), through r = 16 blk + 15
    float x3[1][NTK][4];
    zero(x3);
    const int kk = C - 16 * (blk + 1);
    warp_mma<1, NTK, true, true>(x3, &sm.Tb[16 * (blk + 1)][16 * blk], C + PAD, &Qc[qc_off(blk)][0], DK + PAD, 0, c0,
                                 kk);
    warp_mma<1, NTK, true, true>(x3, &sm.DT[16 * (blk + 1)][16 * blk], C + PAD, &Kc[qc_off(blk)][0], DK + PAD, 0, c0,
                                 kk);
    const int r = 16 * blk + 15;
#pragma unroll
    for (int nt = 0; nt < NTK; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = m0 + frag_row(0, e), c = c0 + frag_col(nt, e);
        const float x = x3[0][nt][e] * __expf(sm.gam[r][c] - sm.gam[j][c]);
        Rk[nt][e] += x;
        Rg[nt][e] -= bf2f(sm.K[j][c]) * x;
      }
  }
  // inside the 16-token blocks, one thread per (block, channel): the block's
  // Q, K, gamma of that channel in registers, each pair's decay computed once
  // for all three sums; the fragment-layout parts meet them in shared memory
  // (dq, dk parts over the now free operand scratch, dgamma over gamma)
  constexpr int SP = DK + GP;
  constexpr int NI = 4 * DK / THREADS;                 // (block, channel) items per thread
  float (*Sq)[SP] = reinterpret_cast<float (*)[SP]>(sm.scratch);
  float (*Sk)[SP] = reinterpret_cast<float (*)[SP]>(sm.scratch2);
  static_assert(sizeof(sm.scratch) >= sizeof(float) * C * SP && sizeof(sm.scratch2) >= sizeof(float) * C * SP,
                "dq / dk staging");
  const int ic = tid % DK;
  float gl[NI][BLK];                                   // gamma of the items' rows, log2 units
  KDA_TR(25);
  __syncthreads();                                     // off-diagonal products done: operand scratch free
#pragma unroll
  for (int it = 0; it < NI; ++it) {
    const int b0 = BLK * (tid / DK + it * (THREADS / DK));
#pragma unroll
    for (int i = 0; i < BLK; ++i) gl[it][i] = sm.gam[b0 + i][ic] * 1.4426950408889634f;
  }
#pragma unroll
  for (int nt = 0; nt < NTK; ++nt)
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      const int i = m0 + frag_row(0, e), c = c0 + frag_col(nt, e);
      *reinterpret_cast<float2*>(&Sq[i][c]) = make_float2(Rq[nt][e], Rq[nt][e + 1]);
      *reinterpret_cast<float2*>(&Sk[i][c]) = make_float2(Rk[nt][e], Rk[nt][e + 1]);
    }
  __syncthreads();                                     // gamma read by every item: it becomes dgamma
#pragma unroll
  for (int nt = 0; nt < NTK; ++nt)
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      const int i = m0 + frag_row(0, e), c = c0 + frag_col(nt, e);
      *reinterpret_cast<float2*>(&sm.gam[i][c]) = make_float2(Rg[nt][e], Rg[nt][e + 1]);
    }
  __syncthreads();
#pragma unroll
  for (int it = 0; it < NI; ++it) {
    const int b0 = BLK * (tid / DK + it * (THREADS / DK));
    float qv[BLK], kv[BLK], rq[BLK], rk[BLK], cl[BLK];
#pragma unroll
    for (int i = 0; i < BLK; ++i) {
      qv[i] = bf2f(sm.Q[b0 + i][ic]);
      kv[i] = bf2f(sm.K[b0 + i][ic]);
      rq[i] = rk[i] = cl[i] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < BLK; ++i) {
#pragma unroll
      for (int j = 0; j <= i; ++j) {
        const float aq = sm.Aqk[b0 + i][b0 + j], ak = sm.M[b0 + i][b0 + j];   // one address per warp
        const float e = j == i ? 1.f : ex2_approx(gl[it][i] - gl[it][j]);
        const float t = kv[j] * e;
        rq[i] = fmaf(aq, t, rq[i]);
        rk[i] = fmaf(ak, t, rk[i]);                    // dAkk is zero on the diagonal
        cl[j] = fmaf(fmaf(aq, qv[i], ak * kv[i]), e, cl[j]);
      }
    }
#pragma unroll
    for (int i = 0; i < BLK; ++i) {
      Sq[b0 + i][ic] += rq[i];
      Sk[b0 + i][ic] += rk[i] + cl[i];
      sm.gam[b0 + i][ic] += qv[i] * rq[i] + kv[i] * (rk[i] - cl[i]);
    }
  }
  __syncthreads();
  KDA_TR(26);
  for (int idx = tid; idx < C * DK / 2; idx += THREADS) {
    const int i = idx / (DK / 2), c = (idx % (DK / 2)) * 2;
    const long long t = ((tok0 + i) * H + h) * DK + c;
    *reinterpret_cast<uint32_t*>(dq + t) = pack_bf16x2(Sq[i][c], Sq[i][c + 1]);
    *reinterpret_cast<uint32_t*>(dk + t) = pack_bf16x2(Sk[i][c], Sk[i][c + 1]);
  }
  // dg = reverse cumsum of dgamma over the chunk (the last row with its extra terms)
  for (int c = tid; c < DK; c += THREADS) {
    float run = sm.colk[c];
    for (int i = C - 1; i >= 0; --i) {
      run += sm.gam[i][c];
      dg[((tok0 + i) * H + h) * DK + c] = run;
    }
  }
  KDA_TR(27);
}

}  // namespace

unsigned long long* g_kda_trace = nullptr;   // host side of the phase trace (kda_set_trace)

template <int DK, int DV>
static int launch_kda_bwd(const KdaIntraBwdArgs& a, cudaStream_t st) {
  const int smem = sizeof(KdaBwdSmem<DK, DV>);
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    if (cudaFuncSetAttribute(kda_intra_bwd_kernel<DK, DV>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return 3;
    attr[dev] = true;
  }
  dim3 grid(static_cast<unsigned>(a.L / C), static_cast<unsigned>(a.H), static_cast<unsigned>(a.B));
  kda_intra_bwd_kernel<DK, DV><<<grid, THREADS, smem, st>>>(
      (const __nv_bfloat16*)a.q, (const __nv_bfloat16*)a.k, (const __nv_bfloat16*)a.v, a.g, a.beta,
      (const __nv_bfloat16*)a.dW, (const __nv_bfloat16*)a.dQh, (const __nv_bfloat16*)a.dKt, a.dA,
      (const __nv_bfloat16*)a.dU, a.dgC, (__nv_bfloat16*)a.dq, (__nv_bfloat16*)a.dk, (__nv_bfloat16*)a.dv, a.dg,
      a.dbeta, a.L, a.H, a.scale, g_kda_trace);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

template <int DK, int DV>
static int launch_kda_fwd(const void* q, const void* k, const void* v, const float* g, const float* beta, void* W,
                          void* Qh, void* Kt, void* A, void* U, float* gC, int B, int L, int H, float scale,
                          cudaStream_t st) {
  const int smem = sizeof(KdaFwdSmem<DK, DV>);
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    if (cudaFuncSetAttribute(kda_intra_fwd_kernel<DK, DV>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return 3;
    attr[dev] = true;
  }
  dim3 grid(static_cast<unsigned>(L / C), static_cast<unsigned>(H), static_cast<unsigned>(B));
  kda_intra_fwd_kernel<DK, DV><<<grid, THREADS, smem, st>>>(
      (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, g, beta, (__nv_bfloat16*)W,
      (__nv_bfloat16*)Qh, (__nv_bfloat16*)Kt, (__nv_bfloat16*)A, (__nv_bfloat16*)U, gC, L, H, scale, g_kda_trace);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int kda_intra_fwd(const void* q, const void* k, const void* v, const float* g, const float* beta, void* W, void* Qh,
                  void* Kt, void* A, void* U, float* gC, int B, int L, int H, int DK, int DV, float scale,
                  cudaStream_t st) {
  if (L % C) return 5;
  if (DK == 128 && DV == 128) return launch_kda_fwd<128, 128>(q, k, v, g, beta, W, Qh, Kt, A, U, gC, B, L, H, scale, st);
  if (DK == 128 && DV == 256) return launch_kda_fwd<128, 256>(q, k, v, g, beta, W, Qh, Kt, A, U, gC, B, L, H, scale, st);
  return 5;
}

void kda_set_trace(unsigned long long* buf) { g_kda_trace = buf; }

int kda_intra_bwd(const KdaIntraBwdArgs& a, cudaStream_t st) {
  if (a.L % C) return 5;
  int rc = 5;
  if (a.DK == 128 && a.DV == 128) rc = launch_kda_bwd<128, 128>(a, st);
  else if (a.DK == 128 && a.DV == 256) rc = launch_kda_bwd<128, 256>(a, st);
  if (rc) return rc;
  return 0;
}

}  // namespace vagus
