// Intra-chunk stage of the chunked gated delta rule (scalar gate), forward
// and backward, one CTA per (batch, head, 64-token chunk), two CTAs per SM.
//
// With gamma = cumsum(g) inside the chunk, G = exp(gamma), D_ij =
// exp(gamma_i - gamma_j) (i >= j, masked before the exp), the forward builds
//     M  = strict_lower(diag(b) (K K^T o D)),   T = (I + M)^{-1}
//     W  = T diag(b G) K          U  = T diag(b) V
//     Qh = s diag(G) Q            Kt = diag(G_C / G) K
//     A  = s (Q K^T o D) (causal, diagonal included),   gC = G_C
// The unit-lower-triangular inverse is a row-by-row forward substitution in
// shared memory (fp32; each row combines up to 63 finished rows, the 64
// columns x 4 partial sums spread over the 256 threads).  The 64 x 64 x dk
// products run on the tensor cores (mma.sync, bf16 in, fp32 accumulate).
//
// The backward takes dW, dQh, dKt (bf16), dA (fp32), dU and dgC from the
// recurrence backward and returns dq, dk, dv, dg, dbeta:
//     dXw = T^T dW,  dXu = T^T dU          (Xw = diag(bG) K, Xu = diag(b) V)
//     dT  = dW Xw^T + dU Xu^T,  dM = -strict_lower(T^T dT T^T)
//     dKK = dM o b D,  dQK = s dA o D,  dD = dM o b KK + s dA o QK
//     dK  = diag(bG) dXw + (dKK + dKK^T) K + dQK^T Q + diag(G_C/G) dKt
//     dQ  = dQK K + s diag(G) dQh,   dV = diag(b) dXu
// plus the per-row scalars (dbeta, and dgamma from G, D, G_C and G_C/G),
// then dg = reverse cumsum(dgamma) within the chunk.
//
// Token-major inputs: q, k (B, L, H, DK), v (B, L, H, DV) bf16; g, beta
// (B, L, H) fp32.  Chunk-major outputs as the recurrence kernels expect.
#include "common.cuh"
#include "kernels.h"
#include "mma.cuh"
#include "tri_inverse.cuh"

namespace vagus {
namespace {

using namespace mma;

constexpr int C = 64;
constexpr int THREADS = 256;

constexpr int cmax(int a, int b) { return a > b ? a : b; }

// Q and V share one buffer: V is fetched (asynchronously, overlapping the
// inverse) once Q has been consumed.  About 94 KB for dk = dv = 256, so two
// CTAs fit on an SM.
template <int DK, int DV>
struct FwdSmem {
  __nv_bfloat16 QV[C][cmax(DK, DV) + PAD];
  __nv_bfloat16 K[C][DK + PAD];
  float M[C][C + 1];             // M, then T (in place)
  __nv_bfloat16 Tb[C][C + PAD];
  float gam[C], beta[C], graw[C];
};

// inclusive prefix sum of g over the chunk (64 values) into gam; warp 0
__device__ __forceinline__ void chunk_cumsum(const float* g_in, float* gam) {
  const int lane = threadIdx.x & 31;
  float a = g_in[2 * lane], b = g_in[2 * lane + 1];
  float s = a + b;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float t = __shfl_up_sync(0xffffffffu, s, o);
    if (lane >= o) s += t;
  }
  gam[2 * lane + 1] = s;
  gam[2 * lane] = s - b;
}

using wy::tri_inverse_inplace;

template <int DK, int DV>
__global__ void __launch_bounds__(THREADS)
intra_fwd_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                 const __nv_bfloat16* __restrict__ v, const float* __restrict__ g, const float* __restrict__ beta,
                 __nv_bfloat16* __restrict__ Wo, __nv_bfloat16* __restrict__ Qho, __nv_bfloat16* __restrict__ Kto,
                 __nv_bfloat16* __restrict__ Ao, __nv_bfloat16* __restrict__ Uo, float* __restrict__ gCo, int L, int H,
                 float scale) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  FwdSmem<DK, DV>& sm = *reinterpret_cast<FwdSmem<DK, DV>*>(smem_raw);
  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int N = gridDim.x;
  const long long bh = (long long)b * H + h;
  const long long cidx = bh * N + n;
  const long long tok0 = (long long)b * L + (long long)n * C;
  const int warp = threadIdx.x / 32;

  constexpr int QP = cmax(DK, DV) + PAD;
  load_tile(&sm.QV[0][0], QP, q + (tok0 * H + h) * DK, (long long)H * DK, C, DK);
  load_tile(&sm.K[0][0], DK + PAD, k + (tok0 * H + h) * DK, (long long)H * DK, C, DK);
  cp_commit();
  if (threadIdx.x < C) {
    sm.graw[threadIdx.x] = g[(tok0 + threadIdx.x) * H + h];
    sm.beta[threadIdx.x] = beta[(tok0 + threadIdx.x) * H + h];
  }
  __syncthreads();
  if (warp == 0) chunk_cumsum(sm.graw, sm.gam);
  cp_wait_all();
  __syncthreads();

  const int m0 = (warp & 3) * 16, n0 = (warp >> 2) * 32;
  {
    float kk[1][4][4], qk[1][4][4];
    zero(kk);
    zero(qk);
    warp_mma<1, 4, false, false>(kk, &sm.K[0][0], DK + PAD, &sm.K[0][0], DK + PAD, m0, n0, DK);
    warp_mma<1, 4, false, false>(qk, &sm.QV[0][0], QP, &sm.K[0][0], DK + PAD, m0, n0, DK);
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int i = m0 + frag_row(0, e), j = n0 + frag_col(nt, e);   // j even; (i, j), (i, j + 1)
        const float d0 = (j <= i) ? __expf(sm.gam[i] - sm.gam[j]) : 0.f;
        const float d1 = (j + 1 <= i) ? __expf(sm.gam[i] - sm.gam[j + 1]) : 0.f;
        sm.M[i][j] = (j < i) ? sm.beta[i] * kk[0][nt][e] * d0 : 0.f;
        sm.M[i][j + 1] = (j + 1 < i) ? sm.beta[i] * kk[0][nt][e + 1] * d1 : 0.f;
        *reinterpret_cast<uint32_t*>(Ao + (cidx * C + i) * C + j) =
            pack_bf16x2(scale * qk[0][nt][e] * d0, scale * qk[0][nt][e + 1] * d1);
      }
  }
  // Qh, Kt out (Q and unscaled K are then free to be overwritten / rescaled)
  const float glast = sm.gam[C - 1];
  for (int idx = threadIdx.x; idx < C * (DK / 8); idx += THREADS) {
    const int i = idx / (DK / 8), c = (idx % (DK / 8)) * 8;
    const float gi = scale * __expf(sm.gam[i]);
    const float ei = __expf(glast - sm.gam[i]);
    const uint4 qv = *reinterpret_cast<const uint4*>(&sm.QV[i][c]);
    const uint4 kv = *reinterpret_cast<const uint4*>(&sm.K[i][c]);
    const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w}, kw[4] = {kv.x, kv.y, kv.z, kv.w};
    uint32_t qo[4], ko[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float2 a2 = unpack_bf16x2(qw[u]), b2 = unpack_bf16x2(kw[u]);
      qo[u] = pack_bf16x2(gi * a2.x, gi * a2.y);
      ko[u] = pack_bf16x2(ei * b2.x, ei * b2.y);
    }
    *reinterpret_cast<uint4*>(Qho + (cidx * C + i) * DK + c) = make_uint4(qo[0], qo[1], qo[2], qo[3]);
    *reinterpret_cast<uint4*>(Kto + (cidx * C + i) * DK + c) = make_uint4(ko[0], ko[1], ko[2], ko[3]);
  }
  if (threadIdx.x == 0) gCo[cidx] = __expf(glast);
  __syncthreads();
  // V into the Q buffer while the inverse runs
  load_tile(&sm.QV[0][0], QP, v + (tok0 * H + h) * DV, (long long)H * DV, C, DV);
  cp_commit();
  tri_inverse_inplace(sm.M);

  // T to bf16; K -> diag(b G) K in place; then V -> diag(b) V
  for (int idx = threadIdx.x; idx < C * C; idx += THREADS) {
    const int i = idx / C, j = idx % C;
    sm.Tb[i][j] = f2bf(sm.M[i][j]);
  }
  for (int idx = threadIdx.x; idx < C * (DK / 8); idx += THREADS) {
    const int i = idx / (DK / 8), c = (idx % (DK / 8)) * 8;
    const float bg = sm.beta[i] * __expf(sm.gam[i]);
    uint4 kv = *reinterpret_cast<const uint4*>(&sm.K[i][c]);
    uint32_t* kw = reinterpret_cast<uint32_t*>(&kv);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float2 b2 = unpack_bf16x2(kw[u]);
      kw[u] = pack_bf16x2(bg * b2.x, bg * b2.y);
    }
    *reinterpret_cast<uint4*>(&sm.K[i][c]) = kv;
  }
  cp_wait_all();
  __syncthreads();
  for (int idx = threadIdx.x; idx < C * (DV / 8); idx += THREADS) {
    const int i = idx / (DV / 8), c = (idx % (DV / 8)) * 8;
    const float bi = sm.beta[i];
    uint4 vv = *reinterpret_cast<const uint4*>(&sm.QV[i][c]);
    uint32_t* vw = reinterpret_cast<uint32_t*>(&vv);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float2 b2 = unpack_bf16x2(vw[u]);
      vw[u] = pack_bf16x2(bi * b2.x, bi * b2.y);
    }
    *reinterpret_cast<uint4*>(&sm.QV[i][c]) = vv;
  }
  __syncthreads();

  // W = T Xw, U = T Xu: warp tile 16 rows x (D / 2) columns
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
    warp_mma<1, NT, false, true>(acc, &sm.Tb[0][0], C + PAD, &sm.QV[0][0], QP, m0, c0, C);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int i = m0 + frag_row(0, e), c = c0 + frag_col(nt, e);
        *reinterpret_cast<uint32_t*>(Uo + (cidx * C + i) * DV + c) = pack_bf16x2(acc[0][nt][e], acc[0][nt][e + 1]);
      }
  }
}

// ------------------------------------------------------------------ backward --

// Backward shared memory, about 110 KB for dk = dv = 256 (two CTAs per SM):
// K stays resident; the feature dimension of Q, V, dW and dU is processed in
// two halves through three half-width buffers.
template <int DK, int DV>
struct BwdSmem {
  static constexpr int HK = DK / 2, HV = DV / 2;
  static constexpr int HP = cmax(cmax(HK, HV), C) + PAD;     // half-buffer pitch (elements)
  __nv_bfloat16 K[C][DK + PAD];
  __nv_bfloat16 H0[C][HP];     // Q lo (KK/QK) | V half (pass A) | dT bf16 | Q half (pass B)
  __nv_bfloat16 H1[C][HP];     // Q hi (KK/QK) | dW half (pass A) | P bf16 | dQK bf16
  __nv_bfloat16 H2[C][HP];     // dU half (pass A) | dW half (pass B)
  float F[C][C + 1];           // M -> T | dM | dKK, then (C x (C + PAD)) bf16 dKK + dKK^T
  __nv_bfloat16 Tb[C][C + PAD];
  float gam[C], beta[C], graw[C];
  float rw[C];     // sum_c dXw K         (-> dbeta * G, dG * beta)
  float ru[C];     // sum_c dXu V         (-> dbeta)
  float rq[C];     // sum_c dQh Q         (-> dG)
  float rk[C];     // sum_c dKt K         (-> dgamma via G_C / G)
  float rm[C];     // sum_j dM KK D       (-> dbeta)
  float dgam[C];
};

// Phase clock of the backward's CTA (0, 0, 0): clock64() at phase boundaries
// into g_gdr_intra_trace[event] (16 u64); null: off.
__device__ unsigned long long* g_gdr_intra_trace_dev = nullptr;
#define GDR_TR(ev)                                                                                       \
  do {                                                                                                   \
    unsigned long long* tr_ = g_gdr_intra_trace_dev;                                                     \
    if (tr_ != nullptr && threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)    \
      tr_[ev] = clock64();                                                                               \
  } while (0)

template <int NT>
__device__ __forceinline__ void row_dot_accumulate(const float (&acc)[1][NT][4], const __nv_bfloat16* X, int ldx,
                                                   int m0, int c0, float* out) {
  // out[i] += sum over this warp's fragment of acc[i][c] * X[i][c]
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
    float s = part[r];
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if ((threadIdx.x & 3) == 0) atomicAdd(&out[m0 + ((threadIdx.x & 31) >> 2) + 8 * r], s);
  }
}

template <int DK, int DV>
__global__ void __launch_bounds__(THREADS, 2)
intra_bwd_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                 const __nv_bfloat16* __restrict__ v, const float* __restrict__ g, const float* __restrict__ beta,
                 const __nv_bfloat16* __restrict__ dW, const __nv_bfloat16* __restrict__ dQh,
                 const __nv_bfloat16* __restrict__ dKt, const float* __restrict__ dA, const __nv_bfloat16* __restrict__ dU, const float* __restrict__ dgC,
                 __nv_bfloat16* __restrict__ dq, __nv_bfloat16* __restrict__ dk, __nv_bfloat16* __restrict__ dv,
                 float* __restrict__ dg, float* __restrict__ dbeta, int L, int H, float scale) {
  using S = BwdSmem<DK, DV>;
  constexpr int HK = S::HK, HV = S::HV, HP = S::HP, KP = DK + PAD;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  S& sm = *reinterpret_cast<S*>(smem_raw);
  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int N = gridDim.x;
  const long long bh = (long long)b * H + h;
  const long long cidx = bh * N + n;
  const long long tok0 = (long long)b * L + (long long)n * C;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int tid = threadIdx.x;
  const int m0 = (warp & 3) * 16, n0 = (warp >> 2) * 32;
  const __nv_bfloat16* qrow = q + (tok0 * H + h) * DK;
  const __nv_bfloat16* krow = k + (tok0 * H + h) * DK;
  const __nv_bfloat16* vrow = v + (tok0 * H + h) * DV;
  const long long qld = (long long)H * DK, vld = (long long)H * DV;

  // ---- phase 1: K, Q; gates; KK, QK (kept in registers); M -> T
  GDR_TR(0);
  load_tile(&sm.K[0][0], KP, krow, qld, C, DK);
  load_tile(&sm.H0[0][0], HP, qrow, qld, C, HK);
  load_tile(&sm.H1[0][0], HP, qrow + HK, qld, C, HK);
  cp_commit();
  if (tid < C) {
    sm.graw[tid] = g[(tok0 + tid) * H + h];
    sm.beta[tid] = beta[(tok0 + tid) * H + h];
    sm.rw[tid] = sm.ru[tid] = sm.rq[tid] = sm.rk[tid] = sm.rm[tid] = sm.dgam[tid] = 0.f;
  }
  __syncthreads();
  if (warp == 0) chunk_cumsum(sm.graw, sm.gam);
  cp_wait_all();
  __syncthreads();
  float kk[1][4][4], qk[1][4][4];
  zero(kk);
  zero(qk);
  warp_mma<1, 4, false, false>(kk, &sm.K[0][0], KP, &sm.K[0][0], KP, m0, n0, DK);
  warp_mma<1, 4, false, false>(qk, &sm.H0[0][0], HP, &sm.K[0][0], KP, m0, n0, HK);
  warp_mma<1, 4, false, false>(qk, &sm.H1[0][0], HP, &sm.K[0][0] + HK, KP, m0, n0, HK);
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = m0 + frag_row(0, e), j = n0 + frag_col(nt, e);
      sm.F[i][j] = (j < i) ? sm.beta[i] * kk[0][nt][e] * __expf(sm.gam[i] - sm.gam[j]) : 0.f;
    }
  __syncthreads();
  GDR_TR(1);
  tri_inverse_inplace(sm.F);
  GDR_TR(2);
  for (int idx = tid; idx < C * C; idx += THREADS) sm.Tb[idx / C][idx % C] = f2bf(sm.F[idx / C][idx % C]);

  // ---- pass A over feature halves: dV, row dots, dT partial products
  float a1[1][4][4], a2[1][4][4];     // dW K^T and dU V^T
  zero(a1);
  zero(a2);
#pragma unroll 1
  for (int hf = 0; hf < 2; ++hf) {
    __syncthreads();
    load_tile(&sm.H0[0][0], HP, vrow + hf * HV, vld, C, HV);
    load_tile(&sm.H2[0][0], HP, dU + cidx * C * DV + hf * HV, DV, C, HV);
    load_tile(&sm.H1[0][0], HP, dW + cidx * C * DK + hf * HK, DK, C, HK);
    cp_commit();
    cp_wait_all();
    __syncthreads();
    {
      // dXu = T^T dU  ->  dV = diag(b) dXu ; ru += dXu . V
      constexpr int NT = HV / 16;
      const int c0 = (warp >> 2) * (HV / 2);
      float acc[1][NT][4];
      zero(acc);
      warp_mma<1, NT, true, true>(acc, &sm.Tb[0][0], C + PAD, &sm.H2[0][0], HP, m0, c0, C);
      row_dot_accumulate<NT>(acc, &sm.H0[0][0], HP, m0, c0, sm.ru);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int i = m0 + frag_row(0, e), c = c0 + frag_col(nt, e);
          *reinterpret_cast<uint32_t*>(dv + ((tok0 + i) * H + h) * DV + hf * HV + c) =
              pack_bf16x2(sm.beta[i] * acc[0][nt][e], sm.beta[i] * acc[0][nt][e + 1]);
        }
    }
    {
      // dXw = T^T dW ; rw += dXw . K
      constexpr int NT = HK / 16;
      const int c0 = (warp >> 2) * (HK / 2);
      float acc[1][NT][4];
      zero(acc);
      warp_mma<1, NT, true, true>(acc, &sm.Tb[0][0], C + PAD, &sm.H1[0][0], HP, m0, c0, C);
      row_dot_accumulate<NT>(acc, &sm.K[0][0] + hf * HK, KP, m0, c0, sm.rw);
    }
    warp_mma<1, 4, false, false>(a1, &sm.H1[0][0], HP, &sm.K[0][0] + hf * HK, KP, m0, n0, HK);
    warp_mma<1, 4, false, false>(a2, &sm.H2[0][0], HP, &sm.H0[0][0], HP, m0, n0, HV);
  }
  __syncthreads();

  GDR_TR(3);
  // ---- dT = (dW K^T) diag(b G) + (dU V^T) diag(b)  (bf16 into H0)
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      const int i = m0 + frag_row(0, e), j = n0 + frag_col(nt, e);
      const float x0 = sm.beta[j] * (__expf(sm.gam[j]) * a1[0][nt][e] + a2[0][nt][e]);
      const float x1 = sm.beta[j + 1] * (__expf(sm.gam[j + 1]) * a1[0][nt][e + 1] + a2[0][nt][e + 1]);
      *reinterpret_cast<uint32_t*>(&sm.H0[i][j]) = pack_bf16x2(x0, x1);
    }
  __syncthreads();
  // P = T^T dT (bf16 into H1), dM = -strict_lower(P T^T) (fragments)
  {
    float p[1][4][4];
    zero(p);
    warp_mma<1, 4, true, true>(p, &sm.Tb[0][0], C + PAD, &sm.H0[0][0], HP, m0, n0, C);
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int i = m0 + frag_row(0, e), j = n0 + frag_col(nt, e);
        *reinterpret_cast<uint32_t*>(&sm.H1[i][j]) = pack_bf16x2(p[0][nt][e], p[0][nt][e + 1]);
      }
  }
  __syncthreads();
  float dm[1][4][4];
  zero(dm);
  warp_mma<1, 4, false, false>(dm, &sm.H1[0][0], HP, &sm.Tb[0][0], C + PAD, m0, n0, C);
  __syncthreads();                            // P (H1) consumed

  GDR_TR(4);
  // ---- elementwise on the fragments: dKK (into F), dQK (bf16 into H1),
  //      gate gradients of D, dbeta partials
  {
    const float* dArow = dA + cidx * C * C;
    float rowg[2] = {0.f, 0.f}, rowm[2] = {0.f, 0.f}, colg[4][2];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) colg[nt][0] = colg[nt][1] = 0.f;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = m0 + frag_row(0, e), j = n0 + frag_col(nt, e);
        float dkk = 0.f, dqk = 0.f;
        if (j <= i) {
          const float d = __expf(sm.gam[i] - sm.gam[j]);
          const float da = dArow[i * C + j];
          dqk = scale * da * d;
          float dd = scale * da * qk[0][nt][e];
          if (j < i) {
            const float dmv = -dm[0][nt][e];
            dkk = dmv * sm.beta[i] * d;
            rowm[e >> 1] += dmv * kk[0][nt][e] * d;
            dd += dmv * sm.beta[i] * kk[0][nt][e];
            const float t = dd * d;
            rowg[e >> 1] += t;
            colg[nt][e & 1] -= t;
          }
        }
        sm.F[i][j] = dkk;
        dm[0][nt][e] = dqk;                   // reuse the register for dQK
      }
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int i = m0 + frag_row(0, e), j = n0 + frag_col(nt, e);
        *reinterpret_cast<uint32_t*>(&sm.H1[i][j]) = pack_bf16x2(dm[0][nt][e], dm[0][nt][e + 1]);
      }
    // row sums over the 4 lanes of a row, column sums over the 8 lanes of a column
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float sg = rowg[r], smv = rowm[r];
      sg += __shfl_xor_sync(0xffffffffu, sg, 1);
      sg += __shfl_xor_sync(0xffffffffu, sg, 2);
      smv += __shfl_xor_sync(0xffffffffu, smv, 1);
      smv += __shfl_xor_sync(0xffffffffu, smv, 2);
      if ((lane & 3) == 0) {
        atomicAdd(&sm.dgam[m0 + (lane >> 2) + 8 * r], sg);
        atomicAdd(&sm.rm[m0 + (lane >> 2) + 8 * r], smv);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float sc = colg[nt][c];
        sc += __shfl_xor_sync(0xffffffffu, sc, 4);
        sc += __shfl_xor_sync(0xffffffffu, sc, 8);
        sc += __shfl_xor_sync(0xffffffffu, sc, 16);
        if (lane < 4) atomicAdd(&sm.dgam[n0 + nt * 8 + lane * 2 + c], sc);
      }
  }
  __syncthreads();
  // dKK + dKK^T as bf16 over F's storage (read everything first)
  __nv_bfloat16 (*dKKb)[C + PAD] = reinterpret_cast<__nv_bfloat16 (*)[C + PAD]>(&sm.F[0][0]);
  {
    float sym[C * C / THREADS];
#pragma unroll
    for (int u = 0; u < C * C / THREADS; ++u) {
      const int idx = tid + u * THREADS, i = idx / C, j = idx % C;
      sym[u] = sm.F[i][j] + sm.F[j][i];
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < C * C / THREADS; ++u) {
      const int idx = tid + u * THREADS, i = idx / C, j = idx % C;
      dKKb[i][j] = f2bf(sym[u]);
    }
  }

  GDR_TR(5);
  // ---- pass B over feature halves: dK, dQ
  const float glast = sm.gam[C - 1];
#pragma unroll 1
  for (int hf = 0; hf < 2; ++hf) {
    __syncthreads();
    load_tile(&sm.H0[0][0], HP, qrow + hf * HK, qld, C, HK);
    load_tile(&sm.H2[0][0], HP, dW + cidx * C * DK + hf * HK, DK, C, HK);
    cp_commit();
    cp_wait_all();
    __syncthreads();
    constexpr int NT = HK / 16;
    const int c0 = (warp >> 2) * (HK / 2);
    const __nv_bfloat16* Kh = &sm.K[0][0] + hf * HK;
    {
      // dK = diag(b G) T^T dW + (dKK + dKK^T) K + dQK^T Q + diag(G_C / G) dKt
      float acc[1][NT][4];
      zero(acc);
      warp_mma<1, NT, true, true>(acc, &sm.Tb[0][0], C + PAD, &sm.H2[0][0], HP, m0, c0, C);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = m0 + frag_row(0, e);
          acc[0][nt][e] *= sm.beta[i] * __expf(sm.gam[i]);
        }
      warp_mma<1, NT, false, true>(acc, &dKKb[0][0], C + PAD, Kh, KP, m0, c0, C);
      warp_mma<1, NT, true, true>(acc, &sm.H1[0][0], HP, &sm.H0[0][0], HP, m0, c0, C);
      float part[2] = {0.f, 0.f};
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int i = m0 + frag_row(0, e), c = c0 + frag_col(nt, e);
          const float ei = __expf(glast - sm.gam[i]);
          const float2 dkt = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(dKt + (cidx * C + i) * DK + hf * HK + c));
          const float2 kv = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(Kh + i * KP + c));
          part[e >> 1] += dkt.x * kv.x + dkt.y * kv.y;
          *reinterpret_cast<uint32_t*>(dk + ((tok0 + i) * H + h) * DK + hf * HK + c) =
              pack_bf16x2(acc[0][nt][e] + ei * dkt.x, acc[0][nt][e + 1] + ei * dkt.y);
        }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float s = part[r];
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        if ((lane & 3) == 0) atomicAdd(&sm.rk[m0 + (lane >> 2) + 8 * r], s);
      }
    }
    {
      // dQ = dQK K + s diag(G) dQh
      float acc[1][NT][4];
      zero(acc);
      warp_mma<1, NT, false, true>(acc, &sm.H1[0][0], HP, Kh, KP, m0, c0, C);
      float part[2] = {0.f, 0.f};
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int i = m0 + frag_row(0, e), c = c0 + frag_col(nt, e);
          const float gi = __expf(sm.gam[i]);
          const float2 dqh = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(dQh + (cidx * C + i) * DK + hf * HK + c));
          const float2 qv = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(&sm.H0[i][c]));
          part[e >> 1] += dqh.x * qv.x + dqh.y * qv.y;
          *reinterpret_cast<uint32_t*>(dq + ((tok0 + i) * H + h) * DK + hf * HK + c) =
              pack_bf16x2(acc[0][nt][e] + scale * gi * dqh.x, acc[0][nt][e + 1] + scale * gi * dqh.y);
        }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float s = part[r];
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        if ((lane & 3) == 0) atomicAdd(&sm.rq[m0 + (lane >> 2) + 8 * r], s);
      }
    }
  }
  __syncthreads();

  GDR_TR(6);
  // ---- per-row scalars, reverse cumsum
  if (warp == 0) {
    float dgl[2], tail = 0.f;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int i = 2 * lane + r;
      const float gi = __expf(sm.gam[i]);
      const float ei = __expf(glast - sm.gam[i]);
      const float dG = sm.beta[i] * sm.rw[i] + scale * sm.rq[i];
      dgl[r] = sm.dgam[i] + dG * gi - ei * sm.rk[i];
      tail += ei * sm.rk[i];
      dbeta[(tok0 + i) * H + h] = gi * sm.rw[i] + sm.ru[i] + sm.rm[i];
    }
    tail = warp_sum(tail);
    if (lane == 31) dgl[1] += tail + dgC[cidx] * __expf(glast);
    // reverse inclusive cumsum over i (64 values, 2 per lane)
    float s = dgl[0] + dgl[1];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float t = __shfl_down_sync(0xffffffffu, s, o);
      if (lane + o < 32) s += t;
    }
    dg[(tok0 + 2 * lane + 1) * H + h] = s - dgl[0];
    dg[(tok0 + 2 * lane) * H + h] = s;
  }
  GDR_TR(7);
}

template <int DK, int DV>
int launch_fwd(const GdrIntraArgs& a, cudaStream_t st) {
  const size_t sm = sizeof(FwdSmem<DK, DV>);
  auto kern = intra_fwd_kernel<DK, DV>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm));
  dim3 grid(static_cast<unsigned>(a.L / C), a.H, static_cast<unsigned>(a.B));
  kern<<<grid, THREADS, sm, st>>>((const __nv_bfloat16*)a.q, (const __nv_bfloat16*)a.k, (const __nv_bfloat16*)a.v,
                                  a.g, a.beta, (__nv_bfloat16*)a.W, (__nv_bfloat16*)a.Qh, (__nv_bfloat16*)a.Kt,
                                  (__nv_bfloat16*)a.A, (__nv_bfloat16*)a.U, a.gC, static_cast<int>(a.L), a.H, a.scale);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

template <int DK, int DV>
int launch_bwd(const GdrIntraBwdArgs& a, cudaStream_t st) {
  const size_t sm = sizeof(BwdSmem<DK, DV>);
  auto kern = intra_bwd_kernel<DK, DV>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm));
  dim3 grid(static_cast<unsigned>(a.f.L / C), a.f.H, static_cast<unsigned>(a.f.B));
  kern<<<grid, THREADS, sm, st>>>((const __nv_bfloat16*)a.f.q, (const __nv_bfloat16*)a.f.k,
                                  (const __nv_bfloat16*)a.f.v, a.f.g, a.f.beta, (const __nv_bfloat16*)a.dW,
                                  (const __nv_bfloat16*)a.dQh, (const __nv_bfloat16*)a.dKt, a.dA,
                                  (const __nv_bfloat16*)a.dU, a.dgC, (__nv_bfloat16*)a.dq, (__nv_bfloat16*)a.dk,
                                  (__nv_bfloat16*)a.dv, a.dg, a.dbeta, static_cast<int>(a.f.L), a.f.H, a.f.scale);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

}  // namespace

int gdr_intra_fwd(const GdrIntraArgs& a, cudaStream_t st) {
  if (a.L % C) return 5;
  if (a.DK == 256 && a.DV == 256) return launch_fwd<256, 256>(a, st);
  if (a.DK == 128 && a.DV == 128) return launch_fwd<128, 128>(a, st);
  if (a.DK == 128 && a.DV == 256) return launch_fwd<128, 256>(a, st);
  return 5;
}

void gdr_intra_set_trace(unsigned long long* buf) {
  cudaMemcpyToSymbol(g_gdr_intra_trace_dev, &buf, sizeof(buf));
}

int gdr_intra_bwd(const GdrIntraBwdArgs& a, cudaStream_t st) {
  if (a.f.L % C) return 5;
  if (a.f.DK == 256 && a.f.DV == 256) return launch_bwd<256, 256>(a, st);
  if (a.f.DK == 128 && a.f.DV == 128) return launch_bwd<128, 128>(a, st);
  if (a.f.DK == 128 && a.f.DV == 256) return launch_bwd<128, 256>(a, st);
  return 5;
}

}  // namespace vagus
