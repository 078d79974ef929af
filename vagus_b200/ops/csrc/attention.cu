// Flash attention (causal with lower-right alignment, or full), forward and
// backward, bf16 in / fp32 statistics, GQA, head dims 64 and 128.
//
// Forward: one CTA per (128 queries, batch * head); 8 warps, 16 query rows
// each.  Key/value tiles of 64 rows stream through a double-buffered
// cp.async ring; S = Q K^T and O += P V run on the tensor cores (mma.sync
// m16n8k16, fp32 accumulate) with the online softmax in registers: the S
// accumulator fragments of two adjacent 8-key tiles are exactly the A
// fragment of the next product, so P never leaves registers.  Writes O and
// the row log-sum-exp (natural log) for the backward.
//
// Backward: one CTA per (64 keys, batch * kv-head); 8 warps.  The CTA keeps
// its K / V tile and accumulates dK, dV in registers while it walks the
// query blocks of every query head that shares the kv head (GQA needs no
// atomics for dK / dV): P = exp(S - lse), dP = dO V^T, dS = P (dP - delta)
// with delta = rowsum(dO o O) from a small pre-pass; P and dS go through
// shared memory as bf16 for dV += P^T dO, dK += dS^T Q and dQ += dS K (fp32
// atomics into a scratch buffer, scaled and rounded by a last pass).
//
// Causal masking is lower-right aligned: query i sits at absolute position
// Lk - Lq + i and sees keys j <= Lk - Lq + i.  Fully masked tiles are skipped.
//
// The forward of problems with Lq, Lk >= 128 and D = Dv in {64, 128} runs on
// the 5th-generation tensor cores instead (attn_fwd_tc below); the mma.sync
// forward above serves the small / odd shapes (decode, Lq < 128).
#include "common.cuh"
#include "gemm.h"
#include "kernels.h"
#include "mma.cuh"

#include <cmath>
#include <cstdlib>

namespace vagus {
namespace {

using namespace mma;

constexpr float kLog2e = 1.4426950408889634f;

// ---------------------------------------------------------------- forward --

constexpr int FQ = 128;      // queries per CTA
constexpr int FK = 64;       // keys per tile
constexpr int FWARPS = 8;

template <int D, int DV>
struct FwdSmem {
  __nv_bfloat16 Q[FQ][D + PAD];
  __nv_bfloat16 K[2][FK][D + PAD];
  __nv_bfloat16 V[2][FK][DV + PAD];
};

template <int D, int DV>
__global__ void __launch_bounds__(FWARPS * 32, 1)
attn_fwd_kernel(const AttnArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  FwdSmem<D, DV>& sm = *reinterpret_cast<FwdSmem<D, DV>*>(smem_raw);
  const int qb = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / a.H, h = bh % a.H;
  const int hk = h / (a.H / a.Hk);
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int q0 = qb * FQ;
  const int offs = a.Lk - a.Lq;                       // lower-right alignment
  const __nv_bfloat16* Qg = reinterpret_cast<const __nv_bfloat16*>(a.q) + b * a.sq_b + h * a.sq_h;
  const __nv_bfloat16* Kg = reinterpret_cast<const __nv_bfloat16*>(a.k) + b * a.sk_b + hk * a.sk_h;
  const __nv_bfloat16* Vg = reinterpret_cast<const __nv_bfloat16*>(a.v) + b * a.sv_b + hk * a.sv_h;

  // tiles: rows past the end are zero-filled
  auto load_rows = [&](__nv_bfloat16* s, int sp, const __nv_bfloat16* g, long long gp, int r0, int nrows,
                       int limit, int cols) {
    const int per_row = cols / 8;
    for (int i = threadIdx.x; i < nrows * per_row; i += blockDim.x) {
      const int r = i / per_row, c = (i - r * per_row) * 8;
      if (r0 + r < limit) cp_async16(s + r * sp + c, g + (long long)(r0 + r) * gp + c);
      else *reinterpret_cast<uint4*>(s + r * sp + c) = make_uint4(0, 0, 0, 0);
    }
  };
  // last key any query of this CTA may see
  const int q_last = min(q0 + FQ, a.Lq) - 1;
  const int k_end = a.causal ? min(a.Lk, q_last + offs + 1) : a.Lk;
  const int ntiles = (k_end + FK - 1) / FK;

  load_rows(&sm.Q[0][0], D + PAD, Qg, a.sq_l, q0, FQ, a.Lq, D);
  if (ntiles > 0) {
    load_rows(&sm.K[0][0][0], D + PAD, Kg, a.sk_l, 0, FK, a.Lk, D);
    load_rows(&sm.V[0][0][0], DV + PAD, Vg, a.sv_l, 0, FK, a.Lk, DV);
  }
  cp_commit();

  constexpr int NO = DV / 8;                          // O n-tiles per warp (all of DV)
  float o[1][NO][4];
  zero(o);
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  const float sl2 = a.scale * kLog2e;
  const int r_lo = q0 + warp * 16 + (lane >> 2);       // this thread's two query rows
  const int rows[2] = {r_lo, r_lo + 8};

  for (int t = 0; t < ntiles; ++t) {
    const int buf = t & 1;
    if (t + 1 < ntiles) {
      load_rows(&sm.K[buf ^ 1][0][0], D + PAD, Kg, a.sk_l, (t + 1) * FK, FK, a.Lk, D);
      load_rows(&sm.V[buf ^ 1][0][0], DV + PAD, Vg, a.sv_l, (t + 1) * FK, FK, a.Lk, DV);
    }
    cp_commit();
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    __syncthreads();

    float s[1][FK / 8][4];
    zero(s);
    warp_mma<1, FK / 8, false, false>(s, &sm.Q[0][0], D + PAD, &sm.K[buf][0][0], D + PAD, warp * 16, 0, D);

    // mask, scale to log2 units, running max
    const int k0 = t * FK;
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int nt = 0; nt < FK / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kj = k0 + nt * 8 + (lane & 3) * 2 + (e & 1);
        const int qi = rows[e >> 1];
        const bool ok = kj < a.Lk && (!a.causal || kj <= qi + offs);
        const float v = ok ? s[0][nt][e] * sl2 : -INFINITY;
        s[0][nt][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      alpha[r] = (mx[r] == -INFINITY) ? 1.f : exp2f(m_r[r] - mx[r]);
      m_r[r] = mx[r];
    }
    float ls[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < FK / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mr = m_r[e >> 1];
        const float p = (mr == -INFINITY) ? 0.f : exp2f(s[0][nt][e] - mr);
        s[0][nt][e] = p;
        ls[e >> 1] += p;
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) l_r[r] = l_r[r] * alpha[r] + ls[r];
#pragma unroll
    for (int nt = 0; nt < NO; ++nt) {
      o[0][nt][0] *= alpha[0]; o[0][nt][1] *= alpha[0];
      o[0][nt][2] *= alpha[1]; o[0][nt][3] *= alpha[1];
    }
    // O += P V: P fragments straight from the S accumulators
    const int l8 = lane & 7, j = lane >> 3;
#pragma unroll
    for (int kk = 0; kk < FK / 16; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16x2(s[0][2 * kk][0], s[0][2 * kk][1]);
      pa[1] = pack_bf16x2(s[0][2 * kk][2], s[0][2 * kk][3]);
      pa[2] = pack_bf16x2(s[0][2 * kk + 1][0], s[0][2 * kk + 1][1]);
      pa[3] = pack_bf16x2(s[0][2 * kk + 1][2], s[0][2 * kk + 1][3]);
#pragma unroll
      for (int nt = 0; nt < NO; nt += 2) {
        uint32_t bfr[4];
        ldsm4t(bfr, &sm.V[buf][kk * 16 + l8 + (j & 1) * 8][nt * 8 + (j >> 1) * 8]);
        mma16816(o[0][nt], pa, bfr[0], bfr[1]);
        mma16816(o[0][nt + 1], pa, bfr[2], bfr[3]);
      }
    }
    __syncthreads();                                   // buffer reused two tiles on
  }
  cp_wait_all();

  // normalise and store
  float inv[2], lse[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float l = l_r[r];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    inv[r] = l > 0.f ? 1.f / l : 0.f;
    lse[r] = l > 0.f ? (m_r[r] + log2f(l)) / kLog2e : -INFINITY;
  }
  __nv_bfloat16* Og = reinterpret_cast<__nv_bfloat16*>(a.o) + b * a.so_b + h * a.so_h;
#pragma unroll
  for (int nt = 0; nt < NO; ++nt)
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      const int qi = rows[e >> 1];
      if (qi < a.Lq) {
        const int c = nt * 8 + (lane & 3) * 2;
        *reinterpret_cast<uint32_t*>(Og + (long long)qi * a.so_l + c) =
            pack_bf16x2(o[0][nt][e] * inv[e >> 1], o[0][nt][e + 1] * inv[e >> 1]);
      }
    }
  if ((lane & 3) == 0) {
#pragma unroll
    for (int r = 0; r < 2; ++r)
      if (rows[r] < a.Lq) a.lse[((long long)b * a.H + h) * a.Lq + rows[r]] = lse[r];
  }
}

// ------------------------------------------------------ tcgen05 forward --
// One CTA per (128 queries, batch * head), 10 warps:
//   warp 0      TMA: the Q tile once, then K / V tiles of 128 keys (K in a
//               two-stage ring, V in NV stages);
//   warp 1      TMEM owner and MMA issuer: S_j = Q K_j^T (M=128, N=128)
//               into a TMEM score buffer (with two buffers, issued one tile
//               ahead; with one, as soon as the softmax warps have read
//               S_{j-1}), then O += P_j V_j (M=128, N=D, K=128 keys) into the
//               TMEM output accumulator;
//   warps 2-9   softmax, two threads per query row (each half of the key
//               columns): tcgen05.ld of the score row, running max / sum in
//               registers (the pair agrees on the max through shared memory),
//               exponentials on the MUFU ex2 unit, P_j written as bf16 into
//               shared memory in the 128-byte-swizzled K-major layout the MMA
//               reads; the output is rescaled in TMEM only when the running
//               max grows by more than 2^8 (otherwise P is taken against the
//               stale max, at most 256x larger, harmless in fp32 / bf16).
// Barriers: q_full, k_full[2] / k_empty[2] and v_full[NV] / v_empty[NV]
// (loader <-> MMA; a K stage frees as soon as its score product is done, so
// K loads run a tile further ahead than V), s_full[NS] / s_free[NS] (MMA <->
// softmax), p_full (softmax -> MMA), o_done (MMA -> softmax: P buffer free
// and O stable).  Every wait is bounded.
extern unsigned long long* g_attn_trace;   // host side of the phase trace (attn_set_trace)

// 2^x on the FMA and integer pipes, for x <= 0 (clamped at -126): x = n + f
// with n = round(x) (adding and subtracting 1.5 * 2^23 rounds in the
// mantissa), 2^f by a cubic least-squares fit on [-1/2, 1/2] (maximum
// relative error 7.5e-5, under half a bf16 ulp: the result is rounded to
// bf16 for the tensor core), 2^n added to the exponent field.  In the
// forward's softmax loop 2 of every 8 exponentials take this path and the
// rest the MUFU unit (measured: 537 -> 523 us at head dim 64; 4 of 8 was
// slower, and the backward, whose transcendental pipe is the busiest, gained
// nothing from 2 or 4 of 8).
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -126.f);
  const float sh = 12582912.f;
  const float t = x + sh;
  const float f = x - (t - sh);
  float q = fmaf(0.05517146f, f, 0.24261086f);
  q = fmaf(q, f, 0.69326099f);
  q = fmaf(q, f, 0.99992809f);
  return __int_as_float(__float_as_int(q) + ((__float_as_int(t) - __float_as_int(sh)) << 23));
}
template <int PX>
__device__ __forceinline__ float ex2_mix(float x, int i) {
  if ((i & 7) < PX) return ex2_poly(x);
  return ex2_approx(x);
}

namespace tcfa {
constexpr int BQ = 128, BKV = 128, THREADS = 320;   // 10 warps
constexpr float kRescale = 8.f;     // log2 units

// Head dim 64 runs two CTAs per SM (the two CTAs' tiles interleave on the
// tensor core and the MUFU): one TMEM score buffer and one V stage, so each
// CTA holds 256 TMEM columns and under 100 KB of shared memory.  Head dim 128
// runs one CTA per SM with two score buffers (S_{j+1} computed while the
// softmax warps work on S_j) and two V stages.
template <int D>
struct Layout {
  static constexpr int CTAS = D == 64 ? 2 : 1;    // CTAs per SM
  static constexpr int NS = D == 64 ? 1 : 2;      // TMEM score buffers
  static constexpr int NV = D == 64 ? 1 : 2;      // V stages (K always has 2)
  static constexpr int Q_BYTES = BQ * D * 2;      // D/64 K-major chunks of 16 KB
  static constexpr int K_BYTES = BKV * D * 2;
  static constexpr int V_BYTES = BKV * D * 2;     // 2 key chunks x D/64 MN-major blocks of 8 KB
  static constexpr int P_BYTES = BQ * BKV * 2;    // 2 K-major chunks of 16 KB
  static constexpr int OFF_K = Q_BYTES;
  static constexpr int OFF_V = OFF_K + 2 * K_BYTES;
  static constexpr int OFF_P = OFF_V + NV * V_BYTES;
  static constexpr int OFF_BAR = OFF_P + P_BYTES;
  // barriers, TMEM slot, then [2][128] row maxima and [2][128] row sums
  static constexpr int BAR_BYTES = 128 + 2 * 2 * BQ * 4;
  static constexpr int SMEM_MIN = CTAS == 1 ? 120 * 1024 : 0;   // one CTA: hold the SM (and its TMEM)
  static constexpr int SMEM = OFF_BAR + BAR_BYTES + 1024 > SMEM_MIN ? OFF_BAR + BAR_BYTES + 1024 : SMEM_MIN;
  static constexpr uint32_t TMEM_S = 0, TMEM_O = NS * BKV, TMEM_COLS = NS == 1 ? 256 : 512;
  static_assert(TMEM_O + D <= TMEM_COLS, "TMEM layout");
  static_assert(CTAS == 1 || SMEM <= 110 * 1024, "two CTAs per SM must fit the SM's shared memory");
};

struct Params {
  int Lq, Lk, H, Hk, causal;
  int lpt;                         // causal order: 0 plain, g > 0 longest query blocks first in groups of g heads
  float sl2;                       // scale * log2(e)
  void* o;
  long long so_b, so_h, so_l;
  float* lse;
  int* err;
  unsigned long long* trace;       // phase clock of the last query block of head 0, [tile][16]; null: off
};
}  // namespace tcfa

template <int D, int PX>
__global__ void __launch_bounds__(tcfa::THREADS, tcfa::Layout<D>::CTAS)
attn_fwd_tc(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
            const __grid_constant__ CUtensorMap mv, const tcfa::Params p) {
  using namespace tcfa;
  using Lt = Layout<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = sm;
  uint8_t* sk = sm + Lt::OFF_K;
  uint8_t* sv = sm + Lt::OFF_V;
  uint8_t* sp = sm + Lt::OFF_P;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Lt::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = bars + 3;
  uint64_t* v_full = bars + 5;
  uint64_t* v_empty = bars + 7;
  uint64_t* s_full = bars + 9;
  uint64_t* s_free = bars + 11;
  uint64_t* p_full = bars + 13;
  uint64_t* o_done = bars + 14;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  // causal: within groups of p.lpt heads, the longest query blocks (most key
  // tiles) launch first, so a group's last wave holds short blocks; the
  // resident CTAs share the K / V of at most a few groups (L2 reuse)
  int qb = blockIdx.x, bh = blockIdx.y;
  if (p.lpt > 0 && p.causal) {
    const int G = p.lpt;
    const int nq = gridDim.x, nbh = gridDim.y;
    const int lin = blockIdx.y * nq + blockIdx.x;
    const int grp = lin / (G * nq);
    const int gsz = min(G, nbh - grp * G);
    const int within = lin - grp * G * nq;
    qb = nq - 1 - within / gsz;
    bh = grp * G + within % gsz;
  }
  const int b = bh / p.H, h = bh % p.H;
  const int hk = h / (p.H / p.Hk);
  const int q0 = qb * BQ;
  const int offs = p.Lk - p.Lq;
  const int q_last = min(q0 + BQ, p.Lq) - 1;
  const int k_end = p.causal ? min(p.Lk, q_last + offs + 1) : p.Lk;
  const int ntiles = k_end > 0 ? (k_end + BKV - 1) / BKV : 0;
  const bool tracing = p.trace != nullptr && qb == static_cast<int>(gridDim.x) - 1 && bh == 0;
#define VAGUS_TRF(tile, ev)                                                     \
  do {                                                                          \
    if (tracing && (tile) < 32) p.trace[(tile) * 16 + (ev)] = clock64();        \
  } while (0)

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 8);
    }
    mbar_init(p_full, 8);
    mbar_init(o_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&mq);
    tma_prefetch_desc(&mk);
    tma_prefetch_desc(&mv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Lt::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- loads
    if (lane == 0 && ntiles > 0) {
      mbar_arrive_expect_tx(q_full, Lt::Q_BYTES);
      for (int c = 0; c < D / 64; ++c) tma_load_4d(sq + c * 16384, &mq, q_full, 64 * c, q0, h, b);
      // order K_0, K_1, V_0, K_2, V_1, ...: K_{j+1} waits for S_{j-1}, V_j for PV_{j-2}
      auto load_k = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(&k_empty[s], ((j >> 1) & 1) ^ 1, abort_flag, p.err, kErrTimeoutProducer)) return false;
        mbar_arrive_expect_tx(&k_full[s], Lt::K_BYTES);
        uint8_t* kd = sk + s * Lt::K_BYTES;
        for (int c = 0; c < D / 64; ++c) tma_load_4d(kd + c * 16384, &mk, &k_full[s], 64 * c, j * BKV, hk, b);
        return true;
      };
      auto load_v = [&](int j) -> bool {
        const int s = j % Lt::NV;
        if (!mbar_wait(&v_empty[s], ((j / Lt::NV) & 1) ^ 1, abort_flag, p.err, kErrTimeoutProducer)) return false;
        mbar_arrive_expect_tx(&v_full[s], Lt::V_BYTES);
        uint8_t* vd = sv + s * Lt::V_BYTES;
        for (int kc = 0; kc < 2; ++kc)
          for (int mb = 0; mb < D / 64; ++mb)
            tma_load_4d(vd + (kc * (D / 64) + mb) * 8192, &mv, &v_full[s], 64 * mb, j * BKV + 64 * kc, hk, b);
        return true;
      };
      bool lok = load_k(0);
      for (int j = 0; lok && j < ntiles; ++j) {
        if (j + 1 < ntiles) lok = load_k(j + 1);
        lok = lok && load_v(j);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0 && ntiles > 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(BQ, BKV, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16(BQ, D, false, true);
      bool ok = mbar_wait(q_full, 0, abort_flag, p.err, kErrTimeoutMma);
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;                    // K stage
        const int sb = j % Lt::NS;              // score buffer
        if (!mbar_wait(&k_full[s], (j >> 1) & 1, abort_flag, p.err, kErrTimeoutMma)) return false;
        if (j >= Lt::NS && !mbar_wait(&s_free[sb], ((j / Lt::NS) - 1) & 1, abort_flag, p.err, kErrTimeoutMma))
          return false;
        tc_fence_after();
        const uint32_t d = tmem_base + Lt::TMEM_S + static_cast<uint32_t>(sb * BKV);
        const uint32_t qa = smem_u32(sq), ka = smem_u32(sk + s * Lt::K_BYTES);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc_mma_f16(d, make_sw128_desc(qa + c * 16384 + kk * 32, 16, 1024),
                       make_sw128_desc(ka + c * 16384 + kk * 32, 16, 1024), idesc_s, (c | kk) ? 1u : 0u);
        tc_commit(&s_full[sb]);
        tc_commit(&k_empty[s]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < ntiles; ++j) {
        if (j + 1 < ntiles && !issue_s(j + 1)) break;
        VAGUS_TRF(j, 0);
        if (!mbar_wait_spin(p_full, j & 1, abort_flag, p.err, kErrTimeoutMma)) break;
        VAGUS_TRF(j, 1);
        const int s = j % Lt::NV;
        if (!mbar_wait(&v_full[s], (j / Lt::NV) & 1, abort_flag, p.err, kErrTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + Lt::TMEM_O;
        const uint32_t pa = smem_u32(sp), va = smem_u32(sv + s * Lt::V_BYTES);
#pragma unroll
        for (int kc = 0; kc < 2; ++kc)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc_mma_f16(d, make_sw128_desc(pa + kc * 16384 + kk * 32, 16, 1024),
                       make_sw128_desc(va + kc * (D / 64) * 8192 + kk * 2048, 8192, 1024), idesc_o,
                       (j > 0 || kc > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&v_empty[s]);
        tc_commit(o_done);
        VAGUS_TRF(j, 2);
      }
    }
  } else {
    // -------------------------------------------------------------- softmax
    // 8 warps: the warp pair (w, w + 4) shares TMEM lane quarter w & 3, i.e.
    // the same 32 query rows, and splits the 128 key columns (and the D
    // output columns) in halves; the pair agrees on the running max through
    // shared memory and a named barrier per quarter.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const int qi = q0 + row;
    const uint32_t t_lane = static_cast<uint32_t>(quarter * 32) << 16;
    float* xmax = reinterpret_cast<float*>(tmem_slot + 2);          // [2][128] partial row maxima
    float* xsum = xmax + 2 * BQ;                                    // [2][128] partial row sums
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    // kernel parameters in registers (the lambdas above take `p` by reference,
    // so reads through it in this loop would be memory loads)
    const float psl2 = p.sl2;
    const int Lk = p.Lk;
    const bool causal = p.causal != 0;
    // a failed (timed-out) wait does not leave the loop: the warp pair must
    // keep meeting at its named barrier, so the remaining tiles run on
    // whatever is in the buffers and the error word reports the failure
    for (int j = 0; j < ntiles; ++j) {
      const int s = j % Lt::NS;
      ok = ok && mbar_wait_spin(&s_full[s], (j / Lt::NS) & 1, abort_flag, p.err, kErrTimeoutEpilogue);
      if (warp == 2 && lane == 0) VAGUS_TRF(j, 3);
      tc_fence_after();
      float x[64];
      const uint32_t sa = tmem_base + t_lane + Lt::TMEM_S + static_cast<uint32_t>(s * BKV + 64 * half);
      tmem_ld_32x32b_x32(sa, *reinterpret_cast<uint32_t(*)[32]>(&x[0]));
      tmem_ld_32x32b_x32(sa + 32, *reinterpret_cast<uint32_t(*)[32]>(&x[32]));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[s]);
      if (warp == 2 && lane == 0) VAGUS_TRF(j, 4);
      const int k0 = j * BKV + 64 * half;
      // tiles wholly visible to every row of the CTA skip the per-element mask
      const bool full = (j * BKV + BKV <= Lk) && (!causal || j * BKV + BKV - 1 <= q0 + offs);
      float mt0 = -INFINITY, mt1 = -INFINITY, mt2 = -INFINITY, mt3 = -INFINITY;
      if (full) {
#pragma unroll
        for (int i = 0; i < 64; i += 4) {
          mt0 = fmaxf(mt0, x[i]); mt1 = fmaxf(mt1, x[i + 1]);
          mt2 = fmaxf(mt2, x[i + 2]); mt3 = fmaxf(mt3, x[i + 3]);
        }
      } else {
        const int lim = causal ? min(Lk - 1, qi + offs) : Lk - 1;   // last visible key
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          if (k0 + i > lim) x[i] = -INFINITY;
          mt0 = fmaxf(mt0, x[i]);
        }
      }
      // raw maxima -> scaled, combined with the partner warp
      float mt = fmaxf(fmaxf(mt0, mt1), fmaxf(mt2, mt3)) * psl2;
      if (warp == 2 && lane == 0) VAGUS_TRF(j, 5);
      xmax[half * BQ + row] = mt;
      asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
      if (warp == 2 && lane == 0) VAGUS_TRF(j, 6);
      mt = fmaxf(mt, xmax[(half ^ 1) * BQ + row]);
      const float m_new = fmaxf(m_run, mt);
      const bool resc = m_new > m_run + kRescale;     // false while the row has seen nothing
      float alpha = 1.f;
      if (resc) {
        alpha = ex2_approx(m_run - m_new);            // 0 when m_run is -inf
        l_run *= alpha;
        m_run = m_new;
      }
      const float nm = (m_run == -INFINITY) ? 0.f : -m_run;
      const float sl2 = (m_run == -INFINITY) ? 0.f : psl2;
      float ls0 = 0.f, ls1 = 0.f;
      // (2 of 8 on the FMA pipe, ex2_poly; packed f16x2 exponentials or 16
      // softmax warps instead of 8 measured no faster)
#pragma unroll
      for (int i = 0; i < 64; i += 2) {
        x[i] = ex2_mix<PX>(fmaf(x[i], sl2, nm), i);
        x[i + 1] = ex2_mix<PX>(fmaf(x[i + 1], sl2, nm), i + 1);
        ls0 += x[i];
        ls1 += x[i + 1];
      }
      if (m_run == -INFINITY) {
#pragma unroll
        for (int i = 0; i < 64; ++i) x[i] = 0.f;
        ls0 = ls1 = 0.f;
      }
      l_run += ls0 + ls1;
      // P packed to bf16 pairs now: the fp32 row is dead before the rescale
      // below needs its own 32 registers
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) pk[i] = pack_bf16x2(x[2 * i], x[2 * i + 1]);
      if (warp == 2 && lane == 0) VAGUS_TRF(j, 7);
      // PV_{j-1} must be done before P is overwritten or O rescaled
      if (j > 0) ok = ok && mbar_wait_spin(o_done, (j - 1) & 1, abort_flag, p.err, kErrTimeoutEpilogue);
      if (warp == 2 && lane == 0) VAGUS_TRF(j, 8);
      if (resc && j > 0) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          uint32_t r[32];
          const uint32_t ta = tmem_base + t_lane + Lt::TMEM_O + static_cast<uint32_t>(half * (D / 2) + 32 * c);
          tmem_ld_32x32b_x32(ta, r);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
          tmem_st_32x32b_x32(ta, r);
        }
        tmem_st_wait();
      }
      // this half's 64 keys are P chunk `half`: bf16, 128-byte-swizzled K-major
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint4 w = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        *reinterpret_cast<uint4*>(sp + half * 16384 + row * 128 + ((u ^ (row & 7)) * 16)) = w;
      }
      if (warp == 2 && lane == 0) VAGUS_TRF(j, 9);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      if (warp == 2 && lane == 0) VAGUS_TRF(j, 10);
    }
    // ------------------------------------------------------------ epilogue
    xsum[half * BQ + row] = l_run;
    asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
    const float l_tot = l_run + xsum[(half ^ 1) * BQ + row];
    __nv_bfloat16* Og = reinterpret_cast<__nv_bfloat16*>(p.o) + b * p.so_b + h * p.so_h;
    const bool have = ok && ntiles > 0 && mbar_wait(o_done, (ntiles - 1) & 1, abort_flag, p.err, kErrTimeoutEpilogue);
    if (have) tc_fence_after();
    const float inv = (have && l_tot > 0.f) ? 1.f / l_tot : 0.f;
#pragma unroll
    for (int c = 0; c < D / 64; ++c) {
      uint32_t r[32];
      const int col = half * (D / 2) + 32 * c;
      if (have) {
        tmem_ld_32x32b_x32(tmem_base + t_lane + Lt::TMEM_O + static_cast<uint32_t>(col), r);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) r[e] = 0u;
      }
      if (qi < p.Lq) {
        __nv_bfloat16* dst = Og + (long long)qi * p.so_l + col;
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          const float* f = reinterpret_cast<const float*>(&r[e]);
          *reinterpret_cast<uint4*>(dst + e) =
              make_uint4(pack_bf16x2(f[0] * inv, f[1] * inv), pack_bf16x2(f[2] * inv, f[3] * inv),
                         pack_bf16x2(f[4] * inv, f[5] * inv), pack_bf16x2(f[6] * inv, f[7] * inv));
        }
      }
    }
    if (qi < p.Lq && half == 0)
      p.lse[((long long)b * p.H + h) * p.Lq + qi] =
          (have && l_tot > 0.f) ? (m_run + log2f(l_tot)) * 0.6931471805599453f : -INFINITY;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Lt::TMEM_COLS);
  }
#undef VAGUS_TRF
}

// --------------------------------------------------------------- backward --

constexpr int BKEYS = 64;    // keys per CTA
constexpr int BQ = 64;       // queries per step
constexpr int BWARPS = 8;

// delta = rowsum(dO o O), fp32; dq_acc zeroed
__global__ void attn_bwd_pre(const AttnBwdArgs a) {
  const long long row = (long long)blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const long long rows = (long long)a.f.B * a.f.H * a.f.Lq;
  if (row >= rows) return;
  const int qi = static_cast<int>(row % a.f.Lq);
  const long long bh = row / a.f.Lq;
  const int b = static_cast<int>(bh / a.f.H), h = static_cast<int>(bh % a.f.H);
  const __nv_bfloat16* o = reinterpret_cast<const __nv_bfloat16*>(a.f.o) + b * a.f.so_b + h * a.f.so_h + qi * a.f.so_l;
  const __nv_bfloat16* d = reinterpret_cast<const __nv_bfloat16*>(a.dO) + b * a.f.so_b + h * a.f.so_h + qi * a.f.so_l;
  float s = 0.f;
  for (int c = lane; c < a.f.Dv; c += 32) s += bf2f(o[c]) * bf2f(d[c]);
  s = warp_sum(s);
  if (lane == 0) a.delta[row] = s;
  float* dq = a.dq_acc + row * a.f.D;
  for (int c = lane; c < a.f.D; c += 32) dq[c] = 0.f;
}

// Vectorised pre-pass for head dims 64 / 128: DV / 8 lanes per row (16-byte
// loads of O and dO), rows striding over the grid; dq_acc zeroed with 16-byte
// stores.
template <int DV>
__global__ void __launch_bounds__(256) attn_bwd_pre_v(const AttnBwdArgs a) {
  constexpr int TPR = DV / 8, RPW = 32 / TPR;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int sub = lane % TPR, rw = lane / TPR;
  const long long rows = (long long)a.f.B * a.f.H * a.f.Lq;
  const int D = a.f.D;
  const long long step = (long long)gridDim.x * 8 * RPW;
  for (long long base = ((long long)blockIdx.x * 8 + warp) * RPW; base < rows; base += step) {
    const long long row = base + rw;
    const bool valid = row < rows;
    float s = 0.f;
    if (valid) {
      const int qi = static_cast<int>(row % a.f.Lq);
      const long long bh = row / a.f.Lq;
      const long long b = bh / a.f.H, h = bh % a.f.H;
      const long long off = b * a.f.so_b + h * a.f.so_h + qi * a.f.so_l + 8 * sub;
      const uint4 ou = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.f.o) + off);
      const uint4 du = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.dO) + off);
      const uint32_t ow[4] = {ou.x, ou.y, ou.z, ou.w}, dw[4] = {du.x, du.y, du.z, du.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 of = unpack_bf16x2(ow[j]), df = unpack_bf16x2(dw[j]);
        s += of.x * df.x + of.y * df.y;
      }
    }
#pragma unroll
    for (int o = 1; o < TPR; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (valid) {
      if (sub == 0) a.delta[row] = s;
      float4* dq = reinterpret_cast<float4*>(a.dq_acc + row * D);
      for (int c = sub; c < D / 4; c += TPR) dq[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
}

__global__ void attn_bwd_post(const AttnBwdArgs a);

// The transpose of RoPE's interleaved-pair rotation on 8 adjacent channels
// (4 pairs): (d0, d1) <- (d0 c + d1 s, -d0 s + d1 c) with the pairs' angles at
// table entries [t0, t0 + 4) (16-byte aligned).
__device__ __forceinline__ void unrotate8(float (&d)[8], const float* cosv, const float* sinv, long long t0) {
  const float4 c4 = *reinterpret_cast<const float4*>(cosv + t0);
  const float4 s4 = *reinterpret_cast<const float4*>(sinv + t0);
  const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const float x0 = d[2 * m], x1 = d[2 * m + 1];
    d[2 * m] = x0 * cc[m] + x1 * sn[m];
    d[2 * m + 1] = -x0 * sn[m] + x1 * cc[m];
  }
}

// dq = scale * dq_acc for head dims 64 / 128: D / 8 lanes per row, 8 values per
// lane (two 16-byte loads, one 16-byte store into dq's strides)
template <int D>
__global__ void __launch_bounds__(256) attn_bwd_post_v(const AttnBwdArgs a) {
  constexpr int TPR = D / 8, RPW = 32 / TPR;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int sub = lane % TPR, rw = lane / TPR;
  const long long rows = (long long)a.f.B * a.f.H * a.f.Lq;
  const float sc = a.f.scale;
  const long long step = (long long)gridDim.x * 8 * RPW;
  for (long long base = ((long long)blockIdx.x * 8 + warp) * RPW; base < rows; base += step) {
    const long long row = base + rw;
    if (row >= rows) continue;
    const long long bh = row / a.f.Lq, l = row - bh * a.f.Lq, b = bh / a.f.H, h = bh - b * a.f.H;
    const float4* src = reinterpret_cast<const float4*>(a.dq_acc + row * D + 8 * sub);
    const float4 v0 = src[0], v1 = src[1];
    float d[8] = {sc * v0.x, sc * v0.y, sc * v0.z, sc * v0.w, sc * v1.x, sc * v1.y, sc * v1.z, sc * v1.w};
    if (a.rope_cos) unrotate8(d, a.rope_cos, a.rope_sin, l * (D / 2) + 4 * sub);
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.dq) + b * a.sdq_b + h * a.sdq_h + l * a.sdq_l +
                              8 * sub) =
        make_uint4(pack_bf16x2(d[0], d[1]), pack_bf16x2(d[2], d[3]), pack_bf16x2(d[4], d[5]), pack_bf16x2(d[6], d[7]));
  }
}

void launch_bwd_post(const AttnBwdArgs& a, cudaStream_t st) {
  const long long rows = (long long)a.f.B * a.f.H * a.f.Lq;
  if ((a.f.D == 64 || a.f.D == 128) && (reinterpret_cast<uintptr_t>(a.dq) & 15u) == 0) {
    const int rpw = 32 / (a.f.D / 8);
    const long long want = (rows + 8LL * rpw - 1) / (8LL * rpw);
    const int grid = static_cast<int>(std::min<long long>(std::max<long long>(want, 1), 148LL * 8));
    if (a.f.D == 64) attn_bwd_post_v<64><<<grid, 256, 0, st>>>(a);
    else attn_bwd_post_v<128><<<grid, 256, 0, st>>>(a);
    return;
  }
  const long long n = rows * a.f.D;
  attn_bwd_post<<<static_cast<unsigned>((n / 4 + 255) / 256), 256, 0, st>>>(a);
}

void launch_bwd_pre(const AttnBwdArgs& a, cudaStream_t st) {
  const long long rows = (long long)a.f.B * a.f.H * a.f.Lq;
  const bool vec = (a.f.Dv == 64 || a.f.Dv == 128) && a.f.D % 4 == 0 && a.f.so_l % 8 == 0 && a.f.so_h % 8 == 0 &&
                   a.f.so_b % 8 == 0 && ((reinterpret_cast<uintptr_t>(a.f.o) | reinterpret_cast<uintptr_t>(a.dO)) & 15u) == 0;
  if (vec) {
    const int rpw = 32 / (a.f.Dv / 8);
    const long long want = (rows + 8LL * rpw - 1) / (8LL * rpw);
    const int grid = static_cast<int>(std::min<long long>(std::max<long long>(want, 1), 148LL * 8));
    if (a.f.Dv == 64) attn_bwd_pre_v<64><<<grid, 256, 0, st>>>(a);
    else attn_bwd_pre_v<128><<<grid, 256, 0, st>>>(a);
    return;
  }
  attn_bwd_pre<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, st>>>(a);
}

template <int D, int DV>
struct BwdSmem {
  __nv_bfloat16 K[BKEYS][D + PAD];
  __nv_bfloat16 V[BKEYS][DV + PAD];
  __nv_bfloat16 Q[BQ][D + PAD];
  __nv_bfloat16 dO[BQ][DV + PAD];
  __nv_bfloat16 P[BQ][BKEYS + PAD];
  __nv_bfloat16 dS[BQ][BKEYS + PAD];
  float lse[BQ], delta[BQ];
};

template <int D, int DV>
__global__ void __launch_bounds__(BWARPS * 32, 1)
attn_bwd_kernel(const AttnBwdArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  BwdSmem<D, DV>& sm = *reinterpret_cast<BwdSmem<D, DV>*>(smem_raw);
  const AttnArgs& f = a.f;
  const int kb = blockIdx.x;
  const int bhk = blockIdx.y;
  const int b = bhk / f.Hk, hk = bhk % f.Hk;
  const int group = f.H / f.Hk;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int k0 = kb * BKEYS;
  const int offs = f.Lk - f.Lq;
  const float sl2 = f.scale * kLog2e;

  auto load_rows = [&](__nv_bfloat16* s, int sp, const __nv_bfloat16* g, long long gp, int r0, int nrows, int limit,
                       int cols) {
    const int per_row = cols / 8;
    for (int i = threadIdx.x; i < nrows * per_row; i += blockDim.x) {
      const int r = i / per_row, c = (i - r * per_row) * 8;
      if (r0 + r < limit) cp_async16(s + r * sp + c, g + (long long)(r0 + r) * gp + c);
      else *reinterpret_cast<uint4*>(s + r * sp + c) = make_uint4(0, 0, 0, 0);
    }
  };
  const __nv_bfloat16* Kg = reinterpret_cast<const __nv_bfloat16*>(f.k) + b * f.sk_b + hk * f.sk_h;
  const __nv_bfloat16* Vg = reinterpret_cast<const __nv_bfloat16*>(f.v) + b * f.sv_b + hk * f.sv_h;
  load_rows(&sm.K[0][0], D + PAD, Kg, f.sk_l, k0, BKEYS, f.Lk, D);
  load_rows(&sm.V[0][0], DV + PAD, Vg, f.sv_l, k0, BKEYS, f.Lk, DV);
  cp_commit();

  // warp tiles: S / dP (64 q x 64 k) as 4 x 2 blocks of 16 x 32;
  // dK, dV (64 keys x D) as 4 x 2 blocks of 16 x D/2
  const int sm0 = (warp & 3) * 16, sn0 = (warp >> 2) * 32;
  constexpr int NK = D / 16, NV = DV / 16;            // n-tiles of the D/2 halves
  float dk[1][NK][4], dv[1][NV][4];
  zero(dk);
  zero(dv);
  // first query that can see key k0 (causal): qi + offs >= k0
  const int q_first = f.causal ? max(0, k0 - offs) : 0;
  const int qb0 = q_first / BQ;
  const int nqb = (f.Lq + BQ - 1) / BQ;

  for (int hh = 0; hh < group; ++hh) {
    const int h = hk * group + hh;
    const __nv_bfloat16* Qg = reinterpret_cast<const __nv_bfloat16*>(f.q) + b * f.sq_b + h * f.sq_h;
    const __nv_bfloat16* dOg = reinterpret_cast<const __nv_bfloat16*>(a.dO) + b * f.so_b + h * f.so_h;
    const long long rowbase = ((long long)b * f.H + h) * f.Lq;
    for (int qb = qb0; qb < nqb; ++qb) {
      const int q0 = qb * BQ;
      __syncthreads();                                   // previous step done with Q, dO, P, dS
      load_rows(&sm.Q[0][0], D + PAD, Qg, f.sq_l, q0, BQ, f.Lq, D);
      load_rows(&sm.dO[0][0], DV + PAD, dOg, f.so_l, q0, BQ, f.Lq, DV);
      cp_commit();
      if (threadIdx.x < BQ) {
        const int qi = q0 + threadIdx.x;
        sm.lse[threadIdx.x] = qi < f.Lq ? f.lse[rowbase + qi] : INFINITY;
        sm.delta[threadIdx.x] = qi < f.Lq ? a.delta[rowbase + qi] : 0.f;
      }
      cp_wait_all();
      __syncthreads();
      // S and dP blocks; P = exp(S - lse) (masked), dS = P (dP - delta)
      float s[1][4][4], dp[1][4][4];
      zero(s);
      zero(dp);
      warp_mma<1, 4, false, false>(s, &sm.Q[0][0], D + PAD, &sm.K[0][0], D + PAD, sm0, sn0, D);
      warp_mma<1, 4, false, false>(dp, &sm.dO[0][0], DV + PAD, &sm.V[0][0], DV + PAD, sm0, sn0, DV);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const int r = sm0 + frag_row(0, e), c = sn0 + frag_col(nt, e);
          const int qi = q0 + r;
          float pv[2], dsv[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int kj = k0 + c + u;
            const bool ok = qi < f.Lq && kj < f.Lk && (!f.causal || kj <= qi + offs);
            const float p = ok ? exp2f(s[0][nt][e + u] * sl2 - sm.lse[r] * kLog2e) : 0.f;
            pv[u] = p;
            dsv[u] = p * (dp[0][nt][e + u] - sm.delta[r]);
          }
          *reinterpret_cast<uint32_t*>(&sm.P[r][c]) = pack_bf16x2(pv[0], pv[1]);
          *reinterpret_cast<uint32_t*>(&sm.dS[r][c]) = pack_bf16x2(dsv[0], dsv[1]);
        }
      __syncthreads();
      // dV += P^T dO, dK += dS^T Q   (rows = keys sm0.., columns = half of D)
      warp_mma<1, NV, true, true>(dv, &sm.P[0][0], BKEYS + PAD, &sm.dO[0][0], DV + PAD, sm0, (warp >> 2) * (DV / 2), BQ);
      warp_mma<1, NK, true, true>(dk, &sm.dS[0][0], BKEYS + PAD, &sm.Q[0][0], D + PAD, sm0, (warp >> 2) * (D / 2), BQ);
      // dQ += dS K  (rows = queries sm0.., columns = half of D), fp32 atomics
      {
        float dq[1][NK][4];
        zero(dq);
        warp_mma<1, NK, false, true>(dq, &sm.dS[0][0], BKEYS + PAD, &sm.K[0][0], D + PAD, sm0, (warp >> 2) * (D / 2),
                                     BKEYS);
#pragma unroll
        for (int nt = 0; nt < NK; ++nt)
#pragma unroll
          for (int e = 0; e < 4; e += 2) {
            const int r = sm0 + frag_row(0, e), c = (warp >> 2) * (D / 2) + frag_col(nt, e);
            const int qi = q0 + r;
            if (qi < f.Lq)
              atomicAdd(reinterpret_cast<float2*>(a.dq_acc + (rowbase + qi) * D + c),
                        make_float2(dq[0][nt][e], dq[0][nt][e + 1]));
          }
      }
    }
  }
  cp_wait_all();                                       // K / V copies (no query block ran)
  // dK (scaled), dV out
  __nv_bfloat16* dKg = reinterpret_cast<__nv_bfloat16*>(a.dk) + b * a.sdk_b + hk * a.sdk_h;
  __nv_bfloat16* dVg = reinterpret_cast<__nv_bfloat16*>(a.dv) + b * a.sdv_b + hk * a.sdv_h;
#pragma unroll
  for (int nt = 0; nt < NK; ++nt)
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      const int r = sm0 + frag_row(0, e), c = (warp >> 2) * (D / 2) + frag_col(nt, e);
      if (k0 + r < f.Lk)
        *reinterpret_cast<uint32_t*>(dKg + (long long)(k0 + r) * a.sdk_l + c) =
            pack_bf16x2(f.scale * dk[0][nt][e], f.scale * dk[0][nt][e + 1]);
    }
#pragma unroll
  for (int nt = 0; nt < NV; ++nt)
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      const int r = sm0 + frag_row(0, e), c = (warp >> 2) * (DV / 2) + frag_col(nt, e);
      if (k0 + r < f.Lk)
        *reinterpret_cast<uint32_t*>(dVg + (long long)(k0 + r) * a.sdv_l + c) = pack_bf16x2(dv[0][nt][e], dv[0][nt][e + 1]);
    }
}

// dq = scale * dq_acc (bf16), dq_acc (B * H, Lq, D) contiguous into dq's strides
__global__ void attn_bwd_post(const AttnBwdArgs a) {
  const long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  const int D = a.f.D;
  const long long n = a.f.B * a.f.H * a.f.Lq * D;
  if (i >= n) return;
  const long long row = i / D, bh = row / a.f.Lq;
  const long long d = i - row * D, l = row - bh * a.f.Lq, b = bh / a.f.H, h = bh - b * a.f.H;
  const float4 v = *reinterpret_cast<const float4*>(a.dq_acc + i);
  const float sc = a.f.scale;
  *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(a.dq) + b * a.sdq_b + h * a.sdq_h + l * a.sdq_l + d) =
      make_uint2(pack_bf16x2(sc * v.x, sc * v.y), pack_bf16x2(sc * v.z, sc * v.w));
}

// ----------------------------------------------------- tcgen05 backward --
// One CTA per (128 keys, batch * kv head), walking every (query head of the
// group, query block) step; 10 warps:
//   warp 0      TMA: K and V once, then Q and dO of each step into a
//               two-stage ring (the next block loads during this one);
//   warp 1      TMEM owner and MMA issuer, per step
//                 S^T = K Q^T and dP^T = V dO^T     (M = 128 keys, N = the block's queries)
//                 dV += P^T dO, dK += dS^T Q          (M = 128 keys, N = D)
//                 dQ into its own TMEM columns:
//                   D = 64:  dQ   = dS K     (M = 128 queries, N = 64)
//                   D = 128: dQ^T = K^T dS^T (M = 128 dims,    N = 64 queries)
//               so the next block's S^T / dP^T products run while dQ is
//               read out;
//   warps 2-9   two threads per key row (one per half of the block's query
//               columns): P^T = exp(S^T scale - lse), dS^T = P^T (dP^T - delta)
//               into shared memory as bf16 (the K-major / MN-major operand of
//               the next products), then stage the dQ rows or columns in
//               shared memory for one bulk tensor reduction (TMA add) into
//               the fp32 dq accumulator -- per-thread global atomics here
//               slowed the tensor core's operand reads several-fold; lse /
//               delta of the next block are fetched while dQ is awaited.  At
//               the end the same warps write dK (scaled) and dV.
// Query blocks are 128 rows for D = 64 and 64 rows for D = 128 (so the Q / dO
// ring fits next to K, V, P^T and dS^T in shared memory, and dQ^T has M = 128).
// delta = rowsum(dO o O) comes from the pre-pass and dq is scaled / rounded
// by the post-pass of the mma.sync backward above.  Every wait is bounded.
namespace tcbw {
constexpr int KROWS = 128, THREADS = 448;     // 14 warps: TMA, MMA, 8 softmax, 4 dQ readout
template <int D>
struct Layout {
  static constexpr int QROWS = D == 64 ? 128 : 64;
  static constexpr int KV_BYTES = KROWS * D * 2;      // K, V: D/64 K-major chunks of [128 keys x 128 B]
  static constexpr int Q_BYTES = QROWS * D * 2;       // Q, dO: D/64 chunks of [QROWS x 128 B]
  static constexpr int QCHUNK = QROWS * 128;          // bytes of one 64-wide chunk of a Q / dO tile
  static constexpr int P_BYTES = KROWS * QROWS * 2;   // P^T, dS^T: QROWS/64 chunks of [128 keys x 128 B]
  static constexpr int OFF_V = KV_BYTES, OFF_Q = 2 * KV_BYTES, OFF_DO = OFF_Q + 2 * Q_BYTES;
  static constexpr int OFF_P = OFF_DO + 2 * Q_BYTES, OFF_DS = OFF_P + P_BYTES;
  static constexpr int OFF_DQ = OFF_DS + P_BYTES;     // fp32 dQ staging for the bulk reduction (32 KB)
  static constexpr int OFF_STAT = OFF_DQ + 32768;     // lse[2][QROWS], delta[2][QROWS]
  static constexpr int OFF_BAR = OFF_STAT + 4 * QROWS * 4;
  static constexpr int SMEM = OFF_BAR + 128 + 1024;
  static constexpr uint32_t C_S = 0, C_DP = QROWS, C_DV = 2 * QROWS, C_DK = 2 * QROWS + D, C_DQ = 384,
                            COLS = 512;
  static_assert(C_DK + D <= C_DQ, "TMEM columns");
  // head dim 64: P^T as bf16 pairs in the last 64 columns, the A operand of dV += P^T dO
  // straight from tensor memory (no shared-memory copy); head dim 128 has no room left
  static constexpr bool P_TMEM = D == 64;
  static constexpr uint32_t C_PT = C_DQ + 64;
  static_assert(!P_TMEM || C_PT + QROWS / 2 <= COLS, "TMEM columns for P^T");
};
struct Params {
  int Lq, Lk, H, Hk, causal;
  float sl2, scale;
  const float* lse;
  const float* delta;
  float* dq_acc;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  long long sdk_b, sdk_h, sdk_l, sdv_b, sdv_h, sdv_l;   // element strides of dk / dv
  const float* rope_cos;       // (Lk, D / 2) or null: dK leaves un-rotated at its key positions
  const float* rope_sin;
  int lpt;                     // causal CTA order: 0 key-block-major per head, 1 key block first, g > 1 in groups of g
  int* err;
  unsigned long long* trace;   // phase clock of CTA (0, 0), [step][16]; null: off
};
}  // namespace tcbw

// host side of the phase trace (attn_set_trace)
unsigned long long* g_attn_trace = nullptr;

template <int D>
__global__ void __launch_bounds__(tcbw::THREADS, 1)
attn_bwd_tc(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
            const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mdo,
            const __grid_constant__ CUtensorMap mdq, const tcbw::Params p) {
  using namespace tcbw;
  using Lt = Layout<D>;
  constexpr int QROWS = Lt::QROWS;
  constexpr int HALF = QROWS / 2;                      // query columns per softmax thread
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sk = sm, *sv = sm + Lt::OFF_V, *sq = sm + Lt::OFF_Q, *sdo = sm + Lt::OFF_DO;
  uint8_t *spt = sm + Lt::OFF_P, *sdst = sm + Lt::OFF_DS, *sdq = sm + Lt::OFF_DQ;
  float* s_lse = reinterpret_cast<float*>(sm + Lt::OFF_STAT);   // [2][QROWS]
  float* s_delta = s_lse + 2 * QROWS;                            // [2][QROWS]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Lt::OFF_BAR);
  uint64_t *kv_full = bars, *q_full = bars + 1, *q_empty = bars + 3, *s_full = bars + 5, *p_full = bars + 6,
           *dq_full = bars + 7, *dq_free = bars + 8, *s_free = bars + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  // causal: key blocks near the start see the most query blocks; launch them
  // first (key block 0 of every head of a group, then block 1, ...) so the
  // last wave holds the short CTAs
  int kb = blockIdx.x, bhk = blockIdx.y;
  if (p.causal) {
    const int mode = p.lpt;                            // 0 plain, 1 all heads, g > 1: groups of g heads
    const int nk = gridDim.x, nbh = gridDim.y;
    const int lin = blockIdx.y * nk + blockIdx.x;
    if (mode == 1) {
      kb = lin / nbh;
      bhk = lin % nbh;
    } else if (mode > 1) {
      const int grp = lin / (mode * nk);
      const int gsz = min(mode, nbh - grp * mode);
      const int within = lin - grp * mode * nk;
      kb = within / gsz;
      bhk = grp * mode + within % gsz;
    }
  }
  const int b = bhk / p.Hk, hk = bhk % p.Hk;
  const int group = p.H / p.Hk;
  const int k0 = kb * KROWS;
  const int offs = p.Lk - p.Lq;
  const int q_first = p.causal ? max(0, k0 - offs) : 0;
  const int qb0 = q_first / QROWS, nqb = (p.Lq + QROWS - 1) / QROWS;
  const int per_head = max(0, nqb - qb0);
  const int nsteps = group * per_head;
  const bool tracing = p.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0;
#define VAGUS_TR(step, ev)                                                      \
  do {                                                                          \
    if (tracing && (step) < 32) p.trace[(step) * 16 + (ev)] = clock64();        \
  } while (0)

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 8);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 4);
    mbar_init(s_free, 8);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&mq);
    tma_prefetch_desc(&mk);
    tma_prefetch_desc(&mv);
    tma_prefetch_desc(&mdo);
    tma_prefetch_desc(&mdq);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Lt::COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tb = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && nsteps > 0) {
      mbar_arrive_expect_tx(kv_full, 2 * Lt::KV_BYTES);
      for (int c = 0; c < D / 64; ++c) {
        tma_load_4d(sk + c * 16384, &mk, kv_full, 64 * c, k0, hk, b);
        tma_load_4d(sv + c * 16384, &mv, kv_full, 64 * c, k0, hk, b);
      }
      for (int st = 0; st < nsteps; ++st) {
        const int h = hk * group + st / per_head, q0 = (qb0 + st % per_head) * QROWS;
        const int s = st & 1;
        if (!mbar_wait(&q_empty[s], ((st >> 1) & 1) ^ 1, abort_flag, p.err, kErrTimeoutProducer)) break;
        mbar_arrive_expect_tx(&q_full[s], 2 * Lt::Q_BYTES);
        for (int c = 0; c < D / 64; ++c) {
          tma_load_4d(sq + s * Lt::Q_BYTES + c * Lt::QCHUNK, &mq, &q_full[s], 64 * c, q0, h, b);
          tma_load_4d(sdo + s * Lt::Q_BYTES + c * Lt::QCHUNK, &mdo, &q_full[s], 64 * c, q0, h, b);
        }
      }
      // the ring's last releases land before the CTA retires
      for (int st = nsteps; st < nsteps + 2; ++st)
        if (!mbar_wait(&q_empty[st & 1], ((st >> 1) & 1) ^ 1, abort_flag, p.err, kErrTimeoutProducer)) break;
    }
  } else if (warp == 1) {
    if (lane == 0 && nsteps > 0) {
      constexpr uint32_t id_s = make_idesc_bf16(KROWS, QROWS, false, false);
      constexpr uint32_t id_kv = make_idesc_bf16(KROWS, D, false, true);
      // D = 64: dQ = dS K (A = dS^T tile read MN-major, B = K MN-major);
      // D = 128: dQ^T = K^T dS^T (A = K tile MN-major, B = dS^T tile MN-major)
      constexpr uint32_t id_q = make_idesc_bf16(128, 64, true, true);
      // base descriptors; every product below offsets them by a compile-time byte count
      const uint64_t dk_k = make_sw128_desc(smem_u32(sk), 16, 1024), dv_k = make_sw128_desc(smem_u32(sv), 16, 1024);
      const uint64_t dp_k = make_sw128_desc(smem_u32(spt), 16, 1024), ds_k = make_sw128_desc(smem_u32(sdst), 16, 1024);
      const uint64_t ds_mn = make_sw128_desc(smem_u32(sdst), 16384, 1024);
      const uint64_t dk_mn = make_sw128_desc(smem_u32(sk), 16384, 1024);
      // S^T and dP^T of step st into their TMEM columns
      auto issue_sdp = [&](int st) {
        const int s = st & 1;
        const uint64_t dq_k = make_sw128_desc(smem_u32(sq + s * Lt::Q_BYTES), 16, 1024);
        const uint64_t ddo_k = make_sw128_desc(smem_u32(sdo + s * Lt::Q_BYTES), 16, 1024);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc_mma_f16(tb + Lt::C_S, desc_add(dk_k, c * 16384 + kk * 32), desc_add(dq_k, c * Lt::QCHUNK + kk * 32), id_s,
                       (c | kk) ? 1u : 0u);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc_mma_f16(tb + Lt::C_DP, desc_add(dv_k, c * 16384 + kk * 32), desc_add(ddo_k, c * Lt::QCHUNK + kk * 32),
                       id_s, (c | kk) ? 1u : 0u);
        tc_commit(s_full);
      };
      // Schedule: S^T / dP^T of step st + 1 go in as soon as the softmax warps
      // have read step st's scores (s_free), so they run while those warps
      // compute P and dS; then step st's dV, dK and dQ.
      bool ok = mbar_wait(kv_full, 0, abort_flag, p.err, kErrTimeoutMma) &&
                mbar_wait(&q_full[0], 0, abort_flag, p.err, kErrTimeoutMma);
      if (ok) {
        tc_fence_after();
        issue_sdp(0);
      }
      for (int st = 0; ok && st < nsteps; ++st) {
        const int s = st & 1;
        VAGUS_TR(st, 0);
        if (st + 1 < nsteps) {
          if (!mbar_wait(&q_full[s ^ 1], ((st + 1) >> 1) & 1, abort_flag, p.err, kErrTimeoutMma)) break;
          if (!mbar_wait(s_free, st & 1, abort_flag, p.err, kErrTimeoutMma)) break;
          tc_fence_after();
          issue_sdp(st + 1);
        }
        VAGUS_TR(st, 1);
        const uint64_t dq_mn = make_sw128_desc(smem_u32(sq + s * Lt::Q_BYTES), Lt::QCHUNK, 1024);
        const uint64_t ddo_mn = make_sw128_desc(smem_u32(sdo + s * Lt::Q_BYTES), Lt::QCHUNK, 1024);
        if (!mbar_wait(p_full, st & 1, abort_flag, p.err, kErrTimeoutMma)) break;
        VAGUS_TR(st, 2);
        tc_fence_after();
        // dV += P^T dO, dK += dS^T Q: K = the block's queries (16 per step)
#pragma unroll
        for (int j = 0; j < QROWS / 16; ++j) {
          const uint32_t acc = (st > 0 || j > 0) ? 1u : 0u;
          const uint32_t a_off = static_cast<uint32_t>((j >> 2) * 16384 + (j & 3) * 32);
          if constexpr (Lt::P_TMEM)
            tc_mma_f16_ts(tb + Lt::C_DV, tb + Lt::C_PT + static_cast<uint32_t>(8 * j), desc_add(ddo_mn, j * 2048),
                          id_kv, acc);
          else
            tc_mma_f16(tb + Lt::C_DV, desc_add(dp_k, a_off), desc_add(ddo_mn, j * 2048), id_kv, acc);
          tc_mma_f16(tb + Lt::C_DK, desc_add(ds_k, a_off), desc_add(dq_mn, j * 2048), id_kv, acc);
        }
        VAGUS_TR(st, 3);
        if (st > 0 && !mbar_wait(dq_free, (st - 1) & 1, abort_flag, p.err, kErrTimeoutMma)) break;
        VAGUS_TR(st, 4);
        tc_fence_after();
        // dQ: K = the 128 keys (8 steps of 16 rows)
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          if constexpr (D == 64)
            tc_mma_f16(tb + Lt::C_DQ, desc_add(ds_mn, kk * 2048), desc_add(dk_mn, kk * 2048), id_q, kk ? 1u : 0u);
          else
            tc_mma_f16(tb + Lt::C_DQ, desc_add(dk_mn, kk * 2048), desc_add(ds_mn, kk * 2048), id_q, kk ? 1u : 0u);
        }
        tc_commit(dq_full);                              // also: P^T / dS^T of step st consumed
        tc_commit(&q_empty[s]);
        VAGUS_TR(st, 5);
      }
    }
  } else if (warp >= 10) {
    // ------------------------------------------------------ dQ readout
    // dQ of each step (complete in TMEM) -> fp32 staging tile -> one bulk
    // reduction into dq_acc (the tensor map clips rows past Lq); off the
    // softmax warps' path, so their next step overlaps it.  Warp w reads TMEM
    // lanes 32 (w & 3) ..; each thread one row (query for D = 64, dim for 128).
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int tq = threadIdx.x - 320;                    // 0..127
    const uint32_t tl = tb + (static_cast<uint32_t>(quarter * 32) << 16);
    bool ok = true;
    for (int st = 0; st < nsteps; ++st) {
      const int h = hk * group + st / per_head, q0 = (qb0 + st % per_head) * QROWS;
      ok = ok && mbar_wait(dq_full, st & 1, abort_flag, p.err, kErrTimeoutEpilogue);
      tc_fence_after();
      uint32_t r[64];
      tmem_ld_32x32b_x32(tl + Lt::C_DQ, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
      tmem_ld_32x32b_x32(tl + Lt::C_DQ + 32u, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_free);
      if (tq == 0) bulk_wait_read<0>();                 // the previous reduction has read the tile
      asm volatile("bar.sync 2, 128;" ::: "memory");
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        if constexpr (D == 64) {
          // dims 32 hf ..: 128-byte swizzled [128 rows][32 fp32] tile per half
          uint8_t* base = sdq + hf * 16384 + row * 128;
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<uint4*>(base + ((u ^ (row & 7)) * 16)) =
                make_uint4(r[32 * hf + 4 * u], r[32 * hf + 4 * u + 1], r[32 * hf + 4 * u + 2], r[32 * hf + 4 * u + 3]);
        } else {
          // dQ^T row = dim `row`, columns = queries 32 hf ..: plain [64 queries][128 dims] tile
          float* base = reinterpret_cast<float*>(sdq) + (32 * hf) * 128 + row;
#pragma unroll
          for (int e = 0; e < 32; ++e) base[e * 128] = __uint_as_float(r[32 * hf + e]);
        }
      }
      fence_proxy_async_smem();
      asm volatile("bar.sync 2, 128;" ::: "memory");
      if (tq == 0 && ok) {
        const int bh = b * p.H + h;
        tma_reduce_add_3d(&mdq, sdq, 0, q0, bh);
        if constexpr (D == 64) tma_reduce_add_3d(&mdq, sdq + 16384, 32, q0, bh);
        bulk_commit();
      }
    }
    if (tq == 0) bulk_wait<0>();                         // reductions performed before the CTA retires
  } else {
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;                 // key row (S^T, dK, dV); query row / dim for dQ
    const uint32_t tl = tb + (static_cast<uint32_t>(quarter * 32) << 16);
    const int t = threadIdx.x - 64;                      // 0..255 over the softmax warps
    const int kj = k0 + row;
    bool ok = true;
    // lse (log2 units) / delta of step st's query block, fetched by threads t < 2 QROWS
    auto fetch_stat = [&](int st) -> float {
      if (st >= nsteps || t >= 2 * QROWS) return 0.f;
      const int h = hk * group + st / per_head, q0 = (qb0 + st % per_head) * QROWS;
      const long long rowbase = ((long long)b * p.H + h) * p.Lq;
      const int qi = q0 + (t < QROWS ? t : t - QROWS);
      if (t < QROWS) return qi < p.Lq ? p.lse[rowbase + qi] * kLog2e : INFINITY;
      return qi < p.Lq ? p.delta[rowbase + qi] : 0.f;
    };
    auto put_stat = [&](int st, float v) {
      if (t < QROWS) s_lse[(st & 1) * QROWS + t] = v;
      else if (t < 2 * QROWS) s_delta[(st & 1) * QROWS + t - QROWS] = v;
    };
    put_stat(0, fetch_stat(0));
    // kernel parameters in registers: the lambdas above take `p` by reference,
    // and reads through that reference inside the hot loop are memory loads
    const float sl2 = p.sl2;
    const int Lk = p.Lk, Lq = p.Lq;
    const bool causal = p.causal != 0;
    for (int st = 0; st < nsteps; ++st) {
      const int q0 = (qb0 + st % per_head) * QROWS;
      const float* lse_s = s_lse + (st & 1) * QROWS + HALF * half;
      const float* del_s = s_delta + (st & 1) * QROWS + HALF * half;
      asm volatile("bar.sync 1, 256;" ::: "memory");     // this step's statistics are in place
      const float nxt = fetch_stat(st + 1);              // the next step's, in flight during this one
      ok = ok && mbar_wait(s_full, st & 1, abort_flag, p.err, kErrTimeoutEpilogue);
      if (t == 0) VAGUS_TR(st, 6);
      tc_fence_after();
      const uint32_t cs = tl + Lt::C_S + static_cast<uint32_t>(HALF * half);
      const uint32_t cd = tl + Lt::C_DP + static_cast<uint32_t>(HALF * half);
      const int qbase = q0 + HALF * half;
      const bool full = (k0 + KROWS <= Lk) && (q0 + QROWS <= Lq) && (!causal || k0 + KROWS - 1 <= q0 + offs);
      // 32 query columns at a time: scores and dP from TMEM (the MMA warp may
      // refill them once the last chunk is read), P^T and dS^T as bf16 into
      // the 128-byte swizzled tiles once the previous step's products are done
#pragma unroll
      for (int c = 0; c < HALF / 32; ++c) {
        float sv[32], dp[32];
        tmem_ld_32x32b_x32(cs + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
        tmem_ld_32x32b_x32(cd + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&dp[0]));
        tmem_ld_wait();
        if (c == HALF / 32 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(s_free);
        }
        if (t == 0 && c == 0) VAGUS_TR(st, 7);
        // lse / delta 4 at a time (shared-memory broadcasts): no 32-wide register copies
        if (full) {
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            const float4 a4 = *reinterpret_cast<const float4*>(lse_s + 32 * c + i);
            const float4 d4 = *reinterpret_cast<const float4*>(del_s + 32 * c + i);
            const float la[4] = {a4.x, a4.y, a4.z, a4.w}, da[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float pr = ex2_approx(fmaf(sv[i + u], sl2, -la[u]));
              sv[i + u] = pr;
              dp[i + u] = pr * (dp[i + u] - da[u]);
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            const float4 a4 = *reinterpret_cast<const float4*>(lse_s + 32 * c + i);
            const float4 d4 = *reinterpret_cast<const float4*>(del_s + 32 * c + i);
            const float la[4] = {a4.x, a4.y, a4.z, a4.w}, da[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int qi = qbase + 32 * c + i + u;
              const bool vis = kj < Lk && qi < Lq && (!causal || kj <= qi + offs);
              const float pr = vis ? ex2_approx(fmaf(sv[i + u], sl2, -la[u])) : 0.f;
              sv[i + u] = pr;
              dp[i + u] = pr * (dp[i + u] - da[u]);
            }
          }
        }
        if (t == 0) VAGUS_TR(st, c == 0 ? 13 : 15);
        if (c == 0 && st > 0) {
          ok = ok && mbar_wait(dq_full, (st - 1) & 1, abort_flag, p.err, kErrTimeoutEpilogue);
          tc_fence_after();                              // P^T in TMEM is rewritten after step st - 1's products
        }
        if constexpr (Lt::P_TMEM) {
          uint32_t pk[16];
#pragma unroll
          for (int u = 0; u < 16; ++u) pk[u] = pack_bf16x2(sv[2 * u], sv[2 * u + 1]);
          tmem_st_32x32b_x16(tl + Lt::C_PT + static_cast<uint32_t>((HALF * half + 32 * c) / 2), pk);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int col = HALF * half + 32 * c + 8 * u;  // query column inside the block
          const uint32_t off =
              static_cast<uint32_t>((col >> 6) * 16384 + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) * 16));
          const float* a8 = &sv[8 * u];
          const float* d8 = &dp[8 * u];
          if constexpr (!Lt::P_TMEM)
            *reinterpret_cast<uint4*>(spt + off) = make_uint4(pack_bf16x2(a8[0], a8[1]), pack_bf16x2(a8[2], a8[3]),
                                                              pack_bf16x2(a8[4], a8[5]), pack_bf16x2(a8[6], a8[7]));
          *reinterpret_cast<uint4*>(sdst + off) = make_uint4(pack_bf16x2(d8[0], d8[1]), pack_bf16x2(d8[2], d8[3]),
                                                             pack_bf16x2(d8[4], d8[5]), pack_bf16x2(d8[6], d8[7]));
        }
        if (t == 0 && c == 0) VAGUS_TR(st, 14);
      }
      if (t == 0) VAGUS_TR(st, 12);
      if constexpr (Lt::P_TMEM) tmem_st_wait();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (t == 0) VAGUS_TR(st, 8);
      if (lane == 0) mbar_arrive(p_full);
      put_stat(st + 1, nxt);
      if (t == 0) VAGUS_TR(st, 11);
    }
    // the last step's products (dV, dK, dQ) are complete once dq_full fires
    if (nsteps > 0) ok = ok && mbar_wait(dq_full, (nsteps - 1) & 1, abort_flag, p.err, kErrTimeoutEpilogue);
    // dK (scaled) and dV rows of this CTA's keys
    const bool have = ok && nsteps > 0;
    if (have) tc_fence_after();
#pragma unroll
    for (int which = 0; which < 2; ++which) {
      __nv_bfloat16* out = which == 0 ? p.dk + b * p.sdk_b + hk * p.sdk_h : p.dv + b * p.sdv_b + hk * p.sdv_h;
      const long long s_l = which == 0 ? p.sdk_l : p.sdv_l;
      const uint32_t base = which == 0 ? Lt::C_DK : Lt::C_DV;
      const float sc = which == 0 ? p.scale : 1.f;
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        uint32_t r[32];
        const int col = half * (D / 2) + 32 * c;
        if (have) {
          tmem_ld_32x32b_x32(tl + base + static_cast<uint32_t>(col), r);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) r[e] = 0u;
        }
        if (kj < p.Lk) {
          __nv_bfloat16* dst = out + (long long)kj * s_l + col;
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            const float* f = reinterpret_cast<const float*>(&r[e]);
            float d[8];
#pragma unroll
            for (int m = 0; m < 8; ++m) d[m] = sc * f[m];
            if (which == 0 && p.rope_cos) unrotate8(d, p.rope_cos, p.rope_sin, (long long)kj * (D / 2) + (col + e) / 2);
            *reinterpret_cast<uint4*>(dst + e) = make_uint4(pack_bf16x2(d[0], d[1]), pack_bf16x2(d[2], d[3]),
                                                            pack_bf16x2(d[4], d[5]), pack_bf16x2(d[6], d[7]));
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tb, Lt::COLS);
  }
#undef VAGUS_TR
}

template <typename Kern>
bool set_smem(Kern kern, size_t bytes) {
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)) ==
         cudaSuccess;
}

template <int D>
int launch_fwd_tc(const AttnArgs& a, cudaStream_t st) {
  using Lt = tcfa::Layout<D>;
  alignas(64) unsigned char mq[128], mk[128], mv[128];
  const unsigned long long dq[4] = {(unsigned long long)D, (unsigned long long)a.Lq, (unsigned long long)a.H,
                                    (unsigned long long)a.B};
  const unsigned long long sq[3] = {(unsigned long long)a.sq_l * 2, (unsigned long long)a.sq_h * 2,
                                    (unsigned long long)a.sq_b * 2};
  const unsigned long long dk[4] = {(unsigned long long)D, (unsigned long long)a.Lk, (unsigned long long)a.Hk,
                                    (unsigned long long)a.B};
  const unsigned long long sk[3] = {(unsigned long long)a.sk_l * 2, (unsigned long long)a.sk_h * 2,
                                    (unsigned long long)a.sk_b * 2};
  const unsigned long long dv[4] = {(unsigned long long)D, (unsigned long long)a.Lk, (unsigned long long)a.Hk,
                                    (unsigned long long)a.B};
  const unsigned long long sv[3] = {(unsigned long long)a.sv_l * 2, (unsigned long long)a.sv_h * 2,
                                    (unsigned long long)a.sv_b * 2};
  const unsigned box_qk[4] = {64u, 128u, 1u, 1u}, box_v[4] = {64u, 64u, 1u, 1u};
  if (!encode_bf16_map(mq, a.q, 4, dq, sq, box_qk) || !encode_bf16_map(mk, a.k, 4, dk, sk, box_qk) ||
      !encode_bf16_map(mv, a.v, 4, dv, sv, box_v))
    return 2;
  tcfa::Params p;
  p.Lq = a.Lq; p.Lk = a.Lk; p.H = a.H; p.Hk = a.Hk; p.causal = a.causal;
  // causal order, measured at B = 4, 16 heads, L = 4096 (plain order: 310 / 425 us): groups of 8 heads
  // at head dim 64 (282 us), of 4 at 128 (403 us)
  p.lpt = D == 64 ? 8 : 4;
  p.sl2 = a.scale * kLog2e;
  p.o = a.o; p.so_b = a.so_b; p.so_h = a.so_h; p.so_l = a.so_l;
  p.lse = a.lse;
  p.err = a.err;
  p.trace = g_attn_trace;
  static bool attr_set[64] = {};
  auto kern = attn_fwd_tc<D, 2>;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lt::SMEM) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
      return 3;
    attr_set[dev] = true;
  }
  dim3 grid(static_cast<unsigned>((a.Lq + tcfa::BQ - 1) / tcfa::BQ), static_cast<unsigned>(a.B * a.H));
  kern<<<grid, tcfa::THREADS, Lt::SMEM, st>>>(*reinterpret_cast<const CUtensorMap*>(mq),
                                               *reinterpret_cast<const CUtensorMap*>(mk),
                                               *reinterpret_cast<const CUtensorMap*>(mv), p);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

template <int D, int DV>
int launch_fwd(const AttnArgs& a, cudaStream_t st) {
  const size_t sm = sizeof(FwdSmem<D, DV>);
  if (!set_smem(attn_fwd_kernel<D, DV>, sm)) return 3;
  dim3 grid(static_cast<unsigned>((a.Lq + FQ - 1) / FQ), static_cast<unsigned>(a.B * a.H));
  attn_fwd_kernel<D, DV><<<grid, FWARPS * 32, sm, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

template <int D>
int launch_bwd_tc(const AttnBwdArgs& a, cudaStream_t st) {
  using Lt = tcbw::Layout<D>;
  const AttnArgs& f = a.f;
  alignas(64) unsigned char mq[128], mk[128], mv[128], mdo[128];
  const unsigned long long dq[4] = {(unsigned long long)D, (unsigned long long)f.Lq, (unsigned long long)f.H,
                                    (unsigned long long)f.B};
  const unsigned long long dk[4] = {(unsigned long long)D, (unsigned long long)f.Lk, (unsigned long long)f.Hk,
                                    (unsigned long long)f.B};
  const unsigned long long sq[3] = {(unsigned long long)f.sq_l * 2, (unsigned long long)f.sq_h * 2,
                                    (unsigned long long)f.sq_b * 2};
  const unsigned long long sk[3] = {(unsigned long long)f.sk_l * 2, (unsigned long long)f.sk_h * 2,
                                    (unsigned long long)f.sk_b * 2};
  const unsigned long long sv[3] = {(unsigned long long)f.sv_l * 2, (unsigned long long)f.sv_h * 2,
                                    (unsigned long long)f.sv_b * 2};
  const unsigned long long so[3] = {(unsigned long long)f.so_l * 2, (unsigned long long)f.so_h * 2,
                                    (unsigned long long)f.so_b * 2};
  const unsigned box[4] = {64u, 128u, 1u, 1u}, box_q[4] = {64u, static_cast<unsigned>(Lt::QROWS), 1u, 1u};
  if (!encode_bf16_map(mq, f.q, 4, dq, sq, box_q) || !encode_bf16_map(mk, f.k, 4, dk, sk, box) ||
      !encode_bf16_map(mv, f.v, 4, dk, sv, box) || !encode_bf16_map(mdo, a.dO, 4, dq, so, box_q))
    return 2;
  // dq_acc (B * H, Lq, D) fp32: D = 64 reduces [128 queries][32 dims] boxes (128-byte
  // swizzle), D = 128 one [64 queries][128 dims] box
  alignas(64) unsigned char mdq[128];
  const unsigned long long ddq[3] = {(unsigned long long)D, (unsigned long long)f.Lq, (unsigned long long)f.B * f.H};
  const unsigned long long sdq[2] = {(unsigned long long)D * 4, (unsigned long long)f.Lq * D * 4};
  const unsigned box_dq[3] = {D == 64 ? 32u : 128u, static_cast<unsigned>(Lt::QROWS), 1u};
  if (!encode_f32_map(mdq, a.dq_acc, 3, ddq, sdq, box_dq, D == 64)) return 2;
  tcbw::Params p;
  p.Lq = f.Lq; p.Lk = f.Lk; p.H = f.H; p.Hk = f.Hk; p.causal = f.causal;
  p.sl2 = f.scale * kLog2e; p.scale = f.scale;
  p.lse = f.lse; p.delta = a.delta; p.dq_acc = a.dq_acc;
  p.dk = (__nv_bfloat16*)a.dk; p.dv = (__nv_bfloat16*)a.dv; p.err = f.err;
  p.sdk_b = a.sdk_b; p.sdk_h = a.sdk_h; p.sdk_l = a.sdk_l;
  p.sdv_b = a.sdv_b; p.sdv_h = a.sdv_h; p.sdv_l = a.sdv_l;
  p.rope_cos = a.rope_cos; p.rope_sin = a.rope_sin;
  // causal order, measured at B = 4, 16 heads, L = 4096: head dim 64 key block first across all heads
  // (905 -> 814 us), head dim 128 in groups of 4 heads (1386 -> 1317 us; all heads at once lost
  // the heads' shared Q / dO reads in L2: 1433 us)
  p.lpt = D == 64 ? 1 : 4;
  p.trace = g_attn_trace;
  static bool attr_set[64] = {};
  auto kern = attn_bwd_tc<D>;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lt::SMEM) != cudaSuccess)
      return 3;
    attr_set[dev] = true;
  }
  const long long rows = (long long)f.B * f.H * f.Lq;
  launch_bwd_pre(a, st);
  dim3 grid(static_cast<unsigned>((f.Lk + tcbw::KROWS - 1) / tcbw::KROWS), static_cast<unsigned>(f.B * f.Hk));
  kern<<<grid, tcbw::THREADS, Lt::SMEM, st>>>(*reinterpret_cast<const CUtensorMap*>(mq),
                                               *reinterpret_cast<const CUtensorMap*>(mk),
                                               *reinterpret_cast<const CUtensorMap*>(mv),
                                               *reinterpret_cast<const CUtensorMap*>(mdo),
                                               *reinterpret_cast<const CUtensorMap*>(mdq), p);
  launch_bwd_post(a, st);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

template <int D, int DV>
int launch_bwd(const AttnBwdArgs& a, cudaStream_t st) {
  const long long rows = (long long)a.f.B * a.f.H * a.f.Lq;
  launch_bwd_pre(a, st);
  const size_t sm = sizeof(BwdSmem<D, DV>);
  if (!set_smem(attn_bwd_kernel<D, DV>, sm)) return 3;
  dim3 grid(static_cast<unsigned>((a.f.Lk + BKEYS - 1) / BKEYS), static_cast<unsigned>(a.f.B * a.f.Hk));
  attn_bwd_kernel<D, DV><<<grid, BWARPS * 32, sm, st>>>(a);
  launch_bwd_post(a, st);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool strides_ok(const AttnArgs& a) {
  // 16-byte rows for cp.async; heads must split evenly for GQA
  const long long s[] = {a.sq_b, a.sq_h, a.sq_l, a.sk_b, a.sk_h, a.sk_l, a.sv_b, a.sv_h, a.sv_l, a.so_b, a.so_h, a.so_l};
  for (long long v : s)
    if (v % 8) return false;
  return aligned16(a.q) && aligned16(a.k) && aligned16(a.v) && aligned16(a.o) && a.Hk > 0 && a.H % a.Hk == 0;
}

}  // namespace

int attn_fwd(const AttnArgs& a, cudaStream_t st) {
  if (!strides_ok(a) || a.Lq <= 0 || a.Lk <= 0) return 5;
  // tensor-core path: every TMA box (128 rows) fits inside its tensor
  static const bool no_tc = std::getenv("VAGUS_ATTN_NO_TC") != nullptr;
  if (!no_tc && a.err && a.Lq >= 128 && a.Lk >= 128 && a.D == a.Dv && (a.D == 64 || a.D == 128))
    return a.D == 64 ? launch_fwd_tc<64>(a, st) : launch_fwd_tc<128>(a, st);
  if (a.D == 64 && a.Dv == 64) return launch_fwd<64, 64>(a, st);
  if (a.D == 128 && a.Dv == 128) return launch_fwd<128, 128>(a, st);
  if (a.D == 64 && a.Dv == 128) return launch_fwd<64, 128>(a, st);
  return 5;
}

void attn_set_trace(unsigned long long* buf) { g_attn_trace = buf; }

int attn_bwd(const AttnBwdArgs& a, cudaStream_t st) {
  if (!strides_ok(a.f) || !aligned16(a.dO) || a.f.Lq <= 0 || a.f.Lk <= 0) return 5;
  // gradient outputs: 16-byte aligned rows (8-element strides) for the vector stores
  const long long gs[] = {a.sdq_b, a.sdq_h, a.sdq_l, a.sdk_b, a.sdk_h, a.sdk_l, a.sdv_b, a.sdv_h, a.sdv_l};
  for (long long x : gs)
    if (x % 8) return 5;
  if (!aligned16(a.dq) || !aligned16(a.dk) || !aligned16(a.dv)) return 5;
  static const bool no_tc = std::getenv("VAGUS_ATTN_NO_TC") != nullptr;
  const bool tc = !no_tc && a.f.err && a.f.Lq >= 128 && a.f.Lk >= 128 && a.f.D == a.f.Dv &&
                  (a.f.D == 64 || a.f.D == 128);
  // un-rotating dq / dk is a step of the tcgen05 path's dQ pass and dK epilogue only
  if (a.rope_cos && (!tc || !a.rope_sin || a.f.Lq != a.f.Lk || !aligned16(a.rope_cos) || !aligned16(a.rope_sin)))
    return 5;
  if (tc) return a.f.D == 64 ? launch_bwd_tc<64>(a, st) : launch_bwd_tc<128>(a, st);
  if (a.f.D == 64 && a.f.Dv == 64) return launch_bwd<64, 64>(a, st);
  if (a.f.D == 128 && a.f.Dv == 128) return launch_bwd<128, 128>(a, st);
  if (a.f.D == 64 && a.f.Dv == 128) return launch_bwd<64, 128>(a, st);
  return 5;
}

}  // namespace vagus
