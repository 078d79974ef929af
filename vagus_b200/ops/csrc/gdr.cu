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
//   gC, dgC: (BH, N) fp32, or (BH, N, DK) for a per-channel (KDA) gate, where
//   gC S scales row k of S by gC[k] and dgC[k] = <S_n row k, dS row k>
//   states, dstates: (BH, N, DV, DK) bf16 (S_n^T, dL/dS_{n+1}^T: value-major)
//   dW, dQh, dKt: (BH, N, C, DK) bf16   dA: (BH, N, C, C) fp32
#include "common.cuh"
#include "gemm.h"
#include "kernels.h"
#include "mma.cuh"

#include <cstdlib>

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

// smem tile [rows][cols] (pitch sp) -> global transposed g[c * gp + r]; rows % 8 == 0
__device__ __forceinline__ void store_tile_t(__nv_bfloat16* g, long long gp, const __nv_bfloat16* s, int sp, int rows,
                                             int cols) {
  for (int i = threadIdx.x; i < cols * (rows / 8); i += blockDim.x) {
    const int c = i % cols, r = (i / cols) * 8;
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      w[j] = static_cast<uint32_t>(__bfloat16_as_ushort(s[(r + 2 * j) * sp + c])) |
             (static_cast<uint32_t>(__bfloat16_as_ushort(s[(r + 2 * j + 1) * sp + c])) << 16);
    *reinterpret_cast<uint4*>(g + c * gp + r) = make_uint4(w[0], w[1], w[2], w[3]);
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
             int DV, int gvec) {
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
    if (states) store_tile_t(states + (cidx * DV + v0) * DK, DK, &sm.S[0][0], DVT + PAD, DK, DVT);

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
    store_tile_t(Vp + (cidx * DV + v0) * C, C, &sm.V[0][0], DVT + PAD, C, DVT);

    // S <- gC S + Kt^T V'  (row k scaled by gC[k] for a per-channel gate)
    const float g = gvec ? 0.f : gC[cidx];
#pragma unroll
    for (int mt = 0; mt < SMT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          S[mt][nt][e] *= gvec ? gC[cidx * DK + srow0 + frag_row(mt, e)] : g;
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

// ------------------------------------------------------ tcgen05 forward scan --
// The same chain on the 5th-generation tensor cores, transposed so the value
// tile is the MMA's M = 128: one CTA per (sequence, 128-wide value tile),
// S^T (value x key, fp32) lives in TMEM, and per chunk
//   D1   = S^T W^T                  (M = 128 values, N = 64 tokens, K = DK)
//   V'^T = U^T - D1                  (state warps: TMEM -> registers -> bf16 smem)
//   S^T += V'^T Kt                   (M = 128, N = DK, K = 64 tokens)
// with S^T copied to bf16 shared memory (the A operand of the next D1) and
// scaled by gC in TMEM by the state warps between the chunks.  Warp 0
// streams W and Kt with TMA into a two-stage ring; warp 1 issues the MMAs and
// the TMA stores of the bf16 S^T (the chunk-entry snapshot) and of V'^T
// straight from the operand tiles, so the snapshots cost the state warps
// nothing; warps 2-9 (two per TMEM lane quarter, one value row and half of
// the columns per thread) do the rest.  Every wait is bounded.
namespace tscan {
constexpr int VT = 128;                  // value tile (MMA M)
template <int DK>
struct Layout {
  static constexpr int W_BYTES = C * DK * 2;     // DK/64 chunks of [64 tokens x 128 B]
  static constexpr int ST_BYTES = VT * DK * 2;   // DK/64 chunks of [128 values x 128 B]
  static constexpr int VTB_BYTES = VT * C * 2;   // [128 values x 64 tokens]
  static constexpr int U_BYTES = C * VT * 2;     // plain row-major [64 tokens][128 values]
  static constexpr int OFF_K = 2 * W_BYTES;
  static constexpr int OFF_ST = 4 * W_BYTES;
  static constexpr int OFF_VT = OFF_ST + ST_BYTES;
  static constexpr int OFF_U = OFF_VT + VTB_BYTES;
  static constexpr int OFF_BAR = OFF_U + U_BYTES;
  static constexpr int SMEM = OFF_BAR + 128 + 1024;
  static constexpr uint32_t C_S = 0, C_D1 = DK, COLS = 512;
};
}  // namespace tscan

template <int DK>
__global__ void __launch_bounds__(320, 1)
gdr_fwd_scan_tc(const __grid_constant__ CUtensorMap mw, const __grid_constant__ CUtensorMap mk,
                const __grid_constant__ CUtensorMap ms, const __grid_constant__ CUtensorMap mv,
                const __nv_bfloat16* __restrict__ U, const float* __restrict__ gC, const float* __restrict__ S0,
                float* __restrict__ S_out, int N, int DV, int gvec, int* err) {
  using namespace tscan;
  using Lt = Layout<DK>;
  extern __shared__ __align__(128) uint8_t smem_raw[];   // re-aligned to 1024 (the swizzle atom) below
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sw = sm, *skt = sm + Lt::OFF_K, *sst = sm + Lt::OFF_ST, *svt = sm + Lt::OFF_VT;
  __nv_bfloat16* su = reinterpret_cast<__nv_bfloat16*>(sm + Lt::OFF_U);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Lt::OFF_BAR);
  uint64_t *w_full = bars, *w_empty = bars + 2, *s_ready = bars + 4, *d1_full = bars + 5, *v_full = bars + 6,
           *s2_done = bars + 7;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int tiles_v = DV / VT;
  const long long bh = blockIdx.x / tiles_v;
  const int v0 = (blockIdx.x % tiles_v) * VT;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&w_full[i], 1);
      mbar_init(&w_empty[i], 1);
    }
    mbar_init(s_ready, 8);
    mbar_init(d1_full, 1);
    mbar_init(v_full, 8);
    mbar_init(s2_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&mw);
    tma_prefetch_desc(&mk);
    tma_prefetch_desc(&ms);
    tma_prefetch_desc(&mv);
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
    if (lane == 0) {
      for (int n = 0; n < N; ++n) {
        const int s = n & 1;
        if (!mbar_wait(&w_empty[s], ((n >> 1) & 1) ^ 1, abort_flag, err, kErrTimeoutProducer)) break;
        mbar_arrive_expect_tx(&w_full[s], 2 * Lt::W_BYTES);
        const int row = static_cast<int>((bh * N + n) * C);
        for (int c = 0; c < DK / 64; ++c) {
          tma_load_2d(sw + s * Lt::W_BYTES + c * 8192, &mw, &w_full[s], 64 * c, row);
          tma_load_2d(skt + s * Lt::W_BYTES + c * 8192, &mk, &w_full[s], 64 * c, row);
        }
      }
      // the last two stages' releases land before the CTA retires
      for (int n = N; n < N + 2; ++n)
        if (!mbar_wait(&w_empty[n & 1], ((n >> 1) & 1) ^ 1, abort_flag, err, kErrTimeoutProducer)) break;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id1 = make_idesc_bf16(VT, C, false, false);
      constexpr uint32_t id2 = make_idesc_bf16(VT, DK, false, true);
      const uint32_t ast = smem_u32(sst), avt = smem_u32(svt);
      for (int n = 0; n < N; ++n) {
        const int s = n & 1;
        const int srow = static_cast<int>((bh * N + n) * DV + v0);   // row of this tile in the value-major outputs
        if (!mbar_wait(&w_full[s], (n >> 1) & 1, abort_flag, err, kErrTimeoutMma)) break;
        if (!mbar_wait(s_ready, n & 1, abort_flag, err, kErrTimeoutMma)) break;
        tc_fence_after();
        const uint32_t aw = smem_u32(sw + s * Lt::W_BYTES), ak = smem_u32(skt + s * Lt::W_BYTES);
#pragma unroll
        for (int c = 0; c < DK / 64; ++c)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc_mma_f16(tb + Lt::C_D1, make_sw128_desc(ast + c * 16384 + kk * 32, 16, 1024),
                       make_sw128_desc(aw + c * 8192 + kk * 32, 16, 1024), id1, (c | kk) ? 1u : 0u);
        bulk_wait_read<0>();              // the previous V'^T store has read its tile
        tc_commit(d1_full);
        for (int c = 0; c < DK / 64; ++c) tma_store_2d(&ms, sst + c * 16384, 64 * c, srow);   // states[n] = S_n^T
        bulk_commit();
        if (!mbar_wait(v_full, n & 1, abort_flag, err, kErrTimeoutMma)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_f16(tb + Lt::C_S, make_sw128_desc(avt + kk * 32, 16, 1024),
                     make_sw128_desc(ak + kk * 2048, 8192, 1024), id2, 1u);
        tma_store_2d(&mv, svt, 0, srow);  // V'^T
        bulk_commit();
        bulk_wait_read<1>();              // the S_n^T store has read its tile
        tc_commit(s2_done);
        tc_commit(&w_empty[s]);
      }
      bulk_wait<0>();
    }
  } else {
    // ------------------------------------------------------------ state warps
    // eight warps, two per TMEM lane quarter: thread (quarter, lane) owns value
    // row v; `half` picks the columns (keys of S^T, tokens of V'^T) it handles
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const int v = quarter * 32 + lane;
    const uint32_t tl = tb + (static_cast<uint32_t>(quarter * 32) << 16);
    const int t = threadIdx.x - 64;                     // 0..255
    constexpr int NB = DK / 64;                         // 32-column blocks of S^T per half
    const int b0 = half * NB;
    bool ok = true;
    // U_n: plain [64][128] bf16 via cp.async by the eight warps
    auto load_u = [&](int n) {
      const __nv_bfloat16* src = U + (bh * N + n) * (long long)C * DV + v0;
      for (int i = t; i < C * (VT / 8); i += 256) {
        const int r = i / (VT / 8), c8 = (i % (VT / 8)) * 8;
        cp_async16(su + r * VT + c8, src + (long long)r * DV + c8);
      }
      cp_commit();
    };
    // 32 fp32 of row v (S^T columns 32 j ..) -> bf16 into the 128-byte swizzled K-major A operand
    auto put_bf16 = [&](int j, const uint32_t (&r)[32]) {
      uint8_t* base = sst + (j >> 1) * 16384 + v * 128;
#pragma unroll
      for (int u = 0; u < 4; ++u)
        *reinterpret_cast<uint4*>(base + ((((j & 1) * 4 + u) ^ (v & 7)) * 16)) =
            make_uint4(pack_bf16x2(__uint_as_float(r[8 * u]), __uint_as_float(r[8 * u + 1])),
                       pack_bf16x2(__uint_as_float(r[8 * u + 2]), __uint_as_float(r[8 * u + 3])),
                       pack_bf16x2(__uint_as_float(r[8 * u + 4]), __uint_as_float(r[8 * u + 5])),
                       pack_bf16x2(__uint_as_float(r[8 * u + 6]), __uint_as_float(r[8 * u + 7])));
    };
    // this thread's part of S^T (fp32) -> bf16 A operand of the next D1
    auto copy_state = [&]() {
      if constexpr (NB == 1) {
        uint32_t r0[32];
        tmem_ld_32x32b_x32(tl + Lt::C_S + static_cast<uint32_t>(32 * b0), r0);
        tmem_ld_wait();
        put_bf16(b0, r0);
      } else {
#pragma unroll 1
        for (int j = b0; j < b0 + NB; j += 2) {
          uint32_t r0[32], r1[32];
          tmem_ld_32x32b_x32(tl + Lt::C_S + static_cast<uint32_t>(32 * j), r0);
          tmem_ld_32x32b_x32(tl + Lt::C_S + static_cast<uint32_t>(32 * j + 32), r1);
          tmem_ld_wait();
          put_bf16(j, r0);
          put_bf16(j + 1, r1);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_ready);
    };
    // S^T *= gC of chunk `ci` in TMEM (overlaps the next D1, which reads only the
    // bf16 copy); a per-channel gate scales column k by gC[ci][k]
    auto scale_state = [&](long long ci) {
      const float g = gvec ? 0.f : gC[ci];
      const float* gv = gC + ci * DK;
#pragma unroll 1
      for (int j = b0; j < b0 + NB; ++j) {
        uint32_t r0[32];
        tmem_ld_32x32b_x32(tl + Lt::C_S + static_cast<uint32_t>(32 * j), r0);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) r0[e] = __float_as_uint(__uint_as_float(r0[e]) * (gvec ? gv[32 * j + e] : g));
        tmem_st_32x32b_x32(tl + Lt::C_S + static_cast<uint32_t>(32 * j), r0);
      }
      tmem_st_wait();
    };
    // initial state into TMEM
#pragma unroll 1
    for (int j = b0; j < b0 + NB; ++j) {
      uint32_t r[32];
#pragma unroll
      for (int e = 0; e < 32; ++e)
        r[e] = __float_as_uint(S0 ? S0[(bh * DK + 32 * j + e) * DV + v0 + v] : 0.f);
      tmem_st_32x32b_x32(tl + Lt::C_S + static_cast<uint32_t>(32 * j), r);
    }
    tmem_st_wait();
    load_u(0);
    copy_state();
    if (N > 0) scale_state(bh * N);
    for (int n = 0; n < N; ++n) {
      const long long cidx = bh * N + n;
      cp_wait_all();
      asm volatile("bar.sync 1, 256;" ::: "memory");     // U_n complete for all eight warps
      uint32_t uu[16];                                   // U_n[32 half + c][v] as bf16 pairs
#pragma unroll
      for (int c = 0; c < 32; c += 2)
        uu[c / 2] = static_cast<uint32_t>(__bfloat16_as_ushort(su[(32 * half + c) * VT + v])) |
                    (static_cast<uint32_t>(__bfloat16_as_ushort(su[(32 * half + c + 1) * VT + v])) << 16);
      asm volatile("bar.sync 1, 256;" ::: "memory");     // every warp has read U_n
      if (n + 1 < N) load_u(n + 1);
      // V'^T row v, tokens 32 half .. 32 half + 31 = U^T - D1
      ok = ok && mbar_wait_spin(d1_full, n & 1, abort_flag, err, kErrTimeoutEpilogue);
      tc_fence_after();
      uint32_t d[32];
      tmem_ld_32x32b_x32(tl + Lt::C_D1 + static_cast<uint32_t>(32 * half), d);
      tmem_ld_wait();
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = 8 * u + 2 * j;
          const float2 uf = unpack_bf16x2(uu[c / 2]);
          w[j] = pack_bf16x2(uf.x - __uint_as_float(d[c]), uf.y - __uint_as_float(d[c + 1]));
        }
        *reinterpret_cast<uint4*>(svt + v * 128 + (((4 * half + u) ^ (v & 7)) * 16)) =
            make_uint4(w[0], w[1], w[2], w[3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(v_full);
      // S_{n+1}: bf16 copy for the next D1, then scaled by gC_{n+1} in TMEM
      ok = ok && mbar_wait_spin(s2_done, n & 1, abort_flag, err, kErrTimeoutEpilogue);
      tc_fence_after();
      if (n + 1 < N) {
        copy_state();
        scale_state(cidx + 1);
      }
    }
    if (S_out) {
#pragma unroll 1
      for (int j = b0; j < b0 + NB; ++j) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tl + Lt::C_S + static_cast<uint32_t>(32 * j), r);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) S_out[(bh * DK + 32 * j + e) * DV + v0 + v] = __uint_as_float(r[e]);
      }
    }
    cp_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tb, Lt::COLS);
  }
}

// ------------------------------------------------------------ forward output --
// O[:, tile] = Qh S_n[:, tile] + A V'[:, tile]; grid (BH * N, DV / 64)

template <int DK>
struct OutSmem {
  __nv_bfloat16 Q[C][DK + PAD];
  __nv_bfloat16 ST[DVT][DK + PAD];     // S_n^T (states are stored value-major)
  __nv_bfloat16 A[C][C + PAD];
  __nv_bfloat16 VT[DVT][C + PAD];      // V'^T
  __nv_bfloat16 O[C][DVT + PAD];
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
  load_tile(&sm.ST[0][0], DK + PAD, states + (cidx * DV + v0) * DK, DK, DVT, DK);
  load_tile(&sm.A[0][0], C + PAD, A + cidx * C * C, C, C, C);
  load_tile(&sm.VT[0][0], C + PAD, Vp + (cidx * DV + v0) * C, C, DVT, C);
  cp_commit();
  cp_wait_all();
  __syncthreads();
  float acc[1][4][4];
  zero(acc);
  warp_mma<1, 4, false, false>(acc, &sm.Q[0][0], DK + PAD, &sm.ST[0][0], DK + PAD, wm0, wn0, DK);
  warp_mma<1, 4, false, false>(acc, &sm.A[0][0], C + PAD, &sm.VT[0][0], C + PAD, wm0, wn0, C);
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      const int r = wm0 + frag_row(0, e), c = wn0 + frag_col(nt, e);
      *reinterpret_cast<uint32_t*>(&sm.O[r][c]) = pack_bf16x2(acc[0][nt][e], acc[0][nt][e + 1]);
    }
  __syncthreads();
  store_tile(O + tok_row0(cidx / N, static_cast<int>(cidx % N), N, H, DV) + v0, (long long)H * DV, &sm.O[0][0],
             DVT + PAD, C, DVT);
}

// ------------------------------------------------ forward output, tcgen05 --
// O_n^T = S_n^T Qh_n^T + V'^T_n A_n^T on the tensor cores, one CTA per chunk:
// M = the value dimension (DV/128 tiles), N = the chunk's 64 tokens, K = the
// key dimension in 64-wide blocks and then the 64 tokens of V'.  Every K block
// pairs a [DV][64] A-operand tile (S^T block, or V'^T) with a [64][64]
// B-operand tile (Qh block, or A), both K-major, both by TMA, through a
// two-stage ring; O^T accumulates in TMEM and the epilogue warps write it
// token-major.  Every wait is bounded.
namespace tout {
template <int DV>
struct Layout {
  static constexpr int A_BYTES = DV * 64 * 2, B_BYTES = 64 * 64 * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int OFF_BAR = 2 * STAGE;
  static constexpr int SMEM = OFF_BAR + 128 + 1024;
  static constexpr int MT = DV / 128;
  static constexpr uint32_t COLS = MT == 1 ? 64 : (MT == 2 ? 128 : 256);
};
}  // namespace tout

template <int DK, int DV>
__global__ void __launch_bounds__(192, 1)
gdr_fwd_out_tc(const __grid_constant__ CUtensorMap m_st, const __grid_constant__ CUtensorMap m_qh,
               const __grid_constant__ CUtensorMap m_vt, const __grid_constant__ CUtensorMap m_a,
               __nv_bfloat16* __restrict__ O, int N, int H, int* err) {
  using Lt = tout::Layout<DV>;
  constexpr int NKB = DK / 64 + 1;                // K blocks: the keys, then the tokens of V'
  extern __shared__ __align__(128) uint8_t smem_raw[];   // re-aligned to 1024 (the swizzle atom) below
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Lt::OFF_BAR);
  uint64_t *full = bars, *empty = bars + 2, *acc_full = bars + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const long long cidx = blockIdx.x;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&m_st);
    tma_prefetch_desc(&m_qh);
    tma_prefetch_desc(&m_vt);
    tma_prefetch_desc(&m_a);
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
    if (lane == 0) {
      for (int kb = 0; kb < NKB; ++kb) {
        const int s = kb & 1;
        if (!mbar_wait(&empty[s], ((kb >> 1) & 1) ^ 1, abort_flag, err, kErrTimeoutProducer)) break;
        uint8_t* a = sm + s * Lt::STAGE;
        uint8_t* bt = a + Lt::A_BYTES;
        mbar_arrive_expect_tx(&full[s], Lt::STAGE);
        const bool keys = kb < DK / 64;
        for (int m = 0; m < DV / 128; ++m)
          tma_load_2d(a + m * 16384, keys ? &m_st : &m_vt, &full[s], keys ? 64 * kb : 0,
                      static_cast<int>(cidx * DV + 128 * m));
        tma_load_2d(bt, keys ? &m_qh : &m_a, &full[s], keys ? 64 * kb : 0, static_cast<int>(cidx * C));
      }
      for (int kb = NKB; kb < NKB + 2; ++kb)
        if (!mbar_wait(&empty[kb & 1], ((kb >> 1) & 1) ^ 1, abort_flag, err, kErrTimeoutProducer)) break;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id = make_idesc_bf16(128, 64, false, false);
      for (int kb = 0; kb < NKB; ++kb) {
        const int s = kb & 1;
        if (!mbar_wait(&full[s], (kb >> 1) & 1, abort_flag, err, kErrTimeoutMma)) break;
        tc_fence_after();
        const uint32_t a = smem_u32(sm + s * Lt::STAGE);
        const uint64_t da = make_sw128_desc(a, 16, 1024), db = make_sw128_desc(a + Lt::A_BYTES, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
          for (int m = 0; m < Lt::MT; ++m)
            tc_mma_f16(tb + 64 * m, desc_add(da, m * 16384 + kk * 32), desc_add(db, kk * 32), id, (kb | kk) ? 1u : 0u);
        tc_commit(&empty[s]);
      }
      tc_commit(acc_full);
    }
  } else {
    const int quarter = warp & 3;
    const uint32_t tl = tb + (static_cast<uint32_t>(quarter * 32) << 16);
    const bool ok = mbar_wait(acc_full, 0, abort_flag, err, kErrTimeoutEpilogue);
    tc_fence_after();
    const int v = quarter * 32 + lane;
    __nv_bfloat16* dst = O + tok_row0(cidx / N, static_cast<int>(cidx % N), N, H, DV) + v;
#pragma unroll 1
    for (int m = 0; m < Lt::MT; ++m) {
      uint32_t r0[32], r1[32];
      tmem_ld_32x32b_x32(tl + 64 * m, r0);
      tmem_ld_32x32b_x32(tl + 64 * m + 32, r1);
      tmem_ld_wait();
      if (ok) {
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          dst[(long long)c * H * DV + 128 * m] = f2bf(__uint_as_float(r0[c]));
          dst[(long long)(c + 32) * H * DV + 128 * m] = f2bf(__uint_as_float(r1[c]));
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
}

// ----------------------------------------------------- tcgen05 backward scan --
// The backward state chain on the tensor cores, transposed like the forward
// scan (value tile = MMA M = 128), one CTA per (sequence, value tile), with
// dS^T (value x key, fp32) in TMEM.  Per chunk, last to first:
//   snapshot  dstates_n = bf16(dS^T)                     (TMA store of the operand tile)
//   D1 = dV'^T = dO^T A + dS^T Kt^T                       (M = 128, N = 64 tokens)
//   dU = dV'  (state warps, from D1);  VN = -dV'^T        (bf16 operand tile)
//   dS^T <- gC dS^T + dO^T Qh + VN W                       (M = 128, N = DK)
// Warp 0 streams A and Kt (single stage, refilled once D1 is done), dO (two
// stages: it feeds both products) and Qh, W (single stage, refilled once the
// state update is done); warp 1 issues the MMAs and the snapshot stores;
// warps 2-9 (two per TMEM lane quarter) copy / scale the state and turn D1
// into VN and dU.  Every wait is bounded.
namespace tbscan {
constexpr int VT = 128;
template <int DK>
struct Layout {
  static constexpr int K_BYTES = C * DK * 2;     // Kt, Qh, W: DK/64 chunks of [64 tokens x 128 B]
  static constexpr int DO_BYTES = C * VT * 2;    // dO: 2 chunks of [64 tokens x 64 values]
  static constexpr int A_BYTES = C * C * 2;
  static constexpr int DT_BYTES = VT * DK * 2;   // bf16 dS^T: DK/64 chunks of [128 values x 128 B]
  static constexpr int VN_BYTES = VT * C * 2;    // -dV'^T: [128 values x 64 tokens]
  static constexpr int OFF_KT = 0, OFF_QH = K_BYTES, OFF_W = 2 * K_BYTES, OFF_DO = 3 * K_BYTES;
  static constexpr int OFF_A = OFF_DO + 2 * DO_BYTES, OFF_DT = OFF_A + A_BYTES, OFF_VN = OFF_DT + DT_BYTES;
  static constexpr int OFF_BAR = OFF_VN + VN_BYTES;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
  static constexpr uint32_t C_S = 0, C_D1 = DK, COLS = 512;
};
}  // namespace tbscan

template <int DK>
__global__ void __launch_bounds__(320, 1)
gdr_bwd_scan_tc(const __grid_constant__ CUtensorMap m_kt, const __grid_constant__ CUtensorMap m_qh,
                const __grid_constant__ CUtensorMap m_w, const __grid_constant__ CUtensorMap m_a,
                const __grid_constant__ CUtensorMap m_do, const __grid_constant__ CUtensorMap m_ds,
                const float* __restrict__ gC, const float* __restrict__ dS_final, __nv_bfloat16* __restrict__ dU,
                float* __restrict__ dS0, int N, int DV, int H, int gvec, int* err) {
  using namespace tbscan;
  using Lt = Layout<DK>;
  extern __shared__ __align__(128) uint8_t smem_raw[];   // re-aligned to 1024 (the swizzle atom) below
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *skt = sm + Lt::OFF_KT, *sqh = sm + Lt::OFF_QH, *sw = sm + Lt::OFF_W, *sdo = sm + Lt::OFF_DO;
  uint8_t *sa = sm + Lt::OFF_A, *sdt = sm + Lt::OFF_DT, *svn = sm + Lt::OFF_VN;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Lt::OFF_BAR);
  uint64_t *a_full = bars, *a_empty = bars + 1, *do_full = bars + 2, *do_empty = bars + 4, *b_full = bars + 6,
           *b_empty = bars + 7, *dt_ready = bars + 8, *d1_full = bars + 9, *vn_ready = bars + 10, *s2_done = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int tiles_v = DV / VT;
  const long long bh = blockIdx.x / tiles_v;
  const int v0 = (blockIdx.x % tiles_v) * VT;

  if (threadIdx.x == 0) {
    mbar_init(a_full, 1);
    mbar_init(a_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&do_full[i], 1);
      mbar_init(&do_empty[i], 1);
    }
    mbar_init(b_full, 1);
    mbar_init(b_empty, 1);
    mbar_init(dt_ready, 8);
    mbar_init(d1_full, 1);
    mbar_init(vn_ready, 8);
    mbar_init(s2_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&m_kt);
    tma_prefetch_desc(&m_qh);
    tma_prefetch_desc(&m_w);
    tma_prefetch_desc(&m_a);
    tma_prefetch_desc(&m_do);
    tma_prefetch_desc(&m_ds);
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
    if (lane == 0) {
      const int b = static_cast<int>(bh / H), h = static_cast<int>(bh % H);
      // j = 0, 1, ... walks the chunks n = N - 1, N - 2, ...
      for (int j = 0; j < N; ++j) {
        const int n = N - 1 - j, s = j & 1;
        const int row = static_cast<int>((bh * N + n) * C);
        if (!mbar_wait(&do_empty[s], ((j >> 1) & 1) ^ 1, abort_flag, err, kErrTimeoutProducer)) break;
        mbar_arrive_expect_tx(&do_full[s], Lt::DO_BYTES);
        for (int i = 0; i < 2; ++i)
          tma_load_3d(sdo + s * Lt::DO_BYTES + i * 8192, &m_do, &do_full[s], v0 + 64 * i, h, b * N * C + n * C);
        if (!mbar_wait(a_empty, (j & 1) ^ 1, abort_flag, err, kErrTimeoutProducer)) break;
        mbar_arrive_expect_tx(a_full, Lt::A_BYTES + Lt::K_BYTES);
        tma_load_2d(sa, &m_a, a_full, 0, row);
        for (int c = 0; c < DK / 64; ++c) tma_load_2d(skt + c * 8192, &m_kt, a_full, 64 * c, row);
        if (!mbar_wait(b_empty, (j & 1) ^ 1, abort_flag, err, kErrTimeoutProducer)) break;
        mbar_arrive_expect_tx(b_full, 2 * Lt::K_BYTES);
        for (int c = 0; c < DK / 64; ++c) {
          tma_load_2d(sqh + c * 8192, &m_qh, b_full, 64 * c, row);
          tma_load_2d(sw + c * 8192, &m_w, b_full, 64 * c, row);
        }
      }
      // the last releases land before the CTA retires
      if (mbar_wait(a_empty, (N & 1) ^ 1, abort_flag, err, kErrTimeoutProducer))
        mbar_wait(b_empty, (N & 1) ^ 1, abort_flag, err, kErrTimeoutProducer);
      for (int j = N; j < N + 2; ++j)
        if (!mbar_wait(&do_empty[j & 1], ((j >> 1) & 1) ^ 1, abort_flag, err, kErrTimeoutProducer)) break;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_a = make_idesc_bf16(VT, C, true, true);     // dO^T (MN) x A (MN)
      constexpr uint32_t id_b = make_idesc_bf16(VT, C, false, false);   // dS^T (K) x Kt (K)
      constexpr uint32_t id_c = make_idesc_bf16(VT, DK, true, true);    // dO^T (MN) x Qh (MN)
      constexpr uint32_t id_d = make_idesc_bf16(VT, DK, false, true);   // VN (K) x W (MN)
      const uint64_t d_a = make_sw128_desc(smem_u32(sa), 16, 1024);
      const uint64_t d_kt = make_sw128_desc(smem_u32(skt), 16, 1024);
      const uint64_t d_qh = make_sw128_desc(smem_u32(sqh), 8192, 1024);
      const uint64_t d_w = make_sw128_desc(smem_u32(sw), 8192, 1024);
      const uint64_t d_dt = make_sw128_desc(smem_u32(sdt), 16, 1024);
      const uint64_t d_vn = make_sw128_desc(smem_u32(svn), 16, 1024);
      for (int j = 0; j < N; ++j) {
        const int n = N - 1 - j, s = j & 1;
        const int srow = static_cast<int>((bh * N + n) * DV + v0);       // this tile's rows in the value-major dstates
        const uint64_t d_do = make_sw128_desc(smem_u32(sdo + s * Lt::DO_BYTES), 8192, 1024);
        if (!mbar_wait(dt_ready, j & 1, abort_flag, err, kErrTimeoutMma)) break;
        if (!mbar_wait(a_full, j & 1, abort_flag, err, kErrTimeoutMma)) break;
        if (!mbar_wait(&do_full[s], (j >> 1) & 1, abort_flag, err, kErrTimeoutMma)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_f16(tb + Lt::C_D1, desc_add(d_do, kk * 2048), desc_add(d_a, kk * 2048), id_a, kk ? 1u : 0u);
#pragma unroll
        for (int c = 0; c < DK / 64; ++c)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc_mma_f16(tb + Lt::C_D1, desc_add(d_dt, c * 16384 + kk * 32), desc_add(d_kt, c * 8192 + kk * 32), id_b,
                       1u);
        tc_commit(d1_full);
        tc_commit(a_empty);
        for (int c = 0; c < DK / 64; ++c) tma_store_2d(&m_ds, sdt + c * 16384, 64 * c, srow);   // dstates_n
        bulk_commit();
        if (!mbar_wait(vn_ready, j & 1, abort_flag, err, kErrTimeoutMma)) break;
        if (!mbar_wait(b_full, j & 1, abort_flag, err, kErrTimeoutMma)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          tc_mma_f16(tb + Lt::C_S, desc_add(d_do, kk * 2048), desc_add(d_qh, kk * 2048), id_c, 1u);
          tc_mma_f16(tb + Lt::C_S, desc_add(d_vn, kk * 32), desc_add(d_w, kk * 2048), id_d, 1u);
        }
        bulk_wait_read<0>();              // the snapshot store has read the dS^T tile
        tc_commit(s2_done);
        tc_commit(b_empty);
        tc_commit(&do_empty[s]);
      }
      bulk_wait<0>();
    }
  } else {
    // ------------------------------------------------------------ state warps
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const int v = quarter * 32 + lane;
    const uint32_t tl = tb + (static_cast<uint32_t>(quarter * 32) << 16);
    constexpr int NB = DK / 64;
    const int b0 = half * NB;
    bool ok = true;
    auto put_bf16 = [&](int jb, const uint32_t (&r)[32]) {
      uint8_t* base = sdt + (jb >> 1) * 16384 + v * 128;
#pragma unroll
      for (int u = 0; u < 4; ++u)
        *reinterpret_cast<uint4*>(base + ((((jb & 1) * 4 + u) ^ (v & 7)) * 16)) =
            make_uint4(pack_bf16x2(__uint_as_float(r[8 * u]), __uint_as_float(r[8 * u + 1])),
                       pack_bf16x2(__uint_as_float(r[8 * u + 2]), __uint_as_float(r[8 * u + 3])),
                       pack_bf16x2(__uint_as_float(r[8 * u + 4]), __uint_as_float(r[8 * u + 5])),
                       pack_bf16x2(__uint_as_float(r[8 * u + 6]), __uint_as_float(r[8 * u + 7])));
    };
    auto copy_state = [&]() {
#pragma unroll 1
      for (int jb = b0; jb < b0 + NB; ++jb) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tl + Lt::C_S + static_cast<uint32_t>(32 * jb), r);
        tmem_ld_wait();
        put_bf16(jb, r);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dt_ready);
    };
    auto scale_state = [&](long long ci) {
      const float g = gvec ? 0.f : gC[ci];
      const float* gv = gC + ci * DK;
#pragma unroll 1
      for (int jb = b0; jb < b0 + NB; ++jb) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tl + Lt::C_S + static_cast<uint32_t>(32 * jb), r);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * (gvec ? gv[32 * jb + e] : g));
        tmem_st_32x32b_x32(tl + Lt::C_S + static_cast<uint32_t>(32 * jb), r);
      }
      tmem_st_wait();
    };
    // initial dS^T
#pragma unroll 1
    for (int jb = b0; jb < b0 + NB; ++jb) {
      uint32_t r[32];
#pragma unroll
      for (int e = 0; e < 32; ++e)
        r[e] = __float_as_uint(dS_final ? dS_final[(bh * DK + 32 * jb + e) * DV + v0 + v] : 0.f);
      tmem_st_32x32b_x32(tl + Lt::C_S + static_cast<uint32_t>(32 * jb), r);
    }
    tmem_st_wait();
    for (int j = 0; j < N; ++j) {
      const int n = N - 1 - j;
      const long long cidx = bh * N + n;
      copy_state();                                      // dstates_n and the operand of D1
      scale_state(cidx);                                 // gC dS^T, before the update accumulates
      ok = ok && mbar_wait_spin(d1_full, j & 1, abort_flag, err, kErrTimeoutEpilogue);
      tc_fence_after();
      uint32_t d[32];
      tmem_ld_32x32b_x32(tl + Lt::C_D1 + static_cast<uint32_t>(32 * half), d);
      tmem_ld_wait();
      // VN row v, tokens 32 half .. : -dV'^T as the K-major operand of the update
#pragma unroll
      for (int u = 0; u < 4; ++u)
        *reinterpret_cast<uint4*>(svn + v * 128 + (((4 * half + u) ^ (v & 7)) * 16)) =
            make_uint4(pack_bf16x2(-__uint_as_float(d[8 * u]), -__uint_as_float(d[8 * u + 1])),
                       pack_bf16x2(-__uint_as_float(d[8 * u + 2]), -__uint_as_float(d[8 * u + 3])),
                       pack_bf16x2(-__uint_as_float(d[8 * u + 4]), -__uint_as_float(d[8 * u + 5])),
                       pack_bf16x2(-__uint_as_float(d[8 * u + 6]), -__uint_as_float(d[8 * u + 7])));
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(vn_ready);
      // dU = dV' (token-major within the chunk), off the critical path
      __nv_bfloat16* du = dU + (cidx * C + 32 * half) * DV + v0 + v;
#pragma unroll
      for (int c = 0; c < 32; ++c) du[(long long)c * DV] = f2bf(__uint_as_float(d[c]));
      ok = ok && mbar_wait_spin(s2_done, j & 1, abort_flag, err, kErrTimeoutEpilogue);
      tc_fence_after();
    }
    if (dS0) {
#pragma unroll 1
      for (int jb = b0; jb < b0 + NB; ++jb) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tl + Lt::C_S + static_cast<uint32_t>(32 * jb), r);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) dS0[(bh * DK + 32 * jb + e) * DV + v0 + v] = __uint_as_float(r[e]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tb, Lt::COLS);
  }
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
             int DV, int H, int gvec) {
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
    store_tile_t(dstates + (cidx * DV + v0) * DK, DK, &sm.dS[0][0], DVT + PAD, DK, DVT);

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

    // dS <- gC dS + Qh^T dO - W^T dV'  (row k scaled by gC[k] for a per-channel gate)
    const float g = gvec ? 0.f : gC[cidx];
#pragma unroll
    for (int mt = 0; mt < SMT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          dS[mt][nt][e] *= gvec ? gC[cidx * DK + srow0 + frag_row(mt, e)] : g;
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
  __nv_bfloat16 VT[2][DVT][C + PAD];     // V'^T
  __nv_bfloat16 ST[2][DVT][64 + PAD];    // S_n^T columns k0..k0+63
  __nv_bfloat16 dST[2][DVT][64 + PAD];   // dS_n^T columns k0..k0+63
  float red[THREADS / 32];
  float rowdot[THREADS];                 // per-channel gate: per-row partial sums
};

__global__ void __launch_bounds__(THREADS, 2)
gdr_bwd_chunk(const __nv_bfloat16* __restrict__ dU, const __nv_bfloat16* __restrict__ dO,
              const __nv_bfloat16* __restrict__ Vp, const __nv_bfloat16* __restrict__ states,
              const __nv_bfloat16* __restrict__ dstates, __nv_bfloat16* __restrict__ dW,
              __nv_bfloat16* __restrict__ dQh, __nv_bfloat16* __restrict__ dKt, float* __restrict__ dA,
              float* __restrict__ dgC, int DK, int DV, int N, int H, int gvec) {
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
    load_tile(&sm.VT[b][0][0], C + PAD, Vp + (cidx * DV + v0) * C, C, DVT, C);
    load_tile(&sm.ST[b][0][0], 64 + PAD, states + (cidx * DV + v0) * DK + k0, DK, DVT, 64);
    load_tile(&sm.dST[b][0][0], 64 + PAD, dstates + (cidx * DV + v0) * DK + k0, DK, DVT, 64);
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
    warp_mma<1, 4, false, true>(aw, &sm.dV[b][0][0], DVT + PAD, &sm.ST[b][0][0], 64 + PAD, wm0, wn0, DVT);
    warp_mma<1, 4, false, true>(aq, &sm.dO[b][0][0], DVT + PAD, &sm.ST[b][0][0], 64 + PAD, wm0, wn0, DVT);
    warp_mma<1, 4, true, true>(ak, &sm.VT[b][0][0], C + PAD, &sm.dST[b][0][0], 64 + PAD, wm0, wn0, DVT);
    if (do_dA) warp_mma<1, 4, false, true>(aa, &sm.dO[b][0][0], DVT + PAD, &sm.VT[b][0][0], C + PAD, wm0, wn0, DVT);
    // THREADS is a multiple of 64: every pass of a thread is on key row threadIdx.x % 64
    for (int i = threadIdx.x; i < 64 * DVT; i += THREADS) {
      const int r = i % 64, c = i / 64;             // key r, value c
      dot += bf2f(sm.ST[b][c][r]) * bf2f(sm.dST[b][c][r]);
    }
    __syncthreads();
  }
  if (gvec) {
    // dgC[k0 + r]: the THREADS / 64 partial sums of row r
    sm.rowdot[threadIdx.x] = dot;
    __syncthreads();
    if (threadIdx.x < 64) {
      float t = 0.f;
      for (int i = threadIdx.x; i < THREADS; i += 64) t += sm.rowdot[i];
      atomicAdd(&dgC[cidx * DK + k0 + threadIdx.x], t);
    }
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
  if (threadIdx.x == 0 && !gvec) {
    float t = 0.f;
    for (int i = 0; i < THREADS / 32; ++i) t += sm.red[i];
    atomicAdd(&dgC[cidx], t);
  }
}

// ------------------------------------------- backward, per chunk, tcgen05 --
// One CTA per chunk: with the value dimension as the contraction (K), the
// chunk's gradient products are all M = 128 tiles over the key dimension:
//   dW^T  = -S dV'^T      dQh^T = S dO^T      dKt^T = dS V'^T      (DK x C)
//   dA    = dO V'^T       (C x C; M = 128 with the upper 64 rows unused)
// S arrives as the value-major snapshot S^T (read MN-major), dS as dL/dS_n
// (K-major), dV' = dU, dO (token-major) and V'^T all by TMA, one 64-wide value
// block per stage of a two-stage ring; the accumulators live in TMEM.  Warps
// 2-5 form dgC = <S, dS> (per key row for a per-channel gate) from the staged
// tiles while the tensor core runs, then write the products.  Every wait is
// bounded.
namespace tchunk {
template <int DK>
struct Layout {
  static constexpr int ST_BYTES = 64 * DK * 2;    // S^T block: DK/64 chunks of [64 v][64 k]
  static constexpr int DS_BYTES = 64 * DK * 2;    // dS^T block: DK/64 chunks of [64 v][64 k]
  static constexpr int T_BYTES = 64 * 64 * 2;     // dO, dU: [64 c][64 v]; V'^T: [64 v][64 c]
  static constexpr int OFF_DO = 0, OFF_DU = T_BYTES, OFF_VT = 2 * T_BYTES, OFF_ST = 3 * T_BYTES;
  static constexpr int OFF_DS = OFF_ST + ST_BYTES;
  static constexpr int STAGE = OFF_DS + DS_BYTES;
  static constexpr int OFF_BAR = 2 * STAGE;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
  static constexpr int MT = DK / 128;             // M tiles over the keys
  static constexpr uint32_t C_DW = 0, C_DQ = 64 * MT, C_DK = 128 * MT, C_DA = 192 * MT;
  static constexpr uint32_t COLS = DK == 256 ? 512 : 256;
};
}  // namespace tchunk

template <int DK>
__global__ void __launch_bounds__(192, 1)
gdr_bwd_chunk_tc(const __grid_constant__ CUtensorMap m_st, const __grid_constant__ CUtensorMap m_ds,
                 const __grid_constant__ CUtensorMap m_du, const __grid_constant__ CUtensorMap m_do,
                 const __grid_constant__ CUtensorMap m_vt, __nv_bfloat16* __restrict__ dW,
                 __nv_bfloat16* __restrict__ dQh, __nv_bfloat16* __restrict__ dKt, float* __restrict__ dA,
                 float* __restrict__ dgC, int DV, int N, int H, int gvec, int* err) {
  using Lt = tchunk::Layout<DK>;
  extern __shared__ __align__(128) uint8_t smem_raw[];   // re-aligned to 1024 (the swizzle atom) below
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Lt::OFF_BAR);
  uint64_t *full = bars, *empty = bars + 2, *acc_full = bars + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(tmem_slot + 2);            // [4] block partial sums

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const long long cidx = blockIdx.x;
  const long long bh = cidx / N;
  const int n = static_cast<int>(cidx % N);
  const int nvb = DV / 64;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1 + 4);      // the MMA commit + the four dgC warps
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&m_st);
    tma_prefetch_desc(&m_ds);
    tma_prefetch_desc(&m_du);
    tma_prefetch_desc(&m_do);
    tma_prefetch_desc(&m_vt);
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
    if (lane == 0) {
      const int b = static_cast<int>(bh / H), h = static_cast<int>(bh % H);
      for (int vb = 0; vb < nvb; ++vb) {
        const int s = vb & 1;
        if (!mbar_wait(&empty[s], ((vb >> 1) & 1) ^ 1, abort_flag, err, kErrTimeoutProducer)) break;
        uint8_t* st = sm + s * Lt::STAGE;
        mbar_arrive_expect_tx(&full[s], Lt::STAGE);
        const int v0 = vb * 64;
        tma_load_3d(st + Lt::OFF_DO, &m_do, &full[s], v0, h, b * N * C + n * C);
        tma_load_2d(st + Lt::OFF_DU, &m_du, &full[s], v0, static_cast<int>(cidx * C));
        tma_load_2d(st + Lt::OFF_VT, &m_vt, &full[s], 0, static_cast<int>(cidx * DV + v0));
        for (int c = 0; c < DK / 64; ++c)
          tma_load_2d(st + Lt::OFF_ST + c * 8192, &m_st, &full[s], 64 * c, static_cast<int>(cidx * DV + v0));
        for (int c = 0; c < DK / 64; ++c)
          tma_load_2d(st + Lt::OFF_DS + c * 8192, &m_ds, &full[s], 64 * c, static_cast<int>(cidx * DV + v0));
      }
      for (int vb = nvb; vb < nvb + 2; ++vb)      // the ring's last releases land before the CTA retires
        if (!mbar_wait(&empty[vb & 1], ((vb >> 1) & 1) ^ 1, abort_flag, err, kErrTimeoutProducer)) break;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = make_idesc_bf16(128, 64, true, false);   // A = S (MN-major), B K-major
      constexpr uint32_t id_v = make_idesc_bf16(128, 64, false, true);   // A = dO K-major, B = V'^T (MN-major)
      constexpr uint32_t id_k = make_idesc_bf16(128, 64, true, true);    // A = dS (MN-major), B = V'^T (MN-major)
      for (int vb = 0; vb < nvb; ++vb) {
        const int s = vb & 1;
        if (!mbar_wait(&full[s], (vb >> 1) & 1, abort_flag, err, kErrTimeoutMma)) break;
        tc_fence_after();
        const uint32_t st = smem_u32(sm + s * Lt::STAGE);
        const uint64_t d_do = make_sw128_desc(st + Lt::OFF_DO, 16, 1024);
        const uint64_t d_du = make_sw128_desc(st + Lt::OFF_DU, 16, 1024);
        const uint64_t d_vt = make_sw128_desc(st + Lt::OFF_VT, 8192, 1024);
        const uint64_t d_st = make_sw128_desc(st + Lt::OFF_ST, 8192, 1024);
        const uint64_t d_ds = make_sw128_desc(st + Lt::OFF_DS, 8192, 1024);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {          // 16 values per step
          const uint32_t acc = (vb | kk) ? 1u : 0u;
#pragma unroll
          for (int m = 0; m < Lt::MT; ++m) {
            tc_mma_f16(tb + Lt::C_DW + 64 * m, desc_add(d_st, m * 16384 + kk * 2048), desc_add(d_du, kk * 32), id_s,
                       acc);
            tc_mma_f16(tb + Lt::C_DQ + 64 * m, desc_add(d_st, m * 16384 + kk * 2048), desc_add(d_do, kk * 32), id_s,
                       acc);
            tc_mma_f16(tb + Lt::C_DK + 64 * m, desc_add(d_ds, m * 16384 + kk * 2048), desc_add(d_vt, kk * 2048), id_k,
                       acc);
          }
          tc_mma_f16(tb + Lt::C_DA, desc_add(d_do, kk * 32), desc_add(d_vt, kk * 2048), id_v, acc);
        }
        tc_commit(&empty[s]);
      }
      tc_commit(acc_full);
    }
  } else {
    // ---------------------------------------------------- dgC, then products
    const int quarter = warp & 3;
    const int t = threadIdx.x - 64;                 // 0..127
    const uint32_t tl = tb + (static_cast<uint32_t>(quarter * 32) << 16);
    bool ok = true;
    float dot[DK / 128] = {};                       // rows k = t + 128 i
    for (int vb = 0; vb < nvb; ++vb) {
      const int s = vb & 1;
      ok = ok && mbar_wait(&full[s], (vb >> 1) & 1, abort_flag, err, kErrTimeoutEpilogue);
      const uint8_t* st = sm + s * Lt::STAGE;
#pragma unroll
      for (int i = 0; i < DK / 128; ++i) {
        const int k = t + 128 * i;
        // S^T and dS^T chunks [v][k]: row v, 16-byte unit ((k & 63) >> 3) ^ (v & 7), element k & 7
        const int off = (k >> 6) * 8192 + (k & 7) * 2;
        float acc = 0.f;
#pragma unroll 8
        for (int v = 0; v < 64; ++v) {
          const int o = off + v * 128 + ((((k & 63) >> 3) ^ (v & 7)) * 16);
          acc = fmaf(bf2f(*reinterpret_cast<const __nv_bfloat16*>(st + Lt::OFF_ST + o)),
                     bf2f(*reinterpret_cast<const __nv_bfloat16*>(st + Lt::OFF_DS + o)), acc);
        }
        dot[i] += acc;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (gvec) {
#pragma unroll
      for (int i = 0; i < DK / 128; ++i) dgC[cidx * DK + t + 128 * i] = dot[i];
    } else {
      float tot = 0.f;
#pragma unroll
      for (int i = 0; i < DK / 128; ++i) tot += dot[i];
      tot = warp_sum(tot);
      if (lane == 0) red[quarter] = tot;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (t == 0) dgC[cidx] = red[0] + red[1] + red[2] + red[3];
    }
    // products: TMEM lane = key row (dA: query row c < 64), columns = the chunk's 64 tokens
    ok = ok && mbar_wait(acc_full, 0, abort_flag, err, kErrTimeoutEpilogue);
    tc_fence_after();
    const int row = quarter * 32 + lane;
#pragma unroll 1
    for (int which = 0; which < 3; ++which) {
      __nv_bfloat16* out = which == 0 ? dW : (which == 1 ? dQh : dKt);
      const uint32_t base = which == 0 ? Lt::C_DW : (which == 1 ? Lt::C_DQ : Lt::C_DK);
      const float sgn = which == 0 ? -1.f : 1.f;
#pragma unroll 1
      for (int m = 0; m < Lt::MT; ++m) {
        uint32_t r0[32], r1[32];
        tmem_ld_32x32b_x32(tl + base + 64 * m, r0);
        tmem_ld_32x32b_x32(tl + base + 64 * m + 32, r1);
        tmem_ld_wait();
        if (ok) {
          __nv_bfloat16* dst = out + (cidx * C) * DK + 128 * m + row;
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            dst[(long long)c * DK] = f2bf(sgn * __uint_as_float(r0[c]));
            dst[(long long)(c + 32) * DK] = f2bf(sgn * __uint_as_float(r1[c]));
          }
        }
      }
    }
    {
      uint32_t r0[32], r1[32];
      tmem_ld_32x32b_x32(tl + Lt::C_DA, r0);
      tmem_ld_32x32b_x32(tl + Lt::C_DA + 32, r1);
      tmem_ld_wait();
      if (ok && row < C) {
        float* dst = dA + (cidx * C + row) * C;
#pragma unroll
        for (int c = 0; c < 32; c += 4) {
          *reinterpret_cast<float4*>(dst + c) = make_float4(__uint_as_float(r0[c]), __uint_as_float(r0[c + 1]),
                                                            __uint_as_float(r0[c + 2]), __uint_as_float(r0[c + 3]));
          *reinterpret_cast<float4*>(dst + 32 + c) = make_float4(__uint_as_float(r1[c]), __uint_as_float(r1[c + 1]),
                                                                 __uint_as_float(r1[c + 2]), __uint_as_float(r1[c + 3]));
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
  static const bool no_tc = std::getenv("VAGUS_GDR_NO_TC") != nullptr;
  if (!no_tc && a.err && a.DV % tscan::VT == 0) {
    using Lt = tscan::Layout<DK>;
    alignas(64) unsigned char mw[128], mk[128], ms[128], mv[128];
    const unsigned long long dims[2] = {(unsigned long long)DK, (unsigned long long)a.BH * a.N * C};
    const unsigned long long strides[1] = {(unsigned long long)DK * 2};
    const unsigned box[2] = {64u, 64u};
    // value-major outputs: states [BH][N][DV][DK], V' [BH][N][DV][C]; 128-row boxes
    const unsigned long long dims_s[2] = {(unsigned long long)DK, (unsigned long long)a.BH * a.N * a.DV};
    const unsigned long long dims_v[2] = {(unsigned long long)C, (unsigned long long)a.BH * a.N * a.DV};
    const unsigned long long strides_v[1] = {(unsigned long long)C * 2};
    const unsigned box_o[2] = {64u, static_cast<unsigned>(tscan::VT)};
    if (!encode_bf16_map(mw, a.W, 2, dims, strides, box) || !encode_bf16_map(mk, a.Kt, 2, dims, strides, box) ||
        !encode_bf16_map(ms, a.states, 2, dims_s, strides, box_o) ||
        !encode_bf16_map(mv, a.Vp, 2, dims_v, strides_v, box_o))
      return 2;
    if (!set_smem(gdr_fwd_scan_tc<DK>, Lt::SMEM)) return 3;
    gdr_fwd_scan_tc<DK><<<static_cast<unsigned>(a.BH * (a.DV / tscan::VT)), 320, Lt::SMEM, st>>>(
        *reinterpret_cast<const CUtensorMap*>(mw), *reinterpret_cast<const CUtensorMap*>(mk),
        *reinterpret_cast<const CUtensorMap*>(ms), *reinterpret_cast<const CUtensorMap*>(mv),
        (const __nv_bfloat16*)a.U, a.gC, a.S0, a.S_out, a.N, a.DV, a.gvec, a.err);
  } else {
    const int grid = static_cast<int>(a.BH * (a.DV / DVT));
    gdr_fwd_scan<DK><<<grid, THREADS, s1, st>>>((const __nv_bfloat16*)a.W, (const __nv_bfloat16*)a.Kt,
                                                (const __nv_bfloat16*)a.U, a.gC, a.S0, (__nv_bfloat16*)a.Vp,
                                                (__nv_bfloat16*)a.states, a.S_out, a.N, a.DV, a.gvec);
  }
  if (!no_tc && a.err && (a.DV == 128 || a.DV == 256 || a.DV == 512)) {
    alignas(64) unsigned char m_st[128], m_qh[128], m_vt[128], m_a[128];
    const unsigned long long BHN = (unsigned long long)a.BH * a.N;
    const unsigned long long d_st[2] = {(unsigned long long)DK, BHN * a.DV}, s_st[1] = {(unsigned long long)DK * 2};
    const unsigned long long d_qh[2] = {(unsigned long long)DK, BHN * C};
    const unsigned long long d_vt[2] = {(unsigned long long)C, BHN * a.DV}, s_c[1] = {(unsigned long long)C * 2};
    const unsigned long long d_a[2] = {(unsigned long long)C, BHN * C};
    const unsigned box_a[2] = {64u, 128u}, box_b[2] = {64u, 64u};
    if (!encode_bf16_map(m_st, a.states, 2, d_st, s_st, box_a) || !encode_bf16_map(m_qh, a.Qh, 2, d_qh, s_st, box_b) ||
        !encode_bf16_map(m_vt, a.Vp, 2, d_vt, s_c, box_a) || !encode_bf16_map(m_a, a.A, 2, d_a, s_c, box_b))
      return 2;
    auto go = [&](auto kern, int smem) -> int {
      if (!set_smem(kern, smem)) return 3;
      kern<<<static_cast<unsigned>(BHN), 192, smem, st>>>(
          *reinterpret_cast<const CUtensorMap*>(m_st), *reinterpret_cast<const CUtensorMap*>(m_qh),
          *reinterpret_cast<const CUtensorMap*>(m_vt), *reinterpret_cast<const CUtensorMap*>(m_a),
          (__nv_bfloat16*)a.O, a.N, a.H, a.err);
      return cudaGetLastError() == cudaSuccess ? 0 : 3;
    };
    if (a.DV == 128) return go(gdr_fwd_out_tc<DK, 128>, tout::Layout<128>::SMEM);
    if (a.DV == 256) return go(gdr_fwd_out_tc<DK, 256>, tout::Layout<256>::SMEM);
    return go(gdr_fwd_out_tc<DK, 512>, tout::Layout<512>::SMEM);
  }
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
  static const bool no_tc_scan = std::getenv("VAGUS_GDR_NO_TC") != nullptr;
  if (!no_tc_scan && a.f.err && a.f.DV % tbscan::VT == 0) {
    using Lt = tbscan::Layout<DK>;
    alignas(64) unsigned char m_kt[128], m_qh[128], m_w[128], m_a[128], m_do[128], m_ds[128];
    const unsigned long long BHN = (unsigned long long)a.f.BH * a.f.N;
    const unsigned long long d_k[2] = {(unsigned long long)DK, BHN * C}, s_k[1] = {(unsigned long long)DK * 2};
    const unsigned long long d_a[2] = {(unsigned long long)C, BHN * C}, s_a[1] = {(unsigned long long)C * 2};
    const unsigned long long d_ds[2] = {(unsigned long long)DK, BHN * a.f.DV};
    const unsigned long long d_do[3] = {(unsigned long long)a.f.DV, (unsigned long long)a.f.H,
                                        (unsigned long long)(a.f.BH / a.f.H) * a.f.N * C};
    const unsigned long long s_do[2] = {(unsigned long long)a.f.DV * 2, (unsigned long long)a.f.H * a.f.DV * 2};
    const unsigned box64[2] = {64u, 64u}, box_ds[2] = {64u, static_cast<unsigned>(tbscan::VT)},
                   box_do[3] = {64u, 1u, 64u};
    if (!encode_bf16_map(m_kt, a.f.Kt, 2, d_k, s_k, box64) || !encode_bf16_map(m_qh, a.f.Qh, 2, d_k, s_k, box64) ||
        !encode_bf16_map(m_w, a.f.W, 2, d_k, s_k, box64) || !encode_bf16_map(m_a, a.f.A, 2, d_a, s_a, box64) ||
        !encode_bf16_map(m_do, a.dO, 3, d_do, s_do, box_do) ||
        !encode_bf16_map(m_ds, a.dstates, 2, d_ds, s_k, box_ds))
      return 2;
    if (!set_smem(gdr_bwd_scan_tc<DK>, Lt::SMEM)) return 3;
    gdr_bwd_scan_tc<DK><<<static_cast<unsigned>(a.f.BH * (a.f.DV / tbscan::VT)), 320, Lt::SMEM, st>>>(
        *reinterpret_cast<const CUtensorMap*>(m_kt), *reinterpret_cast<const CUtensorMap*>(m_qh),
        *reinterpret_cast<const CUtensorMap*>(m_w), *reinterpret_cast<const CUtensorMap*>(m_a),
        *reinterpret_cast<const CUtensorMap*>(m_do), *reinterpret_cast<const CUtensorMap*>(m_ds), a.f.gC,
        a.dS_final, (__nv_bfloat16*)a.dU, a.dS0, a.f.N, a.f.DV, a.f.H, a.f.gvec, a.f.err);
  } else {
  const int grid = static_cast<int>(a.f.BH * (a.f.DV / DVT));
  gdr_bwd_scan<DK><<<grid, THREADS, s1, st>>>((const __nv_bfloat16*)a.f.W, (const __nv_bfloat16*)a.f.Qh,
                                              (const __nv_bfloat16*)a.f.Kt, (const __nv_bfloat16*)a.f.A, a.f.gC,
                                              (const __nv_bfloat16*)a.dO, a.dS_final, (__nv_bfloat16*)a.dU,
                                              (__nv_bfloat16*)a.dstates, a.dS0, a.f.N, a.f.DV, a.f.H, a.f.gvec);
  }
  static const bool no_tc = std::getenv("VAGUS_GDR_NO_TC") != nullptr;
  if (!no_tc && a.f.err && a.f.DV % 64 == 0) {
    using Lt = tchunk::Layout<DK>;
    alignas(64) unsigned char m_st[128], m_ds[128], m_du[128], m_do[128], m_vt[128];
    const unsigned long long BHN = (unsigned long long)a.f.BH * a.f.N;
    const unsigned long long d_st[2] = {(unsigned long long)DK, BHN * a.f.DV};
    const unsigned long long s_st[1] = {(unsigned long long)DK * 2};
    const unsigned long long d_ds[2] = {(unsigned long long)DK, BHN * a.f.DV};
    const unsigned long long d_du[2] = {(unsigned long long)a.f.DV, BHN * C};
    const unsigned long long s_dv[1] = {(unsigned long long)a.f.DV * 2};
    const unsigned long long d_vt[2] = {(unsigned long long)C, BHN * a.f.DV};
    const unsigned long long s_vt[1] = {(unsigned long long)C * 2};
    // dO token-major (B, L, H, DV): {DV, H, B * L}
    const unsigned long long d_do[3] = {(unsigned long long)a.f.DV, (unsigned long long)a.f.H,
                                        (unsigned long long)(a.f.BH / a.f.H) * a.f.N * C};
    const unsigned long long s_do[2] = {(unsigned long long)a.f.DV * 2, (unsigned long long)a.f.H * a.f.DV * 2};
    const unsigned box64[2] = {64u, 64u}, box_do[3] = {64u, 1u, 64u};
    if (!encode_bf16_map(m_st, a.f.states, 2, d_st, s_st, box64) ||
        !encode_bf16_map(m_ds, a.dstates, 2, d_ds, s_st, box64) ||
        !encode_bf16_map(m_du, a.dU, 2, d_du, s_dv, box64) || !encode_bf16_map(m_vt, a.f.Vp, 2, d_vt, s_vt, box64) ||
        !encode_bf16_map(m_do, a.dO, 3, d_do, s_do, box_do))
      return 2;
    if (!set_smem(gdr_bwd_chunk_tc<DK>, Lt::SMEM)) return 3;
    gdr_bwd_chunk_tc<DK><<<static_cast<unsigned>(BHN), 192, Lt::SMEM, st>>>(
        *reinterpret_cast<const CUtensorMap*>(m_st), *reinterpret_cast<const CUtensorMap*>(m_ds),
        *reinterpret_cast<const CUtensorMap*>(m_du), *reinterpret_cast<const CUtensorMap*>(m_do),
        *reinterpret_cast<const CUtensorMap*>(m_vt), (__nv_bfloat16*)a.dW, (__nv_bfloat16*)a.dQh,
        (__nv_bfloat16*)a.dKt, a.dA, a.dgC, a.f.DV, a.f.N, a.f.H, a.f.gvec, a.f.err);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
  }
  dim3 g2(static_cast<unsigned>(a.f.BH * a.f.N), DK / 64);
  gdr_bwd_chunk<<<g2, THREADS, s2, st>>>((const __nv_bfloat16*)a.dU, (const __nv_bfloat16*)a.dO,
                                         (const __nv_bfloat16*)a.f.Vp, (const __nv_bfloat16*)a.f.states,
                                         (const __nv_bfloat16*)a.dstates, (__nv_bfloat16*)a.dW,
                                         (__nv_bfloat16*)a.dQh, (__nv_bfloat16*)a.dKt, a.dA, a.dgC, DK, a.f.DV,
                                         a.f.N, a.f.H, a.f.gvec);
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
