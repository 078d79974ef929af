// Persistent warp-specialised bf16 GEMM for sm_100a on the 5th-generation
// tensor cores.
//
//   C[b] = alpha * op(A[b]) @ op(B[b])^T + beta * S[b]       (mode STORE)
//   C[b] += alpha * op(A[b]) @ op(B[b])^T   (fp32 red.add)    (mode ATOMIC)
//
// A is M x K, B is N x K in the math; each operand may sit in memory either
// K-contiguous ("K-major", the row-major [M][K] / [N][K] tensor) or
// M/N-contiguous ("MN-major", the row-major [K][M] / [K][N] tensor), so the
// three GEMMs of a linear layer (y = x W^T, dx = dy W, dW = dy^T x) all read
// their operands in place without transposes.
//
// One CTA per SM loops over output tiles (128 x BN).  Warp roles:
//   warp 0      TMA producer: 128-byte-swizzled tiles of A and B into a
//               STAGES-deep shared-memory ring (mbarrier full/empty pairs);
//   warp 1      TMEM allocator and MMA issuer: one thread issues
//               tcgen05.mma (M=128, N=BN, K=16) into one of two TMEM
//               accumulators and tcgen05.commit's the smem slot back;
//   warps 2-5   epilogue: tcgen05.ld the accumulator (one TMEM lane = one
//               output row per thread; the load of the next 32 columns is
//               in flight while the current ones are stored), apply
//               alpha/beta/source, store.  Plain bf16 outputs go out through
//               TMA: each warp packs its 32 rows x 32 columns into one of two
//               2 KB shared-memory buffers (64-byte swizzle, conflict-free)
//               and one lane issues a bulk tensor store, so a tile leaves as
//               16 coalesced 2 KB boxes per warp instead of 32-row scattered
//               vector stores; fp32, atomic, source-adding and scatter
//               epilogues store from registers.
// The two accumulators let the epilogue of tile i overlap the main loop of
// tile i+1.  Split-K (mode ATOMIC only) spreads the K range of one tile over
// several work units when there are fewer tiles than SMs (weight gradients).
//
// All waits are bounded (common.cuh); a timeout sets the error word and the
// CTA winds down, releasing its TMEM.
#include "common.cuh"
#include "gemm.h"

#include <algorithm>
#include <type_traits>
#include <cstdio>
#include <cstdlib>
#include <mutex>

namespace vagus {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;            // one 128-byte swizzle row of bf16
constexpr int UMMA_K = 16;
constexpr int NUM_THREADS = 192;  // 6 warps

template <int BN>
struct Cfg {
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;   // two accumulators
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/ + 16384 /*epilogue*/;
};

// Epilogue staging for TMA stores: per epilogue warp two 32 x 32 bf16 boxes.
constexpr int EPI_BOX_BYTES = 32 * 32 * 2;
constexpr int EPI_BYTES = 4 * 2 * EPI_BOX_BYTES;

struct KParams {
  int M, N, K, batch;
  int tiles_m, tiles_n, kb_total;
  int full_tiles, kb_per_split, units;   // see decode_unit
  void* C;
  long long ldc, strideC;
  int c_f32;
  const void* S;
  long long lds, strideS;
  int s_f32;
  float alpha, beta;
  int atomic;
  int vec;          // 16-byte vector access is legal for C and S
  int tma_c;        // plain bf16 output stored through the C tensor map
  int* err;
  // stream-K (atomic outputs, CTA-pair kernel): worker w takes the global
  // k-block range [w * kb_per_worker, (w + 1) * kb_per_worker) of the
  // tiles x kb_total sequence, possibly spanning tiles; partial tiles meet
  // in the atomic epilogue
  int streamk;
  long long kb_per_worker;
  // scatter epilogue (see GemmArgs)
  int scatter, scatter_span, scatter_batch0;
  long long dst_ld, dst_stride;
  void* scatter_dst[16];
};

__device__ __forceinline__ void store_row_chunk(const KParams& p, int b, int row, int col0, const float* v) {
  // v: 32 consecutive values of one output row starting at col0
  if (row >= p.M) return;
  if (!VAGUS_CHECK(b, p.batch) || !VAGUS_CHECK(col0, p.N)) return;
  const bool full = (col0 + 32 <= p.N) && p.vec;
  if (p.atomic) {
    float* c = reinterpret_cast<float*>(p.C) + (long long)b * p.strideC + (long long)row * p.ldc + col0;
    if (full) {
      // 16-byte vector reductions: a quarter of the L2 atomic operations
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        atomicAdd(reinterpret_cast<float4*>(c + j),
                  make_float4(p.alpha * v[j], p.alpha * v[j + 1], p.alpha * v[j + 2], p.alpha * v[j + 3]));
    } else {
      for (int j = 0; j < 32; ++j)
        if (col0 + j < p.N) atomicAdd(c + j, p.alpha * v[j]);
    }
    return;
  }
  float out[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) out[j] = p.alpha * v[j];
  if (p.S != nullptr && p.beta != 0.f) {
    if (p.s_f32) {
      const float* s = reinterpret_cast<const float*>(p.S) + (long long)b * p.strideS + (long long)row * p.lds + col0;
      if (full) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          float4 t = *reinterpret_cast<const float4*>(s + j);
          out[j] += p.beta * t.x; out[j + 1] += p.beta * t.y; out[j + 2] += p.beta * t.z; out[j + 3] += p.beta * t.w;
        }
      } else {
        for (int j = 0; j < 32; ++j) if (col0 + j < p.N) out[j] += p.beta * s[j];
      }
    } else {
      const __nv_bfloat16* s =
          reinterpret_cast<const __nv_bfloat16*>(p.S) + (long long)b * p.strideS + (long long)row * p.lds + col0;
      if (full) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          uint4 t = *reinterpret_cast<const uint4*>(s + j);
          float2 f0 = unpack_bf16x2(t.x), f1 = unpack_bf16x2(t.y), f2 = unpack_bf16x2(t.z), f3 = unpack_bf16x2(t.w);
          out[j] += p.beta * f0.x; out[j + 1] += p.beta * f0.y; out[j + 2] += p.beta * f1.x; out[j + 3] += p.beta * f1.y;
          out[j + 4] += p.beta * f2.x; out[j + 5] += p.beta * f2.y; out[j + 6] += p.beta * f3.x; out[j + 7] += p.beta * f3.y;
        }
      } else {
        for (int j = 0; j < 32; ++j) if (col0 + j < p.N) out[j] += p.beta * bf2f(s[j]);
      }
    }
  }
  if (p.c_f32) {
    float* c = reinterpret_cast<float*>(p.C) + (long long)b * p.strideC + (long long)row * p.ldc + col0;
    if (full) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(c + j) = make_float4(out[j], out[j + 1], out[j + 2], out[j + 3]);
    } else {
      for (int j = 0; j < 32; ++j) if (col0 + j < p.N) c[j] = out[j];
    }
  } else {
    __nv_bfloat16* c;
    if (p.scatter == 1) {
      const int o = row / p.scatter_span;
      c = reinterpret_cast<__nv_bfloat16*>(p.scatter_dst[o]) + (long long)(p.scatter_batch0 + b) * p.dst_stride +
          (long long)(row - o * p.scatter_span) * p.dst_ld + col0;
    } else if (p.scatter == 2) {
      const int o = col0 / p.scatter_span;       // span % 32 == 0: one owner per 32-column chunk
      c = reinterpret_cast<__nv_bfloat16*>(p.scatter_dst[o]) + (long long)(p.scatter_batch0 + b) * p.dst_stride +
          (long long)row * p.dst_ld + (col0 - o * p.scatter_span);
    } else {
      c = reinterpret_cast<__nv_bfloat16*>(p.C) + (long long)b * p.strideC + (long long)row * p.ldc + col0;
    }
    if (full) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 t;
        t.x = pack_bf16x2(out[j], out[j + 1]); t.y = pack_bf16x2(out[j + 2], out[j + 3]);
        t.z = pack_bf16x2(out[j + 4], out[j + 5]); t.w = pack_bf16x2(out[j + 6], out[j + 7]);
        *reinterpret_cast<uint4*>(c + j) = t;
      }
    } else {
      for (int j = 0; j < 32; ++j) if (col0 + j < p.N) c[j] = f2bf(out[j]);
    }
  }
}

// One 32-column chunk of one epilogue warp's 32 rows (v: this thread's row).
// TMA mode: pack to bf16 into the warp's next staging box -- row `lane` at
// byte lane * 64, 16-byte group q stored at q ^ ((lane >> 1) & 3), which is
// the tensor map's 64-byte swizzle and spreads a phase's 8 rows over all
// banks -- then one lane stores the box at (col0, warp_row0, b).  The box
// written two chunks ago must have been read out first (bulk_wait_read<1>).
__device__ __forceinline__ void emit_chunk(const KParams& p, const CUtensorMap* mapC, uint8_t* wbuf, int& sel, int b,
                                           int row, int warp_row0, int col0, const uint32_t (&r)[32], int lane) {
  const float* v = reinterpret_cast<const float*>(r);
  if (!p.tma_c) {
    if (col0 < p.N) store_row_chunk(p, b, row, col0, v);
    return;
  }
  if (col0 >= p.N) return;                 // warp-uniform
  uint8_t* box = wbuf + sel * EPI_BOX_BYTES;
  if (lane == 0) bulk_wait_read<1>();
  __syncwarp();
  uint32_t w[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) w[j] = pack_bf16x2(p.alpha * v[2 * j], p.alpha * v[2 * j + 1]);
  uint4* dst = reinterpret_cast<uint4*>(box + lane * 64);
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int q = 0; q < 4; ++q) dst[q ^ sw] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_3d(mapC, box, col0, warp_row0, b);
    bulk_commit();
  }
  sel ^= 1;
}

// Drains one epilogue warp's 32 accumulator rows of a tile (NCOL columns from
// TMEM address t_row): the tcgen05.ld of the next 32 columns is issued before
// the current ones are converted and stored.
template <int NCOL>
__device__ __forceinline__ void drain_rows(const KParams& p, const CUtensorMap* mapC, uint8_t* wbuf, int& sel, int b,
                                           int row, int warp_row0, int n0, uint32_t t_row, int lane) {
  uint32_t ra[32], rb[32];
  tmem_ld_32x32b_x32(t_row, ra);
#pragma unroll
  for (int c = 0; c < NCOL; c += 64) {
    tmem_ld_wait();
    tmem_regs_ready(ra);
    if (c + 32 < NCOL) tmem_ld_32x32b_x32(t_row + c + 32, rb);
    emit_chunk(p, mapC, wbuf, sel, b, row, warp_row0, n0 + c, ra, lane);
    if (c + 32 < NCOL) {
      tmem_ld_wait();
      tmem_regs_ready(rb);
      if (c + 64 < NCOL) tmem_ld_32x32b_x32(t_row + c + 64, ra);
      emit_chunk(p, mapC, wbuf, sel, b, row, warp_row0, n0 + c + 32, rb, lane);
    }
  }
}

// Work units.  The first `full_tiles` units are whole tiles (all of K); the
// remaining tiles (fewer than one wave) are split `rsplit` ways along K so
// the last wave fills the machine, and their partial products meet in the
// atomic epilogue.  Within the split part the split index varies slowest:
// CTAs running at the same time cover the same K range of neighbouring
// tiles, so the operand panels they share are read from L2 once.
__device__ __forceinline__ void decode_unit(const KParams& p, int u, int& b, int& tm, int& tn, int& kb0, int& kb1) {
  int t;
  if (u < p.full_tiles) {
    t = u;
    kb0 = 0;
    kb1 = p.kb_total;
  } else {
    const int rem = p.batch * p.tiles_m * p.tiles_n - p.full_tiles;
    const int v = u - p.full_tiles;
    const int sp = v / rem;
    t = p.full_tiles + (v - sp * rem);
    kb0 = sp * p.kb_per_split;
    kb1 = min(p.kb_total, kb0 + p.kb_per_split);
  }
  const int per_batch = p.tiles_m * p.tiles_n;
  b = t / per_batch;
  t -= b * per_batch;
  tm = t / p.tiles_n;
  tn = t - tm * p.tiles_n;
}

// Work iterator shared by the three roles: strided units (tile, split), or a
// contiguous stream-K range of k-blocks cut at tile boundaries.
struct WorkIter {
  long long g = 0, end = 0;
  int u = 0, step = 1;
  __device__ WorkIter(const KParams& p, int worker, int nworkers) {
    if (p.streamk) {
      const long long total = (long long)p.batch * p.tiles_m * p.tiles_n * p.kb_total;
      g = (long long)worker * p.kb_per_worker;
      end = g + p.kb_per_worker < total ? g + p.kb_per_worker : total;
    } else {
      u = worker;
      step = nworkers;
    }
  }
  __device__ bool next(const KParams& p, int& b, int& tm, int& tn, int& kb0, int& kb1) {
    if (p.streamk) {
      if (g >= end) return false;
      const int t = static_cast<int>(g / p.kb_total);
      kb0 = static_cast<int>(g - (long long)t * p.kb_total);
      const long long left = end - g;
      kb1 = left < p.kb_total - kb0 ? kb0 + static_cast<int>(left) : p.kb_total;
      g += kb1 - kb0;
      const int per_batch = p.tiles_m * p.tiles_n;
      b = t / per_batch;
      const int r = t - b * per_batch;
      tm = r / p.tiles_n;
      tn = r - tm * p.tiles_n;
      return true;
    }
    if (u >= p.units) return false;
    decode_unit(p, u, b, tm, tn, kb0, kb1);
    u += step;
    return true;
  }
};

// Per-owner tensor maps of a gathered B operand (GemmArgs::gather_*): a
// BN-row box map and an 8-row box map over each owner's rows.
constexpr int kMaxGather = 8;
struct GatherMaps {
  CUtensorMap coarse[kMaxGather];
  CUtensorMap fine[kMaxGather];
  int rows, owners;
};
struct NoGather {};

template <int BN, bool A_MN, bool B_MN, class GM = NoGather>
__global__ void __launch_bounds__(NUM_THREADS, 1)
gemm_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
            const __grid_constant__ CUtensorMap mapC, const KParams p, const __grid_constant__ GM gm) {
  constexpr bool kGather = std::is_same<GM, GatherMaps>::value;
  using C = Cfg<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzle atoms
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;
  uint8_t* epi = smem + C::STAGES * C::STAGE_BYTES;          // 1024-aligned
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(epi + EPI_BYTES);
  uint64_t* empty_bar = full_bar + C::STAGES;
  uint64_t* acc_full = empty_bar + C::STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 128);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&mapA);
    tma_prefetch_desc(&mapB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      WorkIter it(p, blockIdx.x, gridDim.x);
      int b, tm, tn, kb0, kb1;
      while (ok && it.next(p, b, tm, tn, kb0, kb1)) {
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, p.err, kErrTimeoutProducer)) { ok = false; break; }
          uint8_t* sa = tiles + stage * C::STAGE_BYTES;
          uint8_t* sb = sa + C::A_BYTES;
          const int k0 = kb * BK;
          // MN-major operands arrive as 64-wide blocks; a block that starts
          // past the end of M / N is not loaded (its rows only feed output
          // rows the epilogue masks), and the byte count says so.
          int a_blocks = BM / 64, b_blocks = BN / 64;
          if (A_MN) a_blocks = min(a_blocks, (p.M - tm * BM + 63) / 64);
          if (B_MN) b_blocks = min(b_blocks, (p.N - tn * BN + 63) / 64);
          const uint32_t tx = (A_MN ? a_blocks * 8192 : C::A_BYTES) + (B_MN ? b_blocks * 8192 : C::B_BYTES);
          mbar_arrive_expect_tx(&full_bar[stage], tx);
          if (A_MN) {
            for (int j = 0; j < a_blocks; ++j) tma_load_3d(sa + j * 8192, &mapA, &full_bar[stage], tm * BM + 64 * j, k0, b);
          } else {
            tma_load_3d(sa, &mapA, &full_bar[stage], k0, tm * BM, b);
          }
          if constexpr (kGather) {
            // the tile's B rows from their owners: one box when they lie in
            // one owner's rows (or in the last owner's, whose rows past its
            // end only feed masked output columns), else 8-row boxes, each
            // from the owner of its rows (owner boundaries are multiples of 8)
            const int n0 = tn * BN;
            const int o = min(n0 / gm.rows, gm.owners - 1);
            if (n0 + BN <= (o + 1) * gm.rows || o == gm.owners - 1) {
              tma_load_3d(sb, &gm.coarse[o], &full_bar[stage], k0, n0 - o * gm.rows, 0);
            } else {
              for (int r = 0; r < BN / 8; ++r) {
                const int g = n0 + 8 * r;
                const int og = min(g / gm.rows, gm.owners - 1);
                tma_load_3d(sb + r * 1024, &gm.fine[og], &full_bar[stage], k0, g - og * gm.rows, 0);
              }
            }
          } else if (B_MN) {
            for (int j = 0; j < b_blocks; ++j) tma_load_3d(sb + j * 8192, &mapB, &full_bar[stage], tn * BN + 64 * j, k0, b);
          } else {
            tma_load_3d(sb, &mapB, &full_bar[stage], k0, tn * BN, b);
          }
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      WorkIter it(p, blockIdx.x, gridDim.x);
      int b, tm, tn, kb0, kb1;
      for (; ok && it.next(p, b, tm, tn, kb0, kb1); ++local) {
        const int buf = local & 1;
        const uint32_t use = static_cast<uint32_t>(local >> 1);
        if (!mbar_wait(&acc_empty[buf], (use & 1) ^ 1, abort_flag, p.err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, p.err, kErrTimeoutMma)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(tiles + stage * C::STAGE_BYTES);
          const uint32_t b_addr = a_addr + C::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            // K-major: next 16 columns are 32 bytes further along the swizzled row.
            // MN-major: next 16 K-rows are 16 * 128 bytes further down.
            const uint64_t ad = A_MN ? make_sw128_desc(a_addr + kk * 2048, 8192, 1024)
                                     : make_sw128_desc(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? make_sw128_desc(b_addr + kk * 2048, 8192, 1024)
                                     : make_sw128_desc(b_addr + kk * 32, 16, 1024);
            tc_mma_f16(d_tmem, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&empty_bar[stage]);
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit(&acc_full[buf]);
      }
      // let every MMA this thread issued retire before TMEM is released
      tc_commit(drain_bar);
      mbar_wait(drain_bar, 0, abort_flag, p.err, kErrTimeoutMma);
    }
  } else {
    // ----------------------------------------------------------- epilogue
    const int quarter = warp & 3;              // TMEM lane quarter this warp may touch
    const int row_in_tile = quarter * 32 + lane;
    uint8_t* wbuf = epi + quarter * 2 * EPI_BOX_BYTES;
    int sel = 0;
    int local = 0;
    WorkIter it(p, blockIdx.x, gridDim.x);
    int b, tm, tn, kb0, kb1;
    for (; it.next(p, b, tm, tn, kb0, kb1); ++local) {
      const int buf = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1);
      if (!mbar_wait(&acc_full[buf], use & 1, abort_flag, p.err, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(buf * BN);
      drain_rows<BN>(p, &mapC, wbuf, sel, b, tm * BM + row_in_tile, tm * BM + quarter * 32, tn * BN, t_row, lane);
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
    if (p.tma_c && lane == 0) bulk_wait<0>();   // stores out of this warp's boxes are complete
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------- CTA-pair kernel --
// Same roles as above on a cluster of two CTAs (neighbouring SMs) that share
// 256 x 256 output tiles through tcgen05.mma.cta_group::2 (M = 256, N = 256,
// K = 16): CTA r of the pair loads A rows [128 r, 128 r + 128) and B columns
// [128 r, 128 r + 128) of the tile and owns accumulator rows
// [128 r, 128 r + 128) in its TMEM.  Per CTA and k-step that is 32 KB of
// operands for a 128 x 256 x 64 share of the product (48 KB in the one-CTA
// kernel), which is what keeps the tensor pipe fed from L2.
//   * full barriers live in CTA 0: its producer expects both CTAs' bytes and
//     the peer's loads complete on CTA 0's barrier (.cta_group::2 loads);
//   * CTA 0's MMA thread issues everything and commits each stage back to
//     the empty barriers of both CTAs, and each finished tile to both CTAs'
//     accumulator-full barriers (one commit per CTA, no broadcast form);
//   * both CTAs' epilogue warps arrive on CTA 0's accumulator-empty barriers.
namespace pairk {
constexpr int ROWS = 128;                 // rows of A / columns of B per CTA
constexpr int TM = 256, TN = 256;         // pair tile
constexpr int STAGES = 6;
constexpr int A_BYTES = ROWS * BK * 2;
constexpr int B_BYTES = ROWS * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 2 * TN;         // two accumulators (all 512 columns)
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256 + EPI_BYTES;
}  // namespace pairk

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
gemm_pair_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                 const __grid_constant__ CUtensorMap mapC, const KParams p) {
  using namespace pairk;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;
  uint8_t* epi = smem + STAGES * STAGE_BYTES;                // 1024-aligned
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(epi + EPI_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* acc_full = empty_bar + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);         // 4 epilogue warps x 2 CTAs
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&mapA);
    tma_prefetch_desc(&mapB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();                           // barriers of both CTAs initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      WorkIter it(p, cluster, nclusters);
      int b, tm, tn, kb0, kb1;
      while (ok && it.next(p, b, tm, tn, kb0, kb1)) {
        // 64-wide MN-major blocks that start past M / N are not loaded (their
        // rows only feed masked output); both CTAs' counts go to CTA 0's barrier
        int a_blk[2], b_blk[2];
        for (int r = 0; r < 2; ++r) {
          a_blk[r] = A_MN ? max(0, min(ROWS / 64, (p.M - tm * TM - r * ROWS + 63) / 64)) : ROWS / 64;
          b_blk[r] = B_MN ? max(0, min(ROWS / 64, (p.N - tn * TN - r * ROWS + 63) / 64)) : ROWS / 64;
        }
        const uint32_t tx = (a_blk[0] + a_blk[1] + b_blk[0] + b_blk[1]) * 8192;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, p.err, kErrTimeoutProducer)) { ok = false; break; }
          uint8_t* sa = tiles + stage * STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          const uint32_t fb = mapa_shared(smem_u32(&full_bar[stage]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], tx);
          const int k0 = kb * BK;
          const int m0 = tm * TM + (int)rank * ROWS, n0 = tn * TN + (int)rank * ROWS;
          if (A_MN) {
            for (int j = 0; j < a_blk[rank]; ++j) tma_load_3d_pair(sa + j * 8192, &mapA, fb, m0 + 64 * j, k0, b);
          } else {
            tma_load_3d_pair(sa, &mapA, fb, k0, m0, b);
          }
          if (B_MN) {
            for (int j = 0; j < b_blk[rank]; ++j) tma_load_3d_pair(sb + j * 8192, &mapB, fb, n0 + 64 * j, k0, b);
          } else {
            tma_load_3d_pair(sb, &mapB, fb, k0, n0, b);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA (CTA 0 of the pair)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(TM, TN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      WorkIter it(p, cluster, nclusters);
      int b, tm, tn, kb0, kb1;
      for (; ok && it.next(p, b, tm, tn, kb0, kb1); ++local) {
        const int buf = local & 1;
        const uint32_t use = static_cast<uint32_t>(local >> 1);
        if (!mbar_wait(&acc_empty[buf], (use & 1) ^ 1, abort_flag, p.err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * TN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, p.err, kErrTimeoutMma)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(tiles + stage * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            const uint64_t ad = A_MN ? make_sw128_desc(a_addr + kk * 2048, 8192, 1024)
                                     : make_sw128_desc(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? make_sw128_desc(b_addr + kk * 2048, 8192, 1024)
                                     : make_sw128_desc(b_addr + kk * 32, 16, 1024);
            tc_mma_f16_pair(d_tmem, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          const uint32_t e = smem_u32(&empty_bar[stage]);
          tc_commit_pair(mapa_shared(e, 0));
          tc_commit_pair(mapa_shared(e, 1));
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        const uint32_t f = smem_u32(&acc_full[buf]);
        tc_commit_pair(mapa_shared(f, 0));
        tc_commit_pair(mapa_shared(f, 1));
      }
      tc_commit_pair(mapa_shared(smem_u32(drain_bar), 0));
      mbar_wait(drain_bar, 0, abort_flag, p.err, kErrTimeoutMma);
    }
  } else {
    // ----------------------------------------------------------- epilogue
    const int quarter = warp & 3;
    const int warp_row = (int)rank * ROWS + quarter * 32;
    uint8_t* wbuf = epi + quarter * 2 * EPI_BOX_BYTES;
    int sel = 0;
    int local = 0;
    WorkIter it(p, cluster, nclusters);
    int b, tm, tn, kb0, kb1;
    for (; it.next(p, b, tm, tn, kb0, kb1); ++local) {
      const int buf = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1);
      if (!mbar_wait(&acc_full[buf], use & 1, abort_flag, p.err, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(buf * TN);
      drain_rows<TN>(p, &mapC, wbuf, sel, b, tm * TM + warp_row + lane, tm * TM + warp_row, tn * TN, t_row, lane);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[buf]), 0));
    }
    if (p.tma_c && lane == 0) bulk_wait<0>();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();                           // the peer's TMEM and smem stay valid until CTA 0 has drained
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host --

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn get_encode() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    if (std::getenv("VAGUS_GEMM_DEBUG"))
      std::fprintf(stderr, "[gemm] entry point rc %d status %d ptr %p\n", (int)e, (int)q, ptr);
    if (e == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<EncodeFn>(ptr);
  });
  return fn;
}

// 3-D bf16 tensor map: (inner, rows, batch) with a (64, box_rows, 1) box.
bool make_map(CUtensorMap* map, const void* base, long long inner, long long rows, long long batch, long long ld,
              long long bstride, int box_rows) {
  EncodeFn enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)rows, (cuuint64_t)batch};
  // a single matrix still needs a legal (16-byte multiple) batch stride
  if (batch <= 1 || bstride <= 0) bstride = ld * rows;
  cuuint64_t strides[2] = {(cuuint64_t)(ld * 2), (cuuint64_t)(bstride * 2)};
  cuuint32_t box[3] = {64u, (cuuint32_t)box_rows, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  if (std::getenv("VAGUS_GEMM_DEBUG"))
    std::fprintf(stderr, "[gemm] map %p base %p dims %llu %llu %llu strides %llu %llu box %u %u\n", (void*)map, base,
                 (unsigned long long)dims[0], (unsigned long long)dims[1], (unsigned long long)dims[2],
                 (unsigned long long)strides[0], (unsigned long long)strides[1], box[0], box[1]);
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (std::getenv("VAGUS_GEMM_DEBUG")) std::fprintf(stderr, "[gemm] encode -> %d\n", (int)r);
  return r == CUDA_SUCCESS;
}

// C tensor map for the TMA-store epilogue: bf16 (N, M, batch), 32 x 32 boxes,
// 64-byte swizzle.  False (register stores instead) when the output is not a
// plain bf16 store, breaks the TMA rules (16-byte base / pitches), is smaller
// than a box, or VAGUS_GEMM_NO_TMA_STORE is set.
bool make_c_map(CUtensorMap* map, const GemmArgs& a) {
  static const bool off = std::getenv("VAGUS_GEMM_NO_TMA_STORE") != nullptr;
  if (off || a.atomic || a.c_f32 || a.scatter || (a.S != nullptr && a.beta != 0.f)) return false;
  if ((reinterpret_cast<uintptr_t>(a.C) & 15u) || (a.ldc % 8) || (a.batch > 1 && a.strideC % 8)) return false;
  if (a.N < 32 || a.M < 32 || a.ldc < a.N) return false;
  EncodeFn enc = get_encode();
  if (!enc) return false;
  const long long bstride = a.batch > 1 ? a.strideC : a.ldc * a.M;
  cuuint64_t dims[3] = {(cuuint64_t)a.N, (cuuint64_t)a.M, (cuuint64_t)a.batch};
  cuuint64_t strides[2] = {(cuuint64_t)(a.ldc * 2), (cuuint64_t)(bstride * 2)};
  cuuint32_t box[3] = {32u, 32u, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, a.C, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

// Unit plan (see decode_unit): whole tiles for every complete wave, then the
// leftover tiles split along K so that they cover the workers about once
// (atomic outputs only; each split keeps at least 8 k-blocks).  `split_k` > 1
// forces that many splits of every tile.
void plan_units(KParams& p, int tiles, int workers, bool atomic, int split_k) {
  if (atomic && split_k > 1) {
    p.full_tiles = 0;
    p.kb_per_split = (p.kb_total + split_k - 1) / split_k;
  } else if (atomic && split_k != 1) {
    p.full_tiles = (tiles / workers) * workers;
    const int rem = tiles - p.full_tiles;
    // smallest split (at most 8) minimising the makespan ceil(rem * rs / workers) / rs
    int rs = 1;
    double best = 1e30;
    for (int c = 1; rem > 0 && c <= 8 && p.kb_total / c >= 8; ++c) {
      const double t = static_cast<double>((rem * c + workers - 1) / workers) / c;
      if (t < best - 1e-9) { best = t; rs = c; }
    }
    p.kb_per_split = (p.kb_total + rs - 1) / rs;
  } else {
    p.full_tiles = tiles;
    p.kb_per_split = p.kb_total;
  }
  const int rem = tiles - p.full_tiles;
  const int rsplit = rem > 0 ? (p.kb_total + p.kb_per_split - 1) / p.kb_per_split : 0;
  p.units = p.full_tiles + rem * rsplit;
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

bool fill_scatter(KParams& p, const GemmArgs& a);

template <int BN, bool A_MN, bool B_MN, class GM = NoGather>
int launch_t(const GemmArgs& a, cudaStream_t stream) {
  using C = Cfg<BN>;
  constexpr bool kGather = std::is_same<GM, GatherMaps>::value;
  CUtensorMap ma, mb;
  GM gm{};
  // A: K-major -> (K, M) rows of K; MN-major -> (M, K) rows of M.
  bool ok = A_MN ? make_map(&ma, a.A, a.M, a.K, a.batch, a.lda, a.strideA, 64)
                 : make_map(&ma, a.A, a.K, a.M, a.batch, a.lda, a.strideA, BM);
  if constexpr (kGather) {
    gm.rows = a.gather_rows;
    gm.owners = a.gather_n;
    for (int o = 0; ok && o < a.gather_n; ++o)
      ok = make_map(&gm.coarse[o], a.gather_src[o], a.K, a.gather_rows, 1, a.ldb, 0, BN) &&
           make_map(&gm.fine[o], a.gather_src[o], a.K, a.gather_rows, 1, a.ldb, 0, 8);
    mb = gm.coarse[0];                       // unused by the gathering kernel
  } else {
    ok = ok && (B_MN ? make_map(&mb, a.B, a.N, a.K, a.batch, a.ldb, a.strideB, 64)
                     : make_map(&mb, a.B, a.K, a.N, a.batch, a.ldb, a.strideB, BN));
  }
  if (!ok) return 2;
  KParams p;
  p.M = a.M; p.N = a.N; p.K = a.K; p.batch = a.batch;
  p.tiles_m = (a.M + BM - 1) / BM;
  p.tiles_n = (a.N + BN - 1) / BN;
  p.kb_total = (a.K + BK - 1) / BK;
  const int tiles = p.tiles_m * p.tiles_n * a.batch;
  plan_units(p, tiles, num_sms(), a.atomic != 0, a.split_k);
  p.C = a.C; p.ldc = a.ldc; p.strideC = a.strideC; p.c_f32 = a.c_f32;
  p.S = a.S; p.lds = a.lds; p.strideS = a.strideS; p.s_f32 = a.s_f32;
  p.alpha = a.alpha; p.beta = a.beta; p.atomic = a.atomic; p.err = a.err;
  p.streamk = 0;
  p.kb_per_worker = 0;
  {
    const int ce = a.c_f32 ? 4 : 2, se = a.s_f32 ? 4 : 2;
    bool v = (reinterpret_cast<uintptr_t>(a.C) % 16 == 0) && ((a.ldc * ce) % 16 == 0) && ((a.strideC * ce) % 16 == 0);
    if (a.S) v = v && (reinterpret_cast<uintptr_t>(a.S) % 16 == 0) && ((a.lds * se) % 16 == 0) && ((a.strideS * se) % 16 == 0);
    p.vec = v ? 1 : 0;
  }
  if (!fill_scatter(p, a)) return 5;
  CUtensorMap mc = ma;                     // a valid map either way; read only when tma_c
  p.tma_c = make_c_map(&mc, a) ? 1 : 0;
  const int grid = std::min(p.units, num_sms());
  auto kern = gemm_kernel<BN, A_MN, B_MN, GM>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES) != cudaSuccess) return 3;
    attr_set[dev] = true;
  }
  if (std::getenv("VAGUS_GEMM_DEBUG"))
    std::fprintf(stderr, "[gemm] launch grid %d smem %d M %d N %d K %d units %d\n", grid, C::SMEM_BYTES, a.M, a.N,
                 a.K, p.units);
  kern<<<grid, NUM_THREADS, C::SMEM_BYTES, stream>>>(ma, mb, mc, p, gm);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

// Scatter-epilogue fields and the 16-byte vector rule for the destinations;
// false when the request is malformed.
bool fill_scatter(KParams& p, const GemmArgs& a) {
  p.scatter = a.scatter;
  p.scatter_span = a.scatter_span;
  p.scatter_batch0 = a.scatter_batch0;
  p.dst_ld = a.dst_ld;
  p.dst_stride = a.dst_stride;
  for (int i = 0; i < 16; ++i) p.scatter_dst[i] = i < a.scatter_n ? a.scatter_dst[i] : nullptr;
  if (!a.scatter) return true;
  if (a.scatter != 1 && a.scatter != 2) return false;
  if (a.c_f32 || a.atomic || a.scatter_span <= 0 || a.scatter_n < 1 || a.scatter_n > 16) return false;
  const int extent = a.scatter == 1 ? a.M : a.N;
  if ((extent + a.scatter_span - 1) / a.scatter_span > a.scatter_n) return false;
  if (a.scatter == 2 && a.scatter_span % 32) return false;
  bool v = (a.dst_ld * 2) % 16 == 0 && (a.dst_stride * 2) % 16 == 0;
  for (int i = 0; i < a.scatter_n; ++i) {
    if (!a.scatter_dst[i]) return false;
    v = v && reinterpret_cast<uintptr_t>(a.scatter_dst[i]) % 16 == 0;
  }
  if (a.scatter == 2) v = v && (a.scatter_span * 2) % 16 == 0;
  if (!v) p.vec = 0;
  return true;
}

template <bool A_MN, bool B_MN>
int launch_pair(const GemmArgs& a, cudaStream_t stream) {
  using namespace pairk;
  CUtensorMap ma, mb;
  bool ok = A_MN ? make_map(&ma, a.A, a.M, a.K, a.batch, a.lda, a.strideA, 64)
                 : make_map(&ma, a.A, a.K, a.M, a.batch, a.lda, a.strideA, ROWS);
  ok = ok && (B_MN ? make_map(&mb, a.B, a.N, a.K, a.batch, a.ldb, a.strideB, 64)
                   : make_map(&mb, a.B, a.K, a.N, a.batch, a.ldb, a.strideB, ROWS));
  if (!ok) return 2;
  KParams p;
  p.M = a.M; p.N = a.N; p.K = a.K; p.batch = a.batch;
  p.tiles_m = (a.M + TM - 1) / TM;
  p.tiles_n = (a.N + TN - 1) / TN;
  p.kb_total = (a.K + BK - 1) / BK;
  const int clusters_max = num_sms() / 2;
  const int tiles = p.tiles_m * p.tiles_n * a.batch;
  plan_units(p, tiles, clusters_max, a.atomic != 0, a.split_k == -1 ? 1 : a.split_k);
  p.C = a.C; p.ldc = a.ldc; p.strideC = a.strideC; p.c_f32 = a.c_f32;
  p.S = a.S; p.lds = a.lds; p.strideS = a.strideS; p.s_f32 = a.s_f32;
  p.alpha = a.alpha; p.beta = a.beta; p.atomic = a.atomic; p.err = a.err;
  {
    const int ce = a.c_f32 ? 4 : 2, se = a.s_f32 ? 4 : 2;
    bool v = (reinterpret_cast<uintptr_t>(a.C) % 16 == 0) && ((a.ldc * ce) % 16 == 0) && ((a.strideC * ce) % 16 == 0);
    if (a.S) v = v && (reinterpret_cast<uintptr_t>(a.S) % 16 == 0) && ((a.lds * se) % 16 == 0) && ((a.strideS * se) % 16 == 0);
    p.vec = v ? 1 : 0;
  }
  if (!fill_scatter(p, a)) return 5;
  CUtensorMap mc = ma;
  p.tma_c = make_c_map(&mc, a) ? 1 : 0;
  int units = p.units;
  p.streamk = 0;
  p.kb_per_worker = 0;
  if (a.atomic && a.split_k == -1) {
    // stream-K (opt-in: split_k = -1): every pair gets the same number of
    // k-blocks (at least 8).  Slower than split-K on long-K weight gradients
    // here: pairs at different K offsets of one panel lose the L2 sharing.
    const long long total = (long long)tiles * p.kb_total;
    const long long workers = std::max<long long>(1, std::min<long long>(clusters_max, total / 8));
    p.streamk = 1;
    p.kb_per_worker = (total + workers - 1) / workers;
    units = static_cast<int>((total + p.kb_per_worker - 1) / p.kb_per_worker);
  }
  const int clusters = std::min(units, clusters_max);
  auto kern = gemm_pair_kernel<A_MN, B_MN>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess) return 3;
    attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * clusters), 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (std::getenv("VAGUS_GEMM_DEBUG"))
    std::fprintf(stderr, "[gemm] pair launch clusters %d smem %d M %d N %d K %d units %d\n", clusters, SMEM_BYTES,
                 a.M, a.N, a.K, units);
  if (cudaLaunchKernelEx(&cfg, kern, ma, mb, mc, p) != cudaSuccess) return 3;
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int dispatch_pair(const GemmArgs& a, cudaStream_t s) {
  if (!a.a_mn && !a.b_mn) return launch_pair<false, false>(a, s);
  if (!a.a_mn && a.b_mn) return launch_pair<false, true>(a, s);
  if (a.a_mn && !a.b_mn) return launch_pair<true, false>(a, s);
  return launch_pair<true, true>(a, s);
}

template <int BN>
int dispatch_major(const GemmArgs& a, cudaStream_t s) {
  if (!a.a_mn && !a.b_mn) return launch_t<BN, false, false>(a, s);
  if (!a.a_mn && a.b_mn) return launch_t<BN, false, true>(a, s);
  if (a.a_mn && !a.b_mn) return launch_t<BN, true, false>(a, s);
  return launch_t<BN, true, true>(a, s);
}

}  // namespace

bool encode_bf16_map(void* map, const void* base, int rank, const unsigned long long* dims,
                     const unsigned long long* strides, const unsigned* box) {
  EncodeFn enc = get_encode();
  if (!enc || rank < 2 || rank > 5) return false;
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) { d[i] = dims[i]; bx[i] = box[i]; es[i] = 1; }
  for (int i = 0; i < rank - 1; ++i) st[i] = strides[i];
  return enc(reinterpret_cast<CUtensorMap*>(map), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), d,
             st, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_f32_map(void* map, const void* base, int rank, const unsigned long long* dims,
                    const unsigned long long* strides, const unsigned* box, bool swizzle128) {
  EncodeFn enc = get_encode();
  if (!enc || rank < 2 || rank > 5) return false;
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) { d[i] = dims[i]; bx[i] = box[i]; es[i] = 1; }
  for (int i = 0; i < rank - 1; ++i) st[i] = strides[i];
  return enc(reinterpret_cast<CUtensorMap*>(map), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank, const_cast<void*>(base), d,
             st, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
             swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int gemm_launch(const GemmArgs& a, cudaStream_t stream) {
  if (a.M <= 0 || a.N <= 0 || a.batch <= 0) return 0;
  if (a.K <= 0) return 4;
  if (a.gather_n > 0) {
    // gathered B: K-major, one matrix, one-CTA tiles no wider than an owner's rows
    if (a.gather_n > kMaxGather || a.b_mn || a.batch != 1 || a.gather_rows < 128 || a.gather_rows % 8 ||
        (long long)a.gather_n * a.gather_rows < a.N || a.K < 64 || (a.ldb % 8) || a.ldb < a.K)
      return 7;
    for (int o = 0; o < a.gather_n; ++o)
      if (!a.gather_src[o] || (reinterpret_cast<uintptr_t>(a.gather_src[o]) & 15u)) return 1;
    if ((reinterpret_cast<uintptr_t>(a.A) & 15u) || (a.lda % 8)) return 1;
    const long long a_inner = a.a_mn ? a.M : a.K, a_rows = a.a_mn ? a.K : a.M;
    if (a_inner < 64 || a_rows < (a.a_mn ? 64 : BM)) return 6;
    const int bn = (a.block_n == 128 || a.gather_rows < 256 || a.N < 256) ? 128 : 256;
    if (a.a_mn)
      return bn == 128 ? launch_t<128, true, false, GatherMaps>(a, stream) : launch_t<256, true, false, GatherMaps>(a, stream);
    return bn == 128 ? launch_t<128, false, false, GatherMaps>(a, stream) : launch_t<256, false, false, GatherMaps>(a, stream);
  }
  // TMA: base 16-byte aligned, row pitch a multiple of 16 bytes
  auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!aligned(a.A) || !aligned(a.B) || (a.lda % 8) || (a.ldb % 8)) return 1;
  if (a.batch > 1 && ((a.strideA % 8) || (a.strideB % 8))) return 1;
  // block_n: 0 = automatic (CTA pairs with 256 x 256 tiles when M and N
  // reach 256, unless VAGUS_GEMM_NO_PAIR is set), 128 / 256 = one-CTA tiles
  // of that width, 512 = CTA pairs.
  static const bool no_pair = std::getenv("VAGUS_GEMM_NO_PAIR") != nullptr;
  const bool pair = a.block_n == 512 || (a.block_n == 0 && !no_pair && a.M >= 256 && a.N >= 256);
  const int bn = pair ? 128 : (a.block_n > 0 ? a.block_n : (a.N < 256 ? 128 : 256));
  // Every TMA box must fit inside its tensor (the tensor-map encoder does not
  // reject an oversized box reliably); callers route smaller problems elsewhere.
  const long long a_inner = a.a_mn ? a.M : a.K, a_rows = a.a_mn ? a.K : a.M;
  const long long b_inner = a.b_mn ? a.N : a.K, b_rows = a.b_mn ? a.K : a.N;
  const long long a_box = a.a_mn ? 64 : BM, b_box = a.b_mn ? 64 : bn;
  if (a_inner < 64 || a_rows < a_box || b_inner < 64 || b_rows < b_box) return 6;
  if (pair) return dispatch_pair(a, stream);
  return bn == 128 ? dispatch_major<128>(a, stream) : dispatch_major<256>(a, stream);
}

}  // namespace vagus
