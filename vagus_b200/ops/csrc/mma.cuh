// Warp-level bf16 tensor-core helpers (mma.sync m16n8k16 with ldmatrix
// fragment loads from padded shared-memory tiles) and cp.async tile copies,
// shared by the chunked gated delta-rule kernels.  These serve the small
// per-chunk products (64 x 64 x {64, 256}) whose operands live in shared
// memory next to scalar work; the large projection GEMMs use tcgen05.
#pragma once
#include "common.cuh"

namespace vagus {
namespace mma {

constexpr int PAD = 8;       // bf16 elements of row padding (16 bytes): conflict-free ldmatrix


__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void ldsm4t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

// Warp-level D[MT*16 x NT*8] += A[M x K] B[K x N] over k in [0, K).
//   A_T = false: A stored [m][k] (pitch lda);  true: stored [k][m].
//   B_T = false: B stored [n][k] (pitch ldb);  true: stored [k][n].
template <int MT, int NT, bool A_T, bool B_T>
__device__ __forceinline__ void warp_mma(float (&acc)[MT][NT][4], const __nv_bfloat16* As, int lda,
                                         const __nv_bfloat16* Bs, int ldb, int m0, int n0, int K) {
  static_assert(NT % 2 == 0, "NT must be even");
  const int l = threadIdx.x & 31;
  const int j = l >> 3, r8 = l & 7;
  for (int k0 = 0; k0 < K; k0 += 16) {
    uint32_t a[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int mb = m0 + mt * 16;
      if (!A_T) ldsm4(a[mt], As + (mb + r8 + (j & 1) * 8) * lda + k0 + (j >> 1) * 8);
      else ldsm4t(a[mt], As + (k0 + r8 + (j >> 1) * 8) * lda + mb + (j & 1) * 8);
    }
#pragma unroll
    for (int nt = 0; nt < NT; nt += 2) {
      const int nb = n0 + nt * 8;
      uint32_t b[4];
      if (!B_T) ldsm4(b, Bs + (nb + r8 + (j >> 1) * 8) * ldb + k0 + (j & 1) * 8);
      else ldsm4t(b, Bs + (k0 + r8 + (j & 1) * 8) * ldb + nb + (j >> 1) * 8);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        mma16816(acc[mt][nt], a[mt], b[0], b[1]);
        mma16816(acc[mt][nt + 1], a[mt], b[2], b[3]);
      }
    }
  }
}

template <int MT, int NT>
__device__ __forceinline__ void zero(float (&acc)[MT][NT][4]) {
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int jj = 0; jj < NT; ++jj) acc[i][jj][0] = acc[i][jj][1] = acc[i][jj][2] = acc[i][jj][3] = 0.f;
}

// fragment element (mt, nt, e) -> (row, col) inside the warp tile
__device__ __forceinline__ int frag_row(int mt, int e) { return mt * 16 + ((threadIdx.x & 31) >> 2) + (e >= 2 ? 8 : 0); }
__device__ __forceinline__ int frag_col(int nt, int e) { return nt * 8 + ((threadIdx.x & 31) & 3) * 2 + (e & 1); }

// async 16-byte copies of a rows x cols bf16 tile (global pitch gp, smem pitch sp)
__device__ __forceinline__ void cp_async16(void* s, const void* g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(s)), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void load_tile(__nv_bfloat16* s, int sp, const __nv_bfloat16* g, long long gp, int rows,
                                          int cols) {
  const int per_row = cols / 8;
  for (int i = threadIdx.x; i < rows * per_row; i += blockDim.x) {
    const int r = i / per_row, c = (i - r * per_row) * 8;
    cp_async16(s + r * sp + c, g + r * gp + c);
  }
}


}  // namespace mma
}  // namespace vagus
