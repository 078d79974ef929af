// Unit-lower-triangular inverse of a 64 x 64 chunk matrix in shared memory,
// shared by the chunked delta-rule kernels (gdr_intra.cu, kda_intra.cu):
// T = (I + M)^{-1} for a strictly lower triangular M, in place, by 256
// threads.
#pragma once
#include "common.cuh"

namespace vagus {
namespace wy {

constexpr int C = 64;
constexpr int THREADS = 256;

// T = (I + M)^{-1} in place, M strictly lower triangular (row stride C + 1),
// blocked over 16 x 16 tiles so the whole CTA works in parallel with only a
// handful of barriers:
//   1. the four diagonal blocks X_bb = (I + M_bb)^{-1}: one warp per block,
//      one lane per column, forward substitution with the column held in
//      registers (the M rows are warp-wide broadcast reads); written in place;
//   2. off-diagonal blocks by distance d = i - j = 1, 2, 3:
//      X_ij = -X_ii (sum_{k=j}^{i-1} M_ik X_kj).
//      The lower off-diagonal M blocks stay intact until the end (later
//      distances still read them), so X_ij is parked transposed in the
//      (all-zero) upper block (j, i), and the partial sum Y goes there first;
//   3. the parked blocks move to their lower positions, the upper is zeroed.
// Every product is fp32 on the CUDA cores (about 64 K multiply-adds in all).
constexpr int TB16 = 16;

__device__ __forceinline__ void tri_inverse_inplace(float (*M)[C + 1]) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp < 4 && lane < TB16) {
    const int o = warp * TB16, c = lane;
    float x[TB16];
#pragma unroll
    for (int i = 0; i < TB16; ++i) {
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < i; ++j) s += M[o + i][o + j] * x[j];
      x[i] = (i == c) ? 1.f : -s;      // rows above c give s = 0 (x[j] = 0 there)
    }
    __syncwarp(0x0000ffffu);
#pragma unroll
    for (int i = 0; i < TB16; ++i) M[o + i][o + c] = x[i];
  }
  __syncthreads();
  // thread -> element (r, cc) of a 16 x 16 block
  const int r = (threadIdx.x >> 4) & 15, cc = threadIdx.x & 15;
  for (int d = 1; d < 4; ++d) {
    const int nblk = 4 - d;                   // blocks (t + d, t), t < nblk
#pragma unroll
    for (int t = 0; t < 3; ++t) {
      if (t < nblk) {
        const int i = t + d, j = t;
        float y = 0.f;
#pragma unroll
        for (int u = 0; u < TB16; ++u) y += M[i * TB16 + r][j * TB16 + u] * M[j * TB16 + u][j * TB16 + cc];
        for (int k = j + 1; k < i; ++k)       // X_kj parked at (j, k), transposed
#pragma unroll
          for (int u = 0; u < TB16; ++u) y += M[i * TB16 + r][k * TB16 + u] * M[j * TB16 + cc][k * TB16 + u];
        M[j * TB16 + cc][i * TB16 + r] = y;   // Y parked transposed at (j, i)
      }
    }
    __syncthreads();
    float x[3];
#pragma unroll
    for (int t = 0; t < 3; ++t) {
      x[t] = 0.f;
      if (t < nblk) {
        const int i = t + d, j = t;
#pragma unroll
        for (int u = 0; u < TB16; ++u) x[t] -= M[i * TB16 + r][i * TB16 + u] * M[j * TB16 + cc][i * TB16 + u];
      }
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < 3; ++t)
      if (t < nblk) M[t * TB16 + cc][(t + d) * TB16 + r] = x[t];
    __syncthreads();
  }
  for (int idx = threadIdx.x; idx < C * C; idx += THREADS) {
    const int i = idx / C, j = idx % C;
    if ((i >> 4) > (j >> 4)) {                // lower off-diagonal: take the parked value
      M[i][j] = M[j][i];
      M[j][i] = 0.f;
    }
  }
  __syncthreads();
}

}  // namespace wy
}  // namespace vagus
