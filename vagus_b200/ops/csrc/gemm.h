// Host interface of the sm_100a tcgen05 GEMM (gemm.cu).
#pragma once
#include <cuda_runtime.h>

namespace vagus {

struct GemmArgs {
  // math: C[b] (M x N) = alpha * A[b] (M x K) @ B[b] (N x K)^T + beta * S[b]
  const void* A = nullptr;   // bf16; a_mn=false: [M][lda] (K contiguous); true: [K][lda] (M contiguous)
  const void* B = nullptr;   // bf16; b_mn=false: [N][ldb] (K contiguous); true: [K][ldb] (N contiguous)
  long long lda = 0, ldb = 0, strideA = 0, strideB = 0;
  bool a_mn = false, b_mn = false;
  int M = 0, N = 0, K = 0, batch = 1;
  void* C = nullptr;         // bf16 or fp32, [M][ldc]
  long long ldc = 0, strideC = 0;
  int c_f32 = 0;
  const void* S = nullptr;   // optional source for the beta term (bf16 or fp32), [M][lds]
  long long lds = 0, strideS = 0;
  int s_f32 = 0;
  float alpha = 1.f, beta = 0.f;
  int atomic = 0;            // 1: C (fp32) += alpha * A @ B^T with red.add (split-K allowed)
  int split_k = 0;           // 0: automatic (atomic mode only), 1: none, >1: fixed, -1: stream-K (CTA pairs)
  int block_n = 0;           // 0: automatic (128 or 256)
  int* err = nullptr;        // device error word (bounded-wait timeouts)
  // Scatter epilogue (bf16 C, not atomic): the output's rows (scatter = 1) or
  // columns (scatter = 2) fall into blocks of scatter_span; block o is written
  // to scatter_dst[o] -- typically another GPU's buffer through a peer mapping,
  // so the product travels over NVLink from the epilogue itself -- as
  // [scatter_batch0 + b][row - o span | row][col | col - o span] with row pitch
  // dst_ld and batch stride dst_stride (elements).  C is not written.
  int scatter = 0;
  int scatter_span = 0;
  int scatter_n = 0;         // number of destinations (<= 16)
  void* scatter_dst[16] = {};
  long long dst_ld = 0, dst_stride = 0;
  int scatter_batch0 = 0;
  // Gathered B (K-major, batch 1, one-CTA tiles): B's rows live in gather_n
  // buffers of gather_rows rows each (row pitch ldb) -- typically the row
  // shards of a weight held by the GPUs of a group, which the TMA loads of
  // this GEMM then read over NVLink (no multicast) -- rows
  // [o * gather_rows, (o + 1) * gather_rows) in gather_src[o].  `B` is not
  // read.  gather_rows must be a multiple of 8 and at least 128.
  int gather_n = 0;
  int gather_rows = 0;
  const void* gather_src[8] = {};
};

// Returns 0 on launch, nonzero on argument / encode / launch failure.
int gemm_launch(const GemmArgs& args, cudaStream_t stream);

// bf16 tiled tensor map with 128-byte swizzle (the driver's tiled encoder):
// `map` points at a 128-byte CUtensorMap; dims and box in elements
// (innermost first), strides in bytes for dims 1..rank-1.  False on failure.
bool encode_bf16_map(void* map, const void* base, int rank, const unsigned long long* dims,
                     const unsigned long long* strides, const unsigned* box);
// fp32 tiled tensor map, 128-byte swizzle or none (e.g. for bulk reductions).
bool encode_f32_map(void* map, const void* base, int rank, const unsigned long long* dims,
                    const unsigned long long* strides, const unsigned* box, bool swizzle128);

}  // namespace vagus
