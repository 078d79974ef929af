// Scalar-gate activation of a Gated DeltaNet layer from the packed [a | b]
// projection (T x 2H, bf16, row pitch ld):
//   g    = -exp(A_log[h]) * softplus(a + dt_bias[h])     (log decay, fp32)
//   beta = sigmoid(b)                                     (write strength, fp32)
// and the backward, which also reduces dA_log / ddt_bias with one atomic per
// head per CTA.
#include "common.cuh"
#include "kernels.h"

namespace vagus {
namespace {

__global__ void gates_fwd_k(const __nv_bfloat16* __restrict__ ab, long long ld, const float* __restrict__ A_log,
                            const float* __restrict__ dt_bias, float* __restrict__ g, float* __restrict__ beta,
                            long long T, int H) {
  const long long n = T * H;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long t = i / H;
    const int h = static_cast<int>(i - t * H);
    const float a = bf2f(ab[t * ld + h]);
    const float b = bf2f(ab[t * ld + H + h]);
    g[i] = -__expf(A_log[h]) * softplus_f(a + dt_bias[h]);
    beta[i] = sigmoid_f(b);
  }
}

__global__ void gates_bwd_k(const float* __restrict__ dg, const float* __restrict__ dbeta,
                            const __nv_bfloat16* __restrict__ ab, long long ld, const float* __restrict__ A_log,
                            const float* __restrict__ dt_bias, __nv_bfloat16* __restrict__ dab,
                            float* __restrict__ dA_log, float* __restrict__ ddt, long long T, int H) {
  __shared__ float sA[64], sD[64];
  for (int h = threadIdx.x; h < H; h += blockDim.x) { sA[h] = 0.f; sD[h] = 0.f; }
  __syncthreads();
  const long long n = T * H;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long t = i / H;
    const int h = static_cast<int>(i - t * H);
    const float a = bf2f(ab[t * ld + h]);
    const float b = bf2f(ab[t * ld + H + h]);
    const float A = __expf(A_log[h]);
    const float x = a + dt_bias[h];
    const float sp = softplus_f(x);
    const float gv = -A * sp;
    const float d = dg[i];
    const float da = d * (-A) * sigmoid_f(x);     // d softplus = sigmoid
    const float sb = sigmoid_f(b);
    dab[t * ld + h] = f2bf(da);
    dab[t * ld + H + h] = f2bf(dbeta[i] * sb * (1.f - sb));
    atomicAdd(&sA[h], d * gv);                    // dg/dA_log = g
    atomicAdd(&sD[h], da);
  }
  __syncthreads();
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    atomicAdd(&dA_log[h], sA[h]);
    atomicAdd(&ddt[h], sD[h]);
  }
}

inline int grid_for(long long n) {
  long long g = (n + 255) / 256;
  return static_cast<int>(g > 1184 ? 1184 : (g < 1 ? 1 : g));
}

}  // namespace

int gdn_gates_fwd(const void* ab, long long ld, const float* A_log, const float* dt_bias, float* g, float* beta,
                  long long T, int H, cudaStream_t st) {
  gates_fwd_k<<<grid_for(T * H), 256, 0, st>>>((const __nv_bfloat16*)ab, ld, A_log, dt_bias, g, beta, T, H);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int gdn_gates_bwd(const float* dg, const float* dbeta, const void* ab, long long ld, const float* A_log,
                  const float* dt_bias, void* dab, float* dA_log, float* ddt_bias, long long T, int H,
                  cudaStream_t st) {
  if (H > 64) return 5;
  gates_bwd_k<<<grid_for(T * H), 256, 0, st>>>(dg, dbeta, (const __nv_bfloat16*)ab, ld, A_log, dt_bias,
                                               (__nv_bfloat16*)dab, dA_log, ddt_bias, T, H);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

}  // namespace vagus
