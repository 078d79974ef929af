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

// Per-channel (KDA) gate from the low-rank projection f (T x H dk, bf16,
// row pitch ldf) and the write strength from b (T x H, bf16, pitch ldb):
//   g[t, h dk + c] = -exp(A_log[h]) * softplus(f + dt_bias[h dk + c])   (fp32)
//   beta[t, h]     = sigmoid(b)
// One CTA row-strides over tokens, a thread owns 4 adjacent channels.
__global__ void kda_gates_fwd_k(const __nv_bfloat16* __restrict__ f, long long ldf,
                                const __nv_bfloat16* __restrict__ b, long long ldb, const float* __restrict__ A_log,
                                const float* __restrict__ dt_bias, float* __restrict__ g, float* __restrict__ beta,
                                long long T, int H, int dk) {
  const int HK = H * dk;
  const int c = 4 * threadIdx.x;
  const bool act = c < HK;
  const int h = act ? c / dk : 0;
  const float A = act ? __expf(A_log[h]) : 0.f;
  const float4 bias = act ? *reinterpret_cast<const float4*>(dt_bias + c) : make_float4(0.f, 0.f, 0.f, 0.f);
  constexpr int RU = 4;                              // rows per iteration, loads issued together
  for (long long t0 = (long long)blockIdx.x * RU; t0 < T; t0 += (long long)gridDim.x * RU) {
    uint2 u[RU];
#pragma unroll
    for (int r = 0; r < RU; ++r)
      if (act && t0 + r < T) u[r] = *reinterpret_cast<const uint2*>(f + (t0 + r) * ldf + c);
#pragma unroll
    for (int r = 0; r < RU; ++r) {
      const long long t = t0 + r;
      if (t >= T) break;
      if (act) {
        const float2 f0 = unpack_bf16x2(u[r].x), f1 = unpack_bf16x2(u[r].y);
        *reinterpret_cast<float4*>(g + t * HK + c) =
            make_float4(-A * softplus_f(f0.x + bias.x), -A * softplus_f(f0.y + bias.y),
                        -A * softplus_f(f1.x + bias.z), -A * softplus_f(f1.y + bias.w));
      }
      if (threadIdx.x < H) beta[t * H + threadIdx.x] = sigmoid_f(bf2f(b[t * ldb + threadIdx.x]));
    }
  }
}

// Backward: df = dg (-A) sigmoid(f + dt_bias) (bf16, pitch lddf), db = dbeta
// beta (1 - beta) (bf16, pitch lddb), and dA_log[h] += sum dg g, ddt[hc] +=
// sum df -- per-thread register sums over the CTA's tokens, one atomic each.
__global__ void kda_gates_bwd_k(const float* __restrict__ dg, const float* __restrict__ dbeta,
                                const __nv_bfloat16* __restrict__ f, long long ldf,
                                const __nv_bfloat16* __restrict__ b, long long ldb, const float* __restrict__ A_log,
                                const float* __restrict__ dt_bias, __nv_bfloat16* __restrict__ df, long long lddf,
                                __nv_bfloat16* __restrict__ db, long long lddb, float* __restrict__ dA_log,
                                float* __restrict__ ddt, long long T, int H, int dk) {
  const int HK = H * dk;
  const int c = 4 * threadIdx.x;
  const bool act = c < HK;
  const int h = act ? c / dk : 0;
  const float A = act ? __expf(A_log[h]) : 0.f;
  const float4 bias = act ? *reinterpret_cast<const float4*>(dt_bias + c) : make_float4(0.f, 0.f, 0.f, 0.f);
  float sa = 0.f, sd0 = 0.f, sd1 = 0.f, sd2 = 0.f, sd3 = 0.f;
  // RU rows per iteration, their loads issued together (memory-level parallelism)
  constexpr int RU = 4;
  for (long long t0 = (long long)blockIdx.x * RU; t0 < T; t0 += (long long)gridDim.x * RU) {
    uint2 u[RU];
    float4 d4[RU];
#pragma unroll
    for (int r = 0; r < RU; ++r) {
      const long long t = t0 + r;
      if (act && t < T) {
        u[r] = *reinterpret_cast<const uint2*>(f + t * ldf + c);
        d4[r] = *reinterpret_cast<const float4*>(dg + t * HK + c);
      }
    }
#pragma unroll
    for (int r = 0; r < RU; ++r) {
      const long long t = t0 + r;
      if (t >= T) break;
      if (act) {
        const float2 f0 = unpack_bf16x2(u[r].x), f1 = unpack_bf16x2(u[r].y);
        const float x[4] = {f0.x + bias.x, f0.y + bias.y, f1.x + bias.z, f1.y + bias.w};
        const float d[4] = {d4[r].x, d4[r].y, d4[r].z, d4[r].w};
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          o[j] = d[j] * (-A) * sigmoid_f(x[j]);       // d softplus = sigmoid
          sa += d[j] * (-A) * softplus_f(x[j]);       // dg / dA_log = g
        }
        sd0 += o[0]; sd1 += o[1]; sd2 += o[2]; sd3 += o[3];
        *reinterpret_cast<uint2*>(df + t * lddf + c) = make_uint2(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]));
      }
      if (threadIdx.x < H) {
        const float sb = sigmoid_f(bf2f(b[t * ldb + threadIdx.x]));
        db[t * lddb + threadIdx.x] = f2bf(dbeta[t * H + threadIdx.x] * sb * (1.f - sb));
      }
    }
  }
  if (act) {
    atomicAdd(&ddt[c], sd0);
    atomicAdd(&ddt[c + 1], sd1);
    atomicAdd(&ddt[c + 2], sd2);
    atomicAdd(&ddt[c + 3], sd3);
  }
  // dA_log: lanes of one head reduce first (a warp's 128 channels lie in one head when dk is a
  // multiple of 128), so each head takes a few atomics per CTA instead of one per thread
  const unsigned lanes_act = __ballot_sync(0xffffffffu, act);
  const int h0 = __shfl_sync(0xffffffffu, h, 0);
  const bool one_head = __all_sync(0xffffffffu, !act || h == h0);
  if (one_head) {
    const float tot = warp_sum(act ? sa : 0.f);
    if ((threadIdx.x & 31) == 0 && lanes_act) atomicAdd(&dA_log[h0], tot);
  } else if (act) {
    atomicAdd(&dA_log[h], sa);
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

int kda_gates_fwd(const void* f, long long ldf, const void* b, long long ldb, const float* A_log, const float* dt_bias,
                  float* g, float* beta, long long T, int H, int dk, cudaStream_t st) {
  const int HK = H * dk;
  if (HK % 4 || HK / 4 > 1024 || H > HK / 4 || ldf % 4 || (reinterpret_cast<uintptr_t>(f) & 7u)) return 5;
  const long long rows4 = (T + 3) / 4;
  const int grid = static_cast<int>(rows4 < 2368 ? (rows4 < 1 ? 1 : rows4) : 2368);
  kda_gates_fwd_k<<<grid, HK / 4, 0, st>>>((const __nv_bfloat16*)f, ldf, (const __nv_bfloat16*)b, ldb, A_log, dt_bias,
                                          g, beta, T, H, dk);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int kda_gates_bwd(const float* dg, const float* dbeta, const void* f, long long ldf, const void* b, long long ldb,
                  const float* A_log, const float* dt_bias, void* df, long long lddf, void* db, long long lddb,
                  float* dA_log, float* ddt, long long T, int H, int dk, cudaStream_t st) {
  const int HK = H * dk;
  if (HK % 4 || HK / 4 > 1024 || H > HK / 4 || ldf % 4 || lddf % 4 || (reinterpret_cast<uintptr_t>(f) & 7u) ||
      (reinterpret_cast<uintptr_t>(df) & 7u))
    return 5;
  const long long rows4 = (T + 3) / 4;
  const int grid = static_cast<int>(rows4 < 592 ? (rows4 < 1 ? 1 : rows4) : 592);
  kda_gates_bwd_k<<<grid, HK / 4, 0, st>>>(dg, dbeta, (const __nv_bfloat16*)f, ldf, (const __nv_bfloat16*)b, ldb,
                                          A_log, dt_bias, (__nv_bfloat16*)df, lddf, (__nv_bfloat16*)db, lddb, dA_log,
                                          ddt, T, H, dk);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

}  // namespace vagus
