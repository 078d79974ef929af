// Allocation-free entry point of the fused linear cross-entropy.
//
// Declaration: this entry point has no counterpart in the reference.  It
// exists for callers that cannot allocate device memory at call time: code
// embedded in another runtime whose own allocator owns the device's memory
// (a second allocator calling cudaMalloc behind its back would contend with
// its pool or fragment it), and latency-critical loops that must not enter
// the driver's allocation paths (cudaMalloc / cudaFree can synchronise the
// device).  Such a caller still provides every input and output buffer; the
// only memory this routine needs beyond them -- one chunk of bf16 logits and
// a few per-row scalars -- lives in a fixed file-scope device array.
//
//   vagus_fused_linear_ce_noalloc(hidden (N x D bf16), weight (V x D bf16),
//                                 targets (N int64), ...)
//     -> loss_out[0] = mean CE + z_coef * mean(lse^2),  loss_out[1] = the z term
//        dh (N x D bf16)   = d(loss) / d(hidden)
//        dW (V x D fp32)  += d(loss) / d(weight)    (accumulated: zero it first)
//
// Limits: the scratch array is kScratchBytes (32 MiB) per GPU, held from
// library load until process exit.  A chunk needs at least 128 rows of
// logits, so V may be at most about 128 K (128 rows x V x 2 bytes must fit);
// larger problems are rejected with kErrTooLarge before any work is queued.
// N >= 128, D a multiple of 64 and >= 64, V a multiple of 8.
//
// Every call uses the same array and leaves its contents behind; the
// accumulators it needs zeroed are cleared at the start of each call.  Calls
// whose work overlaps on the GPU (two streams, or two host threads without
// ordering) race on the array: serialise them on one stream.
//
// The first call on each device looks up the array's device address with
// cudaGetSymbolAddress (with that device current) and caches it; make that
// first call before any stream capture begins.
#include "common.cuh"
#include "gemm.h"
#include "kernels.h"

namespace vagus {
namespace {

constexpr long long kScratchBytes = 32ll << 20;
constexpr int kMinRows = 128;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_ce_scratch[kScratchBytes];

void* g_scratch_addr[kMaxDevices] = {nullptr};

// sum of per-row losses and of squared log-sum-exps into acc[0], acc[1]
__global__ void ce_rows_reduce(const float* __restrict__ loss, const float* __restrict__ lse, int rows,
                               float* __restrict__ acc) {
  float a = 0.f, b = 0.f;
  for (int i = threadIdx.x; i < rows; i += blockDim.x) {
    a += loss[i];
    b += lse[i] * lse[i];
  }
  a = warp_sum(a);
  b = warp_sum(b);
  if ((threadIdx.x & 31) == 0) {
    atomicAdd(&acc[0], a);
    atomicAdd(&acc[1], b);
  }
}

__global__ void ce_finish(const float* __restrict__ acc, float* __restrict__ out, float inv_n, float z_coef) {
  if (threadIdx.x == 0) {
    const float z = z_coef * acc[1] * inv_n;
    out[0] = acc[0] * inv_n + z;
    out[1] = z;
  }
}

__global__ void ce_clear(float* acc) {
  if (threadIdx.x < 2) acc[threadIdx.x] = 0.f;
}

int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -3;
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_ce_scratch) != cudaSuccess || p == nullptr) return -3;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return 0;
}

}  // namespace
}  // namespace vagus

extern "C" {

enum VagusNoAllocCode {
  kNoAllocOk = 0,
  kErrBadShape = -1,       // N < 128, D not a multiple of 64, V not a multiple of 8, null pointer
  kErrTooLarge = -2,       // 128 rows of logits do not fit the scratch array
  kErrSymbol = -3,         // cudaGetSymbolAddress failed (no device / context)
  kErrLaunch = -4,         // a kernel launch was rejected
};

__attribute__((visibility("default"))) const char* vagus_noalloc_error_string(int code) {
  switch (code) {
    case kNoAllocOk: return "ok";
    case kErrBadShape: return "bad shape: need N >= 128, D % 64 == 0, V % 8 == 0 and non-null buffers";
    case kErrTooLarge: return "problem too large for the fixed 32 MiB scratch array (V too large)";
    case kErrSymbol: return "could not resolve the scratch array's device address";
    case kErrLaunch: return "kernel launch failed";
    default: return "unknown error";
  }
}

__attribute__((visibility("default"))) long long vagus_noalloc_scratch_bytes() { return vagus::kScratchBytes; }

__attribute__((visibility("default"))) int vagus_fused_linear_ce_noalloc(
    const void* hidden, const void* weight, const long long* targets, long long N, int D, int V, float z_coef,
    float* loss_out, void* dh, float* dW, cudaStream_t stream) {
  using namespace vagus;
  if (!hidden || !weight || !targets || !loss_out || !dh || !dW) return kErrBadShape;
  if (N < kMinRows || D < 64 || D % 64 || V < 128 || V % 8) return kErrBadShape;
  // layout: [acc: 2 floats, 256 B][row loss][row lse][logits chunk]
  const long long row_bytes = (long long)V * 2;
  const long long usable = kScratchBytes - 256;
  long long max_rows = usable / (row_bytes + 8);
  max_rows = (max_rows / 64) * 64;
  if (max_rows < kMinRows) return kErrTooLarge;
  void* base = nullptr;
  if (scratch_address(&base) != 0) return kErrSymbol;
  unsigned char* s = static_cast<unsigned char*>(base);
  float* acc = reinterpret_cast<float*>(s);
  float* row_loss = reinterpret_cast<float*>(s + 256);
  float* row_lse = row_loss + max_rows;
  unsigned char* lp = reinterpret_cast<unsigned char*>(row_lse + max_rows);
  lp = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(lp) + 255) & ~uintptr_t(255));
  __nv_bfloat16* logits = reinterpret_cast<__nv_bfloat16*>(lp);
  // chunks of equal size, each at least kMinRows rows
  const long long n_chunks = (N + max_rows - 1) / max_rows;
  const long long per = (N + n_chunks - 1) / n_chunks;
  if (N - (n_chunks - 1) * per < kMinRows) return kErrBadShape;
  ce_clear<<<1, 32, 0, stream>>>(acc);
  const __nv_bfloat16* h = static_cast<const __nv_bfloat16*>(hidden);
  __nv_bfloat16* dhp = static_cast<__nv_bfloat16*>(dh);
  for (long long r0 = 0; r0 < N; r0 += per) {
    const int rows = static_cast<int>(N - r0 < per ? N - r0 : per);
    GemmArgs g;                                            // logits = h W^T
    g.A = h + r0 * D; g.lda = D; g.B = weight; g.ldb = D;
    g.M = rows; g.N = V; g.K = D; g.C = logits; g.ldc = V;
    if (gemm_launch(g, stream) != 0) return kErrLaunch;
    if (softmax_ce(logits, targets + r0, row_loss, row_lse, rows, V, 1.0f / static_cast<float>(N), z_coef,
                   stream) != 0)
      return kErrLaunch;
    ce_rows_reduce<<<1, 256, 0, stream>>>(row_loss, row_lse, rows, acc);
    GemmArgs d;                                            // dh = dlogits W
    d.A = logits; d.lda = V; d.B = weight; d.ldb = D; d.b_mn = true;
    d.M = rows; d.N = D; d.K = V; d.C = dhp + r0 * D; d.ldc = D;
    if (gemm_launch(d, stream) != 0) return kErrLaunch;
    GemmArgs w;                                            // dW += dlogits^T h
    w.A = logits; w.lda = V; w.a_mn = true; w.B = h + r0 * D; w.ldb = D; w.b_mn = true;
    w.M = V; w.N = D; w.K = rows; w.C = dW; w.ldc = D; w.c_f32 = 1; w.atomic = 1;
    if (gemm_launch(w, stream) != 0) return kErrLaunch;
  }
  ce_finish<<<1, 32, 0, stream>>>(acc, loss_out, 1.0f / static_cast<float>(N), z_coef);
  return cudaGetLastError() == cudaSuccess ? kNoAllocOk : kErrLaunch;
}

}  // extern "C"
