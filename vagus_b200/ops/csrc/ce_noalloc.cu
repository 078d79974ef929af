// Allocation-free entry point of the fused linear cross-entropy.  It has no
// counterpart in the reference; its C interface, the callers it serves and
// its limits are stated in ce_noalloc.h.
//
// Working memory: one file-scope device array of kScratchBytes per GPU,
// laid out as
//   [acc: 2 fp32 | status: int32 | pad to 256 B][row loss][row lse][pad][logits chunk, bf16]
// The logits of one chunk of rows are produced by the tcgen05 GEMM, turned
// into the loss gradient in place by softmax_ce, and consumed by the dh and
// dW GEMMs; the per-row losses / lse are reduced into acc.  The GEMMs'
// bounded waits and softmax_ce's target check report into the status word.
#include "ce_noalloc.h"

#include "common.cuh"
#include "gemm.h"
#include "kernels.h"

namespace vagus {
namespace {

constexpr long long kScratchBytes = 32ll << 20;
constexpr int kMinRows = 128;                 // the GEMM's M tile
constexpr int kMaxDevices = 64;
constexpr long long kHeaderBytes = 256;

__device__ __align__(256) unsigned char g_ce_scratch[kScratchBytes];

// Device address of g_ce_scratch per device (host code may not take the
// symbol's address directly: it names a host-side stand-in).
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

// zero the accumulators and the status word
__global__ void ce_clear(float* acc, int* status) {
  if (threadIdx.x < 2) acc[threadIdx.x] = 0.f;
  if (threadIdx.x == 2) *status = 0;
}

int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return VAGUS_NOALLOC_ERR_SYMBOL;
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_ce_scratch) != cudaSuccess || p == nullptr) return VAGUS_NOALLOC_ERR_SYMBOL;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return VAGUS_NOALLOC_OK;
}

// The stream's device must be the current one (the scratch address is per device).
int check_stream(cudaStream_t stream) {
  int cur = 0, sdev = 0;
  if (cudaGetDevice(&cur) != cudaSuccess) return VAGUS_NOALLOC_ERR_SYMBOL;
  if (cudaStreamGetDevice(stream, &sdev) != cudaSuccess) return VAGUS_NOALLOC_ERR_STREAM;
  return sdev == cur ? VAGUS_NOALLOC_OK : VAGUS_NOALLOC_ERR_STREAM;
}

int* status_word(void* base) { return reinterpret_cast<int*>(static_cast<unsigned char*>(base) + 8); }

}  // namespace
}  // namespace vagus

extern "C" {

__attribute__((visibility("default"))) const char* vagus_noalloc_error_string(int code) {
  switch (code) {
    case VAGUS_NOALLOC_OK: return "ok";
    case VAGUS_NOALLOC_ERR_BAD_SHAPE:
      return "bad shape: need N >= 128, D % 64 == 0, V >= 128, V % 8 == 0 and non-null buffers";
    case VAGUS_NOALLOC_ERR_TOO_LARGE: return "problem too large for the fixed 32 MiB scratch array (V too large)";
    case VAGUS_NOALLOC_ERR_SYMBOL: return "could not resolve the scratch array's device address";
    case VAGUS_NOALLOC_ERR_LAUNCH: return "kernel launch or copy failed";
    case VAGUS_NOALLOC_ERR_ROW_SPLIT:
      return "N lies between the chunk size (under 256 rows for V above about 64 K) and 256: no split into chunks "
             "of at least 128 rows";
    case VAGUS_NOALLOC_ERR_STREAM: return "the stream belongs to a device other than the current one";
    default: return "unknown error";
  }
}

__attribute__((visibility("default"))) long long vagus_noalloc_scratch_bytes(void) { return vagus::kScratchBytes; }

__attribute__((visibility("default"))) int vagus_noalloc_status(cudaStream_t stream, int* status) {
  using namespace vagus;
  if (status == nullptr) return VAGUS_NOALLOC_ERR_BAD_SHAPE;
  int rc = check_stream(stream);
  if (rc != VAGUS_NOALLOC_OK) return rc;
  void* base = nullptr;
  if ((rc = scratch_address(&base)) != VAGUS_NOALLOC_OK) return rc;
  if (cudaMemcpyAsync(status, status_word(base), sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
      cudaStreamSynchronize(stream) != cudaSuccess)
    return VAGUS_NOALLOC_ERR_LAUNCH;
  return VAGUS_NOALLOC_OK;
}

__attribute__((visibility("default"))) int vagus_fused_linear_ce_noalloc(
    const void* hidden, const void* weight, const long long* targets, long long N, int D, int V, float z_coef,
    float* loss_out, void* dh, float* dW, cudaStream_t stream) {
  using namespace vagus;
  if (!hidden || !weight || !targets || !loss_out || !dh || !dW) return VAGUS_NOALLOC_ERR_BAD_SHAPE;
  if (N < kMinRows || D < 64 || D % 64 || V < 128 || V % 8) return VAGUS_NOALLOC_ERR_BAD_SHAPE;
  const long long row_bytes = (long long)V * 2;
  const long long usable = kScratchBytes - kHeaderBytes - 256;   // 256: alignment of the logits chunk
  long long max_rows = usable / (row_bytes + 8);
  max_rows = (max_rows / 64) * 64;
  if (max_rows < kMinRows) return VAGUS_NOALLOC_ERR_TOO_LARGE;
  // chunks of (nearly) equal size, each at least kMinRows rows
  const long long n_chunks = (N + max_rows - 1) / max_rows;
  const long long per = (N + n_chunks - 1) / n_chunks;
  if (N - (n_chunks - 1) * per < kMinRows) return VAGUS_NOALLOC_ERR_ROW_SPLIT;
  int rc = check_stream(stream);
  if (rc != VAGUS_NOALLOC_OK) return rc;
  void* base = nullptr;
  if ((rc = scratch_address(&base)) != VAGUS_NOALLOC_OK) return rc;
  unsigned char* s = static_cast<unsigned char*>(base);
  float* acc = reinterpret_cast<float*>(s);
  int* status = status_word(base);
  float* row_loss = reinterpret_cast<float*>(s + kHeaderBytes);
  float* row_lse = row_loss + max_rows;
  unsigned char* lp = reinterpret_cast<unsigned char*>(row_lse + max_rows);
  lp = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(lp) + 255) & ~uintptr_t(255));
  __nv_bfloat16* logits = reinterpret_cast<__nv_bfloat16*>(lp);
  ce_clear<<<1, 32, 0, stream>>>(acc, status);
  const __nv_bfloat16* h = static_cast<const __nv_bfloat16*>(hidden);
  __nv_bfloat16* dhp = static_cast<__nv_bfloat16*>(dh);
  for (long long r0 = 0; r0 < N; r0 += per) {
    const int rows = static_cast<int>(N - r0 < per ? N - r0 : per);
    GemmArgs g;                                            // logits = h W^T
    g.A = h + r0 * D; g.lda = D; g.B = weight; g.ldb = D;
    g.M = rows; g.N = V; g.K = D; g.C = logits; g.ldc = V; g.err = status;
    if (gemm_launch(g, stream) != 0) return VAGUS_NOALLOC_ERR_LAUNCH;
    if (softmax_ce(logits, targets + r0, row_loss, row_lse, rows, V, 1.0f / static_cast<float>(N), z_coef, stream,
                   status) != 0)
      return VAGUS_NOALLOC_ERR_LAUNCH;
    ce_rows_reduce<<<1, 256, 0, stream>>>(row_loss, row_lse, rows, acc);
    GemmArgs d;                                            // dh = dlogits W
    d.A = logits; d.lda = V; d.B = weight; d.ldb = D; d.b_mn = true;
    d.M = rows; d.N = D; d.K = V; d.C = dhp + r0 * D; d.ldc = D; d.err = status;
    if (gemm_launch(d, stream) != 0) return VAGUS_NOALLOC_ERR_LAUNCH;
    GemmArgs w;                                            // dW += dlogits^T h
    w.A = logits; w.lda = V; w.a_mn = true; w.B = h + r0 * D; w.ldb = D; w.b_mn = true;
    w.M = V; w.N = D; w.K = rows; w.C = dW; w.ldc = D; w.c_f32 = 1; w.atomic = 1; w.err = status;
    if (gemm_launch(w, stream) != 0) return VAGUS_NOALLOC_ERR_LAUNCH;
  }
  ce_finish<<<1, 32, 0, stream>>>(acc, loss_out, 1.0f / static_cast<float>(N), z_coef);
  return cudaGetLastError() == cudaSuccess ? VAGUS_NOALLOC_OK : VAGUS_NOALLOC_ERR_LAUNCH;
}

}  // extern "C"
