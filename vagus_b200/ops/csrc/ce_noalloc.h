/* C interface of the allocation-free fused linear cross-entropy
 * (ce_noalloc.cu).  This entry point has no counterpart in the reference.
 *
 * Who it is for: callers that cannot allocate device memory while they run --
 * code embedded in another runtime whose own allocator owns the GPU's memory
 * (a second allocator calling cudaMalloc behind its back would fight its pool
 * or fragment it), and latency-critical loops that must stay out of the
 * driver's allocation paths (cudaMalloc / cudaFree may synchronise the
 * device).  The caller supplies every input and output; the routine's own
 * working memory is one fixed device array inside the library
 * (vagus_noalloc_scratch_bytes(), 32 MiB, held by every GPU that loads the
 * library until the process exits).
 *
 * Shapes: hidden (N x D bf16, row-major), weight (V x D bf16), targets
 * (N int64; a negative target ignores its row; a target >= V is out of range:
 * the row is ignored and the device status records it), loss_out (2 fp32),
 * dh (N x D bf16), dW (V x D fp32, ACCUMULATED: zero it before the first
 * call).  N >= 128, D a multiple of 64, V >= 128 and a multiple of 8, and
 * 128 rows of bf16 logits must fit the array (V up to about 128 K).  For V
 * above about 64 K a chunk holds fewer than 256 rows, and then N may not lie
 * between that chunk size and 256 (a chunk cannot be split into two of at
 * least 128 rows): VAGUS_NOALLOC_ERR_ROW_SPLIT.
 *
 * Streams: `stream` must belong to the current device (the scratch address
 * is per device).  Every call uses the same array and leaves its contents
 * behind; what must start at zero is cleared at the start of each call.
 * Calls whose work overlaps on the GPU (two streams, two host threads without
 * ordering) race on the array: serialise them on one stream.
 *
 * Set-up: the first call on each device looks up the array's device address
 * (cudaGetSymbolAddress, with that device current) and caches it; make that
 * first call before any stream capture begins.
 *
 * Errors: the return code covers what the host can check before queuing work.
 * Failures found on the device -- a tensor-core GEMM wait that ran out of its
 * time budget, an out-of-range target -- are recorded in a status word inside
 * the array, cleared by each call; vagus_noalloc_status() synchronises the
 * stream and returns it (0: none). */
#ifndef VAGUS_CE_NOALLOC_H_
#define VAGUS_CE_NOALLOC_H_

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* return codes of the entry points */
enum VagusNoAllocCode {
  VAGUS_NOALLOC_OK = 0,
  VAGUS_NOALLOC_ERR_BAD_SHAPE = -1,   /* N < 128, D % 64, V < 128 or V % 8, a null buffer */
  VAGUS_NOALLOC_ERR_TOO_LARGE = -2,   /* 128 rows of logits do not fit the scratch array */
  VAGUS_NOALLOC_ERR_SYMBOL = -3,      /* the array's device address could not be resolved */
  VAGUS_NOALLOC_ERR_LAUNCH = -4,      /* a kernel launch or a copy was rejected */
  VAGUS_NOALLOC_ERR_ROW_SPLIT = -5,   /* chunk size < N < 256: no split into chunks of >= 128 rows */
  VAGUS_NOALLOC_ERR_STREAM = -6       /* the stream belongs to another device */
};

/* device status words reported by vagus_noalloc_status() */
enum VagusNoAllocStatus {
  VAGUS_NOALLOC_STATUS_OK = 0,
  /* 1..3: a tensor-core GEMM's producer / MMA / epilogue wait ran out of time */
  VAGUS_NOALLOC_STATUS_BAD_TARGET = 16 /* a target id >= V (that row was ignored) */
};

/* loss_out[0] = mean CE + z_coef * mean(lse^2), loss_out[1] = the z term;
 * dh = dloss/dhidden; dW += dloss/dweight.  Queued on `stream`; returns
 * before the work finishes. */
int vagus_fused_linear_ce_noalloc(const void* hidden, const void* weight, const long long* targets, long long N,
                                  int D, int V, float z_coef, float* loss_out, void* dh, float* dW,
                                  cudaStream_t stream);

/* Waits for `stream`, then stores in *status the device status of the most
 * recent call queued on it (each call clears the word when it starts).
 * Returns a VagusNoAllocCode. */
int vagus_noalloc_status(cudaStream_t stream, int* status);

const char* vagus_noalloc_error_string(int code);
long long vagus_noalloc_scratch_bytes(void);

#ifdef __cplusplus
}
#endif

#endif /* VAGUS_CE_NOALLOC_H_ */
