// Host-side launchers of the sm_100a kernels (no torch types: the .cu files
// compile without the torch headers; bindings.cpp owns tensor checking).
// Every launcher returns 0 on success, nonzero on a launch / argument error.
#pragma once
#include <cuda_runtime.h>

namespace vagus {

// norm.cu
int rmsnorm_fwd(const void* x, int x_f32, const float* gamma, void* y, int y_f32, float* rstd, long long rows, int D,
                float eps, cudaStream_t s);
// dx16 (optional, bf16): a copy of dx; supported for fp32 x / dx with D in {512, 768, 1024, 1536, 2048}
int rmsnorm_bwd(const void* dy, int dy_f32, const void* x, int x_f32, const float* gamma, const float* rstd,
                const float* dres, void* dx, int dx_f32, float* dgamma, long long rows, int D, cudaStream_t s,
                void* dx16 = nullptr);
int rmsnorm_gated_fwd(const void* o, const void* g, long long ldg, int H, const float* gamma, void* y, int y_f32,
                      float* rstd, long long rows, int D, float eps, cudaStream_t s);
int rmsnorm_gated_bwd(const void* dy, const void* o, const void* g, long long ldg, int H, const float* gamma,
                      const float* rstd, void* dO, void* dG, long long lddg, float* dgamma, long long rows, int D,
                      cudaStream_t s);
// ld*: token pitch (elements) of each (B, L, H, D) operand; 0 means dense (H * D)
int qk_norm_rope_fwd(const void* x, const float* gamma, const float* cosv, const float* sinv, void* y, float* rstd,
                     long long rows, int L, int H, int D, float eps, long long ldx, long long ldy, cudaStream_t s);
int qk_norm_rope_bwd(const void* dy, const void* x, const float* gamma, const float* cosv, const float* sinv,
                     const float* rstd, void* dx, float* dgamma, long long rows, int L, int H, int D, long long lddy,
                     long long ldx, long long lddx, cudaStream_t s);

// elementwise.cu
int swiglu_fwd(const void* u, void* s, long long rows, int F, cudaStream_t st);
int swiglu_bwd(const void* ds, const void* u, void* du, long long rows, int F, cudaStream_t st);
int sigmoid_gate_fwd(const void* x, const void* g, void* y, long long n, cudaStream_t st);
int sigmoid_gate_bwd(const void* dy, const void* x, const void* g, void* dx, void* dg, long long n, cudaStream_t st);
// targets >= V are ignored like negative ones; status (optional) then records kErrBadTarget
int softmax_ce(void* logits, const long long* targets, float* loss, float* lse, long long rows, int V, float scale,
               float z_coef, cudaStream_t st, int* status = nullptr);
// V: rows of the table (token ids are checked against it in the bounds-checked build)
int embedding_fwd(const float* W, const long long* tok, void* y, int y_f32, long long n, int D, long long V,
                  cudaStream_t st);
int embedding_bwd(const void* dy, int dy_f32, const long long* tok, float* dW, long long n, int D, long long V,
                  cudaStream_t st);
int adamw_step(float* p, const float* g, float* m, float* v, void* shadow, long long n, float lr, float b1, float b2,
               float eps, float wd, float bc1, float bc2, float gscale, cudaStream_t st);
int muon_momentum(const float* g, float* buf, void* upd, long long n, float mu, int nesterov, float gscale,
                  cudaStream_t st);

// conv.cu: causal depthwise conv (K taps) + SiLU (+ per-head L2 norm) for
// the q / k / v streams of a GatedDeltaNet layer.
int conv_silu_fwd(const void* xp, long long ldx, const float* w, void* y, float* rnorm, long long B, long long L,
                  int D, int K, int head_dim, int l2norm, cudaStream_t st);
int conv_silu_bwd(const void* dy, const void* xp, long long ldx, const float* w, const float* rnorm, void* dx,
                  long long lddx, float* dw, long long B, long long L, int D, int K, int head_dim, int l2norm,
                  cudaStream_t st);

// gdn_gates.cu: per-token scalar gate and write strength from the packed
// projection: g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b).
int gdn_gates_fwd(const void* ab, long long ld, const float* A_log, const float* dt_bias, float* g, float* beta,
                  long long T, int H, cudaStream_t st);
int gdn_gates_bwd(const float* dg, const float* dbeta, const void* ab, long long ld, const float* A_log,
                  const float* dt_bias, void* dab, float* dA_log, float* ddt_bias, long long T, int H,
                  cudaStream_t st);
// Per-channel (KDA) gate g (T x H dk fp32) from the low-rank projection f
// (T x H dk bf16, pitch ldf) and beta (T x H fp32) from b (bf16, pitch ldb),
// and the backward (df, db bf16 into the packed gradient; dA_log, ddt_bias
// accumulated).
int kda_gates_fwd(const void* f, long long ldf, const void* b, long long ldb, const float* A_log, const float* dt_bias,
                  float* g, float* beta, long long T, int H, int dk, cudaStream_t st);
int kda_gates_bwd(const float* dg, const float* dbeta, const void* f, long long ldf, const void* b, long long ldb,
                  const float* A_log, const float* dt_bias, void* df, long long lddf, void* db, long long lddb,
                  float* dA_log, float* ddt, long long T, int H, int dk, cudaStream_t st);

// gdr.cu: inter-chunk state recurrence of the chunked gated delta rule
// (scalar gate), forward scan and reverse-scan backward (see gdr.cu).
struct GdrRecArgs {
  const void* W; const void* Qh; const void* Kt;   // (BH, N, C, DK) bf16
  const void* A;                                   // (BH, N, C, C) bf16
  const void* U;                                   // (BH, N, C, DV) bf16
  const float* gC;                                 // (BH, N), or (BH, N, DK) when gvec
  const float* S0;                                 // (BH, DK, DV) or null
  void* O;                                         // (B, N*C, H, DV) bf16, token-major
  void* Vp;                                        // (BH, N, DV, C) bf16: V'^T (written fwd, read bwd)
  void* states;                                    // (BH, N, DV, DK) bf16 entry states S_n^T (written fwd, read bwd)
  float* S_out;                                    // (BH, DK, DV) or null
  long long BH; int N, DK, DV;
  int H;                                           // heads (BH = B * H)
  int* err = nullptr;                              // device error word (the tcgen05 scan's bounded waits)
  int gvec = 0;                                    // 1: per-channel (KDA) chunk decay gC[k]
};
int gdr_rec_fwd(const GdrRecArgs& a, cudaStream_t st);
struct GdrRecBwdArgs {
  GdrRecArgs f;
  const void* dO;                                  // (B, N*C, H, DV) bf16, token-major
  const float* dS_final;                           // (BH, DK, DV) or null
  void* dW; void* dQh; void* dKt;                  // (BH, N, C, DK) bf16
  float* dA;                                       // (BH, N, C, C) fp32
  void* dU;                                        // (BH, N, C, DV) bf16
  float* dgC;                                      // (BH, N) fp32, zero-initialised (atomics)
  float* dS0;                                      // (BH, DK, DV) or null
  void* dstates;                                   // (BH, N, DV, DK) bf16 scratch: (dL/dS_{n+1})^T per chunk
};
int gdr_rec_bwd(const GdrRecBwdArgs& a, cudaStream_t st);
// gdr_intra.cu: intra-chunk WY / UT stage (scalar gate), forward + backward.
struct GdrIntraArgs {
  const void* q; const void* k; const void* v;   // (B, L, H, DK|DV) bf16 token-major
  const float* g; const float* beta;            // (B, L, H)
  void* W; void* Qh; void* Kt;                  // (B*H, N, C, DK) bf16
  void* A;                                      // (B*H, N, C, C) bf16
  void* U;                                      // (B*H, N, C, DV) bf16
  float* gC;                                    // (B*H, N)
  long long B, L; int H, DK, DV;
  float scale;
};
int gdr_intra_fwd(const GdrIntraArgs& a, cudaStream_t st);
struct GdrIntraBwdArgs {
  GdrIntraArgs f;                               // forward inputs (outputs unused)
  const void* dW; const void* dQh; const void* dKt;   // (BH, N, C, DK) bf16, from gdr_rec_bwd
  const float* dA;
  const void* dU; const float* dgC;
  void* dq; void* dk; void* dv;                 // (B, L, H, DK|DV) bf16
  float* dg; float* dbeta;                      // (B, L, H) fp32
};
int gdr_intra_bwd(const GdrIntraBwdArgs& a, cudaStream_t st);
int gdr_decode(const void* q, const void* k, const void* v, const float* g, const float* beta, float* S, void* o,
               long long BH, int dk, int dv, float scale, cudaStream_t st);

// attention.cu: causal (lower-right aligned) / full softmax attention.
struct AttnArgs {
  const void* q; const void* k; const void* v;  // (B, H, Lq, D), (B, Hk, Lk, D), (B, Hk, Lk, Dv) bf16
  void* o;                                      // (B, H, Lq, Dv) bf16
  float* lse;                                   // (B, H, Lq) fp32
  long long B; int H, Hk, Lq, Lk, D, Dv;
  long long sq_b, sq_h, sq_l, sk_b, sk_h, sk_l, sv_b, sv_h, sv_l, so_b, so_h, so_l;   // element strides
  int causal; float scale;
  int* err = nullptr;                           // device error word (bounded waits of the tcgen05 path)
};
int attn_fwd(const AttnArgs& a, cudaStream_t st);
struct AttnBwdArgs {
  AttnArgs f;
  const void* dO;            // like o (same strides)
  void* dq; void* dk; void* dv;   // (B, H, Lq, D), (B, Hk, Lk, D), (B, Hk, Lk, Dv) bf16, strided:
  long long sdq_b, sdq_h, sdq_l, sdk_b, sdk_h, sdk_l, sdv_b, sdv_h, sdv_l;   // element strides (unit inner)
  float* dq_acc;             // fp32 scratch (B, H, Lq, D)
  float* delta;              // fp32 scratch (B, H, Lq)
  // optional RoPE tables (L, D / 2) fp32, Lq == Lk == L: q and k were rotated by
  // interleaved pairs at their positions, and dq / dk leave un-rotated (the
  // rotation's transpose applied in the dQ pass and the dK epilogue; the
  // tcgen05 path at head dims 64 / 128 only)
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
};
int attn_bwd(const AttnBwdArgs& a, cudaStream_t st);
// Phase clock of the tcgen05 backward's CTA (0, 0): clock64() at 16 phase
// boundaries for each of the first 32 steps into buf[step * 16 + event]
// (device memory, 512 u64); null switches it off.
void attn_set_trace(unsigned long long* buf);

// kda.cu: the gated inner products of the per-channel-gate chunk form.
// Q, K, G (chunks, 64, dk) fp32; Aqk (j <= i), Akk (j < i): (chunks, 64, 64) fp32.
int kda_gated_fwd(const float* Q, const float* K, const float* G, float* Aqk, float* Akk, long long chunks, int dk,
                  cudaStream_t st);
int kda_gated_bwd(const float* Q, const float* K, const float* G, const float* dAqk, const float* dAkk, float* dQ,
                  float* dK, float* dG, long long chunks, int dk, cudaStream_t st);

// kda_intra.cu: the per-channel-gate intra-chunk stage (DK = 128, DV = 128 / 256).
// Forward: q, k (B, L, H, DK), v (B, L, H, DV) bf16, g (B, L, H, DK), beta (B, L, H)
// fp32 -> W, Qh, Kt (BH, N, 64, DK), A (BH, N, 64, 64), U (BH, N, 64, DV) bf16 and
// gC (BH, N, DK) fp32.
int kda_intra_fwd(const void* q, const void* k, const void* v, const float* g, const float* beta, void* W, void* Qh,
                  void* Kt, void* A, void* U, float* gC, int B, int L, int H, int DK, int DV, float scale,
                  cudaStream_t st);
struct KdaIntraBwdArgs {
  const void *q, *k, *v;
  const float *g, *beta;
  const void *dW, *dQh, *dKt, *dU;        // chunk-major bf16
  const float *dA, *dgC;                  // (BH, N, 64, 64), (BH, N, DK) fp32
  void *dq, *dk, *dv;                     // token-major bf16
  float *dg, *dbeta;                      // token-major fp32
  int B, L, H, DK, DV;
  float scale;
};
int kda_intra_bwd(const KdaIntraBwdArgs& a, cudaStream_t st);
// Phase clock of the KDA intra kernels' CTA (0, 0, 0): clock64() at phase
// boundaries into buf[event] (forward 0..15, backward 16..31; device memory,
// 32 u64); null switches it off.
void kda_set_trace(unsigned long long* buf);
// Phase clock of the GDN intra backward's CTA (0, 0, 0) (8 u64 of device
// memory); null switches it off.
void gdr_intra_set_trace(unsigned long long* buf);

// mobius.cu: x_t = (A_t x_{t-1} + B_t) / (C_t x_{t-1} + D_t) along L; A..D, X, gO and the
// gradients (batch, L, R) fp32 contiguous, x0 and gx0 (batch, R).
int mobius_fwd(const float* A, const float* B, const float* C, const float* D, const float* x0, float* X, int batch,
               int L, int R, cudaStream_t st);
int mobius_bwd(const float* A, const float* B, const float* C, const float* D, const float* x0, const float* X,
               const float* gO, float* gA, float* gB, float* gC, float* gD, float* gx0, int batch, int L, int R,
               cudaStream_t st);

// comm.cu: NVLink peer-to-peer all-gather / reduce-scatter over CUDA-IPC
// shared heaps (see comm.cu for the heap layout and the epoch protocol).
constexpr int kMaxCommPeers = 16;
constexpr int kCommAgFlags = 0;                 // byte offsets inside a heap
constexpr int kCommRsFlags = 256;
constexpr long long kCommHeaderBytes = 1024;
struct CommPeers {
  unsigned char* base[kMaxCommPeers];           // every rank's heap, mapped into this process
};
// wait_ns bounds every cross-GPU flag wait (the process group's timeout).
int comm_all_gather(const CommPeers& peers, int rank, int world, unsigned epoch, void* out, long long shard_bytes,
                    long long slot_cap, unsigned long long wait_ns, int* err, cudaStream_t st);
int comm_reduce_scatter(const CommPeers& peers, int rank, int world, unsigned epoch, const void* in, void* out,
                        long long shard_elems, int elem_bytes, float scale, long long ag_cap, long long slot_cap,
                        unsigned long long wait_ns, int* err, cudaStream_t st);
// Cross-GPU epoch barrier on the flag words at byte offset flag_off of every
// heap (kMaxCommPeers u32 per heap): publishes this stream's earlier writes
// (system-scope release), then waits (bounded) until every peer reached epoch.
constexpr int kCommBarFlags = 512;
// all-reduce: "slot staged" flags, "result pushed" flags, two CTA counters
constexpr int kCommArStaged = 640;
constexpr int kCommArPushed = 768;
constexpr int kCommArCount = 896;
// NVLink all-reduce of `n` elements (fp32 or bf16) of `buf` in place, times
// `scale`, over heaps laid out [header][slot 0][slot 1][result 0][result 1]
// (slot_cap bytes each); three launches, no extra synchronisation (see comm.cu).
int comm_all_reduce(const CommPeers& peers, int rank, int world, unsigned epoch, void* buf, long long n,
                    int elem_bytes, float scale, long long slot_cap, unsigned long long wait_ns, int* err,
                    cudaStream_t st);
int comm_barrier(const CommPeers& peers, int rank, int world, int flag_off, unsigned epoch, unsigned long long wait_ns,
                 int* err, cudaStream_t st);
// Block g (blk_bytes each) of src -> heap of rank g / per_rank at
// slot_off + (g % per_rank) * dst_stride + dst_off (peer stores; publish with
// comm_barrier).
int comm_scatter_blocks(const CommPeers& peers, int world, long long slot_off, const void* src, long long blk_bytes,
                        int nblk, int per_rank, long long dst_stride, long long dst_off, cudaStream_t st);

}  // namespace vagus
