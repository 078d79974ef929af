// NVLink peer-to-peer collectives for the FSDP2 parameter all-gather and the
// gradient reduce-scatter, as our own kernels instead of NCCL calls.
//
// Every rank owns one device "heap" (plain cudaMalloc, shared through CUDA
// IPC; no multicast objects) laid out as
//   [AG flags: 64 x u32][RS flags: 64 x u32][pad to 1 KB][AG slot 0][AG slot 1][RS slot 0][RS slot 1]
// and holds the device pointers of every peer's heap.  A collective of epoch
// e (a per-kind counter that advances identically on every rank, since FSDP
// issues its all-gathers and its reduce-scatters in the same order
// everywhere) uses slot e & 1:
//   1. stage:   this rank's contribution -> its own slot (local copy);
//   2. barrier: publish the copy (system-scope release), store e into every
//               peer's flag word for this rank, then wait until every peer's
//               flag in this heap reads >= e (acquire).  The wait is bounded
//               by a caller-given budget (the process group's timeout: ranks
//               legitimately drift apart by seconds -- a checkpoint write, a
//               slow data read); on expiry, or as soon as the error word
//               holds an earlier failure, the kernel records
//               kErrTimeoutPeer and returns;
//   3. combine: all-gather copies each peer's slot into its place in the
//               output; reduce-scatter sums this rank's rows of every peer's
//               slot in fp32, scales (1/world for an average) and casts into
//               the output shard.
// A slot is rewritten two epochs later; by then every peer has passed the
// barrier of the epoch in between, which it reaches only after finishing its
// reads of the slot, so two slots need no second barrier per call.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <cstdint>

namespace vagus {
namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// byte copy with 16-byte vectors for the aligned body
__device__ __forceinline__ void copy_bytes(uint8_t* dst, const uint8_t* src, long long n, long long tid,
                                           long long nthreads) {
  const bool al = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15u) == 0;
  long long body = al ? (n / 16) * 16 : 0;
  for (long long i = tid * 16; i < body; i += nthreads * 16)
    *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<const uint4*>(src + i);
  for (long long i = body + tid; i < n; i += nthreads) dst[i] = src[i];
}

__global__ void stage_k(uint8_t* slot, const uint8_t* src, long long n) {
  copy_bytes(slot, src, n, (long long)blockIdx.x * blockDim.x + threadIdx.x, (long long)gridDim.x * blockDim.x);
}

// one warp: lane p < world signals peer p and waits for peer p's flag
__global__ void barrier_k(const CommPeers peers, int rank, int world, int flag_off, uint32_t epoch,
                          unsigned long long budget_ns, int* err) {
  const int lane = threadIdx.x;
  __threadfence_system();          // the staging copy (previous kernel) is visible system-wide
  if (lane < world) {
    uint32_t* remote = reinterpret_cast<uint32_t*>(peers.base[lane] + flag_off) + rank;
    st_release_sys(remote, epoch);
  }
  bool ok = true;
  if (lane < world) {
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(peers.base[rank] + flag_off) + lane;
    if (ld_acquire_sys(mine) < epoch) {
      const unsigned long long t0 = globaltimer_ns();
      uint32_t spins = 0;
      while (ld_acquire_sys(mine) < epoch) {
        if (((++spins) & 1023u) == 0u) {
          // an earlier failure (another wait that ran out) ends this one too,
          // so a dead peer costs one budget, not one per collective
          if (globaltimer_ns() - t0 > budget_ns || (err != nullptr && *(volatile int*)err != 0)) {
            ok = false;
            break;
          }
        }
      }
    }
  }
  if (!ok) record_error(err, kErrTimeoutPeer);
  __syncwarp();
  __threadfence_system();
}

__global__ void gather_k(const CommPeers peers, int rank, int world, long long slot_off, uint8_t* out,
                         long long n) {
  // blockIdx.y = source rank
  const int src = blockIdx.y;
  if (src == rank || !VAGUS_CHECK(src, world)) return;         // own shard already in place
  copy_bytes(out + (long long)src * n, peers.base[src] + slot_off, n, (long long)blockIdx.x * blockDim.x + threadIdx.x,
             (long long)gridDim.x * blockDim.x);
}

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return bf2f(v); }

template <typename T>
__global__ void reduce_k(const CommPeers peers, int rank, int world, long long slot_off, T* out, long long n,
                         float scale) {
  // this rank's rows [rank * n, rank * n + n) of every peer's slot
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long t0 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if constexpr (sizeof(T) == 4) {
    if ((n & 3) == 0) {
      for (long long i = t0 * 4; i < n; i += stride * 4) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int p = 0; p < world; ++p) {
          const float* s = reinterpret_cast<const float*>(peers.base[p] + slot_off) + (long long)rank * n + i;
          const float4 v = *reinterpret_cast<const float4*>(s);
          acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
        }
        *reinterpret_cast<float4*>(out + i) =
            make_float4(scale * acc.x, scale * acc.y, scale * acc.z, scale * acc.w);
      }
      return;
    }
  }
  for (long long i = t0; i < n; i += stride) {
    float acc = 0.f;
    for (int p = 0; p < world; ++p) {
      const T* s = reinterpret_cast<const T*>(peers.base[p] + slot_off) + (long long)rank * n + i;
      acc += to_f<T>(*s);
    }
    if constexpr (sizeof(T) == 4) out[i] = scale * acc;
    else out[i] = f2bf(scale * acc);
  }
}

// ----------------------------------------------------------- all-reduce --
// Two-shot all-reduce over NVLink, three kernels on the caller's stream:
//   ar_stage_k   copy the buffer into this rank's slot (e & 1); the CTA that
//                finishes last publishes it: system-scope release of epoch e
//                into every peer's "staged" flag for this rank;
//   ar_push_k    every CTA waits (bounded) until all peers staged epoch e,
//                then reduces its part of this rank's 1/world chunk over the
//                peers' slots in fp32, applies `scale`, and stores the result
//                into every rank's result region (e & 1) -- NVLink stores from
//                the reducing threads; the last CTA publishes "pushed";
//   ar_finish_k  waits until all peers pushed epoch e, copies the result out.
// Reuse: slot (e & 1) is rewritten at epoch e + 2 only after this rank's
// ar_finish_k(e + 1), which follows every peer's ar_push_k(e + 1), which
// follows their reads of epoch e; the result region likewise.
struct ArArgs {
  CommPeers peers;
  int rank, world;
  uint32_t epoch;
  long long n;              // elements
  long long slot_cap;       // bytes per slot
  float scale;
  unsigned long long wait_ns;
  int* err;
};

__device__ __forceinline__ uint8_t* ar_slot(const ArArgs& a, int r) {
  return a.peers.base[r] + kCommHeaderBytes + (long long)(a.epoch & 1u) * a.slot_cap;
}
__device__ __forceinline__ uint8_t* ar_result(const ArArgs& a, int r) {
  return a.peers.base[r] + kCommHeaderBytes + 2 * a.slot_cap + (long long)(a.epoch & 1u) * a.slot_cap;
}

// The last CTA of the grid to arrive publishes `epoch` into every peer's flag
// block at flag_off (entry `rank`) after a system-scope fence.
__device__ __forceinline__ void ar_publish_last(const ArArgs& a, int flag_off, int counter) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    uint32_t* cnt = reinterpret_cast<uint32_t*>(a.peers.base[a.rank] + kCommArCount) + counter;
    if (atomicAdd(cnt, 1u) == gridDim.x - 1) {
      *cnt = 0;
      __threadfence_system();
      for (int p = 0; p < a.world; ++p)
        st_release_sys(reinterpret_cast<uint32_t*>(a.peers.base[p] + flag_off) + a.rank, a.epoch);
    }
  }
}

// Every peer's flag at flag_off of this rank's heap reads >= epoch (bounded).
__device__ __forceinline__ bool ar_wait_all(const ArArgs& a, int flag_off) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    const uint32_t* f = reinterpret_cast<const uint32_t*>(a.peers.base[a.rank] + flag_off);
    const unsigned long long t0 = globaltimer_ns();
    for (int p = 0; p < a.world && ok; ++p) {
      uint32_t spins = 0;
      while (ld_acquire_sys(f + p) < a.epoch) {
        if (((++spins) & 1023u) == 0u &&
            (globaltimer_ns() - t0 > a.wait_ns || (a.err != nullptr && *(volatile int*)a.err != 0))) {
          ok = 0;
          break;
        }
      }
    }
    if (!ok) record_error(a.err, kErrTimeoutPeer);
  }
  __syncthreads();
  return ok != 0;
}

template <typename T>
__global__ void ar_stage_k(const ArArgs a, const T* __restrict__ buf) {
  copy_bytes(ar_slot(a, a.rank), reinterpret_cast<const uint8_t*>(buf), a.n * (long long)sizeof(T),
             (long long)blockIdx.x * blockDim.x + threadIdx.x, (long long)gridDim.x * blockDim.x);
  ar_publish_last(a, kCommArStaged, 0);
}

template <typename T>
__global__ void ar_push_k(const ArArgs a) {
  if (!ar_wait_all(a, kCommArStaged)) return;
  // this rank's chunk [lo, hi), 8-element aligned so vector paths stay aligned
  const long long per = ((a.n + a.world - 1) / a.world + 7) / 8 * 8;
  const long long lo = min(a.n, (long long)a.rank * per), hi = min(a.n, lo + per);
  const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x, nt = (long long)gridDim.x * blockDim.x;
  constexpr int V = 16 / sizeof(T);                      // elements per 16-byte vector
  const long long nvec = (hi - lo) / V;
  for (long long v = tid; v < nvec; v += nt) {
    const long long i = lo + v * V;
    float acc[V];
#pragma unroll
    for (int j = 0; j < V; ++j) acc[j] = 0.f;
    for (int p = 0; p < a.world; ++p) {
      const uint4 raw = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(ar_slot(a, p)) + i);
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int j = 0; j < V; ++j) acc[j] += to_f<T>(e[j]);
    }
    uint4 out;
    T* o = reinterpret_cast<T*>(&out);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      if constexpr (sizeof(T) == 4) o[j] = a.scale * acc[j];
      else o[j] = f2bf(a.scale * acc[j]);
    }
    for (int p = 0; p < a.world; ++p)
      *reinterpret_cast<uint4*>(reinterpret_cast<T*>(ar_result(a, p)) + i) = out;
  }
  for (long long i = lo + nvec * V + tid; i < hi; i += nt) {      // ragged tail of the chunk
    float acc = 0.f;
    for (int p = 0; p < a.world; ++p) acc += to_f<T>(reinterpret_cast<const T*>(ar_slot(a, p))[i]);
    T r;
    if constexpr (sizeof(T) == 4) r = a.scale * acc; else r = f2bf(a.scale * acc);
    for (int p = 0; p < a.world; ++p) reinterpret_cast<T*>(ar_result(a, p))[i] = r;
  }
  ar_publish_last(a, kCommArPushed, 1);
}

template <typename T>
__global__ void ar_finish_k(const ArArgs a, T* __restrict__ buf) {
  if (!ar_wait_all(a, kCommArPushed)) return;
  copy_bytes(reinterpret_cast<uint8_t*>(buf), ar_result(a, a.rank), a.n * (long long)sizeof(T),
             (long long)blockIdx.x * blockDim.x + threadIdx.x, (long long)gridDim.x * blockDim.x);
}

int grid_for(long long bytes) {
  long long b = (bytes / 16 + 255) / 256;
  if (b < 1) b = 1;
  if (b > 1184) b = 1184;          // 8 CTAs per SM is plenty for a copy
  return static_cast<int>(b);
}

}  // namespace

int comm_all_gather(const CommPeers& peers, int rank, int world, uint32_t epoch, void* out, long long shard_bytes,
                    long long slot_cap, unsigned long long wait_ns, int* err, cudaStream_t st) {
  if (world < 2 || world > kMaxCommPeers || shard_bytes > slot_cap) return 5;
  const long long slot_off = kCommHeaderBytes + (long long)(epoch & 1u) * slot_cap;
  uint8_t* mine = peers.base[rank] + slot_off;
  uint8_t* o = static_cast<uint8_t*>(out);
  stage_k<<<grid_for(shard_bytes), 256, 0, st>>>(mine, o + (long long)rank * shard_bytes, shard_bytes);
  barrier_k<<<1, 32, 0, st>>>(peers, rank, world, kCommAgFlags, epoch, wait_ns, err);
  dim3 g(static_cast<unsigned>(grid_for(shard_bytes)), static_cast<unsigned>(world));
  gather_k<<<g, 256, 0, st>>>(peers, rank, world, slot_off, o, shard_bytes);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int comm_reduce_scatter(const CommPeers& peers, int rank, int world, uint32_t epoch, const void* in, void* out,
                        long long shard_elems, int elem_bytes, float scale, long long ag_cap, long long slot_cap,
                        unsigned long long wait_ns, int* err, cudaStream_t st) {
  const long long in_bytes = shard_elems * world * elem_bytes;
  if (world < 2 || world > kMaxCommPeers || in_bytes > slot_cap || (elem_bytes != 4 && elem_bytes != 2)) return 5;
  const long long slot_off = kCommHeaderBytes + 2 * ag_cap + (long long)(epoch & 1u) * slot_cap;
  stage_k<<<grid_for(in_bytes), 256, 0, st>>>(peers.base[rank] + slot_off, static_cast<const uint8_t*>(in),
                                              in_bytes);
  barrier_k<<<1, 32, 0, st>>>(peers, rank, world, kCommRsFlags, epoch, wait_ns, err);
  const int g = grid_for(shard_elems * elem_bytes);
  if (elem_bytes == 4)
    reduce_k<float><<<g, 256, 0, st>>>(peers, rank, world, slot_off, static_cast<float*>(out), shard_elems, scale);
  else
    reduce_k<__nv_bfloat16><<<g, 256, 0, st>>>(peers, rank, world, slot_off, static_cast<__nv_bfloat16*>(out),
                                               shard_elems, scale);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int comm_all_reduce(const CommPeers& peers, int rank, int world, uint32_t epoch, void* buf, long long n, int elem_bytes,
                    float scale, long long slot_cap, unsigned long long wait_ns, int* err, cudaStream_t st) {
  const long long bytes = n * elem_bytes;
  if (world < 2 || world > kMaxCommPeers || bytes > slot_cap || (elem_bytes != 4 && elem_bytes != 2) ||
      (reinterpret_cast<uintptr_t>(buf) & 15u) || (slot_cap & 255))
    return 5;
  if (n == 0) return 0;
  ArArgs a;
  a.peers = peers; a.rank = rank; a.world = world; a.epoch = epoch; a.n = n; a.slot_cap = slot_cap;
  a.scale = scale; a.wait_ns = wait_ns; a.err = err;
  // the waiting kernels keep their grids within one wave (one CTA per SM at most)
  const int g_copy = std::min(grid_for(bytes), 148);
  const int g_push = std::min(grid_for(bytes / world), 148);
  if (elem_bytes == 4) {
    ar_stage_k<float><<<g_copy, 256, 0, st>>>(a, static_cast<const float*>(buf));
    ar_push_k<float><<<g_push, 256, 0, st>>>(a);
    ar_finish_k<float><<<g_copy, 256, 0, st>>>(a, static_cast<float*>(buf));
  } else {
    ar_stage_k<__nv_bfloat16><<<g_copy, 256, 0, st>>>(a, static_cast<const __nv_bfloat16*>(buf));
    ar_push_k<__nv_bfloat16><<<g_push, 256, 0, st>>>(a);
    ar_finish_k<__nv_bfloat16><<<g_copy, 256, 0, st>>>(a, static_cast<__nv_bfloat16*>(buf));
  }
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

// ------------------------------------------------------- block scatter --
// Block g of `src` (blk bytes each) goes to rank g / per_rank, into its heap
// at slot_off + (g % per_rank) * dst_stride + dst_off: one pass of NVLink
// stores from this GPU, no staging.  The caller's epoch barrier publishes it.
__global__ void scatter_blocks_k(const CommPeers peers, int world, long long slot_off, const uint8_t* __restrict__ src,
                                 long long blk, int per_rank, long long dst_stride, long long dst_off) {
  const int g = blockIdx.y;
  const int owner = g / per_rank;
  if (!VAGUS_CHECK(owner, world)) return;
  uint8_t* dst = peers.base[owner] + slot_off + (long long)(g % per_rank) * dst_stride + dst_off;
  copy_bytes(dst, src + (long long)g * blk, blk, (long long)blockIdx.x * blockDim.x + threadIdx.x,
             (long long)gridDim.x * blockDim.x);
}

int comm_scatter_blocks(const CommPeers& peers, int world, long long slot_off, const void* src, long long blk_bytes,
                        int nblk, int per_rank, long long dst_stride, long long dst_off, cudaStream_t st) {
  if (world < 2 || world > kMaxCommPeers || nblk <= 0 || nblk > 65535 || per_rank <= 0 || blk_bytes <= 0 ||
      (nblk - 1) / per_rank >= world || slot_off < kCommHeaderBytes)
    return 5;
  const long long vec = (blk_bytes + 15) / 16;
  const int gx = static_cast<int>(std::min<long long>((vec + 255) / 256, std::max(1, 296 / nblk)));
  scatter_blocks_k<<<dim3(gx, nblk), 256, 0, st>>>(peers, world, slot_off, static_cast<const uint8_t*>(src), blk_bytes,
                                                  per_rank, dst_stride, dst_off);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int comm_barrier(const CommPeers& peers, int rank, int world, int flag_off, uint32_t epoch, unsigned long long wait_ns,
                 int* err, cudaStream_t st) {
  if (world < 2 || world > kMaxCommPeers || flag_off < 0 || flag_off + 4 * kMaxCommPeers > kCommHeaderBytes) return 5;
  barrier_k<<<1, 32, 0, st>>>(peers, rank, world, flag_off, epoch, wait_ns, err);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

}  // namespace vagus
