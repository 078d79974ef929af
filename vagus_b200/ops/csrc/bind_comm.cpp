// Bindings of the NVLink peer-to-peer collectives (comm.cu): heap creation
// and CUDA-IPC sharing, and the all-gather / reduce-scatter launches.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <cuda_runtime.h>

#include <cstring>
#include <string>

#include "kernels.h"

int* vagus_device_error_ptr();   // bindings.cpp

namespace {

using torch::Tensor;

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// Bound of every cross-GPU flag wait, in ns.  Ranks drift apart by seconds in
// normal operation (rank 0 writing a checkpoint, a slow read), so this is the
// process group's timeout rather than the 2 s bound of waits inside one CTA.
unsigned long long g_peer_wait_ns = 300ull * 1000000000ull;

void comm_set_wait_budget(double seconds) {
  TORCH_CHECK(seconds > 0.0 && seconds < 86400.0, "comm_set_wait_budget: seconds in (0, 86400)");
  g_peer_wait_ns = static_cast<unsigned long long>(seconds * 1e9);
}

double comm_wait_budget() { return static_cast<double>(g_peer_wait_ns) * 1e-9; }

// Allocates this rank's heap (zeroed) and returns (device pointer, IPC handle bytes).
std::tuple<int64_t, pybind11::bytes> comm_heap_create(int64_t bytes) {
  void* p = nullptr;
  TORCH_CHECK(cudaMalloc(&p, static_cast<size_t>(bytes)) == cudaSuccess, "comm heap: cudaMalloc failed");
  TORCH_CHECK(cudaMemset(p, 0, static_cast<size_t>(bytes)) == cudaSuccess, "comm heap: cudaMemset failed");
  // zeroed before any peer can map it (the flags start below every epoch)
  TORCH_CHECK(cudaDeviceSynchronize() == cudaSuccess, "comm heap: synchronise after zeroing failed");
  cudaIpcMemHandle_t h;
  TORCH_CHECK(cudaIpcGetMemHandle(&h, p) == cudaSuccess, "comm heap: cudaIpcGetMemHandle failed");
  return {reinterpret_cast<int64_t>(p), pybind11::bytes(reinterpret_cast<const char*>(&h), sizeof(h))};
}

// Maps a peer's heap into this process.
int64_t comm_heap_open(pybind11::bytes handle) {
  std::string s = handle;
  TORCH_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "comm heap: bad IPC handle");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, s.data(), sizeof(h));
  void* p = nullptr;
  TORCH_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess,
              "comm heap: cudaIpcOpenMemHandle failed");
  return reinterpret_cast<int64_t>(p);
}

void comm_heap_close(int64_t ptr, bool own) {
  if (own) cudaFree(reinterpret_cast<void*>(ptr));
  else cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr));
}

vagus::CommPeers peers_of(const std::vector<int64_t>& bases) {
  TORCH_CHECK(bases.size() >= 2 && bases.size() <= static_cast<size_t>(vagus::kMaxCommPeers), "comm: world size");
  vagus::CommPeers pr;
  for (int i = 0; i < vagus::kMaxCommPeers; ++i)
    pr.base[i] = i < static_cast<int>(bases.size()) ? reinterpret_cast<unsigned char*>(bases[i]) : nullptr;
  return pr;
}

// out (world * n elements, this rank's shard already at [rank * n, rank * n + n))
void comm_all_gather(Tensor out, std::vector<int64_t> bases, int64_t rank, int64_t epoch, int64_t slot_cap) {
  TORCH_CHECK(out.is_contiguous(), "comm_all_gather: contiguous output");
  const int world = static_cast<int>(bases.size());
  const long long total = out.numel() * out.element_size();
  TORCH_CHECK(total % world == 0, "comm_all_gather: output must split evenly");
  const int rc = vagus::comm_all_gather(peers_of(bases), static_cast<int>(rank), world, static_cast<unsigned>(epoch),
                                        out.data_ptr(), total / world, slot_cap, g_peer_wait_ns, vagus_device_error_ptr(),
                                        stream());
  TORCH_CHECK(rc == 0, "comm_all_gather failed (code ", rc, ")");
}

// in (world * n), out (n), same dtype (fp32 or bf16): out = scale * sum_r in_r[rank * n : rank * n + n]
void comm_reduce_scatter(Tensor out, Tensor in, std::vector<int64_t> bases, int64_t rank, int64_t epoch,
                         double scale, int64_t ag_cap, int64_t slot_cap) {
  TORCH_CHECK(in.is_contiguous() && out.is_contiguous() && in.scalar_type() == out.scalar_type(),
              "comm_reduce_scatter: contiguous tensors of one dtype");
  TORCH_CHECK(in.scalar_type() == at::kFloat || in.scalar_type() == at::kBFloat16, "comm_reduce_scatter: fp32 / bf16");
  const int world = static_cast<int>(bases.size());
  TORCH_CHECK(in.numel() == out.numel() * world, "comm_reduce_scatter: sizes");
  const int rc = vagus::comm_reduce_scatter(peers_of(bases), static_cast<int>(rank), world,
                                            static_cast<unsigned>(epoch), in.data_ptr(), out.data_ptr(), out.numel(),
                                            static_cast<int>(in.element_size()), static_cast<float>(scale), ag_cap,
                                            slot_cap, g_peer_wait_ns, vagus_device_error_ptr(), stream());
  TORCH_CHECK(rc == 0, "comm_reduce_scatter failed (code ", rc, ")");
}

// In-place NVLink all-reduce of a contiguous fp32 / bf16 tensor, times scale
// (heaps: header, two stage slots, two result regions of slot_cap bytes).
void comm_all_reduce(Tensor buf, std::vector<int64_t> bases, int64_t rank, int64_t epoch, double scale,
                     int64_t slot_cap) {
  TORCH_CHECK(buf.is_contiguous() && (buf.scalar_type() == at::kFloat || buf.scalar_type() == at::kBFloat16),
              "comm_all_reduce: contiguous fp32 / bf16");
  const int rc = vagus::comm_all_reduce(peers_of(bases), static_cast<int>(rank), static_cast<int>(bases.size()),
                                        static_cast<unsigned>(epoch), buf.data_ptr(), buf.numel(),
                                        static_cast<int>(buf.element_size()), static_cast<float>(scale), slot_cap,
                                        g_peer_wait_ns, vagus_device_error_ptr(), stream());
  TORCH_CHECK(rc == 0, "comm_all_reduce failed (code ", rc, ")");
}

// Epoch barrier over the heaps (the generic flag block).
void comm_barrier(std::vector<int64_t> bases, int64_t rank, int64_t epoch) {
  const int rc = vagus::comm_barrier(peers_of(bases), static_cast<int>(rank), static_cast<int>(bases.size()),
                                     vagus::kCommBarFlags, static_cast<unsigned>(epoch), g_peer_wait_ns,
                                     vagus_device_error_ptr(), stream());
  TORCH_CHECK(rc == 0, "comm_barrier failed (code ", rc, ")");
}

// Push the blocks of a contiguous tensor to their owners' heaps (see comm.cu).
void comm_scatter_blocks(std::vector<int64_t> bases, int64_t slot_off, Tensor src, int64_t blk_bytes, int64_t nblk,
                         int64_t per_rank, int64_t dst_stride, int64_t dst_off) {
  TORCH_CHECK(src.is_cuda() && src.is_contiguous() && src.numel() * src.element_size() >= blk_bytes * nblk,
              "comm_scatter_blocks: contiguous CUDA source of nblk blocks");
  const int rc = vagus::comm_scatter_blocks(peers_of(bases), static_cast<int>(bases.size()), slot_off, src.data_ptr(),
                                            blk_bytes, static_cast<int>(nblk), static_cast<int>(per_rank), dst_stride,
                                            dst_off, stream());
  TORCH_CHECK(rc == 0, "comm_scatter_blocks failed (code ", rc, ")");
}

// A tensor over `numel` elements of this process's heap at byte offset
// `offset` (no ownership: the heap outlives it).
Tensor comm_heap_view(int64_t ptr, int64_t offset, int64_t numel, at::ScalarType dtype) {
  const int64_t es = c10::elementSize(dtype);
  TORCH_CHECK(offset % es == 0 && numel >= 0, "comm_heap_view: alignment");
  int dev = 0;
  cudaGetDevice(&dev);
  auto opts = torch::TensorOptions().dtype(dtype).device(torch::kCUDA, dev);
  return torch::from_blob(reinterpret_cast<char*>(ptr) + offset, {numel}, [](void*) {}, opts);
}

}  // namespace

void register_comm_ops(pybind11::module& m) {
  m.def("comm_barrier", &comm_barrier);
  m.def("comm_scatter_blocks", &comm_scatter_blocks);
  m.def("comm_set_wait_budget", &comm_set_wait_budget, "bound of cross-GPU flag waits, seconds");
  m.def("comm_wait_budget", &comm_wait_budget);
  m.def("comm_heap_view", &comm_heap_view);
  m.def("comm_heap_create", &comm_heap_create);
  m.def("comm_heap_open", &comm_heap_open);
  m.def("comm_heap_close", &comm_heap_close);
  m.def("comm_all_gather", &comm_all_gather);
  m.def("comm_all_reduce", &comm_all_reduce);
  m.def("comm_reduce_scatter", &comm_reduce_scatter);
}
