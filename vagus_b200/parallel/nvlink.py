"""FSDP2's parameter all-gather and gradient reduce-scatter on our own NVLink
peer-to-peer kernels (``ops/csrc/comm.cu``) instead of NCCL.

FSDP2 lets a module take custom collective objects
(``FSDPModule.set_custom_all_gather`` / ``set_custom_reduce_scatter``);
``use_nvlink_collectives(root, group)`` installs ours on every FSDP unit of a
model.  Each rank allocates one device heap (plain ``cudaMalloc``), shares it
with the other ranks of the group through CUDA IPC (no NVLink multicast
objects), and every collective is three launches on the stream FSDP chose:
stage this rank's contribution into its heap slot, a cross-GPU epoch barrier
(bounded wait; a timeout sets the device error word that
``ops.check_error()`` raises), and the combine step that reads the peers'
slots over NVLink (all-gather: copy into place; reduce-scatter: fp32 sum of
this rank's rows, scale by 1 / world for an average, cast).

Calls the kernels cannot take (a reduction other than sum / average, a
buffer larger than the heap slots) go to NCCL; the decision depends only on
sizes and the op, which are identical on every rank, so the per-kind epoch
counters stay in step.

``MuonExchange`` is the fused product + all-to-all of the sharded Muon
step: the last Newton-Schulz GEMM of each orthogonalised matrix scatters its
output rows from the epilogue straight into the owning ranks' receive buffers
(peer stores over NVLink), then one epoch barrier.

``PeerRowShards`` is the all-gather fused into the consuming GEMM: a weight's
row shards stay in the peers' heaps and the gathered-B GEMM reads them in
place through per-owner TMA maps; ``unit_gather_layout`` gives where each
FSDP2-managed parameter's shard sits in the all-gather staging slots.
``NvlinkAllReduce`` is the all-reduce on the same heaps: DDP's bucket
all-reduce (as a DDP communication hook), FSDP's replicated-parameter
average and the gradient-norm sum.  ``set_dry_run`` switches the FSDP2
hooks off for the exposed-communication probe of ``bench.py``.

Parity: the reference runs these collectives inside FSDP2 on NCCL
(``infra/train/main.py:253-275``); the gradient reduction semantics (average
over the data-parallel group, fp32) are the same.  Its sharded Muon
(``infra/optimizer/muon.py``) all-gathers the Newton-Schulz results; the
update each rank applies is the same.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch.distributed.fsdp._fully_shard._fsdp_api import AllGather, ReduceScatter

from ..ops import native

HEADER = 1024                      # flag words, as comm.cu lays them out

# Bound of every cross-GPU flag wait in the kernels, in seconds.  Ranks drift
# apart by seconds in normal operation (rank 0 writing a checkpoint, a slow
# data read, garbage collection), so the bound is the process group's
# timeout, not the 2 s bound of the waits inside one CTA.
_PEER_WAIT_S = 300.0


def set_peer_wait_seconds(seconds: float) -> None:
    """Bound of the cross-GPU waits of the NVLink collectives (the process
    group's timeout); on expiry the device error word is set and
    ``ops.check_error()`` raises."""
    global _PEER_WAIT_S
    _PEER_WAIT_S = float(seconds)
    from ..ops import _core
    if _core._C is not None:
        _core._C.comm_set_wait_budget(_PEER_WAIT_S)


def open_heaps(group, nbytes: int) -> tuple[int, list[int]]:
    """Allocate this rank's zeroed device heap of ``nbytes``, share it with
    the group over CUDA IPC and map every peer's: (own pointer, every rank's
    base in this process).  Collective over ``group``."""
    C = native()
    C.comm_set_wait_budget(_PEER_WAIT_S)
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    ptr, handle = C.comm_heap_create(int(nbytes))
    handles = [None] * world
    dist.all_gather_object(handles, handle, group=group)
    bases = [ptr if r == rank else C.comm_heap_open(h) for r, h in enumerate(handles)]
    dist.barrier(group=group)
    return ptr, bases


def close_heaps(own: int, bases: list[int]) -> None:
    C = native()
    for b in bases:
        C.comm_heap_close(b, b == own)


_SAME_HOST: dict = {}


def same_host(group) -> bool:
    """True when every rank of ``group`` runs on this machine (CUDA IPC, and
    so these kernels, only reach GPUs of one node).  Collective over the
    group; cached per group."""
    key = id(group)
    if key not in _SAME_HOST:
        import socket
        names = [None] * dist.get_world_size(group)
        dist.all_gather_object(names, socket.gethostname(), group=group)
        _SAME_HOST[key] = len(set(names)) == 1
    return _SAME_HOST[key]


class NvlinkHeap:
    """One IPC-shared device heap per rank of ``group``: 2 all-gather slots of
    ``ag_cap`` bytes and 2 reduce-scatter slots of ``rs_cap`` bytes."""

    def __init__(self, group, ag_cap: int, rs_cap: int):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.ag_cap = (int(ag_cap) + 255) // 256 * 256
        self.rs_cap = (int(rs_cap) + 255) // 256 * 256
        self.own, self.bases = open_heaps(group, HEADER + 2 * self.ag_cap + 2 * self.rs_cap)
        self.ag_epoch = 0
        self.rs_epoch = 0

    def close(self):
        close_heaps(self.own, self.bases)
        self.bases = []


_DRY_RUN = False


def set_dry_run(on: bool) -> None:
    """Timing probe: while on, the FSDP2 all-gather / reduce-scatter hooks
    return without communicating (parameters and gradients are then garbage),
    so a step timed in this mode is the step's compute alone and the
    difference to a normal step is its exposed communication."""
    global _DRY_RUN
    _DRY_RUN = bool(on)


class NvlinkAllGather(AllGather):
    def __init__(self, heap: NvlinkHeap):
        self.heap = heap

    def allocate(self, size, *, dtype, device):
        return torch.empty(*size, dtype=dtype, device=device)

    def __call__(self, output_tensor, input_tensor, group, async_op: bool = False):
        if _DRY_RUN:
            return None
        h = self.heap
        shard_bytes = input_tensor.numel() * input_tensor.element_size()
        if shard_bytes > h.ag_cap or not output_tensor.is_contiguous():
            return dist.all_gather_into_tensor(output_tensor, input_tensor, group=group, async_op=async_op)
        n = input_tensor.numel()
        mine = output_tensor.view(-1)[h.rank * n:(h.rank + 1) * n]
        if mine.data_ptr() != input_tensor.data_ptr():
            mine.copy_(input_tensor.view(-1))
        h.ag_epoch += 1
        native().comm_all_gather(output_tensor, h.bases, h.rank, h.ag_epoch, h.ag_cap)
        return None


class NvlinkReduceScatter(ReduceScatter):
    def __init__(self, heap: NvlinkHeap):
        self.heap = heap

    def allocate(self, size, *, dtype, device):
        return torch.empty(*size, dtype=dtype, device=device)

    def __call__(self, output_tensor, input_tensor, group, op, async_op: bool = False):
        if _DRY_RUN:
            return None
        h = self.heap
        if op == dist.ReduceOp.SUM:
            scale = 1.0
        elif op == dist.ReduceOp.AVG:
            scale = 1.0 / h.world
        else:
            scale = None
        nbytes = input_tensor.numel() * input_tensor.element_size()
        if (scale is None or nbytes > h.rs_cap or input_tensor.dtype not in (torch.float32, torch.bfloat16)
                or input_tensor.dtype != output_tensor.dtype):
            return dist.reduce_scatter_tensor(output_tensor, input_tensor, op=op, group=group, async_op=async_op)
        h.rs_epoch += 1
        native().comm_reduce_scatter(output_tensor, input_tensor.contiguous(), h.bases, h.rank, h.rs_epoch, scale,
                                     h.ag_cap, h.rs_cap)
        return None


class NvlinkAllReduce:
    """In-place all-reduce (sum or average) of fp32 / bf16 tensors over a
    group on our NVLink kernels (``comm.cu``: stage into this rank's heap
    slot, each rank reduces its 1/world chunk over the peers' slots in fp32
    and stores the result into every rank's result region, copy out -- three
    launches, the 1/world of an average folded into the reduction).

    Tensors that are not contiguous, not 16-byte aligned or larger than the
    heap's slots go to NCCL; the choice depends only on sizes and dtypes,
    which are the same on every rank.  ``ddp_hook`` is a DDP communication
    hook (``DistributedDataParallel.register_comm_hook``) averaging each
    gradient bucket this way."""

    def __init__(self, group, cap_bytes: int):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.slot = (int(cap_bytes) + 255) // 256 * 256
        self.own, self.bases = open_heaps(group, HEADER + 4 * self.slot)
        self.epoch = 0
        self.calls = {"nvlink": 0, "nccl": 0}

    def __call__(self, t: torch.Tensor, op=dist.ReduceOp.AVG) -> None:
        ok = (op in (dist.ReduceOp.SUM, dist.ReduceOp.AVG) and t.is_cuda and t.is_contiguous()
              and t.dtype in (torch.float32, torch.bfloat16) and t.numel() * t.element_size() <= self.slot
              and t.data_ptr() % 16 == 0)
        if not ok:
            self.calls["nccl"] += 1
            dist.all_reduce(t, op=op, group=self.group)
            return
        self.calls["nvlink"] += 1
        self.epoch += 1
        scale = 1.0 / self.world if op == dist.ReduceOp.AVG else 1.0
        native().comm_all_reduce(t, self.bases, self.rank, self.epoch, scale, self.slot)

    def ddp_hook(self, _state, bucket):
        # no return annotation: DDP's hook check accepts only none or exactly Future[Tensor]
        buf = bucket.buffer()
        if not buf.is_cuda:
            self(buf, dist.ReduceOp.AVG)
            fut = torch.futures.Future()
            fut.set_result(buf)
            return fut
        # On a side stream, so the bucket's all-reduce overlaps the rest of the
        # backward (as DDP's own NCCL all-reduce does).  The future is
        # CUDA-aware: setting it inside the side stream records an event there,
        # and whoever waits on it (DDP copying the bucket back into the
        # gradients) waits for that event on its own stream.
        side = self._side_stream(buf.device)
        side.wait_stream(torch.cuda.current_stream(buf.device))
        with torch.cuda.stream(side):
            self(buf, dist.ReduceOp.AVG)
            fut = torch.futures.Future(devices=[buf.device])
            fut.set_result(buf)
        return fut

    def _side_stream(self, device):
        st = getattr(self, "_stream", None)
        if st is None or st.device != device:
            st = torch.cuda.Stream(device=device)
            self._stream = st
        return st

    def close(self) -> None:
        close_heaps(self.own, self.bases)
        self.bases = []


def ddp_bucket_cap(model, bucket_cap_mb: float = 25.0) -> int:
    """Bytes a DDP gradient bucket can reach: a bucket closes once it holds
    ``bucket_cap_mb``, so it is at most that plus the largest parameter."""
    largest = max((p.numel() * p.element_size() for p in model.parameters() if p.requires_grad), default=0)
    return int(bucket_cap_mb * 2 ** 20) + largest


def _unit_sizes(root, world: int):
    """Largest FSDP unit (sum of padded parameter numels) among the blocks
    and the root's own parameters; 1-D parameters are replicated, not sharded."""
    from torch.distributed.fsdp import FSDPModule

    def managed(mod, skip):
        total = 0
        for p in mod.parameters():
            if id(p) in skip or p.dim() < 2:
                continue
            d0 = p.shape[0]
            total += ((d0 + world - 1) // world * world) * (p.numel() // max(1, d0))
        return total

    units = [m for m in root.modules() if isinstance(m, FSDPModule)]
    seen: set = set()
    sizes = []
    for m in units:
        if m is root:
            continue
        sizes.append(managed(m, seen))
        seen.update(id(p) for p in m.parameters())
    sizes.append(managed(root, seen))
    return max(sizes) if sizes else 0


def use_nvlink_collectives(root, group=None) -> NvlinkHeap:
    """Install the NVLink collectives on every FSDP unit under ``root``
    (after ``fully_shard``).  Returns the heap (keep it alive), or None when
    the group spans several machines (NCCL stays in place)."""
    from torch.distributed.fsdp import FSDPModule
    group = group or dist.group.WORLD
    if not same_host(group):
        return None                      # ranks on several machines: FSDP2 keeps NCCL
    world = dist.get_world_size(group)
    biggest = _unit_sizes(root, world)
    heap = NvlinkHeap(group, ag_cap=(biggest // world + 64) * 4, rs_cap=(biggest + 64 * world) * 4)
    ag, rs = NvlinkAllGather(heap), NvlinkReduceScatter(heap)
    for m in root.modules():
        if isinstance(m, FSDPModule):
            m.set_custom_all_gather(ag)
            m.set_custom_reduce_scatter(rs)
    return heap


def unit_gather_layout(unit) -> list[dict]:
    """Where each parameter that FSDP2 manages in ``unit`` sits in a rank's
    flat all-gather input -- and so in every peer's all-gather staging slot,
    which is what a GEMM that reads a weight's row shards in place needs:
    FSDP2 concatenates the parameters' dim-0 shards, each padded to
    ``ceil(rows / world)`` rows, in its parameter order.

    One dict per parameter: ``name`` (relative to ``unit``), ``param`` (the
    sharded parameter), ``offset`` (elements of the flat input), ``rows``
    (padded rows per rank), ``shape`` (unsharded) and ``numel``."""
    group = unit._get_fsdp_state()._fsdp_param_group
    out: list[dict] = []
    if group is None:
        return out
    names = {id(p): n for n, p in unit.named_parameters()}
    off = 0
    for fp in group.fsdp_params:
        size = fp.padded_sharded_param_size
        p = fp.sharded_param
        out.append(dict(name=names.get(id(p)), param=p, offset=off, rows=int(size[0]) if len(size) else 0,
                        shape=tuple(fp._orig_size), numel=int(size.numel())))
        off += int(size.numel())
    return out


class MuonExchange:
    """IPC-shared receive buffers for the sharded Muon step: the momentum
    row shards pushed to the matrices' owners (``push_inputs``, in place of an
    all-gather), and the fused Newton-Schulz product + scatter of the results
    (a GEMM followed by an all-to-all, as one kernel over NVLink).

    Each rank's heap holds two slots (alternating by epoch) of ``slot_bytes``;
    a bucket of ``n`` same-shape matrices, row-sharded ``world`` ways, owns a
    block of ``n_pad x rows_l x cols`` bf16 in every slot (``n_pad`` = the
    bucket padded to a multiple of ``world``).  The rank that orthogonalises
    matrix ``g`` writes its rows ``[o rows_l, (o + 1) rows_l)`` into rank
    ``o``'s block at ``g`` (for a tall matrix, processed transposed, the
    column block, stored as ``cols x rows_l``).  A slot is rewritten two
    epochs later, after every peer passed the barrier in between, which it
    reaches only after applying what it read from the slot."""

    def __init__(self, group, slot_bytes: int):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.slot_bytes = (int(slot_bytes) + 255) // 256 * 256
        self.own, self.bases = open_heaps(group, HEADER + 2 * self.slot_bytes)
        self.epoch = 0

    @staticmethod
    def eligible(shape, world: int, device) -> bool:
        rows, cols = shape
        if world < 2 or world > 16 or device.type != "cuda" or rows % world or rows % 8 or cols % 8:
            return False
        rows_l = rows // world
        # a tall matrix scatters 32-column chunks of its transposed product
        return rows <= cols or rows_l % 32 == 0

    @staticmethod
    def block_bytes(n_pad: int, rows_l: int, cols: int) -> int:
        return (n_pad * rows_l * cols * 2 + 255) // 256 * 256

    def _slot(self, epoch: int) -> int:
        return HEADER + (epoch & 1) * self.slot_bytes

    def scatter_fn(self, off: int, batch0: int, rows_l: int, cols: int, transposed: bool):
        """The final product X' = B X + a X of ``_ns_kernels``, scattered into
        the next epoch's slot of every rank."""
        slot = self._slot(self.epoch + 1)
        dst = [b + slot + off for b in self.bases]
        if transposed:      # X' is (cols, rows): column blocks of rows_l, stored (cols, rows_l)
            mode, ld, stride = 2, rows_l, cols * rows_l
        else:               # X' is (rows, cols): row blocks of rows_l, stored (rows_l, cols)
            mode, ld, stride = 1, cols, rows_l * cols

        def last(Bm, X, a):
            rc = native().gemm_scatter(Bm, False, X, True, X, 1.0, a, dst, mode, rows_l, ld, stride, batch0)
            if rc:
                raise RuntimeError(f"gemm_scatter rejected the problem (code {rc})")
        return last

    def push_inputs(self, off: int, local: torch.Tensor, chunk: int) -> None:
        """Send this rank's row shard of each of a bucket's matrices to the
        matrix's owner (the rank that orthogonalises it): matrix g of ``local``
        (n, rows_l, cols) bf16 lands in rank ``g // chunk``'s block at
        ``(g % chunk, rank rows_l : (rank + 1) rows_l)``, laid out (chunk, rows,
        cols), in the next epoch's slot.  Only the owner's rows cross NVLink,
        1/world of what an all-gather of every full momentum moves."""
        n, rows_l, cols = local.shape
        rows = rows_l * self.world
        blk = rows_l * cols * 2
        native().comm_scatter_blocks(self.bases, self._slot(self.epoch + 1), local.contiguous(), blk, n, chunk,
                                     rows * cols * 2, off + self.rank * blk)

    def received_inputs(self, off: int, n: int, chunk: int, rows: int, cols: int) -> torch.Tensor:
        """This rank's ``chunk`` full matrices of the bucket, (chunk, rows,
        cols) bf16 in the heap; the padding past the bucket's ``n`` matrices is
        zeroed (nobody sends it)."""
        t = native().comm_heap_view(self.own, self._slot(self.epoch) + off, chunk * rows * cols,
                                    torch.bfloat16).view(chunk, rows, cols)
        real = max(0, min(chunk, n - self.rank * chunk))
        if real < chunk:
            t[real:].zero_()
        return t

    def barrier(self):
        self.epoch += 1
        native().comm_barrier(self.bases, self.rank, self.epoch)

    def received(self, off: int, n: int, rows_l: int, cols: int, transposed: bool) -> torch.Tensor:
        """This rank's rows of the bucket's n matrices, (n, rows_l, cols) bf16."""
        t = native().comm_heap_view(self.own, self._slot(self.epoch) + off, n * rows_l * cols, torch.bfloat16)
        return t.view(n, cols, rows_l).transpose(1, 2) if transposed else t.view(n, rows_l, cols)

    def close(self):
        close_heaps(self.own, self.bases)
        self.bases = []


class PeerRowShards:
    """A weight whose row shards live in the CUDA-IPC heaps of a group's GPUs
    and are read in place by the GEMM that consumes the weight: the
    all-gather fused into that GEMM (``gemm_gather``: per-owner TMA maps over
    the peers' shards, no multicast), so the gathered weight is never
    materialised and its bytes cross NVLink inside the product's loads.

    Rank r holds rows ``[r rows, (r + 1) rows)`` of a ``(world rows, cols)``
    bf16 matrix (``rows`` a multiple of 8, at least 128).  ``publish()`` is
    the epoch barrier after which the peers may read updated shards;
    ``linear(x, n)`` is ``x @ W[:n]^T``."""

    def __init__(self, group, rows: int, cols: int):
        assert rows % 8 == 0 and rows >= 128 and cols % 8 == 0 and cols >= 64, "shard shape"
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        assert self.world <= 8, "at most 8 owners"
        if not same_host(group):
            raise RuntimeError("PeerRowShards: CUDA IPC reaches the GPUs of one machine only")
        self.rows, self.cols = rows, cols
        self.own, self.bases = open_heaps(group, HEADER + (rows * cols * 2 + 255) // 256 * 256)
        self.epoch = 0

    def local(self) -> torch.Tensor:
        """This rank's shard, (rows, cols) bf16, writable in place."""
        return native().comm_heap_view(self.own, HEADER, self.rows * self.cols, torch.bfloat16).view(self.rows,
                                                                                                     self.cols)

    def publish(self) -> None:
        self.epoch += 1
        native().comm_barrier(self.bases, self.rank, self.epoch)

    def linear(self, x: torch.Tensor, n: int | None = None, out_dtype=torch.bfloat16) -> torch.Tensor:
        n = self.world * self.rows if n is None else n
        x2 = x.reshape(-1, self.cols)
        if x2.dtype != torch.bfloat16 or x2.stride(-1) != 1:
            x2 = x2.to(torch.bfloat16).contiguous()
        out = torch.empty(x2.shape[0], n, device=x.device, dtype=out_dtype)
        rc = native().gemm_gather(x2, False, [b + HEADER for b in self.bases], self.rows, self.cols, out)
        if rc:
            raise RuntimeError(f"gemm_gather rejected the problem (code {rc})")
        return out.view(*x.shape[:-1], n)

    def close(self) -> None:
        close_heaps(self.own, self.bases)
        self.bases = []
