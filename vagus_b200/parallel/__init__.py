"""Data parallelism: one process per GPU, ``torch.distributed`` (NCCL on GPU,
gloo on CPU) for the plumbing.

* DDP (``shard_size`` 1): every rank holds the full fp32 model; gradients are
  averaged by bucketed all-reduces overlapped with backward.
* FSDP2 / HSDP (``shard_size`` > 1): a 2-D (replicate, shard) device mesh;
  parameters, gradients and optimizer state are row-sharded over the shard
  group (fp32 masters, a bf16 copy all-gathered per block for compute, fp32
  gradient reduce-scatter) and replicated across groups.  The 1-D parameters
  stay replicated fp32 and are averaged by one flat all-reduce.

Parity: reference ``infra/train/main.py:195-339`` (setup_distributed,
build_mesh, LMLoss, apply_fsdp, reduce_replicated, unwrap, unsharded,
clip_grad_norm).
"""

from __future__ import annotations

import datetime
import os
from contextlib import contextmanager, nullcontext
from typing import cast

import torch
import torch.distributed as dist
from torch import nn

try:
    from torch.distributed.device_mesh import DeviceMesh, init_device_mesh
    from torch.distributed.fsdp import FSDPModule, MixedPrecisionPolicy, fully_shard
    from torch.distributed.tensor import DTensor
except ImportError:  # pragma: no cover
    DeviceMesh = FSDPModule = DTensor = object  # type: ignore
    init_device_mesh = fully_shard = MixedPrecisionPolicy = None  # type: ignore

DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


def setup_distributed(device: str = "auto", timeout_s: float | None = None):
    """(rank, world, device, is_dist).  Under torchrun (RANK / WORLD_SIZE in
    the environment) the process group is NCCL on GPU, gloo on CPU."""
    if "RANK" in os.environ and "WORLD_SIZE" in os.environ:
        rank = int(os.environ["RANK"])
        world = int(os.environ["WORLD_SIZE"])
        local = int(os.environ.get("LOCAL_RANK", 0))
        kw = {}
        if timeout_s is not None:
            kw["timeout"] = datetime.timedelta(seconds=timeout_s)
            from .nvlink import set_peer_wait_seconds
            set_peer_wait_seconds(timeout_s)        # our kernels' cross-GPU waits end with the group's
        if torch.cuda.is_available():
            dev = torch.device(f"cuda:{local}")
            torch.cuda.set_device(dev)
            if not dist.is_initialized():
                dist.init_process_group(backend="nccl", device_id=dev, **kw)
        else:
            dev = torch.device("cpu")
            if not dist.is_initialized():
                dist.init_process_group(backend="gloo", **kw)
        return rank, world, dev, True
    if device != "auto":
        dev = torch.device(device)
    elif torch.cuda.is_available():
        dev = torch.device("cuda")
    else:
        dev = torch.device("cpu")
    return 0, 1, dev, False


def build_mesh(shard_size: int, device: torch.device, world: int):
    """2-D (replicate, shard) mesh for FSDP2 / HSDP; None for DDP.  Rank r
    sits at (r // shard_size, r % shard_size)."""
    if shard_size <= 1:
        return None
    if world % shard_size:
        raise ValueError(f"world_size {world} is not a multiple of shard_size {shard_size}")
    return init_device_mesh(device.type, (world // shard_size, shard_size), mesh_dim_names=("replicate", "shard"))


class LMLoss(nn.Module):
    """FSDP2 root: forward computes the loss (the fused CE reads the tied head
    weight, which is only unsharded inside the root's forward)."""

    def __init__(self, module: nn.Module, ce_fn):
        super().__init__()
        self.module = module
        self.ce_fn = ce_fn
        self.replicated: list[nn.Parameter] = []

    def forward(self, x, y):
        hidden = self.module(x, return_hidden=True)
        return self.ce_fn(hidden, self.module.head.weight, y)


def apply_fsdp(root: LMLoss, mesh, param_dtype: str = "bfloat16", reduce_dtype: str = "float32",
               reshard_after_forward: bool = True, comm: str = "nccl") -> None:
    """One FSDP2 unit per block plus the root; every 1-D parameter is left out
    (replicated fp32, averaged by ``reduce_replicated``).

    ``comm="nvlink"`` runs FSDP2's parameter all-gathers and gradient
    reduce-scatters on our NVLink peer-to-peer kernels (``parallel.nvlink``)
    instead of NCCL; it applies to a 1-D (pure FSDP) mesh on CUDA, and a 2-D
    HSDP mesh keeps NCCL."""
    pd, rd = DTYPES[param_dtype], DTYPES[reduce_dtype]
    blocks_mp = MixedPrecisionPolicy(param_dtype=None if pd is torch.float32 else pd, reduce_dtype=rd,
                                     cast_forward_inputs=False)
    root_mp = MixedPrecisionPolicy(param_dtype=None, reduce_dtype=rd, cast_forward_inputs=False)
    root.replicated = [p for p in root.parameters() if p.dim() < 2]
    ignored = set(root.replicated)
    for blk in root.module.blocks:
        fully_shard(blk, mesh=mesh, mp_policy=blocks_mp, ignored_params=ignored,
                    reshard_after_forward=reshard_after_forward)
    fully_shard(root, mesh=mesh, mp_policy=root_mp, ignored_params=ignored)
    root.nvlink_heap = None
    root.nvlink_allreduce = None
    if comm == "nvlink" and mesh.ndim == 1 and mesh.device_type == "cuda" and mesh.size() > 1:
        from .nvlink import NvlinkAllReduce, use_nvlink_collectives
        root.nvlink_heap = use_nvlink_collectives(root, mesh.get_group())
        if root.nvlink_heap is not None:
            # the replicated 1-D gradients and the gradient-norm partial sums
            cap = sum(p.numel() * 4 for p in root.replicated) + 4096
            root.nvlink_allreduce = NvlinkAllReduce(mesh.get_group(), cap)
    elif comm not in ("nccl", "nvlink"):
        raise ValueError(f"unknown FSDP collective backend {comm!r} (nccl | nvlink)")


def wrap_ddp(model: nn.Module, device: torch.device, comm: str = "nvlink") -> nn.Module:
    """torch DDP around ``model``; with ``comm="nvlink"`` (CUDA, one machine)
    its bucket all-reduce runs on our NVLink all-reduce kernels through a DDP
    communication hook instead of NCCL."""
    from torch.nn.parallel import DistributedDataParallel as DDP
    cuda = device.type == "cuda"
    ddp = DDP(model, device_ids=[device.index] if cuda else None, output_device=device.index if cuda else None)
    ddp.nvlink_allreduce = None
    if comm == "nvlink" and cuda:
        from .nvlink import NvlinkAllReduce, ddp_bucket_cap, same_host
        if same_host(dist.group.WORLD):
            ar = NvlinkAllReduce(dist.group.WORLD, ddp_bucket_cap(model))
            ddp.register_comm_hook(None, ar.ddp_hook)
            ddp.nvlink_allreduce = ar
    elif comm not in ("nccl", "nvlink"):
        raise ValueError(f"unknown DDP collective backend {comm!r} (nccl | nvlink)")
    return ddp


def _all_reduce(model: nn.Module, t: torch.Tensor, op=dist.ReduceOp.AVG, group=None) -> None:
    """All-reduce through the model's NVLink all-reduce when it has one."""
    ar = getattr(model, "nvlink_allreduce", None)
    if ar is not None and group is None:
        ar(t, op)
    else:
        dist.all_reduce(t, op=op, group=group)


def reduce_replicated(root: LMLoss, mesh=None) -> None:
    grads = [p.grad for p in root.replicated if p.grad is not None]
    if not grads:
        return
    flat = torch.cat([g.flatten() for g in grads])
    _all_reduce(root, flat, dist.ReduceOp.AVG)
    torch._foreach_copy_(grads, list(flat.split([g.numel() for g in grads])))


def unwrap(model: nn.Module) -> nn.Module:
    model = getattr(model, "_orig_mod", model)
    return getattr(model, "module", model)


def optimizer_members(optimizer) -> list:
    return list(getattr(optimizer, "members", [optimizer]))


@contextmanager
def unsharded(model: nn.Module, compute=None):
    units = [m for m in model.modules() if isinstance(m, FSDPModule)]
    for m in units:
        m.unshard()
    try:
        with (compute if compute is not None else nullcontext()):
            yield
    finally:
        for m in units:
            m.reshard()


def clip_grad_norm(model: nn.Module, max_norm: float | None) -> torch.Tensor:
    """Global grad norm (DTensor-aware), clipped in place when max_norm is set."""
    params = [p for p in model.parameters() if p.grad is not None]
    sharded = [p for p in params if isinstance(p.grad, DTensor)]
    plain = [p for p in params if not isinstance(p.grad, DTensor)]
    sq = torch.zeros((), device=params[0].grad.device if params else "cpu")
    ar = getattr(model, "nvlink_allreduce", None)
    if sharded and ar is not None:
        # pure FSDP on NVLink: the local shards' squared norm, summed by one all-reduce on our kernel
        local = [p.grad.to_local() for p in sharded]
        part = torch.stack(torch._foreach_norm([t.float() for t in local])).square().sum().reshape(1)
        ar(part, dist.ReduceOp.SUM)
        sq = sq + part[0]
    for group in ((plain,) if sharded and ar is not None else (sharded, plain)):
        if group:
            n = torch.nn.utils.get_total_norm(cast(list, [p.grad for p in group]), 2.0)
            if isinstance(n, DTensor):
                n = n.full_tensor()
            sq = sq + n.float() ** 2
    total = sq.sqrt()
    if max_norm is not None:
        for group in (sharded, plain):
            if group:
                torch.nn.utils.clip_grads_with_norm_(group, max_norm, total)
    return total
