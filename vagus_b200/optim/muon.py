"""Muon: momentum orthogonalised by a quintic Newton-Schulz iteration, for the
2-D block matrices (everything else trains under AdamW; ``MuonAdamW`` presents
the pair as one optimizer).

Newton-Schulz runs in bf16 on the tcgen05 GEMM when the update lives on a
CUDA device, batched over every same-shape matrix of a bucket:

    A = X X^T            (gram, K-major operands)
    B = b A + c A A      (A symmetric: A A = A A^T, fused alpha/beta epilogue)
    X = a X + B X        (X read N-contiguous, fused alpha/beta epilogue)

Two distributed regimes, per parameter type:
* plain tensors (single GPU, DDP): every rank holds the full gradient; the
  Newton-Schulz *work* is split across ranks (each orthogonalises a
  ceil(n / world) slice of each bucket, zero padded) and the slices are
  all-gathered so every replica applies byte-identical updates;
* DTensors (FSDP2 / HSDP row shards): momentum and decay stay on the local
  shard; the bf16 momentum rows of a bucket are all-gathered over the shard
  group, the Newton-Schulz work is split, the outputs all-gathered back and
  each rank applies its own rows.

Parity: reference ``infra/optimizer/muon.py:42-420`` (coefficient schemes,
functional updates, lr adjustment, Muon, MuonAdamW).
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor
from torch.optim.optimizer import Optimizer

try:
    from torch.distributed.tensor import DTensor, Shard
except ImportError:  # pragma: no cover
    DTensor = type("DTensor", (), {})
    Shard = type("Shard", (), {})

# (a, b, c) per iteration, plus the norm slack the schedule was tuned under.
# 'jordan': the constant quintic of Jordan et al. (repeated ns_steps times);
# 'polar_express': the 5-step minimax schedule of Amsel et al.
# (arXiv:2505.16932) as published by modded-nanogpt.
NS_SCHEMES: dict[str, tuple[list[tuple[float, float, float]], float]] = {
    "jordan": ([(3.4445, -4.7750, 2.0315)], 0.0),
    "polar_express": ([
        (8.156554524902461, -22.48329292557795, 15.878769915207462),
        (4.042929935166739, -2.808917465908714, 0.5000178451051316),
        (3.8916678022926607, -2.772484153217685, 0.5060648178503393),
        (3.285753657755655, -2.3681294933425376, 0.46449024233003106),
        (2.3465413258596377, -1.7097828382687081, 0.42323551169305323),
    ], 2e-2),
}


def _ns_torch(X: Tensor, coeffs) -> Tensor:
    for a, b, c in coeffs:
        A = X @ X.mT
        X = a * X + (b * A + c * (A @ A)) @ X
    return X


def _ns_kernels(X: Tensor, coeffs, last=None) -> Tensor | None:
    """Newton-Schulz on the tcgen05 GEMM.  With ``last``, the final product
    X' = B X + a X is not formed here: ``last(B, X, a)`` is called instead
    (the fused product + scatter over NVLink) and None is returned."""
    from ..ops._core import gemm
    batched = X.dim() == 3
    Xb = X if batched else X[None]
    Xb = Xb.contiguous()
    n, m, k = Xb.shape
    A = torch.empty(n, m, m, device=X.device, dtype=torch.bfloat16)
    Bm = torch.empty_like(A)
    Y = torch.empty_like(Xb)
    for i, (a, b, c) in enumerate(coeffs):
        gemm(Xb, False, Xb, False, A)                              # A = X X^T
        gemm(A, False, A, False, Bm, S=A, alpha=c, beta=b)         # B = c A A^T + b A
        if last is not None and i == len(coeffs) - 1:
            last(Bm, Xb, a)
            return None
        gemm(Bm, False, Xb, True, Y, S=Xb, alpha=1.0, beta=a)      # X' = B X + a X
        Xb, Y = Y, Xb
    return Xb if batched else Xb[0]


def _ns_prepare(G: Tensor, steps: int, eps: float, scheme: str):
    """(X, coeffs, transposed): G in bf16, wide orientation, Frobenius-normalised."""
    coeffs, slack = NS_SCHEMES[scheme]
    if len(coeffs) == 1:
        coeffs = coeffs * steps
    X = G.to(torch.bfloat16)
    transposed = X.size(-2) > X.size(-1)
    if transposed:
        X = X.mT
    X = X / (X.norm(dim=(-2, -1), keepdim=True) * (1 + slack) + eps)
    return X, coeffs, transposed


def _ns_on_kernels(X: Tensor) -> bool:
    return X.is_cuda and X.size(-1) % 8 == 0 and X.size(-2) % 8 == 0 and X.dim() in (2, 3)


def newton_schulz(G: Tensor, steps: int = 5, eps: float = 1e-7, scheme: str = "jordan") -> Tensor:
    """Approximate U V^T of G (..., m, n) by quintic Newton-Schulz in bf16."""
    X, coeffs, transposed = _ns_prepare(G, steps, eps, scheme)
    if _ns_on_kernels(X):
        X = _ns_kernels(X.contiguous(), coeffs)
    else:
        X = _ns_torch(X, coeffs)
    if transposed:
        X = X.mT
    return X


def lr_scale(shape, lr_adjust: str) -> float:
    if lr_adjust == "shape":
        return max(1.0, shape[0] / shape[1]) ** 0.5
    return 0.2 * max(shape[0], shape[1]) ** 0.5


def _momentum(params, grads, bufs, lr, momentum, weight_decay, nesterov):
    torch._foreach_lerp_(bufs, grads, 1 - momentum)
    updates = torch._foreach_lerp(grads, bufs, momentum) if nesterov else bufs
    if weight_decay != 0:
        torch._foreach_mul_(params, 1 - lr * weight_decay)
    return updates


def muon_update(params, grads, momentum_bufs, *, lr, momentum, weight_decay, nesterov, ns_steps, eps,
                lr_adjust="shape", ns_coeffs="jordan", compile_ns=False, world_size=1, rank=0) -> None:
    """Functional Muon over plain tensors; NS work split over ``world_size``."""
    updates = _momentum(params, grads, momentum_bufs, lr, momentum, weight_decay, nesterov)
    buckets: dict[tuple, list[int]] = {}
    for i, u in enumerate(updates):
        buckets.setdefault((tuple(u.shape), u.dtype, u.device), []).append(i)
    for (shape, dtype, device), idx in buckets.items():
        stack = torch.stack([updates[i] for i in idx])
        n = stack.size(0)
        if world_size > 1:
            chunk = -(-n // world_size)
            local = stack[rank * chunk:(rank + 1) * chunk]
            if local.size(0) < chunk:
                local = torch.cat([local, stack.new_zeros((chunk - local.size(0), *shape))])
            local = newton_schulz(local, steps=ns_steps, eps=eps, scheme=ns_coeffs)
            out = torch.empty((chunk * world_size, *shape), dtype=local.dtype, device=device)
            dist.all_gather(list(out.chunk(world_size)), local.contiguous())
            O = out[:n]
        else:
            O = newton_schulz(stack, steps=ns_steps, eps=eps, scheme=ns_coeffs)
        torch._foreach_add_([params[i] for i in idx], list(O.to(dtype).unbind(0)),
                            alpha=-lr * lr_scale(shape, lr_adjust))


def _shard_layout(p):
    dims = [i for i, pl in enumerate(p.placements) if isinstance(pl, Shard)]
    if not dims:
        return None, 1, 0
    assert len(dims) == 1 and p.placements[dims[0]].dim == 0, \
        f"Muon expects row sharding on one mesh dim, got {p.placements}"
    mesh = p.device_mesh
    return mesh.get_group(dims[0]), mesh.size(dims[0]), mesh.get_local_rank(dims[0])


def muon_update_sharded(params, grads, momentum_bufs, *, lr, momentum, weight_decay, nesterov, ns_steps, eps,
                        lr_adjust="shape", ns_coeffs="jordan", compile_ns=False, exchanges=None) -> None:
    """Muon for row-sharded DTensor parameters (FSDP2 / HSDP).

    ``exchanges`` (a dict, kept by the optimizer) turns on the fused NVLink
    path on CUDA (``parallel.nvlink.MuonExchange``): every rank pushes its
    momentum row shard of each matrix to the matrix's owner (one barrier),
    the owner orthogonalises its matrices, the final Newton-Schulz product of
    each is written by the GEMM epilogue straight into the row owners'
    receive buffers on the other GPUs, one epoch barrier follows, and each
    rank applies the rows it received -- in place of two all-gathers of every
    full matrix, which move ``world`` times the bytes.  Buckets the fused
    path cannot take keep the all-gathers."""
    P = [p.to_local() for p in params]
    G = [g.to_local() for g in grads]
    Bf = [b.to_local() for b in momentum_bufs]
    for p, g, b in zip(params, grads, momentum_bufs):
        assert g.placements == p.placements and b.placements == p.placements
    updates = _momentum(P, G, Bf, lr, momentum, weight_decay, nesterov)
    buckets: dict[tuple, list[int]] = {}
    for i, p in enumerate(params):
        buckets.setdefault((tuple(p.shape), p.dtype, p.device, id(p.device_mesh), p.placements), []).append(i)
    plan = []
    for (shape, dtype, device, _, _), idx in buckets.items():
        group, ws, rank = _shard_layout(params[idx[0]])
        plan.append((shape, dtype, device, idx, group, ws, rank))
    # fused-path layout: per group, one receive block per eligible bucket (identical on every rank)
    fused: dict[int, tuple] = {}
    if exchanges is not None:
        from ..parallel.nvlink import MuonExchange
        sizes: dict[int, int] = {}
        for j, (shape, dtype, device, idx, group, ws, rank) in enumerate(plan):
            if not MuonExchange.eligible(shape, ws, device):
                continue
            rows, cols = shape
            chunk = -(-len(idx) // ws)
            off = sizes.get(id(group), 0)
            fused[j] = (off, chunk)
            sizes[id(group)] = off + MuonExchange.block_bytes(chunk * ws, rows // ws, cols)
        from ..parallel.nvlink import same_host
        for j, (shape, dtype, device, idx, group, ws, rank) in enumerate(plan):
            if j in fused and id(group) not in exchanges:
                # CUDA IPC reaches the GPUs of one machine only
                exchanges[id(group)] = MuonExchange(group, sizes[id(group)]) if same_host(group) else None
        for j in list(fused):
            ex = exchanges[id(plan[j][4])]
            if ex is None or ex.slot_bytes < sizes[id(plan[j][4])]:
                del fused[j]            # another machine in the group, or the buckets outgrew the heap
    # fused buckets: each momentum row shard goes straight to the matrix's owner
    # (one NVLink push per bucket and one barrier), not an all-gather of all of them
    for j in fused:
        shape, _, _, idx, group, ws, rank = plan[j]
        local = torch.stack([updates[i] for i in idx]).to(torch.bfloat16)
        exchanges[id(group)].push_inputs(fused[j][0], local, fused[j][1])
    for ex in {id(exchanges[id(plan[j][4])]): exchanges[id(plan[j][4])] for j in fused}.values():
        ex.barrier()
    pending = []
    for j, (shape, dtype, device, idx, group, ws, rank) in enumerate(plan):
        rows, cols = shape
        n = len(idx)
        if j in fused:
            ex = exchanges[id(group)]
            off, chunk = fused[j]
            mine = ex.received_inputs(off, n, chunk, rows, cols)
            X, coeffs, transposed = _ns_prepare(mine, ns_steps, eps, ns_coeffs)
            _ns_kernels(X.contiguous(), coeffs, last=ex.scatter_fn(off, rank * chunk, rows // ws, cols, transposed))
            pending.append((ex, off, idx, shape, dtype, rows // ws, transposed))
            continue
        local = torch.stack([updates[i] for i in idx]).to(torch.bfloat16)
        if ws > 1:
            rows_l = rows // ws
            assert rows % ws == 0 and local.shape[1] == rows_l, \
                f"{shape} is not evenly row-sharded {ws} ways (local {tuple(local.shape[1:])})"
            gathered = torch.empty((ws * n, rows_l, cols), dtype=torch.bfloat16, device=device)
            dist.all_gather_into_tensor(gathered, local.contiguous(), group=group)
            full = gathered.view(ws, n, rows_l, cols).transpose(0, 1).reshape(n, rows, cols)
        else:
            rows_l = rows
            full = local
        chunk = -(-n // ws)
        mine = full[rank * chunk:(rank + 1) * chunk]
        if mine.size(0) < chunk:
            mine = torch.cat([mine, full.new_zeros((chunk - mine.size(0), rows, cols))])
        mine = newton_schulz(mine, steps=ns_steps, eps=eps, scheme=ns_coeffs)
        if ws > 1:
            out = torch.empty((chunk * ws, rows, cols), dtype=mine.dtype, device=device)
            dist.all_gather_into_tensor(out, mine.contiguous(), group=group)
            O = out[:n, rank * rows_l:(rank + 1) * rows_l]
        else:
            O = mine[:n]
        torch._foreach_add_([P[i] for i in idx], list(O.to(dtype).unbind(0)),
                            alpha=-lr * lr_scale(shape, lr_adjust))
    if pending:
        for ex in {id(e[0]): e[0] for e in pending}.values():
            ex.barrier()                 # every peer's products have landed in this rank's buffer
        for ex, off, idx, shape, dtype, rows_l, transposed in pending:
            O = ex.received(off, len(idx), rows_l, shape[1], transposed)
            torch._foreach_add_([P[i] for i in idx], list(O.to(dtype).unbind(0)),
                                alpha=-lr * lr_scale(shape, lr_adjust))


class Muon(Optimizer):
    """Muon for 2-D parameters (anything else is rejected at construction)."""

    def __init__(self, params, lr: float = 0.02, momentum: float = 0.95, weight_decay: float = 0.0, *,
                 nesterov: bool = True, ns_steps: int = 5, eps: float = 1e-7, lr_adjust: str = "shape",
                 ns_coeffs: str = "jordan", compile_ns: bool | None = None, shard: bool = True):
        if lr < 0.0:
            raise ValueError(f"Invalid learning rate: {lr}")
        if not 0.0 <= momentum < 1.0:
            raise ValueError(f"Invalid momentum: {momentum}")
        if weight_decay < 0.0:
            raise ValueError(f"Invalid weight_decay: {weight_decay}")
        if ns_steps < 1:
            raise ValueError(f"Invalid ns_steps: {ns_steps}")
        if lr_adjust not in ("shape", "rms"):
            raise ValueError(f"Invalid lr_adjust: {lr_adjust!r} (expected 'shape' or 'rms')")
        if ns_coeffs not in NS_SCHEMES:
            raise ValueError(f"Invalid ns_coeffs: {ns_coeffs!r} (expected one of {sorted(NS_SCHEMES)})")
        defaults = dict(lr=lr, momentum=momentum, weight_decay=weight_decay, nesterov=nesterov, ns_steps=ns_steps,
                        eps=eps, lr_adjust=lr_adjust, ns_coeffs=ns_coeffs)
        super().__init__(params, defaults)
        # machine-local knobs: deliberately not in defaults / state_dict
        self._compile_ns = bool(compile_ns)
        self._shard = shard
        # fused NVLink exchange of the sharded path (VAGUS_MUON_NCCL=1 keeps the all-gathers)
        import os
        self._exchanges = None if os.environ.get("VAGUS_MUON_NCCL") else {}
        for group in self.param_groups:
            for p in group["params"]:
                if p.dim() != 2:
                    raise ValueError(f"Muon only handles 2D params, got shape {tuple(p.shape)}; "
                                     "give this param to AdamW instead")

    def __setstate__(self, state):
        super().__setstate__(state)
        for group in self.param_groups:
            group.setdefault("nesterov", True)
            group.setdefault("ns_steps", 5)
            group.setdefault("eps", 1e-7)
            group.setdefault("lr_adjust", "shape")
            group.setdefault("ns_coeffs", "jordan")

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        if self._shard and dist.is_available() and dist.is_initialized():
            world_size, rank = dist.get_world_size(), dist.get_rank()
        else:
            world_size, rank = 1, 0
        for group in self.param_groups:
            plain = ([], [], [])
            sharded = ([], [], [])
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.grad.is_sparse:
                    raise RuntimeError("Muon does not support sparse gradients")
                state = self.state[p]
                if not state:
                    state["momentum_buffer"] = torch.zeros_like(p)
                dst = sharded if isinstance(p, DTensor) else plain
                dst[0].append(p)
                dst[1].append(p.grad)
                dst[2].append(state["momentum_buffer"])
            common = dict(lr=group["lr"], momentum=group["momentum"], weight_decay=group["weight_decay"],
                          nesterov=group["nesterov"], ns_steps=group["ns_steps"], eps=group["eps"],
                          lr_adjust=group["lr_adjust"], ns_coeffs=group["ns_coeffs"], compile_ns=self._compile_ns)
            if plain[0]:
                muon_update(*plain, **common, world_size=world_size, rank=rank)
            if sharded[0]:
                ex = self._exchanges if sharded[0][0].device.type == "cuda" else None
                muon_update_sharded(*sharded, **common, exchanges=ex)
        return loss


class MuonAdamW:
    """Muon on the block matrices + AdamW on the rest, as one optimizer."""

    def __init__(self, muon: Muon, adamw: torch.optim.Optimizer):
        self.muon = muon
        self.adamw = adamw

    @property
    def param_groups(self):
        return self.muon.param_groups + self.adamw.param_groups

    @property
    def members(self) -> list[torch.optim.Optimizer]:
        return [self.muon, self.adamw]

    @property
    def state(self):
        return {**self.muon.state, **self.adamw.state}

    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        self.muon.step()
        self.adamw.step()
        return loss

    def zero_grad(self, set_to_none: bool = True) -> None:
        self.muon.zero_grad(set_to_none=set_to_none)
        self.adamw.zero_grad(set_to_none=set_to_none)

    def state_dict(self) -> dict:
        return {"muon": self.muon.state_dict(), "adamw": self.adamw.state_dict()}

    def load_state_dict(self, state_dict: dict) -> None:
        self.muon.load_state_dict(state_dict["muon"])
        self.adamw.load_state_dict(state_dict["adamw"])
