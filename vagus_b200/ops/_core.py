"""Extension loading, the bf16 compute-copy cache and small shared helpers."""

from __future__ import annotations

import torch

_C = None


def native():
    """The compiled sm_100a extension; raises when it cannot be loaded."""
    global _C
    if _C is None:
        from .build import load
        _C = load()
    return _C


def kernels_active(x: torch.Tensor) -> bool:
    """True when ``x`` lives on a CUDA device: the sm_100a kernels then run
    (and their extension must load -- a missing build raises instead of
    silently falling back to eager PyTorch)."""
    if not x.is_cuda:
        return False
    native()
    return True


def check_error() -> None:
    """Raise if a kernel recorded a bounded-wait timeout since the last reset."""
    if _C is None:
        return
    code = _C.error_word()
    if code:
        _C.reset_error()
        raise RuntimeError(f"vagus_b200 kernel watchdog tripped (code {code}): a device wait ran out of time")


class _Bf16Cache:
    """bf16 compute copies of fp32 master weights, rebuilt when the master
    changes (its autograd version counter moves on every in-place update)."""

    def __init__(self):
        self._d: dict[int, tuple[int, int, torch.Tensor]] = {}

    def get(self, w: torch.Tensor) -> torch.Tensor:
        if w.dtype == torch.bfloat16:
            return w if w.is_contiguous() else w.contiguous()
        key = id(w)
        ver = w._version
        hit = self._d.get(key)
        if hit is not None and hit[0] == ver and hit[1] == w.data_ptr():
            return hit[2]
        c = w.detach().to(torch.bfloat16).contiguous()
        self._d[key] = (ver, w.data_ptr(), c)
        return c

    def get_cat(self, ws: list[torch.Tensor]) -> torch.Tensor:
        """Row-concatenation of several masters' bf16 copies (one GEMM operand)."""
        if any(w.dtype != torch.float32 for w in ws):
            # low-precision compute copies (e.g. all-gathered by FSDP) may be
            # refilled in place without a version bump: never cache them
            return torch.cat([w.detach().to(torch.bfloat16) for w in ws], 0).contiguous()
        key = ("cat",) + tuple(id(w) for w in ws)
        vers = tuple((w._version, w.data_ptr()) for w in ws)
        hit = self._d.get(key)
        if hit is not None and hit[0] == vers:
            return hit[2]
        c = torch.cat([w.detach().to(torch.bfloat16) for w in ws], 0).contiguous()
        self._d[key] = (vers, None, c)
        return c

    def clear(self):
        self._d.clear()


BF16 = _Bf16Cache()


def as_bf16_2d(x: torch.Tensor) -> torch.Tensor:
    x2 = x.reshape(-1, x.shape[-1])
    if x2.dtype != torch.bfloat16:
        x2 = x2.to(torch.bfloat16)
    return x2 if x2.stride(-1) == 1 and x2.stride(0) == x2.shape[1] else x2.contiguous()


def autocast_bf16() -> bool:
    return torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16


_GEMM_CODES = {1: "operand base or row pitch not 16-byte aligned", 2: "tensor-map encoding failed",
               3: "kernel launch failed", 4: "K must be positive", 6: "a TMA box exceeds its tensor (shape too small)"}


def gemm(A, a_mn, B, b_mn, C, S=None, alpha=1.0, beta=0.0, atomic=False, split_k=0, block_n=0):
    """C = alpha op(A) op(B)^T + beta S on the tcgen05 GEMM (see gemm.cu)."""
    rc = native().gemm(A, a_mn, B, b_mn, C, S, alpha, beta, atomic, split_k, block_n)
    if rc:
        raise RuntimeError(f"vagus_b200 gemm rejected the problem: {_GEMM_CODES.get(rc, rc)} "
                           f"(A {tuple(A.shape)} mn={a_mn}, B {tuple(B.shape)} mn={b_mn}, C {tuple(C.shape)})")
    return C
