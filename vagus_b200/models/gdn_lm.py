"""Gated delta-rule language model (the LAX / HAX architectures): the
Transformer++ skeleton with the GatedDeltaNet family as token mixer, plus
inter-layer softmax layers and intra-layer parallel (softmax | linear) blocks.

Layer kinds come from ``layer_kinds`` or the cyclic ``layer_pattern``:
``gdn`` (linear mixer alone), ``softmax`` (whole softmax layer), ``parallel``
(``ParallelMixer`` of half-width branches).  ``softmax_rope=False`` makes every
softmax branch NoPE.  ``write`` picks the delta rule's own sigmoid write or a
Kalman gain (``kalman_iso`` / ``kalman_diag``).

Parity: reference ``infra/models/gdn_lm.py:51-349``.
"""

from __future__ import annotations

from typing import Any

import torch
from torch import nn

from .attention import SoftmaxAttention
from .block import Block
from .gdn import GatedDeltaNet
from .kalman import KalmanDeltaNet
from .lm import CausalLM
from .mixer import Mixer
from .parallel_mixer import ParallelMixer
from .rope import RoPE
from .scans import chunk_scan_flops

KINDS = ("gdn", "softmax", "parallel")
WRITES = ("delta", "kalman_iso", "kalman_diag")


class GDNLM(CausalLM):
    def __init__(self, vocab_size: int, dim: int, layer_count: int, head_count: int, key_head_dim: int,
                 value_head_dim: int, ffn_hidden_dim: int | None = None, short_conv_size: int | None = 4,
                 gate: str | bool = "vector", delta: bool = True, gate_rank: int = 64, chunk_size: int = 64,
                 la_impl: str = "auto", la_fused: bool | str | list = False, la_conv_impl: str = "conv1d",
                 la_disable_recompute: bool = False, gate_lower_bound: float | None = None,
                 write: str = "delta", kalman_args: dict | None = None,
                 A_init_range: tuple[float, float] = (1.0, 16.0),
                 dt_init_range: tuple[float, float] = (1e-3, 1e-1), layer_pattern: str = "gdn",
                 layer_kinds: list[str] | None = None, softmax_head_dim: int = 64, softmax_rope: bool = True,
                 softmax_out_gate: bool = False, parallel_width: int | None = None, context_len: int = 2048,
                 rope_base: float = 10000, rmsnorm_eps: float = 1e-6, tie_embedding: bool = True,
                 gate_proj_optimizer: str = "adamw"):
        super().__init__()
        assert gate_proj_optimizer in ("adamw", "muon")
        self.config: dict[str, Any] = dict(
            vocab_size=vocab_size, dim=dim, layer_count=layer_count, head_count=head_count,
            key_head_dim=key_head_dim, value_head_dim=value_head_dim, ffn_hidden_dim=ffn_hidden_dim,
            short_conv_size=short_conv_size, gate=gate, delta=delta, gate_rank=gate_rank,
            chunk_size=chunk_size, la_impl=la_impl, la_fused=la_fused, la_conv_impl=la_conv_impl,
            la_disable_recompute=la_disable_recompute, gate_lower_bound=gate_lower_bound, write=write,
            kalman_args=kalman_args, A_init_range=tuple(A_init_range), dt_init_range=tuple(dt_init_range),
            layer_pattern=layer_pattern, layer_kinds=layer_kinds, softmax_head_dim=softmax_head_dim,
            softmax_rope=softmax_rope, softmax_out_gate=softmax_out_gate, parallel_width=parallel_width,
            context_len=context_len, rope_base=rope_base, rmsnorm_eps=rmsnorm_eps,
            tie_embedding=tie_embedding, gate_proj_optimizer=gate_proj_optimizer)

        if layer_kinds is not None:
            kinds = [k.strip() for k in layer_kinds]
            assert len(kinds) == layer_count, \
                f"layer_kinds has {len(kinds)} entries for layer_count {layer_count}"
        else:
            cycle = [t.strip() for t in layer_pattern.split(",")]
            assert cycle, layer_pattern
            kinds = [cycle[i % len(cycle)] for i in range(layer_count)]
        assert all(k in KINDS for k in kinds), kinds
        self.kinds = kinds

        pw = parallel_width or dim // 2
        if "parallel" in kinds:
            assert pw % softmax_head_dim == 0 and pw % value_head_dim == 0, \
                f"parallel_width {pw} must hold whole softmax ({softmax_head_dim}) and value ({value_head_dim}) heads"
        self.parallel_width = pw

        self.embedding = nn.Embedding(vocab_size, dim)
        self.rope = None
        if any(k != "gdn" for k in kinds) and softmax_rope:
            assert dim % softmax_head_dim == 0
            self.rope = RoPE(dim, softmax_head_dim, context_len, base=rope_base)

        assert write in WRITES, f"write must be one of {WRITES}, got {write!r}"
        self.write = write

        def linear(width: int, out_proj: bool) -> GatedDeltaNet:
            assert width % value_head_dim == 0
            cls, extra = GatedDeltaNet, {}
            if write != "delta":
                cls, extra = KalmanDeltaNet, {"kalman": write.removeprefix("kalman_"), **(kalman_args or {})}
            return cls(**extra, dim=dim, head_count=width // value_head_dim, key_head_dim=key_head_dim,
                       value_head_dim=value_head_dim, short_conv_size=short_conv_size, gate=gate, delta=delta,
                       gate_rank=gate_rank, chunk_size=chunk_size, impl=la_impl, fused=la_fused,
                       conv_impl=la_conv_impl, disable_recompute=la_disable_recompute,
                       gate_lower_bound=gate_lower_bound, A_init_range=tuple(A_init_range),
                       dt_init_range=tuple(dt_init_range), init_std=0.02, layer_count=layer_count,
                       out_proj=out_proj)

        def softmax(width: int, out_proj: bool) -> SoftmaxAttention:
            assert width % softmax_head_dim == 0
            return SoftmaxAttention(dim=width, head_count=width // softmax_head_dim, kv_head_count=None,
                                    v_dim_mult=1, short_conv_size=None, qk_norm=True, rope=self.rope,
                                    init_std=0.02, layer_count=layer_count, in_dim=dim, out_proj=out_proj,
                                    out_gate=softmax_out_gate)

        def mixer(kind: str) -> Mixer:
            if kind == "gdn":
                return linear(head_count * value_head_dim, True)
            if kind == "softmax":
                return softmax(dim, True)
            return ParallelMixer(dim, att=softmax(pw, False), la=linear(pw, False), rmsnorm_eps=rmsnorm_eps,
                                 init_std=0.02, layer_count=layer_count)

        self.blocks = nn.ModuleList([
            Block(dim=dim, ffn_hidden_dim=ffn_hidden_dim, rmsnorm_eps=rmsnorm_eps, mixer=mixer(kind),
                  layer_count=layer_count) for kind in kinds])
        self._finish(vocab_size, dim, rmsnorm_eps, tie_embedding)

    # --- roles -----------------------------------------------------------

    @staticmethod
    def _linear_of(mixer) -> GatedDeltaNet | None:
        if isinstance(mixer, GatedDeltaNet):
            return mixer
        if isinstance(mixer, ParallelMixer):
            return mixer.la
        return None

    @staticmethod
    def _softmax_of(mixer) -> SoftmaxAttention | None:
        if isinstance(mixer, SoftmaxAttention):
            return mixer
        if isinstance(mixer, ParallelMixer):
            return mixer.att
        return None

    @property
    def max_stream_len(self) -> int | None:
        return int(self.config["context_len"]) if self.rope is not None else None

    @torch.no_grad()
    def surprise(self, tokens) -> torch.Tensor:
        """(B, L, layers, H) delta-rule residual ratios (all-GDN layouts only)."""
        x = self.embedding(tokens)
        out = []
        for blk in self.blocks:
            la = self._linear_of(blk.att)
            assert la is not None and la is blk.att, "surprise: all-GDN layouts only"
            out.append(la.residuals(blk.rmsnorm1(x)))
            x = blk(x)
        return torch.stack(out, 2)

    # --- training --------------------------------------------------------

    def param_groups(self) -> dict[str, list[nn.Parameter]]:
        skip = set()
        if self.config["gate_proj_optimizer"] == "adamw":
            for blk in self.blocks:
                skip.update(id(p) for p in getattr(blk.att, "gate_projections", []))
        muon = [p for p in self.blocks.parameters() if p.requires_grad and p.dim() == 2 and id(p) not in skip]
        ids = {id(p) for p in muon}
        decay = [p for p in self.parameters() if p.requires_grad and id(p) not in ids and p.dim() >= 2]
        no_decay = [p for p in self.parameters() if p.requires_grad and p.dim() < 2]
        return {"muon": muon, "adamw_decay": decay, "adamw_no_decay": no_decay}

    def attn_flops_per_token(self, context_len: int) -> float:
        c = self.config
        dk, dv, dim = int(c["key_head_dim"]), int(c["value_head_dim"]), int(c["dim"])
        per_head = chunk_scan_flops(dk, dv, int(c["chunk_size"]), bool(c["delta"]))

        def flops(kind: str) -> float:
            if kind == "gdn":
                return per_head * int(c["head_count"])
            if kind == "softmax":
                return 12 * dim * context_len
            return per_head * (self.parallel_width // dv) + 12 * self.parallel_width * context_len

        return float(sum(flops(k) for k in self.kinds))

    def metric_hooks(self) -> dict:
        return {"slow": [self._metric_probe]}

    @torch.no_grad()
    def _metric_probe(self, ctx) -> dict:
        tokens = ctx.last_batch
        if tokens is None:
            return {}
        x = self.embedding(tokens[:1])
        alpha, mem, beta, srms = [], [], [], []
        worst = None
        for blk in self.blocks:
            h = blk.rmsnorm1(x)
            la = self._linear_of(blk.att)
            if la is not None:
                st = la.gate_stats(h)
                srms.append(float(st["state_rms"]))
                if "alpha" in st:
                    alpha.append(st["alpha"])
                    mem.append(st["mem_len"])
                if "beta" in st:
                    beta.append(st["beta"])
            sm = self._softmax_of(blk.att)
            if sm is not None:
                m = sm.max_attn_logit(h)
                worst = m if worst is None else torch.maximum(worst, m)
            x = x + blk.att(h)
            x = x + blk.ffn(blk.rmsnorm2(x))
        out = {}
        if srms:
            out["gdn/state_rms_max"] = max(srms)
        if alpha:
            a, m = torch.cat(alpha).float(), torch.cat(mem).float()
            out.update({"gdn/alpha_mean": float(a.mean()), "gdn/mem_len_median": float(m.median()),
                        "gdn/mem_len_max": float(m.max())})
        if beta:
            out["gdn/beta_mean"] = float(torch.cat(beta).float().mean())
        if worst is not None:
            out["attn_logit_max"] = float(worst)
        return out
