"""Model registry and components.

A recipe selects a model by name; its ``model_args`` go verbatim into the
constructor.  Every registered model exposes ``param_groups()`` (the
muon / adamw_decay / adamw_no_decay split), ``attn_flops_per_token(ctx)``,
``forward(tokens, return_hidden=)``, a bias-free ``head.weight``, the
Decodable verbs, and optionally ``metric_hooks()``.

Parity: reference ``infra/models/__init__.py:15-22``.
"""

from torch import nn

from .gdn_lm import GDNLM
from .transformer_pp import TransformerPP

MODELS: dict[str, type[nn.Module]] = {"TransformerPP": TransformerPP, "GDNLM": GDNLM}


def build_model(name: str, args: dict) -> nn.Module:
    return MODELS[name](**args)


__all__ = ["MODELS", "build_model", "GDNLM", "TransformerPP"]
