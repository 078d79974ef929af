"""Optimizer factory: maps a model's ``param_groups()`` three-way split
(muon / adamw_decay / adamw_no_decay) onto a concrete optimizer.

Contract of every builder: the returned object exposes step / zero_grad /
state_dict / load_state_dict / param_groups, and each group carries a
``name`` and an ``lr``; ``build_optimizer`` stamps ``base_lr`` on every group
(the schedule multiplies it in each step) after checking that every trainable
parameter lands in exactly one group.

Parity: reference ``infra/optimizer/__init__.py:18-84``.
"""

from __future__ import annotations

import torch

from . import muon
from .adamw import AdamW
from .muon import Muon, MuonAdamW, newton_schulz  # noqa: F401


def build_adamw(model, args: dict):
    groups = model.param_groups()
    args = dict(args)
    wd = args.pop("weight_decay", 0.0)
    if "betas" in args:
        args["betas"] = tuple(args["betas"])
    return AdamW([{"params": groups["muon"] + groups["adamw_decay"], "weight_decay": wd, "name": "decay"},
                  {"params": groups["adamw_no_decay"], "weight_decay": 0.0, "name": "no_decay"}], **args)


def build_muon(model, args: dict):
    groups = model.param_groups()
    args = dict(args)
    adamw_args = dict(args.pop("adamw"))
    if "betas" in adamw_args:
        adamw_args["betas"] = tuple(adamw_args["betas"])
    wd = adamw_args.pop("weight_decay", 0.0)
    m = muon.Muon([{"params": groups["muon"], "name": "muon"}], **args)
    a = AdamW([{"params": groups["adamw_decay"], "weight_decay": wd, "name": "decay"},
               {"params": groups["adamw_no_decay"], "weight_decay": 0.0, "name": "no_decay"}], **adamw_args)
    return muon.MuonAdamW(m, a)


OPTIMIZERS = {"adamw": build_adamw, "muon": build_muon}


def _check_coverage(model, opt) -> None:
    counts: dict[int, int] = {}
    for g in opt.param_groups:
        for p in g["params"]:
            counts[id(p)] = counts.get(id(p), 0) + 1
    names = {id(p): n for n, p in model.named_parameters() if p.requires_grad}
    missing = [n for i, n in names.items() if i not in counts]
    dup = [n for i, n in names.items() if counts.get(i, 0) > 1]
    foreign = len([i for i in counts if i not in names])
    if missing or dup or foreign:
        raise ValueError("optimizer param groups do not cover the model: "
                         f"missing {missing}, in multiple groups {dup}, {foreign} params not in the model")


def build_optimizer(name: str, model, args: dict):
    opt = OPTIMIZERS[name](model, args)
    _check_coverage(model, opt)
    for g in opt.param_groups:
        g["base_lr"] = g["lr"]
    return opt
