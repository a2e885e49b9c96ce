"""build_optimizers: parameter routing into NorMuon and three AdamW groups.

Same signature, routing rules and group layout as the reference's
``build_optimizers`` (transformer_lm/sol_modules.py:428-488):
  value_embeds*                          -> AdamW group, betas (0.75, 0.95), lr ve_lr or embed_lr
  token_embeddings / lm_head / second_embeds -> AdamW embed group, lr embed_lr
  names containing an arch-extra key    -> AdamW no-wd group, lr adam_lr
  remaining params with ndim >= 2        -> NorMuonGNS (weight decay applied)
  remaining 1-D / 0-D params             -> AdamW no-wd group
All AdamW groups have weight_decay 0 and every group stashes ``base_lr``.
"""
from __future__ import annotations

import logging

from .adamw import AdamW
from .normuon import NorMuonGNS

logger = logging.getLogger("sol_b200")

# arch-extra scalar banks / tiny gates (sol_modules.py:445-447)
ADAM_KEYS = ("resid_lambdas", "post_lambdas", "x0_lambdas", "_xsa_alpha", "smear", "skip_gate", "_skip_lambda",
             "_backout", "_second_gate", "_ve_gate")


def route_params(named_params):
    """Returns (muon, embed, norm, ve) parameter lists in named_parameters order."""
    muon, embed, norm, ve = [], [], [], []
    seen = set()
    for name, p in named_params:
        if not p.requires_grad or id(p) in seen:
            continue
        seen.add(id(p))
        if "value_embeds" in name:
            ve.append(p)
        elif ("token_embeddings" in name) or ("lm_head" in name) or ("second_embeds" in name):
            embed.append(p)
        elif any(k in name for k in ADAM_KEYS):
            norm.append(p)
        elif p.ndim >= 2:
            muon.append(p)
        else:
            norm.append(p)
    return muon, embed, norm, ve


def build_optimizers(model, *, muon_lr: float, adam_lr: float, embed_lr: float, weight_decay: float,
                     betas=(0.9, 0.95), eps=1e-8, cautious_wd: bool = False, bf16_master: bool = False,
                     ve_lr: float | None = None, orthogonalizer: str = "gram",
                     coefficients: str = "polar_express", adam_master: str = "none", adam_state_dtype=None,
                     adam_cautious_wd: bool = False):
    """Reference signature plus engine options (orthogonaliser and AdamW storage mode)."""
    inner = getattr(model, "_orig_mod", model)
    muon_params, embed_params, norm_params, ve_params = route_params(inner.named_parameters())
    groups = []
    if embed_params:
        groups.append({"params": embed_params, "lr": embed_lr, "weight_decay": 0.0})
    if ve_params:
        groups.append({"params": ve_params, "lr": ve_lr if ve_lr is not None else embed_lr,
                       "weight_decay": 0.0, "betas": (0.75, 0.95)})
    if norm_params:
        groups.append({"params": norm_params, "lr": adam_lr, "weight_decay": 0.0})
    adamw = AdamW(groups, betas=betas, eps=eps, fused=True, master=adam_master, state_dtype=adam_state_dtype,
                  cautious_wd=adam_cautious_wd)
    muon = NorMuonGNS(muon_params, lr=muon_lr, weight_decay=weight_decay, cautious_wd=cautious_wd,
                      bf16_master=bf16_master, orthogonalizer=orthogonalizer, coefficients=coefficients)
    for opt in (muon, adamw):
        for g in opt.param_groups:
            g["base_lr"] = g["lr"]
    logger.info("optimizers: NorMuonGNS(%d matrices, lr=%.2g, %s) | AdamW embed(%d) + norm/1D(%d) + ve(%d)",
                len(muon_params), muon_lr, orthogonalizer, len(embed_params), len(norm_params), len(ve_params))
    return muon, adamw
