"""sol_b200 — the optimizer step of transformer_lm/train_sol.py on a B200-native engine.

Public surface (names of transformer_lm.sol_modules):
  build_optimizers, NorMuonGNS, EmaWeights, plus AdamW (the fused AdamW that
  build_optimizers returns). ``install()`` points transformer_lm.sol_modules at
  these classes so that train_sol.py runs unchanged.
"""
from .adamw import AdamW
from .clip import clip_grad_norm_
from .ema import EmaWeights
from .normuon import NorMuonGNS
from .routing import build_optimizers, route_params

__all__ = ["AdamW", "EmaWeights", "NorMuonGNS", "build_optimizers", "clip_grad_norm_", "route_params", "install"]


def install(module=None):
    """Replaces build_optimizers/NorMuonGNS/EmaWeights in transformer_lm.sol_modules
    (or in ``module``) with the engine's classes. Returns the patched module."""
    if module is None:
        import importlib
        module = importlib.import_module("transformer_lm.sol_modules")
    module.build_optimizers = build_optimizers
    module.NorMuonGNS = NorMuonGNS
    module.EmaWeights = EmaWeights
    return module
