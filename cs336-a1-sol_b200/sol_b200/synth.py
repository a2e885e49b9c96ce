"""Seeded synthetic parameter sets and gradients for the optimizer step.

The reference trains on OpenWebText; the optimizer step only sees parameter
tensors and their gradients, so the benchmark and the tests use seeded
synthetic tensors with the recipe's names, shapes, dtypes and initialisation
(names/shapes follow SOLTransformerLm as built by transformer_lm/train_sol.py:237-299
with --fused-qkv --value-embeds-k --ve-gates per-head --second-embed --x0-lambdas
--xsa --smear --unet-skips). No data set is involved.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn as nn


@dataclass(frozen=True)
class ModelConfig:
    name: str
    d_model: int
    n_layers: int
    n_heads: int
    d_ff: int
    vocab: int
    ve_k: int = 0
    second_embed: bool = False
    attn_gate: bool = False      # (H, d) per-head output gate, routed to NorMuon
    extras: bool = False         # scalar banks / tiny gates (AdamW no-wd group)
    dtype: torch.dtype = torch.float32
    weight_std: float = 0.02
    ve_std: float = 0.01
    grad_std: float = 1e-3
    grad_hot_rows: float = 0.0   # fraction of rows whose gradient is scaled by 10


# CPU-runnable tiny fp32 step.
C1 = ModelConfig("c1_tiny_fp32", d_model=128, n_layers=2, n_heads=4, d_ff=512, vocab=1024,
                 dtype=torch.float32, grad_std=1e-3)
# B200 leaderboard parameter set (L14 d1024).
C2 = ModelConfig("c2_L14_d1024", d_model=1024, n_layers=14, n_heads=8, d_ff=5632, vocab=32768, ve_k=5,
                 second_embed=True, attn_gate=True, extras=True, dtype=torch.bfloat16, grad_std=1e-4,
                 grad_hot_rows=0.05)
# B300-recipe parameter set (L20).
C5 = ModelConfig("c5_L20_d1024", d_model=1024, n_layers=20, n_heads=8, d_ff=5632, vocab=32768, ve_k=5,
                 second_embed=True, attn_gate=True, extras=True, dtype=torch.bfloat16, grad_std=1e-4,
                 grad_hot_rows=0.05)
# A small bf16 recipe-shaped set for GPU parity tests (every routing case present).
MICRO = ModelConfig("micro_bf16", d_model=128, n_layers=3, n_heads=4, d_ff=384, vocab=512, ve_k=2,
                    second_embed=True, attn_gate=True, extras=True, dtype=torch.bfloat16, grad_std=1e-3,
                    grad_hot_rows=0.05)

CONFIGS = {c.name: c for c in (C1, C2, C5, MICRO)}


def param_specs(cfg: ModelConfig):
    """Ordered (name, shape, init) triples; init in {'normal', 've', 'ones', 'half'}."""
    d, L, H, V = cfg.d_model, cfg.n_layers, cfg.n_heads, cfg.vocab
    specs = []
    if cfg.ve_k:
        specs.append(("value_embeds_k", (cfg.ve_k, V, d), "ve"))
    if cfg.extras:
        specs += [("x0_lambdas", (L,), "half"), ("_skip_lambda", (), "half"), ("_backout", (), "half"),
                  ("_smear_lambda", (), "half")]
        if cfg.second_embed:
            specs.append(("_second_gate", (), "half"))
    specs.append(("token_embeddings.embeddings", (V, d), "normal"))
    for i in range(L):
        p = f"layers.{i}"
        specs.append((f"{p}.norm1.gamma", (d,), "ones"))
        if cfg.extras:
            specs += [(f"{p}.attention._attn_scale", (), "half"), (f"{p}.attention._xsa_alpha", (H,), "half")]
        specs.append((f"{p}.attention._wqkv", (3 * d, d), "normal"))
        if cfg.extras and i >= 1:
            specs += [(f"{p}.attention._ve_gate", (), "half"), (f"{p}.attention._ve_gate_w", (H, 12), "normal")]
        specs.append((f"{p}.attention.wo.weights", (d, d), "normal"))
        if cfg.attn_gate:
            specs.append((f"{p}.attention._attn_gate.weights", (H, d), "normal"))
        specs.append((f"{p}.norm2.gamma", (d,), "ones"))
        specs.append((f"{p}.ffn.w1.weights", (cfg.d_ff, d), "normal"))
        specs.append((f"{p}.ffn.w2.weights", (d, cfg.d_ff), "normal"))
    specs.append(("final_norm.gamma", (d,), "ones"))
    if cfg.extras:
        specs += [("skip_gate.weights", (1, 12), "normal"), ("smear_gate.weights", (1, 12), "normal")]
    if cfg.second_embed:
        specs.append(("second_embeds.weight", (V, d), "normal"))
    return specs


class SyntheticLM(nn.Module):
    """Parameter container whose named_parameters() match the recipe's model."""

    def __init__(self, cfg: ModelConfig, device="cpu", seed: int = 0):
        super().__init__()
        self.cfg = cfg
        meta = torch.device(device).type == "meta"
        g = None if meta else torch.Generator(device=device)
        if g is not None:
            g.manual_seed(seed)
        self._names = []
        for name, shape, init in param_specs(cfg):
            if meta:
                t = torch.empty(shape, device=device, dtype=torch.float32)
            elif init == "normal":
                t = torch.randn(shape, generator=g, device=device, dtype=torch.float32) * cfg.weight_std
            elif init == "ve":
                t = torch.randn(shape, generator=g, device=device, dtype=torch.float32) * cfg.ve_std
            elif init == "ones":
                t = torch.ones(shape, device=device, dtype=torch.float32)
            else:
                t = torch.full(shape, 0.5, device=device, dtype=torch.float32)
            self._register(name, nn.Parameter(t.to(cfg.dtype)))

    def _register(self, dotted: str, p: nn.Parameter):
        parts = dotted.split(".")
        mod = self
        for part in parts[:-1]:
            if not hasattr(mod, part) or not isinstance(getattr(mod, part), nn.Module):
                mod.add_module(part, nn.Module())
            mod = getattr(mod, part)
        mod.register_parameter(parts[-1], p)
        self._names.append(dotted)

    def named_parameters(self, prefix: str = "", recurse: bool = True, remove_duplicate: bool = True):
        # creation order (the order the recipe's model lists them), not module order
        lookup = dict(super().named_parameters(prefix=prefix, recurse=recurse, remove_duplicate=remove_duplicate))
        for n in self._names:
            key = f"{prefix}.{n}" if prefix else n
            if key in lookup:
                yield key, lookup[key]


def make_grads(model: nn.Module, step: int, seed: int = 0, cfg: ModelConfig | None = None):
    """Fresh seeded gradients for every parameter (one call per step)."""
    cfg = cfg or model.cfg
    params = [p for _, p in model.named_parameters()]
    dev = params[0].device
    g = torch.Generator(device=dev)
    g.manual_seed(seed * 1_000_003 + 7919 * (step + 1))
    grads = []
    for p in params:
        x = torch.randn(p.shape, generator=g, device=dev, dtype=torch.float32) * cfg.grad_std
        if cfg.grad_hot_rows > 0 and p.ndim >= 2:
            rows = x.reshape(-1, p.shape[-1])
            hot = torch.rand(rows.shape[0], generator=g, device=dev) < cfg.grad_hot_rows
            rows[hot] *= 10.0
        grads.append(x.to(p.dtype))
    return grads


def set_grads(model: nn.Module, grads):
    for (_, p), gr in zip(model.named_parameters(), grads):
        p.grad = gr


def count_params(cfg: ModelConfig) -> int:
    n = 0
    for _, shape, _ in param_specs(cfg):
        k = 1
        for s in shape:
            k *= s
        n += k
    return n
