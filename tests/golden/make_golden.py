"""Generates tests/golden/ref_digests.json from the reference implementation itself.

Run in the build container, where the reference tree is mounted read-only:
    REF=/path/to/cs336-a1-sol python tests/golden/make_golden.py
It imports transformer_lm.sol_modules (build_optimizers, NorMuonGNS with its
quintic fallback, torch's fused AdamW, EmaWeights), runs the optimizer step of
train_sol.py:460-507 (lr schedule, momentum warmup, muon -> adamw -> ema) on
seeded synthetic parameters/gradients on the CPU, and stores per-tensor digests
(float64 sum, sum of squares and values at fixed sampled indices). It also runs
oracle/ref_step.py on the same inputs and refuses to write the file unless the
oracle is bit-identical to the reference on every tensor.
"""
from __future__ import annotations

import json
import os
import sys
import zlib
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "cs336-a1-sol_b200"))

from oracle import ref_step  # noqa: E402
from sol_b200 import synth  # noqa: E402

OUT = Path(__file__).resolve().parent / "ref_digests.json"

# name -> (config, steps, optimizer kwargs)
CASES = {
    "c1_fp32": (synth.C1, 10, dict(muon_lr=8e-3, adam_lr=1.2e-2, embed_lr=2.4e-2, weight_decay=0.0,
                                    cautious_wd=False, bf16_master=False), 0),
    "micro_bf16_mt_cautious": (synth.MICRO, 6, dict(muon_lr=8e-3, adam_lr=1.2e-2, embed_lr=2.4e-2,
                                                   weight_decay=0.1, cautious_wd=True, bf16_master=True), 300),
    "micro_bf16_plain": (synth.MICRO, 4, dict(muon_lr=8e-3, adam_lr=1.2e-2, embed_lr=2.4e-2, weight_decay=0.1,
                                             cautious_wd=False, bf16_master=False), 0),
}
N_SAMPLES = 24


def lr_frac(it, warmup=5):
    """train_sol.lr_frac during warm-up (train_sol.py:337-342)."""
    return (it + 1) / max(1, warmup)


def momentum_at(it, warmup):
    """train_sol.py:468-475 momentum warm-up 0.85 -> 0.95 (fixed 0.95 when warmup == 0)."""
    if warmup <= 0:
        return None
    return 0.85 + 0.10 * min(1.0, it / warmup)


def digest(t: torch.Tensor, key: str):
    x = t.detach().reshape(-1).to(torch.float64)
    g = torch.Generator().manual_seed(zlib.crc32(key.encode()))
    n = x.numel()
    idx = torch.randint(0, n, (min(N_SAMPLES, n),), generator=g).tolist() if n else []
    return {"sum": float(x.sum()), "sumsq": float((x * x).sum()), "idx": idx, "vals": [float(x[i]) for i in idx],
            "dtype": str(t.dtype), "shape": list(t.shape)}


def collect(model, muon_state, adam, shadows):
    """Tensors to digest: params, NorMuon state, AdamW state, EMA shadows (name -> tensor)."""
    out = {}
    for n, p in model.named_parameters():
        out[f"param/{n}"] = p
    for n, st in muon_state:
        for k, v in st.items():
            if torch.is_tensor(v):
                out[f"muon/{n}/{k}"] = v
    for n, p in model.named_parameters():
        st = adam.state.get(p)
        if st:
            out[f"adam/{n}/exp_avg"] = st["exp_avg"]
            out[f"adam/{n}/exp_avg_sq"] = st["exp_avg_sq"]
    for (n, _), s in zip(model.named_parameters(), shadows):
        out[f"ema/{n}"] = s
    return out


def run_reference(cfg, steps, kw, mwarm):
    ref_path = os.environ.get("REF", "")
    if ref_path and ref_path not in sys.path:
        sys.path.insert(0, ref_path)
    import transformer_lm.sol_modules as sm  # the reference itself
    model = synth.SyntheticLM(cfg, seed=0)
    muon, adamw = sm.build_optimizers(model, **kw)
    ema = sm.EmaWeights(model, 0.999)
    for it in range(steps):
        frac = lr_frac(it)
        for opt in (muon, adamw):
            for g in opt.param_groups:
                g["lr"] = g["base_lr"] * frac
        mom = momentum_at(it, mwarm)
        if mom is not None:
            for g in muon.param_groups:
                g["momentum"] = mom
        synth.set_grads(model, synth.make_grads(model, it, seed=0))
        muon.step()
        adamw.step()
        ema.update()
    names = {id(p): n for n, p in model.named_parameters()}
    mstate = [(names[id(p)], muon.state[p]) for p in muon.param_groups[0]["params"] if p in muon.state]
    return model, collect(model, mstate, adamw, ema.shadow)


def run_oracle(cfg, steps, kw, mwarm):
    model = synth.SyntheticLM(cfg, seed=0)
    step = ref_step.RefStep(model, **kw)
    for it in range(steps):
        frac = lr_frac(it)
        step.muon.group["lr"] = step.muon.group["base_lr"] * frac
        for g in step.adamw.param_groups:
            g["lr"] = g["base_lr"] * frac
        mom = momentum_at(it, mwarm)
        if mom is not None:
            step.muon.group["momentum"] = mom
        synth.set_grads(model, synth.make_grads(model, it, seed=0))
        step.step()
    names = {id(p): n for n, p in model.named_parameters()}
    mstate = [(names[id(p)], st) for p, st in zip(step.muon.params, step.muon.state) if st]
    return model, collect(model, mstate, step.adamw, step.shadow)


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    result = {}
    for name, (cfg, steps, kw, mwarm) in CASES.items():
        _, ref = run_reference(cfg, steps, kw, mwarm)
        _, orc = run_oracle(cfg, steps, kw, mwarm)
        assert ref.keys() == orc.keys(), (name, sorted(set(ref) ^ set(orc)))
        for k in ref:
            a, b = ref[k], orc[k]
            if a.dtype != b.dtype or not torch.equal(a, b):
                raise SystemExit(f"oracle differs from the reference: case {name} tensor {k}")
        result[name] = {"config": cfg.name, "steps": steps, "kwargs": kw, "momentum_warmup": mwarm,
                        "tensors": {k: digest(v, f"{name}/{k}") for k, v in ref.items()}}
        print(f"{name}: {len(ref)} tensors, oracle bit-identical to the reference")
    OUT.write_text(json.dumps(result, indent=1, sort_keys=True))
    print("wrote", OUT, OUT.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
