"""The CPU oracle against golden digests of the reference's own optimizer step.

tests/golden/ref_digests.json was produced by tests/golden/make_golden.py from
transformer_lm.sol_modules of the reference (quintic fallback, torch fused
AdamW, EmaWeights). The oracle must reproduce every digest exactly.
"""
import json
import math
from pathlib import Path

import pytest
import torch

from oracle import ref_step
from sol_b200 import synth

GOLDEN = json.loads((Path(__file__).parent / "golden" / "ref_digests.json").read_text())


def _run(case):
    spec = GOLDEN[case]
    cfg = synth.CONFIGS[spec["config"]]
    kw = spec["kwargs"]
    model = synth.SyntheticLM(cfg, seed=0)
    step = ref_step.RefStep(model, **kw)
    for it in range(spec["steps"]):
        frac = (it + 1) / 5
        step.muon.group["lr"] = step.muon.group["base_lr"] * frac
        for g in step.adamw.param_groups:
            g["lr"] = g["base_lr"] * frac
        if spec["momentum_warmup"] > 0:
            step.muon.group["momentum"] = 0.85 + 0.10 * min(1.0, it / spec["momentum_warmup"])
        synth.set_grads(model, synth.make_grads(model, it, seed=0))
        step.step()
    out = {}
    names = {id(p): n for n, p in model.named_parameters()}
    for n, p in model.named_parameters():
        out[f"param/{n}"] = p
    for p, st in zip(step.muon.params, step.muon.state):
        for k, v in st.items():
            out[f"muon/{names[id(p)]}/{k}"] = v
    for n, p in model.named_parameters():
        st = step.adamw.state.get(p)
        if st:
            out[f"adam/{n}/exp_avg"] = st["exp_avg"]
            out[f"adam/{n}/exp_avg_sq"] = st["exp_avg_sq"]
    for (n, _), s in zip(model.named_parameters(), step.shadow):
        out[f"ema/{n}"] = s
    return spec, out


@pytest.mark.parametrize("case", sorted(GOLDEN))
def test_oracle_matches_reference_digests(case):
    spec, out = _run(case)
    assert set(out) == set(spec["tensors"])
    for k, d in spec["tensors"].items():
        t = out[k]
        assert str(t.dtype) == d["dtype"] and list(t.shape) == d["shape"], k
        x = t.detach().reshape(-1).to(torch.float64)
        vals = [float(x[i]) for i in d["idx"]]
        assert vals == d["vals"], f"{case}: sampled values differ for {k}"
        assert float(x.sum()) == d["sum"] and float((x * x).sum()) == d["sumsq"], f"{case}: sums differ for {k}"


def test_golden_cases_cover_the_paths():
    # fp32 C1 (config 0), bf16 with mantissa tracking + cautious WD, bf16 plain WD
    assert {"c1_fp32", "micro_bf16_mt_cautious", "micro_bf16_plain"} <= set(GOLDEN)
    mt = GOLDEN["micro_bf16_mt_cautious"]["tensors"]
    assert any(k.endswith("/mant_rem") for k in mt)
    assert GOLDEN["c1_fp32"]["steps"] == 10
    for case in GOLDEN.values():
        for d in case["tensors"].values():
            assert all(math.isfinite(v) for v in d["vals"])
