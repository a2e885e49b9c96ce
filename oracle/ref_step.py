"""TEST INFRASTRUCTURE ONLY — CPU restatement of the reference optimizer step.

Each function cites the reference lines it restates
(vincentzed/cs336-a1-sol, transformer_lm/sol_modules.py unless noted).
The operations are the same torch operations in the same order, so on CPU the
results are bit-identical to the reference (pinned by tests/golden/).
"""
from __future__ import annotations

import math
from collections import defaultdict

import torch

QUINTIC = (3.4445, -4.7750, 2.0315)  # sol_modules.py:281


def zeropower_ns5(G: torch.Tensor, steps: int = 5, eps: float = 1e-7) -> torch.Tensor:
    """Quintic Newton-Schulz, bf16 (sol_modules.py:278-293)."""
    assert G.ndim == 2
    a, b, c = QUINTIC
    X = G.bfloat16()
    X = X / (X.norm() + eps)
    transposed = G.size(0) > G.size(1)
    if transposed:
        X = X.t()
    for _ in range(steps):
        A = X @ X.t()
        B = b * A + c * (A @ A)
        X = a * X + B @ X
    if transposed:
        X = X.t()
    return X


def ortho_batch_quintic(U: torch.Tensor, ns_steps: int) -> torch.Tensor:
    """NorMuonGNS._orthogonalize_batch without GNS (sol_modules.py:366-370)."""
    return torch.stack([zeropower_ns5(U[i], steps=ns_steps) for i in range(U.shape[0])])


class RefNorMuon:
    """NorMuonGNS.step (sol_modules.py:372-424) over a list of parameters.

    State per parameter index: momentum_buffer, v_row, mant_rem (as in the reference).
    ``ortho`` maps (U, ns_steps) -> o; default is the quintic fallback.
    """

    def __init__(self, params, lr=2e-3, momentum=0.95, beta2=0.95, nesterov=True, ns_steps=5,
                 weight_decay=0.0, cautious_wd=False, bf16_master=False, ortho=None):
        self.params = list(params)
        self.group = dict(lr=lr, momentum=momentum, beta2=beta2, nesterov=nesterov, ns_steps=ns_steps,
                          weight_decay=weight_decay)
        self.cautious_wd = cautious_wd
        self.bf16_master = bf16_master
        self.ortho = ortho or ortho_batch_quintic
        self.state = [dict() for _ in self.params]
        self.last_o = {}  # shape -> orthogonalised, normalised update of the last step (for tests)

    @torch.no_grad()
    def step(self):
        g = self.group
        beta, beta2 = g["momentum"], g["beta2"]
        ns_steps, nesterov = g["ns_steps"], g["nesterov"]
        lr, wd = g["lr"], g["weight_decay"]
        by_shape = defaultdict(list)
        for i, p in enumerate(self.params):
            if p.grad is not None:
                by_shape[tuple(p.shape)].append(i)
        for shape, idx in by_shape.items():
            params = [self.params[i] for i in idx]
            for i, p in zip(idx, params):
                st = self.state[i]
                if "momentum_buffer" not in st:
                    st["momentum_buffer"] = torch.zeros_like(p)
                    st["v_row"] = torch.zeros_like(p[..., 0:1], dtype=torch.float32)
            bufs = torch.stack([self.state[i]["momentum_buffer"] for i in idx])
            grads = torch.stack([p.grad for p in params])
            v_rows = torch.stack([self.state[i]["v_row"] for i in idx])
            bufs.lerp_(grads, 1 - beta)
            u = grads.lerp(bufs, beta) if nesterov else bufs
            o = self.ortho(u, ns_steps).float()
            vnorm = o.norm(dim=(-2, -1), keepdim=True)
            v_rows.lerp_(o.mul(o).mean(dim=-1, keepdim=True), 1 - beta2)
            o = o * v_rows.sqrt().add(1e-10).reciprocal()
            o = o * (vnorm / o.norm(dim=(-2, -1), keepdim=True).add(1e-10))
            o = o * math.sqrt(max(1.0, shape[-2] / shape[-1]))
            self.last_o[shape] = o.clone()
            for j, (i, p) in enumerate(zip(idx, params)):
                st = self.state[i]
                st["momentum_buffer"].copy_(bufs[j])
                st["v_row"].copy_(v_rows[j])
                mt = self.bf16_master and p.dtype == torch.bfloat16
                if mt:
                    if "mant_rem" not in st:
                        st["mant_rem"] = torch.zeros_like(p)
                    w = p.float().add_(st["mant_rem"].float())
                else:
                    w = p
                if wd:
                    if self.cautious_wd:
                        mask = (o[j] * w) > 0
                        w.mul_(1 - lr * wd * mask.to(w.dtype))
                    else:
                        w.mul_(1 - lr * wd)
                w.add_(o[j].to(w.dtype), alpha=-lr)
                if mt:
                    p.copy_(w)
                    st["mant_rem"].copy_(w.sub_(p.float()))


def make_reference_adamw(groups, betas=(0.9, 0.95), eps=1e-8):
    """The reference's AdamW is torch's fused implementation (sol_modules.py:476).

    The oracle runs torch's own fused AdamW on CPU tensors (the library the
    reference calls), so it is the reference arithmetic by construction.
    """
    return torch.optim.AdamW(groups, betas=betas, eps=eps, fused=True)


def _fma32(a, b, c):
    """fp32 fused multiply-add: a*b + c with one rounding (exact product in float64;
    the float64 sum is then rounded once more to fp32, which matches a true fma
    except in vanishingly rare double-rounding cases)."""
    return (a.double() * b.double() + c.double()).float()


class MasterAdamW:
    """AdamW with a bf16 low-mantissa remainder, fp32 moments and cautious decay.

    torch's fused AdamW element formula (ATen/native/cuda/fused_adam_utils.cuh,
    ADAMW mode: exp_avg = fma(b1, m, fma(-b1, g, g)), the same for exp_avg_sq)
    applied to w = float(p) + float(rem), with NorMuon's cautious mask and
    remainder split (sol_modules.py:406-424).
    """

    def __init__(self, params, lr, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0, cautious=False):
        self.params = list(params)
        self.lr, self.betas, self.eps, self.wd, self.cautious = lr, betas, eps, weight_decay, cautious
        self.state = [dict(step=0, m=torch.zeros_like(p, dtype=torch.float32),
                           v=torch.zeros_like(p, dtype=torch.float32),
                           rem=torch.zeros_like(p) if p.dtype == torch.bfloat16 else None) for p in self.params]

    @torch.no_grad()
    def step(self):
        f32 = lambda x: torch.tensor(x, dtype=torch.float32)  # noqa: E731
        b1, b2 = f32(self.betas[0]), f32(self.betas[1])
        lr, wd, eps = f32(self.lr), f32(self.wd), f32(self.eps)
        for p, st in zip(self.params, self.state):
            if p.grad is None:
                continue
            st["step"] += 1
            t = f32(float(st["step"]))
            bc1 = 1 - torch.pow(b1, t)
            bc2_sqrt = torch.sqrt(1 - torch.pow(b2, t))
            g = p.grad.float()
            w = p.float()
            if st["rem"] is not None:
                w = w + st["rem"].float()
            m = _fma32(b1, st["m"], _fma32(-b1, g, g))
            g2 = g * g
            v = _fma32(b2, st["v"], _fma32(-b2, g2, g2))
            if self.wd:
                lr_wd = lr * wd
                if self.cautious:
                    mask = ((m * w) > 0).float()
                    w = w * (1 - lr_wd * mask)
                else:
                    w = _fma32(-lr_wd, w, w)
            denom = torch.sqrt(v) / bc2_sqrt + eps
            w = w - ((lr / bc1) * m) / denom
            st["m"], st["v"] = m, v
            if st["rem"] is not None:
                pn = w.to(torch.bfloat16)
                st["rem"] = (w - pn.float()).to(torch.bfloat16)
                p.copy_(pn)
            else:
                p.copy_(w)


def ema_update(shadows, params, decay):
    """EmaWeights._update_slow (sol_modules.py:1266-1268): s = lerp(s, p.float(), 1 - decay)."""
    for p, s in zip(params, shadows):
        s.lerp_(p.detach().float(), 1 - decay)


def route(named_params):
    """build_optimizers routing (sol_modules.py:437-466) -> (muon, embed, norm, ve) name lists."""
    adam_keys = ("resid_lambdas", "post_lambdas", "x0_lambdas", "_xsa_alpha", "smear", "skip_gate",
                 "_skip_lambda", "_backout", "_second_gate", "_ve_gate")
    muon, embed, norm, ve = [], [], [], []
    seen = set()
    for name, p in named_params:
        if not p.requires_grad or id(p) in seen:
            continue
        seen.add(id(p))
        if "value_embeds" in name:
            ve.append(name)
        elif ("token_embeddings" in name) or ("lm_head" in name) or ("second_embeds" in name):
            embed.append(name)
        elif any(k in name for k in adam_keys):
            norm.append(name)
        elif p.ndim >= 2:
            muon.append(name)
        else:
            norm.append(name)
    return muon, embed, norm, ve


class RefStep:
    """One full optimizer step of train_sol.py:500-507 on a parameter container:
    muon.step(); adamw.step(); ema.update()  (with the reference's routing and groups)."""

    def __init__(self, model, *, muon_lr, adam_lr, embed_lr, weight_decay, betas=(0.9, 0.95), eps=1e-8,
                 cautious_wd=False, bf16_master=False, ve_lr=None, ema_decay=0.999, ortho=None):
        named = list(model.named_parameters())
        by_name = dict(named)
        muon_n, embed_n, norm_n, ve_n = route(named)
        self.names = [n for n, _ in named]
        self.muon = RefNorMuon([by_name[n] for n in muon_n], lr=muon_lr, weight_decay=weight_decay,
                               cautious_wd=cautious_wd, bf16_master=bf16_master, ortho=ortho)
        groups = []
        if embed_n:
            groups.append({"params": [by_name[n] for n in embed_n], "lr": embed_lr, "weight_decay": 0.0})
        if ve_n:
            groups.append({"params": [by_name[n] for n in ve_n], "lr": ve_lr if ve_lr is not None else embed_lr,
                           "weight_decay": 0.0, "betas": (0.75, 0.95)})
        if norm_n:
            groups.append({"params": [by_name[n] for n in norm_n], "lr": adam_lr, "weight_decay": 0.0})
        self.adamw = make_reference_adamw(groups, betas=betas, eps=eps)
        self.muon.group["base_lr"] = muon_lr            # base_lr stash (sol_modules.py:480-482)
        for g in self.adamw.param_groups:
            g["base_lr"] = g["lr"]
        self.params = [p for _, p in named]
        self.shadow = [p.detach().float().clone() for p in self.params]
        self.ema_decay = ema_decay

    def step(self, ema=True):
        self.muon.step()
        self.adamw.step()
        if ema:
            ema_update(self.shadow, self.params, self.ema_decay)
