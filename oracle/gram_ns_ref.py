"""TEST INFRASTRUCTURE ONLY — CPU restatement of the Gram Newton-Schulz iteration.

The reference calls gram_newton_schulz.GramNewtonSchulz(ns_coefficients=POLAR_EXPRESS_COEFFICIENTS,
gram_newton_schulz_reset_iterations=[2]) (transformer_lm/sol_modules.py:355-359, :369);
that package (gram-newton-schulz==0.1.6) is not in the reference tree, so this is
a restatement of the published method, not of the package: parity unpinned
against the package. It follows the schedule the engine runs:

  X0 = u / (||u||_F * safety + eps), wide orientation (transpose when r > c)
  R = X0 X0^T, Q = I
  for t in range(T):
      if t in resets and t > 0:  X = Q X;  R = X X^T;  Q = I
      P = a_t I + b_t R + c_t R^2;  Q = Q P
      if t < T-1 and t+1 not a restart:  R = P R P
  out = Q X

``store=torch.float16`` (or bfloat16) rounds X0 and every product to that type
as the engine stores them (binary16 is what the engine's Gram mode uses);
``store=None`` runs in float64 (the exact-arithmetic target).
"""
from __future__ import annotations

import torch


def _rnd(x, store):
    return x.to(store).to(x.dtype) if store is not None else x


def gram_ns(U: torch.Tensor, table, resets=(2,), eps=1e-7, safety=1.0, store=None) -> torch.Tensor:
    bf16 = store
    dt = torch.float32 if store is not None else torch.float64
    outs = []
    T = len(table)
    for u in U:
        u = u.to(dt)
        tall = u.shape[0] > u.shape[1]
        X = u.t() if tall else u
        s = 1.0 / (torch.linalg.norm(u) * safety + eps)
        X = _rnd(X * s, bf16)
        R = _rnd(X @ X.t(), bf16)
        Q = None
        pend = 1.0
        for t in range(T):
            a, b, c = (float(v) for v in table[t])
            if t > 0 and t in resets:
                X = _rnd(pend * (Q @ X), bf16)
                R = _rnd(X @ X.t(), bf16)
                Q = None
                pend = 1.0
            R2 = R @ R
            eye = torch.eye(R.shape[0], dtype=dt)
            P = _rnd(a * eye + b * R + c * R2, bf16)
            Q = P if Q is None else _rnd(Q @ P, bf16)
            if t < T - 1 and not (t + 1 in resets):
                T1 = _rnd(P @ R, bf16)
                R = _rnd(T1 @ P, bf16)
        out = pend * (Q @ X)
        out = out.to(torch.bfloat16).to(dt) if store is not None else out
        outs.append(out.t() if tall else out)
    return torch.stack(outs)


def polar_factor(U: torch.Tensor) -> torch.Tensor:
    """Exact orthogonal polar factor U V^T (float64 SVD), the limit of the iteration."""
    outs = []
    for u in U.to(torch.float64):
        Uu, _, Vh = torch.linalg.svd(u, full_matrices=False)
        outs.append(Uu @ Vh)
    return torch.stack(outs)
