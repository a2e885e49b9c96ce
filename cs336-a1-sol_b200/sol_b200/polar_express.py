"""Newton-Schulz coefficient tables.

* ``QUINTIC`` — the constant (a, b, c) of the reference's fallback iteration
  ``zeropower_via_newtonschulz5`` (transformer_lm/sol_modules.py:281).
* ``polar_express(T)`` — a per-step table derived here with the greedy
  minimax procedure of Polar Express (Amsel, Persson, Musco, Gower,
  arXiv:2505.16932). The reference obtains its table from the third-party
  package ``gram-newton-schulz==0.1.6`` (``POLAR_EXPRESS_COEFFICIENTS``,
  imported at sol_modules.py:55 and used at :356); that package is not part of
  the reference tree, so the table is recomputed from the published method:

  1. Singular values of the Frobenius-normalised input lie in [l, u] = [l0, 1].
  2. Each step picks the odd quintic p(x) = a x + b x^3 + c x^5 that minimises
     max |1 - p(x)| over [max(l, cushion * u), u] (Remez exchange with four
     alternation points; the interior extrema are the roots of p'(x), a
     quadratic in x^2).
  3. The polynomial is rescaled so that it is centred on 1 over the true
     interval [l, u] (1 - p(l) = p(u) - 1), and the interval is mapped:
     l <- p(l), u <- p(u).
  4. Safety margin: each polynomial is designed for [l, u * (1 + margin)], so a
     singular value pushed slightly above the nominal top by rounding stays in
     the region where the next polynomial is bounded. Without the margin the
     composition diverges in 16-bit arithmetic for singular values that land at
     the top of an interval (the equioscillation maximum is attained inside the
     interval, so such values are common).

  ``l0``, ``cushion`` and ``margin`` are this library's choices (documented
  defaults); the table is therefore "parity unpinned" against the package's
  own constants.
"""
from __future__ import annotations

import math

QUINTIC = (3.4445, -4.7750, 2.0315)


def _solve4(A, y):
    """Gaussian elimination with partial pivoting for a 4x4 system."""
    n = 4
    M = [list(A[i]) + [y[i]] for i in range(n)]
    for col in range(n):
        piv = max(range(col, n), key=lambda r: abs(M[r][col]))
        M[col], M[piv] = M[piv], M[col]
        if M[col][col] == 0.0:
            raise ZeroDivisionError("singular Remez system")
        for r in range(col + 1, n):
            f = M[r][col] / M[col][col]
            for k in range(col, n + 1):
                M[r][k] -= f * M[col][k]
    x = [0.0] * n
    for r in range(n - 1, -1, -1):
        s = M[r][n] - sum(M[r][k] * x[k] for k in range(r + 1, n))
        x[r] = s / M[r][r]
    return x


def _poly(coef, x):
    a, b, c = coef
    x2 = x * x
    return x * (a + x2 * (b + c * x2))


def optimal_odd_quintic(lo: float, hi: float, iters: int = 100, tol: float = 1e-15):
    """Minimax odd quintic approximation of 1 on [lo, hi] (0 < lo < hi).

    Returns (a, b, c, E) with |1 - p(x)| <= |E| on the interval and equal
    oscillation at lo, the two interior extrema and hi.
    """
    if not (0.0 < lo < hi):
        raise ValueError("need 0 < lo < hi")
    pts = [lo + (hi - lo) * (1.0 - math.cos(math.pi * i / 3.0)) / 2.0 for i in range(4)]
    coef = (0.0, 0.0, 0.0)
    E = 0.0
    for _ in range(iters):
        A = [[x, x ** 3, x ** 5, (-1.0) ** i] for i, x in enumerate(pts)]
        a, b, c, E = _solve4(A, [1.0] * 4)
        coef = (a, b, c)
        # interior extrema: p'(x) = a + 3 b x^2 + 5 c x^4 = 0
        qa, qb, qc = 5.0 * c, 3.0 * b, a
        roots = []
        if abs(qa) > 0.0:
            disc = qb * qb - 4.0 * qa * qc
            if disc >= 0.0:
                sq = math.sqrt(disc)
                for y in ((-qb - sq) / (2.0 * qa), (-qb + sq) / (2.0 * qa)):
                    if y > 0.0:
                        x = math.sqrt(y)
                        if lo < x < hi:
                            roots.append(x)
        roots.sort()
        if len(roots) != 2:
            break  # degenerate: keep the last equioscillating solution
        new = [lo, roots[0], roots[1], hi]
        moved = max(abs(p - q) for p, q in zip(new, pts))
        pts = new
        if moved < tol * hi:
            break
    return coef[0], coef[1], coef[2], E


def polar_express(steps: int = 5, l0: float = 1e-3, cushion: float = 0.02, margin: float = 0.05):
    """Per-step (a, b, c) table of length ``steps`` (float64 values)."""
    lo, hi = float(l0), 1.0
    table = []
    for _ in range(steps):
        top = hi * (1.0 + margin)
        a, b, c, _ = optimal_odd_quintic(max(lo, cushion * top), top)
        pl, pu = _poly((a, b, c), lo), _poly((a, b, c), top)
        k = 2.0 / (pl + pu)
        a, b, c = a * k, b * k, c * k
        table.append((a, b, c))
        lo, hi = _poly((a, b, c), lo), _poly((a, b, c), top)
    return table


def apply_table(table, x: float) -> float:
    """Composition of the table's polynomials at a scalar singular value."""
    for coef in table:
        x = _poly(coef, x)
    return x


def table_for(kind: str, steps: int):
    """Coefficient table of ``steps`` rows for 'quintic' or 'polar_express'."""
    if kind == "quintic":
        return [QUINTIC] * steps
    if kind == "polar_express":
        return polar_express(steps)
    raise ValueError(f"unknown coefficient table {kind!r}")
