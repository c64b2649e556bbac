"""ORACLE (test infrastructure only) -- numpy restatement of CEM-GD's gradient refinement.

Only ``tests/`` may import it; the product package never does.

It restates ``CEMGDSolver._refine_seed_actions`` (reference
``lewm/solvers/cem_gd.py:459-606``): the seed actions (B, K, T, A) are optimized with
Adam (torch defaults: betas 0.9 / 0.999, eps 1e-8, no weight decay) on the mean of their
model costs. After each Adam step the step is retried at factors 1, 1/2, 1/4, 1/10
(backtracking; factor 1 only without it) and each seed keeps the best finite cost below
the cost it had before the step; the parameters are reset to those actions while Adam's
moments carry on. After all steps a seed's refined actions are kept only where their
cost is finite and below the seed's cost. A non-finite cost, loss or gradient ends the
loop early.

The model enters only through ``cost_and_grad(actions) -> (costs (B, K), d mean(costs) /
d actions)`` and ``cost(actions)``; the reference's own test model is the quadratic
embedding cost of ``lewm/solvers/cem_gd.py:748-761`` (``quadratic_cost`` below).
``tests/golden/make_cem_gd_golden.py`` pins this restatement to the reference.
"""

from __future__ import annotations

from typing import Callable, Tuple

import numpy as np

F32 = np.float32


def quadratic_cost(target: np.ndarray):
    """The reference's ``_QuadraticEmbeddingCost``: sum over (T, A) of (a - target)^2, and
    the gradient of the mean over (B, K) of that cost."""
    target = np.asarray(target, dtype=F32)

    def cost(a):
        return ((np.asarray(a, F32) - target) ** 2).sum(axis=(2, 3), dtype=F32).astype(F32)

    def cost_and_grad(a):
        a = np.asarray(a, F32)
        c = cost(a)
        # autograd's order: mean backward (1 / N), then pow backward 2 * (a - target)
        g = ((F32(1.0) / F32(c.size)) * (F32(2.0) * (a - target))).astype(F32)
        return c, g

    return cost, cost_and_grad


def refine(cost_and_grad: Callable, cost: Callable, seed_actions: np.ndarray, seed_costs: np.ndarray, *,
           lr: float, steps: int, backtracking: bool = True) -> Tuple[np.ndarray, np.ndarray, dict]:
    """Returns (accepted actions, accepted costs, {"accept_count", "step_accepted", "model_cost_evals"})."""
    seed = np.asarray(seed_actions, F32)
    seed_c = np.asarray(seed_costs, F32)
    params = seed.copy()
    m = np.zeros_like(params)
    v = np.zeros_like(params)
    beta1, beta2 = 0.9, 0.999  # torch's scalars are Python doubles, rounded once to float32
    w1, b2, w2, eps = F32(1.0 - beta1), F32(beta2), F32(1.0 - beta2), F32(1e-8)
    current = seed_c.copy()
    accepted_any = np.zeros(seed_c.shape, bool)
    factors = [1.0, 0.5, 0.25, 0.1] if backtracking else [1.0]
    width = seed.shape[1]
    evals = 0
    final_a, final_c = seed.copy(), seed_c.copy()
    for t in range(1, steps + 1):
        c, g = cost_and_grad(params)
        evals += width
        if not np.isfinite(c).all() or not np.isfinite(c.mean(dtype=F32)):
            break
        if not np.isfinite(g).all():
            break
        before = params.copy()
        previous = current.copy()
        # torch.optim.Adam on CPU tensors (single-tensor path): m.lerp_(g, 1 - beta1)
        # (weight < 0.5: m + w (g - m)), v * beta2 + (1 - beta2) g g, bias corrections in
        # double, then param + (-step_size * m) / (sqrt(v) / sqrt(bc2) + eps)
        m = (m + w1 * (g - m)).astype(F32)
        v = (v * b2 + (w2 * g) * g).astype(F32)
        step_size = lr / (1.0 - beta1 ** t)
        bc2_sqrt = F32((1.0 - beta2 ** t) ** 0.5)
        denom = (np.sqrt(v) / bc2_sqrt + eps).astype(F32)
        full = (before + (F32(-step_size) * m) / denom).astype(F32)
        update = (full - before).astype(F32)
        best_a, best_c = before, previous
        for f in factors:
            cand = (before + F32(f) * update).astype(F32)
            cc = cost(cand)
            evals += width
            improved = np.isfinite(cc) & (cc < best_c)
            best_a = np.where(improved[..., None, None], cand, best_a)
            best_c = np.where(improved, cc, best_c)
        accepted_any |= best_c < previous
        current = best_c.astype(F32)
        params = best_a.astype(F32)
        final_a, final_c = params.copy(), current.copy()
    keep = np.isfinite(final_c) & (final_c < seed_c)
    out_a = np.where(keep[..., None, None], final_a, seed)
    out_c = np.where(keep, final_c, seed_c)
    return out_a.astype(F32), out_c.astype(F32), {"accept_count": int(keep.sum()),
                                                  "step_accepted": accepted_any, "model_cost_evals": evals}


def model_cost_fns(emb, goal_emb, sd, desc, history_size: int = 3):
    """``cost`` and ``cost_and_grad`` of the LeWM model cost for ``refine``: the gradient of the
    mean over (B, K) of the costs, from the reverse-mode restatement in
    ``oracle/cost_grad_oracle.py`` (float64, returned as float32)."""
    from oracle import cost_grad_oracle as cg

    def cost_and_grad(a):
        c, g = cg.cost_and_grad(emb, goal_emb, a, sd, desc, history_size)
        return c.astype(F32), (g / c.size).astype(F32)

    def cost(a):
        return cost_and_grad(a)[0]

    return cost, cost_and_grad
