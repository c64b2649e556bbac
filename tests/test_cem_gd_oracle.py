"""CEM-GD gradient refinement: the oracle restatement against the reference's own run.

The fixture (``tests/golden/make_cem_gd_golden.py``) holds the reference
``CEMGDSolver._refine_seed_actions`` (``lewm/solvers/cem_gd.py:459-606``) outputs on its
quadratic embedding cost, with and without backtracking.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import cem_gd_oracle as gd
from tests.conftest import GOLDEN
from tests.golden.make_cem_gd_golden import CASES, case_inputs

FIX = np.load(GOLDEN / "cem_gd_refine.npz")


@pytest.mark.parametrize("name", sorted(CASES))
def test_refinement_matches_reference(name):
    shape, lr, steps, bt, seed = CASES[name]
    seed_actions, target = case_inputs(shape, seed)
    cost, cost_and_grad = gd.quadratic_cost(target)
    acts, costs, info = gd.refine(cost_and_grad, cost, seed_actions, cost(seed_actions), lr=lr, steps=steps,
                                  backtracking=bt)
    np.testing.assert_allclose(acts, FIX[f"{name}__actions"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(costs, FIX[f"{name}__costs"], rtol=1e-5, atol=1e-6)
    assert info["accept_count"] == int(FIX[f"{name}__accept_count"])
    assert info["model_cost_evals"] == int(FIX[f"{name}__evals"])


def test_refinement_never_returns_a_worse_cost():
    rng = np.random.default_rng(9)
    seeds = rng.standard_normal((2, 3, 5, 10)).astype(np.float32)
    cost, cost_and_grad = gd.quadratic_cost(rng.standard_normal((2, 1, 5, 10)).astype(np.float32))
    c0 = cost(seeds)
    _, c1, _ = gd.refine(cost_and_grad, cost, seeds, c0, lr=50.0, steps=3)  # steps far past the minimum
    assert (c1 <= c0).all()


def test_non_finite_gradient_stops_and_keeps_the_seeds():
    seeds = np.zeros((1, 2, 5, 4), np.float32)

    def cost(a):
        return np.full(a.shape[:2], 1.0, np.float32)

    def cost_and_grad(a):
        return cost(a), np.full(a.shape, np.nan, np.float32)

    acts, costs, info = gd.refine(cost_and_grad, cost, seeds, cost(seeds), lr=0.1, steps=4)
    np.testing.assert_array_equal(acts, seeds)
    assert info["accept_count"] == 0 and info["model_cost_evals"] == 2
