"""Gradient of the model cost w.r.t. the actions (what CEM-GD steps on): the oracle's
float64 reverse-mode restatement against torch autograd of the reference model (float32),
and against central finite differences."""

from __future__ import annotations

import numpy as np
import pytest

from lewm_flash_b200.model import synthetic_state_dict
from oracle import cost_grad_oracle as cg
from tests.conftest import GOLDEN
from tests.golden.make_cost_grad_golden import (CASES, DESC, FULL_CASES, FULL_DESC, FULL_WEIGHT_SEED, WEIGHT_SEED,
                                                case_inputs)

FIX = np.load(GOLDEN / "cost_grad.npz")
SD = synthetic_state_dict(DESC, WEIGHT_SEED)
FULL_FIX = np.load(GOLDEN / "cost_grad_full.npz")


@pytest.mark.parametrize("name", sorted(CASES))
def test_cost_gradient_matches_reference_autograd(name):
    emb, goal, cand = case_inputs(*CASES[name])
    cost, grad = cg.cost_and_grad(emb, goal, cand, SD, DESC)
    np.testing.assert_allclose(cost, FIX[f"{name}__cost"], rtol=2e-6)
    want = FIX[f"{name}__grad"]
    # float32 autograd against float64: within 1e-4 of the largest gradient entry
    assert np.abs(grad - want).max() <= 1e-4 * np.abs(want).max()


@pytest.mark.parametrize("name", sorted(FULL_CASES))
def test_cost_gradient_matches_reference_autograd_full_width(name):
    """The width-192 / 6-layer predictor the device runs (the fixture its reverse pass is held to)."""
    sd = synthetic_state_dict(FULL_DESC, FULL_WEIGHT_SEED)
    emb, goal, cand = case_inputs(*FULL_CASES[name], desc=FULL_DESC)
    cost, grad = cg.cost_and_grad(emb, goal, cand, sd, FULL_DESC)
    np.testing.assert_allclose(cost, FULL_FIX[f"{name}__cost"], rtol=2e-6)
    want = FULL_FIX[f"{name}__grad"]
    assert np.abs(grad - want).max() <= 1e-4 * np.abs(want).max()


def test_cost_gradient_matches_finite_differences():
    emb, goal, cand = case_inputs(*CASES["h1"])
    _, grad = cg.cost_and_grad(emb, goal, cand, SD, DESC)
    cand = cand.astype(np.float64)
    for idx in [(0, 0, 0, 0), (1, 2, 4, 9), (0, 1, 2, 5)]:
        e = 1e-5
        hi, lo = cand.copy(), cand.copy()
        hi[idx] += e
        lo[idx] -= e
        fd = (cg.cost_and_grad(emb, goal, hi, SD, DESC)[0].sum() - cg.cost_and_grad(emb, goal, lo, SD, DESC)[0].sum())
        assert abs(grad[idx] - fd / (2 * e)) <= 1e-6 * max(1.0, abs(grad[idx]))


def test_refinement_on_the_model_cost_lowers_every_accepted_seed():
    """CEM-GD's refinement (oracle/cem_gd_oracle.py) driven by this gradient on the LeWM model."""
    from oracle import cem_gd_oracle as gd

    emb, goal, cand = case_inputs(*CASES["h3"])
    cost, cost_and_grad = gd.model_cost_fns(emb, goal, SD, DESC)
    seeds = cand[:, :2]
    c0 = cost(seeds)
    acts, c1, info = gd.refine(cost_and_grad, cost, seeds, c0, lr=0.05, steps=3)
    assert (c1 <= c0).all() and info["accept_count"] > 0
    np.testing.assert_allclose(cost(acts), c1, rtol=1e-6)
