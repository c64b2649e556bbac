"""The oracle against the reference's runs at the benchmarked iCEM configurations.

Fixtures from ``tests/golden/make_headline_golden.py`` (the reference's own
``ICEMSolver`` / ``run_static_icem_chain``, fp32 CPU): bucketed iCEM 300 -> 60 over
30 iterations, brown noise, retention 3 / 5, 1 env with history 1 and 4 envs with
history 3; plain CEM 300 / 30 / 30, 1 env, history 1. The oracle's chain, driven by the reference's per-iteration costs,
selects the reference's elites in every iteration and reproduces its refit and
outputs; the oracle's fp32 model cost reproduces the reference's costs of the
first iteration's 300 candidates.
"""

import json

import numpy as np
import pytest

from oracle import icem_oracle as io
from oracle import lewm_oracle as lo
from tests.golden_io import GOLDEN, assert_same_topk, load, weights_of

HEADLINE_CASES = sorted(p.name for p in GOLDEN.glob("icem_headline_*.npz"))


@pytest.mark.parametrize("case", HEADLINE_CASES)
def test_oracle_chain_fed_reference_costs_reproduces_reference(case):
    d = load(case)
    kw = json.loads(str(d["solver"]))
    n = int(d["n_iters"])
    assert io.sample_counts(n, kw["num_samples"], kw["topk"], kw["sample_decay"],
                            kw["sample_count_bucket_size"]) == d["counts"].tolist()
    costs = iter([d[f"cost_{i}"] for i in range(n)])
    trace = []
    act, std, fcost = io.run_static_icem_chain(
        lambda e, g, c: next(costs), d["emb"], d["goal"], d["mean0"], d["var0"],
        [d[f"noise_{i}"] for i in range(n)], topk=kw["topk"], elite_retention=kw["elite_retention"], trace=trace)
    np.testing.assert_allclose(trace[0]["candidates"], d["cand_0"], rtol=1e-6, atol=1e-6)
    for i, t in enumerate(trace):
        assert_same_topk(t["topk_inds"], d[f"inds_{i}"], d[f"cost_{i}"], f"iteration {i}")
        scale = float(np.abs(d[f"mean_{i}"]).max()) + 1.0
        np.testing.assert_allclose(t["mean"], d[f"mean_{i}"], rtol=1e-5, atol=1e-6 * scale)
        np.testing.assert_allclose(t["var"], d[f"std_{i}"], rtol=1e-5, atol=1e-6 * scale)
    scale = float(np.abs(d["solve_actions"]).max()) + 1.0
    np.testing.assert_allclose(act, d["solve_actions"], rtol=1e-5, atol=1e-6 * scale)
    np.testing.assert_allclose(std, d["solve_var"], rtol=1e-5, atol=1e-6 * scale)
    np.testing.assert_allclose(fcost, d["solve_costs"], rtol=2e-6)


@pytest.mark.parametrize("case", HEADLINE_CASES)
def test_oracle_model_cost_of_first_iteration_matches_reference(case):
    d = load(case)
    desc, sd = weights_of(d)
    got = lo.get_cost_from_embeddings(d["emb"], d["goal"], d["cand_0"], sd, desc)
    np.testing.assert_allclose(got, d["cost_0"], rtol=2e-6, atol=1e-5)
