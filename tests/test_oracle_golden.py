"""The oracle against the reference's own outputs (golden fixtures from tests/golden/make_golden.py)."""

import json

import numpy as np
import pytest

from oracle import icem_oracle as io
from oracle import lewm_oracle as lo
from tests.golden_io import CHAIN_CASES, GOLDEN, MODEL_COST_CASES, desc_of, load, weights_of


def test_sample_count_schedules_match_reference():
    cases = json.loads((GOLDEN / "sample_counts.json").read_text())
    assert cases["bucketed_300"]["counts"] == [300, 240, 240, 180, 180, 120, 120, 120] + [60] * 22
    for name, c in cases.items():
        kw = c["kwargs"]
        got = io.sample_counts(kw["n_steps"], kw["num_samples"], kw["topk"], kw.get("sample_decay", 1.0),
                               kw.get("sample_count_bucket_size", 0))
        assert got == c["counts"], name
        assert sum(got) == c["evals"], name


@pytest.mark.parametrize("case", ["raw_b2", "raw_b1", "block_b2", "block1_b2", "white"])
def test_colored_noise_matches_reference(case):
    d = load("colored_noise.npz")
    kw = json.loads(str(d[case + "_kwargs"]))
    got = io.color_white_noise(d[case + "_white"], kw["horizon"], kw["action_dim"], kw["beta"],
                               kw["action_block"], kw["time_axis"])
    np.testing.assert_allclose(got, d[case + "_colored"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("n,beta", [(25, 2.0), (25, 1.0), (5, 2.0), (10, 2.0)])
def test_coloring_matrix_equals_fft_filter(n, beta):
    rng = np.random.default_rng(0)
    x = rng.standard_normal((7, n))
    w = io.coloring_matrix(n, beta)
    freqs = np.fft.rfftfreq(n)
    freqs[0] = 1.0
    scale = freqs ** (-beta / 2)
    scale[0] = scale[1]
    ref = np.fft.irfft(np.fft.rfft(x, axis=-1) * scale, n=n, axis=-1)
    np.testing.assert_allclose(x @ w.T, ref, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("case", MODEL_COST_CASES)
def test_model_cost_matches_reference(case):
    d = load(case)
    desc, sd = weights_of(d)
    pred = lo.rollout_from_embeddings(d["emb"], d["cand"], sd, desc)
    np.testing.assert_allclose(pred, d["pred"], rtol=1e-4, atol=2e-5)
    cost = lo.get_cost_from_embeddings(d["emb"], d["goal"], d["cand"], sd, desc)
    np.testing.assert_allclose(cost, d["cost"], rtol=2e-6, atol=1e-5)


@pytest.mark.parametrize("case", CHAIN_CASES)
def test_icem_chain_matches_reference(case):
    d = load(case)
    desc, sd = weights_of(d)
    kw = json.loads(str(d["solver"]))
    n = int(d["n_iters"])
    noise = [d[f"noise_{i}"] for i in range(n)]
    low = d["low"] if d["low"].size else None
    high = d["high"] if d["high"].size else None
    trace = []
    cost_fn = lambda e, g, c: lo.get_cost_from_embeddings(e, g, c, sd, desc)
    act, std, fcost = io.run_static_icem_chain(
        cost_fn, d["emb"], d["goal"], d["mean0"], d["var0"], noise, topk=kw["topk"],
        elite_retention=kw.get("elite_retention", 0), momentum_alpha=kw.get("momentum_alpha", 0.0),
        return_best_elite=kw.get("return_best_elite", False), action_low=low, action_high=high, trace=trace)
    for i, t in enumerate(trace):
        np.testing.assert_allclose(t["candidates"], d[f"cand_{i}"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(t["costs"], d[f"cost_{i}"], rtol=2e-6, atol=1e-5)
        assert np.array_equal(t["topk_inds"], d[f"inds_{i}"]), f"elite set differs at iteration {i}"
    np.testing.assert_allclose(act, d["actions"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(act, d["solve_actions"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(std, d["std"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(fcost, d["final_cost"], rtol=2e-6, atol=1e-5)
    np.testing.assert_allclose(fcost, d["solve_costs"], rtol=2e-6, atol=1e-5)


def test_chain_fed_reference_costs_selects_reference_elites():
    """Top-k/refit alone, driven by the reference's own per-iteration costs, is bit-exact on indices."""
    for case in CHAIN_CASES:
        d = load(case)
        kw = json.loads(str(d["solver"]))
        for i in range(int(d["n_iters"])):
            vals, inds = io.topk_smallest(d[f"cost_{i}"], kw["topk"])
            assert np.array_equal(inds, d[f"inds_{i}"]), (case, i)
            np.testing.assert_array_equal(vals, d[f"vals_{i}"])


def test_topk_ties_prefer_lower_index_and_nan_last():
    c = np.array([[3.0, 1.0, 1.0, np.nan, 0.5, 1.0]], dtype=np.float32)
    vals, inds = io.topk_smallest(c, 5)
    assert inds.tolist() == [[4, 1, 2, 5, 0]]
    vals, inds = io.topk_smallest(c, 6)
    assert inds[0, -1] == 3


def test_philox_known_answer():
    """Random123's published Philox4x32-10 known-answer vectors (kat_vectors)."""
    z = lambda v: np.array([v], dtype=np.uint64)
    out = io.philox4x32_10((z(0), z(0), z(0), z(0)), (z(0), z(0)))
    assert [int(o[0]) for o in out] == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    out = io.philox4x32_10((z(0xFFFFFFFF),) * 4, (z(0xFFFFFFFF),) * 2)
    assert [int(o[0]) for o in out] == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    out = io.philox4x32_10((z(0x243F6A88), z(0x85A308D3), z(0x13198A2E), z(0x03707344)),
                           (z(0xA4093822), z(0x299F31D0)))
    assert [int(o[0]) for o in out] == [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]
