"""The reference's quadratic-cost solver tests, ported onto the device kernels.

The reference tests drive its solvers with a model whose cost is a quadratic distance to
a target (reference ``tests/test_lewm_icem.py:39-46``,
``tests/test_lewm_icem_static_compile.py:86-110``). The B200 plan fuses the JEPA model
cost, so here the chain runs the library's sampling (``lewm_sample_candidates``) and
elite selection + refit (``lewm_topk_refit``) kernels with that quadratic cost computed
on the device, and is checked against the oracle's ``run_static_icem_chain`` on the same
post-coloring noise.
"""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from lewm_flash_b200.model import ModelDesc, synthetic_state_dict  # noqa: E402
from lewm_flash_b200.runtime import PlanOptions, Runtime  # noqa: E402
from oracle import icem_oracle as io  # noqa: E402

pytestmark = pytest.mark.gpu


def quadratic_cost(cand: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    return ((cand - target) ** 2).sum(dim=(2, 3))


def device_chain(rt, target, mean, std, noise_steps, topk):
    """Slot 0 = mean, the rest mean + std * noise (no retention), quadratic cost, top-k + refit,
    all on the device. Returns the final mean, std, final cost, and per iteration the costs
    and elite indices."""
    opts = PlanOptions(num_samples=noise_steps[0].shape[1], topk=topk, n_steps=len(noise_steps), beta=0.0,
                       elite_retention=0)
    m, s = mean.clone(), std.clone()
    out, costs, idx = None, [], []
    for it, noise in enumerate(noise_steps):
        cand = rt.sample_candidates(opts, noise.shape[1], it, m, s, injected_noise=noise)
        c = quadratic_cost(cand, target)
        out = rt.topk_refit(c, cand, m, s, topk)
        costs.append(c.cpu().numpy())
        idx.append(out["topk_idx"].cpu().numpy())
        m, s = out["mean"], out["std"]
    return m, s, out["final_cost"], costs, idx


@pytest.fixture(scope="module")
def rt():
    desc = ModelDesc()
    r = Runtime(desc, synthetic_state_dict(desc, 0), torch.device("cuda", 0))
    yield r
    r.close()


@pytest.fixture(scope="module")
def rt_a1():
    """A context whose model has one action dim (the sampler works at the model's action dim)."""
    desc = ModelDesc(action_dim=1, smoothed_dim=1)
    r = Runtime(desc, synthetic_state_dict(desc, 0), torch.device("cuda", 0))
    yield r
    r.close()


def test_sampling_rejects_an_action_dim_other_than_the_models(rt):
    dev = torch.device("cuda", 0)
    opts = PlanOptions(num_samples=4, topk=2, n_steps=1)
    with pytest.raises(ValueError):
        rt.sample_candidates(opts, 4, 0, torch.zeros(1, 2, 1, device=dev), torch.ones(1, 2, 1, device=dev))


def test_static_chain_decreases_dummy_quadratic_cost(rt_a1):
    """Reference tests/test_lewm_icem_static_compile.py:86-110 with its inputs: target ones,
    horizon 2, one action dim, noise rows 0 / 1 / 2 / -1, top-2."""
    rt = rt_a1
    dev = torch.device("cuda", 0)
    target = torch.ones(1, 1, 2, 1, device=dev)
    mean = torch.zeros(1, 2, 1, device=dev)
    var = torch.ones_like(mean)
    noise = torch.tensor([[[[0.0], [0.0]], [[1.0], [1.0]], [[2.0], [2.0]], [[-1.0], [-1.0]]]], device=dev)
    before = float(quadratic_cost(mean.unsqueeze(1), target)[0, 0])
    m, s, fc, _, _ = device_chain(rt, target, mean, var, [noise], topk=2)
    rt.sync()
    assert float(fc[0]) <= before
    assert m.shape == mean.shape and s.shape == var.shape
    # costs 2, 0, 2, 8: elites are rows 1 and 0 (tie with row 2 goes to the lower index)
    np.testing.assert_allclose(m.cpu().numpy().ravel(), [0.5, 0.5], rtol=0, atol=0)
    np.testing.assert_allclose(float(fc[0]), 1.0, rtol=0, atol=0)

    want_m, want_s, want_fc = io.run_static_icem_chain(
        lambda e, g, c: ((c - target.cpu().numpy()) ** 2).sum(axis=(2, 3)), np.zeros((1, 1, 4), np.float32),
        np.zeros((1, 1, 4), np.float32), mean.cpu().numpy(), var.cpu().numpy(), [noise.cpu().numpy()], topk=2)
    np.testing.assert_allclose(m.cpu().numpy(), want_m, rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(s.cpu().numpy(), want_s, rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(fc.cpu().numpy(), want_fc, rtol=1e-6)


@pytest.mark.parametrize("B,S,k,steps", [(2, 300, 30, 6), (3, 60, 10, 4)])
def test_quadratic_chain_tracks_oracle_chain(rt, B, S, k, steps):
    """A multi-env, multi-iteration quadratic chain (the reference's QuadraticCostModel,
    tests/test_lewm_icem.py:39-46, at horizon 5 x 10 actions) on the device kernels: fed the
    device's costs, the oracle chain selects the same elites every iteration (bit-exact) and
    refits the same distribution; the chain lowers the cost of the mean."""
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(B * 1000 + S)
    T, A = 5, 10
    target = rng.uniform(-0.8, 0.8, (B, 1, T, A)).astype(np.float32)
    mean = np.zeros((B, T, A), np.float32)
    var = np.ones((B, T, A), np.float32)
    noise = [rng.standard_normal((B, S, T, A)).astype(np.float32) for _ in range(steps)]
    tgt = torch.as_tensor(target, device=dev)
    m, s, fc, costs, idx = device_chain(rt, tgt, torch.as_tensor(mean, device=dev),
                                        torch.as_tensor(var, device=dev),
                                        [torch.as_tensor(n, device=dev) for n in noise], topk=k)
    rt.sync()
    fed = iter(costs)
    trace = []
    want_m, want_s, want_fc = io.run_static_icem_chain(
        lambda e, g, c: next(fed), np.zeros((B, 1, 4), np.float32), np.zeros((B, 1, 4), np.float32), mean, var,
        noise, topk=k, trace=trace)
    for it in range(steps):
        np.testing.assert_array_equal(idx[it], trace[it]["topk_inds"])
    np.testing.assert_allclose(m.cpu().numpy(), want_m, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(s.cpu().numpy(), want_s, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(fc.cpu().numpy(), want_fc, rtol=1e-4)
    start = ((mean[:, None] - target) ** 2).sum(axis=(2, 3))[:, 0]
    end = ((m.cpu().numpy()[:, None] - target) ** 2).sum(axis=(2, 3))[:, 0]
    assert (end < start).all()
