"""The device gradient of the model cost with respect to the action candidates
(``lewm_model_cost_grad``): what CEM-GD's refinement steps on (reference
``lewm/solvers/cem_gd.py:459-606``, torch autograd of ``JEPA.get_cost_from_embeddings``,
``lewm/jepa.py:302-317``).

* against torch autograd of the reference model (``tests/golden/cost_grad_full.npz``, width
  192 / 6 layers, histories 1 to 3, a horizon of 6) and the float64 oracle
  (``oracle/cost_grad_oracle.py``): within 1e-4 of the largest gradient entry;
* against central differences of the device's own float32 model cost;
* weighted costs scale each candidate's gradient; a candidate's gradient does not depend on
  the batch around it (bit for bit);
* through ``install_model_cost``: the reference's own ``CEMGDSolver`` refines on these
  kernels and agrees with the same solver on the reference model's torch autograd.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from lewm_flash_b200.model import synthetic_state_dict
from lewm_flash_b200.runtime import Runtime
from oracle import cost_grad_oracle as cg
from tests.conftest import GOLDEN
from tests.golden.make_cost_grad_golden import FULL_CASES, FULL_DESC, FULL_WEIGHT_SEED, case_inputs

pytestmark = pytest.mark.gpu
FIX = np.load(GOLDEN / "cost_grad_full.npz")
GRAD_TOL = 1e-4  # of the largest gradient entry: float32 forward + reverse against autograd / float64


def _t(x):
    return torch.as_tensor(np.ascontiguousarray(x), dtype=torch.float32, device="cuda:0")


@pytest.fixture(scope="module")
def rt():
    r = Runtime(FULL_DESC, synthetic_state_dict(FULL_DESC, FULL_WEIGHT_SEED), "cuda:0")
    yield r
    r.close()


@pytest.mark.parametrize("name", sorted(FULL_CASES))
def test_gradient_matches_reference_autograd_and_oracle(rt, name):
    emb, goal, cand = case_inputs(*FULL_CASES[name], desc=FULL_DESC)
    H = emb.shape[1]
    cost, grad = rt.model_cost_grad(_t(emb), _t(goal), _t(cand))
    rt.sync()
    cost, grad = cost.cpu().numpy(), grad.cpu().numpy()
    np.testing.assert_allclose(cost, FIX[f"{name}__cost"], rtol=1e-5, atol=1e-5)
    want = FIX[f"{name}__grad"]
    err = np.abs(grad - want).max() / np.abs(want).max()
    _, g64 = cg.cost_and_grad(emb, goal, cand, synthetic_state_dict(FULL_DESC, FULL_WEIGHT_SEED), FULL_DESC)
    err64 = np.abs(grad - g64).max() / np.abs(g64).max()
    print(f"{name} (H={H}): gradient error {err:.2e} against torch autograd, {err64:.2e} against float64")
    assert err <= GRAD_TOL and err64 <= GRAD_TOL


def test_gradient_matches_central_differences(rt):
    emb, goal, cand = case_inputs(*FULL_CASES["full_h3"], desc=FULL_DESC)
    e, g, c = _t(emb), _t(goal), _t(cand)
    _, grad = rt.model_cost_grad(e, g, c)
    rng = np.random.default_rng(3)
    d = _t(rng.standard_normal(cand.shape))
    eps = 5e-2
    hi = rt.model_cost_grad(e, g, c + eps * d)[0]
    lo = rt.model_cost_grad(e, g, c - eps * d)[0]
    rt.sync()
    fd = ((hi - lo) / (2 * eps)).cpu().numpy()
    dd = (grad * d).sum(dim=(2, 3)).cpu().numpy()
    # The float32 costs (~370) resolve a difference to one ulp (3e-5): the quotient carries
    # about 8 ulps / (2 eps) of rounding; the O(eps^2) curvature term stays under 1 %.
    resolution = 8 * float(np.spacing(np.float32(hi.abs().max().item()))) / (2 * eps)
    np.testing.assert_allclose(dd, fd, rtol=1e-2, atol=resolution)


def test_weights_scale_and_batch_independence(rt):
    emb, goal, cand = case_inputs(*FULL_CASES["full_h1"], desc=FULL_DESC)
    e, g, c = _t(emb), _t(goal), _t(cand)
    cost1, g1 = rt.model_cost_grad(e, g, c)
    w = _t(np.array([[0.5, -2.0, 0.0, 3.0], [1.0, 0.25, -1.0, 2.0]], np.float32))
    cost2, g2 = rt.model_cost_grad(e, g, c, cost_weights=w)
    # candidate 1 of env 0 alone, and inside a batch of 300 candidates
    c_one = c[:1, 1:2]
    big = _t(np.random.default_rng(4).standard_normal((1, 300, 5, FULL_DESC.action_dim)))
    big[:, 137] = c_one[:, 0]
    _, g_one = rt.model_cost_grad(e[:1], g[:1], c_one)
    _, g_big = rt.model_cost_grad(e[:1], g[:1], big)
    rt.sync()
    assert torch.equal(cost1, cost2)
    want = g1 * w[..., None, None]
    # Power-of-two weights (and 0) scale every rounding step exactly: the same bits. Weight 3
    # rounds differently along the reverse pass: within 1e-5 of the largest entry.
    exact = torch.tensor([[True, True, True, False], [True, True, True, True]], device=w.device)
    assert torch.equal(g2[exact], want[exact])
    torch.testing.assert_close(g2, want, rtol=0, atol=1e-5 * float(want.abs().max()))
    assert torch.equal(g_one[0, 0], g_big[0, 137])


def test_pred_proj_head_is_rejected():
    from lewm_flash_b200._lib import LewmError
    from lewm_flash_b200.model import ModelDesc

    desc = ModelDesc(pred_proj_hidden=256, pred_proj_norm="layernorm")
    r = Runtime(desc, synthetic_state_dict(desc, 1), "cuda:0")
    x = torch.zeros(1, 1, 192, device="cuda:0")
    with pytest.raises(LewmError, match="UNSUPPORTED_SHAPE"):
        r.model_cost_grad(x, x, torch.zeros(1, 2, 5, 10, device="cuda:0"))
    r.close()


REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


@pytest.mark.skipif(not (REF / "lewm" / "solvers" / "cem_gd.py").is_file(),
                    reason="reference package not installed in baseline/_ref")
@pytest.mark.parametrize("backtracking", [True, False])
def test_reference_cem_gd_solver_refines_on_device_gradient(backtracking):
    """The reference's unmodified CEMGDSolver (CEM seeds, Adam + backtracking refinement)
    with the model cost routed through the B200 kernels, against the same solver on the
    reference model's own torch autograd (float32, the same GPU)."""
    from types import SimpleNamespace

    from tests.test_gpu_dropin import Box, _jepa, _reference

    from lewm_flash_b200.solver import install_model_cost

    ref = _reference()
    from lewm.solvers.cem_gd import CEMGDSolver

    class CLSFeatures(torch.nn.Module):
        """Encoder stand-in: the "pixels" are the CLS features themselves, so JEPA.encode
        (lewm/jepa.py:88-104) returns them as the embeddings and the solver's seed search
        caches them (cem_gd.py:340-347) as it does with the ViT."""

        def forward(self, pixels, interpolate_pos_encoding=True):
            return SimpleNamespace(last_hidden_state=pixels[:, None, :])

    dev = torch.device("cuda", 0)
    kw = dict(batch_size=2, num_samples=64, n_steps=3, topk=8, seed=13, gd_refine_topk=4, gd_steps=3, gd_lr=0.05,
              gd_backtracking=backtracking)
    cfg = SimpleNamespace(horizon=5, action_block=5)
    g = torch.Generator().manual_seed(41)
    obs, goal = torch.randn(2, 1, 192, generator=g), torch.randn(2, 1, 192, generator=g)
    outs = []
    for routed in (True, False):
        model, _ = _jepa(ref, dev)
        model.encoder = CLSFeatures()
        model.set_embedding_cache(True).set_compile_cost(True)
        if routed:
            install_model_cost(model, dev)
        solver = CEMGDSolver(model=model, device=dev, **kw)
        solver.configure(action_space=Box(2), n_envs=2, config=cfg)
        outs.append(solver.solve({"pixels": obs.to(dev), "goal": goal.to(dev)}))
    got, want = outs
    np.testing.assert_allclose(np.asarray(got["costs"]), np.asarray(want["costs"]), rtol=1e-5)
    # Adam's first steps move every coordinate by about lr whatever the gradient's size, so a
    # coordinate whose gradient sits at float32 rounding level (~1e-7 of the largest) may step
    # differently on the two gradients; every other coordinate agrees to 1e-4.
    diff = (got["actions"] - want["actions"]).abs()
    close = diff <= 1e-4 * (1.0 + want["actions"].abs())
    assert close.float().mean().item() >= 0.95, diff.max().item()
    assert diff.max().item() <= 2 * kw["gd_lr"] * kw["gd_steps"]
    gs, ws = got["gd_summary"], want["gd_summary"]
    for key in ("gd_accept_count", "gd_candidate_count", "gd_model_cost_evals", "gd_nan_or_inf_count"):
        assert gs[key] == ws[key], key
    for key in ("gd_cost_delta_mean", "gd_grad_norm_mean", "gd_grad_norm_max"):
        assert abs(gs[key] - ws[key]) <= 1e-4 * (abs(ws[key]) + 1.0), (key, gs[key], ws[key])
    print(f"backtracking={backtracking}: refined costs {np.round(np.asarray(got['costs']), 3).tolist()}, "
          f"accepted {gs['gd_accept_count']} of {gs['gd_candidate_count']}, cost delta {gs['gd_cost_delta_mean']:.4f}, "
          f"actions: {int((~close).sum())} of {close.numel()} coordinates beyond 1e-4 (max {diff.max().item():.1e})")


@pytest.mark.skipif(not (REF / "lewm" / "solvers" / "cem_gd.py").is_file(),
                    reason="reference package not installed in baseline/_ref")
@pytest.mark.parametrize("seed_solver,source", [("cem", "best_elite"), ("icem", "best_elite"), ("cem", "mean")])
def test_b200_cem_gd_solver_matches_reference_solver(seed_solver, source):
    """B200CEMGDSolver (one device seed plan, device-gradient refinement) against the
    reference's CEMGDSolver on the same model cost and the same seed-search noise (its twin's
    _sample_noise): 3 envs in env batches of 2."""
    from types import SimpleNamespace

    from tests.test_gpu_dropin import Box, _jepa, _reference

    from lewm_flash_b200.solver import B200CEMGDSolver, install_model_cost

    ref = _reference()
    from lewm.solvers.cem_gd import CEMGDSolver

    class CLSFeatures(torch.nn.Module):
        def forward(self, pixels, interpolate_pos_encoding=True):
            return SimpleNamespace(last_hidden_state=pixels[:, None, :])

    dev = torch.device("cuda", 0)
    model, _ = _jepa(ref, dev)
    model.encoder = CLSFeatures()
    model.set_embedding_cache(True).set_compile_cost(True)
    install_model_cost(model, dev)
    kw = dict(batch_size=2, num_samples=48, n_steps=4, topk=8, seed=17, gd_seed_solver=seed_solver,
              gd_seed_source=source, gd_refine_topk=3, gd_steps=3, gd_lr=0.05, colored_noise="brown",
              sample_decay=1.25, sample_count_bucket_size=8, elite_retention=2, momentum_alpha=0.1, clip_actions=True)
    cfg = SimpleNamespace(horizon=5, action_block=5)
    g = torch.Generator().manual_seed(43)
    info = {"pixels": torch.randn(3, 1, 192, generator=g).to(dev), "goal": torch.randn(3, 1, 192, generator=g).to(dev)}
    ref_solver = CEMGDSolver(model=model, device=dev, **kw)
    twin = CEMGDSolver(model=model, device=dev, **kw)
    b200 = B200CEMGDSolver(model, device=dev, **kw)
    for s in (ref_solver, twin, b200):
        s.configure(action_space=Box(3, lo=-1.5, hi=1.5), n_envs=3, config=cfg)
    b200.noise_source = twin._sample_noise
    want = ref_solver.solve(dict(info))
    got = b200.solve(dict(info))
    assert set(got) == set(want)
    np.testing.assert_allclose(np.asarray(got["costs"]), np.asarray(want["costs"]), rtol=1e-5)
    torch.testing.assert_close(got["var"][0], want["var"][0], rtol=1e-4, atol=1e-5)
    diff = (got["actions"] - want["actions"]).abs()
    close = diff <= 1e-4 * (1.0 + want["actions"].abs())
    assert close.float().mean().item() >= 0.95 and diff.max().item() <= 2 * kw["gd_lr"] * kw["gd_steps"]
    gs, ws = got["gd_summary"], want["gd_summary"]
    assert set(gs) == set(ws)
    for key in ("gd_accept_count", "gd_candidate_count", "gd_model_cost_evals", "gd_nan_or_inf_count",
                "gd_seed_model_cost_evals", "gd_seed_solver", "gd_seed_source", "gd_refine_topk", "gd_steps"):
        assert gs[key] == ws[key], key
    for key in ("gd_cost_delta_mean", "gd_grad_norm_mean", "gd_grad_norm_max", "gd_accept_rate"):
        assert abs(gs[key] - ws[key]) <= 1e-4 * (abs(ws[key]) + 1.0), (key, gs[key], ws[key])
    print(f"{seed_solver}/{source}: costs {np.round(np.asarray(got['costs']), 3).tolist()}, accepted "
          f"{gs['gd_accept_count']} of {gs['gd_candidate_count']}, {int((~close).sum())} of {close.numel()} action "
          f"coordinates beyond 1e-4")


@pytest.mark.parametrize("H,T,B,S", [(3, 3, 2, 5), (1, 1, 1, 4), (2, 7, 1, 3)])
def test_gradient_edge_shapes_match_oracle(rt, H, T, B, S):
    """A single predictor call (H = T, the window already full), a one-step horizon, and a
    horizon of 7 (a sliding window for five calls) against the float64 oracle."""
    rng = np.random.default_rng(100 + 10 * H + T)
    emb = rng.standard_normal((B, H, FULL_DESC.dim)).astype(np.float32)
    goal = rng.standard_normal((B, 1, FULL_DESC.dim)).astype(np.float32)
    cand = rng.standard_normal((B, S, T, FULL_DESC.action_dim)).astype(np.float32)
    cost, grad = rt.model_cost_grad(_t(emb), _t(goal), _t(cand))
    rt.sync()
    c64, g64 = cg.cost_and_grad(emb, goal, cand, synthetic_state_dict(FULL_DESC, FULL_WEIGHT_SEED), FULL_DESC)
    np.testing.assert_allclose(cost.cpu().numpy(), c64, rtol=1e-5, atol=1e-5)
    err = np.abs(grad.cpu().numpy() - g64).max() / max(np.abs(g64).max(), 1e-30)
    assert err <= GRAD_TOL, err
