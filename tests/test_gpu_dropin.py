"""The drop-in Python surface on a GPU, against the reference's own classes.

Uses the unmodified reference package installed in ``baseline/_ref`` (skipped if
it is absent). A reference ``JEPA`` is built from the reference's classes with the
synthetic width-192 / 6-layer weights, on the GPU. The reference solvers run with
their model cost routed through the B200 kernels (``install_model_cost``), so both
sides see the same costs and the comparison isolates the solver surface:

* ``B200ICEMSolver.solve`` (two env batches, elite retention, clipping, momentum,
  callbacks, ``return_best_elite``, a warm-start ``init_action``) against
  ``ICEMSolver.solve`` (``lewm/solvers/icem.py:471-602``) on the same noise, drawn
  by the reference solver's own ``_sample_noise`` through ``noise_source``;
* ``B200CEMSolver.solve`` twice with ``warm_start`` against ``CEMExactSolver``
  (``lewm/solvers/cem_exact.py:54-383``): actions, var, costs and the
  ``warm_start`` info of both solves;
* the package-level ``run_static_icem_chain`` against the reference's
  (``lewm/solvers/icem_static_compile.py:61-114``) on a noise list whose sample
  counts follow no iCEM schedule;
* ``install_model_cost`` / ``B200ModelCost`` against the reference's fp32
  ``get_cost_from_embeddings`` and against ``Runtime.model_cost``, following the
  JEPA's ``model_cost_autocast_mode()``: "none" (the JEPA default, so every solver
  test here runs the float32 kernels) within the reference's 1e-5 exactness gate,
  "bf16" within the bf16 bound 1e-2.

Tolerances: the two sides compute candidates with different fp32 operation orders
(one rounding apart), so outputs agree to 1e-4 relative rather than bit for bit.
"""

from __future__ import annotations

import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"
pytestmark = pytest.mark.skipif(not (REF / "lewm" / "jepa.py").is_file(),
                                reason="reference package not installed in baseline/_ref")

T, BLOCK = 5, 5


def _reference():
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    from lewm import jepa, module
    from lewm.solvers import cem_exact, icem, icem_static_compile
    return SimpleNamespace(jepa=jepa, module=module, icem=icem, cem=cem_exact, static=icem_static_compile)


def _jepa(ref, device):
    from lewm_flash_b200.model import ModelDesc, synthetic_state_dict

    desc = ModelDesc()
    pred = ref.module.ARPredictor(num_frames=desc.num_frames, depth=desc.depth, heads=desc.heads,
                                  mlp_dim=desc.mlp_dim, input_dim=desc.dim, hidden_dim=desc.dim,
                                  dim_head=desc.dim_head)
    enc = ref.module.Embedder(input_dim=desc.action_dim, smoothed_dim=desc.smoothed_dim, emb_dim=desc.dim,
                              mlp_scale=desc.embed_hidden // desc.dim)
    model = ref.jepa.JEPA(encoder=torch.nn.Identity(), predictor=pred, action_encoder=enc, pred_proj=None)
    model.load_state_dict({k: torch.from_numpy(v) for k, v in synthetic_state_dict(desc, 0).items()}, strict=True)
    return model.to(device).eval(), desc


class Box:
    """gymnasium.spaces.Box stand-in: the solvers read shape, low and high."""

    def __init__(self, n_envs, lo=-2.5, hi=2.5):
        self.shape = (n_envs, 2)
        self.low = lo * np.ones(self.shape, dtype=np.float32)
        self.high = hi * np.ones(self.shape, dtype=np.float32)


def _info(n_envs, H, device, seed):
    g = torch.Generator().manual_seed(seed)
    emb = torch.randn(n_envs, H, 192, generator=g).to(device)
    goal = torch.randn(n_envs, 1, 192, generator=g).to(device)
    # pixels / goal only carry H for JEPA._ensure_cost_embeddings; the cached embeddings skip the encoder.
    return {"emb": emb, "goal_emb": goal, "pixels": torch.zeros(n_envs, H, device=device),
            "goal": torch.zeros(n_envs, H, device=device)}


def _close(a, b, rtol=1e-4, atol=1e-4):
    a = torch.as_tensor(a).float().cpu()
    b = torch.as_tensor(b).float().cpu()
    scale = float(b.abs().max()) + 1.0
    torch.testing.assert_close(a, b, rtol=rtol, atol=atol * scale)


def _histories_close(h_dev, h_ref):
    """ICEMStepSummaryCallback rows. Cost statistics are compared on the scale of the costs
    themselves (~300): the top-k cost std is a difference of nearly equal costs, so a 1e-6
    relative change of the costs moves it by ~1e-3 of its own size."""
    assert len(h_dev) == len(h_ref)
    for rd, rr in zip(h_dev, h_ref):
        assert rd.keys() == rr.keys()
        cost_scale = abs(rr["best_cost_mean"]) + 1.0
        for key in rr:
            if rr[key] is None or isinstance(rr[key], int):
                assert rd[key] == rr[key], key
            elif "cost" in key:
                assert abs(rd[key] - rr[key]) <= 1e-5 * cost_scale, (key, rd[key], rr[key])
            else:
                assert abs(rd[key] - rr[key]) <= 1e-4 * (abs(rr[key]) + 1.0), (key, rd[key], rr[key])


@pytest.fixture(scope="module")
def env():
    ref = _reference()
    dev = torch.device("cuda", 0)
    model, desc = _jepa(ref, dev)
    from lewm_flash_b200.solver import install_model_cost

    install_model_cost(model, dev)
    model.set_embedding_cache(True).set_compile_cost(True)
    return SimpleNamespace(ref=ref, dev=dev, model=model, desc=desc)


ICEM_KW = dict(batch_size=2, num_samples=48, n_steps=4, topk=8, seed=5, elite_retention=2, colored_noise="brown",
               colored_noise_time="raw", momentum_alpha=0.1, sample_decay=1.25, sample_count_bucket_size=8,
               clip_actions=True)


@pytest.mark.gpu
@pytest.mark.parametrize("best_elite", [False, True])
def test_icem_solve_matches_reference_solver(env, best_elite):
    from lewm_flash_b200.solver import B200ICEMSolver

    n_envs, cfg = 3, SimpleNamespace(horizon=T, action_block=BLOCK)
    kw = dict(ICEM_KW, return_best_elite=best_elite)
    ref = env.ref.icem.ICEMSolver(model=env.model, device=env.dev, callbacks=[env.ref.icem.ICEMStepSummaryCallback()],
                                  **kw)
    ref.configure(action_space=Box(n_envs), n_envs=n_envs, config=cfg)
    noise_twin = env.ref.icem.ICEMSolver(model=env.model, device=env.dev, **kw)  # same seed: same noise stream
    noise_twin.configure(action_space=Box(n_envs), n_envs=n_envs, config=cfg)
    b200 = B200ICEMSolver(env.model, device=env.dev, callbacks=[env.ref.icem.ICEMStepSummaryCallback()], **kw)
    b200.configure(action_space=Box(n_envs), n_envs=n_envs, config=cfg)
    b200.noise_source = noise_twin._sample_noise
    assert b200.sample_counts() == ref.sample_counts()
    assert b200.model_cost_evals_per_solve() == ref.model_cost_evals_per_solve()
    assert (b200.n_envs, b200.action_dim, b200.horizon, b200.action_block) == (
        ref.n_envs, ref.action_dim, ref.horizon, ref.action_block)
    # Warm-start prefix: the first two steps of the previous plan, padded with zeros (prepare_init_action).
    init = torch.randn(n_envs, 2, 10, generator=torch.Generator().manual_seed(3)).to(env.dev)
    out_ref = ref.solve(_info(n_envs, 1, env.dev, 11), init_action=init)
    out_dev = b200.solve(_info(n_envs, 1, env.dev, 11), init_action=init)
    assert set(out_dev) == set(out_ref) == {"costs", "mean", "var", "actions", "callbacks"}
    assert out_dev["actions"].device.type == "cpu" and out_dev["actions"].shape == out_ref["actions"].shape
    _close(out_dev["actions"], out_ref["actions"])
    _close(out_dev["mean"][0], out_ref["mean"][0])
    _close(out_dev["var"][0], out_ref["var"][0])
    np.testing.assert_allclose(out_dev["costs"], out_ref["costs"], rtol=1e-5)
    _histories_close(out_dev["callbacks"]["icem_step_summary"], out_ref["callbacks"]["icem_step_summary"])


@pytest.mark.gpu
def test_cem_solve_twice_with_warm_start_matches_reference(env):
    from lewm_flash_b200.solver import B200CEMSolver

    n_envs = 2
    cfg = SimpleNamespace(horizon=T, action_block=BLOCK, receding_horizon=2)
    kw = dict(batch_size=n_envs, num_samples=40, n_steps=3, topk=6, seed=9, warm_start=True)
    ref = env.ref.cem.CEMExactSolver(model=env.model, device=env.dev, **kw)
    ref.configure(action_space=Box(n_envs), n_envs=n_envs, config=cfg)
    twin = env.ref.cem.CEMExactSolver(model=env.model, device=env.dev, **kw)
    b200 = B200CEMSolver(env.model, device=env.dev, **kw)
    b200.configure(action_space=Box(n_envs), n_envs=n_envs, config=cfg)
    # CEMExactSolver draws white noise with torch.randn from its own generator (cem_exact.py:312-319).
    b200.noise_source = lambda b, n: torch.randn(b, n, T, 10, generator=twin.torch_gen, device=env.dev)
    assert b200.last_warm_start_info == ref.last_warm_start_info
    for solve in range(2):
        out_ref = ref.solve(_info(n_envs, 1, env.dev, 20 + solve))
        out_dev = b200.solve(_info(n_envs, 1, env.dev, 20 + solve))
        assert out_dev["warm_start"] == out_ref["warm_start"], solve
        assert out_dev["warm_start"]["used"] == (solve == 1)
        _close(out_dev["actions"], out_ref["actions"])
        _close(out_dev["var"][0], out_ref["var"][0])
        np.testing.assert_allclose(out_dev["costs"], out_ref["costs"], rtol=1e-5)
    b200.reset_warm_start_state("manual")
    ref.reset_warm_start_state("manual")
    assert b200.last_warm_start_info == ref.last_warm_start_info


@pytest.mark.gpu
def test_run_static_icem_chain_accepts_any_noise_list(env):
    from lewm_flash_b200.solver import run_static_icem_chain

    n_envs = 2
    g = torch.Generator(device=env.dev).manual_seed(4)
    counts = [40, 33, 17, 25]  # no iCEM schedule produces these
    noise = [torch.randn(n_envs, c, T, 10, generator=g, device=env.dev) for c in counts]
    info = _info(n_envs, 1, env.dev, 31)
    mean = torch.zeros(n_envs, T, 10, device=env.dev)
    var = torch.ones(n_envs, T, 10, device=env.dev)
    lo, hi = -torch.ones(10, device=env.dev) * 1.5, torch.ones(10, device=env.dev) * 1.5
    kw = dict(topk=7, elite_retention=3, momentum_alpha=0.25, return_best_elite=False, action_low=lo, action_high=hi)
    want = env.ref.static.run_static_icem_chain(env.model.get_cost_from_embeddings, info["emb"], info["goal_emb"],
                                                mean, var, noise, **kw)
    got = run_static_icem_chain(env.model, info["emb"], info["goal_emb"], mean, var, noise, **kw)
    for a, b in zip(got, want):
        _close(a, b)


@pytest.mark.gpu
def test_install_model_cost_routes_reference_cost(env):
    from lewm_flash_b200.solver import _runtime

    g = torch.Generator().manual_seed(8)
    emb = torch.randn(2, 1, 192, generator=g)
    goal = torch.randn(2, 1, 192, generator=g)
    cand = torch.randn(2, 24, T, 10, generator=g)
    got = env.model.get_cost_from_embeddings(emb.to(env.dev), goal.to(env.dev), cand.to(env.dev))
    assert got.dtype == torch.float32 and tuple(got.shape) == (2, 24) and got.is_cuda
    direct = _runtime(env.model, env.dev).model_cost(emb, goal, cand)
    assert torch.equal(got, direct)
    # The reference's own fp32 model cost (a CPU copy of the same JEPA, its method untouched).
    cpu_model, _ = _jepa(env.ref, torch.device("cpu"))
    with torch.inference_mode():
        want = cpu_model.get_cost_from_embeddings(emb, goal, cand)
    rel = ((got.cpu() - want).abs() / want.abs()).max().item()
    assert rel <= 1e-2, rel
    # JEPA.get_cost (compile_cost path, lewm/jepa.py:357-359) reaches the same kernels.
    info = {"emb": emb.to(env.dev)[:, None].expand(2, 24, 1, 192), "goal_emb": goal.to(env.dev)[:, None].expand(2, 24, 1, 192),
            "pixels": torch.zeros(2, 24, 1, device=env.dev), "goal": torch.zeros(2, 24, 1, device=env.dev)}
    via_get_cost = env.model.get_cost(info, cand.to(env.dev))
    assert torch.equal(via_get_cost, got)


@pytest.mark.gpu
def test_model_cost_follows_the_models_autocast_mode(env):
    from lewm_flash_b200.solver import _runtime

    g = torch.Generator().manual_seed(12)
    emb = torch.randn(2, 3, 192, generator=g)
    goal = torch.randn(2, 1, 192, generator=g)
    cand = torch.randn(2, 64, T, 10, generator=g)
    cpu_model, _ = _jepa(env.ref, torch.device("cpu"))
    with torch.inference_mode():
        want = cpu_model.get_cost_from_embeddings(emb, goal, cand)
    args = (emb.to(env.dev), goal.to(env.dev), cand.to(env.dev))
    assert env.model.model_cost_autocast_mode() == "none"
    f32 = env.model.get_cost_from_embeddings(*args)
    assert _runtime(env.model, env.dev).model_cost_autocast_mode() == "none"
    assert torch.allclose(f32.cpu(), want, rtol=1e-5, atol=1e-5), (f32.cpu() - want).abs().max()
    env.model.set_model_cost_autocast("bf16")
    try:
        bf16 = env.model.get_cost_from_embeddings(*args)
        assert _runtime(env.model, env.dev).model_cost_autocast_mode() == "bf16"
        rel = ((bf16.cpu() - want).abs() / want.abs()).max().item()
        assert rel <= 1e-2 and not torch.allclose(bf16.cpu(), want, rtol=1e-5, atol=1e-5), rel
    finally:
        env.model.set_model_cost_autocast("none")
    assert torch.equal(env.model.get_cost_from_embeddings(*args), f32)


@pytest.mark.gpu
def test_static_solver_matches_reference_static_solver(env):
    """B200ICEMStaticSolver against ICEMStaticCompileSolver (eager static chain,
    lewm/solvers/icem_static_compile.py:317-373) on the same noise, with a warmed graph."""
    from lewm_flash_b200.solver import B200ICEMStaticSolver

    n_envs, cfg = 3, SimpleNamespace(horizon=T, action_block=BLOCK)
    kw = dict(ICEM_KW, return_best_elite=False)
    ref = env.ref.static.ICEMStaticCompileSolver(model=env.model, device=env.dev, **kw)
    twin = env.ref.static.ICEMStaticCompileSolver(model=env.model, device=env.dev, **kw)
    b200 = B200ICEMStaticSolver(env.model, device=env.dev, static_chain_compile=True, **kw)
    for s in (ref, twin, b200):
        s.configure(action_space=Box(n_envs), n_envs=n_envs, config=cfg)
    b200.noise_source = twin._sample_noise
    warm = b200.warmup_static_chain_compile(embed_dim=192, history=1, batch_size=n_envs)
    assert warm.enabled and warm.sample_counts == ref.sample_counts()
    out_ref = ref.solve(_info(n_envs, 1, env.dev, 17))
    out_dev = b200.solve(_info(n_envs, 1, env.dev, 17))
    assert set(out_dev) == set(out_ref)
    _close(out_dev["actions"], out_ref["actions"])
    _close(out_dev["var"][0], out_ref["var"][0])
    np.testing.assert_allclose(out_dev["costs"], out_ref["costs"], rtol=1e-5)
    sc_dev, sc_ref = dict(out_dev["static_chain"]), dict(out_ref["static_chain"])
    assert sc_dev.pop("static_chain_warmed") and not sc_ref.pop("static_chain_warmed")
    assert sc_dev.pop("static_chain_compile") and not sc_ref.pop("static_chain_compile")
    assert sc_dev == sc_ref
