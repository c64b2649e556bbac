"""B200PlanningPolicy in front of the reference's own CEMExactSolver, on the CPU.

The unmodified reference package installed in ``baseline/_ref`` (skipped if absent) provides
the JEPA (synthetic width-192 / 6-layer weights) and ``CEMExactSolver`` with its warm start
on (``lewm/solvers/cem_exact.py:198-245``, shift = ``receding_horizon``). The policy drives one
solver through ``get_action``; a twin solver with the same seed is driven by hand the way the
policy's contract says: a solve every ``receding_horizon * action_block`` steps, the previous
plan's unexecuted tail as ``init_action``. Served actions must equal the twin's plans block by
block, bit for bit, and the twin's second solve must report its warm start as used.
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

N_ENVS, RAW, AB, HZ, RH = 2, 2, 5, 5, 2


def _model():
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    from lewm import jepa, module

    from lewm_flash_b200.model import ModelDesc, synthetic_state_dict

    d = ModelDesc()
    pred = module.ARPredictor(num_frames=d.num_frames, depth=d.depth, heads=d.heads, mlp_dim=d.mlp_dim,
                              input_dim=d.dim, hidden_dim=d.dim, dim_head=d.dim_head)
    enc = module.Embedder(input_dim=d.action_dim, smoothed_dim=d.smoothed_dim, emb_dim=d.dim,
                          mlp_scale=d.embed_hidden // d.dim)
    model = jepa.JEPA(encoder=torch.nn.Identity(), predictor=pred, action_encoder=enc, pred_proj=None)
    model.load_state_dict({k: torch.from_numpy(v) for k, v in synthetic_state_dict(d, 0).items()}, strict=True)
    # cached latents: get_cost goes straight to get_cost_from_embeddings (lewm/jepa.py:347-361)
    return model.eval().set_embedding_cache(True).set_compile_cost(True)


class Box:
    def __init__(self, n):
        self.shape = (n, RAW)
        self.low = -np.inf * np.ones(self.shape, np.float32)
        self.high = np.inf * np.ones(self.shape, np.float32)


def _solver(model):
    from lewm.solvers.cem_exact import CEMExactSolver

    return CEMExactSolver(model=model, batch_size=N_ENVS, num_samples=24, n_steps=2, topk=6, device="cpu", seed=11,
                          warm_start=True)


def _info(step):
    g = torch.Generator().manual_seed(100 + step)
    return {"emb": torch.randn(N_ENVS, 1, 192, generator=g), "goal_emb": torch.randn(N_ENVS, 1, 192, generator=g),
            "pixels": torch.zeros(N_ENVS, 1), "goal": torch.zeros(N_ENVS, 1)}


def test_policy_drives_reference_cem_solver_with_warm_start():
    from lewm_flash_b200.policy import B200PlanningPolicy

    torch.manual_seed(0)
    model = _model()
    cfg = SimpleNamespace(horizon=HZ, receding_horizon=RH, action_block=AB)
    policy = B200PlanningPolicy(_solver(model), cfg)
    policy.set_env(SimpleNamespace(num_envs=N_ENVS, action_space=Box(N_ENVS)))
    twin = _solver(model)
    twin.configure(action_space=Box(N_ENVS), n_envs=N_ENVS, config=cfg)

    per_plan = RH * AB
    served, plan_infos = [], []
    with torch.inference_mode():
        for step in range(2 * per_plan):
            info = _info(step)
            if step % per_plan == 0:
                plan_infos.append(info)
            served.append(policy.get_action(info))
    assert policy.solves == 2

    tail, infos = None, []
    with torch.inference_mode():
        for k, info in enumerate(plan_infos):
            out = twin.solve(info, init_action=tail)
            infos.append(twin.last_warm_start_info)
            acts = out["actions"]
            for i in range(per_plan):
                want = acts[:, i // AB, (i % AB) * RAW:(i % AB + 1) * RAW].numpy()
                np.testing.assert_array_equal(served[k * per_plan + i], want.astype(np.float32))
            tail = acts[:, RH:].clone()
    assert infos[0]["used"] is False and infos[1]["used"] is True
    assert policy.solver.last_warm_start_info["used"] is True
