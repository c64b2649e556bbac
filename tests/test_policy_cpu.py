"""B200PlanningPolicy host logic on the CPU: action buffer, replanning cadence, warm-start tail,
scalers and transforms, against a recording stand-in solver.

The policy's semantics come from the reference's side of the stable-worldmodel contract
(``plan_config`` horizon / receding_horizon / action_block, ``prepare_init_action``'s warm-start
padding, ``lewm/eval.py:60-97``); the package itself is not installed, so these tests pin the
bookkeeping directly.
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from lewm_flash_b200.policy import B200PlanningPolicy

RAW, AB, H = 2, 3, 5


class RecordingSolver:
    """Returns (n_envs, horizon, RAW * AB) actions that encode (solve, env, block, column)."""

    def __init__(self, n_envs=4):
        self.n_envs = n_envs
        self.calls = []
        self.configured = None
        self.resets = []

    def configure(self, *, action_space, n_envs, config):
        self.configured = (action_space, n_envs, config)

    def reset_warm_start_state(self, reason="manual"):
        self.resets.append(reason)

    def solve(self, info_dict, init_action=None):
        self.calls.append((info_dict, None if init_action is None else init_action.clone()))
        n = len(next(iter(info_dict.values())))
        return {"actions": _actions(len(self.calls), n), "costs": [0.0] * n}


def _actions(k, n=4):
    """The actions of solve number k (1-based)."""
    return torch.arange(n * H * RAW * AB, dtype=torch.float32).reshape(n, H, RAW * AB) + 1000.0 * k


def _info(n=4, seed=0):
    rng = np.random.default_rng(seed)
    return {"state": torch.as_tensor(rng.standard_normal((n, 1, 3)), dtype=torch.float32),
            "pixels": torch.zeros(n, 1, 3, 8, 8), "goal": torch.zeros(n, 1, 3, 8, 8)}


def test_buffer_cadence_and_block_order():
    solver = RecordingSolver()
    pol = B200PlanningPolicy(solver, SimpleNamespace(horizon=H, receding_horizon=2, action_block=AB))
    steps_per_plan = 2 * AB
    for step in range(3 * steps_per_plan):
        a = pol.get_action(_info())
        assert len(solver.calls) == step // steps_per_plan + 1
        i = step % steps_per_plan
        want = _actions(step // steps_per_plan + 1)[:, i // AB, (i % AB) * RAW:(i % AB + 1) * RAW].numpy()
        np.testing.assert_array_equal(a, want)
        assert a.shape == (4, RAW) and a.dtype == np.float32
        assert pol.buffered_steps == steps_per_plan - i - 1


def test_warm_start_tail_is_next_init_action():
    solver = RecordingSolver()
    pol = B200PlanningPolicy(solver, {"horizon": H, "receding_horizon": 2, "action_block": AB})
    for _ in range(2 * AB + 1):
        pol.get_action(_info())
    assert solver.calls[0][1] is None
    torch.testing.assert_close(solver.calls[1][1], _actions(1)[:, 2:], rtol=0, atol=0)


def test_full_receding_horizon_has_no_tail():
    solver = RecordingSolver()
    pol = B200PlanningPolicy(solver, SimpleNamespace(horizon=H, receding_horizon=H, action_block=AB))
    for _ in range(H * AB + 1):
        pol.get_action(_info())
    assert len(solver.calls) == 2 and solver.calls[1][1] is None


def test_receding_horizon_defaults_to_horizon():
    pol = B200PlanningPolicy(RecordingSolver(), SimpleNamespace(horizon=4, action_block=2))
    assert pol.receding_horizon == 4


@pytest.mark.parametrize("cfg", [dict(horizon=5, receding_horizon=0, action_block=5),
                                 dict(horizon=5, receding_horizon=6, action_block=5),
                                 dict(horizon=0, receding_horizon=1, action_block=5),
                                 dict(horizon=5, receding_horizon=5, action_block=0)])
def test_invalid_plan_config(cfg):
    with pytest.raises(ValueError):
        B200PlanningPolicy(RecordingSolver(), cfg)


def test_solver_shape_mismatch_raises():
    solver = RecordingSolver()
    pol = B200PlanningPolicy(solver, SimpleNamespace(horizon=H + 1, receding_horizon=2, action_block=AB))
    with pytest.raises(ValueError, match="do not match"):
        pol.get_action(_info())


def test_scalers_normalise_observations_and_invert_actions():
    sk = pytest.importorskip("sklearn.preprocessing")
    rng = np.random.default_rng(3)
    state_scaler = sk.StandardScaler().fit(rng.normal(2.0, 3.0, (200, 3)))
    action_scaler = sk.StandardScaler().fit(rng.normal(-1.0, 0.5, (200, RAW)))
    solver = RecordingSolver()
    pol = B200PlanningPolicy(solver, SimpleNamespace(horizon=H, receding_horizon=1, action_block=AB),
                             process={"state": state_scaler, "action": action_scaler})
    info = _info()
    a = pol.get_action(info)
    seen = solver.calls[0][0]["state"].numpy()
    want_state = state_scaler.transform(info["state"].numpy().reshape(-1, 3)).reshape(seen.shape)
    np.testing.assert_allclose(seen, want_state, rtol=1e-6)
    raw = _actions(1)[:, 0, :RAW].numpy()
    np.testing.assert_allclose(a, action_scaler.inverse_transform(raw), rtol=1e-6)
    # the caller's dict is left as it was
    assert info["state"].dtype == torch.float32 and not np.allclose(info["state"].numpy(), seen)


def test_image_transforms_without_encoder():
    solver = RecordingSolver()
    tf = {"pixels": lambda x: x + 1.0, "goal": lambda x: x - 1.0}
    pol = B200PlanningPolicy(solver, SimpleNamespace(horizon=H, receding_horizon=1, action_block=AB), transform=tf)
    pol.get_action(_info())
    seen = solver.calls[0][0]
    assert float(seen["pixels"].mean()) == 1.0 and float(seen["goal"].mean()) == -1.0
    assert "emb" not in seen


def test_set_env_configures_and_reset_replans():
    solver = RecordingSolver()
    cfg = SimpleNamespace(horizon=H, receding_horizon=2, action_block=AB)
    pol = B200PlanningPolicy(solver, cfg)
    env = SimpleNamespace(num_envs=4, action_space=SimpleNamespace(shape=(4, RAW)))
    pol.set_env(env)
    assert solver.configured == (env.action_space, 4, cfg)
    pol.get_action(_info())
    pol.get_action(_info())
    assert len(solver.calls) == 1 and pol.buffered_steps == 2 * AB - 2
    pol.reset()
    assert pol.buffered_steps == 0
    pol.get_action(_info())
    assert len(solver.calls) == 2 and solver.calls[1][1] is None  # the warm start was dropped
    assert solver.resets[-1] == "policy_reset"
