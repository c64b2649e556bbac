"""Receding-horizon planning policy over the B200 solvers.

The reference evaluates its solvers through the policy of stable-worldmodel 0.1.1, a package it
does not vendor: ``lewm/eval.py:93-97`` builds ``WorldModelPolicy(solver=..., config=
PlanConfig(**plan_config), process=..., transform=...)`` and hands it to the world, whose steps
call ``get_action(info_dict)`` (``tools/benchmarks/lewm_plan_benchmark.py:923-935`` wraps that
call to time it). ``B200PlanningPolicy`` takes the same constructor arguments and plays that
role in front of the B200 solvers. What it does follows from the reference's own side of the
contract:

* ``plan_config`` (``lewm/config/eval/pusht.yaml:21-25``): ``horizon`` action blocks per plan,
  ``receding_horizon`` of them executed before the next plan, ``action_block`` raw env actions
  per block (the frameskip). A solver's ``actions`` are ``(n_envs, horizon, raw_dim *
  action_block)``, each block the ``action_block`` raw actions one after another (the layout
  the colored-noise sampler flattens, ``lewm/solvers/icem.py:195-232``).
* warm start: the plan's unexecuted tail (blocks ``receding_horizon ..``) is passed to the next
  solve as ``init_action``, which ``prepare_init_action`` zero-pads to the horizon
  ("stable-worldmodel CEM warm-start padding semantics", ``lewm/solvers/cem_exact.py:13-51``).
  ``CEMExactSolver``'s own warm start shifts by the same ``receding_horizon``
  (``lewm/solvers/cem_exact.py:198-245``).
* ``process``: fitted scalers per dataset column (``lewm/eval.py:70-81``); observation columns
  are normalised before a solve and served actions are mapped back with
  ``process["action"].inverse_transform`` (the solvers plan in the scaler's units).
* ``transform``: the image transforms of ``pixels`` and ``goal`` (``lewm/eval.py:60-64``,
  ``img_transform`` at ``lewm/eval.py:17-26``). Given a ``B200Encoder``, raw uint8 frames skip
  them: ``encode_frames`` applies the same transform inside the encoder's first kernel and the
  embeddings go to the solver as ``emb`` / ``goal_emb`` (the cached-embedding keys of
  ``JEPA._ensure_cost_embeddings``, ``lewm/jepa.py:319-345``).

Calls that only serve the buffer touch no device work: observations are read only when a plan
is due.
"""

from __future__ import annotations

from types import SimpleNamespace
from typing import Any, Optional

import numpy as np
import torch

from .encoder import IMAGENET_MEAN, IMAGENET_STD

_IMAGE_KEYS = ("pixels", "goal")


def _cfg(config: Any, key: str, default: Any = None) -> Any:
    if isinstance(config, dict):
        return config.get(key, default)
    return getattr(config, key, default)


class B200PlanningPolicy:
    """Action buffer + receding-horizon replanning in front of a solver (see the module doc)."""

    def __init__(self, solver: Any, config: Any, process: Optional[dict] = None, transform: Optional[dict] = None,
                 encoder: Any = None, image_mean=IMAGENET_MEAN, image_std=IMAGENET_STD) -> None:
        self.solver = solver
        # a plain dict of plan_config keys is accepted; the solvers read attributes (PlanConfig)
        self.cfg = SimpleNamespace(**config) if isinstance(config, dict) else config
        self.process = dict(process or {})
        self.transform = dict(transform or {})
        self.encoder = encoder
        self.image_mean = tuple(float(v) for v in image_mean)
        self.image_std = tuple(float(v) for v in image_std)
        self.horizon = int(_cfg(config, "horizon"))
        self.receding_horizon = int(_cfg(config, "receding_horizon", self.horizon))
        self.action_block = int(_cfg(config, "action_block", 1))
        if self.horizon <= 0 or self.action_block <= 0:
            raise ValueError(f"horizon and action_block must be positive, got {self.horizon}, {self.action_block}")
        if not 1 <= self.receding_horizon <= self.horizon:
            raise ValueError(f"receding_horizon must be in [1, horizon={self.horizon}], got {self.receding_horizon}")
        self.env = None
        self._buffer: Optional[np.ndarray] = None  # (n_envs, steps left, raw_dim), env units
        self._served = 0
        self._warm: Optional[torch.Tensor] = None  # unexecuted tail of the last plan
        self.solves = 0
        self.last_solve: Optional[dict] = None

    # ------------------------------------------------------------------ world wiring
    def set_env(self, env: Any) -> None:
        """Attach the (vector) env and configure the solver for its action space and env count."""
        self.env = env
        configure = getattr(self.solver, "configure", None)
        if callable(configure):
            configure(action_space=env.action_space, n_envs=int(env.num_envs), config=self.cfg)
        self.reset()

    def reset(self) -> None:
        """Drop the buffered actions and the warm start (episode boundary)."""
        self._buffer = None
        self._served = 0
        self._warm = None
        reset_ws = getattr(self.solver, "reset_warm_start_state", None)
        if callable(reset_ws):
            reset_ws("policy_reset")

    @property
    def buffered_steps(self) -> int:
        """Raw actions left in the buffer (0: the next call plans)."""
        return 0 if self._buffer is None else self._buffer.shape[1] - self._served

    # ------------------------------------------------------------------ planning
    def _prepare(self, info_dict: dict) -> dict:
        """The solver's view of the observation: normalised columns, images encoded or transformed."""
        info = {}
        for key, value in info_dict.items():
            scaler = self.process.get(key)
            if scaler is not None and key not in _IMAGE_KEYS and key != "action":
                arr = np.asarray(value.cpu() if torch.is_tensor(value) else value, dtype=np.float32)
                flat = scaler.transform(arr.reshape(-1, arr.shape[-1])).reshape(arr.shape)
                value = torch.as_tensor(flat, dtype=torch.float32)
            info[key] = value
        if self.encoder is not None and _is_frames(info.get("pixels")) and _is_frames(info.get("goal")):
            info["emb"], info["goal_emb"] = self._encode(info["pixels"], info["goal"])
        else:
            for key in _IMAGE_KEYS:
                tf = self.transform.get(key)
                if tf is not None and key in info:
                    info[key] = tf(info[key])
        return info

    def _encode(self, pixels: torch.Tensor, goal: torch.Tensor):
        """uint8 (B, T, H, W, C) observation frames and (B, G, H, W, C) goal frames -> (B, T, D),
        (B, G, D) embeddings, all frames in one encoder pass."""
        b, t = pixels.shape[:2]
        g = goal.shape[1]
        dev = self.encoder.device
        frames = torch.cat([pixels.reshape(b * t, *pixels.shape[2:]).to(dev, non_blocking=True),
                            goal.reshape(b * g, *goal.shape[2:]).to(dev, non_blocking=True)])
        emb = self.encoder.encode_frames(frames, mean=self.image_mean, std=self.image_std)
        return emb[: b * t].reshape(b, t, -1), emb[b * t:].reshape(b, g, -1)

    def _plan(self, info_dict: dict) -> None:
        info = self._prepare(info_dict)
        out = self.solver.solve(info, init_action=self._warm)
        self.solves += 1
        self.last_solve = out
        actions = out["actions"]
        actions = actions if torch.is_tensor(actions) else torch.as_tensor(actions)
        n_envs, horizon, width = actions.shape
        if horizon != self.horizon or width % self.action_block:
            raise ValueError(f"solver actions {tuple(actions.shape)} do not match horizon {self.horizon} x "
                             f"action_block {self.action_block}")
        r = self.receding_horizon
        self._warm = actions[:, r:].clone() if r < horizon else None
        raw = actions[:, :r].reshape(n_envs, r * self.action_block, width // self.action_block)
        raw = raw.detach().to("cpu", torch.float32).numpy()
        scaler = self.process.get("action")
        if scaler is not None:
            raw = scaler.inverse_transform(raw.reshape(-1, raw.shape[-1])).reshape(raw.shape)
        self._buffer = np.ascontiguousarray(raw, dtype=np.float32)
        self._served = 0

    def get_action(self, info_dict: dict, **kwargs: Any) -> np.ndarray:
        """One raw action per env, ``(n_envs, raw_dim)`` in env units; plans when the buffer is empty."""
        if self.buffered_steps == 0:
            self._plan(info_dict)
        a = self._buffer[:, self._served]
        self._served += 1
        return a

    __call__ = get_action


def _is_frames(x: Any) -> bool:
    """uint8 frames (B, T, H, W, C), the encoder's fused-transform input."""
    return torch.is_tensor(x) and x.dtype == torch.uint8 and x.ndim == 5
