"""Drop-in iCEM / CEM solvers and model-cost helper backed by the B200 kernels.

* ``B200ICEMSolver`` takes exactly the constructor arguments of the reference
  ``ICEMSolver`` (``lewm/solvers/icem.py:258-322``), raises the same
  ``ValueError``s, exposes the same properties and ``configure`` /
  ``sample_counts`` / ``model_cost_evals_per_solve`` / ``solve`` / ``__call__``
  surface and returns the same ``solve`` dict (CPU ``actions``, ``mean``,
  ``var``, ``costs`` and, with callbacks, ``callbacks``). A Hydra config swaps
  ``_target_: lewm.solvers.icem.ICEMSolver`` for
  ``lewm_flash_b200.solver.B200ICEMSolver``.
* ``B200CEMSolver`` is ``CEMExactSolver`` (``lewm/solvers/cem_exact.py:54-383``):
  iCEM with every feature off, plus its receding-horizon warm start.
* ``B200CEMGDSolver`` is ``CEMGDSolver`` (``lewm/solvers/cem_gd.py:38-711``): the seed
  search as one device plan, the gradient refinement on the device gradient.
* ``B200ICEMStaticSolver`` is ``ICEMStaticCompileSolver``
  (``lewm/solvers/icem_static_compile.py:117-373``): the static chain is the device plan.
* ``run_static_icem_chain`` mirrors the reference tensor-only chain
  (``lewm/solvers/icem_static_compile.py:61-114``) with injected noise.
* ``B200ModelCost`` / ``install_model_cost`` replace
  ``JEPA.get_cost_from_embeddings`` (``lewm/jepa.py:302-317``).

The model cost follows the JEPA's ``model_cost_autocast_mode()`` at every call, as
the reference does: "bf16" runs the tensor-core kernels, "none" (a JEPA's default)
the float32 kernels.

All envs of a ``solve`` run as one batched device plan; ``batch_size`` is
accepted for interface compatibility. Noise comes from a counter-based Philox
stream keyed by (seed, solve index, iteration, env, candidate) instead of the
reference's sequential torch generator, so a given seed gives a different (but
deterministic) stream than the reference; parity with the reference is checked
by injecting the reference's noise (``run_static_icem_chain``).
"""

from __future__ import annotations

import math
import time
import warnings
from dataclasses import dataclass
from typing import Any, Optional, Sequence

import numpy as np
import torch

from .runtime import PlanOptions, Runtime

COLORED_NOISE_BETA = {"none": 0.0, "pink": 1.0, "brown": 2.0}


def _runtime(model, device) -> Runtime:
    if isinstance(model, Runtime):
        return model
    cache = getattr(model, "_lewm_b200_runtimes", None)
    if cache is None:
        cache = {}
        try:
            setattr(model, "_lewm_b200_runtimes", cache)
        except Exception:  # pragma: no cover
            pass
    dev = torch.device(device)
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    if key not in cache:
        from .model import extract_state_dict, infer_desc

        desc = infer_desc(model)
        cache[key] = Runtime(desc, extract_state_dict(model, desc), torch.device("cuda", key))
    rt = cache[key]
    # The model's model-cost arithmetic, read at every use as JEPA.get_cost_from_embeddings
    # reads it (lewm/jepa.py:310-317): "none" (a JEPA's default) float32, "bf16" tensor cores.
    mode_of = getattr(model, "model_cost_autocast_mode", None)
    if callable(mode_of):
        rt.set_model_cost_autocast(mode_of())
    return rt


def prepare_init_action(model: Any, info_dict: dict, init_action: Optional[torch.Tensor], horizon: int, *,
                        n_envs: int, action_dim: int) -> torch.Tensor:
    """Warm-start padding of ``prepare_init_action`` (reference ``lewm/solvers/cem_exact.py:13-51``)."""
    if init_action is not None:
        assert init_action.shape[0] == n_envs, f"init_action batch size {init_action.shape[0]} != n_envs {n_envs}"
        assert init_action.shape[2] == action_dim, (
            f"init_action action_dim {init_action.shape[2]} != action_dim {action_dim}")
    n_prev = init_action.shape[1] if init_action is not None else 0
    remaining = horizon - n_prev
    if remaining <= 0:
        return init_action
    if not hasattr(model, "get_action"):
        device = init_action.device if init_action is not None else "cpu"
        tail = torch.zeros(n_envs, remaining, action_dim, device=device)
        return torch.cat([init_action, tail], dim=1) if init_action is not None else tail
    with torch.no_grad():
        tail = model.get_action(info_dict, horizon=remaining, prefix_actions=init_action)
    return torch.cat([init_action.to(tail.device), tail], dim=1) if init_action is not None else tail


class B200ICEMSolver:
    """iCEM solver whose whole iteration loop runs on the B200 plan kernels.

    ``noise_source`` (default None) is the hook for reproducing a reference run: a
    callable ``(batch_size, n_samples) -> (batch_size, n_samples, T, A)`` tensor of
    post-coloring noise, e.g. the ``_sample_noise`` method of a reference
    ``ICEMSolver`` built with the same seed. When set, ``solve`` draws every
    iteration's noise from it in the reference's order (env batch by env batch,
    iteration by iteration, ``lewm/solvers/icem.py:501-521``) and plans on that
    injected noise instead of the in-kernel Philox stream.
    """

    defer_cpu_materialization = True
    noise_source = None

    def __init__(
        self,
        model: Any,
        batch_size: int = 1,
        num_samples: int = 300,
        var_scale: float = 1.0,
        n_steps: int = 30,
        topk: int = 30,
        device: str | torch.device = "cuda",
        seed: int = 1234,
        elite_retention: int = 0,
        colored_noise: str = "none",
        colored_noise_time: str = "raw",
        momentum_alpha: float = 0.0,
        sample_decay: float = 1.0,
        sample_count_bucket_size: int = 0,
        return_best_elite: bool = False,
        clip_actions: bool = False,
        callbacks: list[Any] | None = None,
        history_size: int = 3,
    ) -> None:
        if topk <= 0:
            raise ValueError(f"topk must be positive, got {topk}")
        if num_samples < topk:
            raise ValueError(f"num_samples={num_samples} must be >= topk={topk}")
        if n_steps <= 0:
            raise ValueError(f"n_steps must be positive, got {n_steps}")
        if elite_retention < 0:
            raise ValueError(f"elite_retention must be non-negative, got {elite_retention}")
        if colored_noise not in COLORED_NOISE_BETA:
            raise ValueError(
                f"colored_noise must be one of {sorted(COLORED_NOISE_BETA)}, got {colored_noise!r}")
        if not 0.0 <= momentum_alpha < 1.0:
            raise ValueError(f"momentum_alpha must satisfy 0 <= alpha < 1, got {momentum_alpha}")
        if sample_decay < 1.0:
            raise ValueError(f"sample_decay must be >= 1.0, got {sample_decay}")
        if sample_count_bucket_size < 0:
            raise ValueError(f"sample_count_bucket_size must be non-negative, got {sample_count_bucket_size}")
        if colored_noise_time not in ("block", "raw"):
            raise ValueError(f"colored noise time_axis must be 'block' or 'raw', got {colored_noise_time!r}")
        self.model = model
        self.batch_size = batch_size
        self.var_scale = var_scale
        self.num_samples = num_samples
        self.n_steps = n_steps
        self.topk = topk
        self.device = torch.device(device)
        self.seed = int(seed)
        self.elite_retention = elite_retention
        self.colored_noise = colored_noise
        self.colored_noise_time = colored_noise_time
        self.momentum_alpha = float(momentum_alpha)
        self.sample_decay = float(sample_decay)
        self.sample_count_bucket_size = int(sample_count_bucket_size)
        self.return_best_elite = bool(return_best_elite)
        self.clip_actions = bool(clip_actions)
        self.callbacks = list(callbacks) if callbacks else []
        self.history_size = int(history_size)
        self._action_low: torch.Tensor | None = None
        self._action_high: torch.Tensor | None = None
        self._solves = 0
        try:
            self._dtype = next(model.parameters()).dtype
        except (AttributeError, StopIteration, TypeError):
            self._dtype = torch.float32

    # ------------------------------------------------------------------ reference surface
    def configure(self, *, action_space: Any, n_envs: int, config: Any) -> None:
        self._action_space = action_space
        self._n_envs = n_envs
        self._config = config
        self._action_dim = int(np.prod(action_space.shape[1:]))
        self._configured = True
        if "Box" not in type(action_space).__name__:
            warnings.warn(f"Action space is not Box-like, got {type(action_space)}. "
                          "ICEMSolver may not work as expected.", RuntimeWarning, stacklevel=2)
            return
        if self.clip_actions and hasattr(action_space, "low") and hasattr(action_space, "high"):
            self._action_low = torch.as_tensor(action_space.low[0], device=self.device,
                                               dtype=self.dtype).repeat(self._config.action_block)
            self._action_high = torch.as_tensor(action_space.high[0], device=self.device,
                                                dtype=self.dtype).repeat(self._config.action_block)
        for cb in self.callbacks:
            configure = getattr(cb, "configure", None)
            if callable(configure):
                configure(action_low=self._action_low, action_high=self._action_high)

    @property
    def n_envs(self) -> int:
        return self._n_envs

    @property
    def action_dim(self) -> int:
        return self._action_dim * self._config.action_block

    @property
    def horizon(self) -> int:
        return self._config.horizon

    @property
    def action_block(self) -> int:
        return int(getattr(self._config, "action_block", 1))

    @property
    def dtype(self) -> torch.dtype:
        return self._dtype

    def __call__(self, *args: Any, **kwargs: Any) -> dict[str, Any]:
        return self.solve(*args, **kwargs)

    def sample_count_for_step(self, step: int) -> int:
        if self.sample_decay == 1.0:
            return self.num_samples
        decayed = int(math.ceil(self.num_samples * (self.sample_decay ** (-step))))
        count = max(decayed, min(self.num_samples, 2 * self.topk))
        if self.sample_count_bucket_size > 0:
            count = min(self.num_samples,
                        int(math.ceil(count / self.sample_count_bucket_size)) * self.sample_count_bucket_size)
        return count

    def sample_counts(self) -> list[int]:
        return [self.sample_count_for_step(step) for step in range(self.n_steps)]

    def model_cost_evals_per_solve(self) -> int:
        return sum(self.sample_counts())

    def init_action_distrib(self, n_envs: int, actions: torch.Tensor | None = None):
        var = self.var_scale * torch.ones([n_envs, self.horizon, self.action_dim], dtype=self.dtype)
        mean = torch.zeros([n_envs, 0, self.action_dim], dtype=self.dtype) if actions is None else actions
        remaining = self.horizon - mean.shape[1]
        if remaining > 0:
            new_mean = torch.zeros([n_envs, remaining, self.action_dim], dtype=self.dtype, device=mean.device)
            mean = torch.cat([mean, new_mean], dim=1)
        return mean, var

    # ------------------------------------------------------------------ B200 specifics
    def plan_options(self) -> PlanOptions:
        return PlanOptions(
            num_samples=self.num_samples, topk=self.topk, n_steps=self.n_steps, sample_decay=self.sample_decay,
            sample_count_bucket_size=self.sample_count_bucket_size, elite_retention=self.elite_retention,
            beta=COLORED_NOISE_BETA[self.colored_noise], time_axis=self.colored_noise_time,
            action_block=self.action_block, momentum_alpha=self.momentum_alpha,
            return_best_elite=self.return_best_elite, clip_actions=self._action_low is not None,
            history_size=self.history_size, seed=self.seed)

    @property
    def runtime(self) -> Runtime:
        return _runtime(self.model, self.device)

    def _cost_embeddings(self, info_dict: dict, total_envs: int):
        """(emb (B,H,D), goal_emb (B,G,D)) -- cached tensors if given, else the model's encoder.

        The encoder path mirrors ``ICEMStaticCompileSolver._prepare_cost_embeddings``
        (reference ``lewm/solvers/icem_static_compile.py:212-238``).
        """
        emb = info_dict.get("emb")
        goal = info_dict.get("goal_emb")
        if torch.is_tensor(emb) and torch.is_tensor(goal) and emb.ndim == 3:
            return emb, goal
        expanded = {}
        for key, value in info_dict.items():
            if torch.is_tensor(value):
                tgt = self.dtype if value.is_floating_point() else None
                expanded[key] = value.to(device=self.device, dtype=tgt).unsqueeze(1)
            elif isinstance(value, np.ndarray):
                expanded[key] = value[:, None]
            else:
                expanded[key] = value
        dummy = torch.zeros(total_envs, 1, self.horizon, self.action_dim, device=self.device, dtype=self.dtype)
        if not hasattr(self.model, "_ensure_cost_embeddings"):
            raise RuntimeError("B200ICEMSolver needs emb/goal_emb in info_dict or a JEPA with _ensure_cost_embeddings")
        emb, goal = self.model._ensure_cost_embeddings(expanded, dummy)
        if emb.ndim == 4:
            emb = emb[:, 0]
        if goal.ndim == 4:
            goal = goal[:, 0]
        return emb, goal

    def _injected_noise(self, total_envs: int):
        """Every iteration's noise from ``noise_source``, drawn in the reference's order."""
        if self.noise_source is None:
            return None
        counts = self.sample_counts()
        steps = [[] for _ in counts]
        for start in range(0, total_envs, self.batch_size):
            bs = min(start + self.batch_size, total_envs) - start
            for step, n in enumerate(counts):
                steps[step].append(self.noise_source(bs, n).to(device=self.device, dtype=torch.float32))
        return [torch.cat(chunks, dim=0) for chunks in steps]

    def _plan(self, info_dict: dict, mean: torch.Tensor, var: torch.Tensor, trace: bool, emb_goal=None):
        total_envs = mean.shape[0]
        emb, goal = emb_goal if emb_goal is not None else self._cost_embeddings(info_dict, total_envs)
        # Host embeddings go up without blocking the host: the solve synchronises the stream
        # before it returns, so the caller's buffers are read before they can change.
        emb = emb.to(self.device, torch.float32, non_blocking=True)
        goal = goal.to(self.device, torch.float32, non_blocking=True)
        rt = self.runtime
        opts = self.plan_options()
        plan_index = self._solves
        self._solves += 1
        return rt.plan(opts, emb, goal, mean, var, noise_steps=self._injected_noise(total_envs),
                       action_low=self._action_low, action_high=self._action_high, trace=trace,
                       plan_index=plan_index)

    @torch.inference_mode()
    def solve(self, info_dict: dict, init_action: torch.Tensor | None = None) -> dict[str, Any]:
        outputs: dict[str, Any] = {"costs": [], "mean": [], "var": []}
        total_envs = len(next(iter(info_dict.values())))
        init_action = prepare_init_action(self.model, info_dict, init_action, self.horizon, n_envs=total_envs,
                                          action_dim=self.action_dim)
        mean, var = self.init_action_distrib(total_envs, init_action)
        mean = mean.to(self.device)
        var = var.to(self.device)
        for cb in self.callbacks:
            cb.reset()
        actions, std, fcost, tr = self._plan(info_dict, mean, var, trace=bool(self.callbacks))
        if self.callbacks:
            self._replay_callbacks(tr, mean, var)
        # One device->host read per solve (reference lewm/solvers/icem.py:589-593): the three
        # outputs are queued into pinned host buffers on the plan's stream, then one sync.
        h_cost, h_act, h_std = self._host_outputs(actions, std, fcost)
        h_cost.copy_(fcost, non_blocking=True)
        h_act.copy_(actions, non_blocking=True)
        h_std.copy_(std, non_blocking=True)
        self.runtime.sync()
        outputs["costs"].extend(h_cost.tolist())
        actions_cpu = h_act.clone()
        outputs["actions"] = actions_cpu
        outputs["mean"] = [actions_cpu.clone()]
        outputs["var"] = [h_std.clone()]
        if self.callbacks:
            outputs["callbacks"] = {}
            for cb in self.callbacks:
                cb.end_solve()
                outputs["callbacks"][cb.output_key] = cb.history
        return outputs

    def _host_outputs(self, actions: torch.Tensor, std: torch.Tensor, fcost: torch.Tensor):
        """Pinned host buffers for a solve's final cost, actions and std, kept per shape (the
        results are cloned out of them before ``solve`` returns)."""
        cache = self.__dict__.setdefault("_host_out", {})
        key = (tuple(actions.shape), tuple(fcost.shape))
        if key not in cache:
            cache[key] = (torch.empty(fcost.shape, dtype=torch.float32, pin_memory=True),
                          torch.empty(actions.shape, dtype=torch.float32, pin_memory=True),
                          torch.empty(std.shape, dtype=torch.float32, pin_memory=True))
        return cache[key]

    _callback_n_samples = True  # ICEMSolver passes n_samples to its callbacks; CEMExactSolver does not

    def _replay_callbacks(self, tr, mean0, var0) -> None:
        """Feed the per-iteration plan trace to the reference callback protocol.

        Same calls, in the same order and with the same per-env-batch tensors, as the
        reference's solve loop (``lewm/solvers/icem.py:501-578``): ``start_batch`` once
        per env batch of ``batch_size`` envs, then one call per iteration.
        """
        total = int(mean0.shape[0])
        for start in range(0, total, self.batch_size):
            end = min(start + self.batch_size, total)
            for cb in self.callbacks:
                cb.start_batch()
            prev_mean, prev_var = mean0[start:end], var0[start:end]
            for step, n in enumerate(tr["counts"]):
                cand = tr["candidates"][step][start:end, :n]
                costs = tr["costs"][step][start:end, :n]
                inds = tr["topk_idx"][step][start:end].long()
                vals = tr["topk_val"][step][start:end]
                topk_cand = torch.gather(cand, 1,
                                         inds[:, :, None, None].expand(-1, -1, cand.shape[2], cand.shape[3]))
                m, v = tr["mean"][step][start:end], tr["std"][step][start:end]
                kw = dict(step=step, candidates=cand, costs=costs, topk_vals=vals, topk_inds=inds,
                          topk_candidates=topk_cand, mean=m, var=v, prev_mean=prev_mean, prev_var=prev_var)
                if self._callback_n_samples:
                    kw["n_samples"] = n
                for cb in self.callbacks:
                    cb(**kw)
                prev_mean, prev_var = m, v


@dataclass
class StaticChainWarmupResult:
    """``StaticChainWarmupResult`` (reference ``lewm/solvers/icem_static_compile.py:19-26``)."""

    enabled: bool
    elapsed_s: Optional[float]
    sample_counts: list
    mode: str
    fullgraph: bool
    input_shapes: Optional[dict]


class B200ICEMStaticSolver(B200ICEMSolver):
    """``ICEMStaticCompileSolver`` (reference ``lewm/solvers/icem_static_compile.py:117-373``) on
    the B200 kernels. The reference moves the candidate / model-cost / top-k / refit chain into a
    tensor-only function run eagerly or under ``torch.compile``; here that chain is always the
    device plan (one CUDA graph per plan shape), so ``static_chain_compile`` only selects what
    ``warmup_static_chain_compile`` reports, as in the reference. Same extra arguments and
    ``ValueError``, and ``solve`` adds the reference's ``static_chain`` record."""

    def __init__(self, *args: Any, static_chain_compile: bool = False, static_chain_mode: str = "reduce-overhead",
                 static_chain_fullgraph: bool = False, static_chain_warmup: bool = True, **kwargs: Any) -> None:
        super().__init__(*args, **kwargs)
        if static_chain_mode not in {"default", "reduce-overhead", "max-autotune"}:
            raise ValueError("static_chain_mode must be one of 'default', 'reduce-overhead', or 'max-autotune', "
                             f"got {static_chain_mode!r}")
        self.static_chain_compile = bool(static_chain_compile)
        self.static_chain_mode = static_chain_mode
        self.static_chain_fullgraph = bool(static_chain_fullgraph)
        self.static_chain_warmup = bool(static_chain_warmup)
        self._static_compile_warmed = False

    def warmup_static_chain_compile(self, *, embed_dim: int, history: int = 1,
                                    batch_size: int | None = None) -> StaticChainWarmupResult:
        """Plan once on zero inputs of the given shape, capturing the plan's CUDA graph
        (``warmup_static_chain_compile``, ``icem_static_compile.py:246-315``)."""
        counts = self.sample_counts()
        if not self.static_chain_compile or not self.static_chain_warmup:
            return StaticChainWarmupResult(False, None, counts, self.static_chain_mode, self.static_chain_fullgraph,
                                           None)
        bs = int(batch_size or self.batch_size)
        emb = torch.zeros(bs, history, embed_dim, device=self.device, dtype=self.dtype)
        goal = torch.zeros_like(emb)
        mean = torch.zeros(bs, self.horizon, self.action_dim, device=self.device, dtype=self.dtype)
        var = self.var_scale * torch.ones_like(mean)
        started = time.perf_counter()
        with torch.inference_mode():
            self.runtime.plan(self.plan_options(), emb, goal, mean, var, action_low=self._action_low,
                              action_high=self._action_high)
        torch.cuda.synchronize(self.device)
        self._static_compile_warmed = True
        return StaticChainWarmupResult(
            True, time.perf_counter() - started, counts, self.static_chain_mode, self.static_chain_fullgraph,
            {"emb": list(emb.shape), "goal_emb": list(goal.shape), "mean": list(mean.shape), "var": list(var.shape),
             "noise_steps": [[bs, n, self.horizon, self.action_dim] for n in counts]})

    def solve(self, info_dict: dict, init_action: torch.Tensor | None = None) -> dict[str, Any]:
        outputs = super().solve(info_dict, init_action)
        outputs["static_chain"] = {
            "static_chain_compile": self.static_chain_compile, "static_chain_mode": self.static_chain_mode,
            "static_chain_fullgraph": self.static_chain_fullgraph, "static_chain_warmed": self._static_compile_warmed,
            "sample_counts_per_step": self.sample_counts(),
        }
        return outputs


class B200CEMSolver(B200ICEMSolver):
    """``CEMExactSolver`` semantics (reference ``lewm/solvers/cem_exact.py:54-383``) on the B200 kernels.

    iCEM with every feature off is CEM (reference ``tests/test_lewm_icem.py:56-96``).
    ``warm_start`` shifts the previous solve's mean/var by the receding horizon
    (``_shift_warm_start_distribution``, ``cem_exact.py:193-241``).
    """

    def __init__(self, model: Any, batch_size: int = 1, num_samples: int = 300, var_scale: float = 1.0,
                 n_steps: int = 30, topk: int = 30, device: str | torch.device = "cuda", seed: int = 1234,
                 warm_start: bool = False, callbacks: list[Any] | None = None, history_size: int = 3) -> None:
        super().__init__(model, batch_size=batch_size, num_samples=num_samples, var_scale=var_scale, n_steps=n_steps,
                         topk=topk, device=device, seed=seed, callbacks=callbacks, history_size=history_size)
        self.warm_start = bool(warm_start)
        self._warm_mean: torch.Tensor | None = None
        self._warm_var: torch.Tensor | None = None
        self._warm_signature: tuple | None = None
        self._last_warm_start_info = {"enabled": self.warm_start, "used": False, "reset": False, "reset_reason": None}

    _callback_n_samples = False  # CEMExactSolver's callbacks get no n_samples (cem_exact.py:340-351)

    def configure(self, *, action_space: Any, n_envs: int, config: Any) -> None:
        super().configure(action_space=action_space, n_envs=n_envs, config=config)
        self.reset_warm_start_state("configure")

    @property
    def receding_horizon(self) -> int:
        return int(getattr(self._config, "receding_horizon", self.horizon))

    @property
    def last_warm_start_info(self) -> dict:
        return dict(self._last_warm_start_info)

    def reset_warm_start_state(self, reason: str = "manual") -> None:
        self._warm_mean = None
        self._warm_var = None
        self._warm_signature = None
        self._last_warm_start_info = {"enabled": self.warm_start, "used": False, "reset": True,
                                      "reset_reason": reason}

    def _distribution_signature(self, mean: torch.Tensor, var: torch.Tensor) -> tuple:
        """What a remembered distribution must match to warm-start the next solve
        (``_distribution_signature``, ``cem_exact.py:166-180``)."""
        return (*map(int, mean.shape), *map(int, var.shape), int(self.batch_size), self.receding_horizon,
                torch.device(mean.device), mean.dtype, torch.device(var.device), var.dtype)

    def _shift(self, mean: torch.Tensor, var: torch.Tensor):
        info = {"enabled": self.warm_start, "used": False, "reset": False, "reset_reason": None,
                "receding_horizon": self.receding_horizon}
        if not self.warm_start:
            self._last_warm_start_info = info
            return mean, var
        shift = self.receding_horizon
        if shift <= 0 or shift >= self.horizon:
            info["reset"] = shift >= self.horizon
            info["reset_reason"] = "no_unexecuted_tail" if shift >= self.horizon else "invalid_shift"
            self._last_warm_start_info = info
            return mean, var
        if (self._warm_mean is None or self._warm_var is None
                or self._warm_signature != self._distribution_signature(mean, var)):
            had = self._warm_mean is not None or self._warm_var is not None
            self._warm_mean = self._warm_var = None
            self._warm_signature = None
            info["reset"] = had
            info["reset_reason"] = "signature_mismatch" if had else "no_previous_state"
            self._last_warm_start_info = info
            return mean, var
        m = torch.zeros_like(mean)
        v = self.var_scale * torch.ones_like(var)
        m[:, :-shift] = self._warm_mean[:, shift:].to(mean)
        v[:, :-shift] = self._warm_var[:, shift:].to(var)
        info["used"] = True
        self._last_warm_start_info = info
        return m, v

    @torch.inference_mode()
    def solve(self, info_dict: dict, init_action: torch.Tensor | None = None) -> dict[str, Any]:
        total_envs = len(next(iter(info_dict.values())))
        init_action = prepare_init_action(self.model, info_dict, init_action, self.horizon, n_envs=total_envs,
                                          action_dim=self.action_dim)
        mean, var = self.init_action_distrib(total_envs, init_action)
        mean, var = self._shift(mean.to(self.device), var.to(self.device))
        for cb in self.callbacks:
            cb.reset()
        actions, std, fcost, tr = self._plan(info_dict, mean, var, trace=bool(self.callbacks))
        if self.callbacks:
            self._replay_callbacks(tr, mean, var)
        costs = fcost.cpu().tolist()
        self.runtime.sync()
        out = {"costs": costs, "actions": actions.cpu(), "mean": [actions.cpu()], "var": [std.cpu()],
               "warm_start": self.last_warm_start_info}
        if self.warm_start:
            self._warm_signature = self._distribution_signature(actions, std)
            self._warm_mean, self._warm_var = actions.detach().clone(), std.detach().clone()
        if self.callbacks:
            out["callbacks"] = {}
            for cb in self.callbacks:
                cb.end_solve()
                out["callbacks"][cb.output_key] = cb.history
        return out


class B200CEMGDSolver(B200ICEMSolver):
    """``CEMGDSolver`` (reference ``lewm/solvers/cem_gd.py:38-711``) on the B200 kernels: the
    CEM / iCEM seed search of every env as one device plan, then CEM-GD's refinement (Adam
    with 1 / 1/2 / 1/4 / 1/10 backtracking and per-seed acceptance, ``_refine_seed_actions``,
    ``:459-606``) stepping on the device gradient of the model cost (``lewm_model_cost_grad``).

    Same constructor arguments, ``ValueError`` texts, properties and ``solve`` output (``costs``,
    ``mean``, ``var``, ``actions``, ``gd_summary``) as the reference. The seed search draws its
    noise from the in-kernel Philox stream, or from ``noise_source`` (a reference solver's
    ``_sample_noise``) to reproduce a reference run. The refinement runs env batch by env batch
    of ``batch_size`` as the reference does (its loss is the mean over a batch's seeds, which
    Adam's epsilon sees). The gradient step's forward and reverse pass are one device call:
    ``gd_forward_time_ms_mean`` times it, ``gd_backward_time_ms_mean`` is 0.
    """

    def __init__(self, model: Any | None = None, batch_size: int = 1, num_samples: int = 300, var_scale: float = 1.0,
                 n_steps: int = 30, topk: int = 30, device: str | torch.device = "cuda", seed: int = 1234,
                 elite_retention: int = 0, colored_noise: str = "none", colored_noise_time: str = "raw",
                 momentum_alpha: float = 0.0, sample_decay: float = 1.0, sample_count_bucket_size: int = 0,
                 return_best_elite: bool = False, clip_actions: bool = False, gd_seed_solver: str = "cem",
                 gd_seed_source: str = "best_elite", gd_refine_topk: int = 1, gd_steps: int = 1, gd_lr: float = 0.01,
                 gd_compile_cost: bool = False, gd_backtracking: bool = True, callbacks: list[Any] | None = None,
                 history_size: int = 3) -> None:
        if topk <= 0:
            raise ValueError(f"topk must be positive, got {topk}")
        if num_samples < topk:
            raise ValueError(f"num_samples={num_samples} must be >= topk={topk}")
        if n_steps <= 0:
            raise ValueError(f"n_steps must be positive, got {n_steps}")
        if elite_retention < 0:
            raise ValueError(f"elite_retention must be non-negative, got {elite_retention}")
        if colored_noise not in COLORED_NOISE_BETA:
            raise ValueError(
                f"colored_noise must be one of {sorted(COLORED_NOISE_BETA)}, got {colored_noise!r}")
        if not 0.0 <= momentum_alpha < 1.0:
            raise ValueError(f"momentum_alpha must satisfy 0 <= alpha < 1, got {momentum_alpha}")
        if sample_decay < 1.0:
            raise ValueError(f"sample_decay must be >= 1.0, got {sample_decay}")
        if sample_count_bucket_size < 0:
            raise ValueError(f"sample_count_bucket_size must be non-negative, got {sample_count_bucket_size}")
        if gd_seed_solver not in {"cem", "icem"}:
            raise ValueError(f"gd_seed_solver must be 'cem' or 'icem', got {gd_seed_solver!r}")
        if gd_seed_source not in {"best_elite", "mean"}:
            raise ValueError(f"gd_seed_source must be 'best_elite' or 'mean', got {gd_seed_source!r}")
        if gd_refine_topk <= 0:
            raise ValueError(f"gd_refine_topk must be positive, got {gd_refine_topk}")
        if gd_refine_topk > topk:
            raise ValueError(f"gd_refine_topk={gd_refine_topk} must be <= topk={topk}")
        if gd_steps < 0:
            raise ValueError(f"gd_steps must be non-negative, got {gd_steps}")
        if gd_lr <= 0.0:
            raise ValueError(f"gd_lr must be positive, got {gd_lr}")
        super().__init__(model, batch_size=batch_size, num_samples=num_samples, var_scale=var_scale, n_steps=n_steps,
                         topk=topk, device=device, seed=seed, elite_retention=elite_retention,
                         colored_noise=colored_noise, colored_noise_time=colored_noise_time,
                         momentum_alpha=momentum_alpha, sample_decay=sample_decay,
                         sample_count_bucket_size=sample_count_bucket_size, return_best_elite=return_best_elite,
                         clip_actions=clip_actions, callbacks=callbacks, history_size=history_size)
        self.gd_seed_solver = gd_seed_solver
        self.gd_seed_source = gd_seed_source
        self.gd_refine_topk = int(gd_refine_topk)
        self.gd_steps = int(gd_steps)
        self.gd_lr = float(gd_lr)
        self.gd_compile_cost = bool(gd_compile_cost)
        self.gd_backtracking = bool(gd_backtracking)

    def configure(self, *, action_space: Any, n_envs: int, config: Any) -> None:
        """``CEMGDSolver.configure`` (``cem_gd.py:134-157``): no callback protocol."""
        self._action_space = action_space
        self._n_envs = n_envs
        self._config = config
        self._action_dim = int(np.prod(action_space.shape[1:]))
        self._configured = True
        if "Box" not in type(action_space).__name__:
            warnings.warn(f"Action space is not Box-like, got {type(action_space)}. "
                          "CEMGDSolver may not work as expected.", RuntimeWarning, stacklevel=2)
            return
        if self.clip_actions and hasattr(action_space, "low") and hasattr(action_space, "high"):
            self._action_low = torch.as_tensor(action_space.low[0], device=self.device,
                                               dtype=self.dtype).repeat(self._config.action_block)
            self._action_high = torch.as_tensor(action_space.high[0], device=self.device,
                                                dtype=self.dtype).repeat(self._config.action_block)

    def sample_count_for_step(self, step: int) -> int:
        if self.gd_seed_solver == "cem":
            return self.num_samples
        return super().sample_count_for_step(step)

    def plan_options(self) -> PlanOptions:
        """The seed search: plain CEM (white noise, no decay, retention or momentum) or iCEM
        (``_run_seed_search_batch``, ``cem_gd.py:370-436``); never the best elite as output."""
        icem = self.gd_seed_solver == "icem"
        return PlanOptions(
            num_samples=self.num_samples, topk=self.topk, n_steps=self.n_steps,
            sample_decay=self.sample_decay if icem else 1.0,
            sample_count_bucket_size=self.sample_count_bucket_size if icem else 0,
            elite_retention=self.elite_retention if icem else 0,
            beta=COLORED_NOISE_BETA[self.colored_noise] if icem else 0.0, time_axis=self.colored_noise_time,
            action_block=self.action_block, momentum_alpha=self.momentum_alpha if icem else 0.0,
            return_best_elite=False, clip_actions=self._action_low is not None, history_size=self.history_size,
            seed=self.seed, counts=self.sample_counts())

    def _action_saturation_rate(self, actions: torch.Tensor) -> float | None:
        if self._action_low is None or self._action_high is None:
            return None
        low = self._action_low.to(device=actions.device, dtype=actions.dtype)
        high = self._action_high.to(device=actions.device, dtype=actions.dtype)
        saturated = (actions - low).abs().le(1e-5) | (actions - high).abs().le(1e-5)
        return float(saturated.float().mean().detach().cpu().item())

    def _refine_seed_actions(self, seed_actions: torch.Tensor, seed_costs: torch.Tensor, emb: torch.Tensor,
                             goal_emb: torch.Tensor, *, enable_backtracking: bool | None = None):
        """``_refine_seed_actions`` (``cem_gd.py:459-606``) with the device gradient."""
        rt = self.runtime
        hs = self.history_size
        params = seed_actions.detach().clone().requires_grad_(True)
        optimizer = torch.optim.Adam([params], lr=self.gd_lr)
        current_costs = seed_costs.detach().clone()
        accepted_any = torch.zeros_like(current_costs, dtype=torch.bool)
        forward_times: list[float] = []
        grad_norm_values: list[float] = []
        grad_norm_max = 0.0
        nan_or_inf_count = 0
        refine_width = int(seed_actions.shape[1])
        backtrack = self.gd_backtracking if enable_backtracking is None else enable_backtracking
        factors = [1.0, 0.5, 0.25, 0.1] if backtrack else [1.0]
        evals = 0
        final_actions = seed_actions.detach()
        final_costs = seed_costs.detach()
        n_loss = int(seed_actions.shape[0] * seed_actions.shape[1])  # loss = costs.mean()
        weights = torch.full(tuple(seed_costs.shape), 1.0 / n_loss, device=seed_actions.device)
        for _ in range(self.gd_steps):
            optimizer.zero_grad(set_to_none=True)
            torch.cuda.synchronize(self.device)
            t0 = time.perf_counter()
            costs, grad = rt.model_cost_grad(emb, goal_emb, params.detach(), history_size=hs, cost_weights=weights)
            loss = costs.mean()
            torch.cuda.synchronize(self.device)
            forward_times.append((time.perf_counter() - t0) * 1000.0)
            evals += refine_width
            if not torch.isfinite(costs).all() or not torch.isfinite(loss):
                nan_or_inf_count += int((~torch.isfinite(costs)).sum().item())
                nan_or_inf_count += int(not bool(torch.isfinite(loss).item()))
                break
            if not torch.isfinite(grad).all():
                nan_or_inf_count += int((~torch.isfinite(grad)).sum().item())
                break
            params.grad = grad.to(params.dtype)
            grad_norms = params.grad.detach().flatten(start_dim=2).norm(dim=2)
            grad_norm_values.extend(grad_norms.cpu().flatten().tolist())
            grad_norm_max = max(grad_norm_max, float(grad_norms.max().item()))
            before = params.detach().clone()
            previous_costs = current_costs.detach().clone()
            optimizer.step()
            update = params.detach().clone() - before
            best_actions, best_costs = before, previous_costs
            for factor in factors:
                candidate_actions = before + factor * update
                with torch.no_grad():
                    candidate_costs = rt.model_cost(emb, goal_emb, candidate_actions, history_size=hs)
                evals += refine_width
                finite = torch.isfinite(candidate_costs)
                if not bool(finite.all().item()):
                    nan_or_inf_count += int((~finite).sum().item())
                improved = finite & (candidate_costs < best_costs)
                best_actions = torch.where(improved[..., None, None], candidate_actions, best_actions)
                best_costs = torch.where(improved, candidate_costs, best_costs)
            accepted_any |= best_costs < previous_costs
            current_costs = best_costs.detach()
            with torch.no_grad():
                params.copy_(best_actions)
            final_actions = params.detach().clone()
            final_costs = current_costs
        final_accept = torch.isfinite(final_costs) & (final_costs < seed_costs)
        accepted_actions = torch.where(final_accept[..., None, None], final_actions, seed_actions.detach())
        accepted_costs = torch.where(final_accept, final_costs, seed_costs.detach())
        candidate_count = int(seed_actions.shape[0] * seed_actions.shape[1])
        accept_count = int(final_accept.sum().item())
        cost_delta = (accepted_costs - seed_costs.detach()).detach()
        summary = {
            "gd_seed_solver": self.gd_seed_solver, "gd_seed_source": self.gd_seed_source,
            "gd_refine_topk": self.gd_refine_topk, "gd_steps": self.gd_steps, "gd_lr": self.gd_lr,
            "gd_compile_cost": self.gd_compile_cost,
            "gd_forward_time_ms_mean": sum(forward_times) / len(forward_times) if forward_times else 0.0,
            "gd_grad_norm_mean": sum(grad_norm_values) / len(grad_norm_values) if grad_norm_values else 0.0,
            "gd_grad_norm_max": grad_norm_max,
            "gd_action_saturation_rate": self._action_saturation_rate(accepted_actions),
            "gd_backward_time_ms_mean": 0.0,
            "gd_peak_memory_mb": torch.cuda.max_memory_allocated(self.device) / (1024.0 * 1024.0),
            "gd_cost_delta_mean": float(cost_delta.mean().item()),
            "gd_accept_rate": accept_count / candidate_count if candidate_count else 0.0,
            "gd_accept_count": accept_count, "gd_candidate_count": candidate_count,
            "gd_step_accept_rate": float(accepted_any.float().mean().item()) if accepted_any.numel() else 0.0,
            "gd_nan_or_inf_count": nan_or_inf_count, "gd_model_cost_evals": evals,
        }
        return accepted_actions.detach(), accepted_costs.detach(), summary

    @staticmethod
    def _combine_gd_summaries(summaries: list[dict[str, Any]]) -> dict[str, Any]:
        """``_combine_gd_summaries`` (``cem_gd.py:606-657``): per-batch summaries merged."""
        if not summaries:
            return {}

        def mean_field(key):
            values = [float(s[key]) for s in summaries if isinstance(s.get(key), (int, float))]
            return sum(values) / len(values) if values else None

        candidate_count = sum(int(s.get("gd_candidate_count", 0)) for s in summaries)
        accept_count = sum(int(s.get("gd_accept_count", 0)) for s in summaries)
        cost_delta_total = sum(float(s.get("gd_cost_delta_mean", 0.0)) * int(s.get("gd_candidate_count", 0))
                               for s in summaries)
        peaks = [float(s["gd_peak_memory_mb"]) for s in summaries
                 if isinstance(s.get("gd_peak_memory_mb"), (int, float))]
        first = summaries[0]
        return {
            "gd_seed_solver": first.get("gd_seed_solver"), "gd_seed_source": first.get("gd_seed_source"),
            "gd_refine_topk": first.get("gd_refine_topk"), "gd_steps": first.get("gd_steps"),
            "gd_lr": first.get("gd_lr"), "gd_compile_cost": first.get("gd_compile_cost"),
            "gd_forward_time_ms_mean": mean_field("gd_forward_time_ms_mean"),
            "gd_grad_norm_mean": mean_field("gd_grad_norm_mean"),
            "gd_grad_norm_max": max(float(s.get("gd_grad_norm_max", 0.0)) for s in summaries),
            "gd_action_saturation_rate": mean_field("gd_action_saturation_rate"),
            "gd_backward_time_ms_mean": mean_field("gd_backward_time_ms_mean"),
            "gd_peak_memory_mb": max(peaks) if peaks else None,
            "gd_cost_delta_mean": cost_delta_total / candidate_count if candidate_count else 0.0,
            "gd_accept_rate": accept_count / candidate_count if candidate_count else 0.0,
            "gd_accept_count": accept_count, "gd_candidate_count": candidate_count,
            "gd_nan_or_inf_count": sum(int(s.get("gd_nan_or_inf_count", 0)) for s in summaries),
            "gd_model_cost_evals": max(int(s.get("gd_model_cost_evals", 0)) for s in summaries),
        }

    def solve(self, info_dict: dict, init_action: torch.Tensor | None = None) -> dict[str, Any]:
        """``CEMGDSolver.solve`` (``cem_gd.py:660-711``)."""
        if self.model is None:
            raise RuntimeError("CEMGDSolver.solve requires a model")
        outputs: dict[str, Any] = {"costs": [], "mean": [], "var": []}
        total_envs = len(next(iter(info_dict.values())))
        with torch.inference_mode():
            init_action = prepare_init_action(self.model, info_dict, init_action, self.horizon, n_envs=total_envs,
                                              action_dim=self.action_dim)
            mean, var = self.init_action_distrib(total_envs, init_action)
            mean = mean.to(self.device)
            var = var.to(self.device)
            emb, goal = self._cost_embeddings(info_dict, total_envs)
            _, std, _, tr = self._plan(info_dict, mean, var, trace=True, emb_goal=(emb, goal))
        # Clone out of inference mode: the refinement needs ordinary tensors.
        emb, goal = emb.detach().clone(), goal.detach().clone()
        last = self.n_steps - 1
        k = self.gd_refine_topk
        if self.gd_seed_source == "mean":
            seed_actions = tr["mean"][last].detach().clone().unsqueeze(1)
            seed_costs = self.runtime.model_cost(emb, goal, seed_actions, history_size=self.history_size)
        else:
            n = tr["counts"][last]
            cand = tr["candidates"][last][:, :n]
            idx = tr["topk_idx"][last][:, :k].long()
            seed_actions = torch.gather(cand, 1, idx[:, :, None, None].expand(-1, -1, cand.shape[2], cand.shape[3]))
            seed_actions = seed_actions.detach().clone()
            seed_costs = tr["topk_val"][last][:, :k].detach().clone()
        final_var = std.detach().clone()
        final_actions = torch.empty(total_envs, self.horizon, self.action_dim, device=self.device, dtype=self.dtype)
        summaries = []
        for start in range(0, total_envs, self.batch_size):
            end = min(start + self.batch_size, total_envs)
            refined, refined_costs, summary = self._refine_seed_actions(
                seed_actions[start:end], seed_costs[start:end], emb[start:end], goal[start:end])
            summaries.append(summary)
            best_costs, best_idx = torch.min(refined_costs, dim=1)
            final_actions[start:end] = refined[torch.arange(end - start, device=self.device), best_idx]
            outputs["costs"].extend(best_costs.detach().cpu().tolist())
        self.runtime.sync()
        outputs["actions"] = final_actions.detach().cpu()
        outputs["mean"] = [final_actions.detach().cpu()]
        outputs["var"] = [final_var.detach().cpu()]
        gd_summary = self._combine_gd_summaries(summaries)
        gd_summary["gd_seed_model_cost_evals"] = sum(self.sample_counts()) + (1 if self.gd_seed_source == "mean" else 0)
        outputs["gd_summary"] = gd_summary
        return outputs


def run_static_icem_chain(model, emb: torch.Tensor, goal_emb: torch.Tensor, mean: torch.Tensor, var: torch.Tensor,
                          noise_steps: Sequence[torch.Tensor], *, topk: int, elite_retention: int = 0,
                          momentum_alpha: float = 0.0, return_best_elite: bool = False,
                          action_low: Optional[torch.Tensor] = None, action_high: Optional[torch.Tensor] = None,
                          history_size: int = 3):
    """Reference ``run_static_icem_chain`` (``lewm/solvers/icem_static_compile.py:61-114``) as one device plan.

    ``model`` is a reference ``JEPA`` (its predictor replaces ``cost_fn``) or a
    ``Runtime``. Each noise step is (B, S_i, T, A) post-coloring noise.
    Returns (actions_or_best_elite, std, final_cost) on the device.
    """
    rt = _runtime(model, mean.device if mean.is_cuda else "cuda")
    noise_steps = list(noise_steps)
    if not noise_steps:
        # The reference's loop body never runs and its `assert final_cost is not None` fails.
        raise AssertionError("run_static_icem_chain needs at least one noise step")
    counts = [int(n.shape[1]) for n in noise_steps]
    # Any list of noise tensors: the plan takes their sample counts as given.
    opts = PlanOptions(num_samples=max(counts), topk=topk, n_steps=len(counts), elite_retention=elite_retention,
                       momentum_alpha=momentum_alpha, return_best_elite=return_best_elite,
                       clip_actions=action_low is not None and action_high is not None, history_size=history_size,
                       counts=counts)
    actions, std, fcost, _ = rt.plan(opts, emb, goal_emb, mean, var, noise_steps=noise_steps,
                                     action_low=action_low, action_high=action_high)
    return actions, std, fcost


class _ModelCostWithGrad(torch.autograd.Function):
    """Model costs whose gradient with respect to the action candidates is the device's float32
    reverse pass (``lewm_model_cost_grad``). Candidates are independent, so the pass computes
    every candidate's d cost_c / d cand_c once in the forward and the backward only scales it
    by the incoming d loss / d cost_c."""

    @staticmethod
    def forward(ctx, candidates, rt, emb, goal_emb, history_size):
        costs, grad = rt.model_cost_grad(emb, goal_emb, candidates, history_size=history_size)
        ctx.save_for_backward(grad)
        ctx.cand_meta = (candidates.dtype, candidates.device)
        return costs

    @staticmethod
    def backward(ctx, grad_costs):
        (grad,) = ctx.saved_tensors
        dtype, device = ctx.cand_meta
        g = grad * grad_costs.to(grad.dtype)[..., None, None]
        return g.to(device=device, dtype=dtype), None, None, None, None


class B200ModelCost:
    """``JEPA.get_cost_from_embeddings`` on the B200 kernels (reference ``lewm/jepa.py:302-317``).

    Differentiable with respect to ``action_candidates``: under grad mode with candidates that
    require grad (CEM-GD's refinement, ``lewm/solvers/cem_gd.py:459-606``) the costs come from
    the float32 forward that records the reverse pass, and ``backward`` returns the device
    gradient. The embeddings and goal are constants there (they come from the frozen encoder)."""

    def __init__(self, model, device="cuda"):
        self.model = model
        self.device = torch.device(device)

    @property
    def runtime(self) -> Runtime:
        return _runtime(self.model, self.device)

    def get_cost_from_embeddings(self, emb: torch.Tensor, goal_emb: torch.Tensor, action_candidates: torch.Tensor,
                                 history_size: int = 3) -> torch.Tensor:
        rt = self.runtime
        if torch.is_grad_enabled() and action_candidates.requires_grad:
            if emb.requires_grad or goal_emb.requires_grad:
                raise NotImplementedError("the B200 model cost differentiates with respect to the action candidates "
                                          "only; detach emb / goal_emb")
            return _ModelCostWithGrad.apply(action_candidates, rt, emb.detach(), goal_emb.detach(), int(history_size))
        return rt.model_cost(emb, goal_emb, action_candidates, history_size=history_size)

    __call__ = get_cost_from_embeddings


def install_model_cost(model, device="cuda"):
    """Route ``model.get_cost_from_embeddings`` (and so the reference's compile_cost
    ``JEPA.get_cost`` path, ``lewm/jepa.py:357-359``) through the B200 kernels."""
    mc = B200ModelCost(model, device)
    model.get_cost_from_embeddings = mc.get_cost_from_embeddings
    return mc
