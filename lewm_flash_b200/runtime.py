"""Device runtime: one ``lewm_ctx`` (packed weights + workspace) per model and GPU.

Thin torch-facing wrapper over the C ABI in ``include/lewm_b200.h``. Tensors
passed in are made contiguous float32 on the context's GPU; results are new
device tensors. Every call is asynchronous on the current torch CUDA stream.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Dict, List, Mapping, Optional, Sequence

import numpy as np
import torch

from . import _lib
from .model import ModelDesc, param_shapes


def _dev_index(device) -> int:
    d = torch.device(device)
    if d.type != "cuda":
        raise ValueError(f"the B200 runtime needs a CUDA device, got {d}")
    return d.index if d.index is not None else torch.cuda.current_device()


def pack_canonical(desc: ModelDesc, state_dict: Mapping[str, np.ndarray]) -> np.ndarray:
    """Concatenate the state dict in the order ``lewm_create`` reads it."""
    parts = []
    for name, shape in param_shapes(desc).items():
        arr = np.asarray(state_dict[name], dtype=np.float32)
        if tuple(arr.shape) != tuple(shape):
            raise ValueError(f"{name}: expected {shape}, got {arr.shape}")
        parts.append(arr.reshape(-1))
    return np.ascontiguousarray(np.concatenate(parts), dtype=np.float32)


def desc_to_c(desc: ModelDesc) -> _lib.ModelDescC:
    return _lib.ModelDescC(desc.dim, desc.depth, desc.heads, desc.dim_head, desc.mlp_dim, desc.action_dim,
                           desc.smoothed_dim, desc.embed_hidden, desc.num_frames, desc.pred_proj_hidden,
                           _lib.NORM_CODE[desc.pred_proj_norm])


@dataclass
class PlanOptions:
    """iCEM options in ``ICEMSolver`` terms (reference ``lewm/solvers/icem.py:258-322``)."""

    num_samples: int = 300
    topk: int = 30
    n_steps: int = 30
    sample_decay: float = 1.0
    sample_count_bucket_size: int = 0
    elite_retention: int = 0
    beta: float = 0.0
    time_axis: str = "raw"
    action_block: int = 1
    momentum_alpha: float = 0.0
    return_best_elite: bool = False
    clip_actions: bool = False
    history_size: int = 3
    seed: int = 1234
    # Explicit per-iteration sample counts (one per iteration, each in [topk, num_samples]),
    # e.g. the sample counts of an arbitrary list of injected noise tensors; None follows
    # the ICEMSolver schedule of (num_samples, sample_decay, sample_count_bucket_size).
    counts: Optional[List[int]] = None

    def to_c(self, n_envs: int, horizon: int, history: int, plan_index: int = 0) -> _lib.PlanDescC:
        if self.time_axis not in ("block", "raw"):
            raise ValueError(f"colored noise time_axis must be 'block' or 'raw', got {self.time_axis!r}")
        counts_arr = None
        if self.counts is not None:
            if len(self.counts) != self.n_steps:
                raise ValueError(f"counts has {len(self.counts)} entries, n_steps is {self.n_steps}")
            counts_arr = (C.c_int32 * len(self.counts))(*[int(v) for v in self.counts])
        pd = _lib.PlanDescC(
            int(n_envs), int(horizon), int(history), int(self.history_size), int(self.num_samples), int(self.topk),
            int(self.n_steps), float(self.sample_decay), int(self.sample_count_bucket_size),
            int(self.elite_retention), float(self.beta), 1 if self.time_axis == "raw" else 0, int(self.action_block),
            float(self.momentum_alpha), int(bool(self.return_best_elite)), int(bool(self.clip_actions)),
            int(self.seed) & 0xFFFFFFFFFFFFFFFF, int(plan_index) & 0xFFFFFFFFFFFFFFFF,
            C.cast(counts_arr, C.POINTER(C.c_int32)) if counts_arr is not None else None)
        pd._counts_keep = counts_arr  # the struct holds a raw pointer into this array
        return pd


def sample_counts(opts: PlanOptions, horizon: int = 5, n_envs: int = 1) -> List[int]:
    """Per-iteration sample counts from the C ABI (``lewm_sample_counts``)."""
    pd = opts.to_c(n_envs, horizon, 1)
    out = (C.c_int32 * max(opts.n_steps, 1))()
    evals = C.c_int64(0)
    _lib.check(_lib.lib().lewm_sample_counts(C.byref(pd), out, opts.n_steps, C.byref(evals)))
    return [int(v) for v in out[: opts.n_steps]]


def coloring_matrix(n: int, beta: float) -> np.ndarray:
    out = np.empty((n, n), dtype=np.float64)
    _lib.check(_lib.lib().lewm_coloring_matrix(int(n), float(beta), out.ctypes.data))
    return out


def _f32(t: torch.Tensor, device: torch.device) -> torch.Tensor:
    return t.to(device=device, dtype=torch.float32).contiguous()


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else C.c_void_p(t.data_ptr())


AUTOCAST_MODES = {"none": 0, "bf16": 1}  # LEWM_AUTOCAST_NONE / LEWM_AUTOCAST_BF16


class Runtime:
    """One packed LeWM predictor on one GPU."""

    def __init__(self, desc: ModelDesc, state_dict: Mapping[str, np.ndarray], device="cuda",
                 model_cost_autocast: str = "bf16"):
        self.desc = desc
        self.device = torch.device("cuda", _dev_index(device))
        flat = pack_canonical(desc, state_dict)
        lib = _lib.lib()
        cd = desc_to_c(desc)
        want = lib.lewm_weight_count(C.byref(cd))
        if want == 0:
            _lib.check(2, None)
        if want != flat.size:
            raise ValueError(f"weight count mismatch: C ABI wants {want}, packed {flat.size}")
        h = C.c_void_p()
        _lib.check(lib.lewm_create(C.byref(h), C.byref(cd), flat.ctypes.data, flat.size, self.device.index), None)
        self._h = h
        self.plans_issued = 0
        self._autocast = "bf16"
        self.set_model_cost_autocast(model_cost_autocast)

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.lib().lewm_destroy(self._h)
            self._h = None

    def __del__(self):  # pragma: no cover - interpreter teardown order
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def _stream(self):
        return C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def _check(self, status: int) -> None:
        _lib.check(status, self._h)

    def sync(self) -> None:
        """Synchronize; raise LewmError(LEWM_DEVICE_TIMEOUT) if a device wait expired, or
        LewmError(LEWM_NUMERIC_NAN) if a plan since the last sync produced a NaN final cost."""
        self._check(_lib.lib().lewm_sync_status(self._h, self._stream()))

    def set_wait_limit(self, limit_ns: int) -> None:
        """Time limit of every bounded device-side wait of later launches (0: the 2 s default)."""
        self._check(_lib.lib().lewm_set_wait_limit(self._h, int(limit_ns)))

    def wait_selftest(self) -> None:
        """Enqueue one bounded device wait that can never complete (``lewm_wait_selftest``);
        the next ``sync`` raises LEWM_DEVICE_TIMEOUT."""
        self._check(_lib.lib().lewm_wait_selftest(self._h, self._stream()))

    def set_model_cost_autocast(self, mode: str = "none") -> "Runtime":
        """Arithmetic of later model costs and plans (reference ``JEPA.set_model_cost_autocast``,
        ``lewm/jepa.py:65-69``): "bf16" runs the tensor-core kernels, "none" float32 throughout."""
        if mode not in AUTOCAST_MODES:
            raise ValueError(f"Unsupported model_cost_autocast mode: {mode!r}")
        if mode != self._autocast:
            self._check(_lib.lib().lewm_set_model_cost_autocast(self._h, AUTOCAST_MODES[mode]))
            self._autocast = mode
        return self

    def model_cost_autocast_mode(self) -> str:
        return self._autocast

    # ------------------------------------------------------------------ model cost
    def model_cost(self, emb: torch.Tensor, goal_emb: torch.Tensor, candidates: torch.Tensor,
                   history_size: int = 3) -> torch.Tensor:
        """``JEPA.get_cost_from_embeddings`` semantics (reference ``lewm/jepa.py:302-317``)."""
        args = self._cost_args(emb, goal_emb, candidates)
        out = torch.empty(args["B"], args["S"], device=self.device, dtype=torch.float32)
        self._check(_lib.lib().lewm_model_cost(self._h, _ptr(args["e"]), args["emb_ps"], args["H"], _ptr(args["g"]),
                                               args["goal_ps"], _ptr(args["cand"]), args["B"], args["S"], args["T"],
                                               int(history_size), _ptr(out), self._stream()))
        return out

    def model_cost_grad(self, emb: torch.Tensor, goal_emb: torch.Tensor, candidates: torch.Tensor,
                        history_size: int = 3, cost_weights: Optional[torch.Tensor] = None):
        """Costs (B,S) and d(sum_c w_c cost_c) / d candidates (B,S,T,A), float32 forward and
        reverse pass (``lewm_model_cost_grad``): the gradient CEM-GD steps on
        (reference ``lewm/solvers/cem_gd.py:459-606``). ``cost_weights`` (B,S), default ones."""
        args = self._cost_args(emb, goal_emb, candidates)
        B, S = args["B"], args["S"]
        out = torch.empty(B, S, device=self.device, dtype=torch.float32)
        grad = torch.empty_like(args["cand"])
        w = None if cost_weights is None else _f32(cost_weights.expand(B, S), self.device)
        self._check(_lib.lib().lewm_model_cost_grad(
            self._h, _ptr(args["e"]), args["emb_ps"], args["H"], _ptr(args["g"]), args["goal_ps"], _ptr(args["cand"]),
            B, S, args["T"], int(history_size), _ptr(w), _ptr(out), _ptr(grad), self._stream()))
        return out, grad

    def _cost_args(self, emb: torch.Tensor, goal_emb: torch.Tensor, candidates: torch.Tensor) -> dict:
        dev = self.device
        cand = _f32(candidates, dev)
        if cand.ndim != 4:
            raise ValueError(f"action_candidates must be (B,S,T,A), got {tuple(cand.shape)}")
        B, S, T, A = cand.shape
        if A != self.desc.action_dim:
            raise ValueError(f"action dim {A} != model action_dim {self.desc.action_dim}")
        if emb.ndim == 3:
            e, emb_ps = _f32(emb, dev), 0
            if e.shape[0] != B:
                e = e.expand(B, *e.shape[1:]).contiguous()
        elif emb.ndim == 4:
            e, emb_ps = _f32(emb.expand(B, S, *emb.shape[2:]), dev), 1
        else:
            raise ValueError(f"Expected emb rank 3 or 4, got shape {tuple(emb.shape)}")
        H = int(e.shape[-2])
        if H > T:
            raise ValueError(f"history {H} exceeds horizon {T}")
        if e.shape[-1] != self.desc.dim or goal_emb.shape[-1] != self.desc.dim:
            raise ValueError(f"emb / goal_emb width must be the model dim {self.desc.dim}, got "
                             f"{e.shape[-1]} / {goal_emb.shape[-1]}")
        g = goal_emb[..., -1, :]
        if g.ndim == 2:
            g, goal_ps = _f32(g.expand(B, g.shape[-1]), dev), 0
        elif g.ndim == 3:
            g, goal_ps = _f32(g.expand(B, S, g.shape[-1]), dev), 1
        else:
            raise ValueError(f"goal_emb must be rank 3 or 4, got {tuple(goal_emb.shape)}")
        return {"e": e, "emb_ps": emb_ps, "H": H, "g": g, "goal_ps": goal_ps, "cand": cand, "B": B, "S": S, "T": T}

    # ------------------------------------------------------------------ full plan
    def _check_plan_tensors(self, e: torch.Tensor, g: torch.Tensor, m: torch.Tensor, s: torch.Tensor) -> None:
        """The kernels read every tensor at the model's widths: reject any other shape."""
        if m.ndim != 3 or m.shape[2] != self.desc.action_dim:
            raise ValueError(f"mean must be (B,T,{self.desc.action_dim}), got {tuple(m.shape)}")
        if tuple(s.shape) != tuple(m.shape):
            raise ValueError(f"std shape {tuple(s.shape)} != mean shape {tuple(m.shape)}")
        B = m.shape[0]
        if e.ndim != 3 or e.shape[0] != B or e.shape[2] != self.desc.dim:
            raise ValueError(f"emb must be (B,H,D) with B={B}, D={self.desc.dim}, got {tuple(e.shape)}")
        if tuple(g.shape) != (B, self.desc.dim):
            raise ValueError(f"goal_emb must give (B,D) rows, got {tuple(g.shape)}")

    def plan(self, opts: PlanOptions, emb: torch.Tensor, goal_emb: torch.Tensor, mean: torch.Tensor,
             std: torch.Tensor, noise_steps: Optional[Sequence[torch.Tensor]] = None,
             action_low: Optional[torch.Tensor] = None, action_high: Optional[torch.Tensor] = None,
             trace: bool = False, plan_index: Optional[int] = None):
        """One iCEM solve for every env at once. Returns (actions, std, final_cost, trace|None)."""
        dev = self.device
        m = _f32(mean, dev)
        s = _f32(std, dev)
        e = _f32(emb, dev)
        g = _f32(goal_emb[..., -1, :] if goal_emb.ndim == 3 else goal_emb, dev)
        self._check_plan_tensors(e, g, m, s)
        B, T, A = m.shape
        if plan_index is None:
            plan_index = self.plans_issued
        self.plans_issued += 1
        pd = opts.to_c(B, T, int(e.shape[1]), plan_index)
        counts = sample_counts(opts, T, B) if noise_steps is not None or trace else None
        keep = []
        noise_arr = None
        if noise_steps is not None:
            if len(noise_steps) != opts.n_steps:
                raise ValueError(f"need {opts.n_steps} noise steps, got {len(noise_steps)}")
            ptrs = []
            for i, (n, c) in enumerate(zip(noise_steps, counts)):
                nt = _f32(n, dev)
                if tuple(nt.shape) != (B, c, T, A):
                    raise ValueError(f"noise step {i} must be {(B, c, T, A)}, got {tuple(nt.shape)}")
                keep.append(nt)
                ptrs.append(nt.data_ptr())
            noise_arr = (C.c_void_p * len(ptrs))(*ptrs)
        lo = hi = None
        if opts.clip_actions:
            if action_low is None or action_high is None:
                raise ValueError("clip_actions needs action_low and action_high")
            lo, hi = _f32(action_low.reshape(-1), dev), _f32(action_high.reshape(-1), dev)
            if lo.numel() != A or hi.numel() != A:
                raise ValueError(f"action_low / action_high need {A} values")
        actions = torch.empty(B, T, A, device=dev)
        std_out = torch.empty(B, T, A, device=dev)
        fcost = torch.empty(B, device=dev)
        tr = None
        trc = None
        if trace:
            S, k, n = opts.num_samples, opts.topk, opts.n_steps
            tr = {
                "costs": torch.full((n, B, S), float("nan"), device=dev),
                "topk_idx": torch.empty(n, B, k, device=dev, dtype=torch.int32),
                "topk_val": torch.empty(n, B, k, device=dev),
                "mean": torch.empty(n, B, T, A, device=dev),
                "std": torch.empty(n, B, T, A, device=dev),
                "candidates": torch.full((n, B, S, T, A), float("nan"), device=dev),
                "counts": counts,
            }
            trc = _lib.PlanTraceC(*(C.c_void_p(tr[kk].data_ptr()) for kk in
                                    ("costs", "topk_idx", "topk_val", "mean", "std", "candidates")))
        self._check(_lib.lib().lewm_plan(
            self._h, C.byref(pd), _ptr(e), _ptr(g), _ptr(m), _ptr(s), noise_arr, _ptr(lo), _ptr(hi), _ptr(actions),
            _ptr(std_out), _ptr(fcost), C.byref(trc) if trc is not None else None, self._stream()))
        del keep
        return actions, std_out, fcost, tr

    def profile_plan(self, opts: PlanOptions, emb: torch.Tensor, goal_emb: torch.Tensor, mean: torch.Tensor,
                     std: torch.Tensor, plan_index: int = 0) -> dict:
        """Per-kernel-class device ms / FLOPs / launches of one plan (``lewm_profile_plan``)."""
        dev = self.device
        m, s = _f32(mean, dev), _f32(std, dev)
        e = _f32(emb, dev)
        g = _f32(goal_emb[..., -1, :] if goal_emb.ndim == 3 else goal_emb, dev)
        self._check_plan_tensors(e, g, m, s)
        B, T, _ = m.shape
        pd = opts.to_c(B, T, int(e.shape[1]), plan_index)
        n = len(_lib.KERNEL_CLASSES)
        ms = (C.c_double * n)()
        fl = (C.c_double * n)()
        la = (C.c_int32 * n)()
        self._check(_lib.lib().lewm_profile_plan(self._h, C.byref(pd), _ptr(e), _ptr(g), _ptr(m), _ptr(s), ms, fl, la,
                                                 self._stream()))
        classes = {name: {"ms": ms[i], "flops": fl[i], "launches": int(la[i])}
                   for i, name in enumerate(_lib.KERNEL_CLASSES) if la[i]}
        return {"classes": classes, "launches": int(sum(la))}

    # ------------------------------------------------------------------ pieces
    def topk_refit(self, costs: torch.Tensor, candidates: torch.Tensor, mean: torch.Tensor, std: torch.Tensor,
                   topk: int, momentum_alpha: float = 0.0):
        dev = self.device
        c = _f32(costs, dev)
        cand = _f32(candidates, dev)
        if cand.ndim != 4:
            raise ValueError(f"candidates must be (B,S,T,A), got {tuple(cand.shape)}")
        B, S, T, A = cand.shape
        if tuple(c.shape) != (B, S):
            raise ValueError(f"costs must be {(B, S)}, got {tuple(c.shape)}")
        if tuple(mean.shape) != (B, T, A) or tuple(std.shape) != (B, T, A):
            raise ValueError(f"mean / std must be {(B, T, A)}, got {tuple(mean.shape)} / {tuple(std.shape)}")
        m = _f32(mean, dev).clone()
        s = _f32(std, dev).clone()
        idx = torch.empty(B, topk, device=dev, dtype=torch.int32)
        val = torch.empty(B, topk, device=dev)
        best = torch.empty(B, T, A, device=dev)
        fc = torch.empty(B, device=dev)
        self._check(_lib.lib().lewm_topk_refit(self._h, _ptr(c), _ptr(cand), B, S, T, A, int(topk),
                                               float(momentum_alpha), _ptr(m), _ptr(s), _ptr(idx), _ptr(val),
                                               _ptr(best), _ptr(fc), self._stream()))
        return {"topk_idx": idx, "topk_val": val, "mean": m, "std": s, "best": best, "final_cost": fc}

    def sample_candidates(self, opts: PlanOptions, n_samples: int, iteration: int, mean: torch.Tensor,
                          std: torch.Tensor, injected_noise: Optional[torch.Tensor] = None,
                          action_low: Optional[torch.Tensor] = None, action_high: Optional[torch.Tensor] = None,
                          plan_index: int = 0) -> torch.Tensor:
        dev = self.device
        m = _f32(mean, dev)
        s = _f32(std, dev)
        B, T, A = m.shape
        # The kernel reads and writes the model's action dim per step: every tensor must match it.
        if A != self.desc.action_dim:
            raise ValueError(f"action dim {A} != model action_dim {self.desc.action_dim}")
        if tuple(s.shape) != (B, T, A):
            raise ValueError(f"std shape {tuple(s.shape)} != mean shape {(B, T, A)}")
        if injected_noise is not None and tuple(injected_noise.shape) != (B, n_samples, T, A):
            raise ValueError(f"injected_noise shape {tuple(injected_noise.shape)} != {(B, n_samples, T, A)}")
        pd = opts.to_c(B, T, 1, plan_index)
        nz = None if injected_noise is None else _f32(injected_noise, dev)
        lo = hi = None
        if opts.clip_actions:
            lo, hi = _f32(action_low.reshape(-1), dev), _f32(action_high.reshape(-1), dev)
        out = torch.empty(B, n_samples, T, A, device=dev)
        self._check(_lib.lib().lewm_sample_candidates(self._h, C.byref(pd), int(n_samples), int(iteration), _ptr(m),
                                                      _ptr(s), _ptr(nz), _ptr(lo), _ptr(hi), _ptr(out),
                                                      self._stream()))
        return out
