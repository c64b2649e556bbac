"""ORACLE (test infrastructure only) -- numpy restatement of the iCEM chain.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import this module; the product package never does.

Restated reference functions:

* ``ICEMSolver.sample_count_for_step`` / ``sample_counts`` --
  reference ``lewm/solvers/icem.py:377-394``
* ``make_colored_noise`` / ``_colored_noise_along_time`` /
  ``_normalize_colored_noise`` -- ``lewm/solvers/icem.py:148-250`` (the white
  noise is an input here: the reference draws it from a torch generator)
* ``run_static_icem_chain`` with ``_inject_retained_elites_static`` and
  ``_gather_topk_candidates`` -- ``lewm/solvers/icem_static_compile.py:28-114``
  (bit-identical to ``ICEMSolver.solve`` given the same noise)
* ``init_action_distrib`` / ``prepare_init_action`` --
  ``lewm/solvers/icem.py:396-419``, ``lewm/solvers/cem_exact.py:13-51``

``torch.topk`` leaves the order of equal costs unspecified; this oracle breaks
ties by the lower candidate index (stable sort), the documented order of the
CUDA top-k.

``philox4x32_10`` / ``philox_normal`` restate the counter-based generator the
CUDA sampler uses in its non-injected mode (Salmon et al., "Parallel random
numbers: as easy as 1, 2, 3", SC'11; Box-Muller transform) so tests can check
the device stream value by value.
"""

from __future__ import annotations

import math
from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np

F32 = np.float32
COLORED_NOISE_BETA = {"none": 0.0, "pink": 1.0, "brown": 2.0}


# --------------------------------------------------------------------------- schedule
def sample_count_for_step(step, num_samples, topk, sample_decay=1.0, bucket=0):
    """``ICEMSolver.sample_count_for_step`` (``lewm/solvers/icem.py:377-388``)."""
    if sample_decay == 1.0:
        return num_samples
    decayed = int(math.ceil(num_samples * (sample_decay ** (-step))))
    count = max(decayed, min(num_samples, 2 * topk))
    if bucket > 0:
        count = min(num_samples, int(math.ceil(count / bucket)) * bucket)
    return count


def sample_counts(n_steps, num_samples, topk, sample_decay=1.0, bucket=0) -> List[int]:
    return [sample_count_for_step(s, num_samples, topk, sample_decay, bucket) for s in range(n_steps)]


# --------------------------------------------------------------------------- colored noise
def _color_along_time(white, beta):
    """``_colored_noise_along_time`` after the randn draw (``lewm/solvers/icem.py:173-182``)."""
    n = white.shape[-1]
    if beta <= 0.0 or n <= 1:
        return white.astype(F32)
    freqs = np.fft.rfftfreq(n).astype(F32)
    freqs[0] = 1.0
    scale = np.power(freqs, F32(-beta / 2.0)).astype(F32)
    if scale.size > 1:
        scale[0] = scale[1]
    colored = np.fft.irfft(np.fft.rfft(white.astype(np.float64), axis=-1) * scale, n=n, axis=-1)
    std = colored.std(axis=-1, ddof=1, keepdims=True)
    return (colored / np.maximum(std, 1e-8)).astype(F32)


def white_noise_shape(batch, n_samples, horizon, action_dim, beta, action_block=1, time_axis="raw"):
    """Shape of the ``torch.randn`` draw ``make_colored_noise`` makes."""
    if beta <= 0.0:
        return (batch, n_samples, horizon, action_dim)
    if time_axis == "raw" and action_block > 1:
        return (batch, n_samples, action_dim // action_block, horizon * action_block)
    return (batch, n_samples, action_dim, horizon)


def color_white_noise(white, horizon, action_dim, beta, action_block=1, time_axis="raw"):
    """``make_colored_noise`` given its white draw (``lewm/solvers/icem.py:185-250``)."""
    if time_axis not in ("block", "raw"):
        raise ValueError(f"colored noise time_axis must be 'block' or 'raw', got {time_axis!r}")
    B, S = white.shape[:2]
    if beta <= 0.0:
        return white.astype(F32)
    if time_axis == "raw" and action_block > 1:
        if action_dim % action_block:
            raise ValueError(f"action_dim={action_dim} is not divisible by action_block={action_block}")
        raw = _color_along_time(white, beta)
        return np.ascontiguousarray(raw.swapaxes(-1, -2)).reshape(B, S, horizon, action_dim)
    blk = _color_along_time(white, beta)
    return np.ascontiguousarray(blk.swapaxes(-1, -2))


def coloring_matrix(n, beta):
    """Real n x n matrix W with ``irfft(rfft(x) * scale) == W @ x`` (float64)."""
    eye = np.eye(n)
    if beta <= 0.0 or n <= 1:
        return eye
    freqs = np.fft.rfftfreq(n)
    freqs[0] = 1.0
    scale = freqs ** (-beta / 2.0)
    if scale.size > 1:
        scale[0] = scale[1]
    return np.fft.irfft(np.fft.rfft(eye, axis=0) * scale[:, None], n=n, axis=0)


# --------------------------------------------------------------------------- init / elites
def init_action_distrib(n_envs, horizon, action_dim, var_scale=1.0, init_action=None):
    """``prepare_init_action`` + ``init_action_distrib``: zero-padded mean, std = var_scale."""
    var = np.full((n_envs, horizon, action_dim), var_scale, dtype=F32)
    mean = np.zeros((n_envs, horizon, action_dim), dtype=F32)
    if init_action is not None:
        n = min(horizon, init_action.shape[1])
        mean[:, :n] = init_action[:, :n]
    return mean, var


def topk_smallest(costs, k):
    """Ascending k smallest with lower-index-first ties; NaN sorts after +inf."""
    key = np.where(np.isnan(costs), np.inf, costs)
    nan_rank = np.isnan(costs).astype(np.int8)
    idx = np.lexsort((np.broadcast_to(np.arange(costs.shape[-1]), costs.shape), key, nan_rank), axis=-1)[..., :k]
    return np.take_along_axis(costs, idx, -1), idx


def refit(elites, mean, var, momentum_alpha=0.0):
    """Elite mean / unbiased std with optional momentum (``lewm/solvers/icem.py:555-563``)."""
    e_mean = elites.mean(axis=1, dtype=np.float64).astype(F32)
    e_std = elites.astype(np.float64).std(axis=1, ddof=1).astype(F32)
    if momentum_alpha:
        a = F32(momentum_alpha)
        return (a * mean + (F32(1) - a) * e_mean).astype(F32), (a * var + (F32(1) - a) * e_std).astype(F32)
    return e_mean, e_std


def run_static_icem_chain(cost_fn: Callable, emb, goal_emb, mean, var, noise_steps: Sequence[np.ndarray], *,
                          topk, elite_retention=0, momentum_alpha=0.0, return_best_elite=False,
                          action_low=None, action_high=None, trace: Optional[list] = None):
    """``run_static_icem_chain`` (``lewm/solvers/icem_static_compile.py:61-114``).

    Returns (actions_or_best_elite, std, final_cost). When ``trace`` is a
    list, one dict per iteration (candidates, costs, topk values/indices,
    mean, std) is appended to it.
    """
    batch_mean = np.asarray(mean, dtype=F32)
    batch_var = np.asarray(var, dtype=F32)
    prev_elites = None
    best_elite = None
    final_cost = None
    for noise in noise_steps:
        noise = np.asarray(noise, dtype=F32)
        sampled = noise * batch_var[:, None] + batch_mean[:, None]
        cand = np.concatenate([batch_mean[:, None], sampled[:, 1:]], axis=1).astype(F32)
        if prev_elites is not None and elite_retention > 0:
            n_inject = min(elite_retention, prev_elites.shape[1], cand.shape[1] - 1)
            if n_inject > 0:
                cand[:, 1:1 + n_inject] = prev_elites[:, :n_inject]
        if action_low is not None and action_high is not None:
            cand = np.clip(cand, action_low, action_high).astype(F32)
        costs = np.asarray(cost_fn(emb, goal_emb, cand), dtype=F32)
        vals, inds = topk_smallest(costs, topk)
        elites = np.take_along_axis(cand, inds[:, :, None, None], axis=1)
        prev_elites = elites
        best_elite = elites[:, 0]
        batch_mean, batch_var = refit(elites, batch_mean, batch_var, momentum_alpha)
        final_cost = vals.mean(axis=1, dtype=np.float64).astype(F32)
        if trace is not None:
            trace.append({"candidates": cand, "costs": costs, "topk_vals": vals, "topk_inds": inds,
                          "mean": batch_mean, "var": batch_var})
    if return_best_elite:
        return best_elite, batch_var, final_cost
    return batch_mean, batch_var, final_cost


# --------------------------------------------------------------------------- Philox4x32-10
_M0, _M1 = 0xD2511F53, 0xCD9E8D57
_W0, _W1 = 0x9E3779B9, 0xBB67AE85
_MASK = 0xFFFFFFFF


def philox4x32_10(ctr, key):
    """Philox4x32 with 10 rounds on uint64 arrays (values < 2**32). ctr: 4 arrays, key: 2 arrays."""
    c0, c1, c2, c3 = (np.asarray(c, dtype=np.uint64) for c in ctr)
    k0, k1 = (np.asarray(k, dtype=np.uint64) for k in key)
    for _ in range(10):
        p0 = c0 * np.uint64(_M0)
        p1 = c2 * np.uint64(_M1)
        hi0, lo0 = p0 >> np.uint64(32), p0 & np.uint64(_MASK)
        hi1, lo1 = p1 >> np.uint64(32), p1 & np.uint64(_MASK)
        c0, c1, c2, c3 = (hi1 ^ c1 ^ k0) & np.uint64(_MASK), lo1, (hi0 ^ c3 ^ k1) & np.uint64(_MASK), lo0
        k0 = (k0 + np.uint64(_W0)) & np.uint64(_MASK)
        k1 = (k1 + np.uint64(_W1)) & np.uint64(_MASK)
    return c0, c1, c2, c3


def philox_normal(n, cand, env, it, seed, plan):
    """Standard normals the CUDA sampler draws for one (plan, iteration, env, candidate).

    Draw ``d`` uses counter (d // 4, cand, env, it) and key (seed, plan);
    each block of 4 uint32 words gives two Box-Muller pairs
    (u1 = (w0 + 1) / 2**32 in (0, 1], u2 = w1 / 2**32 in [0, 1)).
    Computed in float64 (the device uses float32 logf/sqrtf/sincospif).
    """
    nblk = (n + 3) // 4
    blk = np.arange(nblk, dtype=np.uint64)
    z = lambda v: np.full(nblk, v, dtype=np.uint64)
    w = philox4x32_10((blk, z(cand), z(env), z(it)), (z(seed & _MASK), z(plan & _MASK)))
    out = np.empty((nblk, 4), dtype=np.float64)
    for j, (a, b) in enumerate(((w[0], w[1]), (w[2], w[3]))):
        u1 = (a.astype(np.float64) + 1.0) / 4294967296.0
        u2 = b.astype(np.float64) / 4294967296.0
        r = np.sqrt(-2.0 * np.log(u1))
        out[:, 2 * j] = r * np.cos(2.0 * np.pi * u2)
        out[:, 2 * j + 1] = r * np.sin(2.0 * np.pi * u2)
    return out.reshape(-1)[:n]
