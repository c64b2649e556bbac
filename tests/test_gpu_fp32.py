"""The float32 model cost (``model_cost_autocast`` "none", ``LEWM_AUTOCAST_NONE``).

The reference computes its model cost in float32 unless ``JEPA.set_model_cost_autocast``
("bf16", ``lewm/jepa.py:65-86``) is set; cfg1 (plain CEM 300 / 30 / 30) is quoted in
float32. Its exactness gate (``tools/benchmarks/check_lewm_cache_exactness.py``) is
``cost_stats`` (``:224-233``: ``torch.allclose`` at atol = rtol = 1e-5, ``:783-784``), then
``compare_rankings`` (``:236-246``: argmin and top-k indices equal) and, where they differ,
``ranking_drift_diagnostics`` (``:249-305``). The device's float32 path is held to it
through the C ABI:

* model costs of every reference fixture at a device width (Identity, LayerNorm and
  BatchNorm ``pred_proj`` heads, histories 1 and 3, width 384 / 12 layers) within 1e-5,
  and a no-norm head against the oracle;
* teacher-forced on the reference's cfg1 / cfg2 / cfg3 trajectories: the costs of every
  iteration's candidates within 1e-5, the argmin equal, the top-k equal up to the order of
  exactly equal costs or explained by near-ties;
* the full float32 plan on the reference's noise stays on the reference's trajectory (any
  elite change only at a tie below 1e-5 relative) and, where it stays through the last
  iteration, returns the reference's actions and final cost;
* switching between "bf16" and "none" gives each mode's own results, bit for bit.
"""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from lewm_flash_b200.model import ModelDesc, synthetic_state_dict
from lewm_flash_b200.runtime import PlanOptions, Runtime
from oracle import lewm_oracle as lo
from tests.golden_io import MODEL_COST_CASES, desc_of, load, weights_of
from tests.test_gpu_headline import HEADLINE_CASES, _opts, _reference_trajectory, ranking_drift

pytestmark = pytest.mark.gpu
ATOL = RTOL = 1e-5  # cost_stats of check_lewm_cache_exactness.py
TIE_REL = 1e-5      # an elite change of the float32 plan must sit at a gap below this


def _t(x, dev="cuda:0"):
    return torch.as_tensor(np.ascontiguousarray(x), dtype=torch.float32, device=dev)


def cost_stats(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return {"allclose": bool(np.allclose(got, want, rtol=RTOL, atol=ATOL)),
            "max_abs": float(np.abs(got - want).max()),
            "max_rel": float((np.abs(got - want) / np.maximum(np.abs(want), 1e-12)).max())}


@pytest.fixture(scope="module")
def runtimes():
    cache = {}
    yield cache
    for rt in cache.values():
        rt.close()


def _rt(cache, d):
    desc, sd = weights_of(d)
    key = (json.dumps(desc.__dict__, sort_keys=True, default=str), int(d["seed"]))
    if key not in cache:
        cache[key] = Runtime(desc, sd, "cuda:0", model_cost_autocast="none")
    return cache[key], desc, sd


# Fixtures at model widths the device kernels are built for (192, 384); the width-64 ones
# serve the oracle's CPU tests.
DEVICE_CASES = [c for c in MODEL_COST_CASES if desc_of(load(c)).dim in (192, 384)]


@pytest.mark.parametrize("case", DEVICE_CASES)
def test_fp32_model_cost_matches_reference_golden(case, runtimes):
    d = load(case)
    rt, desc, sd = _rt(runtimes, d)
    got = rt.model_cost(_t(d["emb"]), _t(d["goal"]), _t(d["cand"])).cpu().numpy()
    rt.sync()
    st = cost_stats(got, d["cost"])
    print(f"{case}: {st}")
    assert st["allclose"], st


@pytest.mark.parametrize("norm,P,H,S", [("none", 256, 1, 64), ("batchnorm", 512, 2, 200), ("layernorm", 2048, 3, 40)])
def test_fp32_pred_proj_matches_oracle(norm, P, H, S):
    desc = ModelDesc(pred_proj_hidden=P, pred_proj_norm=norm)
    sd = synthetic_state_dict(desc, 23)
    rt = Runtime(desc, sd, "cuda:0", model_cost_autocast="none")
    rng = np.random.default_rng(7)
    emb = rng.standard_normal((2, H, desc.dim)).astype(np.float32)
    goal = rng.standard_normal((2, 1, desc.dim)).astype(np.float32)
    cand = rng.standard_normal((2, S, 5, desc.action_dim)).astype(np.float32)
    got = rt.model_cost(_t(emb), _t(goal), _t(cand)).cpu().numpy()
    rt.sync()
    st = cost_stats(got, lo.get_cost_from_embeddings(emb, goal, cand, sd, desc))
    assert st["allclose"], st
    rt.close()


@pytest.mark.parametrize("case", HEADLINE_CASES)
def test_fp32_teacher_forced_costs_and_rankings(case, runtimes):
    d = load(case)
    rt, desc, sd = _rt(runtimes, d)
    kw = json.loads(str(d["solver"]))
    k, n = kw["topk"], int(d["n_iters"])
    traj = _reference_trajectory(d, k, kw["elite_retention"])
    emb, goal = _t(d["emb"]), _t(d["goal"])
    worst, mismatched = 0.0, 0
    for i in range(n):
        ref = d[f"cost_{i}"]
        got = rt.model_cost(emb, goal, _t(traj[i]["candidates"])).cpu().numpy()
        st = cost_stats(got, ref)
        worst = max(worst, st["max_rel"])
        assert st["allclose"], f"iteration {i}: {st}"
        assert np.array_equal(got.argmin(1), ref.argmin(1)) or np.all(
            ref[np.arange(ref.shape[0]), got.argmin(1)] == ref.min(1)), f"iteration {i}: argmin differs"
        drift = ranking_drift(ref, got, k, 2.0 * st["max_abs"])
        mismatched += drift["topk_mismatch_rows"]
        assert drift["explained"], f"iteration {i}: {drift}"
    rt.sync()
    print(f"{case}: {n} iterations, float32 cost max rel err {worst:.2e}, top-k rows with a tie swap {mismatched}")


@pytest.mark.parametrize("case", HEADLINE_CASES)
def test_fp32_full_plan_on_reference_noise(case, runtimes):
    d = load(case)
    rt, desc, sd = _rt(runtimes, d)
    kw = json.loads(str(d["solver"]))
    k, n, retention = kw["topk"], int(d["n_iters"]), kw["elite_retention"]
    counts = [int(c) for c in d["counts"]]
    act, std, fc, tr = rt.plan(_opts(kw), _t(d["emb"]), _t(d["goal"]), _t(d["mean0"]), _t(d["var0"]),
                               noise_steps=[_t(d[f"noise_{i}"]) for i in range(n)], trace=True)
    rt.sync()
    idx_dev = tr["topk_idx"].cpu().numpy()
    B = d["emb"].shape[0]
    keep = max(retention, 1)
    on_track = []
    for b in range(B):
        flip = n
        for i in range(n):
            ref_c = d[f"cost_{i}"][b]
            dev_c = tr["costs"][i, b, :counts[i]].cpu().numpy()
            assert cost_stats(dev_c, ref_c)["allclose"], f"env {b} iteration {i}"
            dev_i, ref_i = idx_dev[i, b].tolist(), d[f"inds_{i}"][b].tolist()
            same_set = set(dev_i) == set(ref_i)
            same_head = [ref_c[a] for a in dev_i[:keep]] == [ref_c[r] for r in ref_i[:keep]]
            if not (same_set and same_head):
                s = np.sort(ref_c)
                gap = (s[k] - s[k - 1]) / abs(s[k - 1]) if not same_set else 0.0
                assert gap <= TIE_REL, f"env {b}: elites changed at iteration {i} with a gap of {gap:.2e}"
                flip = i
                break
            if dev_i[:keep] != ref_i[:keep]:  # equal costs carried over in another order
                flip = i
                break
        on_track.append(flip)
    print(f"{case}: float32 plan on the reference's trajectory for {on_track} of {n} iterations")
    for b, flip in enumerate(on_track):
        if flip == n:
            scale = float(np.abs(d["solve_actions"][b]).max()) + 1.0
            np.testing.assert_allclose(act[b].cpu().numpy(), d["solve_actions"][b], rtol=1e-4, atol=1e-5 * scale)
            np.testing.assert_allclose(std[b].cpu().numpy(), d["solve_var"][b], rtol=1e-4, atol=1e-5 * scale)
            np.testing.assert_allclose(fc[b].cpu().numpy(), d["solve_costs"][b], rtol=RTOL, atol=ATOL)


def test_switching_modes_gives_each_modes_results():
    desc = ModelDesc()
    sd = synthetic_state_dict(desc, 0)
    rng = np.random.default_rng(9)
    emb = _t(rng.standard_normal((2, 1, desc.dim)))
    goal = _t(rng.standard_normal((2, 1, desc.dim)))
    cand = _t(rng.standard_normal((2, 300, 5, desc.action_dim)))
    mean, std = torch.zeros(2, 5, 10, device="cuda:0"), torch.ones(2, 5, 10, device="cuda:0")
    opts = PlanOptions(num_samples=300, topk=30, n_steps=4, sample_decay=1.25, sample_count_bucket_size=60,
                       elite_retention=3, beta=2.0)
    rt = Runtime(desc, sd, "cuda:0")
    assert rt.model_cost_autocast_mode() == "bf16"
    c_bf16 = rt.model_cost(emb, goal, cand).clone()
    p_bf16 = rt.plan(opts, emb, goal, mean, std, plan_index=3)[0].clone()
    rt.set_model_cost_autocast("none")
    c_f32 = rt.model_cost(emb, goal, cand).clone()
    p_f32 = rt.plan(opts, emb, goal, mean, std, plan_index=3)[0].clone()
    p_f32b = rt.plan(opts, emb, goal, mean, std, plan_index=3)[0].clone()  # graph replay
    rt.set_model_cost_autocast("bf16")
    c_bf16b = rt.model_cost(emb, goal, cand)
    p_bf16b = rt.plan(opts, emb, goal, mean, std, plan_index=3)[0]
    rt.sync()
    assert torch.equal(c_bf16, c_bf16b) and torch.equal(p_bf16, p_bf16b)
    assert torch.equal(p_f32, p_f32b)
    want = lo.get_cost_from_embeddings(emb.cpu().numpy(), goal.cpu().numpy(), cand.cpu().numpy(), sd, desc)
    assert cost_stats(c_f32.cpu().numpy(), want)["allclose"]
    assert not cost_stats(c_bf16.cpu().numpy(), want)["allclose"]  # bf16 sits at its own ~1e-3 bound
    with pytest.raises(ValueError):
        rt.set_model_cost_autocast("fp16")
    rt.close()


def test_fp32_costs_do_not_depend_on_the_batch():
    """An env's float32 costs are the same bits alone (64 x 64 GEMM tiles) and inside a batch
    of 64 envs x 300 candidates (the 128 x 128 tiles for the wide GEMMs): every output sums
    its products in the same order whatever the tile."""
    desc = ModelDesc()
    sd = synthetic_state_dict(desc, 0)
    rt = Runtime(desc, sd, "cuda:0", model_cost_autocast="none")
    rng = np.random.default_rng(12)
    emb = _t(rng.standard_normal((64, 3, desc.dim)))
    goal = _t(rng.standard_normal((64, 1, desc.dim)))
    cand = _t(rng.standard_normal((64, 300, 5, desc.action_dim)))
    big = rt.model_cost(emb, goal, cand)
    one = rt.model_cost(emb[5:6], goal[5:6], cand[5:6])
    rt.sync()
    assert torch.equal(big[5:6], one)
    want = lo.get_cost_from_embeddings(emb[5:6].cpu().numpy(), goal[5:6].cpu().numpy(), cand[5:6].cpu().numpy(),
                                       sd, desc)
    assert cost_stats(one.cpu().numpy(), want)["allclose"]
    rt.close()


def test_fp32_profile_and_per_sample_embeddings():
    """lewm_profile_plan reports a float32 plan's model costs under one class (fp32_cost, with
    the canonical GEMM FLOPs of the rows it runs); per-candidate embeddings (rank 4, all equal)
    give the same costs and gradients as per-env ones."""
    desc = ModelDesc()
    sd = synthetic_state_dict(desc, 0)
    rt = Runtime(desc, sd, "cuda:0", model_cost_autocast="none")
    rng = np.random.default_rng(13)
    emb = _t(rng.standard_normal((2, 1, desc.dim)))
    goal = _t(rng.standard_normal((2, 1, desc.dim)))
    mean, std = torch.zeros(2, 5, 10, device="cuda:0"), torch.ones(2, 5, 10, device="cuda:0")
    prof = rt.profile_plan(PlanOptions(num_samples=64, topk=8, n_steps=3), emb, goal, mean, std)
    assert set(prof["classes"]) == {"fp32_cost", "sample", "refit"}, prof["classes"].keys()
    f32 = prof["classes"]["fp32_cost"]
    assert f32["launches"] == 3 and f32["ms"] > 0 and f32["flops"] > 0
    cand = _t(rng.standard_normal((2, 12, 5, desc.action_dim)))
    emb4 = emb[:, None].expand(2, 12, 1, desc.dim).contiguous()
    c3, g3 = rt.model_cost_grad(emb, goal, cand)
    c4, g4 = rt.model_cost_grad(emb4, goal, cand)
    rt.sync()
    assert torch.equal(c3, c4) and torch.equal(g3, g4)
    assert torch.equal(rt.model_cost(emb4, goal, cand), c3)
    rt.close()


@pytest.mark.parametrize("seed", range(8))
def test_fp32_random_shapes_match_oracle(seed):
    """Seeded random geometries (history 1-4, horizon up to 7, history window 1-3, per-env or
    per-candidate embeddings): the float32 costs against the oracle at the 1e-5 gate, and the
    gradient's costs equal to the forward's bit for bit."""
    rng = np.random.default_rng(1000 + seed)
    desc = ModelDesc()
    sd = synthetic_state_dict(desc, 0)
    rt = _SHARED.setdefault("rt", Runtime(desc, sd, "cuda:0", model_cost_autocast="none"))
    H = int(rng.integers(1, 5))
    T = int(rng.integers(H, 8))
    hs = int(rng.integers(1, 4))
    B, S = int(rng.integers(1, 4)), int(rng.integers(1, 40))
    emb = rng.standard_normal((B, H, desc.dim)).astype(np.float32)
    goal = rng.standard_normal((B, 1, desc.dim)).astype(np.float32)
    cand = rng.standard_normal((B, S, T, desc.action_dim)).astype(np.float32)
    got = rt.model_cost(_t(emb), _t(goal), _t(cand), history_size=hs)
    g_cost, _ = rt.model_cost_grad(_t(emb), _t(goal), _t(cand), history_size=hs)
    rt.sync()
    want = lo.get_cost_from_embeddings(emb, goal, cand, sd, desc, history_size=hs)
    st = cost_stats(got.cpu().numpy(), want)
    assert st["allclose"], (H, T, hs, B, S, st)
    assert torch.equal(got, g_cost), (H, T, hs)


_SHARED = {}


_FP32_TILES = """
import sys, numpy as np, torch
from lewm_flash_b200.model import ModelDesc, synthetic_state_dict
from lewm_flash_b200.runtime import Runtime
d = np.load(sys.argv[1])
desc = ModelDesc()
rt = Runtime(desc, synthetic_state_dict(desc, 0), "cuda:0", model_cost_autocast="none")
t = lambda x: torch.as_tensor(x, device="cuda:0")
cost = rt.model_cost(t(d["emb"]), t(d["goal"]), t(d["cand"])).cpu().numpy()
gc, gg = rt.model_cost_grad(t(d["emb"]), t(d["goal"]), t(d["cand"][:, :30]))
rt.sync()
np.save(sys.argv[2], np.concatenate([cost.ravel(), gc.cpu().numpy().ravel(), gg.cpu().numpy().ravel()]))
"""


@pytest.mark.parametrize("S,H", [(300, 1), (40, 3)])
def test_fp32_gemm_tile_shape_does_not_change_bits(tmp_path, S, H):
    # Small GEMM grids run 64 x 32 or 32 x 32 tiles instead of 64 x 64 (forward and reverse
    # pass). Every output keeps its k order, so a process with LEWM_FP32_NARROW=0 (64 x 64
    # tiles everywhere) gives the same costs and gradients bit for bit.
    import os
    import subprocess
    import sys

    rng = np.random.default_rng(S + H)
    desc = ModelDesc()
    np.savez(tmp_path / "in.npz", emb=rng.standard_normal((1, H, desc.dim)).astype(np.float32),
             goal=rng.standard_normal((1, 1, desc.dim)).astype(np.float32),
             cand=rng.standard_normal((1, S, 5, desc.action_dim)).astype(np.float32))
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    outs = []
    for flag in ("1", "0"):
        env = dict(os.environ, LEWM_FP32_NARROW=flag)
        env["PYTHONPATH"] = root + os.pathsep + env.get("PYTHONPATH", "")
        out = tmp_path / f"out{flag}.npy"
        subprocess.run([sys.executable, "-c", _FP32_TILES, str(tmp_path / "in.npz"), str(out)], env=env, cwd=root,
                       check=True, timeout=600)
        outs.append(np.load(out))
    assert np.array_equal(outs[0], outs[1])
