"""Generate the golden fixtures that pin the oracle to the reference.

Runs the reference's own Python code (``lewm/jepa.py``, ``lewm/module.py``,
``lewm/solvers/icem.py``, ``lewm/solvers/icem_static_compile.py``) on CPU in
float32, with seeded synthetic weights from
``lewm_flash_b200.model.synthetic_state_dict`` and seeded inputs, and writes
the inputs and outputs as small ``.npz`` / ``.json`` files next to this script.
Weights are not stored: tests regenerate them from the seed and check the
stored checksum.

Usage (needs the reference checkout; not run by the tests)::

    python tests/golden/make_golden.py --reference /root/reference
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from lewm_flash_b200.model import ModelDesc, STRESS_DESC, state_dict_checksum, synthetic_state_dict  # noqa: E402

SMALL_DESC = ModelDesc(dim=64, depth=2, heads=4, dim_head=16, mlp_dim=256, action_dim=10,
                       smoothed_dim=10, embed_hidden=256, num_frames=3)


def build_reference_jepa(torch, desc: ModelDesc, sd):
    from lewm.jepa import JEPA
    from lewm.module import ARPredictor, Embedder, MLP

    pred = ARPredictor(num_frames=desc.num_frames, depth=desc.depth, heads=desc.heads,
                       mlp_dim=desc.mlp_dim, input_dim=desc.dim, hidden_dim=desc.dim,
                       dim_head=desc.dim_head)
    enc = Embedder(input_dim=desc.action_dim, smoothed_dim=desc.smoothed_dim, emb_dim=desc.dim,
                   mlp_scale=desc.embed_hidden // desc.dim)
    pp = None
    if desc.pred_proj_hidden:
        norm = {"none": None, "layernorm": torch.nn.LayerNorm, "batchnorm": torch.nn.BatchNorm1d}[desc.pred_proj_norm]
        pp = MLP(desc.dim, desc.pred_proj_hidden, desc.dim, norm_fn=norm)
    model = JEPA(encoder=torch.nn.Identity(), predictor=pred, action_encoder=enc, pred_proj=pp)
    state = {k: torch.from_numpy(v) for k, v in sd.items()}
    full = model.state_dict()
    for k in full:
        if k.endswith("num_batches_tracked"):
            state[k] = full[k]
    missing = set(full) - set(state)
    if missing:
        raise RuntimeError(f"synthetic weights miss {sorted(missing)}")
    model.load_state_dict(state, strict=True)
    return model.eval()


def desc_dict(desc: ModelDesc):
    from dataclasses import asdict
    return asdict(desc)


def model_cost_case(torch, name, desc, seed, B, S, T, H, input_seed, emb_rank=3):
    sd = synthetic_state_dict(desc, seed)
    model = build_reference_jepa(torch, desc, sd)
    g = torch.Generator().manual_seed(input_seed)
    if emb_rank == 3:
        emb = torch.randn(B, H, desc.dim, generator=g)
    else:
        emb = torch.randn(B, S, H, desc.dim, generator=g)
    goal = torch.randn(B, 1, desc.dim, generator=g)
    cand = torch.randn(B, S, T, desc.action_dim, generator=g)
    with torch.inference_mode():
        pred = model.rollout_from_embeddings(emb, cand, history_size=3)
        cost = model.get_cost_from_embeddings(emb, goal, cand, history_size=3)
    out = dict(emb=emb.numpy(), goal=goal.numpy(), cand=cand.numpy(), cost=cost.numpy(),
               pred=pred.numpy(), seed=np.int64(seed), checksum=np.float64(state_dict_checksum(sd)),
               desc=json.dumps(desc_dict(desc)))
    np.savez_compressed(HERE / f"model_cost_{name}.npz", **out)
    print(f"model_cost_{name}: cost[0,:4]={cost.reshape(-1)[:4].tolist()}")


def schedules(torch):
    from lewm.solvers.icem import ICEMSolver

    class Dummy(torch.nn.Module):
        pass

    cases = {
        "bucketed_300": dict(num_samples=300, n_steps=30, topk=30, sample_decay=1.25, sample_count_bucket_size=60),
        "stress_3000": dict(num_samples=3000, n_steps=30, topk=300, sample_decay=1.25, sample_count_bucket_size=600),
        "decay2": dict(num_samples=8, n_steps=4, topk=2, sample_decay=2.0),
        "decay2_bucket4": dict(num_samples=12, n_steps=4, topk=2, sample_decay=2.0, sample_count_bucket_size=4),
        "fixed_300": dict(num_samples=300, n_steps=30, topk=30),
    }
    out = {}
    for name, kw in cases.items():
        s = ICEMSolver(model=Dummy(), **kw)
        out[name] = {"kwargs": kw, "counts": s.sample_counts(), "evals": s.model_cost_evals_per_solve()}
    (HERE / "sample_counts.json").write_text(json.dumps(out, indent=1))
    print("sample_counts:", {k: v["evals"] for k, v in out.items()})


def colored(torch):
    from lewm.solvers.icem import make_colored_noise

    cases = [
        ("raw_b2", dict(horizon=5, action_dim=10, beta=2.0, action_block=5, time_axis="raw")),
        ("raw_b1", dict(horizon=5, action_dim=10, beta=1.0, action_block=5, time_axis="raw")),
        ("block_b2", dict(horizon=5, action_dim=10, beta=2.0, action_block=5, time_axis="block")),
        ("block1_b2", dict(horizon=10, action_dim=10, beta=2.0, action_block=1, time_axis="raw")),
        ("white", dict(horizon=5, action_dim=10, beta=0.0, action_block=5, time_axis="raw")),
    ]
    out = {}
    for name, kw in cases.items() if isinstance(cases, dict) else cases:
        g = torch.Generator().manual_seed(7)
        noise = make_colored_noise(batch_size=2, num_samples=6, device="cpu", dtype=torch.float32, generator=g, **kw)
        g = torch.Generator().manual_seed(7)
        beta, blk, ta = kw["beta"], kw["action_block"], kw["time_axis"]
        if beta <= 0:
            shape = (2, 6, kw["horizon"], kw["action_dim"])
        elif ta == "raw" and blk > 1:
            shape = (2, 6, kw["action_dim"] // blk, kw["horizon"] * blk)
        else:
            shape = (2, 6, kw["action_dim"], kw["horizon"])
        white = torch.randn(*shape, generator=g)
        out[name + "_white"] = white.numpy()
        out[name + "_colored"] = noise.numpy()
        out[name + "_kwargs"] = json.dumps(kw)
    np.savez_compressed(HERE / "colored_noise.npz", **out)
    print("colored_noise:", [c[0] for c in cases])


def chain_case(torch, name, desc, seed, solver_kw, n_envs, H, input_seed, clip=False):
    """Noise from ``ICEMSolver._sample_noise``, outputs of ``run_static_icem_chain`` and ``solve``."""
    from types import SimpleNamespace

    from lewm.solvers.icem import ICEMSolver
    from lewm.solvers.icem_static_compile import run_static_icem_chain

    sd = synthetic_state_dict(desc, seed)
    model = build_reference_jepa(torch, desc, sd)
    g = torch.Generator().manual_seed(input_seed)
    emb = torch.randn(n_envs, H, desc.dim, generator=g)
    goal = torch.randn(n_envs, 1, desc.dim, generator=g)

    class Box:
        def __init__(self, shape):
            self.shape = shape
            self.low = -0.8 * np.ones(shape, dtype=np.float32)
            self.high = 0.8 * np.ones(shape, dtype=np.float32)

    cfg = SimpleNamespace(horizon=5, action_block=5)
    space = Box((n_envs, desc.action_dim // 5))
    kw = dict(solver_kw)
    kw["clip_actions"] = clip
    # One env batch, so solve() draws each iteration's noise for all envs at once,
    # in the same order as the up-front draw below.
    kw["batch_size"] = n_envs
    solver = ICEMSolver(model=model, device="cpu", **kw)
    solver.configure(action_space=space, n_envs=n_envs, config=cfg)
    noise = [solver._sample_noise(n_envs, n) for n in solver.sample_counts()]

    trace = []

    def cost_fn(e, gl, cand):
        c = model.get_cost_from_embeddings(e, gl, cand, history_size=3)
        vals, inds = torch.topk(c, k=solver.topk, dim=1, largest=False)
        trace.append(dict(cand=cand.clone(), cost=c.clone(), inds=inds.clone(), vals=vals.clone()))
        return c

    mean, var = solver.init_action_distrib(n_envs, None)
    with torch.inference_mode():
        act, std, fcost = run_static_icem_chain(
            cost_fn, emb, goal, mean, var, noise, topk=solver.topk, elite_retention=solver.elite_retention,
            momentum_alpha=solver.momentum_alpha, return_best_elite=solver.return_best_elite,
            action_low=solver._action_low, action_high=solver._action_high)

    # ICEMSolver.solve draws the same noise from a fresh generator with the same seed.
    solver2 = ICEMSolver(model=model, device="cpu", **kw)
    solver2.configure(action_space=space, n_envs=n_envs, config=cfg)
    model.set_embedding_cache(True).set_compile_cost(True)
    # pixels/goal only carry H (JEPA._ensure_cost_embeddings reads pixels.size(2) after the
    # solver expands it to (envs, samples, H)); the cached embeddings skip the encoder.
    info = {"emb": emb, "goal_emb": goal, "pixels": torch.zeros(n_envs, H), "goal": torch.zeros(n_envs, H)}
    solved = solver2.solve(info)
    model.set_embedding_cache(False).set_compile_cost(False)
    same = bool(torch.equal(solved["actions"], act)) and bool(torch.equal(solved["var"][0], std))

    out = dict(emb=emb.numpy(), goal=goal.numpy(), mean0=mean.numpy(), var0=var.numpy(),
               actions=act.numpy(), std=std.numpy(), final_cost=fcost.numpy(),
               solve_actions=solved["actions"].numpy(), solve_costs=np.asarray(solved["costs"], np.float32),
               low=(solver._action_low.numpy() if solver._action_low is not None else np.zeros(0, np.float32)),
               high=(solver._action_high.numpy() if solver._action_high is not None else np.zeros(0, np.float32)),
               seed=np.int64(seed), checksum=np.float64(state_dict_checksum(sd)),
               desc=json.dumps(desc_dict(desc)), solver=json.dumps(kw), n_iters=np.int64(len(noise)))
    for i, (n, t) in enumerate(zip(noise, trace)):
        out[f"noise_{i}"] = n.numpy()
        out[f"cand_{i}"] = t["cand"].numpy()
        out[f"cost_{i}"] = t["cost"].numpy()
        out[f"inds_{i}"] = t["inds"].numpy()
        out[f"vals_{i}"] = t["vals"].numpy()
    np.savez_compressed(HERE / f"icem_chain_{name}.npz", **out)
    print(f"icem_chain_{name}: solve==static {same}; final_cost={fcost.tolist()}")
    if not same:
        raise RuntimeError("ICEMSolver.solve and run_static_icem_chain disagree")


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", required=True, help="reference checkout (its lewm/ is imported)")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import torch

    torch.set_num_threads(8)
    schedules(torch)
    colored(torch)
    model_cost_case(torch, "small_h1", SMALL_DESC, 11, B=2, S=7, T=5, H=1, input_seed=1)
    model_cost_case(torch, "small_h3", SMALL_DESC, 12, B=2, S=5, T=5, H=3, input_seed=2)
    model_cost_case(torch, "small_h3_rank4", SMALL_DESC, 12, B=2, S=3, T=5, H=3, input_seed=3, emb_rank=4)
    model_cost_case(torch, "small_ppln", SMALL_DESC.replace(pred_proj_hidden=96, pred_proj_norm="layernorm"),
                    13, B=1, S=6, T=5, H=1, input_seed=4)
    model_cost_case(torch, "small_ppbn", SMALL_DESC.replace(pred_proj_hidden=96, pred_proj_norm="batchnorm"),
                    14, B=1, S=6, T=5, H=1, input_seed=5)
    model_cost_case(torch, "full_h1", ModelDesc(), 0, B=1, S=6, T=5, H=1, input_seed=6)
    model_cost_case(torch, "full_h3", ModelDesc(), 0, B=2, S=4, T=5, H=3, input_seed=7)
    model_cost_case(torch, "full_ppln", ModelDesc(pred_proj_hidden=2048, pred_proj_norm="layernorm"), 3,
                    B=1, S=4, T=5, H=1, input_seed=8)
    model_cost_case(torch, "full_ppbn_h3", ModelDesc(pred_proj_hidden=2048, pred_proj_norm="batchnorm"), 4,
                    B=2, S=5, T=5, H=3, input_seed=10)
    model_cost_case(torch, "stress_h3", STRESS_DESC, 5, B=1, S=2, T=10, H=3, input_seed=9)
    base = dict(num_samples=24, n_steps=5, topk=6, seed=3, var_scale=1.0)
    chain_case(torch, "brown_ret", ModelDesc(), 0,
               dict(base, elite_retention=2, colored_noise="brown", colored_noise_time="raw", momentum_alpha=0.2,
                    sample_decay=1.25, sample_count_bucket_size=6), n_envs=2, H=1, input_seed=21)
    chain_case(torch, "best_clip", ModelDesc(), 0,
               dict(base, elite_retention=3, colored_noise="pink", colored_noise_time="raw",
                    return_best_elite=True), n_envs=1, H=1, input_seed=22, clip=True)
    chain_case(torch, "cem_white_h3", ModelDesc(), 0, dict(base), n_envs=2, H=3, input_seed=23)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
