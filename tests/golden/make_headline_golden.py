"""Generate reference-run fixtures of the benchmarked iCEM configurations.

Runs the reference's own ``ICEMSolver`` (``lewm/solvers/icem.py``) and
``run_static_icem_chain`` (``lewm/solvers/icem_static_compile.py``) on CPU in
float32, on seeded synthetic weights (``lewm_flash_b200.model.synthetic_state_dict``,
width 192, 6 layers) and seeded N(0,1) latents, at the full solver settings of the
benchmark:

* ``icem_headline_cfg2``: bucketed iCEM 300 -> 60 samples over 30 iterations
  (2820 candidates), 30 elites, brown noise over raw time (action block 5),
  elite retention 3, 1 env, history 1, horizon 5;
* ``icem_headline_cfg2_ret5``: the same with elite retention 5;
* ``icem_headline_cfg3``: the same solver for 4 envs with history 3 (a subset of
  the 64-env batched configuration; envs are independent);
* ``icem_headline_cfg1``: plain CEM, 300 samples / 30 elites / 30 iterations
  (``ICEMSolver`` with white noise, no sample decay, no elite retention), 1 env,
  history 1: the float32 configuration.

The noise of every iteration is drawn by ``ICEMSolver._sample_noise``; the
fixture stores it with the reference's per-iteration costs, top-k indices and
values, the refit mean / std after each iteration, and the outputs of
``run_static_icem_chain`` and of ``ICEMSolver.solve`` (which draws the same noise
from a fresh generator with the same seed; the script checks that both agree bit
for bit). Weights are not stored: tests regenerate them from the seed and check
the stored checksum.

Usage (needs the reference checkout; not run by the tests)::

    python tests/golden/make_headline_golden.py --reference /root/reference
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(HERE))

from lewm_flash_b200.model import ModelDesc, state_dict_checksum, synthetic_state_dict  # noqa: E402

CEM_SOLVER = dict(num_samples=300, n_steps=30, topk=30, sample_decay=1.0, sample_count_bucket_size=0,
                  colored_noise="none", colored_noise_time="raw", elite_retention=0, seed=0, var_scale=1.0)
HEADLINE_SOLVER = dict(num_samples=300, n_steps=30, topk=30, sample_decay=1.25, sample_count_bucket_size=60,
                       colored_noise="brown", colored_noise_time="raw", elite_retention=3, seed=0, var_scale=1.0)


def headline_case(torch, name, solver_kw, n_envs, H, input_seed):
    from make_golden import build_reference_jepa, desc_dict

    from lewm.solvers.icem import ICEMSolver
    from lewm.solvers.icem_static_compile import run_static_icem_chain

    desc = ModelDesc()
    sd = synthetic_state_dict(desc, 0)
    model = build_reference_jepa(torch, desc, sd)
    g = torch.Generator().manual_seed(input_seed)
    emb = torch.randn(n_envs, H, desc.dim, generator=g)
    goal = torch.randn(n_envs, 1, desc.dim, generator=g)

    class Box:
        def __init__(self, shape):
            self.shape = shape
            self.low = -np.inf * np.ones(shape, dtype=np.float32)
            self.high = np.inf * np.ones(shape, dtype=np.float32)

    cfg = SimpleNamespace(horizon=5, action_block=5)
    space = Box((n_envs, desc.action_dim // 5))
    kw = dict(solver_kw, batch_size=n_envs)
    solver = ICEMSolver(model=model, device="cpu", **kw)
    solver.configure(action_space=space, n_envs=n_envs, config=cfg)
    noise = [solver._sample_noise(n_envs, n) for n in solver.sample_counts()]
    trace = []

    def cost_fn(e, gl, cand):
        c = model.get_cost_from_embeddings(e, gl, cand, history_size=3)
        vals, inds = torch.topk(c, k=solver.topk, dim=1, largest=False)
        elites = torch.gather(cand, 1, inds[:, :, None, None].expand(-1, -1, cand.shape[2], cand.shape[3]))
        trace.append(dict(cand=cand.clone(), cost=c.clone(), inds=inds.clone(), vals=vals.clone(),
                          mean=elites.mean(dim=1), std=elites.std(dim=1)))
        return c

    mean, var = solver.init_action_distrib(n_envs, None)
    with torch.inference_mode():
        act, std, fcost = run_static_icem_chain(
            cost_fn, emb, goal, mean, var, noise, topk=solver.topk, elite_retention=solver.elite_retention,
            momentum_alpha=solver.momentum_alpha, return_best_elite=solver.return_best_elite)

    solver2 = ICEMSolver(model=model, device="cpu", **kw)
    solver2.configure(action_space=space, n_envs=n_envs, config=cfg)
    model.set_embedding_cache(True).set_compile_cost(True)
    info = {"emb": emb, "goal_emb": goal, "pixels": torch.zeros(n_envs, H), "goal": torch.zeros(n_envs, H)}
    solved = solver2.solve(info)
    model.set_embedding_cache(False).set_compile_cost(False)
    same = bool(torch.equal(solved["actions"], act)) and bool(torch.equal(solved["var"][0], std))
    if not same:
        raise RuntimeError("ICEMSolver.solve and run_static_icem_chain disagree")

    out = dict(emb=emb.numpy(), goal=goal.numpy(), mean0=mean.numpy(), var0=var.numpy(),
               actions=act.numpy(), std=std.numpy(), final_cost=fcost.numpy(),
               solve_actions=solved["actions"].numpy(), solve_var=solved["var"][0].numpy(),
               solve_costs=np.asarray(solved["costs"], np.float32),
               counts=np.asarray(solver.sample_counts(), np.int64), seed=np.int64(0),
               checksum=np.float64(state_dict_checksum(sd)), desc=json.dumps(desc_dict(desc)),
               solver=json.dumps(kw), n_iters=np.int64(len(noise)), history=np.int64(H))
    out["cand_0"] = trace[0]["cand"].numpy()
    for i, (n, t) in enumerate(zip(noise, trace)):
        out[f"noise_{i}"] = n.numpy()
        out[f"cost_{i}"] = t["cost"].numpy()
        out[f"inds_{i}"] = t["inds"].numpy()
        out[f"vals_{i}"] = t["vals"].numpy()
        out[f"mean_{i}"] = t["mean"].numpy()
        out[f"std_{i}"] = t["std"].numpy()
    np.savez_compressed(HERE / f"icem_headline_{name}.npz", **out)
    print(f"icem_headline_{name}: {len(noise)} iterations, {sum(solver.sample_counts())} candidates per env; "
          f"final_cost={fcost.tolist()}")


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", required=True, help="reference checkout (its lewm/ is imported)")
    ap.add_argument("--only", nargs="*", help="case names to (re)generate (default: all)")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import torch

    torch.set_num_threads(8)
    cases = {
        "cfg2": (HEADLINE_SOLVER, 1, 1, 31),
        "cfg2_ret5": (dict(HEADLINE_SOLVER, elite_retention=5), 1, 1, 32),
        "cfg3": (HEADLINE_SOLVER, 4, 3, 33),
        "cfg1": (CEM_SOLVER, 1, 1, 34),
    }
    for name, (kw, n_envs, H, seed) in cases.items():
        if not args.only or name in args.only:
            headline_case(torch, name, kw, n_envs=n_envs, H=H, input_seed=seed)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
