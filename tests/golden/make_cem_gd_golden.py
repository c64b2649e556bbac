"""Generate the golden fixture that pins the CEM-GD refinement oracle to the reference.

Runs the reference ``CEMGDSolver._refine_seed_actions`` (``lewm/solvers/cem_gd.py:459-606``)
on CPU in float32 with the reference's quadratic embedding cost
(``lewm/solvers/cem_gd.py:748-761``): the settings of its own
``run_dummy_quadratic_refinement`` (zero seeds, target ones, (2, 1, 5, 4)) and seeded
random seeds / targets of shape (3, 4, 5, 10), with and without backtracking, and writes
``cem_gd_refine.npz`` next to this script.

Usage (needs the reference checkout; not run by the tests)::

    python tests/golden/make_cem_gd_golden.py --reference /root/reference
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# name: (shape, lr, steps, backtracking, seed; seed < 0: zero seeds and target ones)
CASES = {
    "dummy_lr0.01_s1": ((2, 1, 5, 4), 0.01, 1, True, -1),
    "dummy_lr0.5_s3": ((2, 1, 5, 4), 0.5, 3, True, -1),
    "rand_lr0.05_s5_bt": ((3, 4, 5, 10), 0.05, 5, True, 1),
    "rand_lr0.3_s4_nobt": ((3, 4, 5, 10), 0.3, 4, False, 2),
    "rand_lr2.0_s3_bt": ((3, 4, 5, 10), 2.0, 3, True, 3),
}


def case_inputs(shape, seed):
    if seed < 0:
        return np.zeros(shape, np.float32), np.ones(shape, np.float32)
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(shape).astype(np.float32),
            rng.uniform(-1.0, 1.0, (shape[0], 1, *shape[2:])).astype(np.float32))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="reference checkout (its lewm/ is imported)")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference)))
    import torch

    from lewm.solvers.cem_gd import CEMGDSolver, _QuadraticEmbeddingCost

    out = {}
    for name, (shape, lr, steps, bt, seed) in CASES.items():
        seed_actions, target = case_inputs(shape, seed)
        model = _QuadraticEmbeddingCost(torch.from_numpy(target))
        emb = torch.zeros(shape[0], 1, 3)
        seed_t = torch.from_numpy(seed_actions)
        seed_costs = model.get_cost_from_embeddings(emb, emb, seed_t)
        solver = CEMGDSolver(model=model, gd_steps=steps, gd_lr=lr, topk=max(1, shape[1]), num_samples=300)
        acts, costs, summary = solver._refine_seed_actions(seed_t, seed_costs, emb, emb, enable_backtracking=bt)
        out[f"{name}__actions"] = acts.numpy()
        out[f"{name}__costs"] = costs.numpy()
        out[f"{name}__accept_count"] = np.array(summary["gd_accept_count"])
        out[f"{name}__evals"] = np.array(summary["gd_model_cost_evals"])
        print(name, float(seed_costs.mean()), "->", float(costs.mean()), summary["gd_accept_count"])
    np.savez(HERE / "cem_gd_refine.npz", **out)


if __name__ == "__main__":
    main()
