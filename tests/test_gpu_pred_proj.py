"""The predictor's pred_proj MLP head on the device (JEPA.predict, lewm/jepa.py:106-114).

``JEPA.predict`` sends every predictor output row through ``pred_proj``: Identity, or the
reference ``MLP`` (``lewm/module.py:217-240``: Linear(192 -> P), LayerNorm / BatchNorm1d
in eval / none, GELU, Linear(P -> 192)). The rollout keeps only each call's last row, so
the device runs the head on the new prediction of every candidate after each predictor
call (the encoder's projector kernels) before the cost or the next window. Checked
through the C ABI against reference fixtures (LayerNorm head, history 1; BatchNorm head,
history 3; ``tests/golden/make_golden.py``) and against the float32 oracle at 300
candidates, within the 1e-2 bf16-rollout bound, and inside a full plan.
"""

import numpy as np
import pytest
import torch

from lewm_flash_b200.model import ModelDesc, synthetic_state_dict
from lewm_flash_b200.runtime import PlanOptions, Runtime
from oracle import icem_oracle as io
from oracle import lewm_oracle as lo
from tests.golden_io import load, weights_of

pytestmark = pytest.mark.gpu
COST_RTOL = 1e-2


def cuda(x):
    return torch.as_tensor(np.asarray(x), dtype=torch.float32, device="cuda:0")


def rel(got, want):
    return np.abs(np.asarray(got, np.float64) - want) / np.maximum(np.abs(want), 1e-6)


@pytest.mark.parametrize("case", ["model_cost_full_ppln.npz", "model_cost_full_ppbn_h3.npz"])
def test_pred_proj_model_cost_matches_reference_golden(case):
    d = load(case)
    desc, sd = weights_of(d)
    assert desc.pred_proj_hidden == 2048
    rt = Runtime(desc, sd, "cuda:0")
    got = rt.model_cost(cuda(d["emb"]), cuda(d["goal"]), cuda(d["cand"])).cpu().numpy()
    rt.sync()
    err = rel(got, d["cost"])
    assert err.max() <= COST_RTOL, f"max rel err {err.max():.3e}"
    rt.close()


@pytest.mark.parametrize("norm,P,H,S", [("layernorm", 2048, 1, 300), ("batchnorm", 2048, 3, 130),
                                        ("none", 256, 1, 64), ("batchnorm", 512, 2, 200)])
def test_pred_proj_model_cost_matches_oracle(norm, P, H, S):
    desc = ModelDesc(pred_proj_hidden=P, pred_proj_norm=norm)
    sd = synthetic_state_dict(desc, 21)
    rt = Runtime(desc, sd, "cuda:0")
    rng = np.random.default_rng(5)
    emb = rng.standard_normal((2, H, desc.dim)).astype(np.float32)
    goal = rng.standard_normal((2, 1, desc.dim)).astype(np.float32)
    cand = rng.standard_normal((2, S, 5, desc.action_dim)).astype(np.float32)
    got = rt.model_cost(cuda(emb), cuda(goal), cuda(cand)).cpu().numpy()
    rt.sync()
    want = lo.get_cost_from_embeddings(emb, goal, cand, sd, desc)
    assert rel(got, want).max() <= COST_RTOL
    # The head changes the costs: the Identity-head model gives different ones.
    plain = Runtime(ModelDesc(), {k: v for k, v in sd.items() if not k.startswith("pred_proj")}, "cuda:0")
    other = plain.model_cost(cuda(emb), cuda(goal), cuda(cand)).cpu().numpy()
    plain.sync()
    assert rel(other, want).max() > 0.05
    rt.close()
    plain.close()


def test_pred_proj_plan_matches_oracle_replay():
    desc = ModelDesc(pred_proj_hidden=2048, pred_proj_norm="layernorm")
    sd = synthetic_state_dict(desc, 22)
    rt = Runtime(desc, sd, "cuda:0")
    rng = np.random.default_rng(6)
    emb = rng.standard_normal((2, 1, desc.dim)).astype(np.float32)
    goal = rng.standard_normal((2, 1, desc.dim)).astype(np.float32)
    mean = np.zeros((2, 5, 10), np.float32)
    std = np.ones_like(mean)
    opts = PlanOptions(num_samples=64, topk=8, n_steps=3, elite_retention=2, sample_decay=1.25,
                       sample_count_bucket_size=16)
    counts = [64, 64, 48]
    noise = [rng.standard_normal((2, c, 5, 10)).astype(np.float32) for c in counts]
    act, sdv, fc, tr = rt.plan(opts, cuda(emb), cuda(goal), cuda(mean), cuda(std),
                               noise_steps=[cuda(n) for n in noise], trace=True)
    rt.sync()
    assert tr["counts"] == counts
    for i, c in enumerate(counts):  # device costs against the fp32 model on the device's candidates
        cand = tr["candidates"][i, :, :c].cpu().numpy()
        want = lo.get_cost_from_embeddings(emb, goal, cand, sd, desc)
        assert rel(tr["costs"][i, :, :c].cpu().numpy(), want).max() <= COST_RTOL, i
    # The chain replayed by the oracle on the device's own costs reproduces its elites and outputs.
    costs = iter([tr["costs"][i, :, :c].cpu().numpy() for i, c in enumerate(counts)])
    trace = []
    a_o, s_o, f_o = io.run_static_icem_chain(lambda e, g, cc: next(costs), emb, goal, mean, std, noise, topk=8,
                                             elite_retention=2, trace=trace)
    for i, t in enumerate(trace):
        assert np.array_equal(t["topk_inds"], tr["topk_idx"][i].cpu().numpy()), i
    np.testing.assert_allclose(act.cpu().numpy(), a_o, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(fc.cpu().numpy(), f_o, rtol=1e-5)
    # Graph replay (in-kernel noise) gives the same bits as direct launches of the same plan.
    a1 = rt.plan(opts, cuda(emb), cuda(goal), cuda(mean), cuda(std), plan_index=4)[0].clone()
    a2 = rt.plan(opts, cuda(emb), cuda(goal), cuda(mean), cuda(std), plan_index=4)[0]
    rt.sync()
    assert torch.equal(a1, a2)
    rt.close()
