"""C ABI and host logic, no GPU: exports, schedules, option checks, weight packing order."""

import ctypes
import json
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from lewm_flash_b200 import _lib
from lewm_flash_b200.model import ModelDesc, STRESS_DESC, param_shapes, synthetic_state_dict
from lewm_flash_b200.runtime import PlanOptions, Runtime, coloring_matrix, pack_canonical, sample_counts
from lewm_flash_b200.solver import B200CEMSolver, B200ICEMSolver
from oracle import icem_oracle as io
from tests.golden_io import GOLDEN

HEADER = Path(__file__).resolve().parents[1] / "include" / "lewm_b200.h"


def header_symbols():
    return sorted(set(re.findall(r"LEWM_API\s+[\w\s\*]*?\b(lewm_\w+)\s*\(", HEADER.read_text())))


def test_library_exports_every_header_symbol():
    names = header_symbols()
    assert len(names) >= 11
    h = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in names if not hasattr(h, n)]
    assert not missing, missing
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"


def test_sample_counts_match_reference_schedules():
    cases = json.loads((GOLDEN / "sample_counts.json").read_text())
    for name, c in cases.items():
        kw = c["kwargs"]
        opts = PlanOptions(num_samples=kw["num_samples"], topk=kw["topk"], n_steps=kw["n_steps"],
                           sample_decay=kw.get("sample_decay", 1.0),
                           sample_count_bucket_size=kw.get("sample_count_bucket_size", 0))
        assert sample_counts(opts) == c["counts"], name


@pytest.mark.parametrize("n,beta", [(25, 2.0), (25, 1.0), (5, 2.0), (10, 2.0), (50, 1.0), (7, 0.0)])
def test_coloring_matrix_matches_oracle(n, beta):
    np.testing.assert_allclose(coloring_matrix(n, beta), io.coloring_matrix(n, beta), rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("kw,msg", [
    (dict(topk=0), "topk must be positive"),
    (dict(num_samples=4, topk=8), "must be >= topk"),
    (dict(n_steps=0), "n_steps must be positive"),
    (dict(elite_retention=-1), "elite_retention must be non-negative"),
    (dict(momentum_alpha=1.0), "momentum_alpha must satisfy"),
    (dict(sample_decay=0.5), "sample_decay must be >= 1.0"),
    (dict(sample_count_bucket_size=-3), "sample_count_bucket_size must be non-negative"),
])
def test_plan_option_checks_mirror_reference_value_errors(kw, msg):
    with pytest.raises(ValueError, match=msg):
        sample_counts(PlanOptions(**kw))
    solver_kw = dict(kw)
    if "sample_count_bucket_size" in solver_kw:
        pass
    with pytest.raises(ValueError, match=msg):
        B200ICEMSolver(model=None, **solver_kw)


def test_solver_rejects_unknown_noise_color():
    with pytest.raises(ValueError, match="colored_noise must be one of"):
        B200ICEMSolver(model=None, colored_noise="blue")


def test_solver_schedule_and_evals():
    s = B200ICEMSolver(model=None, num_samples=300, n_steps=30, topk=30, sample_decay=1.25,
                       sample_count_bucket_size=60)
    assert s.sample_counts() == [300, 240, 240, 180, 180, 120, 120, 120] + [60] * 22
    assert s.model_cost_evals_per_solve() == 2820
    assert B200CEMSolver(model=None).sample_counts() == [300] * 30


@pytest.mark.parametrize("desc", [ModelDesc(), STRESS_DESC,
                                  ModelDesc(pred_proj_hidden=2048, pred_proj_norm="layernorm"),
                                  ModelDesc(pred_proj_hidden=512, pred_proj_norm="batchnorm"),
                                  ModelDesc(pred_proj_hidden=256, pred_proj_norm="none")])
def test_weight_count_matches_reference_state_dict(desc):
    lib = _lib.lib()
    cd = __import__("lewm_flash_b200.runtime", fromlist=["desc_to_c"]).desc_to_c(desc)
    n = lib.lewm_weight_count(ctypes.byref(cd))
    want = sum(int(np.prod(s)) for k, s in param_shapes(desc).items())
    assert n == want
    flat = pack_canonical(desc, synthetic_state_dict(desc, 0))
    assert flat.size == n


def test_unsupported_shapes_are_rejected():
    lib = _lib.lib()
    from lewm_flash_b200.runtime import desc_to_c

    # pred_proj heads run at width 192 with a hidden width that is a multiple of 256
    for bad in (ModelDesc(dim=64, heads=4, dim_head=16, mlp_dim=256, embed_hidden=256), ModelDesc(dim_head=32),
                ModelDesc(pred_proj_hidden=96, pred_proj_norm="layernorm"),
                STRESS_DESC.replace(pred_proj_hidden=2048, pred_proj_norm="layernorm")):
        assert lib.lewm_weight_count(ctypes.byref(desc_to_c(bad))) == 0


def test_runtime_needs_cuda_device():
    with pytest.raises(ValueError, match="needs a CUDA device"):
        Runtime(ModelDesc(), synthetic_state_dict(ModelDesc(), 0), device="cpu")


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU error path")
def test_create_without_gpu_fails_loudly():
    desc = ModelDesc()
    flat = pack_canonical(desc, synthetic_state_dict(desc, 0))
    from lewm_flash_b200.runtime import desc_to_c

    h = ctypes.c_void_p()
    st = _lib.lib().lewm_create(ctypes.byref(h), ctypes.byref(desc_to_c(desc)), flat.ctypes.data, flat.size, 0)
    assert st == 5 and not h.value
    assert b"CUDA" in _lib.lib().lewm_last_error(None)


def _unopened_runtime(desc: ModelDesc) -> Runtime:
    """A Runtime without a device context: enough for the argument checks, which run first."""
    rt = object.__new__(Runtime)
    rt.desc = desc
    rt.device = torch.device("cpu")
    rt.plans_issued = 0
    return rt


@pytest.mark.parametrize("case", ["plan_action_dim", "plan_std", "plan_emb_width", "plan_goal_width",
                                  "cost_emb_width", "refit_costs", "refit_mean", "sample_action_dim",
                                  "sample_noise"])
def test_wrappers_reject_tensors_the_kernels_would_overrun(case):
    """Every kernel reads and writes at the model's widths, so the wrappers reject any other
    shape with ValueError before anything reaches the device."""
    desc = ModelDesc()
    rt = _unopened_runtime(desc)
    D, A = desc.dim, desc.action_dim
    z = torch.zeros
    opts = PlanOptions(num_samples=8, topk=2, n_steps=1)
    calls = {
        "plan_action_dim": lambda: rt.plan(opts, z(1, 1, D), z(1, 1, D), z(1, 5, A - 1), z(1, 5, A - 1)),
        "plan_std": lambda: rt.plan(opts, z(1, 1, D), z(1, 1, D), z(1, 5, A), z(1, 4, A)),
        "plan_emb_width": lambda: rt.plan(opts, z(1, 1, D - 1), z(1, 1, D), z(1, 5, A), z(1, 5, A)),
        "plan_goal_width": lambda: rt.plan(opts, z(1, 1, D), z(1, 1, D + 1), z(1, 5, A), z(1, 5, A)),
        "cost_emb_width": lambda: rt.model_cost(z(1, 1, D - 64), z(1, 1, D), z(1, 4, 5, A)),
        "refit_costs": lambda: rt.topk_refit(z(1, 3), z(1, 4, 5, A), z(1, 5, A), z(1, 5, A), 2),
        "refit_mean": lambda: rt.topk_refit(z(1, 4), z(1, 4, 5, A), z(1, 5, 1), z(1, 5, A), 2),
        "sample_action_dim": lambda: rt.sample_candidates(opts, 4, 0, z(1, 2, 1), z(1, 2, 1)),
        "sample_noise": lambda: rt.sample_candidates(opts, 4, 0, z(1, 5, A), z(1, 5, A), injected_noise=z(1, 3, 5, A)),
    }
    with pytest.raises(ValueError):
        calls[case]()


def test_sample_count_schedule_fuzzed_against_oracle():
    """The C ABI's schedule (lewm_sample_counts) equals the oracle restatement of
    ICEMSolver.sample_count_for_step (reference lewm/solvers/icem.py:377-394) on random
    sample sizes, elite counts, decays and buckets."""
    hyp = pytest.importorskip("hypothesis")
    st = hyp.strategies
    from oracle import icem_oracle as io

    @hyp.settings(max_examples=300, deadline=None, derandomize=True)
    @hyp.given(S=st.integers(1, 4096), k=st.integers(1, 512), n=st.integers(1, 40),
               decay=st.sampled_from([1.0, 1.1, 1.25, 1.5, 2.0, 3.0]), bucket=st.integers(0, 700))
    def check(S, k, n, decay, bucket):
        hyp.assume(k <= S)
        opts = PlanOptions(num_samples=S, topk=k, n_steps=n, sample_decay=decay, sample_count_bucket_size=bucket)
        assert sample_counts(opts) == io.sample_counts(n, S, k, decay, bucket)

    check()


def test_coloring_matrix_fuzzed_against_oracle():
    """lewm_coloring_matrix equals the oracle's rfft / scale / irfft filter as a matrix
    (reference lewm/solvers/icem.py:173-182) for every colored length up to 128 and any beta."""
    hyp = pytest.importorskip("hypothesis")
    st = hyp.strategies

    @hyp.settings(max_examples=150, deadline=None, derandomize=True)
    @hyp.given(n=st.integers(2, 128), beta=st.floats(0.0, 3.0, allow_nan=False))
    def check(n, beta):
        np.testing.assert_allclose(coloring_matrix(n, beta), io.coloring_matrix(n, beta), rtol=1e-10, atol=1e-11)

    check()
