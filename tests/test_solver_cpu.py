"""Host-side solver logic against the reference's own code (no GPU needed).

The warm-start padding (``prepare_init_action``, ``lewm/solvers/cem_exact.py:13-51``),
the initial distribution (``init_action_distrib``, ``lewm/solvers/icem.py:396-419``),
the schedule and the receding-horizon warm-start shift of ``CEMExactSolver``
(``_shift_warm_start_distribution``, ``lewm/solvers/cem_exact.py:193-241``) are host
code in the B200 solvers; they must give the reference's tensors and info dicts.
Uses the reference package in ``baseline/_ref`` (skipped if it is absent).
"""

from __future__ import annotations

import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from lewm_flash_b200.solver import B200CEMSolver, B200ICEMSolver, prepare_init_action

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"
pytestmark = pytest.mark.skipif(not (REF / "lewm" / "jepa.py").is_file(),
                                reason="reference package not installed in baseline/_ref")


def _ref():
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    from lewm.solvers import cem_exact, icem
    return cem_exact, icem


class Box:
    def __init__(self, n_envs):
        self.shape = (n_envs, 2)
        self.low = -np.ones(self.shape, np.float32)
        self.high = np.ones(self.shape, np.float32)


class NoActionModel(torch.nn.Module):
    """A model without get_action: prepare_init_action pads with zeros."""


@pytest.mark.parametrize("n_prev", [None, 0, 2, 5, 6])
def test_prepare_init_action_matches_reference(n_prev):
    cem_exact, _ = _ref()
    init = None if n_prev is None else torch.randn(3, n_prev, 10, generator=torch.Generator().manual_seed(1))
    got = prepare_init_action(NoActionModel(), {}, init, 5, n_envs=3, action_dim=10)
    want = cem_exact.prepare_init_action(NoActionModel(), {}, init, 5, n_envs=3, action_dim=10)
    assert torch.equal(got, want)


def test_prepare_init_action_asserts_like_reference():
    cem_exact, _ = _ref()
    bad = torch.zeros(2, 1, 10)
    for fn in (prepare_init_action, cem_exact.prepare_init_action):
        with pytest.raises(AssertionError, match="init_action batch size 2 != n_envs 3"):
            fn(NoActionModel(), {}, bad, 5, n_envs=3, action_dim=10)


@pytest.mark.parametrize("prefix", [None, 2])
def test_init_action_distrib_and_schedule_match_reference(prefix):
    _, icem = _ref()
    kw = dict(num_samples=300, n_steps=30, topk=30, sample_decay=1.25, sample_count_bucket_size=60, var_scale=0.7)
    cfg = SimpleNamespace(horizon=5, action_block=5)
    ref = icem.ICEMSolver(model=NoActionModel(), **kw)
    ours = B200ICEMSolver(NoActionModel(), device="cpu", **kw)
    for s in (ref, ours):
        s.configure(action_space=Box(3), n_envs=3, config=cfg)
    init = None if prefix is None else torch.randn(3, prefix, 10, generator=torch.Generator().manual_seed(2))
    a = prepare_init_action(NoActionModel(), {}, init, 5, n_envs=3, action_dim=10)
    for got, want in zip(ours.init_action_distrib(3, a), ref.init_action_distrib(3, a)):
        assert torch.equal(got, want)
    assert ours.sample_counts() == ref.sample_counts()
    assert ours.model_cost_evals_per_solve() == ref.model_cost_evals_per_solve() == 2820


@pytest.mark.parametrize("case", ["fresh", "used", "signature_mismatch", "no_unexecuted_tail", "invalid_shift",
                                  "disabled"])
def test_warm_start_shift_matches_reference(case):
    cem_exact, _ = _ref()
    receding = {"no_unexecuted_tail": 5, "invalid_shift": 0}.get(case, 2)
    cfg = SimpleNamespace(horizon=5, action_block=5, receding_horizon=receding)
    kw = dict(num_samples=40, n_steps=3, topk=6, var_scale=0.5, warm_start=case != "disabled")
    ref = cem_exact.CEMExactSolver(model=NoActionModel(), **kw)
    ours = B200CEMSolver(NoActionModel(), device="cpu", **kw)
    for s in (ref, ours):
        s.configure(action_space=Box(2), n_envs=2, config=cfg)
    assert ours.last_warm_start_info == ref.last_warm_start_info
    g = torch.Generator().manual_seed(5)
    prev_m, prev_v = torch.randn(2, 5, 10, generator=g), torch.rand(2, 5, 10, generator=g)
    if case != "fresh":
        ref._remember_warm_start_distribution(prev_m, prev_v)
        ours._warm_signature = ours._distribution_signature(prev_m, prev_v)
        ours._warm_mean, ours._warm_var = prev_m.clone(), prev_v.clone()
    n = 3 if case == "signature_mismatch" else 2
    mean, var = torch.zeros(n, 5, 10), 0.5 * torch.ones(n, 5, 10)
    got = ours._shift(mean, var)
    want = ref._shift_warm_start_distribution(mean, var)
    for a, b in zip(got, want):
        assert torch.equal(a, b)
    assert ours.last_warm_start_info == ref.last_warm_start_info
    if case == "used":
        assert ours.last_warm_start_info["used"] is True


CEMGD_BAD_ARGS = [dict(topk=0), dict(num_samples=10, topk=20), dict(n_steps=0), dict(elite_retention=-1),
                  dict(colored_noise="blue"), dict(momentum_alpha=1.0), dict(sample_decay=0.5),
                  dict(sample_count_bucket_size=-1), dict(gd_seed_solver="mppi"), dict(gd_seed_source="last"),
                  dict(gd_refine_topk=0), dict(gd_refine_topk=31), dict(gd_steps=-1), dict(gd_lr=0.0)]


@pytest.mark.parametrize("bad", CEMGD_BAD_ARGS)
def test_cem_gd_solver_rejects_like_reference(bad):
    """B200CEMGDSolver raises the reference CEMGDSolver's ValueErrors (lewm/solvers/cem_gd.py:67-101)."""
    from lewm_flash_b200.solver import B200CEMGDSolver

    _ref()
    from lewm.solvers.cem_gd import CEMGDSolver

    with pytest.raises(ValueError) as want:
        CEMGDSolver(model=None, **bad)
    with pytest.raises(ValueError) as got:
        B200CEMGDSolver(None, **bad)
    assert str(got.value) == str(want.value)


@pytest.mark.parametrize("kw", [dict(), dict(gd_seed_solver="icem", sample_decay=1.25, sample_count_bucket_size=60),
                                dict(gd_seed_solver="cem", sample_decay=1.25, sample_count_bucket_size=60),
                                dict(gd_seed_solver="icem", sample_decay=1.1, num_samples=100, topk=10)])
def test_cem_gd_solver_schedule_and_surface_match_reference(kw):
    from lewm_flash_b200.solver import B200CEMGDSolver

    _ref()
    from lewm.solvers.cem_gd import CEMGDSolver

    cfg = SimpleNamespace(horizon=5, action_block=5)
    ref = CEMGDSolver(model=None, **kw)
    dev = B200CEMGDSolver(None, **kw)
    for s in (ref, dev):
        s.configure(action_space=Box(2), n_envs=2, config=cfg)
    assert dev.sample_counts() == ref.sample_counts()
    assert dev.model_cost_evals_per_solve() == ref.model_cost_evals_per_solve()
    assert (dev.n_envs, dev.action_dim, dev.horizon, dev.action_block) == (
        ref.n_envs, ref.action_dim, ref.horizon, ref.action_block)
    m_ref, v_ref = ref.init_action_distrib(2, None)
    m_dev, v_dev = dev.init_action_distrib(2, None)
    assert torch.equal(m_ref, m_dev) and torch.equal(v_ref, v_dev)
    opts = dev.plan_options()
    assert opts.counts == ref.sample_counts()
    icem = dev.gd_seed_solver == "icem"
    assert opts.beta == (COLORED[dev.colored_noise] if icem else 0.0)
    assert opts.elite_retention == (dev.elite_retention if icem else 0) and not opts.return_best_elite


COLORED = {"none": 0.0, "pink": 1.0, "brown": 2.0}


def test_static_solver_surface_matches_reference():
    """B200ICEMStaticSolver: ICEMStaticCompileSolver's extra arguments, ValueError and the
    disabled-warmup record (lewm/solvers/icem_static_compile.py:117-258)."""
    from lewm_flash_b200.solver import B200ICEMStaticSolver

    _ref()
    from lewm.solvers.icem_static_compile import ICEMStaticCompileSolver

    with pytest.raises(ValueError) as want:
        ICEMStaticCompileSolver(model=None, static_chain_mode="fast")
    with pytest.raises(ValueError) as got:
        B200ICEMStaticSolver(None, static_chain_mode="fast")
    assert str(got.value) == str(want.value)
    kw = dict(num_samples=300, topk=30, sample_decay=1.25, sample_count_bucket_size=60, static_chain_mode="default")
    ref = ICEMStaticCompileSolver(model=None, **kw)
    dev = B200ICEMStaticSolver(None, **kw)
    cfg = SimpleNamespace(horizon=5, action_block=5)
    for s in (ref, dev):
        s.configure(action_space=Box(1), n_envs=1, config=cfg)
    assert dev.sample_counts() == ref.sample_counts()
    r, d = ref.warmup_static_chain_compile(embed_dim=192), dev.warmup_static_chain_compile(embed_dim=192)
    assert (d.enabled, d.elapsed_s, d.sample_counts, d.mode, d.fullgraph, d.input_shapes) == (
        r.enabled, r.elapsed_s, r.sample_counts, r.mode, r.fullgraph, r.input_shapes)
