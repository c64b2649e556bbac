"""Failure detection on the GPU, in forms that fault, trap or hang nothing.

* Bounded waits: every device-side wait of the kernels is bounded by the
  context's wait limit (%globaltimer). ``lewm_wait_selftest`` enqueues one wait on
  a barrier that nothing ever completes; with a 200 us limit it runs out, the
  kernel sets the timeout bit and returns, ``lewm_sync_status`` reports
  LEWM_DEVICE_TIMEOUT once, and the same context then plans normally.
* Numerics: a plan whose final costs are NaN (a host-built weight blob with a NaN
  in the final LayerNorm bias) makes ``lewm_sync_status`` report LEWM_NUMERIC_NAN;
  the status is cleared by that read.
"""

from __future__ import annotations

import time

import numpy as np
import pytest
import torch

from lewm_flash_b200._lib import LewmError
from lewm_flash_b200.model import ModelDesc, synthetic_state_dict
from lewm_flash_b200.runtime import PlanOptions, Runtime


def _inputs(dev, B=1):
    g = torch.Generator().manual_seed(0)
    emb = torch.randn(B, 1, 192, generator=g).to(dev)
    goal = torch.randn(B, 1, 192, generator=g).to(dev)
    return emb, goal, torch.zeros(B, 5, 10, device=dev), torch.ones(B, 5, 10, device=dev)


@pytest.mark.gpu
def test_expired_wait_reports_timeout_and_context_stays_usable():
    dev = torch.device("cuda", 0)
    desc = ModelDesc()
    rt = Runtime(desc, synthetic_state_dict(desc, 0), dev)
    emb, goal, mean, std = _inputs(dev)
    opts = PlanOptions(num_samples=32, topk=4, n_steps=2)
    before = rt.plan(opts, emb, goal, mean, std, plan_index=3)[0].clone()
    rt.sync()
    rt.set_wait_limit(200_000)  # 200 us
    t0 = time.perf_counter()
    rt.wait_selftest()
    with pytest.raises(LewmError) as err:
        rt.sync()
    elapsed = time.perf_counter() - t0
    assert err.value.status_name == "LEWM_DEVICE_TIMEOUT"
    assert elapsed < 1.5, f"the 200 us wait took {elapsed:.3f} s to report"
    rt.sync()  # the read cleared the status word
    rt.set_wait_limit(0)  # back to the 2 s default
    after = rt.plan(opts, emb, goal, mean, std, plan_index=3)[0]
    rt.sync()
    assert torch.equal(before, after)
    rt.close()


@pytest.mark.gpu
def test_nan_final_cost_reports_numeric_nan():
    dev = torch.device("cuda", 0)
    desc = ModelDesc()
    sd = synthetic_state_dict(desc, 0)
    sd["predictor.transformer.norm.bias"] = sd["predictor.transformer.norm.bias"].copy()
    sd["predictor.transformer.norm.bias"][7] = np.nan
    rt = Runtime(desc, sd, dev)
    emb, goal, mean, std = _inputs(dev, B=2)
    _, _, fcost, _ = rt.plan(PlanOptions(num_samples=32, topk=4, n_steps=2), emb, goal, mean, std)
    with pytest.raises(LewmError) as err:
        rt.sync()
    assert err.value.status_name == "LEWM_NUMERIC_NAN"
    assert torch.isnan(fcost).all()
    rt.sync()  # cleared
    rt.close()
