"""Helpers that load the committed golden fixtures and regenerate their weights."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

from lewm_flash_b200.model import ModelDesc, state_dict_checksum, synthetic_state_dict

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name: str):
    return np.load(GOLDEN / name, allow_pickle=False)


def desc_of(d) -> ModelDesc:
    return ModelDesc(**json.loads(str(d["desc"])))


def weights_of(d):
    """Regenerate the fixture's synthetic weights and check them against its checksum."""
    desc = desc_of(d)
    sd = synthetic_state_dict(desc, int(d["seed"]))
    got = state_dict_checksum(sd)
    want = float(d["checksum"])
    assert abs(got - want) <= 1e-9 * max(1.0, abs(want)), f"weight generator drifted: {got} != {want}"
    return desc, sd


MODEL_COST_CASES = sorted(p.name for p in GOLDEN.glob("model_cost_*.npz"))
CHAIN_CASES = sorted(p.name for p in GOLDEN.glob("icem_chain_*.npz"))


def assert_same_topk(idx, want, costs, what=""):
    """Top-k indices equal to the reference's up to the order of exactly equal costs.

    ``torch.topk`` leaves the order of equal values unspecified (its CPU kernel put index
    239 before 160 at one tie of the CEM fixture); the device and the oracle order ties by
    the lower index. So: the same index set per row, and the same cost at every rank."""
    idx, want, costs = np.asarray(idx), np.asarray(want), np.asarray(costs)
    assert idx.shape == want.shape, what
    for b in range(idx.shape[0]):
        assert np.array_equal(np.sort(idx[b]), np.sort(want[b])), f"{what}: elite sets differ in row {b}"
        assert np.array_equal(costs[b][idx[b]], costs[b][want[b]]), f"{what}: elite order differs in row {b}"
