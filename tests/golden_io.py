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
