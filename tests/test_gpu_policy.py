"""B200PlanningPolicy on the GPU: uint8 frames -> fused-transform encoder -> B200ICEMSolver plan
-> action buffer, against the same pieces called one by one.

* the embeddings the policy hands the solver are ``encode_frames`` of the observation and goal
  frames (one encoder pass over both), so the policy's first plan equals a twin solver's plan
  on those embeddings bit for bit (same seed, same plan index);
* every served action is the twin plan's block ``i // action_block``, raw action
  ``i % action_block``, mapped back through the action scaler;
* the second plan, ``receding_horizon * action_block`` steps later, warm-starts from the first
  plan's unexecuted tail, as the twin does when given that tail as ``init_action``.
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

N_ENVS, RAW, AB, HZ, RH = 3, 2, 5, 5, 2


class Box:
    def __init__(self, n):
        self.shape = (n, RAW)
        self.low = -np.ones(self.shape, np.float32)
        self.high = np.ones(self.shape, np.float32)


def _solver(rt, dev):
    from lewm_flash_b200.solver import B200ICEMSolver

    s = B200ICEMSolver(rt, num_samples=60, topk=10, n_steps=4, elite_retention=2, colored_noise="brown",
                       sample_decay=1.25, sample_count_bucket_size=20, seed=7, history_size=1, device=dev)
    s.configure(action_space=Box(N_ENVS), n_envs=N_ENVS, config=SimpleNamespace(horizon=HZ, receding_horizon=RH,
                                                                                   action_block=AB))
    return s


def test_policy_frames_to_actions_matches_the_pieces():
    from sklearn.preprocessing import StandardScaler

    from lewm_flash_b200.encoder import B200Encoder, EncoderDesc, flat_weights, synthetic_weights
    from lewm_flash_b200.model import ModelDesc, synthetic_state_dict
    from lewm_flash_b200.policy import B200PlanningPolicy
    from lewm_flash_b200.runtime import Runtime

    dev = torch.device("cuda:0")
    desc = ModelDesc()
    rt = Runtime(desc, synthetic_state_dict(desc, 0), dev)
    edesc = EncoderDesc(image_size=56, depth=2, proj_hidden=512)
    vit, proj = synthetic_weights(edesc, 0)
    enc = B200Encoder(edesc, flat_weights(vit, proj, edesc), dev)
    rng = np.random.default_rng(0)
    scaler = StandardScaler().fit(rng.normal(0.3, 2.0, (100, RAW)))
    cfg = SimpleNamespace(horizon=HZ, receding_horizon=RH, action_block=AB)
    policy = B200PlanningPolicy(_solver(rt, dev), cfg, process={"action": scaler}, encoder=enc)
    env = SimpleNamespace(num_envs=N_ENVS, action_space=Box(N_ENVS))
    policy.set_env(env)
    twin = _solver(rt, dev)

    def frames(seed):
        g = np.random.default_rng(seed)
        return {"pixels": torch.as_tensor(g.integers(0, 256, (N_ENVS, 1, 56, 56, 3), dtype=np.uint8)),
                "goal": torch.as_tensor(g.integers(0, 256, (N_ENVS, 1, 56, 56, 3), dtype=np.uint8))}

    served = []
    infos = []
    for step in range(2 * RH * AB):
        info = frames(step)
        if step % (RH * AB) == 0:
            infos.append(info)
        served.append(policy.get_action(info))
    assert policy.solves == 2

    tail = None
    for k, info in enumerate(infos):
        both = torch.cat([info["pixels"].reshape(-1, 56, 56, 3), info["goal"].reshape(-1, 56, 56, 3)]).to(dev)
        emb = enc.encode_frames(both)
        out = twin.solve({"emb": emb[:N_ENVS].reshape(N_ENVS, 1, -1), "goal_emb": emb[N_ENVS:].reshape(N_ENVS, 1, -1)},
                         init_action=tail)
        acts = out["actions"]
        for i in range(RH * AB):
            raw = acts[:, i // AB, (i % AB) * RAW:(i % AB + 1) * RAW].numpy()
            np.testing.assert_array_equal(served[k * RH * AB + i], scaler.inverse_transform(raw).astype(np.float32))
        tail = acts[:, RH:].clone()
    rt.close()
