"""Generate the golden fixtures that pin the encoder oracle to the reference.

Builds the reference ``JEPA`` (``lewm/jepa.py``) with a transformers ``ViTModel``
encoder and the reference projector ``MLP`` (``lewm/module.py:217-240``), loads the
seeded synthetic weights of ``lewm_flash_b200.encoder.synthetic_weights``, runs the
reference ``JEPA.encode`` (``lewm/jepa.py:88-104``) on CPU in float32 over seeded
pixels of shape (b, t, C, H, W), and writes the embeddings next to this script as
``encoder_<case>.npz``. Weights and pixels are not stored: tests regenerate them from
the seeds and check the stored checksums.

Usage (needs the reference checkout; not run by the tests)::

    python tests/golden/make_encoder_golden.py --reference /root/reference
"""

from __future__ import annotations

import argparse
import json
import sys
from dataclasses import asdict
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from lewm_flash_b200.encoder import EncoderDesc, synthetic_weights  # noqa: E402
from oracle.vit_oracle import synthetic_pixels  # noqa: E402

CASES = {
    # name: (desc, weight seed, pixel seed, (b, t))
    "small_bn": (EncoderDesc(image_size=56, depth=2, proj_hidden=512, proj_norm="batchnorm"), 11, 21, (2, 2)),
    "small_ln": (EncoderDesc(image_size=56, depth=2, proj_hidden=512, proj_norm="layernorm"), 12, 22, (3, 1)),
    "small_none_p16": (EncoderDesc(image_size=64, patch_size=16, depth=3, proj_hidden=256, proj_norm="none"), 13, 23,
                       (1, 2)),
}


def weights_checksum(vit: dict, proj: dict) -> float:
    return float(sum(np.float64(v).sum() * (i + 1) for i, (_, v) in enumerate(sorted({**vit, **{
        "proj." + k: w for k, w in proj.items()}}.items()))))


def build_reference(torch, desc: EncoderDesc, vit: dict, proj: dict):
    from transformers import ViTConfig, ViTModel

    from lewm.jepa import JEPA
    from lewm.module import MLP

    cfg = ViTConfig(hidden_size=desc.hidden, num_hidden_layers=desc.depth, num_attention_heads=desc.heads,
                    intermediate_size=desc.mlp_dim, image_size=desc.image_size, patch_size=desc.patch_size,
                    num_channels=desc.channels, layer_norm_eps=desc.ln_eps)
    encoder = ViTModel(cfg, add_pooling_layer=False)
    encoder.load_state_dict({k: torch.from_numpy(v) for k, v in vit.items()}, strict=True)
    norm = {"none": None, "layernorm": torch.nn.LayerNorm, "batchnorm": torch.nn.BatchNorm1d}[desc.proj_norm]
    projector = MLP(desc.hidden, desc.proj_hidden, desc.proj_out, norm_fn=norm)
    state = {k: torch.from_numpy(v) for k, v in proj.items()}
    full = projector.state_dict()
    for k in full:
        if k.endswith("num_batches_tracked"):
            state[k] = full[k]
    projector.load_state_dict(state, strict=True)
    return JEPA(encoder=encoder, predictor=None, action_encoder=None, projector=projector).eval()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="reference checkout (its lewm/ is imported)")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "lewm"))
    sys.path.insert(0, str(Path(args.reference)))
    import torch

    torch.manual_seed(0)
    for name, (desc, wseed, pseed, (b, t)) in CASES.items():
        vit, proj = synthetic_weights(desc, wseed)
        model = build_reference(torch, desc, vit, proj)
        pix = synthetic_pixels(b * t, desc, pseed)
        info = {"pixels": torch.from_numpy(pix).reshape(b, t, *pix.shape[1:])}
        with torch.no_grad():
            emb = model.encode(info)["emb"].numpy()
        np.savez(HERE / f"encoder_{name}.npz", desc=json.dumps(asdict(desc)), weight_seed=wseed, pixel_seed=pseed,
                 bt=np.array([b, t]), checksum=weights_checksum(vit, proj),
                 pixel_checksum=float(np.float64(pix).sum()), emb=emb.astype(np.float32))
        print(name, emb.shape, float(np.abs(emb).max()))


if __name__ == "__main__":
    main()
