"""Observation encoder: oracle pinned to the reference and to transformers, host-side checks.

The reference step is ``JEPA.encode`` (reference ``lewm/jepa.py:88-104``): CLS row of a
transformers ``ViTModel`` and the projector ``MLP`` (reference ``lewm/module.py:217-240``).
"""

from __future__ import annotations

import ctypes as C
import json
from dataclasses import asdict

import numpy as np
import pytest

from lewm_flash_b200 import _lib
from lewm_flash_b200.encoder import (EncoderDesc, flat_weights, projector_param_names, synthetic_weights,
                                     vit_param_names, weight_count)
from oracle import vit_oracle as vo
from tests.conftest import GOLDEN

ENCODER_CASES = sorted(p.name for p in GOLDEN.glob("encoder_*.npz"))


def load_case(name):
    d = np.load(GOLDEN / name, allow_pickle=False)
    desc = EncoderDesc(**json.loads(str(d["desc"])))
    vit, proj = synthetic_weights(desc, int(d["weight_seed"]))
    from tests.golden.make_encoder_golden import weights_checksum

    assert abs(weights_checksum(vit, proj) - float(d["checksum"])) <= 1e-9 * max(1.0, abs(float(d["checksum"])))
    b, t = (int(x) for x in d["bt"])
    pix = vo.synthetic_pixels(b * t, desc, int(d["pixel_seed"]))
    assert abs(float(np.float64(pix).sum()) - float(d["pixel_checksum"])) <= 1e-6 * abs(float(d["pixel_checksum"]))
    return desc, vit, proj, pix, d["emb"].reshape(b * t, -1)


def test_encoder_fixtures_exist():
    assert len(ENCODER_CASES) >= 3


@pytest.mark.parametrize("name", ENCODER_CASES)
def test_oracle_matches_reference_jepa_encode(name):
    """The numpy restatement equals the reference JEPA.encode (ViTModel + MLP projector) output."""
    desc, vit, proj, pix, want = load_case(name)
    got = vo.encode(vit, proj, desc, pix)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=2e-5)


def test_oracle_matches_transformers_vit_full_size():
    """224 px, patch 14, 12 layers: the restated ViT forward against the installed ViTModel."""
    torch = pytest.importorskip("torch")
    transformers = pytest.importorskip("transformers")
    desc = EncoderDesc()
    vit, _ = synthetic_weights(desc, 3)
    cfg = transformers.ViTConfig(hidden_size=desc.hidden, num_hidden_layers=desc.depth,
                                 num_attention_heads=desc.heads, intermediate_size=desc.mlp_dim,
                                 image_size=desc.image_size, patch_size=desc.patch_size,
                                 num_channels=desc.channels, layer_norm_eps=desc.ln_eps)
    m = transformers.ViTModel(cfg, add_pooling_layer=False).eval()
    m.load_state_dict({k: torch.from_numpy(v) for k, v in vit.items()}, strict=True)
    pix = vo.synthetic_pixels(2, desc, 4)
    with torch.no_grad():
        ref = m(torch.from_numpy(pix), interpolate_pos_encoding=True).last_hidden_state[:, 0].numpy()
    np.testing.assert_allclose(vo.vit_cls(vit, desc, pix), ref, rtol=1e-4, atol=2e-5)


def test_bf16_operand_mode_stays_near_float32():
    """The bf16-operand oracle (the GPU numerics) is within 1e-2 of the float32 forward, max-normalized."""
    desc = EncoderDesc(image_size=56, depth=4)
    vit, proj = synthetic_weights(desc, 5)
    pix = vo.synthetic_pixels(3, desc, 6)
    a = vo.encode(vit, proj, desc, pix)
    b = vo.encode(vit, proj, desc, pix, operand_bf16=True)
    assert 0 < np.abs(a - b).max() / np.abs(a).max() < 1e-2


def test_bf16_rounding_is_nearest_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -3.0e-3, 65504.0], dtype=np.float32)
    got = vo.bf16(x)
    import torch

    want = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("norm", ["none", "layernorm", "batchnorm"])
def test_weight_count_matches_state_dicts(norm):
    desc = EncoderDesc(proj_norm=norm)
    vit, proj = synthetic_weights(desc, 0)
    assert set(vit) == set(vit_param_names(desc))
    assert set(proj) == set(projector_param_names(desc))
    assert weight_count(desc) == flat_weights(vit, proj, desc).size


@pytest.mark.parametrize("kw,status", [
    (dict(hidden=384, heads=6), "LEWM_UNSUPPORTED_SHAPE"),
    (dict(image_size=256, patch_size=14), "LEWM_UNSUPPORTED_SHAPE"),
    (dict(image_size=448, patch_size=14), "LEWM_UNSUPPORTED_SHAPE"),   # 1025 tokens > 272
    (dict(proj_hidden=2000), "LEWM_UNSUPPORTED_SHAPE"),
    (dict(proj_out=256), "LEWM_UNSUPPORTED_SHAPE"),
    (dict(mlp_dim=700), "LEWM_UNSUPPORTED_SHAPE"),
    (dict(depth=0), "LEWM_INVALID_ARG"),
    (dict(ln_eps=0.0), "LEWM_INVALID_ARG"),
])
def test_unsupported_encoder_desc_is_rejected_before_device_work(kw, status):
    desc = EncoderDesc(**kw)
    lib = _lib.lib()
    assert lib.lewm_encoder_weight_count(C.byref(desc.c())) == 0
    enc = C.c_void_p()
    w = np.zeros(8, np.float32)
    st = lib.lewm_encoder_create(C.byref(enc), C.byref(desc.c()), w.ctypes.data_as(C.c_void_p), w.size, 0)
    assert _lib.STATUS[st] == status
    assert not enc.value
    assert lib.lewm_encoder_last_error(None)


def test_wrong_weight_length_is_invalid_arg():
    desc = EncoderDesc(image_size=56, depth=1)
    n = weight_count(desc)
    w = np.zeros(n - 1, np.float32)
    enc = C.c_void_p()
    st = _lib.lib().lewm_encoder_create(C.byref(enc), C.byref(desc.c()), w.ctypes.data_as(C.c_void_p), w.size, 0)
    assert _lib.STATUS[st] == "LEWM_INVALID_ARG"
    assert b"expected" in _lib.lib().lewm_encoder_last_error(None)


def test_unknown_projector_norm_raises_value_error():
    with pytest.raises(ValueError):
        EncoderDesc(proj_norm="groupnorm").c()


def test_desc_round_trips_through_json():
    desc = EncoderDesc(image_size=64, patch_size=16)
    assert EncoderDesc(**json.loads(json.dumps(asdict(desc)))) == desc
    assert desc.tokens == 17


def test_img_transform_matches_torchvision_policy_transform():
    """The oracle's frame normalization equals the reference transform bit for bit
    (lewm/eval.py:17-26: ToImage, ToDtype(float32, scale=True), Normalize, Resize)."""
    torch = pytest.importorskip("torch")
    tv = pytest.importorskip("torchvision.transforms.v2")
    from lewm_flash_b200.encoder import IMAGENET_MEAN, IMAGENET_STD

    desc = EncoderDesc()
    frames = vo.synthetic_frames(2, desc, 3)
    tf = tv.Compose([tv.ToImage(), tv.ToDtype(torch.float32, scale=True),
                     tv.Normalize(mean=list(IMAGENET_MEAN), std=list(IMAGENET_STD)), tv.Resize(size=desc.image_size)])
    want = np.stack([tf(f).numpy() for f in frames])
    got = vo.img_transform(frames, IMAGENET_MEAN, IMAGENET_STD)
    np.testing.assert_array_equal(got, want)
