"""Observation encoder on the B200 kernels against the oracle and the reference fixtures.

Tolerances (max |gpu - ref| / max |ref| over the embedding batch): 1e-2 against the
bf16-operand oracle (the kernels' own rounding points), 2e-2 against the float32
forward and the reference JEPA.encode fixtures (bf16 operand rounding alone moves the
embedding by about 0.7 %). Rows of different images never mix, so batching is checked
bit-exactly.
"""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from lewm_flash_b200.encoder import B200Encoder, EncoderDesc, flat_weights, install_encoder, synthetic_weights  # noqa: E402
from oracle import vit_oracle as vo  # noqa: E402
from tests.test_encoder_cpu import ENCODER_CASES, load_case  # noqa: E402

pytestmark = pytest.mark.gpu


def rel(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


def run(enc: B200Encoder, pix: np.ndarray) -> np.ndarray:
    out = enc.encode_pixels(torch.from_numpy(pix).cuda())
    enc.sync()
    return out.cpu().numpy()


@pytest.fixture(scope="module")
def full():
    desc = EncoderDesc()
    vit, proj = synthetic_weights(desc, 7)
    return desc, vit, proj, B200Encoder(desc, flat_weights(vit, proj, desc))


def test_full_size_encoder_matches_oracle(full):
    """224 px, patch 14 (257 tokens), 12 layers, 2048-wide BatchNorm projector."""
    desc, vit, proj, enc = full
    pix = vo.synthetic_pixels(3, desc, 8)
    got = run(enc, pix)
    assert np.isfinite(got).all()
    e16 = vo.encode(vit, proj, desc, pix, operand_bf16=True)
    e32 = vo.encode(vit, proj, desc, pix)
    assert rel(got, e16) <= 1e-2, rel(got, e16)
    assert rel(got, e32) <= 2e-2, rel(got, e32)


def test_batch_rows_are_independent_bits(full):
    """An image's embedding does not depend on the batch it is encoded in."""
    desc, _, _, enc = full
    pix = vo.synthetic_pixels(5, desc, 9)
    batched = run(enc, pix)
    for i in range(5):
        np.testing.assert_array_equal(run(enc, pix[i:i + 1])[0], batched[i])


@pytest.mark.parametrize("name", ENCODER_CASES)
def test_encoder_matches_reference_fixture(name):
    """LayerNorm / BatchNorm / no projector norm, patch 14 and 16, against JEPA.encode outputs."""
    desc, vit, proj, pix, want = load_case(name)
    enc = B200Encoder(desc, flat_weights(vit, proj, desc))
    got = run(enc, pix)
    assert rel(got, want) <= 2e-2, rel(got, want)
    assert rel(got, vo.encode(vit, proj, desc, pix, operand_bf16=True)) <= 1e-2


@pytest.mark.parametrize("image_size,patch_size", [(224, 16), (112, 14)])
def test_attention_geometries(image_size, patch_size):
    """197 tokens (two query tiles, one S MMA of N 208, the second warpgroup on keys 144..207)
    and 65 tokens (one query tile, N 80) against the oracle."""
    desc = EncoderDesc(image_size=image_size, patch_size=patch_size, depth=2, proj_hidden=512)
    vit, proj = synthetic_weights(desc, 15)
    enc = B200Encoder(desc, flat_weights(vit, proj, desc))
    pix = vo.synthetic_pixels(3, desc, 16)
    got = run(enc, pix)
    assert rel(got, vo.encode(vit, proj, desc, pix, operand_bf16=True)) <= 1e-2
    assert rel(got, vo.encode(vit, proj, desc, pix)) <= 2e-2


def test_more_than_one_tile_of_images_and_workspace_growth():
    """130 images: the CLS / projector GEMMs span two 128-row tiles; the workspace grows
    from a smaller batch and the results do not depend on the history of the encoder."""
    desc = EncoderDesc(image_size=56, depth=2, proj_hidden=512)
    vit, proj = synthetic_weights(desc, 10)
    enc = B200Encoder(desc, flat_weights(vit, proj, desc))
    pix = vo.synthetic_pixels(130, desc, 11)
    small = run(enc, pix[:3])
    got = run(enc, pix)
    np.testing.assert_array_equal(got[:3], small)
    assert rel(got, vo.encode(vit, proj, desc, pix, operand_bf16=True)) <= 1e-2
    assert enc.encode_pixels(torch.empty(0, 3, 56, 56, device="cuda")).shape == (0, desc.proj_out)


def test_pixels_of_the_wrong_size_raise():
    desc = EncoderDesc(image_size=56, depth=1, proj_hidden=256)
    vit, proj = synthetic_weights(desc, 1)
    enc = B200Encoder(desc, flat_weights(vit, proj, desc))
    with pytest.raises(ValueError):
        enc.encode_pixels(torch.zeros(1, 3, 64, 64, device="cuda"))


def test_install_encoder_routes_model_encode():
    """install_encoder swaps model.encode (JEPA.encode semantics: (b, t) pixels -> (b, t, D) emb)."""
    transformers = pytest.importorskip("transformers")
    desc = EncoderDesc(image_size=56, depth=2, proj_hidden=512, proj_norm="batchnorm")
    vit, proj = synthetic_weights(desc, 12)
    cfg = transformers.ViTConfig(hidden_size=desc.hidden, num_hidden_layers=desc.depth,
                                 num_attention_heads=desc.heads, intermediate_size=desc.mlp_dim,
                                 image_size=desc.image_size, patch_size=desc.patch_size,
                                 num_channels=desc.channels, layer_norm_eps=desc.ln_eps)

    class Projector(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.net = torch.nn.Sequential(torch.nn.Linear(desc.hidden, desc.proj_hidden),
                                           torch.nn.BatchNorm1d(desc.proj_hidden), torch.nn.GELU(),
                                           torch.nn.Linear(desc.proj_hidden, desc.proj_out))

    model = torch.nn.Module()
    model.encoder = transformers.ViTModel(cfg, add_pooling_layer=False).eval()
    model.encoder.load_state_dict({k: torch.from_numpy(v) for k, v in vit.items()}, strict=True)
    model.projector = Projector().eval()
    sd = {k: torch.from_numpy(v) for k, v in proj.items()}
    sd["net.1.num_batches_tracked"] = torch.tensor(0)
    model.projector.load_state_dict(sd, strict=True)
    enc = install_encoder(model)
    assert enc.desc == desc
    pix = vo.synthetic_pixels(4, desc, 13)
    info = model.encode({"pixels": torch.from_numpy(pix).reshape(2, 2, *pix.shape[1:]).cuda()})
    enc.sync()
    got = info["emb"].cpu().numpy()
    assert got.shape == (2, 2, desc.proj_out)
    assert rel(got.reshape(4, -1), vo.encode(vit, proj, desc, pix)) <= 2e-2


def test_uint8_frames_equal_transformed_pixels_bits(full):
    """lewm_encode_u8 (policy image transform fused into the first kernel) equals lewm_encode
    on the oracle-transformed float pixels bit for bit, and rejects frames of another size."""
    from lewm_flash_b200.encoder import IMAGENET_MEAN, IMAGENET_STD

    desc, _, _, enc = full
    frames = vo.synthetic_frames(3, desc, 14)
    got = enc.encode_frames(torch.from_numpy(frames).cuda())
    enc.sync()
    want = run(enc, vo.img_transform(frames, IMAGENET_MEAN, IMAGENET_STD))
    np.testing.assert_array_equal(got.cpu().numpy(), want)
    with pytest.raises(ValueError):
        enc.encode_frames(torch.zeros(1, 112, 112, 3, dtype=torch.uint8, device="cuda"))
