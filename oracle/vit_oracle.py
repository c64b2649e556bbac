"""ORACLE (test infrastructure only) -- numpy restatement of the observation encoder.

This module is the CPU checker for the B200 encoder kernels. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it; the
product package never does.

It restates ``JEPA.encode`` (reference ``lewm/jepa.py:88-104``): the CLS row of
``last_hidden_state`` of a transformers ``ViTModel`` (third-party: transformers,
built by stable-pretraining 0.1.7 ``vit_hf``, reference
``tools/benchmarks/stage_lewm_weights.py:72-78``; not vendored in the reference),
then the projector ``MLP`` (reference ``lewm/module.py:217-240``). The ViTModel
algorithm restated here is the published ViT forward (Dosovitskiy et al. 2021) as
transformers implements it:

* patch embedding: Conv2d(C, D, kernel = stride = patch) over the image, flattened
  row-major over the patch grid; CLS token prepended; learned position embedding
  added (no interpolation when the image matches the configured size);
* per layer (pre-norm): ``h = x + Wo . softmax(Q K^T / sqrt(64)) V`` with
  ``Q, K, V = LN_before(x) . W^T + b`` split into heads of 64, then
  ``x = h + W2 . GELU(W1 . LN_after(h) + b1) + b2``; LayerNorm eps from the config;
* final LayerNorm.

Parity is pinned two ways: ``tests/test_encoder_cpu.py`` runs the installed
transformers ``ViTModel`` on the same weights and compares, and
``tests/golden/make_encoder_golden.py`` runs the reference ``JEPA.encode`` with the
reference ``MLP`` projector and commits the embeddings as fixtures.

``operand_bf16=True`` rounds every tensor-core operand to bfloat16 at the points the
B200 kernels do (patch pixels, weights, LayerNorm outputs, Q, K, V, softmax
probabilities, attention output, GELU hidden, projector hidden), accumulating in
float32, so the GPU result can be checked against a tighter bound than against the
float32 forward.
"""

from __future__ import annotations

from typing import Mapping

import numpy as np

try:  # erf for the exact GELU (ViTConfig.hidden_act "gelu", nn.GELU())
    from scipy.special import erf as _erf
except Exception:  # pragma: no cover - scipy is in the image
    _erf = np.vectorize(__import__("math").erf)

F32 = np.float32


def bf16(a: np.ndarray) -> np.ndarray:
    """Round float32 to the nearest bfloat16 (ties to even), returned as float32."""
    u = np.ascontiguousarray(a, dtype=F32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(F32)


def layer_norm(x: np.ndarray, g, b, eps: float) -> np.ndarray:
    """torch.nn.functional.layer_norm over the last axis (biased variance)."""
    x = x.astype(F32)
    mu = x.mean(-1, keepdims=True, dtype=np.float64).astype(F32)
    var = ((x - mu) ** 2).mean(-1, keepdims=True, dtype=np.float64).astype(F32)
    y = (x - mu) / np.sqrt(var + F32(eps))
    if g is not None:
        y = y * g + b
    return y.astype(F32)


def gelu(x: np.ndarray) -> np.ndarray:
    return (0.5 * x * (1.0 + _erf(x / np.sqrt(2.0)))).astype(F32)


def _mm(a: np.ndarray, w: np.ndarray, rb: bool) -> np.ndarray:
    """a . w^T in float32 (operands rounded to bf16 when rb)."""
    if rb:
        a, w = bf16(a), bf16(w)
    return (a.astype(F32) @ w.astype(F32).T).astype(F32)


def patchify(pixels: np.ndarray, p: int) -> np.ndarray:
    """(N, C, H, W) -> (N, (H/p)(W/p), C p p) in Conv2d weight order, row-major over the grid."""
    n, c, h, w = pixels.shape
    g_h, g_w = h // p, w // p
    x = pixels.reshape(n, c, g_h, p, g_w, p).transpose(0, 2, 4, 1, 3, 5)
    return x.reshape(n, g_h * g_w, c * p * p).astype(F32)


def vit_cls(vit: Mapping[str, np.ndarray], desc, pixels: np.ndarray, operand_bf16: bool = False) -> np.ndarray:
    """CLS row of ViTModel.last_hidden_state: (N, hidden)."""
    rb = operand_bf16
    g = lambda k: np.asarray(vit[k], dtype=F32)  # noqa: E731
    D, H = desc.hidden, desc.heads
    dh = D // H
    n = pixels.shape[0]
    patches = patchify(np.asarray(pixels, dtype=F32), desc.patch_size)
    wp = g("embeddings.patch_embeddings.projection.weight").reshape(D, -1)
    tok = _mm(patches.reshape(-1, patches.shape[-1]), wp, rb).reshape(n, -1, D) + g(
        "embeddings.patch_embeddings.projection.bias")
    cls = np.broadcast_to(g("embeddings.cls_token").reshape(1, 1, D), (n, 1, D))
    x = np.concatenate([cls, tok], axis=1) + g("embeddings.position_embeddings").reshape(1, -1, D)
    x = x.astype(F32)
    T = x.shape[1]
    for i in range(desc.depth):
        p = f"encoder.layer.{i}."
        h = layer_norm(x, g(p + "layernorm_before.weight"), g(p + "layernorm_before.bias"), desc.ln_eps)
        h2 = h.reshape(-1, D)
        qkv = []
        for t in ("query", "key", "value"):
            y = _mm(h2, g(p + f"attention.attention.{t}.weight"), rb) + g(p + f"attention.attention.{t}.bias")
            y = y.reshape(n, T, H, dh).transpose(0, 2, 1, 3)  # (n, H, T, dh)
            qkv.append(bf16(y) if rb else y)
        q, k, v = qkv
        s = np.einsum("nhqd,nhkd->nhqk", q, k).astype(F32) / F32(np.sqrt(dh))
        s = s - s.max(-1, keepdims=True)
        e = np.exp(s).astype(F32)
        if rb:
            e = bf16(e)
        o = np.einsum("nhqk,nhkd->nhqd", e, v).astype(F32) / e.sum(-1, keepdims=True)
        o = o.transpose(0, 2, 1, 3).reshape(-1, D)
        x = x + (_mm(o, g(p + "attention.output.dense.weight"), rb) + g(p + "attention.output.dense.bias")).reshape(
            n, T, D)
        h = layer_norm(x, g(p + "layernorm_after.weight"), g(p + "layernorm_after.bias"), desc.ln_eps).reshape(-1, D)
        m = gelu(_mm(h, g(p + "intermediate.dense.weight"), rb) + g(p + "intermediate.dense.bias"))
        x = x + (_mm(m, g(p + "output.dense.weight"), rb) + g(p + "output.dense.bias")).reshape(n, T, D)
        x = x.astype(F32)
    return layer_norm(x[:, 0], g("layernorm.weight"), g("layernorm.bias"), desc.ln_eps)


def projector(proj: Mapping[str, np.ndarray], desc, x: np.ndarray, operand_bf16: bool = False) -> np.ndarray:
    """Reference MLP (``lewm/module.py:217-240``): Linear -> norm -> GELU -> Linear (eval mode)."""
    rb = operand_bf16
    g = lambda k: np.asarray(proj[k], dtype=F32)  # noqa: E731
    h = _mm(x, g("net.0.weight"), rb) + g("net.0.bias")
    if desc.proj_norm == "layernorm":
        h = layer_norm(h, g("net.1.weight"), g("net.1.bias"), desc.proj_eps)
    elif desc.proj_norm == "batchnorm":  # BatchNorm1d in eval: running statistics
        h = (h - g("net.1.running_mean")) / np.sqrt(g("net.1.running_var") + F32(desc.proj_eps)) * g(
            "net.1.weight") + g("net.1.bias")
    h = gelu(h.astype(F32))
    return (_mm(h, g("net.3.weight"), rb) + g("net.3.bias")).astype(F32)


def encode(vit, proj, desc, pixels: np.ndarray, operand_bf16: bool = False) -> np.ndarray:
    """JEPA.encode on (N, C, H, W) pixels -> (N, proj_out)."""
    return projector(proj, desc, vit_cls(vit, desc, pixels, operand_bf16), operand_bf16)


def img_transform(frames: np.ndarray, mean, std) -> np.ndarray:
    """Policy image transform (reference ``lewm/eval.py:17-26``: torchvision v2 ``ToImage``,
    ``ToDtype(float32, scale=True)``, ``Normalize``, ``Resize``) on uint8 frames (N, H, W, C)
    already at the target size: (u * float32(1/255) - mean) / std per channel, rounded
    after each float32 step, returned as (N, C, H, W)."""
    u = np.asarray(frames, dtype=np.uint8).astype(F32).transpose(0, 3, 1, 2)
    m = np.asarray(mean, dtype=F32).reshape(1, -1, 1, 1)
    s = np.asarray(std, dtype=F32).reshape(1, -1, 1, 1)
    return ((u * F32(1.0 / 255.0)) - m) / s


def synthetic_frames(n: int, desc, seed: int) -> np.ndarray:
    """Seeded uint8 frames (N, H, W, C) standing in for rendered observations."""
    rng = np.random.default_rng(seed)
    return rng.integers(0, 256, size=(n, desc.image_size, desc.image_size, desc.channels), dtype=np.uint8)


def synthetic_pixels(n: int, desc, seed: int) -> np.ndarray:
    """Seeded stand-in for normalized observations: uint8 noise images through the
    ImageNet mean / std normalization the policy applies (values about -2.1 .. 2.6)."""
    rng = np.random.default_rng(seed)
    raw = rng.integers(0, 256, size=(n, desc.channels, desc.image_size, desc.image_size)).astype(F32) / 255.0
    mean = np.array([0.485, 0.456, 0.406][: desc.channels], dtype=F32).reshape(1, -1, 1, 1)
    std = np.array([0.229, 0.224, 0.225][: desc.channels], dtype=F32).reshape(1, -1, 1, 1)
    return ((raw - mean) / std).astype(F32)
