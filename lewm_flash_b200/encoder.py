"""Observation encoder on the B200 kernels: ``JEPA.encode`` (reference ``lewm/jepa.py:88-104``).

The reference encodes pixels with a transformers ``ViTModel`` (stable-pretraining
0.1.7 ``vit_hf``, reference ``tools/benchmarks/stage_lewm_weights.py:72-78``), keeps the
CLS row of ``last_hidden_state`` and applies the projector ``MLP`` (reference
``lewm/module.py:217-240``). The planner reaches it through
``JEPA._ensure_cost_embeddings`` (reference ``lewm/jepa.py:319-345``) whenever
``info_dict`` carries pixels instead of cached embeddings.

``B200Encoder`` runs that whole step through ``lewm_encode`` (``include/lewm_b200.h``);
``install_encoder(model)`` swaps ``model.encode`` for it, so the reference's own
``_ensure_cost_embeddings`` and every solver on top of it use the B200 kernels.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Any, Callable, Optional

import numpy as np
import torch

from . import _lib

NORMS = ("none", "layernorm", "batchnorm")
# ImageNet statistics of the policy image transform (reference lewm/eval.py:17-26).
IMAGENET_MEAN = (0.485, 0.456, 0.406)
IMAGENET_STD = (0.229, 0.224, 0.225)


@dataclass
class EncoderDesc:
    """ViTConfig fields plus the projector MLP shape (defaults: ViT-tiny, patch 14, 224 px)."""

    image_size: int = 224
    patch_size: int = 14
    channels: int = 3
    hidden: int = 192
    depth: int = 12
    heads: int = 3
    mlp_dim: int = 768
    ln_eps: float = 1e-12
    proj_hidden: int = 2048
    proj_out: int = 192
    proj_norm: str = "batchnorm"
    proj_eps: float = 1e-5

    @property
    def tokens(self) -> int:
        return (self.image_size // self.patch_size) ** 2 + 1

    def c(self) -> _lib.EncoderDescC:
        if self.proj_norm not in NORMS:
            raise ValueError(f"proj_norm must be one of {NORMS}, got {self.proj_norm!r}")
        return _lib.EncoderDescC(self.image_size, self.patch_size, self.channels, self.hidden, self.depth, self.heads,
                                 self.mlp_dim, float(self.ln_eps), self.proj_hidden, self.proj_out,
                                 _lib.NORM_CODE[self.proj_norm], float(self.proj_eps))


def vit_param_names(desc: EncoderDesc) -> list[str]:
    """ViTModel state-dict names in ``lewm_encoder_create`` order."""
    names = ["embeddings.cls_token", "embeddings.position_embeddings",
             "embeddings.patch_embeddings.projection.weight", "embeddings.patch_embeddings.projection.bias"]
    for i in range(desc.depth):
        p = f"encoder.layer.{i}."
        names += [p + "layernorm_before.weight", p + "layernorm_before.bias"]
        for t in ("query", "key", "value"):
            names += [p + f"attention.attention.{t}.weight", p + f"attention.attention.{t}.bias"]
        names += [p + "attention.output.dense.weight", p + "attention.output.dense.bias",
                  p + "layernorm_after.weight", p + "layernorm_after.bias",
                  p + "intermediate.dense.weight", p + "intermediate.dense.bias",
                  p + "output.dense.weight", p + "output.dense.bias"]
    return names + ["layernorm.weight", "layernorm.bias"]


def projector_param_names(desc: EncoderDesc) -> list[str]:
    """Projector ``MLP`` (``nn.Sequential`` of Linear, norm, GELU, Linear) state-dict names."""
    norm = {"none": [], "layernorm": ["net.1.weight", "net.1.bias"],
            "batchnorm": ["net.1.weight", "net.1.bias", "net.1.running_mean", "net.1.running_var"]}[desc.proj_norm]
    return ["net.0.weight", "net.0.bias", *norm, "net.3.weight", "net.3.bias"]


def flat_weights(vit_state: dict, proj_state: dict, desc: EncoderDesc) -> np.ndarray:
    """Concatenate ViTModel + projector tensors into the float32 vector ``lewm_encoder_create`` takes."""
    parts = []
    for n in vit_param_names(desc):
        parts.append(np.asarray(_np(vit_state[n]), dtype=np.float32).reshape(-1))
    for n in projector_param_names(desc):
        parts.append(np.asarray(_np(proj_state[n]), dtype=np.float32).reshape(-1))
    return np.ascontiguousarray(np.concatenate(parts))


def _np(t) -> np.ndarray:
    return t.detach().float().cpu().numpy() if torch.is_tensor(t) else np.asarray(t)


def synthetic_weights(desc: EncoderDesc, seed: int = 0) -> tuple[dict, dict]:
    """Seeded random ViT + projector state dicts (numpy float32) with the reference shapes.

    Weights N(0, 0.02) like the ViT initializer, LayerNorm / BatchNorm affines near 1 / 0,
    BatchNorm running statistics away from the identity so the folding is exercised.
    """
    rng = np.random.default_rng(seed)
    D, M, P, T = desc.hidden, desc.mlp_dim, desc.proj_hidden, desc.tokens

    def w(*shape, s=0.02):
        return (rng.standard_normal(shape) * s).astype(np.float32)

    def gamma(n):
        return (1.0 + rng.standard_normal(n) * 0.05).astype(np.float32)

    vit = {"embeddings.cls_token": w(1, 1, D), "embeddings.position_embeddings": w(1, T, D),
           "embeddings.patch_embeddings.projection.weight": w(D, desc.channels, desc.patch_size, desc.patch_size),
           "embeddings.patch_embeddings.projection.bias": w(D)}
    for i in range(desc.depth):
        p = f"encoder.layer.{i}."
        vit[p + "layernorm_before.weight"], vit[p + "layernorm_before.bias"] = gamma(D), w(D)
        for t in ("query", "key", "value"):
            vit[p + f"attention.attention.{t}.weight"] = w(D, D, s=0.06)
            vit[p + f"attention.attention.{t}.bias"] = w(D)
        vit[p + "attention.output.dense.weight"], vit[p + "attention.output.dense.bias"] = w(D, D), w(D)
        vit[p + "layernorm_after.weight"], vit[p + "layernorm_after.bias"] = gamma(D), w(D)
        vit[p + "intermediate.dense.weight"], vit[p + "intermediate.dense.bias"] = w(M, D, s=0.04), w(M)
        vit[p + "output.dense.weight"], vit[p + "output.dense.bias"] = w(D, M), w(D)
    vit["layernorm.weight"], vit["layernorm.bias"] = gamma(D), w(D)
    proj = {"net.0.weight": w(P, D, s=0.05), "net.0.bias": w(P),
            "net.3.weight": w(desc.proj_out, P, s=0.02), "net.3.bias": w(desc.proj_out)}
    if desc.proj_norm == "layernorm":
        proj["net.1.weight"], proj["net.1.bias"] = gamma(P), w(P)
    elif desc.proj_norm == "batchnorm":
        proj["net.1.weight"], proj["net.1.bias"] = gamma(P), w(P)
        proj["net.1.running_mean"] = (rng.standard_normal(P) * 0.1).astype(np.float32)
        proj["net.1.running_var"] = rng.uniform(0.5, 1.5, P).astype(np.float32)
    return vit, proj


def desc_from_modules(vit_model, projector) -> EncoderDesc:
    """EncoderDesc of a transformers ViTModel and a reference projector ``MLP``."""
    cfg = vit_model.config
    lin0, norm, _, lin3 = list(projector.net)
    if isinstance(norm, torch.nn.BatchNorm1d):
        kind, eps = "batchnorm", float(norm.eps)
    elif isinstance(norm, torch.nn.LayerNorm):
        kind, eps = "layernorm", float(norm.eps)
    else:
        kind, eps = "none", 1e-5
    size = cfg.image_size if isinstance(cfg.image_size, int) else cfg.image_size[0]
    patch = cfg.patch_size if isinstance(cfg.patch_size, int) else cfg.patch_size[0]
    return EncoderDesc(image_size=size, patch_size=patch, channels=cfg.num_channels, hidden=cfg.hidden_size,
                       depth=cfg.num_hidden_layers, heads=cfg.num_attention_heads, mlp_dim=cfg.intermediate_size,
                       ln_eps=float(cfg.layer_norm_eps), proj_hidden=lin0.out_features, proj_out=lin3.out_features,
                       proj_norm=kind, proj_eps=eps)


def encoder_flops(desc: EncoderDesc) -> float:
    """Algorithmic FLOPs of one image: patch GEMM, per layer QKV / attention scores and
    values / out-proj / MLP over all tokens, projector on the CLS row (norms excluded)."""
    T, D, M, P = desc.tokens, desc.hidden, desc.mlp_dim, desc.proj_hidden
    k_patch = desc.channels * desc.patch_size ** 2
    layer = 2 * T * (3 * D * D + D * D + 2 * D * M) + 4 * T * T * D
    return float(2 * (T - 1) * k_patch * D + desc.depth * layer + 2 * D * P + 2 * P * desc.proj_out)


def encoder_launches(desc: EncoderDesc) -> int:
    """Kernel launches of one ``lewm_encode`` call."""
    return 2 + 5 * desc.depth + 1 + (3 if desc.proj_norm == "layernorm" else 2)


def weight_count(desc: EncoderDesc) -> int:
    return int(_lib.lib().lewm_encoder_weight_count(C.byref(desc.c())))


class B200Encoder:
    """pixels (N, C, H, W) float32 -> embeddings (N, proj_out) float32 on the B200 kernels."""

    def __init__(self, desc: EncoderDesc, weights: np.ndarray, device: Any = "cuda",
                 action_encoder: Optional[Callable] = None):
        self.desc = desc
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.action_encoder = action_encoder
        w = np.ascontiguousarray(weights, dtype=np.float32)
        lib = _lib.lib()
        self._enc = C.c_void_p()
        _lib.check_encoder(lib.lewm_encoder_create(C.byref(self._enc), C.byref(desc.c()),
                                                   w.ctypes.data_as(C.c_void_p), w.size, self.device.index))

    @classmethod
    def from_modules(cls, vit_model, projector, device: Any = "cuda", action_encoder=None) -> "B200Encoder":
        desc = desc_from_modules(vit_model, projector)
        return cls(desc, flat_weights(vit_model.state_dict(), projector.state_dict(), desc), device, action_encoder)

    def __del__(self):
        enc = getattr(self, "_enc", None)
        if enc is not None and enc.value:
            try:
                _lib.lib().lewm_encoder_destroy(enc)
            except Exception:
                pass
            self._enc = None

    def encode_pixels(self, pixels: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """ViT CLS row + projector for a batch of images (device tensors, stream-ordered)."""
        d = self.desc
        if pixels.ndim != 4 or tuple(pixels.shape[1:]) != (d.channels, d.image_size, d.image_size):
            raise ValueError(f"pixels must be (N, {d.channels}, {d.image_size}, {d.image_size}), "
                             f"got {tuple(pixels.shape)}")
        pix = pixels.to(device=self.device, dtype=torch.float32).contiguous()
        n = pix.shape[0]
        if out is None:
            out = torch.empty(n, d.proj_out, device=self.device, dtype=torch.float32)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check_encoder(_lib.lib().lewm_encode(self._enc, C.c_void_p(pix.data_ptr()), n,
                                                  C.c_void_p(out.data_ptr()), C.c_void_p(stream)), self._enc)
        return out

    def encode_frames(self, frames: torch.Tensor, mean=IMAGENET_MEAN, std=IMAGENET_STD,
                      out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Raw uint8 frames (N, H, W, C) -> embeddings: the policy image transform
        (``ToImage``, ``ToDtype(float32, scale=True)``, ``Normalize``, ``Resize`` to the encoder
        size; reference ``lewm/eval.py:17-26``) fused into the encoder's first kernel. Frames
        must already be at the encoder size, where that ``Resize`` is the identity."""
        d = self.desc
        if frames.dtype != torch.uint8 or frames.ndim != 4 or tuple(frames.shape[1:]) != (
                d.image_size, d.image_size, d.channels):
            raise ValueError(f"frames must be uint8 (N, {d.image_size}, {d.image_size}, {d.channels}), "
                             f"got {frames.dtype} {tuple(frames.shape)}")
        if len(mean) != d.channels or len(std) != d.channels:
            raise ValueError("mean / std need one value per channel")
        fr = frames.to(self.device).contiguous()
        n = fr.shape[0]
        if out is None:
            out = torch.empty(n, d.proj_out, device=self.device, dtype=torch.float32)
        m = (C.c_float * d.channels)(*[float(v) for v in mean])
        sd = (C.c_float * d.channels)(*[float(v) for v in std])
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check_encoder(_lib.lib().lewm_encode_u8(self._enc, C.c_void_p(fr.data_ptr()), n, m, sd,
                                                     C.c_void_p(out.data_ptr()), C.c_void_p(stream)), self._enc)
        return out

    def sync(self) -> None:
        """Synchronize the current stream and raise if a bounded device wait expired."""
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check_encoder(_lib.lib().lewm_encoder_sync_status(self._enc, C.c_void_p(stream)), self._enc)

    def encode(self, info: dict) -> dict:
        """``JEPA.encode`` (reference ``lewm/jepa.py:88-104``): info["pixels"] (b, t, C, H, W) -> info["emb"]
        (b, t, proj_out); info["act_emb"] from the model's action encoder when "action" is present."""
        pixels = info["pixels"].float()
        b, t = pixels.shape[:2]
        emb = self.encode_pixels(pixels.reshape(b * t, *pixels.shape[2:]))
        info["emb"] = emb.reshape(b, t, -1)
        if "action" in info:
            if self.action_encoder is None:
                raise RuntimeError("info has 'action' but the encoder was built without an action encoder")
            info["act_emb"] = self.action_encoder(info["action"])
        return info

    __call__ = encode


def install_encoder(model, device: Any = "cuda") -> B200Encoder:
    """Route ``model.encode`` (and so ``JEPA._ensure_cost_embeddings`` and the solvers that call it)
    through the B200 encoder built from ``model.encoder`` and ``model.projector``."""
    enc = B200Encoder.from_modules(model.encoder, model.projector, device,
                                   action_encoder=getattr(model, "action_encoder", None))
    model.encode = enc.encode
    return enc
