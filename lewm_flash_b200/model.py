"""LeWM predictor description, seeded synthetic weights and state-dict plumbing.

The predictor stack mirrors the reference modules:

* ``ARPredictor`` (reference ``lewm/module.py:244-285``): learned position
  embedding of ``num_frames`` rows, a ``Transformer`` of ``depth``
  ``ConditionalBlock`` layers (AdaLN-zero, ``lewm/module.py:88-111``) and a
  final affine ``LayerNorm`` (``lewm/module.py:147,183``).
* ``Embedder`` action encoder (``lewm/module.py:189-214``): Conv1d(k=1),
  Linear, SiLU, Linear.
* optional ``pred_proj`` head ``MLP`` (``lewm/module.py:217-240``).

Parameter names are the reference ``JEPA`` state-dict names
(``predictor.*``, ``action_encoder.*``, ``pred_proj.*``) so a trained
reference checkpoint loads unchanged.
"""

from __future__ import annotations

import dataclasses
from dataclasses import dataclass
from typing import Dict, Mapping

import numpy as np

NORM_KINDS = ("none", "layernorm", "batchnorm")


@dataclass(frozen=True)
class ModelDesc:
    """Static shape of one LeWM predictor + action encoder.

    Defaults are the LeWM Push-T predictor: width 192, 6 layers, 16 heads of
    64, MLP 4x, action dim 2 x frameskip 5 = 10 (reference
    ``lewm/module.py:247-262``; ``lewm/config/eval/pusht.yaml``).
    """

    dim: int = 192
    depth: int = 6
    heads: int = 16
    dim_head: int = 64
    mlp_dim: int = 768
    action_dim: int = 10
    smoothed_dim: int = 10
    embed_hidden: int = 768
    num_frames: int = 3
    pred_proj_hidden: int = 0
    pred_proj_norm: str = "none"

    def __post_init__(self) -> None:
        if self.pred_proj_norm not in NORM_KINDS:
            raise ValueError(f"pred_proj_norm must be one of {NORM_KINDS}, got {self.pred_proj_norm!r}")
        for name in ("dim", "depth", "heads", "dim_head", "mlp_dim", "action_dim",
                     "smoothed_dim", "embed_hidden", "num_frames"):
            if getattr(self, name) <= 0:
                raise ValueError(f"{name} must be positive, got {getattr(self, name)}")
        if self.pred_proj_hidden < 0:
            raise ValueError("pred_proj_hidden must be >= 0")

    @property
    def inner_dim(self) -> int:
        return self.heads * self.dim_head

    def replace(self, **kw) -> "ModelDesc":
        return dataclasses.replace(self, **kw)


# Scaled-stress predictor: width 384, 12 layers, horizon 10.
STRESS_DESC = ModelDesc(dim=384, depth=12, heads=16, dim_head=64, mlp_dim=1536,
                        action_dim=10, smoothed_dim=10, embed_hidden=1536, num_frames=3)


def param_shapes(desc: ModelDesc) -> Dict[str, tuple]:
    """Reference state-dict names and shapes, in canonical (packing) order."""
    D, inner, mlp = desc.dim, desc.inner_dim, desc.mlp_dim
    shapes: Dict[str, tuple] = {}
    p = "predictor."
    shapes[p + "pos_embedding"] = (1, desc.num_frames, D)
    for l in range(desc.depth):
        q = f"{p}transformer.layers.{l}."
        shapes[q + "adaLN_modulation.1.weight"] = (6 * D, D)
        shapes[q + "adaLN_modulation.1.bias"] = (6 * D,)
        shapes[q + "attn.norm.weight"] = (D,)
        shapes[q + "attn.norm.bias"] = (D,)
        shapes[q + "attn.to_qkv.weight"] = (3 * inner, D)
        shapes[q + "attn.to_out.0.weight"] = (D, inner)
        shapes[q + "attn.to_out.0.bias"] = (D,)
        shapes[q + "mlp.net.0.weight"] = (D,)
        shapes[q + "mlp.net.0.bias"] = (D,)
        shapes[q + "mlp.net.1.weight"] = (mlp, D)
        shapes[q + "mlp.net.1.bias"] = (mlp,)
        shapes[q + "mlp.net.4.weight"] = (D, mlp)
        shapes[q + "mlp.net.4.bias"] = (D,)
    shapes[p + "transformer.norm.weight"] = (D,)
    shapes[p + "transformer.norm.bias"] = (D,)
    a = "action_encoder."
    shapes[a + "patch_embed.weight"] = (desc.smoothed_dim, desc.action_dim, 1)
    shapes[a + "patch_embed.bias"] = (desc.smoothed_dim,)
    shapes[a + "embed.0.weight"] = (desc.embed_hidden, desc.smoothed_dim)
    shapes[a + "embed.0.bias"] = (desc.embed_hidden,)
    shapes[a + "embed.2.weight"] = (D, desc.embed_hidden)
    shapes[a + "embed.2.bias"] = (D,)
    if desc.pred_proj_hidden:
        h = desc.pred_proj_hidden
        shapes["pred_proj.net.0.weight"] = (h, D)
        shapes["pred_proj.net.0.bias"] = (h,)
        if desc.pred_proj_norm == "layernorm":
            shapes["pred_proj.net.1.weight"] = (h,)
            shapes["pred_proj.net.1.bias"] = (h,)
        elif desc.pred_proj_norm == "batchnorm":
            shapes["pred_proj.net.1.weight"] = (h,)
            shapes["pred_proj.net.1.bias"] = (h,)
            shapes["pred_proj.net.1.running_mean"] = (h,)
            shapes["pred_proj.net.1.running_var"] = (h,)
        shapes["pred_proj.net.3.weight"] = (D, h)
        shapes["pred_proj.net.3.bias"] = (D,)
    return shapes


def _is_norm_param(name: str) -> bool:
    """LayerNorm / BatchNorm affine parameters (attn.norm, FFN net.0, final norm, head norm)."""
    return (
        ".attn.norm." in name
        or ".mlp.net.0." in name
        or "transformer.norm." in name
        or name in ("pred_proj.net.1.weight", "pred_proj.net.1.bias")
    )


def synthetic_state_dict(desc: ModelDesc, seed: int = 0, adaln_scale: float = 1.0) -> Dict[str, np.ndarray]:
    """Seeded random-init weights with the reference parameter names.

    Linear layers use the PyTorch default bound U(+-1/sqrt(fan_in)); the
    position embedding is N(0, 1) as in ``ARPredictor.__init__``. LayerNorm
    affine parameters are perturbed away from (1, 0) so they are exercised.
    The AdaLN-zero modulation Linear is zero-initialised by the reference
    (``lewm/module.py:102-103``), which makes every block the identity; here it
    is re-randomised with bound ``adaln_scale/sqrt(dim)`` so every block and
    every action matters. Uses numpy's PCG64 stream, which is stable across
    numpy versions, so the same seed gives the same weights everywhere.
    """
    rng = np.random.default_rng(np.random.PCG64(seed))
    out: Dict[str, np.ndarray] = {}
    for name, shape in param_shapes(desc).items():
        if name.endswith("pos_embedding"):
            v = rng.standard_normal(shape)
        elif name.endswith("running_mean"):
            v = 0.1 * rng.standard_normal(shape)
        elif name.endswith("running_var"):
            v = rng.uniform(0.5, 1.5, shape)
        elif _is_norm_param(name):
            v = (1.0 + 0.1 * rng.standard_normal(shape)) if name.endswith("weight") else 0.05 * rng.standard_normal(shape)
        else:
            # Linear / Conv1d weight or bias: fan_in is the last weight dim(s).
            wname = name[: -len("bias")] + "weight" if name.endswith("bias") else name
            wshape = param_shapes(desc)[wname]
            fan_in = int(np.prod(wshape[1:]))
            bound = 1.0 / np.sqrt(fan_in)
            if "adaLN_modulation" in name:
                bound *= adaln_scale
            v = rng.uniform(-bound, bound, shape)
        out[name] = np.ascontiguousarray(v, dtype=np.float32)
    return out


def state_dict_checksum(sd: Mapping[str, np.ndarray]) -> float:
    """Order-independent float64 checksum used to pin regenerated weights."""
    return float(sum(np.asarray(v, dtype=np.float64).sum() * (1 + (i % 7)) for i, (k, v) in enumerate(sorted(sd.items()))))


def extract_state_dict(model, desc: ModelDesc) -> Dict[str, np.ndarray]:
    """Pull the hot-path parameters out of a reference ``JEPA`` module.

    Accepts any object whose ``state_dict()`` carries the reference names
    (``predictor.*``, ``action_encoder.*``, optional ``pred_proj.*``).
    """
    sd = model.state_dict()
    out: Dict[str, np.ndarray] = {}
    for name, shape in param_shapes(desc).items():
        if name not in sd:
            raise KeyError(f"model state_dict is missing {name!r}")
        t = sd[name]
        arr = t.detach().to("cpu").float().numpy() if hasattr(t, "detach") else np.asarray(t, dtype=np.float32)
        if tuple(arr.shape) != tuple(shape):
            raise ValueError(f"{name}: expected shape {shape}, got {tuple(arr.shape)}")
        out[name] = np.ascontiguousarray(arr, dtype=np.float32)
    return out


def infer_desc(model) -> ModelDesc:
    """Read a ``ModelDesc`` off a reference ``JEPA`` (predictor/action encoder/pred_proj)."""
    pred = model.predictor
    tr = pred.transformer
    blk = tr.layers[0]
    D = int(pred.pos_embedding.shape[-1])
    heads = int(blk.attn.heads)
    inner = int(blk.attn.to_qkv.weight.shape[0]) // 3
    enc = model.action_encoder
    pp_hidden, pp_norm = 0, "none"
    pp = getattr(model, "pred_proj", None)
    net = getattr(pp, "net", None)
    if net is not None:
        pp_hidden = int(net[0].weight.shape[0])
        kind = type(net[1]).__name__
        pp_norm = {"LayerNorm": "layernorm", "BatchNorm1d": "batchnorm", "Identity": "none"}[kind]
    if not isinstance(tr.input_proj, type(tr.norm)) and hasattr(tr.input_proj, "weight"):
        raise ValueError("predictor input/hidden/output widths must be equal (Identity projections)")
    return ModelDesc(
        dim=D,
        depth=len(tr.layers),
        heads=heads,
        dim_head=inner // heads,
        mlp_dim=int(blk.mlp.net[1].weight.shape[0]),
        action_dim=int(enc.patch_embed.weight.shape[1]),
        smoothed_dim=int(enc.patch_embed.weight.shape[0]),
        embed_hidden=int(enc.embed[0].weight.shape[0]),
        num_frames=int(pred.pos_embedding.shape[1]),
        pred_proj_hidden=pp_hidden,
        pred_proj_norm=pp_norm,
    )
