"""ORACLE (test infrastructure only) -- numpy restatement of the LeWM model-cost path.

This module is the CPU checker for the CUDA path. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import it; the product package never does.

It restates, in float32 numpy, the reference's tensor-only model cost
``JEPA.get_cost_from_embeddings`` (reference ``lewm/jepa.py:302-317``):

* ``rollout_from_embeddings`` -- ``lewm/jepa.py:262-300``
* ``JEPA.predict`` + ``pred_proj`` -- ``lewm/jepa.py:106-114``
* ``ARPredictor`` / ``Transformer`` / ``ConditionalBlock`` / ``Attention`` /
  ``FeedForward`` / ``modulate`` -- ``lewm/module.py:6-8,38-111,131-187,244-285``
* ``Embedder`` -- ``lewm/module.py:189-214``
* ``MLP`` head -- ``lewm/module.py:217-240``
* ``cost_from_rollout`` -- ``lewm/jepa.py:246-260``

Parity is pinned against the reference itself: ``tests/golden/make_golden.py``
imports the reference classes, runs them on seeded weights and inputs, and
commits the outputs as fixtures that ``tests/test_oracle_golden.py`` checks.

The action encoder is evaluated once over the whole action sequence instead of
on the growing prefix each step; the Embedder is per-timestep, and the
reference's own test pins the two as equal
(``tests/test_lewm_jepa_cache.py:181-194``).
"""

from __future__ import annotations

from typing import Mapping

import numpy as np

try:  # erf for the exact (non-tanh) GELU used by nn.GELU()
    from scipy.special import erf as _erf
except Exception:  # pragma: no cover - scipy is in the image
    _erf = np.vectorize(__import__("math").erf)

F32 = np.float32


def layer_norm(x, weight=None, bias=None, eps=1e-5):
    """``nn.LayerNorm`` over the last dim (biased variance)."""
    x = x.astype(F32, copy=False)
    mu = x.mean(-1, keepdims=True, dtype=np.float64).astype(F32)
    xc = x - mu
    var = (xc * xc).mean(-1, keepdims=True, dtype=np.float64).astype(F32)
    y = xc / np.sqrt(var + F32(eps))
    if weight is not None:
        y = y * weight + bias
    return y.astype(F32, copy=False)


def silu(x):
    # exp(-x) overflows to inf for x below about -88: x / inf = -0, the limit of SiLU.
    with np.errstate(over="ignore"):
        return (x / (F32(1) + np.exp(-x))).astype(F32, copy=False)


def gelu(x):
    return (F32(0.5) * x * (F32(1) + _erf(x / np.sqrt(F32(2))).astype(F32))).astype(F32, copy=False)


def linear(x, w, b=None):
    """``nn.Linear``; flattened to one 2-D GEMM so numpy hands it to BLAS in one call."""
    lead = x.shape[:-1]
    y = np.ascontiguousarray(x, dtype=F32).reshape(-1, x.shape[-1]) @ w.T
    if b is not None:
        y += b
    return y.reshape(*lead, w.shape[0]).astype(F32, copy=False)


def embedder(act, sd: Mapping[str, np.ndarray], prefix: str = "action_encoder."):
    """``Embedder.forward`` (reference ``lewm/module.py:205-214``). act (..., A)."""
    x = act.astype(F32)
    wc = sd[prefix + "patch_embed.weight"][:, :, 0]
    x = linear(x, wc, sd[prefix + "patch_embed.bias"])  # Conv1d k=1 over channels
    x = linear(x, sd[prefix + "embed.0.weight"], sd[prefix + "embed.0.bias"])
    x = silu(x)
    return linear(x, sd[prefix + "embed.2.weight"], sd[prefix + "embed.2.bias"])


def attention(x, sd, q, heads, dim_head):
    """``Attention.forward`` with causal SDPA (``lewm/module.py:75-85``). x (N, w, D)."""
    N, w, _ = x.shape
    xn = layer_norm(x, sd[q + "attn.norm.weight"], sd[q + "attn.norm.bias"], 1e-5)
    qkv = linear(xn, sd[q + "attn.to_qkv.weight"])
    inner = heads * dim_head
    qh = qkv[..., :inner].reshape(N, w, heads, dim_head).transpose(0, 2, 1, 3)
    kh = qkv[..., inner:2 * inner].reshape(N, w, heads, dim_head).transpose(0, 2, 1, 3)
    vh = qkv[..., 2 * inner:].reshape(N, w, heads, dim_head).transpose(0, 2, 1, 3)
    scores = (qh @ kh.transpose(0, 1, 3, 2)) * F32(dim_head ** -0.5)
    mask = np.triu(np.ones((w, w), dtype=bool), 1)
    scores = np.where(mask, F32(-np.inf), scores)
    scores = scores - scores.max(-1, keepdims=True)
    p = np.exp(scores)
    p = p / p.sum(-1, keepdims=True)
    out = (p @ vh).transpose(0, 2, 1, 3).reshape(N, w, inner)
    return linear(out, sd[q + "attn.to_out.0.weight"], sd[q + "attn.to_out.0.bias"])


def feed_forward(x, sd, q):
    """``FeedForward.forward`` (``lewm/module.py:38-53``)."""
    h = layer_norm(x, sd[q + "mlp.net.0.weight"], sd[q + "mlp.net.0.bias"], 1e-5)
    h = gelu(linear(h, sd[q + "mlp.net.1.weight"], sd[q + "mlp.net.1.bias"]))
    return linear(h, sd[q + "mlp.net.4.weight"], sd[q + "mlp.net.4.bias"])


def ar_predictor(x, c, sd, desc):
    """``ARPredictor.forward`` (``lewm/module.py:276-285``). x, c: (N, w, D)."""
    w = x.shape[1]
    D = desc.dim
    x = (x + sd["predictor.pos_embedding"][:, :w]).astype(F32)
    for l in range(desc.depth):
        q = f"predictor.transformer.layers.{l}."
        mod = linear(silu(c), sd[q + "adaLN_modulation.1.weight"], sd[q + "adaLN_modulation.1.bias"])
        sh_msa, sc_msa, g_msa, sh_mlp, sc_mlp, g_mlp = (mod[..., i * D:(i + 1) * D] for i in range(6))
        h = layer_norm(x, eps=1e-6) * (F32(1) + sc_msa) + sh_msa
        x = x + g_msa * attention(h, sd, q, desc.heads, desc.dim_head)
        h = layer_norm(x, eps=1e-6) * (F32(1) + sc_mlp) + sh_mlp
        x = x + g_mlp * feed_forward(h, sd, q)
    return layer_norm(x, sd["predictor.transformer.norm.weight"], sd["predictor.transformer.norm.bias"], 1e-5)


def pred_proj(x, sd, desc):
    """``JEPA.pred_proj``: Identity or ``MLP`` (``lewm/module.py:217-240``)."""
    if not desc.pred_proj_hidden:
        return x
    h = linear(x, sd["pred_proj.net.0.weight"], sd["pred_proj.net.0.bias"])
    if desc.pred_proj_norm == "layernorm":
        h = layer_norm(h, sd["pred_proj.net.1.weight"], sd["pred_proj.net.1.bias"], 1e-5)
    elif desc.pred_proj_norm == "batchnorm":  # eval-mode BatchNorm1d, eps 1e-5
        h = ((h - sd["pred_proj.net.1.running_mean"]) / np.sqrt(sd["pred_proj.net.1.running_var"] + F32(1e-5))
             * sd["pred_proj.net.1.weight"] + sd["pred_proj.net.1.bias"]).astype(F32)
    h = gelu(h)
    return linear(h, sd["pred_proj.net.3.weight"], sd["pred_proj.net.3.bias"])


def rollout_from_embeddings(emb, cand, sd, desc, history_size=3):
    """``JEPA.rollout_from_embeddings`` (``lewm/jepa.py:262-300``).

    emb (B, H, D) or (B, S, H, D); cand (B, S, T, A). Returns (B, S, T+1, D).
    """
    cand = np.asarray(cand, dtype=F32)
    B, S, T = cand.shape[:3]
    emb = np.asarray(emb, dtype=F32)
    H = emb.shape[-2]
    if emb.ndim == 3:
        emb = np.broadcast_to(emb[:, None], (B, S) + emb.shape[1:])
    elif emb.ndim != 4:
        raise ValueError(f"Expected emb rank 3 or 4, got shape {tuple(emb.shape)}")
    hist = np.array(emb.reshape(B * S, H, -1), dtype=F32)
    act_emb = embedder(cand.reshape(B * S, T, -1), sd)
    HS = history_size
    for t in range(T - H + 1):
        end = H + t
        start = max(0, end - HS)
        x = hist[:, -HS:]
        c = act_emb[:, start:end]
        pred = pred_proj(ar_predictor(x, c, sd, desc), sd, desc)[:, -1:]
        hist = np.concatenate([hist, pred], axis=1)
    return hist.reshape(B, S, hist.shape[1], -1)


def cost_from_rollout(pred_emb, goal_emb):
    """``JEPA.cost_from_rollout`` (``lewm/jepa.py:246-260``): terminal squared distance."""
    goal = goal_emb[..., -1:, :]
    while goal.ndim < pred_emb.ndim:
        goal = goal[:, None]
    d = pred_emb[..., -1, :] - goal[..., -1, :]
    return (d * d).sum(-1, dtype=np.float64).astype(F32)


def get_cost_from_embeddings(emb, goal_emb, cand, sd, desc, history_size=3):
    """``JEPA.get_cost_from_embeddings`` (``lewm/jepa.py:302-317``) -> (B, S) float32."""
    pred = rollout_from_embeddings(emb, cand, sd, desc, history_size)
    return cost_from_rollout(pred, np.asarray(goal_emb, dtype=F32))
