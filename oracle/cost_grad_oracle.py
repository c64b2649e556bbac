"""ORACLE (test infrastructure only) -- gradient of the LeWM model cost w.r.t. the actions.

Only ``tests/`` may import it; the product package never does.

CEM-GD (reference ``lewm/solvers/cem_gd.py:459-606``) refines actions with the gradient of
``JEPA.get_cost_from_embeddings`` (reference ``lewm/jepa.py:302-317``) with respect to the
action candidates. This module restates that forward (the same algorithm as
``oracle/lewm_oracle.py``: Embedder, AdaLN-zero blocks with causal window attention,
final LayerNorm, autoregressive rollout over the growing / sliding window, terminal
squared distance) on a small reverse-mode tape in float64, and returns the costs and
d sum(costs) / d candidates. ``tests/golden/make_cost_grad_golden.py`` pins it to torch
autograd of the reference model.

Each op keeps its inputs and a backward rule; ``backward`` walks the tape in reverse
creation order, summing gradients over broadcast dimensions.
"""

from __future__ import annotations

import itertools
from typing import Mapping, Sequence

import numpy as np

try:
    from scipy.special import erf as _erf
except Exception:  # pragma: no cover - scipy is in the image
    _erf = np.vectorize(__import__("math").erf)

F64 = np.float64
_ids = itertools.count()


class V:
    """A tape value: array, gradient, parents and the rule mapping the output gradient to theirs."""

    __slots__ = ("v", "g", "parents", "rule", "id")

    def __init__(self, v, parents: Sequence["V"] = (), rule=None):
        self.v = np.asarray(v, dtype=F64)
        self.g = None
        self.parents = tuple(parents)
        self.rule = rule
        self.id = next(_ids)


def const(a) -> V:
    return V(a)


def _unbroadcast(g: np.ndarray, shape) -> np.ndarray:
    while g.ndim > len(shape):
        g = g.sum(0)
    for i, n in enumerate(shape):
        if n == 1 and g.shape[i] != 1:
            g = g.sum(i, keepdims=True)
    return g


def add(a: V, b: V) -> V:
    return V(a.v + b.v, (a, b), lambda g: (_unbroadcast(g, a.v.shape), _unbroadcast(g, b.v.shape)))


def mul(a: V, b: V) -> V:
    return V(a.v * b.v, (a, b), lambda g: (_unbroadcast(g * b.v, a.v.shape), _unbroadcast(g * a.v, b.v.shape)))


def linear(x: V, w: np.ndarray, b=None) -> V:
    """x . w^T (+ b) with constant weights."""
    w = np.asarray(w, F64)
    y = x.v @ w.T
    if b is not None:
        y = y + np.asarray(b, F64)
    return V(y, (x,), lambda g: (g @ w,))


def matmul(a: V, b: V) -> V:
    return V(a.v @ b.v, (a, b), lambda g: (g @ np.swapaxes(b.v, -1, -2), np.swapaxes(a.v, -1, -2) @ g))


def reshape(x: V, shape) -> V:
    s0 = x.v.shape
    return V(x.v.reshape(shape), (x,), lambda g: (g.reshape(s0),))


def transpose(x: V, axes) -> V:
    inv = np.argsort(axes)
    return V(x.v.transpose(axes), (x,), lambda g: (g.transpose(inv),))


def take(x: V, idx) -> V:
    s0 = x.v.shape

    def rule(g):
        out = np.zeros(s0, F64)
        out[idx] += g
        return (out,)

    return V(x.v[idx], (x,), rule)


def concat(xs: Sequence[V], axis: int) -> V:
    sizes = [x.v.shape[axis] for x in xs]
    cuts = np.cumsum(sizes)[:-1]
    return V(np.concatenate([x.v for x in xs], axis=axis), xs, lambda g: tuple(np.split(g, cuts, axis=axis)))


def silu(x: V) -> V:
    s = 1.0 / (1.0 + np.exp(-x.v))
    return V(x.v * s, (x,), lambda g: (g * (s + x.v * s * (1.0 - s)),))


def gelu(x: V) -> V:
    cdf = 0.5 * (1.0 + _erf(x.v / np.sqrt(2.0)))
    pdf = np.exp(-0.5 * x.v * x.v) / np.sqrt(2.0 * np.pi)
    return V(x.v * cdf, (x,), lambda g: (g * (cdf + x.v * pdf),))


def layer_norm(x: V, w=None, b=None, eps: float = 1e-5) -> V:
    n = x.v.shape[-1]
    mu = x.v.mean(-1, keepdims=True)
    xc = x.v - mu
    rstd = 1.0 / np.sqrt((xc * xc).mean(-1, keepdims=True) + eps)
    xh = xc * rstd
    w64 = None if w is None else np.asarray(w, F64)
    y = xh if w is None else xh * w64 + np.asarray(b, F64)

    def rule(g):
        gx = g if w64 is None else g * w64
        return (rstd / n * (n * gx - gx.sum(-1, keepdims=True) - xh * (gx * xh).sum(-1, keepdims=True)),)

    return V(y, (x,), rule)


def causal_softmax(s: V) -> V:
    w = s.v.shape[-1]
    mask = np.triu(np.ones((w, w), dtype=bool), 1)
    z = np.where(mask, -np.inf, s.v)
    z = z - z.max(-1, keepdims=True)
    p = np.exp(z)
    p = p / p.sum(-1, keepdims=True)
    return V(p, (s,), lambda g: (p * (g - (g * p).sum(-1, keepdims=True)),))


def backward(out: V, seed: np.ndarray) -> None:
    order, seen, stack = [], set(), [out]
    while stack:  # every node reachable from the output
        n = stack.pop()
        if n.id in seen:
            continue
        seen.add(n.id)
        order.append(n)
        stack.extend(n.parents)
    order.sort(key=lambda n: n.id, reverse=True)  # creation order is a topological order
    out.g = np.asarray(seed, F64)
    for n in order:
        if n.g is None or n.rule is None:
            continue
        for p, gp in zip(n.parents, n.rule(n.g)):
            p.g = gp if p.g is None else p.g + gp


# ----------------------------------------------------------------- the model cost on the tape
def _embedder(act: V, sd) -> V:
    p = "action_encoder."
    x = linear(act, sd[p + "patch_embed.weight"][:, :, 0], sd[p + "patch_embed.bias"])
    x = silu(linear(x, sd[p + "embed.0.weight"], sd[p + "embed.0.bias"]))
    return linear(x, sd[p + "embed.2.weight"], sd[p + "embed.2.bias"])


def _attention(x: V, sd, q: str, heads: int, dh: int) -> V:
    N, w, _ = x.v.shape
    inner = heads * dh
    xn = layer_norm(x, sd[q + "attn.norm.weight"], sd[q + "attn.norm.bias"], 1e-5)
    qkv = linear(xn, sd[q + "attn.to_qkv.weight"])

    def head(i):
        part = take(qkv, (Ellipsis, slice(i * inner, (i + 1) * inner)))
        return transpose(reshape(part, (N, w, heads, dh)), (0, 2, 1, 3))

    qh, kh, vh = head(0), head(1), head(2)
    s = mul(matmul(qh, transpose(kh, (0, 1, 3, 2))), const(dh ** -0.5))
    out = matmul(causal_softmax(s), vh)
    out = reshape(transpose(out, (0, 2, 1, 3)), (N, w, inner))
    return linear(out, sd[q + "attn.to_out.0.weight"], sd[q + "attn.to_out.0.bias"])


def _feed_forward(x: V, sd, q: str) -> V:
    h = layer_norm(x, sd[q + "mlp.net.0.weight"], sd[q + "mlp.net.0.bias"], 1e-5)
    h = gelu(linear(h, sd[q + "mlp.net.1.weight"], sd[q + "mlp.net.1.bias"]))
    return linear(h, sd[q + "mlp.net.4.weight"], sd[q + "mlp.net.4.bias"])


def _predictor(x: V, c: V, sd, desc) -> V:
    w, D = x.v.shape[1], desc.dim
    x = add(x, const(np.asarray(sd["predictor.pos_embedding"], F64)[:, :w]))
    one = const(1.0)
    for l in range(desc.depth):
        q = f"predictor.transformer.layers.{l}."
        mod = linear(silu(c), sd[q + "adaLN_modulation.1.weight"], sd[q + "adaLN_modulation.1.bias"])
        sh1, sc1, g1, sh2, sc2, g2 = (take(mod, (Ellipsis, slice(i * D, (i + 1) * D))) for i in range(6))
        h = add(mul(layer_norm(x, eps=1e-6), add(one, sc1)), sh1)
        x = add(x, mul(g1, _attention(h, sd, q, desc.heads, desc.dim_head)))
        h = add(mul(layer_norm(x, eps=1e-6), add(one, sc2)), sh2)
        x = add(x, mul(g2, _feed_forward(h, sd, q)))
    return layer_norm(x, sd["predictor.transformer.norm.weight"], sd["predictor.transformer.norm.bias"], 1e-5)


def cost_and_grad(emb: np.ndarray, goal_emb: np.ndarray, cand: np.ndarray, sd: Mapping[str, np.ndarray], desc,
                  history_size: int = 3):
    """Costs (B, S) of ``get_cost_from_embeddings`` and d sum(costs) / d cand (B, S, T, A),
    float64. emb (B, H, D), goal_emb (B, G, D), cand (B, S, T, A); Identity pred_proj."""
    if desc.pred_proj_hidden:
        raise NotImplementedError("the gradient oracle covers the Identity pred_proj head")
    cand = np.asarray(cand, F64)
    B, S, T, A = cand.shape
    H, D = emb.shape[-2], emb.shape[-1]
    leaf = V(cand)
    act = reshape(leaf, (B * S, T, A))
    act_emb = _embedder(act, sd)
    hist = const(np.broadcast_to(np.asarray(emb, F64)[:, None], (B, S, H, D)).reshape(B * S, H, D))
    HS = history_size
    for t in range(T - H + 1):
        end = H + t
        start = max(0, end - HS)
        n = hist.v.shape[1]
        x = take(hist, (slice(None), slice(max(0, n - HS), n)))
        c = take(act_emb, (slice(None), slice(start, end)))
        pred = take(_predictor(x, c, sd, desc), (slice(None), slice(-1, None)))
        hist = concat([hist, pred], axis=1)
    last = take(hist, (slice(None), -1))
    goal = np.broadcast_to(np.asarray(goal_emb, F64)[:, -1][:, None], (B, S, D)).reshape(B * S, D)
    d = add(last, const(-goal))
    cost = V((d.v * d.v).sum(-1), (d,), lambda g: (2.0 * d.v * g[:, None],))
    backward(cost, np.ones(B * S))
    return cost.v.reshape(B, S), leaf.g
