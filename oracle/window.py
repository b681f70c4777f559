"""TEST INFRASTRUCTURE ONLY: numpy restatement of Mimi's windowed streaming attention and of
the Mimi transformer layer around it.

Follows the reference after in_proj: MimiStreamingMultiheadAttention::forward
(ptts/src/transformer.rs:419-468: RoPE at the cache's absolute offset, append, scores scaled by
1/sqrt(D), the mask, softmax, trim), KvCache (transformer.rs:257-317: append concatenates,
trim keeps the last context - 1 rows, absolute_offset counts every row) and the mask of
StreamingTransformer::forward (transformer.rs:762-785: key visible iff 0 <= query - key <
context). RoPE as rope.rs:37-95 (interleaved pairs, f32 angle). With `bf16`, rotated k and v
are rounded to bf16 as they enter the cache (the library's bf16 cache). The layer
(mimi_layer) follows MimiStreamingMultiheadAttention::forward (transformer.rs:419-468: in_proj
without bias, the packed [t, 3, heads, D] split, RoPE, the cache, out_proj) inside
StreamingTransformerLayer::forward (transformer.rs:591-634: LayerNorm eps 1e-5, the layer
scales of layer_scale.rs:14-16, GELU erf or the tanh form of transformer.rs:498-503). Parity
unpinned, like the rest of the oracle; only tests use it.
"""
from __future__ import annotations

import numpy as np


def _round_bf16(x):
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def rope(x, positions, inv_freq):
    """x [rows, heads, D], positions [rows] -> rotated (f32 angle, f64 arithmetic)."""
    ang = (np.asarray(positions, np.float32)[:, None] * inv_freq.astype(np.float32)[None, :]).astype(np.float32)
    c, s = np.cos(ang.astype(np.float64))[:, None, :], np.sin(ang.astype(np.float64))[:, None, :]
    x = np.asarray(x, np.float64)
    y = np.empty_like(x)
    y[..., 0::2] = x[..., 0::2] * c - x[..., 1::2] * s
    y[..., 1::2] = x[..., 0::2] * s + x[..., 1::2] * c
    return y


class KvCache:
    """One stream's Mimi cache."""

    def __init__(self, context: int):
        self.context = context
        self.k = np.zeros((0, 8, 64))
        self.v = np.zeros((0, 8, 64))
        self.offset = 0


def attend(cache: KvCache, q, k, v, inv_freq, *, bf16: bool):
    """q [t, H, D], k/v [t, KVH, D] -> [t, H*D]; the cache is appended and trimmed."""
    t, H, D = q.shape
    rep = H // k.shape[1]
    pos = cache.offset + np.arange(t)
    qr = rope(q, pos, inv_freq)
    kr = np.repeat(rope(k, pos, inv_freq), rep, axis=1)
    vr = np.repeat(np.asarray(v, np.float64), rep, axis=1)
    if bf16:
        kr = _round_bf16(kr).astype(np.float64)
        vr = _round_bf16(vr).astype(np.float64)
    K = np.concatenate([cache.k, kr])
    V = np.concatenate([cache.v, vr])
    kv_len = cache.k.shape[0]
    seq = np.arange(t)[:, None] + kv_len
    key = np.arange(K.shape[0])[None, :]
    visible = (key <= seq) & (seq < key + cache.context)
    scores = np.einsum("thd,khd->htk", qr, K) / np.sqrt(D)
    scores = np.where(visible[None], scores, -np.inf)
    scores -= scores.max(-1, keepdims=True)
    p = np.exp(scores)
    p /= p.sum(-1, keepdims=True)
    out = np.einsum("htk,khd->thd", p, V).reshape(t, H * D)
    keep = max(cache.context - 1, 0)
    cache.k, cache.v = K[max(K.shape[0] - keep, 0):], V[max(V.shape[0] - keep, 0):]
    cache.offset += t
    return out


def layer_norm(x, g, b, eps=1e-5):
    x = np.asarray(x, np.float64)
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    return (x - mu) / np.sqrt(var + eps) * g + b


def gelu(x, form="erf"):
    x = np.asarray(x, np.float64)
    if form == "tanh":  # x sigmoid(2u), u = sqrt(2/pi) (x + 0.044715 x^3)
        u2 = (x * x * 0.07135482 + 1.595769) * x
        return x / (1.0 + np.exp(-u2))
    from scipy.special import erf
    return 0.5 * x * (1.0 + erf(x / np.sqrt(2.0)))


def mimi_layer(t: dict, prefix: str, x, cache: KvCache, inv_freq, heads: int, *, bf16: bool, gelu_form="erf"):
    """One StreamingTransformerLayer of Mimi on one stream's rows x [t, d] (float64): returns
    the new rows; the stream's cache for this layer is appended and trimmed."""
    g = lambda n: np.asarray(t[prefix + n], np.float64)
    rows, d = x.shape
    D = d // heads
    h = layer_norm(x, g("norm1.weight"), g("norm1.bias"))
    packed = (h @ g("self_attn.in_proj.weight").T).reshape(rows, 3, heads, D)
    a = attend(cache, packed[:, 0], packed[:, 1], packed[:, 2], inv_freq, bf16=bf16)
    a = a @ g("self_attn.out_proj.weight").T
    if prefix + "layer_scale_1.scale" in t:
        a = a * g("layer_scale_1.scale")
    x = x + a
    h = layer_norm(x, g("norm2.weight"), g("norm2.bias"))
    f = gelu(h @ g("linear1.weight").T, gelu_form) @ g("linear2.weight").T
    if prefix + "layer_scale_2.scale" in t:
        f = f * g("layer_scale_2.scale")
    return x + f


def mimi_forward(t: dict, layers: int, x, caches, inv_freq, heads: int, *, bf16: bool, gelu_form="erf"):
    """StreamingTransformer::forward (transformer.rs:742-808) of Mimi's layers on one stream:
    caches[l] is the stream's KvCache of layer l."""
    x = np.asarray(x, np.float64)
    for l in range(layers):
        x = mimi_layer(t, f"layers.{l}.", x, caches[l], inv_freq, heads, bf16=bf16, gelu_form=gelu_form)
    return x
