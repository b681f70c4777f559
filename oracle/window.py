"""TEST INFRASTRUCTURE ONLY: numpy restatement of Mimi's windowed streaming attention.

Follows the reference after in_proj: MimiStreamingMultiheadAttention::forward
(ptts/src/transformer.rs:419-468: RoPE at the cache's absolute offset, append, scores scaled by
1/sqrt(D), the mask, softmax, trim), KvCache (transformer.rs:257-317: append concatenates,
trim keeps the last context - 1 rows, absolute_offset counts every row) and the mask of
StreamingTransformer::forward (transformer.rs:762-785: key visible iff 0 <= query - key <
context). RoPE as rope.rs:37-95 (interleaved pairs, f32 angle). With `bf16`, rotated k and v
are rounded to bf16 as they enter the cache (the library's bf16 cache). Parity unpinned, like
the rest of the oracle; only tests use it.
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
