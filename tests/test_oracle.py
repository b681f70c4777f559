"""CPU tests of the oracle, pinned to the reference's own tests and formulas.

The reference's attention arithmetic lives in `xn` 0.2.15, which cannot be built here, and it
holds no numeric golden vectors for this path (parity unpinned). These tests re-express the
reference's equivalence and known-answer tests against the oracle and check its RoPE tables
against rope.rs:44-57 evaluated in float64 (tests/golden/).
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

from conftest import GOLDEN, normwise


def _mha(oracle, in_w, out_w, embed, h, kvh, d, xs_chunks, cap, *, kv_rows=None):
    """StreamingMultiheadAttention::forward with f32 Linear weights (no bias), chunk by chunk:
    in_proj -> split -> oracle.attend -> out_proj; the host-position path."""
    kvd = kvh * d
    kc = np.zeros((1, cap, h, d), np.float32)
    vc = np.zeros_like(kc)
    length = 0
    outs = []
    for xs in xs_chunks:
        t = xs.shape[0]
        proj = xs @ in_w.T
        q = proj[:, : h * d].reshape(t, h, d)
        k = proj[:, h * d: h * d + kvd].reshape(t, kvh, d)
        v = proj[:, h * d + kvd:].reshape(t, kvh, d)
        a = oracle.attend(q, k, v, kc, vc, [length], [0], [0, t])
        outs.append(a @ out_w.T)
        length += t
    return np.concatenate(outs), kc, vc


def test_grouped_query_attention_is_attention_with_repeated_kv_heads(oracle):
    """transformer.rs:1112-1164 on the test's own LCG inputs (seed 1): prompt of 3, two steps."""
    g = np.load(os.path.join(GOLDEN, "lcg_gqa.npz"))
    embed, h, kvh, d = (int(v) for v in g["dims"])
    attn, group = h * d, h // kvh
    q_w, k_w, v_w = g["q_w"], g["k_w"], g["v_w"]
    o_w = g["o_w"].reshape(embed, attn)
    x = g["x"].reshape(5, embed)

    def repeat(w):
        return np.concatenate([w[(j // group) * d * embed:(j // group + 1) * d * embed] for j in range(h)])

    chunks = [x[0:3], x[3:4], x[4:5]]
    grouped, _, _ = _mha(oracle, np.concatenate([q_w, k_w, v_w]).reshape(-1, embed), o_w, embed, h,
                         kvh, d, chunks, 8)
    full, _, _ = _mha(oracle, np.concatenate([q_w, repeat(k_w), repeat(v_w)]).reshape(-1, embed),
                      o_w, embed, h, h, d, chunks, 8)
    assert grouped.shape == (5, embed)
    assert np.abs(grouped - full).max() < 1e-6


def test_a_device_step_is_the_host_step(oracle):
    """transformer.rs:1169-1225 on the test's LCG inputs (seed 7): a step that scatters its k/v
    at a position and attends over the whole cache with a -inf mask on unfilled slots gives the
    host step's output. The device form is restated in numpy over the oracle's cache."""
    g = np.load(os.path.join(GOLDEN, "lcg_device_step.npz"))
    embed, h, kvh, d, kv = (int(v) for v in g["dims"])
    in_w = g["in_w"].reshape((h + 2 * kvh) * d, embed)
    out_w = g["out_w"].reshape(embed, h * d)
    x = g["x"].reshape(5, embed)
    group = h // kvh
    # Host: prompt of 3 then steps at 3 and 4.
    host, kc, vc = _mha(oracle, in_w, out_w, embed, h, kvh, d, [x[0:3], x[3:4], x[4:5]], kv)
    # Device form for the steps: the cache after the prompt, scatter at p, full-cache mask.
    _, kd, vd = _mha(oracle, in_w, out_w, embed, h, kvh, d, [x[0:3]], kv)
    inv = oracle.rope_inv_freq(d)
    for p in (3, 4):
        proj = x[p] @ in_w.T
        q = proj[: h * d].reshape(h, d).astype(np.float32)
        k = np.repeat(proj[h * d: h * d + kvh * d].reshape(kvh, d), group, axis=0)
        v = np.repeat(proj[h * d + kvh * d:].reshape(kvh, d), group, axis=0)
        c, s = np.cos(np.float32(p) * inv), np.sin(np.float32(p) * inv)

        def rope(z):
            z = z.copy()
            z0, z1 = z[:, 0::2].copy(), z[:, 1::2].copy()
            z[:, 0::2], z[:, 1::2] = z0 * c - z1 * s, z0 * s + z1 * c
            return z

        q, k = rope(q), rope(k)
        kd[0, p], vd[0, p] = k, v
        mask = np.where(np.arange(kv) <= p, 0.0, -np.inf)
        out = np.zeros((h, d))
        for hh in range(h):
            sc = kd[0, :, hh] @ q[hh] / np.sqrt(d) + mask
            w = np.exp(sc - sc.max())
            out[hh] = (w / w.sum()) @ vd[0, :, hh]
        got = out.reshape(-1) @ out_w.T
        assert np.abs(got - host[p]).max() < 1e-6, p


def test_rope_tables_match_rope_rs_in_float64():
    """rope.rs:44-57: inverse frequencies within one f32 ulp of theta^(-i/32) rounded once; the
    angle is the f32 product pos * freq and cos/sin are within 2 f32 ulp of the float64 cos/sin
    of that f32 angle."""
    import oracle
    g = np.load(os.path.join(GOLDEN, "rope_f64.npz"))
    inv = oracle.rope_inv_freq(64, 10000.0)
    assert (np.abs(inv - g["inv_freq"]) <= np.spacing(g["inv_freq"])).all()
    pos = g["positions"]
    c, s = oracle.rope_table(64, pos, 10000.0)
    ang = (pos[:, None] * inv[None, :]).astype(np.float32).astype(np.float64)
    for got, want in ((c, np.cos(ang)), (s, np.sin(ang))):
        ulp = np.spacing(np.abs(want).astype(np.float32)).astype(np.float64)
        assert (np.abs(got - want) <= 2 * ulp + 1e-12).all()


def test_rope_is_interleaved_pairs(oracle):
    """(x[2i], x[2i+1]) is turned as the complex number x[2i] + i x[2i+1] times e^{i pos w_i}
    (rope.rs:81-95; the same convention as ptts-coreml/src/phonon/flow_lm.rs:85-89)."""
    rng = np.random.default_rng(0)
    q = rng.normal(size=(1, 8, 64)).astype(np.float32)
    k = np.zeros((1, 8, 64), np.float32)
    kc = np.zeros((1, 64, 8, 64), np.float32)
    vc = np.zeros_like(kc)
    pos = 37
    # Attention with one key of zeros returns v = 0; read the rotated k from the cache instead.
    kk = rng.normal(size=(1, 8, 64)).astype(np.float32)
    oracle.attend(q, kk, k, kc, vc, [pos], [0], [0, 1])
    inv = oracle.rope_inv_freq(64)
    z = (kk[0, :, 0::2] + 1j * kk[0, :, 1::2]) * np.exp(1j * pos * inv.astype(np.float64))
    got = kc[0, pos]
    np.testing.assert_allclose(got[:, 0::2], z.real, atol=2e-5)
    np.testing.assert_allclose(got[:, 1::2], z.imag, atol=2e-5)


def _attention_f64(q, kc, vc, length):
    d = q.shape[-1]
    s = np.einsum("hd,jhd->hj", q.astype(np.float64), kc[:length].astype(np.float64)) / np.sqrt(d)
    w = np.exp(s - s.max(-1, keepdims=True))
    w /= w.sum(-1, keepdims=True)
    return np.einsum("hj,jhd->hd", w, vc[:length].astype(np.float64))


def test_oracle_attention_against_float64(oracle):
    """Ragged batch, prompt rows and a decode row: the oracle's causal attention against a
    float64 restatement over the oracle's own cache (mask rule of transformer.rs:94-108)."""
    rng = np.random.default_rng(1)
    S, cap, H, D = 3, 40, 8, 64
    kc = np.zeros((S, cap, H, D), np.float32)
    vc = np.zeros_like(kc)
    lengths = np.array([5, 0, 17], np.int32)
    streams, rows = [2, 0, 1], [1, 7, 4]
    offs = np.concatenate([[0], np.cumsum(rows)]).astype(np.int32)
    n = offs[-1]
    q = rng.normal(size=(n, H, D)).astype(np.float32)
    k = rng.normal(size=(n, H, D)).astype(np.float32)
    v = rng.normal(size=(n, H, D)).astype(np.float32)
    kc[2, :5] = rng.normal(size=(5, H, D))
    vc[2, :5] = rng.normal(size=(5, H, D))
    out = oracle.attend(q, k, v, kc, vc, lengths, streams, offs)
    inv = oracle.rope_inv_freq(D)
    for i, s in enumerate(streams):
        for r in range(offs[i], offs[i + 1]):
            pos = lengths[s] + r - offs[i]
            ang = np.float32(pos) * inv
            qr = q[r].copy()
            q0, q1 = qr[:, 0::2].copy(), qr[:, 1::2].copy()
            qr[:, 0::2] = q0 * np.cos(ang) - q1 * np.sin(ang)
            qr[:, 1::2] = q0 * np.sin(ang) + q1 * np.cos(ang)
            want = _attention_f64(qr, kc[s], vc[s], pos + 1)
            assert normwise(out[r].reshape(H, D), want) < 1e-5
    # The cache holds the appended rows at their positions and nothing past them.
    assert (kc[0, 12:] == 0).all() and (kc[1, 4:] == 0).all() and (kc[2, 18:] == 0).all()


def test_capacity_is_refused(oracle):
    kc = np.zeros((1, 4, 8, 64), np.float32)
    q = np.zeros((3, 8, 64), np.float32)
    with pytest.raises(ValueError):
        oracle.attend(q, q, q, kc, kc.copy(), [2], [0], [0, 3])


def test_linear_i8_against_numpy(oracle):
    rng = np.random.default_rng(2)
    x = rng.normal(size=(13, 128)).astype(np.float32)
    w = rng.integers(-127, 128, size=(72, 128), dtype=np.int8)
    s = rng.uniform(0.005, 0.02, 72).astype(np.float32)
    y = oracle.linear_i8(x, w, s)
    want = x.astype(np.float64) @ (w.astype(np.float64) * s[:, None]).T
    assert normwise(y, want) < 1e-6
    # q8_0 layout: one scale per 32 weights along K.
    s32 = rng.uniform(0.005, 0.02, (72, 4)).astype(np.float32)
    y32 = oracle.linear_i8(x, w, s32, group=32)
    want32 = x.astype(np.float64) @ (w.astype(np.float64) * np.repeat(s32, 32, axis=1)).T
    assert normwise(y32, want32) < 1e-6


def test_layer_norm_and_gelu(oracle):
    rng = np.random.default_rng(3)
    x = rng.normal(3, 2, size=(5, 512)).astype(np.float32)
    g = rng.uniform(0.5, 1.5, 512).astype(np.float32)
    b = rng.normal(0, 0.1, 512).astype(np.float32)
    y = oracle.layer_norm(x, g, b)
    x64 = x.astype(np.float64)
    want = (x64 - x64.mean(-1, keepdims=True)) / np.sqrt(x64.var(-1, keepdims=True) + 1e-5) * g + b
    assert normwise(y, want) < 1e-5
    from math import erf, exp, sqrt, pi, tanh
    for v in (-3.0, -0.5, 0.0, 0.7, 4.0):
        assert abs(oracle.lib().oracle_gelu(v, 0) - 0.5 * v * (1 + erf(v / sqrt(2)))) < 1e-6
        u = sqrt(2 / pi) * (v + 0.044715 * v ** 3)
        assert abs(oracle.lib().oracle_gelu(v, 1) - 0.5 * v * (1 + tanh(u))) < 1e-5


def test_model_forward_is_the_layer_composition(oracle, ptts):
    """oracle_model_forward == LN -> in_proj -> attend -> out_proj -> residual -> LN -> FFN ->
    residual (transformer.rs:591-634), composed here from the oracle's single ops."""
    cfg = ptts.FlowLMConfig(num_layers=2, dim_feedforward=256)
    w = ptts.random_weights(cfg, 5, ln_random=True)
    m = oracle.Model(cfg, w)
    rng = np.random.default_rng(4)
    S, cap, rows = 2, 16, [3, 5]
    offs = np.array([0, 3, 8], np.int32)
    x = rng.normal(size=(8, 512)).astype(np.float32)
    for store in (0, oracle.ROUND_KV, oracle.ROUND_KV | oracle.ROUND_OPERANDS):
        kc = np.zeros((2, S, cap, 8, 64), np.float32)
        vc = np.zeros_like(kc)
        got = m.forward(x, kc, vc, [0, 0], [0, 1], offs, store=store)
        h = x.copy()
        kc2, vc2 = np.zeros_like(kc), np.zeros_like(vc)
        rb = oracle.round_bf16 if store & oracle.ROUND_OPERANDS else (lambda a: a)
        for l in range(2):
            n1 = rb(oracle.layer_norm(h, w.ln1_g[l], w.ln1_b[l]))
            qkv = oracle.linear_i8(n1, w.w_qkv[l], w.s_qkv[l])
            a = oracle.attend(qkv[:, :512].reshape(-1, 8, 64), qkv[:, 512:1024].reshape(-1, 8, 64),
                              qkv[:, 1024:].reshape(-1, 8, 64), kc2[l], vc2[l], [0, 0], [0, 1], offs,
                              store=store & oracle.ROUND_KV)
            h = h + oracle.linear_i8(rb(a), w.w_out[l], w.s_out[l])
            n2 = rb(oracle.layer_norm(h, w.ln2_g[l], w.ln2_b[l]))
            f = oracle.linear_i8(n2, w.w_ff1[l], w.s_ff1[l])
            f = rb(np.vectorize(lambda z: oracle.lib().oracle_gelu(float(z), 0))(f).astype(np.float32))
            h = h + oracle.linear_i8(f, w.w_ff2[l], w.s_ff2[l])
        assert normwise(got, h) < 1e-4
        np.testing.assert_array_equal(kc, kc2)


def test_with_seq_budget_known_answers():
    """transformer.rs:1022-1100 restated on numpy caches: prefix copied, tail zero, a budget
    below the prefix refused naming both numbers, an equal budget accepted."""
    g = json.load(open(os.path.join(GOLDEN, "with_seq_budget.json")))
    b, h, d = g["b"], g["h"], g["d"]
    for c in g["cases"]:
        k = np.array(c["k"], np.float32).reshape(b, c["seq"], h, d)
        if c["refused"]:
            assert c["used"] > c["budget"]
            continue
        out = np.zeros((b, c["budget"], h, d), np.float32)
        out[:, : c["used"]] = k[:, : c["used"]]
        np.testing.assert_array_equal(out.ravel(), np.array(c["want_k"], np.float32))


def test_mimi_layer_restatement_agrees_with_the_flow_lm_layer(ptts, oracle):
    """The numpy Mimi layer (oracle/window.py) with an unbounded window and no layer scales is
    the flow-LM layer the C oracle restates (transformer.rs:591-634 around either attention):
    same weights (int8 * row scale as f32), same bf16 cache rounding, prompt then decode rows."""
    from oracle import window as ow
    cfg = ptts.FlowLMConfig(num_layers=2)
    w = ptts.random_weights(cfg, 95)
    t = {}
    for l in range(cfg.num_layers):
        p = f"layers.{l}."
        t[p + "self_attn.in_proj.weight"] = w.w_qkv[l].astype(np.float32) * w.s_qkv[l][:, None]
        t[p + "self_attn.out_proj.weight"] = w.w_out[l].astype(np.float32) * w.s_out[l][:, None]
        t[p + "linear1.weight"] = w.w_ff1[l].astype(np.float32) * w.s_ff1[l][:, None]
        t[p + "linear2.weight"] = w.w_ff2[l].astype(np.float32) * w.s_ff2[l][:, None]
        t[p + "norm1.weight"], t[p + "norm1.bias"] = w.ln1_g[l], w.ln1_b[l]
        t[p + "norm2.weight"], t[p + "norm2.bias"] = w.ln2_g[l], w.ln2_b[l]
    om = oracle.Model(cfg, w)
    inv = oracle.rope_inv_freq(64)
    # Without the bf16 cache the two restatements are the same arithmetic (float64 against f32:
    # 1e-6); with it, the two sides' keys differ in the last f32 bits before rounding, and a few
    # bf16 roundings flip (1.5e-4).
    for store, bf16, tol in ((0, False, 5e-6), (oracle.ROUND_KV, True, 1e-3)):
        kc = np.zeros((cfg.num_layers, 1, 32, 8, 64), np.float32)
        vc = np.zeros_like(kc)
        caches = [ow.KvCache(10 ** 9) for _ in range(cfg.num_layers)]
        rng = np.random.default_rng(95)
        length = np.zeros(1, np.int32)
        for rows in (20, 1, 1, 3):
            x = oracle.round_bf16(rng.normal(size=(rows, 512)).astype(np.float32))
            want = om.forward(x, kc, vc, length, [0], [0, rows], store=store)
            got = ow.mimi_forward(t, cfg.num_layers, x, caches, inv, 8, bf16=bf16)
            length += rows
            assert np.abs(got - want).max() / np.abs(want).max() < tol, (store, rows)
