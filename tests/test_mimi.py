"""Mimi's transformer layers (MimiStreamingMultiheadAttention inside StreamingTransformerLayer,
transformer.rs:395-468 and :591-634) through ptts_b200_forward: f32 linears without biases, the
packed q/k/v split, RoPE at each stream's absolute position, windowed attention over the last
`context` positions, and the layer scales. Checked against the numpy restatement in
oracle/window.py over prompts and decode rows whose positions run past the window and past the
cache's slots (slots wrap), per call. Metric: ||gpu - oracle||_inf / ||oracle||_inf <= 2e-3 (bf16
cache, f32-grade linears). The oracle runs in float64 and rounds the rotated k and the v rows to
bf16 where the library's cache stores them."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import normwise

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _calls():
    # (stream, rows) per call; a window of 12 over 20 slots takes at most 9 rows per call.
    return ([[(0, 9), (1, 5), (2, 1)], [(0, 7), (2, 9)], [(1, 9), (2, 6)]] +
            [[(0, 1), (1, 1), (2, 1)]] * 14 + [[(2, 9), (0, 3)]] + [[(0, 1), (1, 1), (2, 1)]] * 6)


@pytest.mark.parametrize("gelu_form", ["erf", "tanh"])
def test_mimi_layers_match_the_oracle(ptts, cuda, gelu_form):
    import torch
    import oracle
    from oracle import window as ow
    cfg = ptts.FlowLMConfig(num_layers=2, gelu=gelu_form)
    tensors = ptts.random_mimi_tensors(cfg, 91, layer_scale=0.5)
    model = ptts.Transformer(cfg)
    model.load_mimi(tensors)
    S, cap, ctx = 3, 20, 12
    kv = ptts.KvState(cfg.num_layers, S, cap, dtype="bf16")
    kv.set_window(list(range(S)), ctx)
    caches = [[ow.KvCache(ctx) for _ in range(cfg.num_layers)] for _ in range(S)]
    inv = oracle.rope_inv_freq(64)
    g = torch.Generator().manual_seed(91)
    worst = []
    for call in _calls():
        streams = [s for s, _ in call]
        rows = [r for _, r in call]
        x = torch.randn(sum(rows), 512, generator=g).bfloat16()
        y = model.forward(kv, x.to(cuda), streams, rows).cpu().numpy()
        at = 0
        for s, r in call:
            want = ow.mimi_forward(tensors, cfg.num_layers, x[at:at + r].float().numpy(), caches[s], inv, 8,
                                   bf16=True, gelu_form=gelu_form)
            worst.append(normwise(y[at:at + r], want))
            at += r
    kv.check()
    assert list(kv.lengths()) == [c[0].offset for c in caches]
    assert max(kv.lengths()) > cap + ctx  # positions ran past the slots and the window
    print(gelu_form, "mimi layers: worst normwise", max(worst), "over", len(worst), "stream-calls")
    assert max(worst) < TOL


def test_layer_scale_folds_into_the_residual_linears(ptts, cuda):
    """ptts_b200_model_set_layer_scale on an int8 flow-LM layer: ones change nothing (bit for
    bit), a scale s gives x + s * attn and x + s * ff, and clearing restores the layer."""
    import torch
    cfg = ptts.FlowLMConfig(num_layers=1)
    w = ptts.random_weights(cfg, 93)
    model = ptts.Transformer(cfg)
    model.load(w)
    g = torch.Generator().manual_seed(93)
    x = torch.randn(40, 512, generator=g).bfloat16().to(cuda)

    def run():
        kv = ptts.KvState(1, 2, 64, dtype="bf16")
        return model.forward(kv, x, [0, 1], [25, 15]).clone()

    plain = run()
    model.set_layer_scale(0, np.ones(512, np.float32), np.ones(512, np.float32))
    assert torch.equal(run(), plain)
    # With scales on both branches, and the branches on their own (the other scale zero).
    s1 = np.random.default_rng(93).uniform(0.2, 2.0, 512).astype(np.float32)
    model.set_layer_scale(0, s1, np.zeros(512, np.float32))
    attn_only = run()
    model.set_layer_scale(0, np.zeros(512, np.float32), np.zeros(512, np.float32))
    nothing = run()
    assert torch.equal(nothing, x.float())  # both branches scaled to zero: the input passes through
    model.set_layer_scale(0, np.ones(512, np.float32), np.zeros(512, np.float32))
    attn_unscaled = run()
    got = (attn_only - nothing).cpu().numpy()
    want = (attn_unscaled - nothing).cpu().numpy() * s1
    assert normwise(got, want) < 1e-5
    model.set_layer_scale(0, None, None)
    assert torch.equal(run(), plain)


def test_a_q8_mimi_transformer_matches_the_f32_one(ptts, cuda):
    """transformer.rs:1321-1338: a Mimi transformer whose linears are quantized to q8_0
    (prepare_q8 / apply_q8) gives the f32 one's outputs within a relative RMS error of 1e-2,
    and not exactly. Here over windowed prompts and decode rows past the window, through the
    q8_0 layer loader (f16 hi/lo planes for prompts, block-scaled int8 widened on chip for
    decode rows), with the layer scales."""
    import torch
    cfg = ptts.FlowLMConfig(num_layers=2)
    tensors = ptts.random_mimi_tensors(cfg, 95, layer_scale=0.5)
    S, cap, ctx = 3, 20, 12
    outs = []
    for q8 in (False, True):
        model = ptts.Transformer(cfg)
        model.load_mimi(tensors, q8_0=q8)
        kv = ptts.KvState(cfg.num_layers, S, cap, dtype="bf16")
        kv.set_window(list(range(S)), ctx)
        g = torch.Generator().manual_seed(95)
        ys = []
        for call in _calls():
            streams = [s for s, _ in call]
            rows = [r for _, r in call]
            x = torch.randn(sum(rows), 512, generator=g).bfloat16()
            ys.append(model.forward(kv, x.to(cuda), streams, rows).cpu().numpy())
        kv.check()
        outs.append(np.concatenate(ys))
    want, got = outs
    err = float(np.sqrt(np.sum((got - want) ** 2) / np.sum(want ** 2)))
    print("q8_0 against f32 Mimi layers: relative RMS error", err)
    assert 0.0 < err < 0.01
