"""More than 8 heads (the reference's 1024-wide, 16-head test config, ptts/tests/fixtures/
config.json:3-4): the cache keeps each group of 8 heads as its own block and every kernel runs
per group, so a 16-head attention must be, bit for bit, two 8-head attentions side by side:
outputs, cache rows, ring evictions, windowed streams, prefix loads and stream copies. The layer
stack at that shape is checked against the oracle (transformer.rs:183-251, :591-634)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import normwise

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _scenario(ptts, cuda, heads, kv_heads, data, dtype):
    """One pass of the attention op over two layers and five streams of a KvState with `heads`
    heads: a loaded prefix (stream 2), prompts in one call (streams 0, 1, 2, 4; stream 4 then a
    ring), a windowed stream's prompt in its own call (stream 3), 9 decode steps over all five
    (the ring evicts its 3 oldest frames when its 6 frame slots are full), a copy of stream 1
    into a second cache and a reset of stream 2. Returns every output and both caches' rows."""
    import torch
    kv = ptts.KvState(2, 5, 200, num_heads=heads, dtype=dtype)
    for layer in range(2):
        kv.load_prefix(layer, 2, data["pre_k"][layer].to(cuda), data["pre_v"][layer].to(cuda))
    kv.set_window([3], 24)
    outs = []

    def call(layer, i, streams, rows):
        q, k, v = (data[n][layer][i].to(cuda) for n in ("q", "k", "v"))
        outs.append(ptts.attend(kv, layer, q, k, v, streams, rows, out_dtype="f32").cpu())

    for layer in range(2):
        call(layer, 0, [0, 1, 2, 4], [150, 7, 33, 12])
    kv.advance([0, 1, 2, 4], [150, 7, 33, 12])
    for layer in range(2):
        call(layer, 1, [3], [40])
    kv.advance([3], [40])
    kv.start_ring([4])
    in_view = 0
    for i in range(9):
        if in_view == 6:
            kv.evict(4, 12, [12, 13, 14])
            in_view -= 3
        kv.set_ring_slot(4, 12 + i % 6)
        for layer in range(2):
            call(layer, 2 + i, [0, 1, 2, 3, 4], [1] * 5)
        kv.advance([0, 1, 2, 3, 4], [1] * 5)
        in_view += 1
    other = ptts.KvState(2, 2, 220, num_heads=heads, dtype=dtype)
    other.copy_stream(1, kv, 1)
    kv.reset([2])
    kv.check()
    other.check()

    def rows(state):
        out = []
        for layer in range(2):
            for t in state.tensors(layer)[:2]:
                S, cap = t.shape[0], t.shape[1]
                out.append(t.reshape(S, cap, heads, 64).float().cpu())
        return out

    return outs, rows(kv), rows(other), kv.lengths().copy()


def _inputs(heads, kv_heads, seed, dtype):
    """Per call: q [n, heads, 64], k and v [n, kv_heads, 64]; the prefix [40, heads, 64]."""
    import torch
    g = torch.Generator().manual_seed(seed)
    t = torch.bfloat16 if dtype == "bf16" else torch.float32
    sizes = [202, 40] + [5] * 9  # the prompt call, the windowed prompt, 9 steps
    d = {n: [[torch.randn(s, h, 64, generator=g).to(t) for s in sizes] for _ in range(2)]
         for n, h in (("q", heads), ("k", kv_heads), ("v", kv_heads))}
    d["pre_k"] = [torch.randn(40, heads, 64, generator=g).to(t) for _ in range(2)]
    d["pre_v"] = [torch.randn(40, heads, 64, generator=g).to(t) for _ in range(2)]
    return d


def _half(d, part, heads, kv_heads):
    """The 8 heads of group `part` and their key/value heads, as an 8-head input."""
    qh, kh = heads // 2, kv_heads // 2
    cut = lambda x, n: x[:, part * n:(part + 1) * n].contiguous()
    out = {n: [[cut(x, qh if n == "q" else kh) for x in per_layer] for per_layer in d[n]]
           for n in ("q", "k", "v")}
    out["pre_k"] = [cut(x, qh) for x in d["pre_k"]]
    out["pre_v"] = [cut(x, qh) for x in d["pre_v"]]
    return out


@pytest.mark.parametrize("kernel,dtype,kv_heads", [("fa", "bf16", 16), ("fa", "bf16", 4), ("tc1", "bf16", 16),
                                                   ("core", "bf16", 16), ("core", "f32", 16)])
def test_sixteen_heads_are_two_groups_of_eight(ptts, cuda, monkeypatch, kernel, dtype, kv_heads):
    if kernel != "fa":
        monkeypatch.setenv("PTTS_B200_PREFILL", kernel)
    d = _inputs(16, kv_heads, 61, dtype)
    outs, rows, copied, lengths = _scenario(ptts, cuda, 16, kv_heads, d, dtype)
    halves = [_scenario(ptts, cuda, 8, kv_heads // 2, _half(d, p, 16, kv_heads), dtype) for p in (0, 1)]
    for i, o in enumerate(outs):
        for p in (0, 1):
            assert np.array_equal(o[:, 512 * p:512 * (p + 1)].numpy(), halves[p][0][i].numpy()), (i, p)
    for whole, a, b in zip(rows + copied, halves[0][1] + halves[0][2], halves[1][1] + halves[1][2]):
        assert np.array_equal(whole[:, :, :8].numpy(), a.numpy())
        assert np.array_equal(whole[:, :, 8:].numpy(), b.numpy())
    np.testing.assert_array_equal(lengths, halves[0][3])


def test_sixteen_head_stack_matches_the_oracle(ptts, oracle, cuda):
    """The reference's 1024-wide, 16-head, ff 4096 shape (2 layers): ragged prompts over 130
    streams, then decode steps (two lanes from 128 rows), against the oracle."""
    import torch
    cfg = ptts.FlowLMConfig(d_model=1024, num_heads=16, num_kv_heads=16, num_layers=2, dim_feedforward=4096)
    w = ptts.random_weights(cfg, 71)
    model = ptts.Transformer(cfg)
    model.load(w)
    om = oracle.Model(cfg, w)
    S = 130
    rows = np.random.default_rng(72).integers(1, 7, size=S).astype(np.int32)
    rows[0] = 140  # one prompt over two 128-row tiles
    cap = int(rows.max()) + 8
    kv = ptts.KvState(cfg.num_layers, S, cap, num_heads=16, dtype="bf16")
    shape = (cfg.num_layers, S, cap, 16, 64)
    kc, vc = np.zeros(shape, np.float32), np.zeros(shape, np.float32)
    streams = list(range(S))
    offs = np.concatenate([[0], np.cumsum(rows)]).astype(np.int32)
    g = torch.Generator().manual_seed(73)
    x = torch.randn(int(offs[-1]), 1024, generator=g).bfloat16()
    y = model.forward(kv, x.to(cuda), streams, rows.tolist())
    lengths = np.zeros(S, np.int32)
    want = om.forward(x.float().numpy(), kc, vc, lengths, streams, offs, store=oracle.ROUND_KV)
    errs = [normwise(y.float().cpu().numpy(), want)]
    lengths += rows
    for _ in range(3):
        xs = torch.randn(S, 1024, generator=g).bfloat16()
        y = model.step(kv, streams, xs.to(cuda))
        want = om.forward(xs.float().numpy(), kc, vc, lengths, streams, np.arange(S + 1, dtype=np.int32),
                          store=oracle.ROUND_KV)
        lengths += 1
        errs.append(normwise(y.float().cpu().numpy(), want))
    kv.check()
    print("16 heads, 1024 wide: prompt and decode normwise", ["%.2e" % e for e in errs])
    assert max(errs) < TOL
    # Layer 0's cache rows (group blocks read back as [S, cap, 16, 64]) against the oracle's:
    # both round the same f32 values to bf16, so they agree to a rounding flip (one bf16 ulp,
    # 2^-8 of the largest value).
    kt, vt, _ = kv.tensors(0)
    got_k = kt.reshape(S, cap, 16, 64).float().cpu().numpy()
    got_v = vt.reshape(S, cap, 16, 64).float().cpu().numpy()
    for s in (0, 5, 129):
        n = int(lengths[s])
        assert normwise(got_k[s, :n], kc[0, s, :n]) < 2 ** -8
        assert normwise(got_v[s, :n], vc[0, s, :n]) < 2 ** -8
