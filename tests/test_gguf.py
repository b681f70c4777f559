"""GGUF checkpoints with q8_0 linears (loader.rs:15-67, examples/quantize.rs:46-47): the key
remap against the reference's own test vectors (CPU), and a q8_0 model loaded from a GGUF file
against the oracle with 32-wide scale blocks (GPU)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import normwise
from gguf_fixture import write

TOL = 2e-3


def test_remap_key_renames_and_drops(ptts):
    """loader.rs:484-527 (remap_key_renames_and_drops, flow_lm_flow_is_renamed_not_dropped)."""
    for dropped in ["flow_lm.flow.w_s_t", "mimi.quantizer.vq.something", "mimi.quantizer.logvar_proj.weight"]:
        assert ptts.gguf_remap_key(dropped) is None, dropped
    cases = [
        ("flow_lm.condition_provider.conditioners.speaker_wavs.output_proj.weight", "flow_lm.speaker_proj_weight"),
        ("flow_lm.condition_provider.conditioners.transcript_in_segment.emb.weight", "flow_lm.conditioner.emb.weight"),
        ("flow_lm.backbone.layers.0.linear1.weight", "flow_lm.transformer.layers.0.linear1.weight"),
        ("mimi.model.decoder.layers.0.weight", "mimi.decoder.layers.0.weight"),
        ("mimi.decoder.layers.0.weight", "mimi.decoder.layers.0.weight"),
        ("flow_lm.flow.layers.0.weight", "flow_lm.flow_net.layers.0.weight"),
    ]
    for src, dst in cases:
        assert ptts.gguf_remap_key(src) == dst, src


def test_q8_0_quantizer_is_the_published_format(ptts):
    """quantize_q8_0 (the q8_0 of Q8Linear::from_linear, q8.rs:29-35): per 32 weights an f16
    d = max |w| / 127 and int8 q = round(w / d), laid out as the GGUF blocks; dequantized with
    the stored f16 d, every weight is within half a step of the original plus the f16 rounding
    of d over at most 127 steps (d (1/2 + 127 * 2^-11)), and all-zero blocks stay zero."""
    from gguf_fixture import q8_0_blocks
    rng = np.random.default_rng(97)
    w = rng.normal(0.0, 0.05, (48, 96)).astype(np.float32)
    w[3, 32:64] = 0.0
    blocks = ptts.quantize_q8_0(w)
    assert blocks.shape == (48, 3 * 34) and blocks.dtype == np.uint8
    b = blocks.reshape(48, 3, 34)
    d = b[..., :2].copy().view(np.float16).reshape(48, 3).astype(np.float32)
    q = b[..., 2:].copy().view(np.int8).astype(np.float32)
    np.testing.assert_array_equal(blocks, q8_0_blocks(q.reshape(48, 96).astype(np.int8), d))
    deq = (q * d[..., None]).reshape(48, 96)
    assert np.all(np.abs(deq - w) <= (0.5 + 127 * 2.0 ** -11) * np.repeat(d, 32, axis=1) * (1 + 1e-3) + 1e-12)
    assert np.all(deq[3, 32:64] == 0.0) and d[3, 1] == 0.0


def _q8_layers(cfg, seed):
    """Per layer: int8 q ~ U{-127..127} and f16 block scales ~ U(0.005, 0.02) for the four
    linears (the regime of the int8 tests), LayerNorm gain 1/16."""
    rng = np.random.default_rng(seed)
    d, hd, ff = cfg.d_model, cfg.num_heads * cfg.head_dim, cfg.dim_feedforward
    nqkv = hd + 2 * cfg.num_kv_heads * cfg.head_dim
    shapes = {"in_proj": (nqkv, d), "out_proj": (d, hd), "linear1": (ff, d), "linear2": (d, ff)}
    layers = []
    for _ in range(cfg.num_layers):
        lay = {}
        for k, (n, kk) in shapes.items():
            q = rng.integers(-127, 128, size=(n, kk), dtype=np.int8)
            s = rng.uniform(0.005, 0.02, size=(n, kk // 32)).astype(np.float16).astype(np.float32)
            lay[k] = (q, s)
        layers.append(lay)
    return layers


def _oracle_weights(ptts, cfg, layers):
    g = lambda k, i: np.stack([lay[k][i] for lay in layers])
    L, d = cfg.num_layers, cfg.d_model
    ln = lambda v: np.full((L, d), v, np.float32)
    return ptts.Weights(g("in_proj", 0), g("in_proj", 1), g("out_proj", 0), g("out_proj", 1),
                        g("linear1", 0), g("linear1", 1), g("linear2", 0), g("linear2", 1),
                        ln(ptts.LN_GAIN), ln(0.0), ln(ptts.LN_GAIN), ln(0.0))


def _upstream(name: str) -> str:
    """A flow-head tensor's key as an upstream checkpoint spells it (before remap_key)."""
    return "flow_lm." + (name.replace("flow_net.", "flow.", 1) if name.startswith("flow_net.") else name)


def _write_checkpoint(ptts, path, cfg, layers, flow_w):
    t = []
    for l, lay in enumerate(layers):
        p = f"flow_lm.backbone.layers.{l}."
        t += [(p + "self_attn.in_proj.weight", "q8_0", lay["in_proj"]),
              (p + "self_attn.out_proj.weight", "q8_0", lay["out_proj"]),
              (p + "linear1.weight", "q8_0", lay["linear1"]),
              (p + "linear2.weight", "q8_0", lay["linear2"])]
        for n in ("norm1", "norm2"):
            t += [(p + n + ".weight", "f32", np.full(cfg.d_model, ptts.LN_GAIN, np.float32)),
                  (p + n + ".bias", "f32", np.zeros(cfg.d_model, np.float32))]
    for name, v in flow_w.items():
        t.append((_upstream(name), "f16" if name == "bos_emb" else "f32", v))
    # Tensors the loader drops or leaves to others.
    t += [("flow_lm.flow.w_s_t.weight", "f32", np.ones(4, np.float32)),
          ("mimi.model.decoder.conv.weight", "f32", np.ones(3, np.float32)),
          ("flow_lm.emb_mean", "f32", np.zeros(32, np.float32))]
    write(str(path), t)


@pytest.mark.gpu
def test_q8_0_checkpoint_matches_the_oracle(ptts, oracle, cuda, tmp_path):
    """A 2-layer q8_0 model and the flow head from one GGUF file (upstream key names), then
    prompts below and above 4096 rows (the two tcgen05 row tiles) and decode steps, against
    the oracle with 32-wide scale blocks; the flow head samples against its oracle."""
    import torch
    from oracle import flow as of
    cfg = ptts.FlowLMConfig(num_layers=2, scale_group=32)
    fcfg = ptts.PHONON_FLOW
    layers = _q8_layers(cfg, 31)
    flow_w = ptts.random_flow_weights(fcfg, 32)
    flow_w["bos_emb"] = flow_w["bos_emb"].astype(np.float16).astype(np.float32)
    path = tmp_path / "model.q8.gguf"
    _write_checkpoint(ptts, path, cfg, layers, flow_w)
    model = ptts.Transformer(cfg)
    flow = ptts.Flow(fcfg)
    model.load_gguf(str(path), flow)
    om = oracle.Model(cfg, _oracle_weights(ptts, cfg, layers))
    g = torch.Generator().manual_seed(33)
    for rows in ([30, 7, 1, 12], [1030, 1030, 1031, 1029]):
        S, cap = len(rows), max(rows) + 8
        kv = ptts.KvState(cfg.num_layers, S, cap, dtype="bf16")
        shape = (cfg.num_layers, S, cap, cfg.num_heads, cfg.head_dim)
        kc, vc = np.zeros(shape, np.float32), np.zeros(shape, np.float32)
        streams = list(range(S))
        offs = np.concatenate([[0], np.cumsum(rows)]).astype(np.int32)
        x = torch.randn(int(offs[-1]), 512, generator=g).bfloat16()
        y = model.forward(kv, x.to(cuda), streams, rows)
        lengths = np.zeros(S, np.int32)
        want = om.forward(x.float().numpy(), kc, vc, lengths, streams, offs, store=oracle.ROUND_KV)
        errs = [normwise(y.cpu().numpy(), want)]
        lengths += np.array(rows, np.int32)
        for _ in range(3):
            xs = torch.randn(S, 512, generator=g).bfloat16()
            y = model.step(kv, streams, xs.to(cuda))
            want = om.forward(xs.float().numpy(), kc, vc, lengths, streams, np.arange(S + 1, dtype=np.int32),
                              store=oracle.ROUND_KV)
            lengths += 1
            errs.append(normwise(y.cpu().numpy(), want))
        kv.check()
        print(sum(rows), "rows: prompt and decode normwise", ["%.2e" % e for e in errs])
        assert max(errs) < TOL
    t = np.random.default_rng(34).normal(size=(9, 512)).astype(np.float32)
    z = np.random.default_rng(35).normal(size=(9, 32)).astype(np.float32)
    lat, eos = flow.sample(torch.from_numpy(t).to(cuda), torch.from_numpy(z).to(cuda))
    want_l, want_e = of.sample_from_noise(fcfg, flow_w, t, z)
    assert normwise(lat.cpu().numpy(), want_l) < TOL and normwise(eos.cpu().numpy(), want_e) < TOL


@pytest.mark.gpu
def test_gguf_refusals(ptts, cuda, tmp_path):
    """Missing or misshaped tensors and broken files are refused, naming what is wrong."""
    cfg = ptts.FlowLMConfig(num_layers=2)
    layers = _q8_layers(cfg, 41)
    model = ptts.Transformer(cfg)
    full = tmp_path / "full.gguf"
    _write_checkpoint(ptts, full, cfg, layers, {})
    model.load_gguf(str(full))  # no flow head asked for: its tensors may be absent
    short = tmp_path / "short.gguf"
    _write_checkpoint(ptts, short, cfg, layers[:1], {})
    with pytest.raises(ptts.PttsError, match="missing: flow_lm.transformer.layers.1.self_attn.in_proj.weight"):
        model.load_gguf(str(short))
    bad = [dict(lay) for lay in layers]
    q, s = bad[1]["linear2"]
    bad[1]["linear2"] = (q[:, :1024], s[:, :32])
    misshaped = tmp_path / "misshaped.gguf"
    _write_checkpoint(ptts, misshaped, cfg, bad, {})
    with pytest.raises(ptts.PttsError, match="layers.1.linear2.weight: expected dims"):
        model.load_gguf(str(misshaped))
    junk = tmp_path / "junk.gguf"
    junk.write_bytes(b"GGML" + bytes(64))
    with pytest.raises(ptts.PttsError, match="not a GGUF file"):
        model.load_gguf(str(junk))
    cut = tmp_path / "cut.gguf"
    cut.write_bytes(full.read_bytes()[:-1000])
    with pytest.raises(ptts.PttsError, match="past the end"):
        model.load_gguf(str(cut))
    flow = ptts.Flow(ptts.PHONON_FLOW)
    with pytest.raises(ptts.PttsError, match="flow tensor missing"):
        model.load_gguf(str(full), flow)


@pytest.mark.gpu
def test_q8_0_widened_on_chip_equals_the_planes(ptts, cuda, tmp_path, monkeypatch):
    """Below 4096 rows a q8_0 layer's linears read the int8 values and block scales and widen
    them on chip into the f16 hi/lo weights its planes hold (lo mostly f16 subnormals); with
    the same MMA order that is bit for bit the planes path (PTTS_B200_Q8=planes), prompts and
    decode steps alike. Layer 1 has blocks whose scale over the row's power of two is not an
    exact f16 (2^10 below the rest): that layer keeps to its planes."""
    import torch
    cfg = ptts.FlowLMConfig(num_layers=2, scale_group=32)
    layers = _q8_layers(cfg, 51)
    # Blocks of mixed magnitude in a row: the row's power of two then sits well above some.
    for lay, f in zip(layers, (1.0 / 8, 1.0 / 1024)):
        q, s = lay["linear1"]
        s[:, ::7] *= f
        lay["linear1"] = (q, s.astype(np.float16).astype(np.float32))
    path = tmp_path / "model.q8.gguf"
    _write_checkpoint(ptts, path, cfg, layers, {})
    rows, S = [30, 7, 1, 12], 4
    x = torch.randn(sum(rows), 512, generator=torch.Generator().manual_seed(52)).bfloat16()
    xs = [torch.randn(S, 512, generator=torch.Generator().manual_seed(53 + i)).bfloat16() for i in range(3)]

    def run():
        model = ptts.Transformer(cfg)
        model.load_gguf(str(path))
        kv = ptts.KvState(cfg.num_layers, S, max(rows) + 8, dtype="bf16")
        out = [model.forward(kv, x.to(cuda), list(range(S)), rows).cpu()]
        out += [model.step(kv, list(range(S)), v.to(cuda)).cpu() for v in xs]
        kv.check()
        return out

    monkeypatch.delenv("PTTS_B200_Q8", raising=False)
    on_chip = run()
    monkeypatch.setenv("PTTS_B200_Q8", "planes")
    planes = run()
    for a, b in zip(on_chip, planes):
        assert torch.equal(a, b)
