"""The flow head (FlowLM's frame tail and its SimpleMLPAdaLN flow net) against the numpy oracle
(oracle/flow.py), and the oracle against the reference's own unit test of the time norms.

Metric: ||gpu - oracle||_inf / ||oracle||_inf <= 2e-3 (the flow net's linears run on the tensor
cores with bf16 hi/lo activations and, for f32 weights, bf16 hi/lo weights).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import normwise

TOL = 2e-3


def test_time_norms_follow_their_formulas():
    """mlp.rs:253-277: the row [1, 2, 3, 6] with alpha = 2 under both time norms."""
    from oracle import flow as of
    xs = np.array([[1.0, 2.0, 3.0, 6.0]])
    alpha = np.full(4, 2.0)
    n, eps = 4.0, 1e-5
    mean = xs.sum() / n
    var = ((xs - mean) ** 2).sum() / (n - 1)
    ms = (xs * xs).sum() / n
    np.testing.assert_allclose(of.time_norm(xs, alpha, "rms"), 2.0 * xs / np.sqrt(ms + eps), atol=1e-5)
    np.testing.assert_allclose(of.time_norm(xs, alpha, "rms_var"), 2.0 * xs / np.sqrt(var + eps), atol=1e-5)


def test_pointwise_is_noise_plus_drifting(ptts):
    """FlowType::Pointwise adds the noise to the flow net's output, FlowType::Drifting returns
    it (flow_lm.rs:379-381): same weights, same inputs."""
    from oracle import flow as of
    rng = np.random.default_rng(1)
    cfg_d = ptts.FlowConfig(flow_dim=128, flow_depth=2, flow_type="drifting")
    cfg_p = ptts.FlowConfig(flow_dim=128, flow_depth=2, flow_type="pointwise")
    W = ptts.random_flow_weights(cfg_d, 2)
    t = rng.normal(size=(5, 512)).astype(np.float32)
    z = rng.normal(size=(5, 32)).astype(np.float32)
    ld, ed = of.sample_from_noise(cfg_d, W, t, z)
    lp, ep = of.sample_from_noise(cfg_p, W, t, z)
    np.testing.assert_allclose(lp, z + ld, rtol=1e-12, atol=1e-12)
    np.testing.assert_array_equal(ed, ep)


def test_flow_tensor_names_are_the_checkpoint_keys(ptts):
    """FlowLM::load and SimpleMLPAdaLN::load paths (flow_lm.rs:196-283, mlp.rs:179-201)."""
    sh = ptts.PHONON_FLOW.shapes()
    assert sh["flow_net.res_blocks.5.adaLN_modulation.1.weight"] == (1536, 512)
    assert sh["flow_net.time_embed.1.mlp.0.weight"] == (512, 256)
    assert sh["flow_net.final_layer.linear.weight"] == (32, 512)
    assert "flow_net.res_blocks.6.in_ln.weight" not in sh
    assert "flow_net.time_embed.0.freqs" not in ptts.FlowConfig(flow_type="drifting").shapes()


def _flow(ptts, cfg, seed, **kw):
    W = ptts.random_flow_weights(cfg, seed, **kw)
    f = ptts.Flow(cfg)
    f.load(W)
    return f, W


@pytest.mark.gpu
@pytest.mark.parametrize("kind", [
    dict(),                                                   # phonon: LSD, 1 step, rms
    dict(lsd_steps=2, time_norm="rms_var"),                   # pocket-tts norm, two solver steps
    dict(flow_type="pointwise", flow_depth=3),
    dict(flow_type="drifting", flow_depth=2, flow_dim=256),
], ids=["lsd1-rms", "lsd2-rmsvar", "pointwise", "drifting"])
@pytest.mark.parametrize("exact", [True, False], ids=["bf16-weights", "f32-weights"])
def test_flow_sample_matches_the_oracle(ptts, cuda, kind, exact):
    import torch
    from oracle import flow as of
    cfg = ptts.FlowConfig(**kind)
    f, W = _flow(ptts, cfg, 3, bf16_exact=exact)
    rng = np.random.default_rng(4)
    n = 37
    t = rng.normal(size=(n, cfg.d_model)).astype(np.float32)
    z = rng.normal(size=(n, cfg.ldim)).astype(np.float32)
    latent, eos = f.sample(torch.from_numpy(t).to(cuda), torch.from_numpy(z).to(cuda))
    want_l, want_e = of.sample_from_noise(cfg, W, t, z)
    el, ee = normwise(latent.cpu().numpy(), want_l), normwise(eos.cpu().numpy(), want_e)
    print(kind, exact, "latent", el, "eos", ee)
    assert el < TOL and ee < TOL


@pytest.mark.gpu
@pytest.mark.parametrize("S", [6, 200])
def test_frames_match_the_oracle(ptts, oracle, cuda, S):
    """A prompt, then frames from bos_emb: input_linear -> device step -> out_norm -> flow
    sample, per frame against the oracle fed the same latents (flow_lm.rs:392-410). 200 streams
    run the step as two lanes."""
    import torch
    from oracle import flow as of
    mcfg = ptts.FlowLMConfig(num_layers=2)
    fcfg = ptts.PHONON_FLOW
    w = ptts.random_weights(mcfg, 7)
    model = ptts.Transformer(mcfg)
    model.load(w)
    om = oracle.Model(mcfg, w)
    f, W = _flow(ptts, fcfg, 8, condition=True)
    P, cap = 20, 40
    kv = ptts.KvState(mcfg.num_layers, S, cap, dtype="bf16")
    shape = (mcfg.num_layers, S, cap, mcfg.num_heads, mcfg.head_dim)
    kc, vc = np.zeros(shape, np.float32), np.zeros(shape, np.float32)
    g = torch.Generator().manual_seed(9)
    prompt = torch.randn(S * P, 512, generator=g).bfloat16()
    streams = list(range(S))
    model.forward(kv, prompt.to(cuda), streams, [P] * S)
    lengths = np.zeros(S, np.int32)
    om.forward(prompt.float().numpy(), kc, vc, lengths, streams,
               np.arange(0, S * P + 1, P, dtype=np.int32), store=oracle.ROUND_KV)
    lengths += P
    latent = None
    for frame in range(4):
        z = torch.randn(S, fcfg.ldim, generator=g)
        got_l, got_e = f.frame(model, kv, streams, latent, z.to(cuda))
        x = oracle.round_bf16(of.frame_input(fcfg, W, None if latent is None else latent.cpu().numpy())
                              .astype(np.float32))
        if latent is None:
            x = np.repeat(x, S, 0)
        hidden = om.forward(x, kc, vc, lengths, streams, np.arange(S + 1, dtype=np.int32), store=oracle.ROUND_KV)
        lengths += 1
        want_l, want_e = of.sample_from_noise(fcfg, W, of.out_norm(W, hidden), z.numpy())
        el = normwise(got_l.cpu().numpy(), want_l)
        ee = normwise(got_e.cpu().numpy(), want_e)
        print("frame", frame, "latent", el, "eos", ee)
        assert el < TOL and ee < TOL
        latent = got_l
    np.testing.assert_array_equal(kv.lengths(), lengths)


@pytest.mark.gpu
def test_flow_loader_refuses_bad_tensors(ptts, cuda):
    """Unknown names and wrong sizes are refused when set, missing tensors at finish, and
    sampling before finish (ptts_b200_last_error names the tensor)."""
    import torch
    cfg = ptts.FlowConfig(flow_dim=128, flow_depth=1)
    f = ptts.Flow(cfg)
    with pytest.raises(ptts.PttsError, match="unknown flow tensor"):
        f.set("flow_net.res_blocks.1.in_ln.weight", np.ones(128, np.float32))
    with pytest.raises(ptts.PttsError, match="expected 128"):
        f.set("flow_net.res_blocks.0.in_ln.weight", np.ones(64, np.float32))
    W = ptts.random_flow_weights(cfg, 1)
    W.pop("flow_net.final_layer.linear.bias")
    with pytest.raises(ptts.PttsError, match="final_layer.linear.bias"):
        f.load(W)
    t = torch.zeros(2, 512, device=cuda)
    with pytest.raises(ptts.PttsError, match="not finished"):
        f.sample(t, torch.zeros(2, 32, device=cuda))
