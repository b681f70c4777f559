"""TEST INFRASTRUCTURE ONLY: numpy restatement of the flow head (FlowLM's frame tail).

Follows the reference, in float64 with the f32 inputs it is given:
  * SimpleMLPAdaLN (ptts/src/mlp.rs:158-247): input_proj, cond_embed, y = t_emb + c, SiLU, the
    residual blocks, the final layer;
  * ResBlock::forward (mlp.rs:115-133): adaLN chunks (shift, scale, gate) in that order,
    LayerNorm eps 1e-6 with affine in_ln, modulate x (1 + scale) + shift (mlp.rs:4-11),
    linear -> SiLU -> linear, x + gate * h;
  * FinalLayer::forward (mlp.rs:150-157): LayerNorm eps 1e-6 without affine, adaLN (shift,
    scale), linear;
  * TimestepEmbedder (mlp.rs:54-81): cat(cos, sin)(t * freqs), linear1, SiLU, linear2, then
    the RMS norm (Rms: x a / sqrt(mean(x^2) + 1e-5); RmsVar: x a / sqrt(var_unbiased(x) + 1e-5));
    time_embedding averages the embedders (mlp.rs:204-211);
  * lsd_time_embeddings / lsd_decode (flow_lm.rs:84-112), sample_from_noise (flow_lm.rs:360-384)
    and the frame (sample_next_latent_step, flow_lm.rs:392-410 with backbone, :296-324).
Pinned by the reference's own unit test of the two time norms (mlp.rs:253-277), which
tests/test_flow.py re-expresses; otherwise parity unpinned, like the rest of the oracle.
Only tests and bench.py's CPU legs use it; the CUDA library never does.
"""
from __future__ import annotations

import numpy as np


def silu(x):
    return x / (1.0 + np.exp(-x))


def layer_norm(x, w=None, b=None, eps=1e-5):
    x = np.asarray(x, np.float64)
    mean = x.mean(-1, keepdims=True)
    var = ((x - mean) ** 2).mean(-1, keepdims=True)
    y = (x - mean) / np.sqrt(var + eps)
    if w is not None:
        y = y * w + b
    return y


def linear(x, w, b=None):
    y = np.asarray(x, np.float64) @ np.asarray(w, np.float64).T
    return y + b if b is not None else y


def time_norm(x, alpha, kind: str):
    """TimestepEmbedder::normalize (mlp.rs:70-81)."""
    x = np.asarray(x, np.float64)
    n = x.shape[-1]
    if kind == "rms":
        ms = (x * x).sum(-1, keepdims=True) / n
        return x / np.sqrt(ms + 1e-5) * alpha
    mean = x.sum(-1, keepdims=True) / n
    var = ((x - mean) ** 2).sum(-1, keepdims=True) / (n - 1)
    return x / np.sqrt(var + 1e-5) * alpha


def timestep_embed(W: dict, i: int, t: float, kind: str):
    p = f"flow_net.time_embed.{i}."
    args = (np.float32(t) * W[p + "freqs"].astype(np.float32)).astype(np.float64)  # f32 angle
    emb = np.concatenate([np.cos(args), np.sin(args)])
    h = silu(linear(emb, W[p + "mlp.0.weight"], W[p + "mlp.0.bias"]))
    y = linear(h, W[p + "mlp.2.weight"], W[p + "mlp.2.bias"])
    return time_norm(y, W[p + "mlp.3.alpha"], kind)


def time_embeddings(cfg, W: dict):
    """lsd_time_embeddings: one [flow_dim] row per solver step, conditioned on (i/N, (i+1)/N)."""
    N = cfg.lsd_steps
    out = []
    for i in range(N):
        s, t = np.float32(i) / np.float32(N), np.float32(i + 1) / np.float32(N)
        out.append((timestep_embed(W, 0, s, cfg.time_norm) + timestep_embed(W, 1, t, cfg.time_norm)) / 2.0)
    return out


def flow_net(cfg, W: dict, c, t_emb, x):
    """SimpleMLPAdaLN::forward: c [n, d], t_emb [C] or None, x [n, ldim] -> [n, ldim]."""
    C = cfg.flow_dim
    h = linear(x, W["flow_net.input_proj.weight"], W["flow_net.input_proj.bias"])
    y = linear(c, W["flow_net.cond_embed.weight"], W["flow_net.cond_embed.bias"])
    if t_emb is not None:
        y = y + t_emb
    y_act = silu(y)
    for b in range(cfg.flow_depth):
        p = f"flow_net.res_blocks.{b}."
        ada = linear(y_act, W[p + "adaLN_modulation.1.weight"], W[p + "adaLN_modulation.1.bias"])
        shift, scale, gate = ada[:, :C], ada[:, C:2 * C], ada[:, 2 * C:]
        g = layer_norm(h, W[p + "in_ln.weight"], W[p + "in_ln.bias"], 1e-6) * (1.0 + scale) + shift
        g = linear(silu(linear(g, W[p + "mlp.0.weight"], W[p + "mlp.0.bias"])),
                   W[p + "mlp.2.weight"], W[p + "mlp.2.bias"])
        h = h + gate * g
    p = "flow_net.final_layer."
    ada = linear(y_act, W[p + "adaLN_modulation.1.weight"], W[p + "adaLN_modulation.1.bias"])
    shift, scale = ada[:, :C], ada[:, C:]
    g = layer_norm(h, None, None, 1e-6) * (1.0 + scale) + shift
    return linear(g, W[p + "linear.weight"], W[p + "linear.bias"])


def sample_from_noise(cfg, W: dict, t_out, noise):
    """FlowLM::sample_from_noise: t_out [n, d] (after out_norm), noise [n, ldim] ->
    (latent [n, ldim], eos [n])."""
    t_out = np.asarray(t_out, np.float64)
    noise = np.asarray(noise, np.float64)
    eos = linear(t_out, W["out_eos.weight"], W["out_eos.bias"])[:, 0]
    if cfg.flow_type == "lsd":
        cur = noise
        for t_emb in time_embeddings(cfg, W):
            cur = cur + flow_net(cfg, W, t_out, t_emb, cur) / cfg.lsd_steps
        latent = cur
    elif cfg.flow_type == "drifting":
        latent = flow_net(cfg, W, t_out, None, noise)
    else:  # pointwise
        latent = noise + flow_net(cfg, W, t_out, None, noise)
    return latent, eos


def frame_input(cfg, W: dict, latent):
    """input_linear(latent) (+ the summed conditions), the backbone's input row; latent None
    starts from bos_emb (StepInput::Bos)."""
    if latent is None:
        latent = W["bos_emb"][None, :]
    x = linear(latent, W["input_linear.weight"])
    if "condition" in W:
        x = x + W["condition"]
    return x


def out_norm(W: dict, hidden):
    """The backbone's out_norm (flow_lm.rs:316), LayerNorm eps 1e-5."""
    return layer_norm(hidden, W["out_norm.weight"], W["out_norm.bias"], 1e-5)
