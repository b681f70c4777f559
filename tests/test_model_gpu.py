"""GPU parity of the whole flow-LM stack (ptts_b200_forward / ptts_b200_step) against the
oracle's StreamingTransformer::forward restatement.

Hidden states are the f32 residual stream after the last layer (per frame). The oracle runs
with store=ROUND_KV: rotated k and v rows are rounded to bf16 as they enter the cache, the one
16-bit storage point of the library's layer stack (GEMM inputs travel as f16 hi/lo pairs, which
keep f32-grade precision). Metric: ||gpu - oracle||_inf / ||oracle||_inf <= 2e-3.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import normwise

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _f32(t):
    return t.float().cpu().numpy()


def _setup(ptts, oracle, cfg, seed, S, cap, cuda):
    w = ptts.random_weights(cfg, seed)
    model = ptts.Transformer(cfg)
    model.load(w)
    om = oracle.Model(cfg, w)
    kv = ptts.KvState(cfg.num_layers, S, cap, dtype="bf16")
    shape = (cfg.num_layers, S, cap, cfg.num_heads, cfg.head_dim)
    return model, om, kv, np.zeros(shape, np.float32), np.zeros(shape, np.float32)


def _report(name, got, want):
    rowerr = np.abs(got - want).max(1) / np.abs(want).max()
    print(f"{name}: normwise {normwise(got, want):.3e}, median row {np.median(rowerr):.2e}, "
          f"rows > 1e-3: {(rowerr > 1e-3).sum()}/{len(rowerr)}")
    return normwise(got, want)


def test_prefill_then_decode_matches_the_oracle(ptts, oracle, cuda):
    """Ragged prompts (host path, t > 1) then host-position decode steps (t = 1), 31m shape."""
    import torch
    cfg = ptts.PHONON_31M
    S, cap = 6, 96
    model, om, kv, kc, vc = _setup(ptts, oracle, cfg, 3, S, cap, cuda)
    rows = [17, 40, 1, 33, 8, 25]
    streams = [4, 0, 5, 2, 1, 3]
    offs = np.concatenate([[0], np.cumsum(rows)]).astype(np.int32)
    x = torch.randn(int(offs[-1]), 512).bfloat16()
    y = model.forward(kv, x.to(cuda), streams, rows)
    kv.check()
    lengths = np.zeros(S, np.int32)
    kc32, vc32 = kc.copy(), vc.copy()
    want = om.forward(_f32(x), kc, vc, lengths, streams, offs, store=oracle.ROUND_KV)
    err = _report("prefill vs mirror", _f32(y), want)
    _report("prefill vs f32", _f32(y), om.forward(_f32(x), kc32, vc32, lengths, streams, offs, store=0))
    assert err < TOL
    for i, s in enumerate(streams):
        lengths[s] += rows[i]
    np.testing.assert_array_equal(kv.lengths(), lengths)
    worst = 0.0
    for frame in range(4):
        xs = torch.randn(S, 512).bfloat16()
        order = list(range(S))
        y = model.forward(kv, xs.to(cuda), order, [1] * S)
        want = om.forward(_f32(xs), kc, vc, lengths, order, np.arange(S + 1, dtype=np.int32), store=oracle.ROUND_KV)
        lengths += 1
        worst = max(worst, normwise(_f32(y), want))
    kv.check()
    print("decode normwise:", worst)
    assert worst < TOL
    for l in range(cfg.num_layers):
        kt, vt, _ = kv.tensors(l)
        for s in range(S):
            n = lengths[s]
            assert (_f32(kt[s, n:]) == 0).all() and (_f32(vt[s, n:]) == 0).all()
            d = np.abs(_f32(kt[s, :n]) - kc[l, s, :n]).max() / max(np.abs(kc[l, s, :n]).max(), 1e-30)
            assert d < 0.05, (l, s, d)


def test_a_device_step_is_the_host_step(ptts, cuda):
    """transformer.rs:1169-1225: the graph-replayed step (positions on the device) gives the
    host step's output and cache, frame after frame."""
    import torch
    cfg = ptts.FlowLMConfig(num_layers=3)
    w = ptts.random_weights(cfg, 9)
    model = ptts.Transformer(cfg)
    model.load(w)
    S, cap = 5, 40
    kvs = [ptts.KvState(cfg.num_layers, S, cap, dtype="bf16") for _ in range(2)]
    prompt = torch.randn(3 * S, 512).bfloat16().to(cuda)
    for kv in kvs:
        model.forward(kv, prompt, list(range(S)), [3] * S)
    streams = [3, 1, 4]
    for frame in range(5):
        x = torch.randn(len(streams), 512).bfloat16().to(cuda)
        host = model.forward(kvs[0], x, streams, [1] * len(streams))
        dev = model.step(kvs[1], streams, x)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(_f32(dev), _f32(host))
    np.testing.assert_array_equal(kvs[0].lengths(), kvs[1].lengths())
    for l in range(cfg.num_layers):
        np.testing.assert_array_equal(_f32(kvs[0].tensors(l)[0]), _f32(kvs[1].tensors(l)[0]))
    # The device lengths match the host mirror.
    np.testing.assert_array_equal(_f32(kvs[1].tensors(0)[2]).astype(np.int32), kvs[1].lengths())
    # A step past the capacity is refused on the host.
    full = ptts.KvState(cfg.num_layers, 1, 1, dtype="bf16")
    model.step(full, [0], torch.randn(1, 512).bfloat16().to(cuda))
    with pytest.raises(ptts.CapacityError):
        model.step(full, [0], torch.randn(1, 512).bfloat16().to(cuda))


def test_config4_decode_frames(ptts, oracle, cuda):
    """Config 4 (seed 3) shortened to 12 frames: 31m shape, 64 streams, prefix 128, per-frame
    hidden states of the device step against the oracle."""
    import torch
    cfg = ptts.PHONON_31M
    B, prefix, frames = 64, 128, 12
    model, om, kv, kc, vc = _setup(ptts, oracle, cfg, 3, B, prefix + frames, cuda)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(B * prefix, 512, generator=g).bfloat16()
    streams = list(range(B))
    offs = np.arange(0, B * prefix + 1, prefix, dtype=np.int32)
    model.forward(kv, x.to(cuda), streams, [prefix] * B)
    lengths = np.zeros(B, np.int32)
    om.forward(_f32(x), kc, vc, lengths, streams, offs, store=oracle.ROUND_KV)
    lengths += prefix
    errs = []
    for f in range(frames):
        xs = torch.randn(B, 512, generator=g).bfloat16()
        y = model.step(kv, streams, xs.to(cuda))
        want = om.forward(_f32(xs), kc, vc, lengths, streams, np.arange(B + 1, dtype=np.int32), store=oracle.ROUND_KV)
        lengths += 1
        errs.append(normwise(_f32(y), want))
    kv.check()
    print("config4 per-frame normwise:", ["%.2e" % e for e in errs])
    assert max(errs) < TOL


def test_two_lane_steps_match_the_oracle(ptts, oracle, cuda):
    """Decode steps of 200 streams, which run as two lanes (rows 0-95 and 96-199 on two CUDA
    streams inside the step graph): ragged prefixes and a permuted subset of the arena's
    streams, per step against the oracle."""
    import torch
    cfg = ptts.FlowLMConfig(num_layers=2)
    S, cap = 240, 48
    model, om, kv, kc, vc = _setup(ptts, oracle, cfg, 41, S, cap, cuda)
    rng = np.random.default_rng(41)
    rows = rng.integers(1, 40, size=S).astype(np.int32)
    offs = np.concatenate([[0], np.cumsum(rows)]).astype(np.int32)
    g = torch.Generator().manual_seed(41)
    x = torch.randn(int(offs[-1]), 512, generator=g).bfloat16()
    model.forward(kv, x.to(cuda), list(range(S)), rows.tolist())
    lengths = np.zeros(S, np.int32)
    om.forward(_f32(x), kc, vc, lengths, list(range(S)), offs, store=oracle.ROUND_KV)
    lengths += rows
    streams = [int(v) for v in rng.permutation(S)[:200]]
    errs = []
    for _ in range(3):
        xs = torch.randn(len(streams), 512, generator=g).bfloat16()
        y = model.step(kv, streams, xs.to(cuda))
        want = om.forward(_f32(xs), kc, vc, lengths, streams, np.arange(len(streams) + 1, dtype=np.int32),
                          store=oracle.ROUND_KV)
        lengths[streams] += 1
        errs.append(normwise(_f32(y), want))
    kv.check()
    np.testing.assert_array_equal(kv.lengths(), lengths)
    print("two-lane steps normwise:", ["%.2e" % e for e in errs])
    assert max(errs) < TOL


@pytest.mark.parametrize("env", [{"PTTS_B200_GEMM": "mma"}, {"PTTS_B200_PREFILL": "core"}],
                         ids=["mma-sync-linears", "cuda-core-prefill"])
def test_kernel_variants_match_the_oracle(ptts, oracle, cuda, monkeypatch, env):
    """The opt-in variants (mma.sync linears; the CUDA-core prefill attention) on the same
    prefill + decode as the default path, against the oracle."""
    import torch
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    cfg = ptts.PHONON_31M
    S, cap = 4, 160
    model, om, kv, kc, vc = _setup(ptts, oracle, cfg, 5, S, cap, cuda)
    rows = [130, 7, 64, 1]
    streams = [2, 0, 3, 1]
    offs = np.concatenate([[0], np.cumsum(rows)]).astype(np.int32)
    g = torch.Generator().manual_seed(5)
    x = torch.randn(int(offs[-1]), 512, generator=g).bfloat16()
    y = model.forward(kv, x.to(cuda), streams, rows)
    lengths = np.zeros(S, np.int32)
    want = om.forward(_f32(x), kc, vc, lengths, streams, offs, store=oracle.ROUND_KV)
    errs = [normwise(_f32(y), want)]
    for i, s in enumerate(streams):
        lengths[s] += rows[i]
    for frame in range(3):
        xs = torch.randn(S, 512, generator=g).bfloat16()
        y = model.step(kv, list(range(S)), xs.to(cuda))
        want = om.forward(_f32(xs), kc, vc, lengths, list(range(S)), np.arange(S + 1, dtype=np.int32),
                          store=oracle.ROUND_KV)
        lengths += 1
        errs.append(normwise(_f32(y), want))
    kv.check()
    print(env, "normwise:", ["%.2e" % e for e in errs])
    assert max(errs) < TOL


def test_long_prompts_match_the_oracle(ptts, oracle, cuda):
    """Prompts of 4096+ rows in one call (the linears' 64-row tcgen05 tiles, the tcgen05
    prefill attention over 1000+ keys), then a decode step."""
    import torch
    cfg = ptts.FlowLMConfig(num_layers=2)
    rows = [1100, 1003, 1200, 900]
    S, cap = len(rows), max(rows) + 4
    model, om, kv, kc, vc = _setup(ptts, oracle, cfg, 17, S, cap, cuda)
    g = torch.Generator().manual_seed(18)
    streams = [2, 0, 3, 1]
    offs = np.concatenate([[0], np.cumsum(rows)]).astype(np.int32)
    x = torch.randn(int(offs[-1]), 512, generator=g).bfloat16()
    y = model.forward(kv, x.to(cuda), streams, rows)
    lengths = np.zeros(S, np.int32)
    want = om.forward(_f32(x), kc, vc, lengths, streams, offs, store=oracle.ROUND_KV)
    errs = [normwise(_f32(y), want)]
    for i, s in enumerate(streams):
        lengths[s] += rows[i]
    xs = torch.randn(S, 512, generator=g).bfloat16()
    y = model.step(kv, list(range(S)), xs.to(cuda))
    want = om.forward(_f32(xs), kc, vc, lengths, list(range(S)), np.arange(S + 1, dtype=np.int32),
                      store=oracle.ROUND_KV)
    errs.append(normwise(_f32(y), want))
    kv.check()
    print("long prompts", ["%.2e" % e for e in errs])
    assert max(errs) < TOL


def test_full_config5_shard_on_sampled_streams(ptts, oracle, cuda):
    """The benchmark's whole per-GPU workload: the 40m stack (9 layers), 512 streams with
    prompts of U{32..512} rows (seed 4, 139k rows in one prefill: the persistent prompt
    linears and the tcgen05 prefill attention), then decode steps of all 512 streams (two
    lanes, compact-ring attention). Streams never interact, so the oracle runs only a sample of
    them, on their own prompts and inputs, and every sampled stream's rows are compared."""
    import importlib
    import torch
    wl = importlib.import_module("xn_ptts_b200.workloads")
    cfg = ptts.PHONON_40M
    B = 512
    prefixes = np.asarray(wl.prefix_lengths(4096, 32, 512, 4)[:B], np.int32)
    cap = int(prefixes.max()) + 4
    w = ptts.random_weights(cfg, 4)
    model = ptts.Transformer(cfg)
    model.load(w)
    kv = ptts.KvState(cfg.num_layers, B, cap, dtype="bf16")
    offs = np.concatenate([[0], np.cumsum(prefixes)]).astype(np.int32)
    g = torch.Generator().manual_seed(4)
    x = torch.randn(int(offs[-1]), 512, generator=g).bfloat16()
    y = model.forward(kv, x.to(cuda), list(range(B)), prefixes.tolist())
    y = _f32(y)
    steps = [torch.randn(B, 512, generator=g).bfloat16() for _ in range(3)]
    ys = [_f32(model.step(kv, list(range(B)), xs.to(cuda))) for xs in steps]
    kv.check()
    np.testing.assert_array_equal(kv.lengths(), prefixes + len(steps))

    sample = np.random.default_rng(4).choice(B, size=8, replace=False)
    sample.sort()
    om = oracle.Model(cfg, w)
    shape = (cfg.num_layers, len(sample), cap, cfg.num_heads, cfg.head_dim)
    kc, vc = np.zeros(shape, np.float32), np.zeros(shape, np.float32)
    xf = _f32(x)
    rows = prefixes[sample]
    o_offs = np.concatenate([[0], np.cumsum(rows)]).astype(np.int32)
    xin = np.concatenate([xf[offs[b]:offs[b + 1]] for b in sample])
    lengths = np.zeros(len(sample), np.int32)
    local = list(range(len(sample)))
    want = om.forward(xin, kc, vc, lengths, local, o_offs, store=oracle.ROUND_KV)
    got = np.concatenate([y[offs[b]:offs[b + 1]] for b in sample])
    errs = [_report("config-5 prefill (sampled streams)", got, want)]
    lengths += rows
    for i, xs in enumerate(steps):
        want = om.forward(_f32(xs)[sample], kc, vc, lengths, local,
                          np.arange(len(sample) + 1, dtype=np.int32), store=oracle.ROUND_KV)
        lengths += 1
        errs.append(_report(f"config-5 step {i}", ys[i][sample], want))
    assert max(errs) < TOL


def test_grouped_query_attention_in_the_stack(ptts, oracle, cuda):
    """num_kv_heads < num_heads through the whole stack (transformer.rs:1112-1164's equivalence,
    here against the oracle's GQA): a ragged prompt and decode steps."""
    import torch
    cfg = ptts.FlowLMConfig(num_layers=2, num_kv_heads=4)
    S, cap = 4, 64
    model, om, kv, kc, vc = _setup(ptts, oracle, cfg, 23, S, cap, cuda)
    g = torch.Generator().manual_seed(24)
    rows = [20, 3, 33, 9]
    streams = [1, 3, 0, 2]
    offs = np.concatenate([[0], np.cumsum(rows)]).astype(np.int32)
    x = torch.randn(int(offs[-1]), 512, generator=g).bfloat16()
    y = model.forward(kv, x.to(cuda), streams, rows)
    lengths = np.zeros(S, np.int32)
    errs = [normwise(_f32(y), om.forward(_f32(x), kc, vc, lengths, streams, offs, store=oracle.ROUND_KV))]
    for i, s in enumerate(streams):
        lengths[s] += rows[i]
    for _ in range(3):
        xs = torch.randn(S, 512, generator=g).bfloat16()
        y = model.step(kv, list(range(S)), xs.to(cuda))
        errs.append(normwise(_f32(y), om.forward(_f32(xs), kc, vc, lengths, list(range(S)),
                                                 np.arange(S + 1, dtype=np.int32), store=oracle.ROUND_KV)))
        lengths += 1
    kv.check()
    print("gqa", ["%.2e" % e for e in errs])
    assert max(errs) < TOL


def test_kernel_stamps_of_a_two_lane_step(ptts, cuda):
    """The kernel timeline (ptts_b200_model_stamps) of a two-lane step: every launch of both
    lanes is stamped, each kernel starts after its predecessor in the lane ended, and the
    stamped step's output equals an unstamped step's bit for bit."""
    import torch
    cfg = ptts.FlowLMConfig(num_layers=2)
    S, P = 160, 12
    w = ptts.random_weights(cfg, 61)
    model = ptts.Transformer(cfg)
    model.load(w)
    kvs = [ptts.KvState(cfg.num_layers, S, 32, dtype="bf16") for _ in range(2)]
    g = torch.Generator().manual_seed(61)
    x = torch.randn(S * P, 512, generator=g).bfloat16().to(cuda)
    for kv in kvs:
        model.forward(kv, x, list(range(S)), [P] * S)
    xs = torch.randn(S, 512, generator=g).bfloat16().to(cuda)
    plain = model.step(kvs[0], list(range(S)), xs).clone()
    model.stamps(64)
    stamped = model.step(kvs[1], list(range(S)), xs).clone()
    st = model.read_stamps()
    model.stamps(0)
    assert torch.equal(plain, stamped)
    kernels = ["ln1", "in_proj", "attention", "out_proj", "ln2", "linear1", "linear2"]
    for lane in (0, 1):
        seq = [e for e in st if e["lane"] == lane]
        assert [e["kernel"] for e in seq] == kernels * cfg.num_layers + ["ln_out"]
        assert [e["layer"] for e in seq[:-1]] == [l for l in range(cfg.num_layers) for _ in kernels]
        for a, b in zip(seq, seq[1:]):
            assert 0 <= b["entry_us"] <= b["start_us"] <= b["end_us"]
            assert b["entry_us"] <= b["last_entry_us"] <= b["end_us"]
            assert b["start_us"] >= a["end_us"] - 0.1, (a, b)
    with pytest.raises(ptts.PttsError, match="stamps are off"):
        model.read_stamps()
    model.step(kvs[0], list(range(S)), xs)  # the unstamped graph again
    kvs[0].check()
