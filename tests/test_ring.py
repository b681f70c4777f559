"""Ring caches (StreamingTransformer::start_ring / set_ring_slot / evict, transformer.rs:840-929):
the reference's two ring tests (transformer.rs:1359-1419) re-expressed on the GPU path, with the
oracle run on the ring's kept rows as the strict reference.

The oracle keeps a ring stream's rows compacted (only the kept rows, in the order written):
attention does not depend on key order, and a ring's length equals its number of kept rows, so
appending at the length reproduces the ring's RoPE positions. Eviction there drops the rows and
rotates every kept key past the prefix back by the count (rounded to bf16 again, as the cache
holds bf16).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import normwise

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _rotate_back(oracle, k, shift):
    """RotaryEmbedding::shift_back then rotate (rope.rs:26-35, :37-95) on rows [n, H, D]:
    angle f32(-shift) * inv_freq[i], interleaved pairs, f32 arithmetic, bf16 storage."""
    inv = oracle.rope_inv_freq(64).astype(np.float32)
    ang = (np.float32(-shift) * inv).astype(np.float32)
    c = np.cos(ang.astype(np.float64)).astype(np.float32)
    s = np.sin(ang.astype(np.float64)).astype(np.float32)
    x0, x1 = k[..., 0::2].astype(np.float32), k[..., 1::2].astype(np.float32)
    y = np.empty_like(k, dtype=np.float32)
    y[..., 0::2] = x0 * c - x1 * s
    y[..., 1::2] = x0 * s + x1 * c
    return oracle.round_bf16(y)


@pytest.mark.parametrize("path", ["forward", "step"])
def test_evicting_leaves_the_cache_of_a_sequence_without_them(ptts, oracle, cuda, path):
    """transformer.rs:1359-1395: a 5-row prompt and 6 frame slots whose oldest 3 frames go
    whenever they are full, over 15 frames (three evictions, the later ones wrapping round the
    ring so the kept frames lie in two runs). One layer, where a row's key and value depend on
    its own input and position alone: every frame must see what it would have seen had the
    evicted frames never been there. Checked against the oracle on the kept rows (strict) and
    against a plain sequence of the prompt and the frames in view (semantic: the kept keys
    carry one more bf16 rounding)."""
    import torch
    cfg = ptts.FlowLMConfig(num_layers=1)
    w = ptts.random_weights(cfg, 11)
    model = ptts.Transformer(cfg)
    model.load(w)
    om = oracle.Model(cfg, w)
    P, SLOTS, FR = 5, 6, 15
    cap = P + SLOTS
    g = torch.Generator().manual_seed(12)
    prompt = torch.randn(P, 512, generator=g).bfloat16()
    frames = torch.randn(FR, 512, generator=g).bfloat16()
    kv = ptts.KvState(1, 1, cap, dtype="bf16")
    model.forward(kv, prompt.to(cuda), [0], [P])
    kv.start_ring([0])
    kc = np.zeros((1, 1, cap, 8, 64), np.float32)
    vc = np.zeros_like(kc)
    lengths = np.zeros(1, np.int32)
    om.forward(prompt.float().numpy(), kc, vc, lengths, [0], np.array([0, P], np.int32), store=oracle.ROUND_KV)
    lengths[0] = P
    slot_of_row = list(range(P))
    in_view, worst, worst_sem = 0, 0.0, 0.0
    for i in range(FR):
        if in_view == SLOTS:
            oldest = i - in_view
            slots = [P + (oldest + j) % SLOTS for j in range(3)]
            kv.evict(0, P, slots)
            keep = [r for r, s in enumerate(slot_of_row) if s not in slots]
            k_kept, v_kept = kc[:, 0, keep].copy(), vc[:, 0, keep].copy()
            k_kept[:, P:] = _rotate_back(oracle, k_kept[:, P:], len(slots))
            kc[:, 0] = 0
            vc[:, 0] = 0
            kc[:, 0, :len(keep)] = k_kept
            vc[:, 0, :len(keep)] = v_kept
            slot_of_row = [slot_of_row[r] for r in keep]
            lengths[0] -= len(slots)
            in_view -= len(slots)
            assert kv.lengths()[0] == P + in_view
        slot = P + i % SLOTS
        kv.set_ring_slot(0, slot)
        x = frames[i:i + 1]
        got = (model.forward(kv, x.to(cuda), [0], [1]) if path == "forward" else model.step(kv, [0], x.to(cuda)))
        got = got.float().cpu().numpy()
        want = om.forward(x.float().numpy(), kc, vc, lengths, [0], np.array([0, 1], np.int32), store=oracle.ROUND_KV)
        lengths[0] += 1
        slot_of_row.append(slot)
        in_view += 1
        worst = max(worst, normwise(got, want))
        # The plain sequence without the evicted frames.
        plain = ptts.KvState(1, 1, cap, dtype="bf16")
        model.forward(plain, prompt.to(cuda), [0], [P])
        for j in range(i + 1 - in_view, i + 1):
            ref = model.forward(plain, frames[j:j + 1].to(cuda), [0], [1])
        worst_sem = max(worst_sem, normwise(got, ref.float().cpu().numpy()))
        plain.close()
    kv.check()
    print(path, "ring vs oracle", worst, "ring vs plain sequence", worst_sem)
    assert worst < TOL
    assert worst_sem < 1e-2


@pytest.mark.parametrize("S,rings", [(3, [1]), (160, [1, 130])], ids=["one-lane", "two-lanes"])
def test_ring_and_appended_streams_share_a_batch(ptts, oracle, cuda, S, rings):
    """A decode batch mixing ring streams (each with a hole from an eviction) and appended
    streams: every row against the oracle (a ring stream on its kept rows). 160 streams run the
    step as two lanes, with a ring stream in each."""
    import torch
    cfg = ptts.FlowLMConfig(num_layers=2)
    w = ptts.random_weights(cfg, 21)
    model = ptts.Transformer(cfg)
    model.load(w)
    om = oracle.Model(cfg, w)
    P, cap = 8, 16
    streams = list(range(S))
    g = torch.Generator().manual_seed(22)
    kv = ptts.KvState(cfg.num_layers, S, cap, dtype="bf16")
    prompt = torch.randn(S * P, 512, generator=g).bfloat16()
    model.forward(kv, prompt.to(cuda), streams, [P] * S)
    shape = (cfg.num_layers, S, cap, 8, 64)
    kc, vc = np.zeros(shape, np.float32), np.zeros(shape, np.float32)
    lengths = np.zeros(S, np.int32)
    om.forward(prompt.float().numpy(), kc, vc, lengths, streams, np.arange(0, S * P + 1, P, dtype=np.int32),
               store=oracle.ROUND_KV)
    lengths += P
    kv.start_ring(rings)
    # Evict slots 5 and 6 of each ring stream (past a prefix of 4): rows 5, 6 go, 7 rotates back by 2.
    keep = [0, 1, 2, 3, 4, 7]
    for r in rings:
        kv.evict(r, 4, [5, 6])
        for l in range(cfg.num_layers):
            k_kept, v_kept = kc[l, r, keep].copy(), vc[l, r, keep].copy()
            k_kept[4:] = _rotate_back(oracle, k_kept[4:], 2)
            kc[l, r] = 0
            vc[l, r] = 0
            kc[l, r, :6] = k_kept
            vc[l, r, :6] = v_kept
        lengths[r] -= 2
        kv.set_ring_slot(r, 5)
    worst = 0.0
    for frame in range(3):
        if frame:
            for r in rings:
                kv.set_ring_slot(r, 8 + frame)  # fresh slots past the filled ones
        x = torch.randn(S, 512, generator=g).bfloat16()
        got = model.step(kv, streams, x.to(cuda)).float().cpu().numpy()
        want = om.forward(x.float().numpy(), kc, vc, lengths, streams, np.arange(S + 1, dtype=np.int32),
                          store=oracle.ROUND_KV)
        lengths += 1
        worst = max(worst, normwise(got, want))
    kv.check()
    np.testing.assert_array_equal(kv.lengths(), lengths)
    print("mixed batch", S, worst)
    assert worst < TOL


def test_misuse_of_a_ring_is_refused(ptts, cuda):
    """transformer.rs:1396-1419, plus the calls this library adds."""
    import torch
    cfg = ptts.FlowLMConfig(num_layers=1)
    model = ptts.Transformer(cfg)
    model.load(ptts.random_weights(cfg, 5))
    kv = ptts.KvState(1, 1, 8, dtype="bf16")
    row = lambda n: torch.randn(n, 512).bfloat16().to(cuda)
    model.forward(kv, row(4), [0], [4])
    with pytest.raises(ptts.PttsError, match="not a ring"):
        kv.set_ring_slot(0, 4)
    kv.start_ring([0])
    other = ptts.KvState(1, 1, 10, dtype="bf16")
    with pytest.raises(ptts.PttsError, match="cannot be resized"):
        other.copy_stream(0, kv, 0)
    kv.set_ring_slot(0, 4)
    model.forward(kv, row(1), [0], [1])
    with pytest.raises(ptts.PttsError, match="slot 2 holds no row past the prefix"):
        kv.evict(0, 4, [2])
    with pytest.raises(ptts.PttsError, match="slot 5 holds no row"):
        kv.evict(0, 4, [5])
    # Refused as a whole: slot 4 stays in the cache.
    with pytest.raises(ptts.PttsError):
        kv.evict(0, 4, [4, 5])
    kv.set_ring_slot(0, 4)
    with pytest.raises(ptts.PttsError, match="still holds a row"):
        model.forward(kv, row(1), [0], [1])
    kv.evict(0, 4, [4])
    model.forward(kv, row(1), [0], [1])
    # What this library adds: prompts, lengths, slots out of range, and reset.
    with pytest.raises(ptts.PttsError, match="one row at a time"):
        model.forward(kv, row(2), [0], [2])
    with pytest.raises(ptts.PttsError, match="eviction"):
        kv.set_lengths([0], [3])
    with pytest.raises(ptts.PttsError, match="8-slot ring"):
        kv.set_ring_slot(0, 8)
    with pytest.raises(ptts.PttsError, match="cannot evict 9 of 5"):
        kv.evict(0, 0, list(range(9)))
    assert kv.lengths()[0] == 5
    kv.check()
    kv.reset([0])
    with pytest.raises(ptts.PttsError, match="not a ring"):
        kv.set_ring_slot(0, 0)
    model.forward(kv, row(3), [0], [3])  # an appended stream again
    assert kv.lengths()[0] == 3


@pytest.mark.parametrize("S", [12, 150], ids=["in-launch", "copied"])
def test_set_ring_slots_is_set_ring_slot_for_each_stream(ptts, cuda, S):
    """ptts_b200_kv_set_ring_slots sets every listed ring's write slot in one call: frames
    stepped after it equal, bit for bit, the same frames stepped after one set_ring_slot per
    stream, on a second cache (both list forms: carried in the launch, and copied). A list
    naming a stream twice, or a stream that is not a ring, is refused and changes nothing: the
    frame after the refusals still matches."""
    import torch
    cfg = ptts.FlowLMConfig(num_layers=2)
    w = ptts.random_weights(cfg, 25)
    model = ptts.Transformer(cfg)
    model.load(w)
    P, cap = 6, 20
    streams = list(range(S))
    g = torch.Generator().manual_seed(26)
    prompt = torch.randn(S * P, 512, generator=g).bfloat16().to(cuda)
    kvs = [ptts.KvState(cfg.num_layers, S, cap, dtype="bf16") for _ in range(2)]
    rings = streams[: S - 2]  # two appended streams stay in the batch
    for kv in kvs:
        model.forward(kv, prompt, streams, [P] * S)
        kv.start_ring(rings)
        for r in rings[::3]:
            kv.evict(r, 2, [3, 4])

    def frame(f):
        # Free slots past the prompt, a different one per frame for each ring.
        slots = [(f + 3 * r) % (cap - P) + P for r in rings]
        for r, sl in zip(rings, slots):
            kvs[0].set_ring_slot(r, sl)
        kvs[1].set_ring_slots(rings, slots)
        x = torch.randn(S, 512, generator=g).bfloat16().to(cuda)
        a, b = model.step(kvs[0], streams, x), model.step(kvs[1], streams, x)
        torch.cuda.synchronize()
        assert torch.equal(a, b), f

    for f in range(4):
        frame(f)
    with pytest.raises(ptts.PttsError, match="twice"):
        kvs[1].set_ring_slots([rings[0], rings[0]], [P, P + 1])
    with pytest.raises(ptts.PttsError, match="not a ring"):
        kvs[1].set_ring_slots([rings[0], S - 1], [P, P])
    frame(4)
    for kv in kvs:
        kv.check()
    np.testing.assert_array_equal(kvs[0].lengths(), kvs[1].lengths())
    for l in range(cfg.num_layers):
        for t1, t2 in zip(kvs[0].tensors(l)[:2], kvs[1].tensors(l)[:2]):
            assert torch.equal(t1, t2)
