"""Windowed streams (Mimi's KvCache with a context, transformer.rs:257-317 and :395-468) through
the attention op, against the numpy restatement in oracle/window.py: prompts and decode steps
whose positions run past the capacity (the slots wrap), mixed in one call with an appended
stream, for bf16 and f32 caches; and the calls that refuse windowed streams."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import normwise

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,tol", [("bf16", 2e-3), ("f32", 1e-5)])
@pytest.mark.parametrize("kv_heads", [8, 4])
def test_windowed_attention_matches_mimi_kvcache(ptts, cuda, dtype, tol, kv_heads):
    import torch
    import oracle
    from oracle import window as ow
    cap, ctx = 12, 5
    kv = ptts.KvState(1, 3, cap, dtype=dtype)
    kv.set_window([0, 2], ctx)
    caches = [ow.KvCache(ctx), ow.KvCache(10 ** 9), ow.KvCache(ctx)]  # stream 1 appends
    inv = oracle.rope_inv_freq(64)
    g = torch.Generator().manual_seed(51)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    calls = [([0, 1, 2], [4, 3, 2])] + [([0, 1, 2], [1, 1, 1])] * 8 + [([2, 0], [1, 1])] * 9 + \
            [([0, 2], [8, 3])] + [([0, 2], [1, 1])] * 4
    worst = 0.0
    for streams, rows in calls:
        n = sum(rows)
        q = torch.randn(n, 8, 64, generator=g).to(tdt)
        k = torch.randn(n, kv_heads, 64, generator=g).to(tdt)
        v = torch.randn(n, kv_heads, 64, generator=g).to(tdt)
        out = ptts.attend(kv, 0, q.to(cuda), k.to(cuda), v.to(cuda), streams, rows).cpu().numpy()
        kv.advance(streams, rows)
        at = 0
        for s, r in zip(streams, rows):
            want = ow.attend(caches[s], q[at:at + r].float().numpy(), k[at:at + r].float().numpy(),
                             v[at:at + r].float().numpy(), inv, bf16=dtype == "bf16")
            worst = max(worst, normwise(out[at:at + r], want))
            at += r
    kv.check()
    assert list(kv.lengths()) == [c.offset for c in caches]
    print(dtype, kv_heads, "worst normwise", worst)
    assert worst < tol


def test_windowed_streams_refuse_what_they_cannot_do(ptts, cuda):
    import torch
    kv = ptts.KvState(1, 2, 8, dtype="bf16")
    with pytest.raises(ptts.PttsError, match="context must be in 1..8"):
        kv.set_window([0], 9)
    kv.set_window([0], 5)
    row = lambda n, h=8: torch.randn(n, h, 64).bfloat16().to(cuda)
    # At most capacity - context + 1 = 4 rows per call.
    with pytest.raises(ptts.CapacityError, match="at most 4 rows per call"):
        ptts.attend(kv, 0, row(5), row(5), row(5), [0], [5])
    ptts.attend(kv, 0, row(4), row(4), row(4), [0], [4])
    kv.advance([0], [4])
    with pytest.raises(ptts.PttsError, match="not empty"):
        kv.set_window([0], 3)
    with pytest.raises(ptts.PttsError, match="windowed"):
        kv.start_ring([0])
    with pytest.raises(ptts.PttsError, match="keeps its position"):
        kv.set_lengths([0], [2])
    cfg = ptts.FlowLMConfig(num_layers=1)
    model = ptts.Transformer(cfg)
    model.load(ptts.random_weights(cfg, 1))
    # The device step is the flow LM's (transformer.rs:603-605): windowed streams go through
    # ptts_b200_forward (tests/test_mimi.py) or the attention op.
    with pytest.raises(ptts.PttsError, match="not the device step"):
        model.step(kv, [0], torch.randn(1, 512).bfloat16().to(cuda))
    # Positions keep growing past the capacity through decode calls.
    for _ in range(10):
        ptts.attend(kv, 0, row(1), row(1), row(1), [0], [1])
        kv.advance([0], [1])
    assert kv.lengths()[0] == 14
    kv.check()
    kv.reset([0])
    ptts.attend(kv, 0, row(6), row(6), row(6), [0], [6])  # appended again: 6 rows fit in 8 slots
