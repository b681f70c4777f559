"""The decode attention that allocates nothing (ptts_b200_attend_decode_noalloc).

Some hosts of this library cannot allocate device memory while they run: a real-time audio
engine plans every allocation before its frame loop, a server may own all device memory through
its own pool, and a foreign runtime may hand over only raw pointers. For them the split-KV
decode takes its working memory from a fixed array inside the library. This test drives that
entry point through the C ABI, twice in a row on the same cache, and checks each call's output
and cache writes against the ordinary entry point (ptts_b200_attend) on an identical copy of the
cache, within the tolerance the other tests use. It also checks that the second call leaves the
device's free memory unchanged and that an oversized batch is refused.

This file is named to be collected last, so a run that stops at the first failure has already
run every other test.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import normwise

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _f32(t):
    return t.float().cpu().numpy()


def test_noalloc_decode_matches_the_allocating_entry_point(ptts, cuda):
    import torch
    g = torch.Generator(device=cuda).manual_seed(21)
    S, cap = 37, 700
    lengths = torch.randint(0, 600, (S,), generator=torch.Generator().manual_seed(21)).numpy().astype(np.int32)
    ref = ptts.KvState(1, S, cap, dtype="bf16")
    rk, rv, _ = ref.tensors(0)
    rk.normal_(generator=g)
    rv.normal_(generator=g)
    ref.set_lengths(np.arange(S, dtype=np.int32), lengths)
    # The caller-owned copy: plain torch buffers, as a host with its own memory would hold them.
    kc, vc = rk.clone(), rv.clone()
    dev_lengths = torch.from_numpy(lengths).to(cuda)
    streams = np.array([5, 0, 36, 17, 2, 9, 30, 11], np.int32)
    dev_streams = torch.from_numpy(streams).to(cuda)
    n = len(streams)
    out = torch.empty(n, 512, dtype=torch.float32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    torch.cuda.synchronize()
    for call in range(2):
        q, k, v = (torch.randn(n, 8, 64, generator=g, device=cuda).bfloat16() for _ in range(3))
        want = ptts.attend(ref, 0, q, k, v, streams, np.ones(n, np.int32), out_dtype="f32")
        ptts.attend_decode_noalloc(kc, vc, dev_lengths, dev_streams, q, k, v, out=out, err=err)
        torch.cuda.synchronize()
        if call == 1:
            free_before = torch.cuda.mem_get_info()[0]
            ptts.attend_decode_noalloc(kc, vc, dev_lengths, dev_streams, q, k, v, out=out, err=err)
            torch.cuda.synchronize()
            assert torch.cuda.mem_get_info()[0] == free_before, "the no-alloc call allocated"
        assert int(err.item()) == 0
        assert normwise(_f32(out), _f32(want)) < TOL, call
        np.testing.assert_array_equal(_f32(kc), _f32(ref.tensors(0)[0]))
        np.testing.assert_array_equal(_f32(vc), _f32(ref.tensors(0)[1]))
        ref.advance(streams, np.ones(n, np.int32))
        dev_lengths[dev_streams.long()] += 1
    ref.check()


def test_noalloc_refuses_an_oversized_batch(ptts, cuda):
    import torch
    kc = torch.zeros(2, 4, 8, 64, dtype=torch.bfloat16, device=cuda)
    lengths = torch.zeros(2, dtype=torch.int32, device=cuda)
    streams = torch.zeros(1025, dtype=torch.int32, device=cuda)
    q = torch.zeros(1025, 8, 64, dtype=torch.bfloat16, device=cuda)
    out = torch.empty(1025, 512, dtype=torch.float32, device=cuda)
    with pytest.raises(ptts.PttsError) as e:
        ptts.attend_decode_noalloc(kc, kc, lengths, streams, q, q, q, out=out)
    assert "1024" in e.value.msg
