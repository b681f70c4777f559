"""The decode attention that allocates nothing (ptts_b200_attend_decode_noalloc).

Some hosts of this library cannot allocate device memory while they run: a real-time audio
engine plans every allocation before its frame loop, a server may own all device memory through
its own pool, and a foreign runtime may hand over only raw pointers. For them the split-KV
decode takes its working memory from a fixed array inside the library. These tests drive that
entry point through the C ABI, two calls in a row on the same cache, and check each call's output
and cache writes against the ordinary entry point (ptts_b200_attend) on an identical copy of the
cache. Both run the same plan and the same kernels on the same number of CTAs, so the outputs
must agree bit for bit. Covered: grouped key/value heads, bf16 and f32 caches and outputs, a
full 1024-row call whose last stream is cut across the last CTAs (the partial records' highest
slot), the refusal of an oversized batch, and rows the kernels refuse (a stream index out of
range, a repeated stream, a position at the capacity): those write nothing, read nothing, come
back as zero rows and set their bits in the error word, while the other rows are unaffected.

This file is named to be collected last, so a run that stops at the first failure has already
run every other test.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _pair(ptts, cuda, S, cap, kv_dtype, lengths, seed):
    """The library's KvState and a caller-owned copy (plain torch buffers) of the same cache."""
    import torch
    g = torch.Generator(device=cuda).manual_seed(seed)
    ref = ptts.KvState(1, S, cap, dtype=kv_dtype)
    rk, rv, _ = ref.tensors(0)
    rk.normal_(generator=g)
    rv.normal_(generator=g)
    ref.set_lengths(np.arange(S, dtype=np.int32), lengths)
    return ref, rk.clone(), rv.clone(), g


@pytest.mark.parametrize("kv_heads,kv_dtype,out_dtype", [(8, "bf16", "f32"), (2, "bf16", "bf16"),
                                                          (1, "bf16", "f32"), (8, "f32", "f32"),
                                                          (4, "f32", "bf16")])
def test_noalloc_decode_matches_the_allocating_entry_point(ptts, cuda, kv_heads, kv_dtype, out_dtype):
    import torch
    S, cap = 37, 700
    lengths = torch.randint(0, 600, (S,), generator=torch.Generator().manual_seed(21)).numpy().astype(np.int32)
    ref, kc, vc, g = _pair(ptts, cuda, S, cap, kv_dtype, lengths, 21)
    dev_lengths = torch.from_numpy(lengths).to(cuda)
    streams = np.array([5, 0, 36, 17, 2, 9, 30, 11], np.int32)
    dev_streams = torch.from_numpy(streams).to(cuda)
    n = len(streams)
    odt = torch.bfloat16 if out_dtype == "bf16" else torch.float32
    out = torch.empty(n, 512, dtype=odt, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    torch.cuda.synchronize()
    for call in range(2):
        q = torch.randn(n, 8, 64, generator=g, device=cuda).bfloat16()
        k, v = (torch.randn(n, kv_heads, 64, generator=g, device=cuda).bfloat16() for _ in range(2))
        want = ptts.attend(ref, 0, q, k, v, streams, np.ones(n, np.int32), out_dtype=out_dtype)
        ptts.attend_decode_noalloc(kc, vc, dev_lengths, dev_streams, q, k, v, out=out, err=err)
        torch.cuda.synchronize()
        if call == 1:
            free_before = torch.cuda.mem_get_info()[0]
            ptts.attend_decode_noalloc(kc, vc, dev_lengths, dev_streams, q, k, v, out=out, err=err)
            torch.cuda.synchronize()
            assert torch.cuda.mem_get_info()[0] == free_before, "the no-alloc call allocated"
        assert int(err.item()) == 0
        assert torch.equal(out, want), (call, (out.float() - want.float()).abs().max().item())
        assert torch.equal(kc, ref.tensors(0)[0]) and torch.equal(vc, ref.tensors(0)[1])
        ref.advance(streams, np.ones(n, np.int32))
        dev_lengths[dev_streams.long()] += 1
    ref.check()


def test_noalloc_full_batch_with_cut_streams_at_the_last_ctas(ptts, cuda):
    """1024 rows (the limit): short streams, then a last stream long enough to span the last
    CTAs of the split, so its partial records land at the highest slot (row 1023 + last CTA)."""
    import torch
    S, cap = 1024, 4200
    rng = np.random.default_rng(5)
    lengths = rng.integers(0, 300, size=S).astype(np.int32)
    lengths[-1] = 4100
    lengths[700] = 2500  # another cut stream mid-batch
    ref, kc, vc, g = _pair(ptts, cuda, S, cap, "bf16", lengths, 5)
    dev_lengths = torch.from_numpy(lengths).to(cuda)
    streams = rng.permutation(S - 1).astype(np.int32)
    streams = np.concatenate([streams, [S - 1]]).astype(np.int32)  # the long stream is the last row
    dev_streams = torch.from_numpy(streams).to(cuda)
    n = S
    out = torch.empty(n, 512, dtype=torch.float32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    for call in range(2):
        q, k, v = (torch.randn(n, 8, 64, generator=g, device=cuda).bfloat16() for _ in range(3))
        want = ptts.attend(ref, 0, q, k, v, streams, np.ones(n, np.int32), out_dtype="f32")
        ptts.attend_decode_noalloc(kc, vc, dev_lengths, dev_streams, q, k, v, out=out, err=err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert torch.equal(out, want), (call, (out - want).abs().max().item())
        assert torch.equal(kc, ref.tensors(0)[0]) and torch.equal(vc, ref.tensors(0)[1])
        ref.advance(streams, np.ones(n, np.int32))
        dev_lengths[dev_streams.long()] += 1
    ref.check()


def test_noalloc_refused_rows_write_nothing_and_come_back_zero(ptts, cuda):
    """Rows naming a stream out of range (-1 and S), repeating an earlier row's stream, or
    sitting at the capacity are refused: zero output rows, their error bits set, no cache row
    written; the valid rows equal the allocating entry point's output over those rows alone."""
    import torch
    S, cap = 24, 300
    lengths = np.random.default_rng(9).integers(1, 250, size=S).astype(np.int32)
    lengths[7] = cap  # full: its next row does not fit
    ref, kc, vc, g = _pair(ptts, cuda, S, cap, "bf16", lengths, 9)
    dev_lengths = torch.from_numpy(lengths).to(cuda)
    # Stream 0 has no valid row: an out-of-range index must not land there.
    #                  ok  bad  ok  dup-of-3 full  ok  bad ok
    streams = np.array([3, -1, 12, 3, 7, 5, S, 19], np.int32)
    refused = np.array([0, 1, 0, 1, 1, 0, 1, 0], bool)
    n = len(streams)
    dev_streams = torch.from_numpy(streams).to(cuda)
    out = torch.full((n, 512), 7.0, dtype=torch.float32, device=cuda)
    for call in range(2):
        err = torch.zeros(1, dtype=torch.int32, device=cuda)
        q, k, v = (torch.randn(n, 8, 64, generator=g, device=cuda).bfloat16() for _ in range(3))
        ok = np.flatnonzero(~refused)
        want = ptts.attend(ref, 0, q[ok], k[ok], v[ok], streams[ok], np.ones(len(ok), np.int32), out_dtype="f32")
        ptts.attend_decode_noalloc(kc, vc, dev_lengths, dev_streams, q, k, v, out=out, err=err)
        torch.cuda.synchronize()
        bits = int(err.item())
        assert bits & ptts.DEVERR_BOUNDS and bits & ptts.DEVERR_DUPLICATE and bits & ptts.DEVERR_CAPACITY, bits
        assert torch.equal(out[torch.from_numpy(ok).to(cuda)], want)
        assert (out[torch.from_numpy(np.flatnonzero(refused)).to(cuda)] == 0).all()
        # Only the valid rows' slots changed: the caller's cache equals the reference's, which
        # saw the valid rows alone.
        assert torch.equal(kc, ref.tensors(0)[0]) and torch.equal(vc, ref.tensors(0)[1])
        ref.advance(streams[ok], np.ones(len(ok), np.int32))
        dev_lengths[torch.from_numpy(streams[ok]).long().to(cuda)] += 1
        out.fill_(7.0)
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
