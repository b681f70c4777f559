"""Seeded synthetic inputs for the five configurations of the flow-LM attention path.

The reference measures only with its own bench on real checkpoints, which are not present; every
configuration here is random data in the named shapes (torch.Generator for reproducibility):

1. single-stream f32 decode, 512 steps, q/k/v ~ N(0, 1) per step in the order q, k, v (seed 0)
2. bf16 prefill, one stream of 256 rows, q/k/v ~ N(0, 1) / sqrt(64) (seed 1)
3. ragged bf16 decode, 256 streams, prefilled lengths ~ U{64..2048}, cached rows ~ N(0, 1)
   (treated as already rotated), 100 steps of q/k/v ~ N(0, 1) (seed 2)
4. 31m decode step (6 layers), 64 streams, prefix 128, 250 frames, int8 weights (seed 3)
5. 40m (9 layers), 4096 streams sharded 512 per GPU, prefixes ~ U{32..512}, 250 frames (seed 4)
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


def _gen(seed: int):
    import torch
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def config1_steps(steps: int = 512, seed: int = 0):
    """[(q, k, v)] per step, each float32 [1, 8, 64]."""
    import torch
    g = _gen(seed)
    out = []
    for _ in range(steps):
        q = torch.randn(1, 8, 64, generator=g)
        k = torch.randn(1, 8, 64, generator=g)
        v = torch.randn(1, 8, 64, generator=g)
        out.append((q, k, v))
    return out


def config2(seed: int = 1, rows: int = 256):
    """q, k, v bf16 [rows, 8, 64] ~ N(0, 1) / sqrt(64)."""
    import torch
    g = _gen(seed)
    q, k, v = (torch.randn(rows, 8, 64, generator=g) / 8.0 for _ in range(3))
    return q.bfloat16(), k.bfloat16(), v.bfloat16()


@dataclass
class RaggedDecode:
    lengths: np.ndarray          # [B] prefilled lengths
    prefix_k: list               # per stream bf16 [L, 8, 64] (CPU torch)
    prefix_v: list
    seed: int

    def steps(self, n: int):
        """Yields (q, k, v) bf16 [B, 8, 64] for n steps (deterministic per seed)."""
        import torch
        g = _gen(self.seed + 1000)
        B = len(self.lengths)
        for _ in range(n):
            yield tuple(torch.randn(B, 8, 64, generator=g).bfloat16() for _ in range(3))


def config3(B: int = 256, seed: int = 2, lo: int = 64, hi: int = 2048) -> RaggedDecode:
    import torch
    g = _gen(seed)
    lengths = torch.randint(lo, hi + 1, (B,), generator=g).numpy().astype(np.int32)
    pk, pv = [], []
    for L in lengths:
        pk.append(torch.randn(int(L), 8, 64, generator=g).bfloat16())
        pv.append(torch.randn(int(L), 8, 64, generator=g).bfloat16())
    return RaggedDecode(lengths, pk, pv, seed)


def prefix_lengths(n: int, lo: int, hi: int, seed: int) -> np.ndarray:
    import torch
    return torch.randint(lo, hi + 1, (n,), generator=_gen(seed)).numpy().astype(np.int32)


def hidden_rows(n: int, d: int, seed: int):
    """bf16 [n, d] ~ N(0, 1): stand-in for the flow LM's per-frame input rows."""
    import torch
    return torch.randn(n, d, generator=_gen(seed)).bfloat16()
