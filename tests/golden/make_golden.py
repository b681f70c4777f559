"""Generate the golden fixtures under tests/golden/ (run from the repo root).

The reference holds no numeric golden vectors for the attention path (its CUDA/CPU arithmetic
lives in the un-vendored `xn` crate). What it does hold, and what these fixtures restate:

- lcg_gqa.npz — the inputs of `grouped_query_attention_is_attention_with_repeated_kv_heads`
  (ptts/src/transformer.rs:1112-1164): a 64-bit LCG (multiplier 6364136223846793005, increment
  1442695040888963407, value (state >> 40) / 2^24 - 0.5) seeded 1, drawn in the test's order
  q_w, k_w, v_w, o_w, x for embed 6, h 4, kvh 2, d 2.
- lcg_device_step.npz — the inputs of `a_device_step_is_the_host_step` (transformer.rs:1169-1225),
  the same LCG seeded 7: in_w, out_w, x.
- with_seq_budget.json — the known answers of `with_seq_budget_tests` (transformer.rs:1022-1100):
  a cache whose k[b, s, h, d] = s + 100 h (v = -k), copied into a larger budget: the first
  `used` slots equal the pattern, the rest are zero, a smaller budget is refused with a message
  naming both numbers, an equal budget is accepted.
- rope_f64.npz — the inverse frequencies of rope.rs:44-48 (1 / theta^(i/32), head_dim 64,
  theta 10000) with the power taken in float64 and rounded once to f32 (libm powf may differ by
  one ulp), and the positions at which the tests check the tables (0..63 and a stride-61 sample
  up to 4095).

Each expected output here comes from the reference's own test code or from the rope.rs formula,
not from this repository's oracle.
"""
from __future__ import annotations

import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
MASK = (1 << 64) - 1


class Lcg:
    def __init__(self, seed: int):
        self.state = seed

    def take(self, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        for i in range(n):
            self.state = (self.state * 6364136223846793005 + 1442695040888963407) & MASK
            out[i] = np.float32(self.state >> 40) / np.float32(1 << 24) - np.float32(0.5)
        return out


def lcg_gqa():
    embed, h, kvh, d = 6, 4, 2, 2
    attn = h * d
    r = Lcg(1)
    q_w, k_w, v_w = r.take(attn * embed), r.take(kvh * d * embed), r.take(kvh * d * embed)
    o_w, x = r.take(embed * attn), r.take(5 * embed)
    return dict(q_w=q_w, k_w=k_w, v_w=v_w, o_w=o_w, x=x, dims=np.array([embed, h, kvh, d]))


def lcg_device_step():
    embed, h, kvh, d, kv = 6, 4, 2, 2, 8
    r = Lcg(7)
    in_w = r.take((h + 2 * kvh) * d * embed)
    out_w = r.take(embed * h * d)
    x = r.take(5 * embed)
    return dict(in_w=in_w, out_w=out_w, x=x, dims=np.array([embed, h, kvh, d, kv]))


def with_seq_budget():
    b, h, d = 1, 2, 3
    cases = []
    for seq, used, budget in [(4, 3, 10), (4, 2, 8), (4, 3, 2), (4, 3, 3)]:
        k = np.zeros((b, seq, h, d), np.float32)
        for s in range(seq):
            for hh in range(h):
                k[0, s, hh, :] = s + 100 * hh
        case = dict(seq=seq, used=used, budget=budget, k=k.ravel().tolist(),
                    v=(-k).ravel().tolist(), refused=used > budget)
        if used <= budget:
            want_k = np.zeros((b, budget, h, d), np.float32)
            want_k[:, :used] = k[:, :used]
            case["want_k"] = want_k.ravel().tolist()
            case["want_v"] = (-want_k).ravel().tolist()
        cases.append(case)
    return dict(b=b, h=h, d=d, cases=cases)


def rope_f64():
    head_dim, theta = 64, np.float32(10000.0)
    half = head_dim // 2
    inv = np.array([np.float32(1.0) / np.float32(np.float64(theta) ** (np.float64(np.float32(i) / np.float32(half))))
                    for i in range(half)], np.float32)
    pos = np.array(sorted(set(range(64)) | set(range(0, 4096, 61)) | {2047, 2048, 4095}), np.float32)
    return dict(inv_freq=inv, positions=pos)


def main():
    np.savez_compressed(os.path.join(HERE, "lcg_gqa.npz"), **lcg_gqa())
    np.savez_compressed(os.path.join(HERE, "lcg_device_step.npz"), **lcg_device_step())
    with open(os.path.join(HERE, "with_seq_budget.json"), "w") as f:
        json.dump(with_seq_budget(), f)
    np.savez_compressed(os.path.join(HERE, "rope_f64.npz"), **rope_f64())


if __name__ == "__main__":
    main()
