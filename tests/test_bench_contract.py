"""bench.py's reference arm on CPU: one JSON line with the keys the benchmark contract names, and
no work (and no output) on ranks other than 0. The arm times the C oracle port of the
reference's CPU path over a small sample of the config-5 shard."""
from __future__ import annotations

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench(*args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, env=e,
                          capture_output=True, text=True, timeout=300)


def test_reference_arm_prints_one_contract_line():
    r = _bench("--impl", "reference", "--steps", "1", "--warmup", "3")
    assert r.returncode == 0, r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["steps"] == 1 and d["warmup"] == 3 and d["higher_is_better"] is True
    assert d["value"] > 0 and d["unit"] == "frames/s"
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_is_rank_zero_only():
    r = _bench("--impl", "reference", "--steps", "1", "--warmup", "3", env={"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == ""


def test_fewer_than_three_warmup_steps_are_refused():
    r = _bench("--impl", "reference", "--steps", "1", "--warmup", "2")
    assert r.returncode != 0
    assert "warmup" in r.stderr


def test_q8_0_layers_are_the_published_block_layout(ptts):
    """bench.py --weights q8_0 packs the int8 weights as GGUF q8_0 blocks: per 32 weights an
    f16 scale, then the 32 int8 (W = q * d), each row's scale in every block of the row. Checked
    against the test fixture's own writer of that layout, and by decoding the blocks back."""
    import numpy as np
    sys.path.insert(0, ROOT)
    import bench
    from gguf_fixture import q8_0_blocks
    cfg = ptts.FlowLMConfig(num_layers=2)
    w = ptts.random_weights(cfg, 5)
    layers = bench.q8_0_layers(w, cfg)
    assert len(layers) == 2
    for l, layer in enumerate(layers):
        for name in ("in_proj", "out_proj", "linear1", "linear2"):
            q, s = w.layer(l)[name], w.layer(l)[name + "_scale"]
            n, k = q.shape
            d = np.repeat(s.astype(np.float16)[:, None], k // 32, axis=1)
            np.testing.assert_array_equal(layer[name], q8_0_blocks(q, d))
            blocks = layer[name].reshape(n, k // 32, 34)
            back = blocks[:, :, 2:].view(np.int8).astype(np.float32) * blocks[:, :, :2].copy().view(np.float16).astype(np.float32)
            np.testing.assert_array_equal(back.reshape(n, k), q.astype(np.float32) * s.astype(np.float16).astype(np.float32)[:, None])
        for name in ("norm1_weight", "norm1_bias", "norm2_weight", "norm2_bias"):
            np.testing.assert_array_equal(layer[name], w.layer(l)[name])
