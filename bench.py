"""Benchmark: flow-LM decode frames/s (config 5 shard) with decode-attention GB/s vs HBM peak.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--repeats R] [--impl ours|reference]

Workload (config 5, the largest single-GPU configuration): the 40m flow LM shape
(9 layers, d_model 512, 8 heads of 64, ff 2048), random-init int8 per-output-channel weights
(scales U(0.005, 0.02), seed 4), 512 independent streams per GPU (GPU g holds streams
512g..512g+511 of 4096), prefixes U{32..512} prefilled before timing, then decode frames: one
row per stream per frame through all layers (QKV + RoPE + KV append + split-KV attention +
out_proj + FFN) replayed as one CUDA graph. A step = one frame for all streams of a GPU.

Timed window. Config 5 runs 250 frames, and a frame's KV read grows with its index (2.7 GB at
frame 5, 3.8 GB on average, 4.8 GB at frame 249 per GPU). K < 250 timed frames sit in the middle
of the window (frames (250 - K) / 2 ..), with the W warm-up frames just before them, so they see
the window's average KV; the K-frame region is timed R times from that same start (lengths set
back between repeats, outside the timed region) and ms_per_step is the median, with min and
max beside it. K >= 250 frames cycle the whole window from frame 0 (lengths return to the
prefixes every 250 frames), timed once.

value  = stream-frames per second over all GPUs, inputs resident in HBM.
e2e    = the same through ptts_b200_step with pinned HOST input/output (H2D + D2H per step).
roofline = the decode-attention kernel: algorithmic bytes (K and V rows read for every
           attended position, q read, output written) / its CUDA-event duration in a traced
           pass over the same frames, against MEASURED_PEAKS.json's HBM copy bandwidth.
decode_attn = config 3 (256 ragged streams, lengths U{64..2048}, bf16 KV, 100-step window) run
           through the attention op in the same process: the op's algorithmic GB/s and the
           decode kernel's own fraction of the HBM peak.
cpu_baseline = the C oracle (a port of the reference's CPU path) on the host cores, on a
           sample of 16 streams of the same workload.
Multi-GPU: one process per GPU (torchrun), independent shards, no data-path collective and no
NCCL: the start/stop barriers and the max over ranks of the timed duration go through a gloo
process group on host tensors.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

STREAMS_PER_GPU = 512
TOTAL_STREAMS = 4096
FRAMES = 250
SEED = 4
PREFIX_LO, PREFIX_HI = 32, 512
METRIC = "decode attn GB/s (% HBM peak) & flow-LM frames/sec at 1/2/4/8 B200"
CPU_SAMPLE_STREAMS = 16


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def traffic_per_launch():
    """DRAM bytes / algorithmic bytes of the decode-attention kernel from a committed ncu
    summary of a smaller case; traffic grows in proportion to the KV rows read."""
    path = os.path.join(ROOT, "profiles", "decode_attn_traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def shard_streams(rank: int, world: int):
    """Stream ids of a rank: contiguous blocks of STREAMS_PER_GPU (GPU g gets 512g..512g+511)."""
    if world * STREAMS_PER_GPU > TOTAL_STREAMS:
        raise ValueError(f"{world} ranks x {STREAMS_PER_GPU} streams exceed {TOTAL_STREAMS}")
    return list(range(rank * STREAMS_PER_GPU, (rank + 1) * STREAMS_PER_GPU))


def barrier(dist):
    """Start/stop barrier of the timed region (no-op on one process; gloo, host side)."""
    if dist is None:
        return
    dist.barrier()


def max_over_ranks(dist, ms: float) -> float:
    """The slowest rank's duration: the job's time (a host tensor through gloo)."""
    if dist is None:
        return ms
    import torch
    t = torch.tensor([ms], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_over_ranks(dist, v: float) -> list:
    """Every rank's value, in rank order (one element on one process)."""
    if dist is None:
        return [v]
    import torch
    t = torch.tensor([v], dtype=torch.float64)
    out = [torch.zeros_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    return [float(x.item()) for x in out]


def timing_window(steps: int, warmup: int):
    """(first warm-up frame, first timed frame) in the 250-frame window. K < 250 timed frames
    are centred in the window, the warm-up frames just before them; K >= 250 cycle the window
    from frame 0 (warm-up frames first)."""
    if steps >= FRAMES:
        return 0, warmup % FRAMES
    first = (FRAMES - steps) // 2
    return max(first - warmup, 0), first


def spread(values) -> dict:
    vs = sorted(values)
    return {"min": vs[0], "median": statistics.median(vs), "max": vs[-1]}


def load():
    import __graft_entry__ as ge
    return ge.load_package(), ge.load_workloads()


def shard_prefixes(wl, rank: int):
    """Prefix lengths of a rank's streams, cut from the job-wide U{32..512} draw (seed 4)."""
    allp = wl.prefix_lengths(TOTAL_STREAMS, PREFIX_LO, PREFIX_HI, SEED)
    ids = shard_streams(rank, 1 + rank)
    return allp[ids[0]:ids[-1] + 1]


def cpu_baseline(ptts, wl, cfg, weights, steps: int | None = None, warmup: int = 0, start: int = 0,
                 budget_s: float = 12.0):
    """The oracle on the host cores: a sample of CPU_SAMPLE_STREAMS streams of rank 0's shard,
    prefilled (untimed), then decode frames from frame `start` of the window (lengths set to
    prefix + start; the cache rows of the frames skipped stay zero, which changes no arithmetic
    count), `warmup` untimed frames, then frames timed until `steps` frames or `budget_s`
    seconds. Frames past the window's end cycle it (lengths return to the prefixes)."""
    import numpy as np
    import torch
    import oracle

    n = CPU_SAMPLE_STREAMS
    prefixes = shard_prefixes(wl, 0)[:n].astype(np.int32)
    cap = int(prefixes.max()) + FRAMES
    om = oracle.Model(cfg, weights)
    shape = (cfg.num_layers, n, cap, cfg.num_heads, cfg.head_dim)
    kc = np.zeros(shape, np.float32)
    vc = np.zeros(shape, np.float32)
    g = torch.Generator().manual_seed(SEED * 7919)
    offs = np.concatenate([[0], np.cumsum(prefixes)]).astype(np.int32)
    x = torch.randn(int(offs[-1]), cfg.d_model, generator=g).bfloat16().float().numpy()
    lengths = np.zeros(n, np.int32)
    streams = np.arange(n, dtype=np.int32)
    threads = oracle.threads()
    om.forward(x, kc, vc, lengths, streams, offs, store=oracle.ROUND_KV, n_threads=threads)
    one = np.arange(n + 1, dtype=np.int32)
    frames = [torch.randn(n, cfg.d_model, generator=g).bfloat16().float().numpy() for _ in range(8)]
    state = {"f": start % FRAMES}

    def frame():
        f = state["f"]
        lengths = prefixes + f
        om.forward(frames[f % len(frames)], kc, vc, lengths, streams, one, store=oracle.ROUND_KV,
                   n_threads=threads)
        state["f"] = (f + 1) % FRAMES

    for _ in range(warmup):
        frame()
    done, t0 = 0, time.perf_counter()
    while True:
        frame()
        done += 1
        el = time.perf_counter() - t0
        if (steps is not None and done >= steps) or (steps is None and el >= budget_s) or done >= 4 * FRAMES:
            break
    el = time.perf_counter() - t0
    return {"value": n * done / el, "unit": "frames/s", "cores": threads, "kind": "port",
            "sample": f"{n} streams of the config-5 shard (prefixes U{{32..512}}), {done} decode frames "
                      f"of the 40m stack from frame {start % FRAMES} of the 250-frame window, after an "
                      f"untimed prefill and {warmup} untimed frames; C oracle with OpenMP",
            "seconds": el, "frames": done}


def run_reference(args):
    """--impl reference: the reference's CPU path (the C oracle port) on the host cores, over
    the same timed frames of the window as the GPU arm (see timing_window)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    ptts, wl = load()
    cfg = ptts.PHONON_40M
    weights = ptts.random_weights(cfg, SEED)
    import oracle
    oracle.lib()
    w0, t0 = timing_window(args.steps, args.warmup)
    cb = cpu_baseline(ptts, wl, cfg, weights, steps=args.steps, warmup=t0 - w0 if args.steps < FRAMES else args.warmup,
                      start=w0)
    per_frame = cb["seconds"] / cb["frames"]
    value = CPU_SAMPLE_STREAMS / per_frame
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "frames/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": per_frame * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (bf16-rounded storage)", "data": "synthetic",
        "config": {"workload": "config5 shard: 40m flow LM, prefixes U{32..512}, decode frames",
                   "streams_sampled": CPU_SAMPLE_STREAMS, "timed_frames": [t0, t0 + args.steps],
                   "extrapolated": f"stream-frames/s of {CPU_SAMPLE_STREAMS} sampled streams of the "
                                   f"{STREAMS_PER_GPU}-stream shard: streams never interact, so the "
                                   "per-stream rate is the shard's; ms_per_step is the time of one "
                                   f"frame of the {CPU_SAMPLE_STREAMS} sampled streams"},
        "cpu_baseline": {"value": value, "unit": "frames/s", "cores": cb["cores"], "kind": "port",
                         "sample": cb["sample"]},
        "e2e": {"value": value, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_spec(args, ptts, wl, rank):
    """(cfg, streams per GPU, prefix lengths of this rank, seed, description) of the workload."""
    import numpy as np
    if args.workload == "config4":
        cfg = ptts.PHONON_31M
        B = 64
        prefixes = np.full(B, 128, np.int32)
        seed = 3
        desc = ("config4: 31m flow LM (6 layers, d 512, 8x64 heads, ff 2048), 64 streams/GPU, "
                "prefix 128, 250-frame decode window")
    else:
        cfg = ptts.PHONON_40M
        B = STREAMS_PER_GPU
        prefixes = shard_prefixes(wl, rank)
        seed = SEED
        desc = ("config5 shard: 40m flow LM (9 layers, d 512, 8x64 heads, ff 2048), 512 streams/GPU, "
                "prefixes U{32..512}, 250-frame decode window")
    if args.layers:
        cfg = ptts.FlowLMConfig(num_layers=args.layers)
        desc += f" [profiling override: {args.layers} layers]"
    return cfg, B, prefixes, seed, desc


def q8_0_layers(weights, cfg) -> list:
    """The same int8 weights as GGUF q8_0 linears (blocks of 34 bytes per 32 weights: an f16
    scale d, then the 32 int8 q; W = q * d, the published ggml layout): every block of a row takes
    that row's scale, rounded to f16. Norms as they are."""
    import numpy as np
    out = []
    for l in range(cfg.num_layers):
        w = weights.layer(l)
        layer = {}
        for name in ("in_proj", "out_proj", "linear1", "linear2"):
            q = np.ascontiguousarray(w[name])
            n, k = q.shape
            d = np.repeat(w[name + "_scale"].astype(np.float16)[:, None], k // 32, axis=1)
            blocks = np.zeros((n, k // 32, 34), np.uint8)
            blocks[:, :, :2] = np.ascontiguousarray(d).view(np.uint8).reshape(n, k // 32, 2)
            blocks[:, :, 2:] = q.view(np.uint8).reshape(n, k // 32, 32)
            layer[name] = blocks.reshape(n, -1)
        for name in ("norm1_weight", "norm1_bias", "norm2_weight", "norm2_bias"):
            layer[name] = w[name]
        out.append(layer)
    return out


def run_ours(args):
    import numpy as np
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    dist = None
    if world > 1:
        # Host-side plumbing only (barriers, the max over ranks): the data path has no
        # collective, so no NCCL communicator is created.
        import datetime
        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))

    ptts, wl = load()
    cfg, B, prefixes, seed, desc = workload_spec(args, ptts, wl, rank)
    L = cfg.num_layers
    weights = ptts.random_weights(cfg, seed)
    model = ptts.Transformer(cfg, local)
    if args.weights == "q8_0":
        for l, layer in enumerate(q8_0_layers(weights, cfg)):
            model.load_layer_q8_0(l, layer)
    else:
        model.load(weights)
    cap = int(prefixes.max()) + FRAMES
    streams = np.arange(B, dtype=np.int32)
    stream = torch.cuda.current_stream()

    def fresh_state():
        # Prompts on a scratch state first load every kernel (the linears' 32- and 128-row
        # tiles) and build the RoPE table for this capacity, so the timed prefill includes no
        # first-use module loading.
        scratch = ptts.KvState(L, 4, max(cap, 1100), dtype="bf16", device=local)
        for n in (130, 1100):
            model.forward(scratch, torch.zeros(4 * n, cfg.d_model, device=dev).bfloat16(),
                          [0, 1, 2, 3], [n] * 4)
            scratch.reset([0, 1, 2, 3])
        torch.cuda.synchronize()
        scratch.close()
        kv = ptts.KvState(L, B, cap, dtype="bf16", device=local)
        g = torch.Generator(device=dev).manual_seed(seed * 1000 + rank)
        x = torch.randn(int(prefixes.sum()), cfg.d_model, generator=g, device=dev).bfloat16()
        # An untimed prefill of the same prompts sizes the forward workspace (its allocations
        # are not prefill work), then the streams are emptied and the timed prefill runs.
        model.forward(kv, x, streams, prefixes)
        kv.reset(streams)
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        model.forward(kv, x, streams, prefixes)
        t1.record()
        torch.cuda.synchronize()
        del x
        return kv, t0.elapsed_time(t1)

    kv, prefill_ms = fresh_state()
    g = torch.Generator(device=dev).manual_seed(seed * 2000 + rank)
    x_frames = torch.randn(FRAMES, B, cfg.d_model, generator=g, device=dev).bfloat16()
    y = torch.empty(B, cfg.d_model, dtype=torch.float32, device=dev)

    state = {"f": 0}

    def goto(f):
        """Window position f: every stream's length prefix + f (a host call, outside timing)."""
        kv.set_lengths(streams, prefixes + (f % FRAMES))
        state["f"] = f % FRAMES
        torch.cuda.synchronize()

    def step(x_src, out):
        f = state["f"]
        if f == FRAMES:
            kv.set_lengths(streams, prefixes)
            f = 0
        model.step(kv, streams, x_src(f), out=out)
        state["f"] = f + 1

    def timed(x_src, out, k: int, start: int):
        goto(start)
        barrier(dist)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(k):
            step(x_src, out)
        e1.record(stream)
        e1.synchronize()
        mine = e0.elapsed_time(e1)
        return max_over_ranks(dist, mine), mine

    w0, t0 = timing_window(args.steps, args.warmup)
    cycling = args.steps >= FRAMES

    def run_repeats(x_src, out, min_repeats):
        """Warm-up frames (before the timed start), then R timed regions of K frames, each from
        the same start. Returns per-repeat job times (max over ranks) and this rank's own."""
        goto(w0)
        for _ in range(args.warmup):
            step(x_src, out)
        torch.cuda.synchronize()
        if cycling:
            job, mine = timed_cycle(x_src, out)
            return [job], [mine]
        jobs, mine = [], []
        r = 0
        target = args.repeats if args.repeats > 0 else min_repeats
        while r < target:
            j, m = timed(x_src, out, args.steps, t0)
            jobs.append(j)
            mine.append(m)
            r += 1
            if args.repeats <= 0 and r == min_repeats:
                # Auto: at least min_repeats, and at least ~1 s of timed work in all, so the
                # 200 ms clock sampler sees the timed region (the same count on every rank).
                want = int(np.ceil(1000.0 / max(statistics.median(jobs), 1e-3)))
                target = max(min_repeats, min(want, 200))
        return jobs, mine

    def timed_cycle(x_src, out):
        # K >= 250: one region, frames cycling the whole window from the warm-up's end.
        barrier(dist)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step(x_src, out)
        e1.record(stream)
        e1.synchronize()
        m = e0.elapsed_time(e1)
        return max_over_ranks(dist, m), m

    # ---- device-resident inputs --------------------------------------------------------------
    dev_src = lambda f: x_frames[f]
    # The sampler's process starts before the warm-up, so its start-up does not stall the host
    # inside the timed region.
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.5)
    jobs, mine = run_repeats(dev_src, y, 15)
    clocks = sampler.stop()
    ms = statistics.median(jobs)
    value = world * B * args.steps / (ms / 1e3)
    lanes = ptts.step_lanes(B)
    launches_per_step = 1 + lanes * (2 + 7 * L)  # advance + per lane: plan, final reduce and per
    #                       layer LN1, in_proj, attention (merge fused), out_proj, LN2, linear1, linear2
    wraps = (t0 + args.steps - 1) // FRAMES if not cycling else (args.warmup + args.steps) // FRAMES
    gpu_launches = len(jobs) * (args.steps * launches_per_step + wraps)
    per_rank = gather_over_ranks(dist, statistics.median(mine) / args.steps)

    # ---- end to end through pinned host buffers ------------------------------------------------
    x_host = x_frames.cpu().pin_memory()
    y_host = torch.empty(B, cfg.d_model, dtype=torch.float32).pin_memory()
    host_src = lambda f: x_host[f]
    ejobs, _ = run_repeats(host_src, y_host, 15)
    ms_e2e = statistics.median(ejobs)
    e2e = {"value": world * B * args.steps / (ms_e2e / 1e3), "unit": "frames/s",
           "h2d_bytes_per_step": B * cfg.d_model * 2, "d2h_bytes_per_step": B * cfg.d_model * 4,
           "ms_per_step": ms_e2e / args.steps, "repeats": len(ejobs)}

    # ---- traced pass: decode-attention launch durations with CUDA events ------------------------
    # The same frames as the timed region (its first repeat).
    goto(w0)
    for _ in range(args.warmup):
        step(dev_src, y)
    if not cycling:
        goto(t0)
    torch.cuda.synchronize()
    ptts.set_tracing(True)
    ptts.trace(reset=True)
    for _ in range(min(args.steps, FRAMES)):
        step(dev_src, y)
    torch.cuda.synchronize()
    tr = ptts.trace(reset=True)
    ptts.set_tracing(False)
    peak, peak_kind = peaks()
    per_launch_bytes = tr["attn_bytes"] / max(tr["attn_launches"], 1)
    per_launch_ms = tr["attn_ms"] / max(tr["attn_launches"], 1)
    achieved = per_launch_bytes / (per_launch_ms / 1e3) / 1e9
    traffic = traffic_per_launch()
    ratio = traffic.get("dram_over_algorithmic") if traffic else None
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                if peak_kind == "measured" else "fallback 6.65 TB/s",
                "traffic": ratio * per_launch_bytes if ratio else None,
                "kernel": "decode_attn_kernel<bf16> (split-KV)",
                "algorithmic_bytes_per_launch": per_launch_bytes,
                "launch_ms": per_launch_ms, "launches_timed": tr["attn_launches"],
                "attn_share_of_traced_step": tr["attn_ms"] / max(tr["step_ms"], 1e-9)}
    if traffic:
        roofline["traffic_source"] = "scaled from profiles/decode_attn_traffic.json: " + traffic.get("source", "")
    kv_bytes_per_step = tr["attn_bytes"] / max(tr["steps"], 1)

    # ---- kernel timeline inside the graph (device stamps), for the attention as it runs there --
    # Events around a launch cut it off from its neighbours; the stamps do not. The last of a few
    # graph-replayed steps is read, at the middle of the timed frames: per attention launch, from
    # its first CTA past the wait on its predecessor to its last CTA done (and from its first
    # CTA's start, which also counts the copies issued before that wait).
    mid = (t0 + args.steps // 2) % FRAMES if not cycling else FRAMES // 2
    goto(max(mid - 2, 0))
    model.stamps(lanes * (2 + 8 * L))
    while state["f"] <= mid:
        step(dev_src, y)
    torch.cuda.synchronize()
    stamps = model.read_stamps()
    model.stamps(0)
    att = [e for e in stamps if e["kernel"] == "attention"]
    kv_rows = float(prefixes.sum()) + B * (mid + 1)  # attended keys of the stamped step
    bytes_stamped = L * (kv_rows * 2 * 1024 + B * 512 * 6)
    busy = sum(e["end_us"] - e["start_us"] for e in att)
    busy_entry = sum(e["end_us"] - e["entry_us"] for e in att)
    if att and busy > 0:
        roofline["in_frame"] = {
            "source": "device stamps (globaltimer) of the attention launches of one graph-replayed step "
                      f"(frame {mid} of the window)",
            "launches": len(att), "us_per_launch": busy / len(att),
            "bytes_per_launch": bytes_stamped / len(att),
            "achieved": bytes_stamped / (busy / 1e6) / 1e9,
            "frac": bytes_stamped / (busy / 1e6) / 1e9 / peak,
            "us_per_launch_from_first_cta": busy_entry / len(att),
            "frac_from_first_cta": bytes_stamped / (busy_entry / 1e6) / 1e9 / peak,
            "step_us": max(e["end_us"] for e in stamps)}
    if args.timeline:
        with open(args.timeline, "w") as f:
            f.write("lane layer kernel       entry_us  start_us    end_us last_entry_us\n")
            for e in stamps:
                f.write(f"{e['lane']:4d} {e['layer']:5d} {e['kernel']:10s} {e['entry_us']:9.2f} "
                        f"{e['start_us']:9.2f} {e['end_us']:9.2f} {e['last_entry_us']:9.2f}\n")

    # ---- whole frames: input_linear -> step -> out_norm -> EOS + flow net (ptts_b200_frame) ----
    # An extra line item (the headline value above is the backbone step the configs define):
    # each frame feeds its latent back as the next input, as FlowLM's sampler does.
    flow_frame = None
    if args.workload == "config5" and not args.no_flow:
        fcfg = ptts.PHONON_FLOW
        flow = ptts.Flow(fcfg, device=local)
        flow.load(ptts.random_flow_weights(fcfg, seed, bf16_exact=True))
        noise = torch.randn(FRAMES, B, fcfg.ldim, generator=g, device=dev)
        fstate = {"lat": None}

        def frame():
            f = state["f"]
            if f == FRAMES:
                kv.set_lengths(streams, prefixes)
                f = 0
            fstate["lat"], _ = flow.frame(model, kv, streams, fstate["lat"], noise[f])
            state["f"] = f + 1

        k = min(args.steps, FRAMES)
        goto(w0)
        for _ in range(args.warmup):
            frame()
        goto(t0 if not cycling else 0)
        barrier(dist)
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(k):
            frame()
        f1.record(stream)
        f1.synchronize()
        fms = max_over_ranks(dist, f0.elapsed_time(f1))
        flow_frame = {"value": world * B * k / (fms / 1e3), "unit": "frames/s", "frames": k,
                      "ms_per_frame": fms / k, "ms_head_per_frame": fms / k - ms / args.steps,
                      "head": "flow_dim 512, depth 6, ldim 32, LSD 1 step (phonon shape), bf16 weights, "
                              "latent fed back each frame"}
        flow.close()
    kv.check()
    del kv

    # ---- config 3 through the attention op: the north star's decode-attention figure ------------
    decode_attn = None
    if args.workload == "config5" and not args.no_config3 and rank == 0 and world == 1:
        decode_attn = config3_attention(ptts, 200, args.warmup, local)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload == "config5" and not args.layers:
        cb = cpu_baseline(ptts, wl, cfg, weights, warmup=t0 - w0 if not cycling else args.warmup, start=w0)
        cpu = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "frames/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random-init int8 weights and N(0,1) hidden rows)",
            "config": {"workload": desc,
                       "streams_per_gpu": B, "total_streams": world * B, "layers": L,
                       "kv_capacity": cap, "parallelism": f"stream-sharded x{world}, no collectives",
                       "lanes": lanes,
                       "weights": "int8, one f32 scale per output row" if args.weights == "int8" else
                                  "GGUF q8_0 blocks (an f16 scale per 32 weights), the same int8 values",
                       "timed_frames": "whole window, cycled from frame 0" if cycling else [t0, t0 + args.steps],
                       "repeats": len(jobs),
                       "l2": f"inputs larger than L2: {kv_bytes_per_step / 1e9:.2f} GB of KV read per step per GPU"
                             if kv_bytes_per_step > 126e6 else "KV per step fits in L2 (no flush)"},
            "ms_per_step_spread": {k: v / args.steps for k, v in spread(jobs).items()},
            "ms_per_step_per_rank": {**spread(per_rank), "ranks": per_rank},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": gpu_launches,
            "gpu_launches_per_step": launches_per_step,
            "clocks": clocks, "prefill_ms": prefill_ms, "frame_with_flow_head": flow_frame,
            "prefill_rows_per_s": world * float(prefixes.sum()) / (prefill_ms / 1e3),
            "decode_attn": decode_attn,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        barrier(dist)
        dist.destroy_process_group()


def config3_attention(ptts, steps: int, warmup: int, device: int) -> dict:
    """Config 3 (seed 2) through the attention op, for the bench line's `decode_attn` object:
    256 ragged streams (prefilled lengths U{64..2048}, bf16 cache), one query per stream per
    step (RoPE + append + split-KV attention, then kv_advance), `steps` steps cycling the 100-step
    window. Reports the op's algorithmic GB/s (CUDA events around all steps), the decode
    kernel's own GB/s and fraction of the HBM peak (CUDA events around each launch, a traced
    pass over the same steps) and the clocks sampled meanwhile."""
    import numpy as np
    import torch

    dev = torch.device(f"cuda:{device}")
    B, window = 256, 100
    lengths = torch.randint(64, 2049, (B,), generator=torch.Generator().manual_seed(2)).numpy().astype(np.int32)
    cap = int(lengths.max()) + window
    kv = ptts.KvState(1, B, cap, dtype="bf16", device=device)
    g = torch.Generator(device=dev).manual_seed(2)
    kt, vt, _ = kv.tensors(0)
    kt.normal_(generator=g)
    vt.normal_(generator=g)
    streams = np.arange(B, dtype=np.int32)
    ones = np.ones(B, np.int32)
    kv.set_lengths(streams, lengths)
    pool = [torch.randn(window, B, 8, 64, generator=g, device=dev).bfloat16() for _ in range(3)]
    out = torch.empty(B, 512, dtype=torch.bfloat16, device=dev)
    state = {"s": 0}

    def bytes_of_step(lens):
        return float(((lens.astype(np.int64) + 1) * 2048).sum() + B * (1024 + 2048 + 1024))

    def step(acc):
        s = state["s"]
        if s and s % window == 0:
            kv.set_lengths(streams, lengths)
        i = s % window
        acc.append(bytes_of_step(lengths + i))
        ptts.attend(kv, 0, pool[0][i], pool[1][i], pool[2][i], streams, ones, out=out)
        kv.advance(streams, ones)
        state["s"] = s + 1

    junk = []
    sampler = ClockSampler(device)
    sampler.start()
    time.sleep(0.5)
    for _ in range(warmup):
        step(junk)
    kv.set_lengths(streams, lengths)
    state["s"] = 0
    torch.cuda.synchronize()
    acc = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step(acc)
    e1.record()
    e1.synchronize()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    kv.set_lengths(streams, lengths)
    state["s"] = 0
    ptts.set_tracing(True)
    ptts.trace(reset=True)
    for _ in range(steps):
        step(junk)
    tr = ptts.trace(reset=True)
    ptts.set_tracing(False)
    kv.check()
    kv.close()
    peak, kind = peaks()
    per_bytes = tr["attn_bytes"] / max(tr["attn_launches"], 1)
    per_ms = tr["attn_ms"] / max(tr["attn_launches"], 1)
    achieved = per_bytes / (per_ms / 1e3) / 1e9
    return {"workload": "config3: 256 ragged streams, lengths U{64..2048} (seed 2), bf16 KV, one query "
                        "per stream per step, 100-step window",
            "steps": steps, "op_gbs": sum(acc) / (ms / 1e3) / 1e9, "op_ms_per_step": ms / steps,
            "kernel": "decode_attn_kernel<bf16> (split-KV, wide ring)", "achieved": achieved,
            "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "peak_kind": f"{kind} (MEASURED_PEAKS.json hbm_gbs)" if kind == "measured" else "fallback 6.65 TB/s",
            "launch_ms": per_ms, "algorithmic_bytes_per_launch": per_bytes,
            "launches_timed": tr["attn_launches"], "clocks": clocks}


def run_config3(args):
    """--workload config3: the attention op alone over config 3 (see config3_attention), K steps
    after W warm-up steps; value = the op's algorithmic GB/s."""
    import torch
    ptts, _ = load()
    torch.cuda.set_device(0)
    d = config3_attention(ptts, args.steps, args.warmup, 0)
    print(json.dumps({
        "metric": "decode attn GB/s (config 3: 256 ragged streams, L0 U{64..2048}, bf16 KV)",
        "value": d["op_gbs"], "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": d["op_ms_per_step"], "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config3", "streams": 256, "window": 100},
        "roofline": {"bound": "hbm", "achieved": d["achieved"], "peak": d["peak"], "unit": "GB/s",
                     "frac": d["frac"], "peak_kind": d["peak_kind"], "launch_ms": d["launch_ms"],
                     "algorithmic_bytes_per_launch": d["algorithmic_bytes_per_launch"],
                     "kernel": d["kernel"]},
        "clocks": d["clocks"]}), flush=True)


def run_config2(args):
    """Config 2 (seed 1): one bf16 prompt of 256 rows, q/k/v ~ N(0,1)/sqrt(64), causal over
    itself: RoPE + append + prefill attention on the tensor cores. Each step re-runs the prompt
    on a cache emptied by kv_set_lengths. value = latency per call; the roofline is the
    algorithmic causal flop count 4 * 8 * 64 * sum(1..256) = 67.4 MFLOP over the measured
    bf16 tensor peak (tiny contraction: reported, not a target)."""
    import numpy as np
    import torch

    ptts, wl = load()
    torch.cuda.set_device(0)
    dev = torch.device("cuda:0")
    q, k, v = (t.to(dev) for t in wl.config2(seed=1))
    kv = ptts.KvState(1, 1, 256, dtype="bf16")
    out = torch.empty(256, 512, dtype=torch.float32, device=dev)
    zero = np.zeros(1, np.int32)

    def step():
        kv.set_lengths([0], zero)
        ptts.attend(kv, 0, q, k, v, [0], [256], out=out)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    flops = 4 * 8 * 64 * sum(range(1, 257))
    try:
        peak = float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["bf16_tflops"])
        kind = "measured"
    except Exception:
        peak, kind = 1590.0, "fallback"
    achieved = flops / (ms / 1e3) / 1e12
    print(json.dumps({
        "metric": "prefill attention latency (config 2: one 256-row causal prompt, bf16 KV)",
        "value": ms, "unit": "ms", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": False, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config2", "rows": 256,
                   "note": "per call: plan, RoPE + append, tcgen05 prefill attention (2 query tiles x 8 heads, one head per CTA for so few tiles); the host side (Python wrapper, the list copy, three launches) takes about as long as the kernels"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_kind": kind,
                     "algorithmic_flops_per_call": flops}}), flush=True)
    kv.check()


def run_ring(args):
    """Ring caches in the config-5 frame (StreamingTransformer::start_ring / set_ring_slot /
    evict, transformer.rs:840-929): the shard's 512 streams on the 40m stack, prompts
    U{32..512} prefilled, then every stream a ring of 200 frame slots past its prompt. 200
    frames fill the slots, the oldest 50 of every ring are evicted (the kept keys past the
    prompt rotated back), and the timed frames write into the freed slots: per frame one
    ptts_b200_kv_set_ring_slots call for all 512 rings and one graph-replayed step. Every
    frame's attention reads each ring's slots up to its highest filled one (prompt + 200), the
    50 evicted ones masked; roofline bytes count all slots read."""
    import numpy as np
    import torch

    ring, evict = 200, 50
    if args.warmup + args.steps + 5 > evict:
        raise SystemExit(f"--warmup + --steps + 5 traced frames must fit the {evict} freed slots")
    ptts, wl = load()
    torch.cuda.set_device(0)
    dev = torch.device("cuda:0")
    cfg, B, prefixes, seed, desc = workload_spec(args, ptts, wl, 0)
    model = ptts.Transformer(cfg, 0)
    model.load(ptts.random_weights(cfg, seed))
    cap = int(prefixes.max()) + ring
    streams = np.arange(B, dtype=np.int32)
    kv = ptts.KvState(cfg.num_layers, B, cap, dtype="bf16")
    g = torch.Generator(device=dev).manual_seed(seed * 1000)
    model.forward(kv, torch.randn(int(prefixes.sum()), cfg.d_model, generator=g, device=dev).bfloat16(),
                  streams, prefixes)
    kv.start_ring(streams)
    xs = [torch.randn(B, cfg.d_model, generator=g, device=dev).bfloat16() for _ in range(8)]
    y = torch.empty(B, cfg.d_model, dtype=torch.float32, device=dev)
    for f in range(ring):
        kv.set_ring_slots(streams, prefixes + f)
        model.step(kv, streams, xs[f % 8], out=y)
    t0 = time.perf_counter()
    for st in streams:
        p = int(prefixes[st])
        kv.evict(int(st), p, list(range(p, p + evict)))
    torch.cuda.synchronize()
    evict_ms = (time.perf_counter() - t0) * 1e3
    state = {"f": 0}

    def frame():
        kv.set_ring_slots(streams, prefixes + state["f"])  # the freed slots, oldest first
        model.step(kv, streams, xs[state["f"] % 8], out=y)
        state["f"] += 1

    for _ in range(args.warmup):
        frame()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        frame()
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    ptts.set_tracing(True)
    ptts.trace(reset=True)
    for _ in range(5):
        frame()
    torch.cuda.synchronize()
    tr = ptts.trace(reset=True)
    ptts.set_tracing(False)
    kv.check()
    peak, peak_kind = peaks()
    per_launch_bytes = tr["attn_bytes"] / max(tr["attn_launches"], 1)
    per_launch_ms = tr["attn_ms"] / max(tr["attn_launches"], 1)
    achieved = per_launch_bytes / (per_launch_ms / 1e3) / 1e9
    print(json.dumps({
        "metric": "flow-LM frames/s with ring caches (a hole of 50 evicted frames in each ring)",
        "value": B / (ms / 1e3), "unit": "frames/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "dtype": "bf16",
        "data": "synthetic (seeded random-init int8 weights and N(0,1) hidden rows)",
        "config": {"workload": "ring: config5 shard (40m, 512 streams, prefixes U{32..512}), rings of "
                               f"{ring} frame slots, {evict} evicted, timed frames in the freed slots",
                   "lanes": ptts.step_lanes(B)},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "kernel": "decode_attn_kernel<bf16> (split-KV, ring masks)",
                     "algorithmic_bytes_per_launch": per_launch_bytes, "launch_ms": per_launch_ms,
                     "launches_timed": tr["attn_launches"]},
        "evict_ms_all_streams": evict_ms}), flush=True)


def run_mimi(args):
    """Mimi's transformer, the phonon codec's (2 layers, d 512, 8 heads, ff 2048, context 250:
    MimiStreamingMultiheadAttention inside StreamingTransformerLayer, transformer.rs:395-468 and
    :591-634), decoding one frame per stream for 512 windowed streams per GPU whose positions
    lie past the window, through ptts_b200_forward (windowed streams run the host-position path,
    not the graph-replayed step). Random f32 layers with layer scales 0.01, synthetic rows. A
    step is one frame for all streams; value = stream-frames/s. The attention reads the last
    250 K and V rows of every stream in both layers (bf16, 1 KB per row each)."""
    import numpy as np
    import torch

    ptts, wl = load()
    torch.cuda.set_device(0)
    dev = torch.device("cuda:0")
    cfg, ctx = ptts.MIMI_TRANSFORMER, ptts.MIMI_CONTEXT
    B, cap, prompt = 512, 512, 260  # a call adds at most cap - ctx + 1 = 263 rows to a stream
    model = ptts.Transformer(cfg)
    model.load_mimi(ptts.random_mimi_tensors(cfg, 7))
    kv = ptts.KvState(cfg.num_layers, B, cap, dtype="bf16")
    streams = list(range(B))
    kv.set_window(streams, ctx)
    g = torch.Generator(device=dev).manual_seed(7)
    for s0 in range(0, B, 64):  # the prompts, 64 streams per call
        x = torch.randn(64 * prompt, cfg.d_model, generator=g, device=dev).bfloat16()
        model.forward(kv, x, streams[s0:s0 + 64], [prompt] * 64)
    frames = [torch.randn(B, cfg.d_model, generator=g, device=dev).bfloat16() for _ in range(4)]
    ones = [1] * B

    def step(i):
        model.forward(kv, frames[i % 4], streams, ones)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        step(args.warmup + i)
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    kv.check()
    kv_bytes = B * cfg.num_layers * ctx * 2 * 1024
    print(json.dumps({
        "metric": "Mimi transformer decode (windowed streams past the 250-position window)",
        "value": B / (ms / 1e3), "unit": "frames/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "dtype": "bf16",
        "data": "synthetic (random f32 layers, layer scale 0.01, N(0,1) rows)",
        "config": {"workload": "mimi: 2 layers, d 512, 8 heads, ff 2048, context 250, 512 streams, "
                               f"positions {prompt + args.warmup}..{prompt + args.warmup + args.steps}",
                   "path": "ptts_b200_forward, one row per stream (host positions, no graph)"},
        "kv_bytes_per_step": kv_bytes,
        "kv_gbs_over_the_whole_step": kv_bytes / (ms / 1e3) / 1e9}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--repeats", type=int, default=0,
                    help="timed regions of K frames from the same centred start (0: at least 15 and "
                         "at least 1 s of timed work); K >= 250 frames are timed once")
    ap.add_argument("--no-config3", action="store_true",
                    help="skip the decode_attn object (config 3 through the attention op)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--timeline", default="",
                    help="write the kernel timeline (device stamps) of one decode step to this file")
    ap.add_argument("--no-flow", action="store_true",
                    help="skip the extra line item: whole frames with the flow head (ptts_b200_frame)")
    ap.add_argument("--workload", choices=["config5", "config4", "config3", "config2", "mimi", "ring"],
                    default="config5",
                    help="config5: the flow-LM frame, 512 streams/GPU (default); config4: 31m, "
                         "64 streams, prefix 128; config3: the attention op alone; config2: one "
                         "256-row prompt; mimi: Mimi's transformer decoding 512 windowed streams; "
                         "ring: the config-5 frame with ring caches after an eviction")
    ap.add_argument("--weights", choices=["int8", "q8_0"], default="int8",
                    help="int8 with per-row scales (default), or the same values as GGUF q8_0 blocks "
                         "(the published checkpoints' format: f16-plane linears)")
    ap.add_argument("--layers", type=int, default=0,
                    help="profiling aid: override the layer count (recorded in config.workload)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "config3":
        run_config3(args)
    elif args.workload == "config2":
        run_config2(args)
    elif args.workload == "mimi":
        run_mimi(args)
    elif args.workload == "ring":
        run_ring(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
