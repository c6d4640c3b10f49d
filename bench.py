#!/usr/bin/env python
"""Benchmark of the quantized-decoder hot path on B200 (libaexis_cuda).

Headline: the batch-1 Q4 group-32 dequant-GEMV sweep over
(K, N) = (1024,3072), (1024,512), (1024,3584), (3584,1024), (1024,151936), in
algorithmic HBM GB/s. One step = one pass over the five GEMVs (fp16 x and y,
fp16 scales, fp32 accumulation). Weight sets are rotated among copies whose
total is > 4x L2, so no step finds its weights in L2. Steps are replayed from
CUDA graphs (programmatic dependent launch between the GEMVs).

Also reported: config 1 (Q8 GEMV) and config 3 (the 24-layer synthetic Q4
decoder: 512-token prompt, 64 greedy tokens, tokens/s), the dominant kernel's
roofline, the CPU oracle baseline, clocks during the timed region, and the
end-to-end number through the C ABI with host buffers.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

N > 1 runs under torchrun: the sweep does not shard (a GEMV has no exchange),
so every rank runs the same workload as an independent replica; value is the
aggregate over ranks, timed as the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from aiimage_b200 import synth  # noqa: E402

SWEEP = synth.Q4_SWEEP
GROUP = 32
SWEEP_BYTES = [synth.gemv_bytes(4, n, k, GROUP) for (k, n) in SWEEP]
STEP_BYTES = sum(SWEEP_BYTES)
L2_BYTES = 126 * 1024 * 1024
DOMINANT = 4  # (1024, 151936): the lm_head-sized GEMV, 93% of a step's bytes


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def measured_tflops():
    """Dense fp16/bf16 tensor peak for a kernel timed alone (burst figure)."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def profile_traffic(name: str):
    """DRAM bytes per launch from a committed ncu summary (profiles/<name>),
    line 'traffic_bytes_per_launch: <int>'; None when absent."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        for line in open(path):
            if line.strip().startswith("traffic_bytes_per_launch:"):
                return int(line.split(":", 1)[1].strip().split()[0])
    except OSError:
        pass
    return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {"gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
               "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100}

    def __init__(self, index: int, period_s: float = 0.005):
        self.index, self.period = index, period_s
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception as e:  # NVML missing: report no samples
            self.error = str(e)
        return self

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                try:
                    r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                except AttributeError:
                    r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
                for name, bit in self.REASONS.items():
                    if r & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *exc):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(self.samples)}


def dist_setup(n_gpus: int):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        # NCCL's communicator set-up log (rank count, channels, NVLS) goes to
        # stderr, so that rank 0's one JSON line stands alone on stdout; an
        # explicit NCCL_DEBUG / NCCL_DEBUG_FILE request is kept.
        if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION"):
            os.environ["NCCL_DEBUG"] = "INFO"
            os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
            os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def process_group_info(world: int):
    """The communicator the timings ran over (None at N=1): backend, world size, NCCL version."""
    if world == 1:
        return None
    import torch
    import torch.distributed as dist
    v = torch.cuda.nccl.version()
    return {"backend": dist.get_backend(), "world_size": dist.get_world_size(),
            "nccl": ".".join(str(x) for x in v) if isinstance(v, tuple) else str(v),
            "log": "NCCL_DEBUG=INFO (subsystem INIT) on stderr"}


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    import torch
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


class Sweep:
    """The config-2 weight sets, uploaded `copies` times, and per-copy graphs."""

    def __init__(self, ops, seed: int = 1):
        import torch
        self.ops = ops
        self.copies = max(2, -(-4 * L2_BYTES // STEP_BYTES))  # total > 4x L2
        host = [synth.q4_weights(n, k, GROUP, seed, tag=(k, n)) for (k, n) in SWEEP]
        self.w = [[ops.new_int4_weight_only_upload(p, s, n, k, GROUP) for (p, s), (k, n) in zip(host, SWEEP)]
                  for _ in range(self.copies)]
        self.x_host = [synth.activations(k, seed, tag=(k, n)) for (k, n) in SWEEP]
        # The step's activations and outputs each live in one buffer (host and
        # device), so a step moves its inputs and results with one copy each way.
        xo = np.cumsum([0] + [x.size for x in self.x_host])
        yo = np.cumsum([0] + [n for (k, n) in SWEEP])
        x_flat = np.concatenate([x.ravel() for x in self.x_host])
        self.x_all = torch.from_numpy(x_flat).cuda()
        self.x_all_pin = torch.from_numpy(x_flat).pin_memory()
        self.y_all = torch.zeros(int(yo[-1]), dtype=torch.float16, device="cuda")
        self.y_all_pin = torch.zeros(int(yo[-1]), dtype=torch.float16).pin_memory()
        self.x = [self.x_all[xo[i]:xo[i + 1]].view(1, -1) for i in range(len(SWEEP))]
        self.y = [self.y_all[yo[i]:yo[i + 1]].view(1, -1) for i in range(len(SWEEP))]

    def gemv(self, copy: int, i: int):
        k, n = SWEEP[i]
        self.ops.set_int8_gemm_weights(None)
        self.ops.set_int4_gemm_weights(self.w[copy][i])
        self.ops.gemm2d_pack4_linear_texture_a(self.x[i], None, 1, n, k, True, 1.0, 1.0, False, 4, self.y[i])

    def step(self, copy: int):
        for i in range(len(SWEEP)):
            self.gemv(copy, i)

    def graph_steps(self, fn, n: int):
        """Capture n consecutive steps fn(i % copies), i = 0..n-1, into one graph."""
        import torch
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for i in range(n):
                    fn(i % self.copies)
        torch.cuda.current_stream().wait_stream(s)
        return g

    def graph(self, fn, reps: int):
        """Capture `reps` rotations of fn(copy) over all copies into one graph."""
        import torch
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for _ in range(reps):
                    for c in range(self.copies):
                        fn(c)
        torch.cuda.current_stream().wait_stream(s)
        return g


class StepGraphs:
    """Graphs that replay exactly n steps of fn(copy), copies rotating so no
    two consecutive steps read the same weights: a chunk of C steps (C a
    multiple of the copy count) replayed n // C times, then one graph of the
    n % C remaining steps (copies 0.. again, after a chunk that ended on the
    last copy)."""

    def __init__(self, sw, fn, n: int, max_chunk: int = 240):
        self.copies = sw.copies
        c = self.copies * max(1, min(n, max_chunk) // self.copies)
        self.chunk = c if n >= c else 0
        self.reps = n // c if self.chunk else 0
        rem = n - self.reps * c
        self.g_chunk = sw.graph_steps(fn, c) if self.chunk else None
        self.g_rem = sw.graph_steps(fn, rem) if rem else None
        self.n = n

    def replay(self):
        for _ in range(self.reps):
            self.g_chunk.replay()
        if self.g_rem is not None:
            self.g_rem.replay()


# SM cycles of the spin queued ahead of a timed region (about 1 ms at 1.9 GHz).
LAUNCH_COVER_CYCLES = 2_000_000


def cover_launches():
    """Queue a short device-side spin ahead of a start event. The host then
    submits the timed graphs while the stream is still busy, so the events
    bracket the steps' device time rather than the host's launch latency (a
    20-step region lasts well under a millisecond; with idle streams its first
    graph submission, slower still with several ranks sharing the host, would
    count as GPU time)."""
    import torch
    torch.cuda._sleep(LAUNCH_COVER_CYCLES)


def time_steps(graphs: StepGraphs, world: int) -> float:
    """CUDA-event time of exactly graphs.n steps, barrier + synchronize on both sides."""
    import torch
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cover_launches()
    start.record()
    graphs.replay()
    end.record()
    end.synchronize()
    barrier(world)
    return start.elapsed_time(end) / 1e3


def load_window(graphs: StepGraphs, seconds: float):
    """Replays the same steps for about `seconds` (untimed): the clock
    sampler's window around the timed region, so it holds many NVML samples
    taken under the same load."""
    import torch
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        graphs.replay()
        torch.cuda.synchronize()


def run_gpu(args):
    import torch
    world, rank, local = dist_setup(args.gpus)
    from aiimage_b200.ops import AexisOps
    from aiimage_b200 import native
    native.lib()  # fails loudly when the CUDA library is missing
    ops = AexisOps(local)
    sw = Sweep(ops)
    copies = sw.copies
    for c in range(copies):  # first calls outside capture (kernel attributes, occupancy)
        sw.step(c)
    torch.cuda.synchronize()
    timed = StepGraphs(sw, sw.step, args.steps)
    warm = StepGraphs(sw, sw.step, args.warmup)
    warm.replay()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        load_window(timed, 0.25)
        secs = time_steps(timed, world)
        load_window(timed, 0.1)
    secs = max_over_ranks(secs, world)
    value = world * args.steps * STEP_BYTES / secs / 1e9

    # Dominant kernel alone: back-to-back launches over rotating copies.
    def dom(c):
        sw.gemv(c, DOMINANT)
    dom_reps = max(1, 120 // copies)
    g_dom = sw.graph(dom, dom_reps)
    g_dom.replay()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_rep = 5
    cover_launches()
    ev0.record()
    for _ in range(n_rep):
        g_dom.replay()
    ev1.record()
    ev1.synchronize()
    dom_launches = n_rep * dom_reps * copies
    dom_s = ev0.elapsed_time(ev1) / 1e3 / dom_launches
    peak, peak_kind = measured_peak()
    achieved = SWEEP_BYTES[DOMINANT] / dom_s / 1e9
    traffic = profile_traffic("gemv_mma_q4_1024x151936.md")

    # Per-shape throughput (each GEMV alone, same method), config 1 Q8 GEMV.
    per_shape = {}
    for i, (k, n) in enumerate(SWEEP):
        g = sw.graph(lambda c, i=i: sw.gemv(c, i), max(1, 120 // copies))
        g.replay()
        torch.cuda.synchronize()
        cover_launches()
        ev0.record()
        g.replay()
        ev1.record()
        ev1.synchronize()
        t = ev0.elapsed_time(ev1) / 1e3 / (max(1, 120 // copies) * copies)
        per_shape[f"{k}x{n}"] = {"us": round(t * 1e6, 3), "GB/s": round(SWEEP_BYTES[i] / t / 1e9, 1),
                                 "frac": round(SWEEP_BYTES[i] / t / 1e9 / peak, 3)}
    q8 = bench_q8(ops, peak)

    # End to end through the C ABI with host buffers: per step, H2D of the five
    # activations from pinned memory (one packed copy), the five gemm calls, D2H
    # of the five outputs (one packed copy).
    stream = torch.cuda.current_stream()

    def e2e_step(c):
        sw.x_all.copy_(sw.x_all_pin, non_blocking=True)
        sw.step(c)
        sw.y_all_pin.copy_(sw.y_all, non_blocking=True)
        stream.synchronize()

    e2e_steps = max(1, min(args.steps, 200))
    for c in range(min(args.warmup, copies)):
        e2e_step(c)
    barrier(world)
    ev0.record()
    for i in range(e2e_steps):
        e2e_step(i % copies)
    ev1.record()
    ev1.synchronize()
    e2e_s = max_over_ranks(ev0.elapsed_time(ev1) / 1e3, world)
    h2d = sum(k * 2 for k, n in SWEEP)
    d2h = sum(n * 2 for k, n in SWEEP)

    decoder = None
    if not args.skip_decoder:
        try:
            decoder = bench_decoder(ops, peak)
        except Exception as e:  # reported, never silently replaced
            decoder = {"error": f"{type(e).__name__}: {e}"}

    hybrid = None
    if not args.skip_decoder:
        try:
            hybrid = bench_hybrid_decoder(ops, peak)
        except Exception as e:
            hybrid = {"error": f"{type(e).__name__}: {e}"}

    config4 = None
    if not args.skip_config4:
        try:
            config4 = bench_config4(ops, peak, world, rank)
        except Exception as e:
            config4 = {"error": f"{type(e).__name__}: {e}"}

    config5 = None
    if not args.skip_config5:
        try:
            config5 = bench_config5(ops, world, rank)
        except Exception as e:
            config5 = {"error": f"{type(e).__name__}: {e}"}

    w8a8 = None
    if not args.skip_w8a8:
        try:
            w8a8 = bench_w8a8(ops, peak)
        except Exception as e:
            w8a8 = {"error": f"{type(e).__name__}: {e}"}

    sampler = None
    if not args.skip_sampler:
        try:
            sampler = bench_sampler(ops, peak)
        except Exception as e:
            sampler = {"error": f"{type(e).__name__}: {e}"}

    linear_attn = None
    if not args.skip_linear_attention:
        try:
            linear_attn = bench_linear_attention(ops, peak)
        except Exception as e:
            linear_attn = {"error": f"{type(e).__name__}: {e}"}

    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu:
        cpu = cpu_baseline(args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": "Q4 g32 dequant-GEMV sweep, algorithmic HBM GB/s (batch 1)",
            "value": round(value, 1),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(secs / args.steps * 1e3, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "int4 weights, fp16 act/scales, fp32 accumulate",
            "data": "synthetic (seeded PCG64; BASELINE config 2 shapes and distributions)",
            "config": sweep_config(world),
            "timing": {"graphs": f"exactly {args.steps} steps: {timed.reps} replay(s) of a {timed.chunk}-step graph"
                                 f" + one {args.steps - timed.reps * timed.chunk}-step graph",
                       "events": "CUDA events on the launching stream, barrier + synchronize both sides"},
            "roofline": {"bound": "hbm", "kernel": "gemv_mma_kernel q4 g32 fp16-x int8-MMA path (1024x151936)",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "algorithmic_bytes_per_launch": SWEEP_BYTES[DOMINANT],
                         "us_per_launch": round(dom_s * 1e6, 3), "peak_source": peak_kind + " (MEASURED_PEAKS.json hbm_gbs)"},
            "per_shape": per_shape,
            "config1_q8": q8,
            "decoder": decoder,
            "hybrid_decoder": hybrid,
            "config4": config4,
            "config5": config5,
            "linear_attention": linear_attn,
            "sampler": sampler,
            "w8a8": w8a8,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_steps * STEP_BYTES * world / e2e_s / 1e9, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": "aexis_cuda_gemm via ctypes, pinned host x/y, sync per step"},
            "process_group": process_group_info(world),
            "gpu_launches": args.steps * len(SWEEP),
            "clocks": {**clk.summary(), "window": "NVML every 5 ms over 0.25 s of the same step graphs, the"
                                                  " timed region, then 0.1 s more"},
        }
        print(json.dumps(line), flush=True)
    ops.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def sweep_config(world: int) -> dict:
    """The workload, identical in both arms (the reference arm rotates the same weight copies in host memory)."""
    copies = max(2, -(-4 * L2_BYTES // STEP_BYTES))
    return {"workload": "config2_q4_g32_gemv_sweep_m1", "shapes_KxN": [list(s) for s in SWEEP],
            "bytes_per_step": STEP_BYTES, "weight_copies": copies,
            "l2": f"weights rotated over {copies} copies ({copies * STEP_BYTES / 2**20:.0f} MiB > 4x L2)",
            "parallelism": f"replicas x{world}"}


def bench_q8(ops, peak):
    """Q8 K=1024 N=3584 GEMV (rotated copies, graph)."""
    import torch
    k, n = 1024, 3584
    p, s = synth.q8_weights(n, k, seed=0)
    b = synth.gemv_bytes(8, n, k)
    copies = max(2, -(-4 * L2_BYTES // b))
    ws = [ops.new_int8_weight_only_upload(p, s, n, k) for _ in range(copies)]
    x = torch.from_numpy(synth.activations(k, seed=0)).cuda()
    y = torch.zeros((1, n), dtype=torch.float16, device="cuda")

    def call(c):
        ops.set_int4_gemm_weights(None)
        ops.set_int8_gemm_weights(ws[c])
        ops.gemm2d_pack4_linear_texture_a(x, None, 1, n, k, True, 1.0, 1.0, False, 4, y)

    call(0)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        with torch.cuda.graph(g, stream=st):
            for c in range(copies):
                call(c)
    torch.cuda.current_stream().wait_stream(st)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cover_launches()
    e0.record()
    for _ in range(3):
        g.replay()
    e1.record()
    e1.synchronize()
    t = e0.elapsed_time(e1) / 1e3 / (3 * copies)
    return {"shape_KxN": [k, n], "bytes": b, "us": round(t * 1e6, 3), "GB/s": round(b / t / 1e9, 1),
            "frac": round(b / t / 1e9 / peak, 3)}


def bench_decoder(ops, peak, prompt_len: int = 512, new_tokens: int = 64):
    """24-layer synthetic Q4 decoder, 512-token prompt, then
    64 greedy tokens. Device tokens/s from the graph-chained generate call
    (one H2D token in, one D2H of the 64 ids out), and the per-token host
    round-trip rate (aexis_cuda_decoder_step: id in, greedy id out)."""
    import torch
    from aiimage_b200.decoder import DecoderSession
    cfg = synth.QWEN35_08B_Q4
    model = synth.SyntheticDecoder(cfg, seed=3)
    prompt = model.prompt(prompt_len, seed=30)
    sess = DecoderSession(ops, cfg).load(model)
    sess.prefill(prompt[:-1])
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    toks = sess.generate(prompt[-1:], new_tokens)  # decode steps at positions prompt_len-1 ..
    gen_s = time.perf_counter() - t0
    sess.reset()
    sess.prefill(prompt[:-1])
    nxt = int(prompt[-1])
    t0 = time.perf_counter()
    for _ in range(new_tokens):
        nxt = sess.step(nxt)
    step_s = time.perf_counter() - t0
    kv_mean = cfg.n_layers * 2 * cfg.n_kv_heads * cfg.head_dim * 2 * (prompt_len - 1 + new_tokens // 2)
    bytes_tok = model.weight_bytes_per_token() + kv_mean
    # The same generate call under the persistent schedule (one cooperative
    # kernel for every emitting step), reported beside the default graphs.
    persist = None
    sess.set_schedule(-1)
    if sess.schedule() == 1:
        sess.reset()
        sess.generate(prompt[:8], 2)  # first use packs the weight stream: not timed
        sess.reset()
        sess.prefill(prompt[:-1])
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        ptoks = sess.generate(prompt[-1:], new_tokens)
        ps = time.perf_counter() - t0
        persist = {"tokens_per_s": round(new_tokens / ps, 1), "ms_per_token": round(ps / new_tokens * 1e3, 4),
                   "same_tokens": ptoks == toks}
    sess.close()
    n = new_tokens
    return {"workload": f"config3_q4_decoder_prompt{prompt_len}_greedy{n}", "tokens_per_s": round(n / gen_s, 1),
            "ms_per_token": round(gen_s / n * 1e3, 4), "e2e_tokens_per_s_host_roundtrip": round(n / step_s, 1),
            "bytes_per_token": bytes_tok, "GB/s": round(bytes_tok * n / gen_s / 1e9, 1),
            "frac": round(bytes_tok * n / gen_s / 1e9 / peak, 3), "first_tokens": toks[:8],
            "kernels_per_token": 2 + 5 * cfg.n_layers + 1, "schedule": "graph per step",
            "persistent_schedule": persist}


def bench_hybrid_decoder(ops, peak, prompt_len: int = 512, new_tokens: int = 64):
    """The hybrid Qwen3.5 stack (18 linear-attention blocks, ShortConv + Gated
    Delta Rule, and 6 full-attention blocks; Q4 g32, vocab 151936): 512-token
    prompt, then 64 greedy tokens through the graph-chained generate call.
    Bytes per token: every weight once, the 6 KV caches at the mean context,
    and per linear-attention layer the fp32 GDR state read and written
    (2 x 16 x 128 x 128 x 4 bytes) plus the conv cache (3 rows read, 4
    written, 6144 channels)."""
    import torch
    from aiimage_b200.decoder import DecoderSession
    cfg = synth.QWEN35_08B_HYBRID_Q4
    model = synth.SyntheticDecoder(cfg, seed=6, norm_mean=1.0, balanced_q4=True)
    prompt = model.prompt(prompt_len, seed=60)
    sess = DecoderSession(ops, cfg).load(model)
    sess.prefill(prompt[:-1])
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    toks = sess.generate(prompt[-1:], new_tokens)
    gen_s = time.perf_counter() - t0
    sess.close()
    kinds = cfg.layer_types()
    n_full, n_lin = kinds.count(0), kinds.count(1)
    kv_mean = n_full * 2 * cfg.n_kv_heads * cfg.head_dim * 2 * (prompt_len - 1 + new_tokens // 2)
    state = n_lin * (2 * cfg.lin_heads * cfg.lin_kdim * cfg.lin_vdim * 4
                     + (2 * cfg.conv_kernel - 1) * cfg.conv_channels() * 4)
    bytes_tok = model.weight_bytes_per_token() + kv_mean + state
    n = new_tokens
    return {"workload": f"qwen35_hybrid_q4_decoder_prompt{prompt_len}_greedy{n} (18 linear + 6 full attention)",
            "tokens_per_s": round(n / gen_s, 1), "ms_per_token": round(gen_s / n * 1e3, 4),
            "bytes_per_token": bytes_tok, "recurrent_state_bytes_per_token": state,
            "GB/s": round(bytes_tok * n / gen_s / 1e9, 1), "frac": round(bytes_tok * n / gen_s / 1e9 / peak, 3),
            "first_tokens": toks[:8], "kernels_per_token": 2 + 5 * cfg.n_layers + 1,
            "timing": "host clock around one generate call (one H2D token in, one D2H of the ids out)"}


def bench_config4(ops, peak, world: int, rank: int, steps: int = 128, total_seqs: int = 256, per_batch: int = 32):
    """the Q8 decoder of config 3's shape, 256 sequences
    with contexts U[256, 4096] (seeded), split over the ranks (strong
    scaling: rank r decodes sequences r*256/G ..), 32 per batch, 128 greedy
    steps per batch. The contexts are synthetic KV fills (stand-ins for the
    prefill, outside the timed region); only the decode steps are timed, on
    the device (CUDA events around each batch's generate call)."""
    import torch
    from aiimage_b200.decoder import BatchSession, DecoderSession
    d = synth.QWEN35_08B_Q8.as_dict()
    d.update(kv_capacity=256)
    cfg = synth.DecoderCfg(**d)
    model = synth.SyntheticDecoder(cfg, seed=4)
    dec = DecoderSession(ops, cfg).load(model)
    rng = np.random.default_rng([4, 256, 4096])
    ctx_all = rng.integers(256, 4097, size=total_seqs).astype(np.int32)
    first_all = rng.integers(0, cfg.vocab, size=total_seqs).astype(np.int32)
    lo, hi = rank * total_seqs // world, (rank + 1) * total_seqs // world
    cap = 4096 + steps
    batch = BatchSession(dec, max_batch=per_batch, kv_capacity=cap, max_steps=steps)
    # Warm-up: graph capture and first launches on the first batch.
    batch.fill_context(ctx_all[lo:lo + per_batch], seed=4, first_seq_id=lo)
    batch.generate(first_all[lo:lo + per_batch], 3)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dev_s, tokens, kv_bytes, first_ids = 0.0, 0, 0, None
    kv_row = cfg.n_layers * 2 * cfg.n_kv_heads * cfg.head_dim * 2  # K+V bytes per position, all layers
    for b0 in range(lo, hi, per_batch):
        b1 = min(hi, b0 + per_batch)
        batch.fill_context(ctx_all[b0:b1], seed=4, first_seq_id=b0)
        torch.cuda.synchronize()
        e0.record()
        out = batch.generate(first_all[b0:b1], steps)
        e1.record()
        e1.synchronize()
        dev_s += e0.elapsed_time(e1) / 1e3
        tokens += (b1 - b0) * steps
        kv_bytes += int(sum(int(c) * steps + steps * (steps + 1) // 2 for c in ctx_all[b0:b1])) * kv_row
        if first_ids is None:
            first_ids = out[:4, 0].tolist()
    total_s = max_over_ranks(dev_s, world)
    w_bytes = model.weight_bytes_per_token() - cfg.hidden * 2  # linears + norms (embedding rows counted per token)
    n_steps = (hi - lo + per_batch - 1) // per_batch * steps
    byts = w_bytes * n_steps + kv_bytes
    batch.close()
    dec.close()
    return {"workload": "config4_q8_decoder_batch32_ctxU256-4096_greedy128", "gpus": world,
            "scaling": "strong", "sequences": total_seqs, "sequences_this_rank": hi - lo,
            "tokens_per_s": round(total_seqs * steps / total_s, 1),
            "tokens_per_s_per_gpu": round(tokens / dev_s, 1),
            "ms_per_step": round(dev_s / n_steps * 1e3, 4),
            "bytes_per_step_mean": int(byts / n_steps), "GB/s": round(byts / dev_s / 1e9, 1),
            "frac": round(byts / dev_s / 1e9 / peak, 3), "first_ids": first_ids,
            "timing": "device (CUDA events around each batch's generate), max over ranks"}


def bench_w8a8(ops, peak):
    """W8A8 activation fake-quantisation (SetInt8ActivationQuantization) on the Q8 paths: the config-1 GEMV
    (K 1024, N 3584, batch 1) and the same weights at 32 rows (tensor cores), each timed with and without the
    activation codes. Weights rotate over copies larger than L2 (GEMV) inside a CUDA graph; CUDA events."""
    import torch
    import types
    k, n = 1024, 3584
    p, s = synth.q8_weights(n, k, seed=0)
    b = synth.gemv_bytes(8, n, k)
    copies = max(2, -(-4 * L2_BYTES // b))
    ws = [ops.new_int8_weight_only_upload(p, s, n, k) for _ in range(copies)]
    out = {}
    for rows in (1, 32):
        x = torch.from_numpy(synth.activations(k, seed=0, m=rows)).cuda()
        y = torch.zeros((rows, n), dtype=torch.float16, device="cuda")
        for quant in (False, True):
            ops.set_int8_activation_quantization(types.SimpleNamespace(mode="Int8W8A8", activation_scale=0.03,
                                                                       activation_zero_point=0) if quant else None)

            def call(c):
                ops.set_int4_gemm_weights(None)
                ops.set_int8_gemm_weights(ws[c])
                ops.gemm2d_pack4_linear_texture_a(x, None, rows, n, k, True, 1.0, 1.0, False, 4, y)

            for c in range(copies):
                call(c)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            st = torch.cuda.Stream()
            st.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(st):
                with torch.cuda.graph(g, stream=st):
                    for c in range(copies):
                        call(c)
            torch.cuda.current_stream().wait_stream(st)
            g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            cover_launches()
            e0.record()
            for _ in range(3):
                g.replay()
            e1.record()
            e1.synchronize()
            t = e0.elapsed_time(e1) / 1e3 / (3 * copies)
            out[f"rows{rows}_{'w8a8' if quant else 'w8a16'}_us"] = round(t * 1e6, 3)
    ops.set_int8_activation_quantization(None)
    out["workload"] = "Q8 K1024 N3584 (config 1 weights), activation scale 0.03, zero point 0"
    out["timing"] = "CUDA events over graph replays, weights rotated over copies > L2"
    return out


def bench_sampler(ops, peak):
    """Device sampling (Qwen35Sampler.Select with Qwen35SamplingConfig's defaults: T 0.3, top-k 50, top-p 0.8,
    repetition penalty 1.1 over a 64-token history) on the 151936-wide vocabulary, batch 1 (one decode step)
    and batch 256 (config 5's rows). Logits already on the device; CUDA events over back-to-back calls."""
    import torch
    vocab = 151936
    out = {}
    for rows in (1, 256):
        g = torch.Generator(device="cuda").manual_seed(11)
        logits = torch.randn((rows, vocab), generator=g, device="cuda", dtype=torch.float32) * 4
        hist = torch.zeros((rows, (vocab + 31) // 32), dtype=torch.int32, device="cuda")
        toks = torch.randint(0, vocab, (64, rows), generator=g, device="cuda", dtype=torch.int32)
        for t in range(64):
            ops.sample_history_add(hist, rows, vocab, toks[t])
        u = torch.rand(rows, generator=g, device="cuda", dtype=torch.float64)
        ids = torch.empty(rows, dtype=torch.int32, device="cuda")
        for _ in range(5):
            ops.sample(logits, rows, vocab, hist, 1.1, 0.3, 50, 0.8, u, ids)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = 50
        e0.record()
        for _ in range(n):
            ops.sample(logits, rows, vocab, hist, 1.1, 0.3, 50, 0.8, u, ids)
        e1.record()
        e1.synchronize()
        t = e0.elapsed_time(e1) / 1e3 / n
        read = rows * vocab * 4
        out[f"rows{rows}"] = {"us_per_call": round(t * 1e6, 2), "logits_GB/s": round(read / t / 1e9, 1)}
        # The whole vocabulary (top_k 0): the radix select by probability mass.
        for _ in range(3):
            ops.sample(logits, rows, vocab, hist, 1.1, 0.3, 0, 0.8, u, ids)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(10):
            ops.sample(logits, rows, vocab, hist, 1.1, 0.3, 0, 0.8, u, ids)
        e1.record()
        e1.synchronize()
        out[f"rows{rows}_top_k0"] = {"us_per_call": round(e0.elapsed_time(e1) / 10 * 1e3, 2)}
    out["workload"] = ("Qwen35Sampler.Select defaults (T 0.3, top-k 50, top-p 0.8, penalty 1.1), vocab 151936;"
                       " *_top_k0: the same with top-k 0 (the whole vocabulary)")
    out["timing"] = "CUDA events over 50 back-to-back calls, logits resident"
    return out


def bench_linear_attention(ops, peak, prefill: int = 512):
    """Linear-attention layers of Qwen3.5-0.8B (18 of its 24 blocks), batch-1
    decode: the Gated Delta Rule over 16 heads with key/value dims 128 and the
    causal ShortConv over 6144 channels (kernel 4). One decode launch of the
    GDR reads and writes the fp32 state once (2 x 1 MiB); the states rotate
    over copies larger than L2 (updated in place), each launch timed inside a
    graph by CUDA events. Also one 512-token prefill call (state kept on chip)."""
    import torch
    heads, kd, vd = 16, 128, 128
    rng = np.random.default_rng(17)
    state_bytes = heads * kd * vd * 4
    copies = max(2, -(-2 * L2_BYTES // state_bytes))
    states = [torch.from_numpy(rng.normal(0, 0.05, heads * kd * vd).astype(np.float32)).cuda() for _ in range(copies)]

    def vec(n, mu=0.0, sd=0.5):
        return torch.from_numpy(rng.normal(mu, sd, n).astype(np.float32)).cuda()

    a_log, dt = vec(heads, -1.0, 0.2), vec(heads, 0.0, 0.2)
    b, a = vec(prefill * heads, 0, 0.4), vec(prefill * heads, 0, 0.4)
    q, k, v = vec(prefill * heads * kd), vec(prefill * heads * kd), vec(prefill * heads * vd)
    out = torch.zeros(prefill * heads * vd, dtype=torch.float32, device="cuda")

    def gdr(c, first=0, count=1):
        ops.gated_delta_rule_pack4(a_log, dt, b, a, q, k, v, states[c], out, states[c], heads, kd, vd, prefill,
                                   token_index=first, token_count=count)

    groups, kernel = 6144, 4
    ld = groups
    conv_w = vec(groups * kernel, 0, 0.3)
    conv_x = vec(ld)
    conv_cache = vec(kernel * ld)
    conv_out = torch.zeros(ld, dtype=torch.float32, device="cuda")

    def conv(c):
        ops.short_conv_pack4(conv_w, conv_x, conv_cache, conv_out, conv_cache, groups, kernel, 1, kernel)

    def timed(fn, launches):
        for c in range(min(launches, 3)):
            fn(c)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            with torch.cuda.graph(g, stream=st):
                for c in range(launches):
                    fn(c)
        torch.cuda.current_stream().wait_stream(st)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        cover_launches()
        e0.record()
        for _ in range(3):
            g.replay()
        e1.record()
        e1.synchronize()
        return e0.elapsed_time(e1) / 1e3 / (3 * launches)

    gdr_s = timed(lambda c: gdr(c % copies), copies)
    gdr_bytes = 2 * state_bytes + 4 * heads * (2 * kd + 2 * vd) + 4 * 2 * heads
    conv_s = timed(conv, 64)
    conv_bytes = 4 * (groups * kernel + 2 * kernel * groups + 2 * groups)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gdr(0, 0, prefill)
    e0.record()
    for c in range(1, 4):
        gdr(c, 0, prefill)
    e1.record()
    e1.synchronize()
    pre_s = e0.elapsed_time(e1) / 1e3 / 3
    return {"workload": "qwen35_08b_linear_attention_decode_b1 (GDR 16 heads x 128 x 128; ShortConv 6144 ch, k4)",
            "gdr_decode_us": round(gdr_s * 1e6, 3), "gdr_decode_bytes": gdr_bytes,
            "gdr_decode_GB/s": round(gdr_bytes / gdr_s / 1e9, 1),
            "gdr_decode_frac": round(gdr_bytes / gdr_s / 1e9 / peak, 3),
            "gdr_state_copies": copies,
            "short_conv_decode_us": round(conv_s * 1e6, 3), "short_conv_bytes": conv_bytes,
            "gdr_prefill_tokens": prefill, "gdr_prefill_us": round(pre_s * 1e6, 1),
            "gdr_prefill_tokens_per_s": round(prefill / pre_s, 1),
            "timing": "CUDA events around graph replays (decode), back-to-back calls (prefill)"}


def bench_config5(ops, world: int, rank: int, reps: int = 10):
    """lm_head 151936 x 1024 Q8 per row, batch 256 fp16
    hidden states, greedy argmax + top-50 per row. G > 1: vocab shards with
    the NCCL exchange (aiimage_b200.sharded); rank 0 checks the ids against a
    single-GPU run of the whole vocabulary."""
    import torch
    from aiimage_b200.sharded import ShardedLmHead
    from aiimage_b200.sharded import keys_to_ids as sharded_ids
    vocab, hidden, m, k = 151936, 1024, 256, 50
    p, s = synth.q8_weights(vocab, hidden, seed=5, tag=(vocab, hidden))
    x = torch.from_numpy(synth.activations(hidden, seed=5, tag=(m, hidden), m=m)).cuda()
    head = ShardedLmHead(ops, p, s, vocab, hidden, world, rank)
    logits = torch.empty((m, head.n), dtype=torch.float32, device="cuda")
    for _ in range(3):
        ids, vals, idx = head.forward(x, k, logits)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        ids, vals, idx = head.forward(x, k, logits)
    e1.record()
    e1.synchronize()
    call_s = max_over_ranks(e0.elapsed_time(e1) / 1e3 / reps, world)
    # GEMM alone (the dominant kernel of the call), this rank's shard.
    e0.record()
    for _ in range(reps):
        head.shard_logits(x, logits)
    e1.record()
    e1.synchronize()
    gemm_s = e0.elapsed_time(e1) / 1e3 / reps
    # The selection alone on this rank's logits: top-k, then the greedy keys from its lists.
    keys = torch.empty(m, dtype=torch.int64, device="cuda")
    tv = torch.empty((m, k), dtype=torch.float32, device="cuda")
    ti = torch.empty((m, k), dtype=torch.int32, device="cuda")
    e0.record()
    for _ in range(reps):
        ops.top_k(logits, head.n, m, k, tv, ti)
    e1.record()
    e1.synchronize()
    topk_s = e0.elapsed_time(e1) / 1e3 / reps
    e0.record()
    for _ in range(reps):
        ops.topk_greedy_keys(logits, head.n, m, k, tv, ti, head.lo, keys)
    e1.record()
    e1.synchronize()
    argmax_s = e0.elapsed_time(e1) / 1e3 / reps
    # The exchange alone (G > 1) on a buffer this rank's GEMM already filled, max over ranks as the whole
    # call: the call's own path (peer memory: push + merge), then the collective path (one NCCL
    # all-gather + aexis_cuda_topk_merge) for comparison.
    exchange_s = collective_s = None
    if world > 1:
        from aiimage_b200.sharded import pack_views, packed_words
        buf = torch.empty(packed_words(m, k), dtype=torch.int32, device="cuda")
        head.shard_topk(x, k, *pack_views(buf, m, k))

        def time_merge():
            head.merge(buf, m, k)
            torch.cuda.synchronize()
            barrier(world)
            e0.record()
            for _ in range(reps):
                head.merge(buf, m, k)
            e1.record()
            e1.synchronize()
            return max_over_ranks(e0.elapsed_time(e1) / 1e3 / reps, world)

        peer = head.uses_peer_exchange()
        exchange_s = time_merge()
        head.exchange_mode = "collective"
        collective_s = time_merge()
        head.exchange_mode = "auto"
    # The whole call as one CUDA graph (G = 1, or the peer exchange): the same kernels without the host's
    # launch gaps, replayed `reps` times; its results are the ones checked against one GPU below.
    graph_s = None
    if world == 1 or head.uses_peer_exchange():
        from aiimage_b200.sharded import pack_views, packed_words
        gbuf = torch.empty(packed_words(m, k), dtype=torch.int32, device="cuda")
        gk, gv, gi = pack_views(gbuf, m, k)
        g_ids = torch.empty(m, dtype=torch.int64, device="cuda")
        g_v = torch.empty((m, k), dtype=torch.float32, device="cuda")
        g_i = torch.empty((m, k), dtype=torch.int32, device="cuda")

        def one_call():
            head.shard_topk(x, k, gk, gv, gi)
            if world > 1:
                head.merge_into(gbuf, m, k, g_ids, g_v, g_i)

        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                one_call()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        barrier(world)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            one_call()
        graph.replay()
        torch.cuda.synchronize()
        barrier(world)
        cover_launches()
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        e1.synchronize()
        graph_s = max_over_ranks(e0.elapsed_time(e1) / 1e3 / reps, world)
        if world > 1:
            ids, vals, idx = g_ids, g_v, g_i.to(torch.int64)
        else:
            ids, vals, idx = sharded_ids(gk), gv, gi.to(torch.int64)
        del graph
    flops = 2.0 * m * vocab * hidden
    peak, kind = measured_tflops()
    best_s = graph_s if graph_s is not None else call_s
    out = {"workload": "config5_lm_head_q8_151936x1024_batch256_argmax_top50", "gpus": world,
           "ms_per_call": round(best_s * 1e3, 4), "TFLOP/s": round(flops / best_s / 1e12, 1),
           "timing": ("one CUDA graph per call (top-k GEMM, and at G > 1 the peer push and merge), replayed"
                      if graph_s is not None else "host loop of calls"),
           "ms_per_call_host_loop": round(call_s * 1e3, 4),
           "gemm_rank_ms": round(gemm_s * 1e3, 4),
           "greedy_keys_from_topk_rank_ms": round(argmax_s * 1e3, 4), "topk_rank_ms": round(topk_s * 1e3, 4),
           "gemm_rank_TFLOP/s": round(2.0 * m * head.n * hidden / gemm_s / 1e12, 1),
           "gemm_frac_of_tensor_peak": round(2.0 * m * head.n * hidden / gemm_s / 1e12 / peak, 3),
           "tensor_peak": f"{peak} TFLOP/s ({kind}, MEASURED_PEAKS.json bf16_tflops)",
           "first_ids": ids[:6].tolist()}
    if exchange_s is not None:
        out["exchange_ms"] = round(exchange_s * 1e3, 4)
        out["exchange"] = ((f"peer memory: aexis_cuda_topk_push of {packed_words(m, k) * 4} B (keys + top-{k} values"
                            f" and indices) into every rank's receive buffer over NVLink + aexis_cuda_topk_merge_peers"
                            f" (waits on the epoch flags)") if peer else
                           f"NCCL all-gather of {packed_words(m, k) * 4} B per rank + aexis_cuda_topk_merge") + \
            ", max over ranks"
        out["exchange_collective_ms"] = round(collective_s * 1e3, 4)
    if world > 1 and rank == 0:
        full = ShardedLmHead(ops, p, s, vocab, hidden, 1, 0)
        ids1, _, idx1 = full.forward(x, k)
        out["ids_match_single_gpu"] = bool(torch.equal(ids1, ids))
        out["top50_match_single_gpu"] = bool(torch.equal(idx1, idx))
        full.w.free()
    head.close()
    head.w.free()
    return out


def cpu_baseline(budget_s: float = 12.0):
    """The CPU oracle (restated reference path) on the same sweep, all host
    threads, bounded to ~budget_s of work, rotating the same weight copies as
    the GPU arm (host memory)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    O.build()
    copies = sweep_config(1)["weight_copies"]
    host = [synth.q4_weights(n, k, GROUP, 1, tag=(k, n)) for (k, n) in SWEEP]
    sets = [[(p.copy(), s.astype(np.float32)) for p, s in host] for _ in range(copies)]
    xs = [synth.activations(k, 1, tag=(k, n)).astype(np.float32) for (k, n) in SWEEP]
    passes, t0 = 0, time.perf_counter()
    while True:
        for (p, s), x, (k, n) in zip(sets[passes % copies], xs, SWEEP):
            O.gemm(x, 4, p, s, GROUP, n)
        passes += 1
        el = time.perf_counter() - t0
        if el >= budget_s or passes >= 60:
            break
    return {"value": round(passes * STEP_BYTES / el / 1e9, 3), "unit": "GB/s", "cores": O.num_threads(),
            "kind": "port", "sample": f"{passes} full sweep pass(es) of config 2 through the C++ oracle "
                                      f"(sequential fp32 per output, OpenMP over outputs), weights rotated over "
                                      f"{copies} host copies, {el:.1f} s"}


def run_only(args):
    """Single-kernel / single-path modes for profiling (not the bench contract):
    --only dominant   W + K launches of the (1024, 151936) Q4 GEMV, rotating
                      over copies larger than L2, no graphs
    --only decoder    the config-3 decoder with --prompt-len / --new-tokens
    --only hybrid     the hybrid Qwen3.5 decoder (18 linear + 6 full attention), same flags
    --only tcgemm     the config-5 lm_head GEMM alone (M=256, tensor cores)
    --only config4    one config-4 batch (32 sequences, --new-tokens steps)
    --only linear_attention  the Qwen3.5 GatedDeltaRule / ShortConv decode kernels
    --only sampler    the device sampler (Qwen35Sampler defaults) at 1 and 256 rows
    --only w8a8       the Q8 GEMV / 32-row GEMM with and without W8A8 activation codes"""
    import torch
    torch.cuda.set_device(0)
    from aiimage_b200.ops import AexisOps
    ops = AexisOps(0)
    peak, _ = measured_peak()
    if args.only == "decoder":
        out = bench_decoder(ops, peak, args.prompt_len, args.new_tokens)
    elif args.only == "hybrid":
        out = bench_hybrid_decoder(ops, peak, args.prompt_len, args.new_tokens)
    elif args.only == "linear_attention":
        out = bench_linear_attention(ops, peak)
    elif args.only == "sampler":
        out = bench_sampler(ops, peak)
    elif args.only == "w8a8":
        out = bench_w8a8(ops, peak)
    elif args.only == "topk":
        m, vocab, k = 256, 151936, 50
        g = torch.Generator(device="cuda").manual_seed(5)
        logits = torch.randn((m, vocab), generator=g, device="cuda", dtype=torch.float32)
        vals = torch.empty((m, k), dtype=torch.float32, device="cuda")
        idx = torch.empty((m, k), dtype=torch.int32, device="cuda")
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for i in range(args.warmup + args.steps):
            if i == args.warmup:
                e0.record()
            ops.top_k(logits, vocab, m, k, vals, idx)
        e1.record()
        e1.synchronize()
        t = e0.elapsed_time(e1) / 1e3 / max(1, args.steps)
        out = {"kernel": "topk 256x151936 k50", "us": round(t * 1e6, 2),
               "GB/s": round(m * vocab * 4 / t / 1e9, 1)}
    elif args.only == "config4":
        out = bench_config4(ops, peak, 1, 0, steps=args.new_tokens, total_seqs=32)
    elif args.only == "tcgemm":
        vocab, hidden, m = 151936, 1024, 256
        p, s = synth.q8_weights(vocab, hidden, seed=5, tag=(vocab, hidden))
        w = ops.new_int8_weight_only_upload(p, s, vocab, hidden)
        x = torch.from_numpy(synth.activations(hidden, seed=5, tag=(m, hidden), m=m)).cuda()
        y = torch.empty((m, vocab), dtype=torch.float32, device="cuda")
        ops.set_int8_gemm_weights(w)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for i in range(args.warmup + args.steps):
            if i == args.warmup:
                e0.record()
            ops.gemm2d_pack4_tiled_texture_a(x, None, m, vocab, hidden, True, 1.0, 1.0, False, 4, y)
        e1.record()
        e1.synchronize()
        t = e0.elapsed_time(e1) / 1e3 / max(1, args.steps)
        out = {"kernel": "gemm_q8_tc 256x151936x1024", "us": round(t * 1e6, 2),
               "TFLOP/s": round(2.0 * m * vocab * hidden / t / 1e12, 1)}
    else:
        k, n = SWEEP[DOMINANT]
        p, s = synth.q4_weights(n, k, GROUP, 1, tag=(k, n))
        copies = max(2, -(-2 * L2_BYTES // SWEEP_BYTES[DOMINANT]))
        ws = [ops.new_int4_weight_only_upload(p, s, n, k, GROUP) for _ in range(copies)]
        x = torch.from_numpy(synth.activations(k, 1, tag=(k, n))).cuda()
        y = torch.zeros((1, n), dtype=torch.float16, device="cuda")
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for i in range(args.warmup + args.steps):
            if i == args.warmup:
                e0.record()
            ops.set_int4_gemm_weights(ws[i % copies])
            ops.gemm2d_pack4_linear_texture_a(x, None, 1, n, k, True, 1.0, 1.0, False, 4, y)
        e1.record()
        e1.synchronize()
        t = e0.elapsed_time(e1) / 1e3 / max(1, args.steps)
        out = {"kernel": "gemv q4 1024x151936", "launches": args.warmup + args.steps, "copies": copies,
               "us_per_launch_incl_host_gaps": round(t * 1e6, 2)}
    print(json.dumps({"only": args.only, **out}), flush=True)
    ops.close()


def run_reference(args):
    """--impl reference: the reference's CPU path for this workload (the C++
    oracle restating AexisGemm2DPack4LinearTextureA / AexisGemm2DReadB) on all
    host threads, over the same weight copies the GPU arm rotates (host
    memory, step i reads copy i % copies). Under torchrun only rank 0 runs."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    O.build()
    cfg = sweep_config(world)
    copies = cfg["weight_copies"]
    host = [synth.q4_weights(n, k, GROUP, 1, tag=(k, n)) for (k, n) in SWEEP]
    sets = [[(p.copy(), s.astype(np.float32)) for p, s in host] for _ in range(copies)]
    xs = [synth.activations(k, 1, tag=(k, n)).astype(np.float32) for (k, n) in SWEEP]

    def step(c):
        for (p, s), x, (k, n) in zip(sets[c], xs, SWEEP):
            O.gemm(x, 4, p, s, GROUP, n)

    for i in range(args.warmup):
        step(i % copies)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(i % copies)
    el = time.perf_counter() - t0
    value = args.steps * STEP_BYTES / el / 1e9
    line = {"impl": "reference", "metric": "Q4 g32 dequant-GEMV sweep, algorithmic HBM GB/s (batch 1)",
            "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int4 weights, fp16 act/scales, fp32 accumulate",
            "data": "synthetic (seeded PCG64; BASELINE config 2 shapes and distributions)",
            "config": cfg,
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": O.num_threads(), "kind": "port",
                             "sample": f"{args.steps} full sweep passes through the C++ oracle (sequential fp32 per"
                                       f" output, OpenMP over outputs), weights rotated over {copies} host copies"},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=30)
    ap.add_argument("--impl", choices=["aexis", "reference"], default="aexis")
    ap.add_argument("--skip-decoder", action="store_true", help="omit the config-3 decoder measurement")
    ap.add_argument("--skip-cpu", action="store_true", help="omit the CPU oracle baseline")
    ap.add_argument("--skip-config5", action="store_true", help="omit the config-5 lm_head measurement")
    ap.add_argument("--skip-config4", action="store_true", help="omit the config-4 batched decoder measurement")
    ap.add_argument("--skip-sampler", action="store_true", help="omit the device sampler measurement")
    ap.add_argument("--skip-w8a8", action="store_true", help="omit the W8A8 GEMV/GEMM measurement")
    ap.add_argument("--skip-linear-attention", action="store_true",
                    help="omit the GatedDeltaRule / ShortConv decode measurement")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--only", choices=["dominant", "decoder", "hybrid", "tcgemm", "config4", "topk", "linear_attention", "sampler", "w8a8"], help="profiling mode (see run_only)")
    ap.add_argument("--prompt-len", type=int, default=512)
    ap.add_argument("--new-tokens", type=int, default=64)
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.only:
        run_only(args)
    elif args.impl == "reference":
        if args.steps > 20:
            args.steps = 20  # each reference step is a full CPU pass (~0.5 s); bound the run
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
