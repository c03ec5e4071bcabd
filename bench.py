"""Benchmark of the decoder token loop: greedy decode tokens/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

A step is one greedy decode step of the workload's stream (one token through
28 layers, the tied lm_head and the argmax). The default workload is
configs[2] of the benchmark definition: Qwen3-ASR-1.7B decoder, q4 weights
(seed 1), 375 N(0,1) audio rows + 16 text ids, q8 KV cache, 448 greedy tokens
(W + K = 448 by default). Weights (0.91 GB) exceed the 126 MB L2, so no flush
is needed between steps.

The same line carries a `streams64` object: configs[3] of the benchmark
definition, 64 independent streams per GPU of the same model (prefixes
uniform in [100, 1500] audio rows + 16 text ids, each prefilled on the tensor
cores when its slot begins), timed over greedy steps of all 64 slots with the
batched tensor-core step, with its own roofline and end-to-end figures.

Under torchrun (N > 1) every rank holds a full weight replica and decodes its
own independent streams (streams shard across GPUs with no exchange): value =
tokens of all ranks / the slowest rank's device time.

`--impl reference` times the CPU restatement of the reference's Zig decode
path (oracle/, the reference itself cannot be built here: no Zig toolchain)
on the host cores, on a bounded sample of the same workload.
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tokens/s, 1.7B q4, 1 & 64 streams/GPU at 1/2/4/8 GPU; % of HBM roofline"
KV_BYTES_PER_POSITION = 28 * 2 * (1024 + 1024 // 64 * 2)  # all layers, K and V, q8 codes + f16 scales
# DRAM bytes (read + write) per decoded token of decode_kernel at cfg2, from one
# ncu capture of a 16-token launch (dram__bytes_read.sum 15.058 GB +
# dram__bytes_write.sum 29.3 MB, divided by 16 tokens).
DECODE_TRAFFIC_PER_TOKEN = (15.058409e9 + 29.326592e6) / 16


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=440)
    p.add_argument("--warmup", type=int, default=8)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", default="cfg2_1p7b_q4_b1")
    p.add_argument("--chunk", type=int, default=64, help="decode steps per device launch")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--streams-workload", default="cfg3_1p7b_q4_s64",
                   help="multi-stream workload measured beside the main one ('none' to skip)")
    p.add_argument("--streams-steps", type=int, default=200)
    return p.parse_args()


def algorithmic_bytes(model, first_position: int, steps: int) -> float:
    """Bytes one greedy step must move, summed over `steps` steps starting at
    `first_position`: every weight payload once (the tied embedding once, as
    the lm_head), one embedding row, the norm vectors, the q8 KV rows read
    (position + 1 rows) and the row written."""
    c = model.config
    weights = sum(t.payload.nbytes for t in model.tensors if t.fmt != 0)
    norms = sum(t.payload.nbytes for t in model.tensors if t.fmt == 0)
    embed_row = c.text_hidden_size // 64 * (2 + (32 if model.fmt == 16 else 64))
    per_pos = c.text_layers * 2 * (c.kv_width + c.kv_width // 64 * 2)
    total = 0.0
    for i in range(steps):
        p = first_position + i
        total += weights + norms + embed_row + (p + 1) * per_pos + per_pos
    return total


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.device)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peak() -> tuple[float, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def config_block(w, args, world):
    return {"workload": w.name, "model": "Qwen3-ASR-1.7B decoder" if w.config.text_hidden_size == 2048
            else "Qwen3-ASR-0.6B decoder", "weights": "q4" if w.fmt == 16 else "q8", "kv_cache": "q8",
            "streams_per_gpu": w.streams, "prompt": f"{w.audio_rows} audio rows + {w.text_ids} text ids",
            "decode_tokens": args.warmup + args.steps, "l2": "weights 0.91 GB > 126 MB L2 (no flush needed)",
            "parallelism": f"stream-replicas x{world}"}


def oracle_decode_rate(model, prompt, threads: int, budget_s: float = 20.0, max_steps: int = 64):
    """Times the CPU port's greedy steps on a bounded sample: prefill of the
    prompt's text ids only, then decode steps until `budget_s` has passed."""
    import oracle as O
    from tests.parity import oracle_model

    om = oracle_model(model, threads=threads)
    c = model.config
    text = prompt.tokens[prompt.tokens != c.token_audio_pad][:8]
    nxt = om.prefill(text, np.zeros((0, c.text_hidden_size), np.float32), 0)
    t0 = time.perf_counter()
    steps = 0
    while steps < max_steps and (steps < 2 or time.perf_counter() - t0 < budget_s):
        nxt = om.step(nxt)
        steps += 1
    dt = time.perf_counter() - t0
    om.close()
    del O
    return steps / dt, steps, dt, len(text)


def run_reference(args, rank):
    from qwenscriber_b200 import synthetic

    if rank != 0:
        return
    w = synthetic.workloads()[args.workload]
    model = synthetic.make_model(w.config, w.fmt, w.seed)
    prompt = synthetic.make_prompt(w.config, w.audio_rows if isinstance(w.audio_rows, int) else w.audio_rows[0],
                                   w.text_ids, w.seed)
    threads = os.cpu_count() or 1
    rate, steps, dt, pre = oracle_decode_rate(model, prompt, threads, budget_s=60.0, max_steps=max(2, args.steps))
    sample = (f"{steps} greedy steps after a {pre}-token text prefill (positions {pre}..{pre + steps - 1}; the "
              f"workload decodes at positions ~{w.audio_rows}+: attention is <3% of a step's bytes), {dt:.1f} s")
    line = {"metric": METRIC, "value": rate, "unit": "tokens/s", "n_gpus": args.gpus, "steps": steps,
            "warmup": 0, "ms_per_step": 1000.0 / rate, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": config_block(w, args, 1),
            "cpu_baseline": {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": rate, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "CPU restatement of the reference's Zig decode path (oracle/); the Zig reference cannot be "
                    "built here (no zig toolchain)"}
    print(json.dumps(line), flush=True)


def streams_bytes(model, positions: list[int], steps: int) -> float:
    """Algorithmic bytes of `steps` batched steps: every weight payload once
    per step (shared by all slots), the norm vectors, and per slot its
    embedding row, its (position + 1) q8 KV rows read and the row written."""
    c = model.config
    weights = sum(t.payload.nbytes for t in model.tensors if t.fmt != 0)
    norms = sum(t.payload.nbytes for t in model.tensors if t.fmt == 0)
    embed_row = c.text_hidden_size // 64 * (2 + (32 if model.fmt == 16 else 64))
    per_pos = c.text_layers * 2 * (c.kv_width + c.kv_width // 64 * 2)
    total = 0.0
    for i in range(steps):
        total += weights + norms
        for p0 in positions:
            p = p0 + i
            total += embed_row + (p + 1) * per_pos + per_pos
    return total


def measure_streams(args, model, w, rank, local_rank, barrier, world):
    """The multi-stream workload on this rank's GPU: every slot's prompt is
    prefilled at qwc_stream_begin, then `streams_steps` greedy steps of all
    slots are timed on the device (qwc_streams_run_timed), then 32 steps
    through qwc_streams_step (host buffers each step) for the end-to-end figure."""
    import dataclasses

    import torch

    from qwenscriber_b200 import runtime as rt
    from qwenscriber_b200 import shards, synthetic

    m = dataclasses.replace(model, config=w.config)
    gm = rt.CudaModel(local_rank)
    synthetic.load_into(m, gm, cache_format=rt.CACHE_Q8, streams=w.streams)
    gm.set_option(rt.OPTION_IGNORE_EOS, 1)
    # This rank's global streams (shards.shard): their own prefix lengths and prompts.
    lengths = synthetic.prefix_lengths(w, world, rank)
    ids = shards.shard(w.streams * world, world, rank)
    prompts = [synthetic.make_prompt(w.config, lengths[s], w.text_ids, w.seed, stream=ids[s])
               for s in range(w.streams)]
    plen = [len(p.tokens) for p in prompts]
    warm, e2e_steps = 4, 32
    steps = min(args.streams_steps, w.decode - 1 - warm - e2e_steps)
    t0 = time.perf_counter()
    for s in range(w.streams):  # each prompt prefilled on the tensor cores, 64 positions per step
        gm.stream_begin(s, prompts[s].tokens, prompts[s].audio, w.decode)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    gm.streams_run_timed(warm)
    positions = [plen[s] + warm for s in range(w.streams)]
    barrier()
    launches0 = gm.launches()
    with ClockSampler(local_rank) as clocks:
        ms = gm.streams_run_timed(steps)
    launches = gm.launches() - launches0
    barrier()
    ms = shards.max_over_ranks(ms)
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        gm.streams_step(w.streams)
    e2e_s = time.perf_counter() - t0
    barrier()
    e2e_s = shards.max_over_ranks(e2e_s)
    gm.close()
    tokens = steps * w.streams * world
    bytes_total = streams_bytes(m, positions, steps)
    peak, peak_kind = measured_peak()
    achieved = bytes_total / (ms / 1000.0) / 1e9
    return {
        "workload": w.name, "streams_per_gpu": w.streams,
        "value": shards.aggregate_rate(steps * w.streams, world, ms / 1000.0), "unit": "tokens/s",
        "ms_per_step": ms / steps, "steps": steps, "warmup": warm,
        "prompt": f"{w.text_ids} text ids after U[{w.audio_rows[0]}, {w.audio_rows[1]}] audio rows per stream "
                  f"({sum(plen)} prompt positions in all, prefilled in {prefill_s:.2f} s, 64 positions per "
                  f"tensor-core step)",
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_kind": peak_kind, "bytes_per_step": bytes_total / steps},
        "e2e": {"value": shards.aggregate_rate(e2e_steps * w.streams, world, e2e_s), "unit": "tokens/s",
                "h2d_bytes_per_step": 64 * 16, "d2h_bytes_per_step": 64 * 4 + 16,
                "includes": "qwc_streams_step: slot descriptors up, one graph replay, tokens down, per step"},
        "gpu_launches": launches, "clocks": clocks.summary(),
    }


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from qwenscriber_b200 import runtime as rt
    from qwenscriber_b200 import shards, synthetic

    torch.cuda.set_device(local_rank)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=torch.device(
            "cuda", local_rank))
    w = synthetic.workloads()[args.workload]
    model = synthetic.make_model(w.config, w.fmt, w.seed)
    rows = w.audio_rows if isinstance(w.audio_rows, int) else w.audio_rows[0]
    prompt = synthetic.make_prompt(w.config, rows, w.text_ids, w.seed, stream=rank)
    gm = rt.CudaModel(local_rank)
    synthetic.load_into(model, gm, cache_format=rt.CACHE_Q8)
    gm.set_option(rt.OPTION_IGNORE_EOS, 1)
    gm.set_option(rt.OPTION_STEP_CHUNK, args.chunk)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- device-timed decode (inputs resident in HBM) ----
    gm.decode_begin(prompt.tokens, prompt.audio, args.warmup + args.steps + 1)
    gm.run_timed(args.warmup)
    first_position = len(prompt.tokens) + args.warmup
    barrier()
    launches0 = gm.launches()
    with ClockSampler(local_rank) as clocks:
        ms = gm.run_timed(args.steps)
    launches = gm.launches() - launches0
    barrier()
    ms = shards.max_over_ranks(ms)
    gm.decode_end()

    # ---- end to end through the public API: prompt upload + prefill + K steps, tokens read each step ----
    barrier()
    t0 = time.perf_counter()
    gm.decode_begin(prompt.tokens, prompt.audio, args.steps + 1)
    for _ in range(args.steps):
        gm.decode_step()
    e2e_s = time.perf_counter() - t0
    gm.decode_end()
    barrier()
    e2e_s = shards.max_over_ranks(e2e_s)

    streams = None
    if args.streams_workload != "none":
        streams = measure_streams(args, model, synthetic.workloads()[args.streams_workload], rank, local_rank,
                                  barrier, world)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        rate, steps, dt, pre = oracle_decode_rate(model, prompt, threads, budget_s=20.0, max_steps=64)
        cpu = {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample": f"{steps} greedy steps of the same model after a {pre}-token text prefill, {dt:.1f} s"}

    if rank == 0:
        tokens = args.steps * world
        value = shards.aggregate_rate(args.steps, world, ms / 1000.0)
        bytes_total = algorithmic_bytes(model, first_position, args.steps)
        peak, peak_kind = measured_peak()
        achieved = bytes_total / (ms / 1000.0) / 1e9
        h2d = (prompt.tokens.nbytes + prompt.audio.nbytes) / args.steps
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32 (q4 codes dequantized exactly in registers)", "data": "synthetic",
            "config": config_block(w, args, world),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind,
                         "traffic": DECODE_TRAFFIC_PER_TOKEN if args.workload == "cfg2_1p7b_q4_b1" else None,
                         "traffic_unit": "bytes per step, from an ncu capture of decode_kernel at cfg2",
                         "bytes_per_step": bytes_total / args.steps,
                         "kernel": "decode_kernel (persistent, one launch per %d steps)" % args.chunk},
            "e2e": {"value": shards.aggregate_rate(args.steps, world, e2e_s), "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
                    "includes": "prompt upload + prefill of %d positions + %d decode steps via qwc_decode_step"
                                % (len(prompt.tokens), args.steps)},
            "gpu_launches": launches,
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
            "streams64": streams,
        }
        print(json.dumps(line), flush=True)
    gm.close()
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
