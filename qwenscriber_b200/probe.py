"""Runs one workload for profiling: load, prefill, then a few device-timed steps.

    python -m qwenscriber_b200.probe [--workload NAME] [--steps K]
    python -m qwenscriber_b200.probe --gemm ROWS COLS [--steps K]
    python -m qwenscriber_b200.probe --workload cfg2_1p7b_q4_b1 --trace

--trace (single-stream workloads) runs one more launch with the phase
timeline on (QWC_OPTION_TRACE) and prints, per stage of a layer, the mean
time from the previous barrier to the stage's input being ready, the compute
time, and the grid-barrier wait, over CTAs and the middle layers.

Single-stream workloads prefill with qwc_decode_begin and time K greedy
steps of the persistent decode kernel (qwc_decode_run_timed); multi-stream
workloads begin every slot (tensor-core prefill) and time K batched steps
(qwc_streams_run_timed). Prints the device time and the kernels launched
before the timed steps, which is the skip count a profiler needs to land on
them.

--gemm times K calls of qwc_op_gemm_streams on a random q4 matrix of ROWS x
COLS against 64 stream columns, after 3 untimed calls: each call launches the
activation packing, the GEMM and the split-K sum; a profiler filtered on
gemm_streams_kernel skips 3 launches to land on the first timed one.
"""

from __future__ import annotations

import argparse
import sys

from . import quant
from . import runtime as rt
from . import synthetic


def main(argv=None) -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--workload", default="cfg3_1p7b_q4_s64")
    p.add_argument("--steps", type=int, default=1)
    p.add_argument("--chunk", type=int, default=16, help="decode steps per launch (single stream)")
    p.add_argument("--streams", type=int, default=0, help="override the workload's streams per GPU")
    p.add_argument("--gemm", type=int, nargs=2, metavar=("ROWS", "COLS"), help="time the stream GEMM op alone")
    p.add_argument("--trace", action="store_true", help="print the per-stage timeline of one decode launch")
    a = p.parse_args(argv)
    if a.gemm:
        return gemm(*a.gemm, a.steps)
    w = synthetic.workloads()[a.workload]
    if a.streams:
        import dataclasses

        w = dataclasses.replace(w, streams=a.streams)
    model = synthetic.make_model(w.config, w.fmt, w.seed)
    gm = rt.CudaModel(0)
    synthetic.load_into(model, gm, cache_format=rt.CACHE_Q8, streams=w.streams)
    gm.set_option(rt.OPTION_IGNORE_EOS, 1)
    gm.set_option(rt.OPTION_STEP_CHUNK, a.chunk)
    if w.streams > 1:
        lengths = synthetic.prefix_lengths(w)
        for s in range(w.streams):
            pr = synthetic.make_prompt(w.config, lengths[s], w.text_ids, w.seed, stream=s)
            gm.stream_begin(s, pr.tokens, pr.audio, w.decode)
        before = gm.launches()
        ms = gm.streams_run_timed(a.steps)
        tokens = a.steps * w.streams
    else:
        pr = synthetic.make_prompt(w.config, w.audio_rows, w.text_ids, w.seed)
        gm.decode_begin(pr.tokens, pr.audio, a.steps + 1 + (min(a.chunk, 8) if a.trace else 0))
        before = gm.launches()
        ms = gm.run_timed(a.steps)
        tokens = a.steps
    print(f"{w.name}: {a.steps} steps, {ms / a.steps:.3f} ms/step, {tokens / (ms / 1000.0):.0f} tokens/s; "
          f"kernels before the timed steps: {before}")
    if a.trace and w.streams <= 1:
        gm.set_option(rt.OPTION_TRACE, 1)
        gm.run_timed(min(a.chunk, 8))
        print_trace(gm.debug_trace(), w.config.text_layers)
    gm.close()
    return 0


STAGES = ("qkv", "attention", "o", "gate", "up", "down")


def print_trace(raw, layers: int) -> None:
    """Per-stage means of the decode kernel's phase timeline (three stamps per
    stage: input ready, output done, barrier passed), over CTAs and layers
    1 .. layers - 2, in microseconds; brackets hold the mean over layers of
    the slowest CTA."""
    import numpy as np

    tr = raw.reshape(-1, 512).astype(np.int64)
    ev = (tr - tr[:, 0].min()) / 1000.0
    per = len(STAGES)
    print(f"{'stage':10s} {'input':>16s} {'compute':>16s} {'barrier':>16s}")
    for si, name in enumerate(STAGES):
        cols = []
        for k in range(3):
            means, maxes = [], []
            for layer in range(1, layers - 1):
                q = layer * per + si
                stamps = [ev[:, q * 3 - 1], ev[:, q * 3], ev[:, q * 3 + 1], ev[:, q * 3 + 2]]
                d = stamps[k + 1] - stamps[k]
                means.append(d.mean())
                maxes.append(d.max())
            cols.append(f"{np.mean(means):6.2f} [{np.mean(maxes):6.2f}]")
        print(f"{name:10s} " + " ".join(f"{c:>16s}" for c in cols))
    span = [ev[:, (layer + 1) * per * 3 - 1].max() - ev[:, layer * per * 3 - 1].max() for layer in range(1, layers - 1)]
    q = layers * per
    lm = [(ev[:, q * 3 + k] - ev[:, q * 3 + k - 1]).mean() for k in range(3)]
    print(f"layer {np.mean(span):.2f} us; lm_head input {lm[0]:.2f} compute {lm[1]:.2f} barrier {lm[2]:.2f} us; "
          f"per token and CTA: tiles in hand {tr[:, 509].mean() / 1000:.1f} us, waiting for tiles "
          f"{tr[:, 510].mean() / 1000:.1f} us, at grid barriers {tr[:, 511].mean() / 1000:.1f} us")


def gemm(rows: int, cols: int, reps: int) -> int:
    import numpy as np
    import torch

    L = rt.lib()
    rng = np.random.default_rng(0)
    groups = cols // 64
    scales = torch.from_numpy((np.abs(rng.standard_normal((rows, groups))) * 0.003).astype(np.float16)
                              .view(np.uint16)).cuda()
    codes = torch.from_numpy(rng.integers(0, 256, size=(rows, groups * 32), dtype=np.uint8)).cuda()
    x = torch.randn(64, cols, device="cuda")
    out = torch.zeros(64, rows, device="cuda")

    def call():
        rt.check(L.qwc_op_gemm_streams(quant.Q4, scales.data_ptr(), codes.data_ptr(), rows, cols,
                                       x.data_ptr(), 64, out.data_ptr(), None), "qwc_op_gemm_streams")

    for _ in range(3):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        call()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / reps
    print(f"stream gemm q4 {rows} x {cols}, 64 columns: {us:.1f} us per op call (packing + GEMM + split-K sum)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
