"""Runs one workload for profiling: load, prefill, then a few device-timed steps.

    python -m qwenscriber_b200.probe [--workload NAME] [--steps K]

Single-stream workloads prefill with qwc_decode_begin and time K greedy
steps of the persistent decode kernel (qwc_decode_run_timed); multi-stream
workloads begin every slot (tensor-core prefill) and time K batched steps
(qwc_streams_run_timed). Prints the device time and the kernels launched
before the timed steps, which is the skip count a profiler needs to land on
them.
"""

from __future__ import annotations

import argparse
import sys

from . import runtime as rt
from . import synthetic


def main(argv=None) -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--workload", default="cfg3_1p7b_q4_s64")
    p.add_argument("--steps", type=int, default=1)
    p.add_argument("--chunk", type=int, default=16, help="decode steps per launch (single stream)")
    p.add_argument("--streams", type=int, default=0, help="override the workload's streams per GPU")
    a = p.parse_args(argv)
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
        gm.decode_begin(pr.tokens, pr.audio, a.steps + 1)
        before = gm.launches()
        ms = gm.run_timed(a.steps)
        tokens = a.steps
    print(f"{w.name}: {a.steps} steps, {ms / a.steps:.3f} ms/step, {tokens / (ms / 1000.0):.0f} tokens/s; "
          f"kernels before the timed steps: {before}")
    gm.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
