"""Per-kernel device time of one decoding step of config 5 (oumu_b200.engine.Engine, captured as one CUDA graph):
the kernels a step launches, how often, and their share of the step.

    python tests/perf_step_kernels.py [--takes 32] [--steps 3] [--lm-tc qkv,o,gu,down]
        torch profiler (CUDA activity) over `steps` graph replays: one line per kernel name.
    ncu --profile-from-start off --metrics gpu__time_duration.sum --clock-control none --csv \\
        --log-file launches.csv python tests/perf_step_kernels.py --ncu
        one replay between cudaProfilerStart / cudaProfilerStop, for an ncu launch list of exactly one step.
"""
import argparse
import collections
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

from oumu_b200 import engine, synth  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--takes", type=int, default=32)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--ncu", action="store_true", help="one replay inside cudaProfilerStart/Stop, nothing printed")
    ap.add_argument("--lm-tc", default=None, help="LM projections on the library's GEMM (comma list; 'none': cuBLAS)")
    args = ap.parse_args()
    B = args.takes
    kw = {} if args.lm_tc is None else {"lm_tc": () if args.lm_tc == "none" else tuple(args.lm_tc.split(","))}
    e = engine.Engine(B, **kw)
    margin = 2 * (args.steps + 8)
    e.prime([int(v) for v in synth.uniform_int(synth.config_seed(5), B, 330, 4096 - margin)])
    g = e.capture()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    if args.ncu:
        torch.cuda.profiler.start()
        g.replay()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        return 0
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(args.steps):
            g.replay()
        torch.cuda.synchronize()
    evs = [ev for ev in prof.events() if ev.device_type == torch.autograd.DeviceType.CUDA]
    tot = collections.defaultdict(lambda: [0, 0.0])
    for ev in evs:
        t = tot[ev.name[:100]]
        t[0] += 1
        t[1] += ev.device_time_total
    busy = sum(v[1] for v in tot.values()) / args.steps
    print(f"takes {B}: {sum(v[0] for v in tot.values()) / args.steps:.0f} kernels per step, "
          f"{busy / 1e3:.3f} ms of kernel time per step")
    for k, (n, t) in sorted(tot.items(), key=lambda kv: -kv[1][1]):
        print(f"{t / args.steps / 1e3:8.3f} ms {n / args.steps:5.0f}x {t / n:8.2f} us  {100 * t / args.steps / busy:5.1f} %"
              f"  {k}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
