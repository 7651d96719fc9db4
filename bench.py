#!/usr/bin/env python
"""Benchmark of the attention hot path on the configuration BASELINE's metric is quoted on (config 2):
decode attention of 28 layers x 64 takes per GPU, 16 q / 2 kv heads, hd 128, bf16 KV slots of 4096 positions,
per-take lengths uniform in [330, 4096], one query per take per layer, all layers in one captured CUDA graph.

One step = for each of the 28 layers, one launch of the fused decode layer: rope of q/k at each take's position, k/v
written into the take's slot, and the split-KV decode attention with the combine fused in.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

For N > 1 it runs under torchrun, one rank per GPU; every rank owns its own 64 takes (takes are independent,
no collective on the data path), so scaling is weak: N x 64 lengths are drawn from the seed and dealt out so that
every GPU holds about the same KV bytes. Rank 0 prints one JSON line.
--impl reference times the reference algorithm's CPU restatement (oracle/, all host threads) on the same workload.
"""
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

METRIC = "decode-attn HBM GB/s (% of 8 TB/s) at 64 takes×KV4096; patches/sec at 1/2/4/8 B200"
NQ, NK, HD, MAXLEN, LAYERS, TAKES = 16, 2, 128, 4096, 28, 64
LEN_LO, LEN_HI = 330, 4096
NOMINAL_HBM_GBS = 8000.0
WORKLOAD = ("config 2: decode attention, 28 layers x 64 takes per GPU, 16 q / 2 kv heads, hd 128, bf16 KV slots "
            "of 4096, per-take lengths U[330,4096], one query per take per layer, one CUDA graph per step")


# The JSON line is the only thing on standard output: everything else (NCCL's banner, library messages) is sent to
# standard error by pointing file descriptor 1 there, and the line is written to the original standard output.
_STDOUT_FD = None


def quiet_stdout():
    global _STDOUT_FD
    if _STDOUT_FD is None:
        sys.stdout.flush()
        _STDOUT_FD = os.dup(1)
        os.dup2(2, 1)


def emit(line):
    sys.stdout.flush()
    data = (json.dumps(line) + "\n").encode()
    os.write(_STDOUT_FD if _STDOUT_FD is not None else 1, data)


def shard_lengths(seed, per_rank, world, rank, lo, hi):
    """This rank's per_rank take lengths: world * per_rank lengths drawn from the seed (the first per_rank of them are
    the one-GPU draw), dealt out longest first to the rank with the fewest cached positions so far, each rank taking
    per_rank takes, as a host placing takes on GPUs balances their KV bytes. Kept in draw order. (Independent draws
    per rank differed by up to 18 % in bytes, and the max-over-ranks time then measured that imbalance.)"""
    from oumu_b200 import synth
    allv = [int(v) for v in synth.uniform_int(seed, world * per_rank, lo, hi)]
    if world == 1:
        return allv
    load, mine = [0] * world, [[] for _ in range(world)]
    for i in sorted(range(len(allv)), key=lambda i: (-allv[i], i)):
        r = min((q for q in range(world) if len(mine[q]) < per_rank), key=lambda q: (load[q], q))
        mine[r].append(i)
        load[r] += allv[i]
    return [allv[i] for i in sorted(mine[rank])]


def take_lengths(rank, world=1):
    return shard_lengths(0x5EED + 1, TAKES, world, rank, LEN_LO, LEN_HI)


def bytes_per_layer(lens):
    """Algorithmic bytes of one layer's decode attention: K and V of the L_s valid positions of each take, its
    q heads read and its output written (2*nk*L*hd*2 + 2*nq*hd*2 per take)."""
    return int(sum(2 * NK * int(L) * HD * 2 + 2 * NQ * HD * 2 for L in lens))


def rank_reduce(x, op, dist=None, device="cpu"):
    """x reduced over the ranks of the default process group (op "max" for device times, "sum" for bytes);
    x itself without a group. Every rank must call it at the same point."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return x
    import torch
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def committed_traffic():
    """DRAM bytes per attention launch from the committed ncu summary (profiles/), scaled to one full launch."""
    p = os.path.join(ROOT, "profiles", "decode_attn_config2.md")
    try:
        for line in open(p):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":")[1])
    except OSError:
        pass
    return None


class ClockSampler:
    """SM clock and clock-event reasons sampled with NVML every 10 ms while active (read-only queries)."""

    REASONS = {0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x4: "sw_power_cap",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, index):
        self.samples, self.reasons, self.ok = [], set(), False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            uuid = None
            try:
                import torch
                uuid = "GPU-" + str(torch.cuda.get_device_properties(index).uuid)
            except Exception:
                pass
            self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid) if uuid else pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # no NVML: the line says so
            self.err = str(e)

    def sample(self):
        nv = self.nv
        try:
            self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
            r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            for bit, name in self.REASONS.items():
                if r & bit:
                    self.reasons.add(name)
        except Exception:
            pass

    def _run(self):
        while not self.stop:
            self.sample()
            time.sleep(0.01)

    def __enter__(self):
        # one sample on entry and one on exit in the caller's thread (a short timed region can end before the
        # sampling thread gets scheduled), the thread's in between
        if self.ok:
            self.sample()
            self.stop = False
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self.sample()
            self.stop = True
            self.t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": getattr(self, "err", "no samples")}
        return {"sm_mhz": float(statistics.median(self.samples)), "sm_max_mhz": float(self.max_mhz),
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ------------------------------------------------------------------------------------------------------------
# CPU leg: the reference algorithm's fp32 restatement (oracle/) on the host cores
# ------------------------------------------------------------------------------------------------------------

def cpu_inputs(lens, layers, seed):
    from oumu_b200 import synth
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(layers):
        qkv = synth.f32_to_bf16(rng.standard_normal((TAKES, (NQ + 2 * NK) * HD), dtype=np.float32))
        kc = np.zeros((TAKES, NK, MAXLEN, HD), np.uint16)
        vc = np.zeros_like(kc)
        for s, L in enumerate(lens):  # only the valid positions are read
            kc[s, :, :L] = synth.f32_to_bf16(rng.standard_normal((NK, L, HD), dtype=np.float32))
            vc[s, :, :L] = synth.f32_to_bf16(rng.standard_normal((NK, L, HD), dtype=np.float32))
        out.append((qkv, kc, vc))
    return out


def host_threads():
    """Host threads this process may run on. The oracle's OpenMP pool is set to it explicitly: torchrun exports
    OMP_NUM_THREADS=1 to every rank, which would otherwise leave the CPU evaluation on one thread."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_time(lens, layers, min_seconds):
    """Times the oracle's decode attention over `layers` layers of the workload until min_seconds have passed;
    returns (GB/s, threads, seconds, sample description)."""
    from oracle import cpu
    cpu.set_threads(host_threads())
    data = cpu_inputs(lens, layers, 7)
    ln = np.asarray(lens, np.int32)
    nbytes, reps, t0 = 0, 0, time.perf_counter()
    while True:
        for qkv, kc, vc in data:
            cpu.attn_decode(qkv, kc, vc, None, ln, TAKES, NQ, NK, HD, MAXLEN, HD ** -0.5)
            nbytes += bytes_per_layer(lens)
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= min_seconds:
            break
    return nbytes / dt / 1e9, cpu.threads(), dt, f"{reps} x {layers} layer(s) x {TAKES} takes of config 2"


def reference_arm(args, rank, world):
    if rank != 0:
        return 0
    from oracle import cpu
    cpu.set_threads(host_threads())
    lens = take_lengths(0)
    data = cpu_inputs(lens, 1, 7)
    qkv, kc, vc = data[0]
    ln = np.asarray(lens, np.int32)
    group = 8  # takes per step: each step is a bounded sample of the workload, rotating over the 64 takes

    def one(i):
        s0 = (i * group) % TAKES
        sl = slice(s0, s0 + group)
        cpu.attn_decode(qkv[sl], kc[sl], vc[sl], None, ln[sl], group, NQ, NK, HD, MAXLEN, HD ** -0.5)
        return bytes_per_layer(lens[sl])

    for i in range(args.warmup):
        one(i)
    nbytes, t0 = 0, time.perf_counter()
    for i in range(args.steps):
        nbytes += one(args.warmup + i)
    dt = time.perf_counter() - t0
    gbs = nbytes / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * dt / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) bf16 q/k/v, per-take lengths U[330,4096])",
        "config": {"workload": WORKLOAD, "takes_per_gpu": TAKES, "layers": LAYERS, "maxlen": MAXLEN,
                   "same_config": False,
                   "sampled": f"a rate measured on a sample of the workload: each step is one layer of {group} of "
                              f"the {TAKES} takes (rotating over them) on rank 0's host; GB/s of that sample"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cpu.threads(), "kind": "port",
                         "sample": f"each step: one layer of {group} of the 64 takes (rotating), fp32 C "
                                   "restatement of kernels/voxcpm.cu:131-185 (OpenMP, all host threads)"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference implements this path only as CUDA kernels; its CPU form is the oracle port",
    }
    emit(line)
    return 0


# ------------------------------------------------------------------------------------------------------------
# GPU arm
# ------------------------------------------------------------------------------------------------------------

STEP_TAKES = 32
STEP_WORKLOAD = ("config 5: random-init VoxCPM2-shaped decoding step per GPU, one CUDA graph: 9 DiT passes "
                 "(10 timesteps, CFG 2.0, 4 layers) -> local encoder (4 layers) -> base LM (28 layers, hidden 2048, "
                 "SwiGLU 6144) -> FSQ -> residual LM (8 layers); KV slots of 4096, lengths U[330, 4096)")


def patches_leg(args, dev, rank, max_over_ranks, sum_over_ranks, barrier, world=1):
    """Config 5: the whole decoding step (oumu_b200.engine) for --step-takes takes per GPU, as one CUDA graph;
    patches/s over all ranks, device-resident and end to end (the step's noise uploaded from pinned host memory,
    the new patch and the stop flags read back and waited for every step, as Engine::decode reads `stop`,
    src/model.rs:785-794)."""
    import torch
    from oumu_b200 import engine, synth
    B, K, W = args.step_takes, args.step_steps, max(3, min(args.warmup, 5))
    margin = 2 * (K + W) + 4  # every replay advances every take by one position; lengths reset between legs
    lens = shard_lengths(synth.config_seed(5), B, world, rank, LEN_LO, MAXLEN - margin)
    e = engine.Engine(B, maxlen=MAXLEN, max_steps=4 * (K + W) + 8, device=dev)
    e.prime(lens, seed=5 + rank)
    from oumu_b200 import _lib
    c0 = _lib.CALLS[0]
    graph = e.capture()  # one eager step + the capture: each of this library's launches is called twice
    launches = (_lib.CALLS[0] - c0) // 2

    local = []  # this rank's own times, for the per-rank record

    def timed(fn):
        e.set_lens(lens)
        for _ in range(W):
            fn()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(K):
            fn()
        b.record()
        torch.cuda.synchronize()
        local.append(a.elapsed_time(b) / K)
        return max_over_ranks(a.elapsed_time(b))

    ms = timed(graph.replay)
    noise_host = torch.empty((B, engine.PATCH), dtype=torch.bfloat16).pin_memory()
    noise_host.normal_()
    patch_host = torch.empty((B, engine.PATCH), dtype=torch.bfloat16).pin_memory()
    stop_host = torch.empty((B,), dtype=torch.int32).pin_memory()
    stream = torch.cuda.current_stream()

    def e2e_step():
        e.noise.copy_(noise_host, non_blocking=True)
        graph.replay()
        patch_host.copy_(e.cond, non_blocking=True)  # cond holds this step's patch after the step
        stop_host.copy_(e.stop, non_blocking=True)
        stream.synchronize()

    e2e_ms = timed(e2e_step)
    patches = sum_over_ranks(B * K)
    # after the timed region: every rank's finished patches and stop steps to every rank, the sharded decode's one
    # collective (once per text)
    gathered = None
    if world > 1:
        gp, gs = engine.gather_patches(e.patches, e.stop)
        torch.cuda.synchronize()
        gathered = {"takes": int(gp.shape[0]), "bytes_per_rank": int(e.patches.numel() * 2 + e.stop.numel() * 4)}
    kv = 2 * 2 * 128 * 2 * (len(e.base.layers) + len(e.res.layers)) * int(sum(int(v) + W + K // 2 for v in lens))
    wbytes = e.step_weight_bytes()
    flops = e.step_flops()
    del graph
    return {
        "value": round(patches / (ms / 1e3), 1), "unit": "patches/s", "takes_per_gpu": B, "steps": K, "warmup": W,
        "ms_per_step": round(ms / K, 4), "workload": STEP_WORKLOAD, "scaling": "weak",
        "layers": {"base": len(e.base.layers), "residual": len(e.res.layers), "encoder": len(e.enc.layers),
                   "dit": len(e.dit.layers), "dit_passes": len(e.sched)},
        "per_step_per_gpu": {"weight_bytes": wbytes, "kv_bytes_mean": kv, "gemm_flops": flops},
        "e2e": {"value": round(patches / (e2e_ms / 1e3), 1), "unit": "patches/s",
                "h2d_bytes_per_step": noise_host.numel() * 2, "d2h_bytes_per_step": B * (engine.PATCH * 2 + 4),
                "ms_per_step": round(e2e_ms / K, 4),
                "path": "pinned host noise -> device, graph replay, patch + stop flags -> pinned host, host sync"},
        "gpu_launches_per_step": launches,
        "patches_gathered": gathered,
        "_local_ms_per_step": local,
    }

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-step", action="store_true", help="skip the end-to-end decoding-step leg (patches/s)")
    ap.add_argument("--step-takes", type=int, default=STEP_TAKES, help="takes per GPU of the decoding-step leg")
    ap.add_argument("--step-steps", type=int, default=30, help="timed decoding steps of the decoding-step leg")
    args = ap.parse_args()
    quiet_stdout()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        return reference_arm(args, rank, world)

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    from oumu_b200 import build, ops
    if rank == 0 or world == 1:
        build.build()
    if world > 1:
        dist.barrier()
    lens = take_lengths(rank, world)
    W = (NQ + 2 * NK) * HD
    gen = torch.Generator(device=dev)
    gen.manual_seed(0x5EED + 1 + rank)

    def rnd(*shape):
        return torch.randn(shape, generator=gen, device=dev, dtype=torch.float32).to(torch.bfloat16)

    qkv_all = rnd(LAYERS, TAKES, W)
    kc = [rnd(TAKES, NK, MAXLEN, HD) for _ in range(LAYERS)]
    vc = [rnd(TAKES, NK, MAXLEN, HD) for _ in range(LAYERS)]
    att_all = torch.zeros((LAYERS, TAKES, NQ * HD), dtype=torch.bfloat16, device=dev)
    cs, sn = ops.rotary_tables(MAXLEN, HD)
    cs, sn = cs.to(dev), sn.to(dev)
    ln = torch.tensor(lens, dtype=torch.int32, device=dev)
    ws = ops.decode_workspace(TAKES, NQ, NK, HD, MAXLEN, dev)
    per_layer = bytes_per_layer(lens)
    per_step = LAYERS * per_layer

    def step():
        for l in range(LAYERS):
            ops.step_tf_attention(qkv_all[l], kc[l], vc[l], att_all[l], ws, cs, sn, None, ln, TAKES, NQ, NK, HD,
                                  MAXLEN)

    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        step()  # eager once (first-use set-up outside the capture)
        # programmatic dependent launch between the step's kernels (the step writes no length and no cache
        # position below the newest one, the condition oumu_set_pdl states)
        ops.set_pdl(True)
        with torch.cuda.graph(graph, stream=stream):
            step()
        ops.set_pdl(False)
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        return rank_reduce(x, "max", dist if world > 1 else None, dev)

    def sum_over_ranks(x):
        return rank_reduce(x, "sum", dist if world > 1 else None, dev)

    def per_rank(vals):
        """Every rank's values (a list of floats of the same length on each rank), gathered to every rank."""
        if world == 1:
            return [list(vals)]
        t = torch.tensor([float(v) for v in vals], dtype=torch.float64, device=dev)
        out = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(out, t)
        return [[float(x) for x in o.tolist()] for o in out]

    # ---- device-resident timing ----
    t_end = time.perf_counter() + 0.3
    while time.perf_counter() < t_end:  # let the clocks settle (untimed)
        graph.replay()
        torch.cuda.synchronize()
    for _ in range(args.warmup):
        graph.replay()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        e0.record()
        for _ in range(args.steps):
            graph.replay()
        e1.record()
        clocks.sample()  # the replays are queued: the GPU is busy with them now
        torch.cuda.synchronize()
    ms_local = e0.elapsed_time(e1)
    ms = max_over_ranks(ms_local)
    barrier()
    total_bytes = sum_over_ranks(per_step * args.steps)
    value = total_bytes / (ms / 1e3) / 1e9

    # ---- dominant kernel: its mean duration per launch inside the timed region (the graph holds nothing else:
    #      LAYERS launches of the fused decode layer per step, CUDA events on the launching stream) ----
    launch_ms = ms / (args.steps * LAYERS)
    achieved = per_layer / (launch_ms / 1e3) / 1e9
    # and the same launches serialised, for reference: the step captured without programmatic dependent launch, so
    # each launch starts only once the one before it has completed and its ramp-up and tail overlap nothing. (Events
    # around eager launches would add the host's launch time whenever it exceeds a kernel's.)
    graph_ser = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph_ser, stream=stream):
            step()
    torch.cuda.current_stream().wait_stream(stream)
    reps = max(2, min(10, args.steps // 20))
    graph_ser.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        graph_ser.replay()
    b.record()
    torch.cuda.synchronize()
    del graph_ser
    kern_ms_local = a.elapsed_time(b) / (reps * LAYERS)
    kern_ms = max_over_ranks(kern_ms_local)
    peak, peak_kind = measured_peak()
    traffic = committed_traffic()

    # ---- end to end through the C ABI: host qkv in, host attention out, every step. As a serving loop runs it: two
    #      device buffer sets (one captured graph each), step i+1's inputs copied in and step i-1's outputs copied out
    #      on the copy engines while step i computes ----
    qkv_host = torch.empty_like(qkv_all, device="cpu").pin_memory()
    qkv_host.copy_(qkv_all)
    att_host = torch.empty_like(att_all, device="cpu").pin_memory()
    h2d, d2h = qkv_all.numel() * 2, att_all.numel() * 2
    qkv_b, att_b = [qkv_all, torch.empty_like(qkv_all)], [att_all, torch.empty_like(att_all)]
    graph2 = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        ops.set_pdl(True)
        with torch.cuda.graph(graph2, stream=stream):
            for l in range(LAYERS):
                ops.step_tf_attention(qkv_b[1][l], kc[l], vc[l], att_b[1][l], ws, cs, sn, None, ln, TAKES, NQ, NK,
                                      HD, MAXLEN)
        ops.set_pdl(False)
    torch.cuda.current_stream().wait_stream(stream)
    graphs = [graph, graph2]
    s_comp = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev = lambda: torch.cuda.Event()  # noqa: E731
    done_in, done_comp, done_out = [ev(), ev()], [ev(), ev()], [ev(), ev()]
    for b in range(2):  # every event recorded once, so the first waits pass
        for e in (done_in[b], done_comp[b], done_out[b]):
            e.record(s_comp)

    def e2e_steps(n):
        for i in range(n):
            b = i & 1
            s_in.wait_event(done_comp[b])            # step i-2 has read qkv_b[b]
            with torch.cuda.stream(s_in):
                qkv_b[b].copy_(qkv_host, non_blocking=True)
            done_in[b].record(s_in)
            s_comp.wait_event(done_in[b])
            s_comp.wait_event(done_out[b])           # step i-2's output has left att_b[b]
            graphs[b].replay()
            done_comp[b].record(s_comp)
            s_out.wait_event(done_comp[b])
            with torch.cuda.stream(s_out):
                att_host.copy_(att_b[b], non_blocking=True)
            done_out[b].record(s_out)
        s_comp.wait_stream(s_in)
        s_comp.wait_stream(s_out)

    e2e_steps(args.warmup)
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(s_comp)
    s_in.wait_event(f0)
    s_out.wait_event(f0)
    e2e_steps(args.steps)
    f1.record(s_comp)
    torch.cuda.synchronize()
    e2e_ms_local = f0.elapsed_time(f1)
    e2e_ms = max_over_ranks(e2e_ms_local)
    # the same loop serialised on one stream (copy in, step, copy out, in order), for comparison
    barrier()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record(s_comp)
    for _ in range(args.steps):
        qkv_b[0].copy_(qkv_host, non_blocking=True)
        graphs[0].replay()
        att_host.copy_(att_b[0], non_blocking=True)
    g1.record(s_comp)
    torch.cuda.synchronize()
    e2e_serial_ms = max_over_ranks(g0.elapsed_time(g1))
    del graph2
    e2e_value = total_bytes / (e2e_ms / 1e3) / 1e9
    errword = ops.device_error()
    barrier()

    step = None if args.no_step else patches_leg(args, dev, rank, max_over_ranks, sum_over_ranks, barrier, world)
    step_local = step.pop("_local_ms_per_step") if step else [0.0, 0.0]
    # per-rank record (the line's times are the max over ranks): which GPU sets them, and at what clock
    ck = clocks.summary()
    ranks = per_rank([ms_local / args.steps, ms_local / (args.steps * LAYERS), kern_ms_local,
                      e2e_ms_local / args.steps, ck["sm_mhz"] or 0.0, step_local[0], step_local[-1]])

    cpu_base = None
    if world == 1 and not args.no_cpu:
        gbs, thr, secs, sample = cpu_time(lens, 2, 10.0)
        cpu_base = {"value": round(gbs, 3), "unit": "GB/s", "cores": thr, "kind": "port",
                    "sample": f"{sample} ({secs:.1f} s), fp32 C restatement of kernels/voxcpm.cu:131-185"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) bf16 q/k/v, per-take lengths U[330,4096])",
            "config": {"workload": WORKLOAD, "takes_per_gpu": TAKES, "layers": LAYERS, "maxlen": MAXLEN,
                       "mean_len": float(np.mean(lens)), "bytes_per_step_per_gpu": per_step,
                       "l2": "inputs larger than L2 (3.7 GB of K/V per step per GPU)",
                       "parallelism": f"takes sharded over {world} GPU(s), no collective on the data path"},
            "pct_of_8TBps_per_gpu": round(100 * value / world / NOMINAL_HBM_GBS, 2),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "peak_kind": peak_kind, "kernel": "dec::k_attn_decode<128, fused>",
                         "kernel_ms": round(launch_ms, 5), "kernel_ms_alone": round(kern_ms, 5),
                         "algorithmic_bytes_per_launch": per_layer},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms / args.steps, 4),
                    "serialised_value": round(total_bytes / (e2e_serial_ms / 1e3) / 1e9, 2),
                    "serialised_ms_per_step": round(e2e_serial_ms / args.steps, 4),
                    "path": "pinned host qkv -> device, graph of C-ABI calls, attention output -> pinned host; "
                            "double-buffered: the copies of neighbouring steps overlap a step's compute"},
            "cpu_baseline": cpu_base,
            "clocks": ck,
            "per_rank": [{"rank": r, "ms_per_step": round(v[0], 4), "kernel_ms": round(v[1], 5),
                          "kernel_ms_alone": round(v[2], 5), "e2e_ms_per_step": round(v[3], 4),
                          "sm_mhz_median": v[4], "patches_ms_per_step": round(v[5], 4),
                          "patches_e2e_ms_per_step": round(v[6], 4)} for r, v in enumerate(ranks)],
            "gpu_launches": LAYERS * args.steps,
            "device_error": errword,
            "patches_per_s": step,
        }
        emit(line)
    del graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
