"""Per-kernel timing of the attention hot path at the benchmark configurations, for this library ("ours") and for
the reference's own kernels ("ref", oracle/_ref/voxcpm_ref.fatbin with the launch shapes of src/model.rs).
Also the small, self-contained cases used for ncu captures.

    python tests/perf_cases.py CASE [--impl ours|ref] [--reps N] [--warmup N] [--layers N]

CASE: decode (config 2: 64 takes, slots of 4096, lengths U[330,4096]; per layer)
      step (config 2 per layer: decode prologue + attention)
      decode1 (config 1: one take, 512 of 4096 positions)
      decode1_long (one take, all 4096 positions of its slot)
      prefill (config 3: T = 1024 causal, 16 q / 2 kv heads, hd 128; per layer; --T for other prompt lengths)
      replicate (config 3: the prompt KV of one layer, K and V, into 64 slots of 4096)
      prefill_kv (config 3 per layer in one launch: prefill + k/v into all 64 slots; and the separate launches)
      locdit (config 4: 512 sequences x 12 tokens, 16 heads, hd 64)
      locdit_ref (the reference's DiT shape: 512 sequences x 11 tokens, 16 q / 2 kv heads, hd 128)
      locdit_ref_rope (the same with the rope: one launch for ours, rope then attention for the reference)
      locenc (the local encoder at 256 takes: 256 sequences x 5 tokens, 16 q / 2 kv heads, hd 128, rope)
      loop (config 5 decoding loop, 32 takes, --reps steps: host loop reading the stop flags after every replay
            against the same graph inside one launch with the stop test on the device; per step)
The step, prefill and short-sequence cases launch this library's kernels with programmatic dependent launch unless
--pdl 0. Prints one JSON line: mean milliseconds per launch (CUDA events on the launching stream, after warm-up) and the
algorithmic bytes / FLOPs per launch. With --impl ref and per-take lengths, the reference kernel (one shared
position) runs once per take with slot-offset pointers; "decode_shared" instead runs every take at the mean length.
"""
import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)

from oumu_b200 import ops, synth  # noqa: E402

NQ, NK, HD = 16, 2, 128


def rnd(shape, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(shape, generator=g, device="cuda", dtype=torch.float32).to(torch.bfloat16)


GRAPH = True
PROFILE = False


def timed(fn, reps, warmup):
    """Mean device milliseconds per call: `reps` calls captured in one CUDA graph and replayed (so host launch
    overhead is excluded), CUDA events around the replay on the launching stream; --eager times calls one by one."""
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    if not GRAPH:
        evs = []
        for i in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn(i)
            b.record()
            evs.append((a, b))
        torch.cuda.synchronize()
        return float(np.mean([a.elapsed_time(b) for a, b in evs]))
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for i in range(reps):
                fn(i)
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if PROFILE:  # only the timed replay between cudaProfilerStart / Stop (ncu --profile-from-start off)
        torch.cuda.profiler.start()
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    if PROFILE:
        torch.cuda.profiler.stop()
    del g
    return a.elapsed_time(b) / reps


def case_decode(args, impl, lens, shared=False):
    B, maxlen = len(lens), 4096
    layers = args.layers
    qkv = [rnd((B, (NQ + 2 * NK) * HD), 10 + l) for l in range(layers)]
    kc = [rnd((B, NK, maxlen, HD), 100 + l) for l in range(layers)]
    vc = [rnd((B, NK, maxlen, HD), 200 + l) for l in range(layers)]
    att = torch.zeros((B, NQ * HD), dtype=torch.bfloat16, device="cuda")
    nbytes = int(sum(2 * NK * int(L) * HD * 2 + 2 * NQ * HD * 2 for L in lens))
    if impl == "ours":
        ws = ops.decode_workspace(B, NQ, NK, HD, maxlen)
        ln = torch.tensor(lens, dtype=torch.int32, device="cuda")

        def fn(i):
            l = i % layers
            ops.attn_decode(qkv[l], kc[l], vc[l], att, ws, None, ln, B, NQ, NK, HD, maxlen, HD ** -0.5)
    else:
        from oracle import refkern
        part = torch.zeros(B * NQ * (maxlen // 64) * (HD + 2), dtype=torch.float32, device="cuda")
        if shared:
            pos = torch.tensor([int(round(np.mean(lens))) - 1], dtype=torch.int32, device="cuda")

            def fn(i):
                l = i % layers
                refkern.attn_decode(qkv[l], kc[l], vc[l], part, att, pos, B, NQ, NK, HD, maxlen, HD ** -0.5)
        else:
            pos = torch.tensor([int(L) - 1 for L in lens], dtype=torch.int32, device="cuda")
            row, slot, nsp = (NQ + 2 * NK) * HD, NK * maxlen * HD, maxlen // 64

            def fn(i):
                l = i % layers
                for s in range(B):
                    refkern.attn_decode(qkv[l].data_ptr() + 2 * s * row, kc[l].data_ptr() + 2 * s * slot,
                                        vc[l].data_ptr() + 2 * s * slot, part.data_ptr() + 4 * s * NQ * nsp * (HD + 2),
                                        att.data_ptr() + 2 * s * NQ * HD, pos.data_ptr() + 4 * s, 1, NQ, NK, HD,
                                        maxlen, HD ** -0.5)
    ms = timed(fn, args.reps, args.warmup)
    return dict(ms=ms, bytes=nbytes, GBps=nbytes / ms / 1e6)


def case_step(args, lens):
    """Config 2 step of `layers` layers: decode prologue + decode attention per layer (two launches), captured
    with programmatic dependent launch as bench.py does; per-layer time."""
    B, maxlen = len(lens), 4096
    layers = args.layers
    qkv = [rnd((B, (NQ + 2 * NK) * HD), 10 + l) for l in range(layers)]
    kc = [rnd((B, NK, maxlen, HD), 100 + l) for l in range(layers)]
    vc = [rnd((B, NK, maxlen, HD), 200 + l) for l in range(layers)]
    att = torch.zeros((B, NQ * HD), dtype=torch.bfloat16, device="cuda")
    cs, sn = ops.rotary_tables(maxlen, HD)
    cs, sn = cs.cuda(), sn.cuda()
    ws = ops.decode_workspace(B, NQ, NK, HD, maxlen)
    ln = torch.tensor(lens, dtype=torch.int32, device="cuda")
    nbytes = int(sum(2 * NK * int(L) * HD * 2 + 2 * NQ * HD * 2 for L in lens))

    def fn(i):
        l = i % layers
        ops.step_tf_attention(qkv[l], kc[l], vc[l], att, ws, cs, sn, None, ln, B, NQ, NK, HD, maxlen)
    ops.set_pdl(args.pdl)
    ms = timed(fn, args.reps, args.warmup)
    ops.set_pdl(False)
    return dict(ms=ms, bytes=nbytes, GBps=nbytes / ms / 1e6, pdl=args.pdl)


def case_loop(args, B=32):
    """Config 5: `reps` decoding steps of the captured step graph, (a) replayed from the host loop of
    Engine::decode (src/model.rs:784-793: one replay, then the stop flags read back, per step) and (b) as one launch
    of the device-side loop (ops.DecodeLoop). No take asks to stop early (min_len above max_steps), so both run the
    same steps; milliseconds per step, wall clock around the whole loop (it includes the host reads)."""
    import time
    from oumu_b200 import engine
    steps = args.reps
    e = engine.Engine(B, max_steps=steps + 1, min_len=10 ** 6)
    e.prime([int(v) for v in synth.uniform_int(synth.config_seed(5), B, 330, 4096 - 2 * steps - 8)])
    g = e.capture(keep_graph=True)  # the capture's eager step is step 1
    s0 = [t.clone() for t in (e.ctr, e.stop, e.lens)]
    out = {}
    for mode in ("host", "device", "host", "device"):  # the first pair warms up
        for t, v in zip((e.ctr, e.stop, e.lens), s0):
            t.copy_(v)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        e.decode(g, device_loop=mode == "device")
        torch.cuda.synchronize()
        out[mode] = (time.perf_counter() - t0) * 1e3 / steps
        assert int(e.ctr[1]) == steps + 1
    return dict(ms=out["device"], host_ms=out["host"], steps=steps, takes=B)


def case_prefill(args, impl, T=1024):
    layers = args.layers
    qkv = [rnd((T, (NQ + 2 * NK) * HD), 300 + l) for l in range(layers)]
    out = torch.zeros((T, NQ * HD), dtype=torch.bfloat16, device="cuda")
    flops = 4 * NQ * HD * T * (T + 1) // 2
    K = ops if impl == "ours" else __import__("oracle.refkern", fromlist=["x"])

    def fn(i):
        K.attn_full(qkv[i % layers], out, T, T, 1, NQ, NK, HD, HD ** -0.5)
    ms = timed_pdl(fn, args, impl)
    return dict(ms=ms, flops=flops, TFLOPs=flops / ms / 1e9, pdl=args.pdl if impl == "ours" else 0)


def case_replicate(args, impl, B=64, maxlen=4096, T=1024):
    c = [rnd((B, NK, maxlen, HD), 400 + k) for k in range(2)]
    K = ops if impl == "ours" else __import__("oracle.refkern", fromlist=["x"])
    nbytes = 2 * (NK * T * HD * 2) * B  # per cache: slot 0 read once + B-1 slots written, K and V

    def fn(i):
        K.kv_replicate(c[0], B, NK, maxlen, HD, T)
        K.kv_replicate(c[1], B, NK, maxlen, HD, T)
    ms = timed(fn, args.reps, args.warmup)
    return dict(ms=ms, bytes=nbytes, GBps=nbytes / ms / 1e6)


def case_prefill_kv(args, B=64, maxlen=4096, T=1024):
    """Config 3 per layer in one launch: causal prefill + the prompt's k/v into all B slots (oumu_attn_prefill_kv);
    against it, the separate launches (kv_write, attention, replication of K and V)."""
    layers = args.layers
    qkv = [rnd((T, (NQ + 2 * NK) * HD), 300 + l) for l in range(layers)]
    out = torch.zeros((T, NQ * HD), dtype=torch.bfloat16, device="cuda")
    kc, vc = rnd((B, NK, maxlen, HD), 401), rnd((B, NK, maxlen, HD), 402)
    flops = 4 * NQ * HD * T * (T + 1) // 2

    def fused(i):
        ops.attn_prefill_kv(qkv[i % layers], out, kc, vc, T, B, NQ, NK, HD, maxlen, HD ** -0.5)

    def separate(i):
        ops.kv_write(qkv[i % layers], kc, vc, None, 1, T, NQ, NK, HD, maxlen)
        ops.attn_full(qkv[i % layers], out, T, T, 1, NQ, NK, HD, HD ** -0.5)
        ops.kv_replicate(kc, B, NK, maxlen, HD, T)
        ops.kv_replicate(vc, B, NK, maxlen, HD, T)
    ms = timed_pdl(fused, args, "ours")
    ms_sep = timed_pdl(separate, args, "ours")
    return dict(ms=ms, ms_separate=ms_sep, flops=flops, TFLOPs=flops / ms / 1e9,
                kv_bytes_written=2 * B * NK * T * HD * 2, pdl=args.pdl)


def timed_pdl(fn, args, impl):
    """timed(), with this library's launches made with programmatic dependent launch when --pdl 1 (ours only)."""
    if impl != "ours":
        return timed(fn, args.reps, args.warmup)
    prev = ops.set_pdl(bool(args.pdl))
    try:
        return timed(fn, args.reps, args.warmup)
    finally:
        ops.set_pdl(prev)


def case_small(args, impl, nseq, seq, nq, nk, hd, rope=False):
    rows, W = nseq * seq, (nq + 2 * nk) * hd
    layers = max(args.layers, 8)  # rotate inputs so consecutive calls do not hit L2
    qkv = [rnd((rows, W), 500 + l) for l in range(layers)]
    out = torch.zeros((rows, nq * hd), dtype=torch.bfloat16, device="cuda")
    nbytes = rows * (nq + 2 * nk) * hd * 2 + rows * nq * hd * 2
    K = ops if impl == "ours" else __import__("oracle.refkern", fromlist=["x"])
    if rope:
        from oracle import cpu  # the reference builds its rotary tables on the host (src/model.rs:337-349)
        cs, sn = (torch.from_numpy(t).cuda() for t in cpu.rotary_tables(seq, hd))

    def fn(i):
        if rope and impl == "ours":  # one launch: rope + attention (Engine::full's DiT call)
            K.attn_full_rope(qkv[i % layers], out, cs, sn, rows, seq, 0, nq, nk, hd, hd ** -0.5)
            return
        if rope:  # the reference's two launches; q and k are rotated again on each call (timing only)
            K.rope(qkv[i % layers], cs, sn, None, rows, seq, nq, nk, hd)
        K.attn_full(qkv[i % layers], out, rows, seq, 0, nq, nk, hd, hd ** -0.5)
    ms = timed_pdl(fn, args, impl)
    return dict(ms=ms, bytes=nbytes, GBps=nbytes / ms / 1e6, pdl=args.pdl if impl == "ours" else 0)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case")
    ap.add_argument("--impl", default="ours", choices=["ours", "ref"])
    ap.add_argument("--reps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--eager", action="store_true", help="time calls one by one instead of graph replay")
    ap.add_argument("--pdl", type=int, default=1,
                    help="programmatic dependent launch on/off for this library's kernels (step, prefill and "
                         "short-sequence cases)")
    ap.add_argument("--T", type=int, default=1024, help="prefill case: prompt length")
    ap.add_argument("--profile", action="store_true",
                    help="bracket the timed graph replay with cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    args = ap.parse_args()
    global GRAPH, PROFILE
    GRAPH = not args.eager
    PROFILE = args.profile
    if args.impl == "ours":
        from oumu_b200 import build
        build.build()
    lens2 = synth.uniform_int(synth.config_seed(1), 64, 330, 4096)
    c = args.case
    if c == "decode":
        r = case_decode(args, args.impl, lens2)
    elif c == "step":
        r = case_step(args, lens2)
    elif c == "decode_shared":
        r = case_decode(args, args.impl, lens2, shared=True)
    elif c == "decode1":
        r = case_decode(args, args.impl, [512])
    elif c == "decode1_long":
        r = case_decode(args, args.impl, [4096])
    elif c == "prefill":
        r = case_prefill(args, args.impl, T=args.T)
    elif c == "replicate":
        r = case_replicate(args, args.impl)
    elif c == "prefill_kv":
        r = case_prefill_kv(args)
    elif c == "loop":
        r = case_loop(args)
    elif c == "locdit":
        r = case_small(args, args.impl, 512, 12, 16, 16, 64)
    elif c == "locdit_ref":
        r = case_small(args, args.impl, 512, 11, 16, 2, 128)
    elif c == "locdit_ref_rope":
        r = case_small(args, args.impl, 512, 11, 16, 2, 128, rope=True)
    elif c == "locenc":
        r = case_small(args, args.impl, 256, 5, 16, 2, 128, rope=True)
    else:
        raise SystemExit(f"unknown case {c}")
    r.update(case=c, impl=args.impl, reps=args.reps)
    print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
