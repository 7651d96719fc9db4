"""The decoding step of config 5 run through the reference's own kernels, for a like-for-like patches/s comparison
with oumu_b200.engine on the same GPU.

Same weights, buffers and launch order as oumu_b200.engine.Engine (which restates Engine::step, src/model.rs:725-773),
but every non-GEMM kernel is the reference's (oracle/_ref/voxcpm_ref.fatbin, launched with the grids of
src/model.rs): rmsnorm / add_rmsnorm / silu_mul / rope / kv_write / attn_decode + attn_combine / attn_full /
dit_build / gather_rows / cfg_euler / enc_build / silu_inplace / fsq_act / copy2d / fill_bias / step_end. GEMMs are
cuBLAS as in the reference for M > 8 (src/gpu.rs:186-229), the bias pre-filled by fill_bias and accumulated with
beta = 1. The reference decodes every take at one shared position (src/model.rs:596-615): the takes are primed at
the mean of config 5's per-take lengths, so both steps read the same number of KV bytes.

    python tests/perf_step_ref.py [--takes 32] [--steps 20]
Prints one JSON line (ms per step and patches/s for the reference kernels and for this library).
"""
import argparse
import ctypes
import json
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

from oracle import refkern as rk  # noqa: E402
from oumu_b200 import engine, synth  # noqa: E402
from oumu_b200.engine import DIT_SEQ, DIT_X0, ENC_SEQ, EPS, FSQ, HD, LM, LOC, NK, NQ  # noqa: E402

P, I, F = rk.P, rk.I, rk.F


def L(v):
    return ctypes.c_int64(int(v))


def k1(name, n, args):
    """Gpu::k1: one thread per element, 256 per block."""
    rk.launch(name, ((int(n) + 255) // 256, 1, 1), 256, 0, args)


class RefStep(engine.Engine):
    """Engine whose step launches the reference kernels (see the module docstring)."""

    def __init__(self, B, **kw):
        super().__init__(B, lm_tc=(), **kw)
        self.part = torch.empty(B * NQ * (self.maxlen // 64) * (HD + 2), dtype=torch.float32, device=self.device)
        self.seeds = torch.arange(B, dtype=torch.int32, device=self.device)
        self.noise_table = None  # [N][64][4] fp32: the noise kernel replays it (verification mode) instead of hashing
        self.z2 = {}

    def lin(self, lin, x, out):
        """Lin::fwd (src/model.rs:27-45): fill_bias, then y += x W^T (cuBLAS, beta = 1)."""
        if lin.b is None:
            return torch.matmul(x, lin.w.t(), out=out)
        rows, n = out.shape
        k1("fill_bias", rows * n, [P(out), P(lin.b), I(rows), I(n), I(out.stride(0))])
        return out.addmm_(x, lin.w.t())

    def _post_attn(self, tf, li, x, sc, out):
        l = tf.layers[li]
        rows, h = x.shape
        self.lin(l["o"], sc["att"], sc["tmp"])
        rk.launch("add_rmsnorm", (rows, 1, 1), 256, 0, [P(x), P(sc["tmp"]), P(l["ln2"]), P(sc["xn"]), I(h), F(EPS)])
        self.lin(l["gu"], sc["xn"], sc["gu"])
        k1("silu_mul", rows * tf.ffn, [P(sc["gu"]), P(sc["act"]), I(rows), I(tf.ffn)])
        self.lin(l["down"], sc["act"], sc["tmp"])
        last = li + 1 == len(tf.layers)
        w, o = (tf.norm, out) if last else (tf.layers[li + 1]["ln1"], sc["xn"])
        rk.launch("add_rmsnorm", (rows, 1, 1), 256, 0, [P(x), P(sc["tmp"]), P(w), P(o), I(h), F(EPS)])

    def full(self, tf, x, rows, seq, out):
        sc = self._sc(rows, tf.h, tf.ffn)
        rk.launch("rmsnorm", (rows, 1, 1), 256, 0, [P(x), P(tf.layers[0]["ln1"]), P(sc["xn"]), I(tf.h), F(EPS)])
        for li, l in enumerate(tf.layers):
            self.lin(l["qkv"], sc["xn"], sc["qkv"])
            if tf.rope:
                rk.rope(sc["qkv"], self.cos, self.sin, None, rows, seq, NQ, NK, HD)
            rk.attn_full(sc["qkv"], sc["att"], rows, seq, 0, NQ, NK, HD, HD ** -0.5)
            self._post_attn(tf, li, x, sc, out)
        return out

    def step_tf(self, tf, x, out):
        B = self.B
        sc = self._sc(B, tf.h, tf.ffn)
        rk.launch("rmsnorm", (B, 1, 1), 256, 0, [P(x), P(tf.layers[0]["ln1"]), P(sc["xn"]), I(tf.h), F(EPS)])
        for li, l in enumerate(tf.layers):
            self.lin(l["qkv"], sc["xn"], sc["qkv"])
            if tf.rope:
                rk.rope(sc["qkv"], self.cos, self.sin, self.ctr, B, 0, NQ, NK, HD)
            rk.kv_write(sc["qkv"], tf.kc[li], tf.vc[li], self.ctr, B, 1, NQ, NK, HD, self.maxlen)
            rk.attn_decode(sc["qkv"], tf.kc[li], tf.vc[li], self.part, sc["att"], self.ctr, B, NQ, NK, HD,
                           self.maxlen, HD ** -0.5)
            self._post_attn(tf, li, x, sc, out)
        return out

    def encode(self, feat, n, y):
        self.lin(self.enc_in, feat.view(n * 4, 64), self.xp[:n * 4])
        rk.launch("enc_build", (n, ENC_SEQ, 1), 256, 0, [P(self.enc_seq), P(self.enc_special), P(self.xp), I(LOC)])
        self.full(self.enc, self.enc_seq, n * ENC_SEQ, ENC_SEQ, self.enc_hout)
        cls = self.z2.setdefault("cls", torch.empty((n, LOC), dtype=torch.bfloat16, device=self.device))
        rk.launch("gather_rows", (n, 1, 1), 256, 0, [P(self.enc_hout), P(cls), I(ENC_SEQ), I(0), I(1), I(LOC)])
        return self.lin(self.enc_to_lm, cls, y)

    def step(self):
        B = self.B
        z = self.z2
        tok = z.setdefault("tok", torch.empty((2 * B * 4, LOC), dtype=torch.bfloat16, device=self.device))
        dit_o = z.setdefault("dit_o", torch.empty((2 * B * 4, 64), dtype=torch.bfloat16, device=self.device))
        self.lin(self.lm_to_dit, self.lm_h, self.mu[:, :LOC])
        self.lin(self.res_to_dit, self.res_h, self.mu[:, LOC:])
        self.lin(self.dit_cond, self.cond.view(B * 4, 64), self.condp)
        rk.launch("noise", (B, 1, 1), 256, 0, [P(self.x), P(self.noise_table), P(self.ctr.data_ptr() + 4),
                                               P(self.seeds), I(B)])
        for i, (_, dt) in enumerate(self.sched):
            self.lin(self.dit_in, self.x.view(B * 4, 64), self.xp)
            rk.launch("dit_build", (2 * B, DIT_SEQ, 1), 256, 0, [P(self.dit_seq), P(self.mu), P(self.temb[i]),
                                                                 P(self.condp), P(self.xp), I(B), I(LOC)])
            self.full(self.dit, self.dit_seq, 2 * B * DIT_SEQ, DIT_SEQ, self.dit_hout)
            rk.launch("gather_rows", (2 * B, 4, 1), 256, 0, [P(self.dit_hout), P(tok), I(DIT_SEQ), I(DIT_X0), I(4),
                                                             I(LOC)])
            self.lin(self.dit_out, tok, dit_o)
            rk.launch("cfg_euler", (B, 1, 1), 256, 0, [P(self.x), P(dit_o), I(B), F(dt), F(self.cfg)])
        self.encode(self.x, B, self.base_x)
        k1("copy2d", B * LM, [P(self.base_x), I(LM), P(self.fus.data_ptr() + 2 * LM), I(2 * LM), I(B), I(LM)])
        self.lin(self.stop_proj, self.lm_h, self.stop_h)
        k1("silu_inplace", B * LM, [P(self.stop_h), L(B * LM)])
        self.lin(self.stop_head, self.stop_h, self.stop_l)
        self.step_tf(self.base, self.base_x, self.lm_raw)
        self.lin(self.fsq_in, self.lm_raw, self.q)
        k1("fsq_act", B * FSQ, [P(self.q), L(B * FSQ), F(9.0)])
        self.lin(self.fsq_out, self.q, self.lm_h)
        k1("copy2d", B * LM, [P(self.lm_h), I(LM), P(self.fus), I(2 * LM), I(B), I(LM)])
        self.lin(self.fusion, self.fus, self.res_x)
        self.step_tf(self.res, self.res_x, self.res_h)
        self.cond.copy_(self.x)
        rk.launch("step_end", (1, 1, 1), 256, 0, [P(self.stop_l), P(self.x), P(self.patches), P(self.stop),
                                                  P(self.ctr), I(B), I(self.min_len), I(self.max_steps)])

    def capture(self):
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            self.step()
            s.synchronize()
            with torch.cuda.graph(g, stream=s):
                self.step()
        torch.cuda.current_stream().wait_stream(s)
        return g


def time_graph(e, lens, steps, shared_pos=None):
    g = e.capture()
    e.set_lens(lens)
    if shared_pos is not None:
        e.ctr.copy_(torch.tensor([shared_pos, 0, 0, 0], dtype=torch.int32))
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e.set_lens(lens)
    if shared_pos is not None:
        e.ctr.copy_(torch.tensor([shared_pos, 0, 0, 0], dtype=torch.int32))
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    del g
    return a.elapsed_time(b) / steps


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--takes", type=int, default=32)
    ap.add_argument("--steps", type=int, default=20)
    args = ap.parse_args()
    if not rk.available():
        print(json.dumps({"unavailable": "oracle/_ref/voxcpm_ref.fatbin not built"}))
        return 0
    B = args.takes
    margin = 2 * (args.steps + 8)
    lens = [int(v) for v in synth.uniform_int(synth.config_seed(5), B, 330, 4096 - margin)]
    mean_pos = int(round(sum(lens) / B)) - 1
    ref = RefStep(B)
    ref.prime(lens)
    ms_ref = time_graph(ref, lens, args.steps, shared_pos=mean_pos)
    del ref
    torch.cuda.empty_cache()
    ours = engine.Engine(B)
    ours.prime(lens)
    ms_ours = time_graph(ours, lens, args.steps)
    print(json.dumps({"takes": B, "steps": args.steps, "mean_len": mean_pos + 1,
                      "reference_kernels": {"ms_per_step": round(ms_ref, 4), "patches_per_s": round(B / ms_ref * 1e3, 1)},
                      "ours": {"ms_per_step": round(ms_ours, 4), "patches_per_s": round(B / ms_ours * 1e3, 1)},
                      "speedup": round(ms_ref / ms_ours, 3)}), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
