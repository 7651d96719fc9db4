"""Decoding step of a VoxCPM2-shaped model on one GPU, for end-to-end throughput (patches per second).

A host-side restatement of the reference engine's per-step launch sequence, `Engine::step` (src/model.rs:725-773):
DiT passes with classifier-free guidance (src/model.rs:733-749) -> local encoder on the new patch (:751) -> stop
head (:754-756) -> base LM step (:758) -> FSQ -> fusion -> residual LM step (:759-764) -> step end (:766-772).
Every kernel outside the GEMMs is this library's, through the C ABI: the fused decode layer of the LMs
(oumu_attn_decode_step), the small-sequence attention of the DiT and the local encoder (oumu_attn_full) with its
rope, and the step glue of include/oumu_step.h. The LM projections (qkv, o, gate|up, down at 1 row per take) run
on this library's tcgen05 GEMM (oumu_gemm); the DiT's and the heads' GEMMs are cuBLAS through torch (bf16 in and
out, fp32 accumulate, bias added in the epilogue and rounded once, as the reference's gemm_ex with beta = 1 over a
bias-filled output, src/gpu.rs:186-229, kernels/voxcpm.cu:70-76).

Weights are random (seeded N(0, 0.02) bf16; norm weights 1 + N(0, 0.02)) and the KV slots hold random prompt
state: the step is for timing, not for audio. The whole step is captured as one CUDA graph and replayed, the
positions advancing on the device (src/model.rs:777-796). Dimensions follow src/model.rs:9-25; the layer counts the
reference reads from config.json (src/model.rs:430-433) are arguments.
"""
import math

import numpy as np
import torch

from . import ops

LM, LM_FFN, LOC, LOC_FFN, FSQ = 2048, 6144, 1024, 4096, 512
NQ, NK, HD = 16, 2, 128
QKV, QW = (NQ + 2 * NK) * HD, NQ * HD
PATCH, ENC_SEQ, DIT_SEQ, DIT_X0 = 256, 5, 11, 7
EPS = 1e-5


def _rb(v):
    return np.float32(torch.tensor(float(v), dtype=torch.float32).to(torch.bfloat16).float().item())


def schedule(n):
    """(t, dt) of every diffusion pass that runs the DiT: the sway-sampled schedule of UnifiedCFM in fp32 with its
    bf16 roundings (src/model.rs:292-318); 9 passes for 10 timesteps."""
    f = np.float32
    steps = n + 1
    step = f(-1.0) / f(n)
    lin = [_rb(f(1.0) + step * f(i) if i < steps // 2 else f(0.0) - step * f(steps - 1 - i)) for i in range(steps)]
    ts = []
    for t in lin:
        a = _rb(f(math.pi / 2) * t)
        e = _rb(_rb(_rb(np.cos(a)) - f(1.0)) + t)
        ts.append(_rb(t + e))
    zero_init = max(1, int(steps * 0.04))
    t, dt = ts[0], _rb(ts[0] - ts[1])
    out = []
    for s in range(1, steps):
        if s > zero_init:
            out.append((float(t), float(dt)))
        t = _rb(t - dt)
        if s < steps - 1:
            dt = _rb(t - ts[s + 1])
    return out


def gather_patches(patches, stop, group=None):
    """Every rank's finished patches [B][max_steps][PATCH] and stop steps [B] in rank order (rank r's takes at
    [r*B, (r+1)*B)): the one collective of a decode sharded over GPUs by takes, once per text after the last step (the
    reference keeps every take on one GPU and reads them back there, src/model.rs:785-796). torch.distributed
    all_gather over the process group's backend (NCCL for device tensors, gloo for host tensors; the tensors cross as
    their bytes); without a process group, the tensors themselves."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return patches, stop
    world = dist.get_world_size(group)

    def allgather(t):
        wire = t.contiguous().view(torch.uint8)  # bytes: every backend carries them, whatever the element type
        parts = [torch.empty_like(wire) for _ in range(world)]
        dist.all_gather(parts, wire, group=group)
        return torch.cat(parts).view(t.dtype)

    return allgather(patches), allgather(stop)


class _Init:
    def __init__(self, seed, device):
        self.g = torch.Generator(device=device)
        self.g.manual_seed(seed)
        self.device = device

    def w(self, *shape, std=0.02):
        return (torch.randn(shape, generator=self.g, device=self.device) * std).to(torch.bfloat16)

    def norm(self, n):
        return (1.0 + torch.randn(n, generator=self.g, device=self.device) * 0.02).to(torch.bfloat16)


class Lin:
    """y = x W^T (+ b), weight [n][k] bf16 (src/model.rs:27-45). `tc`: through this library's tensor-core GEMM
    (oumu_gemm) instead of cuBLAS. `swiglu` (with tc, for an MLP's gate|up projection): the call writes the SwiGLU
    activation [rows][n/2] instead (oumu_gemm_swiglu), the weight kept with its rows interleaved for it."""

    def __init__(self, ini, n, k, bias, tc=False, swiglu=False):
        self.w = ini.w(n, k)
        self.b = ini.w(n) if bias else None
        self.tc = tc
        self.swiglu = bool(tc and swiglu)
        if self.swiglu:
            self.w = ops.swiglu_interleave(self.w)
            self.b = ops.swiglu_interleave(self.b) if self.b is not None else None

    def standard_weight(self):
        """The weight in [n][k] row order (the gate rows, then the up rows, for a SwiGLU projection)."""
        return ops.swiglu_deinterleave(self.w) if self.swiglu else self.w

    def __call__(self, x, out):
        if self.swiglu:
            return ops.gemm_swiglu(x, self.w, out, bias_il=self.b)
        if self.tc:
            return ops.gemm(x, self.w, out, bias=self.b)
        if self.b is None:
            return torch.matmul(x, self.w.t(), out=out)
        return torch.addmm(self.b, x, self.w.t(), out=out)

    def nbytes(self):
        return 2 * (self.w.numel() + (self.b.numel() if self.b is not None else 0))


class Tf:
    """One transformer stack (src/model.rs:47-63,111-138): per layer ln1, qkv, o, ln2, gate|up, down; final norm;
    with `slots`, one K and one V cache [slots][NK][maxlen][HD] per layer."""

    def __init__(self, ini, n, h, ffn, rope, slots=0, maxlen=0, tc=()):
        self.h, self.ffn, self.rope = h, ffn, rope
        self.layers = [dict(ln1=ini.norm(h), qkv=Lin(ini, QKV, h, False, "qkv" in tc), o=Lin(ini, h, QW, False, "o" in tc),
                            ln2=ini.norm(h), gu=Lin(ini, 2 * ffn, h, False, "gu" in tc, "swiglu" in tc),
                            down=Lin(ini, h, ffn, False, "down" in tc)) for _ in range(n)]
        self.norm = ini.norm(h)
        shape = (slots, NK, maxlen, HD)
        self.kc = [torch.zeros(shape, dtype=torch.bfloat16, device=ini.device) for _ in range(n)] if slots else []
        self.vc = [torch.zeros(shape, dtype=torch.bfloat16, device=ini.device) for _ in range(n)] if slots else []

    def gemm_params(self):
        return sum(l[k].w.numel() for l in self.layers for k in ("qkv", "o", "gu", "down"))

    def weight_bytes(self):
        return 2 * (self.gemm_params() + sum(l["ln1"].numel() + l["ln2"].numel() for l in self.layers)
                    + self.norm.numel())


class Engine:
    """Weights, KV slots and step buffers for B takes (src/model.rs:184-243, 404-529)."""

    # LM projections that run on this library's GEMM (oumu_gemm) instead of cuBLAS: all four by default. With
    # programmatic dependent launch through the norm / SwiGLU kernels between them, each GEMM streams its weights
    # while the preceding kernel finishes: 4.68 ms per captured step against 4.77 ms on cuBLAS (32 takes, the same
    # B200). lm_tc=() selects cuBLAS.
    # "swiglu": the gate|up GEMM writes the SwiGLU activation itself (oumu_gemm_swiglu), one launch per layer fewer.
    LM_TC = ("qkv", "o", "gu", "down", "swiglu")

    def __init__(self, B, maxlen=4096, timesteps=10, base_layers=28, res_layers=8, enc_layers=4, dit_layers=4,
                 cfg=2.0, max_steps=256, min_len=2, seed=0, device="cuda", lm_tc=LM_TC):
        if not 1 <= B <= 1024:
            raise ValueError("takes per GPU must be in 1..1024")
        self.B, self.maxlen, self.cfg, self.max_steps, self.min_len = B, maxlen, cfg, max_steps, min_len
        self.device = dev = torch.device(device)
        ini = _Init(seed, dev)
        self.base = Tf(ini, base_layers, LM, LM_FFN, True, B, maxlen, tc=lm_tc)
        self.res = Tf(ini, res_layers, LM, LM_FFN, False, B, maxlen, tc=lm_tc)  # no rope (src/model.rs:445)
        self.enc = Tf(ini, enc_layers, LOC, LOC_FFN, True)
        self.dit = Tf(ini, dit_layers, LOC, LOC_FFN, True)
        L = lambda n, k, b=True: Lin(ini, n, k, b)  # noqa: E731
        self.enc_in, self.enc_to_lm = L(LOC, 64), L(LM, LOC)
        self.enc_special = ini.w(LOC)
        self.dit_in, self.dit_cond, self.dit_out = L(LOC, 64), L(LOC, 64), L(64, LOC)
        self.fsq_in, self.fsq_out, self.fusion = L(FSQ, LM), L(LM, FSQ), L(LM, 2 * LM)
        self.lm_to_dit, self.res_to_dit = L(LOC, LM), L(LOC, LM)
        self.stop_proj, self.stop_head = L(LM, LM), L(2, LM, False)
        self.sched = schedule(timesteps)
        self._temb(ini)
        cs, sn = ops.rotary_tables(maxlen, HD)
        self.cos, self.sin = cs.to(dev), sn.to(dev)
        z = lambda *s: torch.zeros(s, dtype=torch.bfloat16, device=dev)  # noqa: E731
        # per-take state (StepBufs, src/model.rs:184-243)
        self.x, self.cond, self.noise = z(B, PATCH), z(B, PATCH), z(B, PATCH)
        self.lm_h, self.res_h = z(B, LM), z(B, LM)
        self.mu, self.condp, self.xp = z(B, 2 * LOC), z(B * 4, LOC), z(B * 4, LOC)
        self.dit_seq, self.dit_hout = z(2 * B * DIT_SEQ, LOC), z(2 * B * DIT_SEQ, LOC)
        self.dit_o = z(2 * B * DIT_SEQ, 64)
        self.enc_seq, self.enc_hout = z(B * ENC_SEQ, LOC), z(B * ENC_SEQ, LOC)
        self.fus, self.base_x, self.lm_raw, self.res_x = z(B, 2 * LM), z(B, LM), z(B, LM), z(B, LM)
        self.q, self.stop_h, self.stop_l = z(B, FSQ), z(B, LM), z(B, 2)
        self.patches = z(B, max_steps, PATCH)
        self.lens = torch.ones(B, dtype=torch.int32, device=dev)
        self.ctr = torch.zeros(4, dtype=torch.int32, device=dev)
        self.stop = torch.full((B,), -1, dtype=torch.int32, device=dev)
        self.ws = ops.decode_workspace(B, NQ, NK, HD, maxlen, dev)
        self._scratch = {}

    def _temb(self, ini):
        """Time embedding of every DiT pass, time_mlp(sinusoid(t)) + delta_time_mlp(sinusoid(0))
        (src/model.rs:351-371), computed once."""
        dev = self.device
        t1, t2, d1, d2 = (Lin(ini, LOC, LOC, True) for _ in range(4))
        half = LOC // 2
        freqs = torch.exp(torch.arange(half, device=dev, dtype=torch.float32) * -(math.log(10000.0) / (half - 1)))

        def sinus(t):
            a = 1000.0 * t * freqs
            return torch.cat([a.sin(), a.cos()]).to(torch.bfloat16)

        n = len(self.sched)
        tin = torch.stack([sinus(t) for t, _ in self.sched])
        zin = torch.stack([sinus(0.0)] * n)

        def mlp(a, b, v):
            h = torch.empty((n, LOC), dtype=torch.bfloat16, device=dev)
            a(v, h)
            torch.nn.functional.silu(h, inplace=True)
            return b(h, torch.empty_like(h))

        self.temb = (mlp(t1, t2, tin).float() + mlp(d1, d2, zin).float()).to(torch.bfloat16).contiguous()

    def _lins(self):
        return [v for v in vars(self).values() if isinstance(v, Lin)]

    def step_weight_bytes(self):
        """Bytes of every weight one step reads (each at least once)."""
        return sum(tf.weight_bytes() for tf in (self.base, self.res, self.enc, self.dit)) + sum(
            l.nbytes() for l in self._lins())

    def step_flops(self):
        """GEMM FLOPs of one step (2 per multiply-add), attention excluded."""
        B, T = self.B, len(self.sched)
        lm = 2 * B * (self.base.gemm_params() + self.res.gemm_params())
        dit = T * 2 * (2 * B * DIT_SEQ) * (self.dit.gemm_params() + 64 * LOC) + T * 2 * B * 4 * 64 * LOC
        enc = 2 * B * ENC_SEQ * self.enc.gemm_params()
        heads = 2 * B * (2 * LOC * LM + 4 * 64 * LOC + LM * LOC + FSQ * LM * 2 + 2 * LM * LM + LM * LM + 2 * LM)
        return lm + dit + enc + heads

    def prime(self, lens, seed=1):
        """Every take holds a prompt: random bf16 K/V in its slots and random hidden states; lens[s] is the number
        of positions take s attends over in the next step (its newest position, lens[s] - 1, is written by it)."""
        lens = [int(v) for v in lens]
        if len(lens) != self.B or min(lens) < 1 or max(lens) > self.maxlen:
            raise ValueError("one length in 1..maxlen per take")
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        for tf in (self.base, self.res):
            for c in tf.kc + tf.vc:
                c.normal_(generator=g)
        for t in (self.lm_h, self.res_h, self.cond, self.noise):
            t.normal_(generator=g)
        self.set_lens(lens)

    def set_lens(self, lens):
        self.lens.copy_(torch.as_tensor([int(v) for v in lens], dtype=torch.int32))
        self.ctr.zero_()
        self.stop.fill_(-1)

    def _sc(self, rows, h, ffn):
        """Scratch of one transformer call site (the reference's Scratch, src/model.rs:245-270, per row count)."""
        key = (rows, h)
        if key not in self._scratch:
            z = lambda *s: torch.empty(s, dtype=torch.bfloat16, device=self.device)  # noqa: E731
            self._scratch[key] = dict(xn=z(rows, h), qkv=z(rows, QKV), att=z(rows, QW), tmp=z(rows, h),
                                      gu=z(rows, 2 * ffn), act=z(rows, ffn))
        return self._scratch[key]

    # ---- transformer passes (src/model.rs:532-632) ----
    def _post_attn(self, tf, li, x, sc, out):
        """o_proj, residual + norm, SwiGLU MLP, residual + the next layer's input norm (src/model.rs:621-631)."""
        l = tf.layers[li]
        l["o"](sc["att"], sc["tmp"])
        ops.rmsnorm(x, l["ln2"], sc["xn"], EPS, d=sc["tmp"])
        if l["gu"].swiglu:  # gate|up projection and SwiGLU in one launch
            l["gu"](sc["xn"], sc["act"])
        else:
            l["gu"](sc["xn"], sc["gu"])
            ops.silu_mul(sc["gu"], sc["act"])
        l["down"](sc["act"], sc["tmp"])
        last = li + 1 == len(tf.layers)
        ops.rmsnorm(x, tf.norm if last else tf.layers[li + 1]["ln1"], out if last else sc["xn"], EPS, d=sc["tmp"])

    def full(self, tf, x, rows, seq, out):
        """Independent non-causal sequences of length seq (the DiT and the local encoder, src/model.rs:532-571)."""
        sc = self._sc(rows, tf.h, tf.ffn)
        ops.rmsnorm(x, tf.layers[0]["ln1"], sc["xn"], EPS)
        for li, l in enumerate(tf.layers):
            l["qkv"](sc["xn"], sc["qkv"])
            ops.full_attention(sc["qkv"], sc["att"], rows, seq, 0, NQ, NK, HD,
                               cos_t=self.cos if tf.rope else None, sin_t=self.sin if tf.rope else None)
            self._post_attn(tf, li, x, sc, out)
        return out

    def step_tf(self, tf, x, out):
        """One position per take through an LM: per layer the fused decode layer (rope + kv_write + split-KV
        attention, src/model.rs:573-619) between the GEMMs."""
        B = self.B
        sc = self._sc(B, tf.h, tf.ffn)
        ops.rmsnorm(x, tf.layers[0]["ln1"], sc["xn"], EPS)
        for li, l in enumerate(tf.layers):
            l["qkv"](sc["xn"], sc["qkv"])
            ops.step_tf_attention(sc["qkv"], tf.kc[li], tf.vc[li], sc["att"], self.ws, self.cos, self.sin, None,
                                  self.lens, B, NQ, NK, HD, self.maxlen, rope_on=tf.rope)
            self._post_attn(tf, li, x, sc, out)
        return out

    def encode(self, feat, n, y):
        """Local encoder over n patches [n][4][64] -> its first token's output projected to LM width
        (src/model.rs:634-644)."""
        self.enc_in(feat.view(n * 4, 64), self.xp[:n * 4])
        ops.build_seq(self.enc_seq, self.enc_special, self.xp, n, ENC_SEQ, LOC)
        self.full(self.enc, self.enc_seq, n * ENC_SEQ, ENC_SEQ, self.enc_hout)
        cls = self.enc_hout.view(n, ENC_SEQ, LOC)[:, 0]  # rows ENC_SEQ apart, a strided GEMM operand
        return self.enc_to_lm(cls, y)

    def step(self):
        """One decoding step for every take; device work only, so it can be captured (src/model.rs:725-773)."""
        B = self.B
        self.lm_to_dit(self.lm_h, self.mu[:, :LOC])
        self.res_to_dit(self.res_h, self.mu[:, LOC:])
        self.dit_cond(self.cond.view(B * 4, 64), self.condp)
        self.x.copy_(self.noise)
        for i, (_, dt) in enumerate(self.sched):
            self.dit_in(self.x.view(B * 4, 64), self.xp)
            ops.build_seq(self.dit_seq, self.temb[i], self.xp, 2 * B, DIT_SEQ, LOC, mu=self.mu, condp=self.condp, B=B)
            self.full(self.dit, self.dit_seq, 2 * B * DIT_SEQ, DIT_SEQ, self.dit_hout)
            self.dit_out(self.dit_hout, self.dit_o)  # all 11 tokens; cfg_euler reads the 4 noisy ones in place
            ops.cfg_euler(self.x, self.dit_o, B, DIT_SEQ, DIT_X0, dt, self.cfg)
        self.encode(self.x, B, self.base_x)
        self.fus[:, LM:].copy_(self.base_x)
        self.stop_proj(self.lm_h, self.stop_h)
        ops.silu_(self.stop_h)
        self.stop_head(self.stop_h, self.stop_l)
        self.step_tf(self.base, self.base_x, self.lm_raw)
        self.fsq_in(self.lm_raw, self.q)
        ops.fsq_(self.q, 9.0)
        self.fsq_out(self.q, self.lm_h)
        self.fus[:, :LM].copy_(self.lm_h)
        self.fusion(self.fus, self.res_x)
        self.step_tf(self.res, self.res_x, self.res_h)
        self.cond.copy_(self.x)
        ops.step_end(self.stop_l, self.x, self.patches, self.stop, self.ctr, self.lens, B, self.min_len,
                     self.max_steps)

    def capture(self, keep_graph=False):
        """The step as one CUDA graph (src/model.rs:779-783), programmatic edges into the decode layers. The step
        runs once eagerly first (buffers, cuBLAS handles), which advances the state by one step. keep_graph=True
        keeps the cudaGraph_t for decode(device_loop=True) and instantiates the graph for replay."""
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph(keep_graph=keep_graph)
        with torch.cuda.stream(s):
            self.step()
            s.synchronize()
            prev = ops.set_pdl(True)
            try:
                with torch.cuda.graph(g, stream=s):
                    self.step()
            finally:
                ops.set_pdl(prev)
            if keep_graph:
                g.instantiate()
        torch.cuda.current_stream().wait_stream(s)
        return g

    def decode(self, graph, device_loop=True):
        """Steps until every take has stopped or max_steps patches exist; the number of patches of every take
        (Engine::decode, src/model.rs:777-796: stop step + 1, or max_steps for a take that never stopped).
        device_loop=False replays `graph` and reads the stop flags after every step, as the reference does;
        device_loop=True runs the whole loop as one graph launch with the stop test on the device (`graph` from
        capture(keep_graph=True)) and reads the flags once."""
        if device_loop:
            if getattr(self, "_loop_graph", None) is not graph:
                if getattr(self, "_loop", None) is not None:
                    self._loop.close()
                self.loop_status = torch.zeros(2, dtype=torch.int32, device=self.device)
                self._loop = ops.DecodeLoop(graph, self.stop, self.ctr, self.loop_status, self.B, self.max_steps)
                self._loop_graph = graph
            self._loop.launch()
            stops = self.stop.cpu()
            if int(self.loop_status[1]) != 0:
                raise RuntimeError("decoding loop ended at its step cap while ctr[1] < max_steps")
        else:
            stops = self.stop.cpu()
            for _ in range(int(self.ctr[1]), self.max_steps):
                if bool((stops >= 0).all()):
                    break
                graph.replay()
                stops = self.stop.cpu()
        return [int(v) + 1 if v >= 0 else self.max_steps for v in stops.tolist()]
