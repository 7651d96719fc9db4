"""Host-side mirror of the reference's attention launch interface, over the C ABI.

Each function has the reference kernel's name and argument meaning (kernels/voxcpm.cu, launched from
src/model.rs) and takes torch CUDA tensors for the buffers; launches go to the current torch stream, so every call
can be recorded inside a CUDA graph capture. Errors raise OumuError with the library's status.
bf16 buffers may be torch.bfloat16 or 16-bit integer tensors holding bf16 bit patterns.
"""
import torch

from . import _lib

HD_SUPPORTED = (64, 128)


def _p(t):
    return None if t is None else t.data_ptr()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def rotary_tables(maxlen, hd, ext=None):
    """cos, sin fp32 [maxlen][hd/2] built on the host (src/model.rs:337-349), as CPU tensors."""
    import ctypes
    import numpy as np
    cs = np.empty((maxlen, hd // 2), dtype=np.float32)
    sn = np.empty_like(cs)
    ext_arr = None if ext is None else np.ascontiguousarray(ext, dtype=np.float64)
    _lib.call("oumu_rotary_tables", maxlen, hd,
              None if ext_arr is None else ext_arr.ctypes.data_as(ctypes.c_void_p),
              cs.ctypes.data_as(ctypes.c_void_p), sn.ctypes.data_as(ctypes.c_void_p))
    return torch.from_numpy(cs), torch.from_numpy(sn)


def rope(qkv, cos_t, sin_t, pos, rows, seq, nq, nk, hd):
    """In-place rotary embedding (kernels/voxcpm.cu:100-115); pos: int32 device tensor or None when seq > 0."""
    _lib.call("oumu_rope", _p(qkv), _p(cos_t), _p(sin_t), _p(pos), rows, seq, nq, nk, hd, _stream())


def kv_write(qkv, kc, vc, pos, slots, rows, nq, nk, hd, maxlen):
    """k/v of `rows` positions of every slot into the caches at *pos (or 0) (kernels/voxcpm.cu:117-129)."""
    _lib.call("oumu_kv_write", _p(qkv), _p(kc), _p(vc), _p(pos), slots, rows, nq, nk, hd, maxlen, _stream())


def decode_prologue(qkv, kc, vc, cos_t, sin_t, pos, lens, B, nq, nk, hd, maxlen):
    """rope + kv_write of one decode position per take, one launch (src/model.rs:580-595)."""
    _lib.call("oumu_decode_prologue", _p(qkv), _p(kc), _p(vc), _p(cos_t), _p(sin_t), _p(pos), _p(lens), B, nq, nk,
              hd, maxlen, _stream())


def decode_workspace_bytes(B, nq, nk, hd, maxlen):
    return int(_lib.load().oumu_attn_decode_workspace(B, nq, nk, hd, maxlen))


def decode_workspace(B, nq, nk, hd, maxlen, device=None):
    """A zero-filled workspace for attn_decode (counters start at zero; every call leaves them at zero)."""
    n = decode_workspace_bytes(B, nq, nk, hd, maxlen)
    if n == 0:
        raise ValueError("unsupported decode shape")
    return torch.zeros(n, dtype=torch.uint8, device=device or "cuda")


def reference_part_bytes(B, nq, hd, maxlen, att_ch=64):
    """Size of the reference's StepBufs::att_part (src/model.rs:237)."""
    return 4 * B * nq * (maxlen // att_ch) * (hd + 2)


def attn_decode(qkv, kc, vc, out, workspace, pos, lens, B, nq, nk, hd, maxlen, scale):
    """Split-KV decode attention with the combine fused (replaces attn_decode + attn_combine,
    kernels/voxcpm.cu:131-185). Lengths: lens[s] (int32 device tensor) or *pos + 1."""
    _lib.call("oumu_attn_decode", _p(qkv), _p(kc), _p(vc), _p(out), _p(workspace), workspace.numel(), _p(pos),
              _p(lens), B, nq, nk, hd, maxlen, float(scale), _stream())


def attn_decode_step(qkv, kc, vc, out, workspace, cos_t, sin_t, pos, lens, B, nq, nk, hd, maxlen, scale):
    """One decode layer in one launch: rope + kv_write of the newest position fused into the split-KV attention
    (replaces rope + kv_write + attn_decode + attn_combine of Engine::step_tf, src/model.rs:580-615)."""
    _lib.call("oumu_attn_decode_step", _p(qkv), _p(kc), _p(vc), _p(out), _p(workspace), workspace.numel(),
              _p(cos_t), _p(sin_t), _p(pos), _p(lens), B, nq, nk, hd, maxlen, float(scale), _stream())


def attn_decode_reset(workspace, B, nq, nk, hd, maxlen):
    _lib.call("oumu_attn_decode_reset", _p(workspace), workspace.numel(), B, nq, nk, hd, maxlen, _stream())


def attn_full(qkv, out, rows, seq, causal, nq, nk, hd, scale):
    """Attention inside independent sequences of length seq (kernels/voxcpm.cu:262-297)."""
    _lib.call("oumu_attn_full", _p(qkv), _p(out), rows, seq, int(bool(causal)), nq, nk, hd, float(scale), _stream())


def kv_replicate(c, B, nk, maxlen, hd, T):
    """Slot 0 -> slots 1..B-1 for positions < T (kernels/voxcpm.cu:407-413)."""
    _lib.call("oumu_kv_replicate", _p(c), B, nk, maxlen, hd, T, _stream())


def set_pdl(enable):
    """Programmatic dependent launch for the decode kernels (see oumu_set_pdl); returns the previous setting."""
    return bool(_lib.load().oumu_set_pdl(1 if enable else 0))


def device_error(reset=False):
    """The library's device-side error word on the current device (synchronises)."""
    return int(_lib.load().oumu_device_error(1 if reset else 0))


# ------------------------------------------------------------------------------------------------------------
# The attention launch sequences of Engine (src/model.rs), per layer
# ------------------------------------------------------------------------------------------------------------

def step_tf_attention(qkv, kc, vc, att, workspace, cos_t, sin_t, ctr, lens, B, nq, nk, hd, maxlen, rope_on=True,
                      fused=True):
    """One decode position of one layer for every take, as Engine::step_tf does (src/model.rs:578-615): one fused
    launch (rope + kv_write + split-KV attention with the combine), or with fused=False the prologue launch then
    the attention launch."""
    cs, sn = (cos_t, sin_t) if rope_on else (None, None)
    pos = ctr if lens is None else None
    if fused:
        attn_decode_step(qkv, kc, vc, att, workspace, cs, sn, pos, lens, B, nq, nk, hd, maxlen, 1.0 / hd ** 0.5)
        return
    decode_prologue(qkv, kc, vc, cs, sn, ctr, lens, B, nq, nk, hd, maxlen)
    attn_decode(qkv, kc, vc, att, workspace, pos, lens, B, nq, nk, hd, maxlen, 1.0 / hd ** 0.5)


def attn_full_rope(qkv, att, cos_t, sin_t, rows, seq, causal, nq, nk, hd, scale):
    """Rope at positions r % seq + attention in one launch (small grouped sequences); qkv is left unrotated."""
    _lib.call("oumu_attn_full_rope", _p(qkv), _p(att), _p(cos_t), _p(sin_t), rows, seq, int(bool(causal)), nq, nk,
              hd, float(scale), _stream())
    return att


def rope_fusable(seq, nq, nk):
    """Shapes oumu_attn_full_rope takes (the grouped small-sequence kernel)."""
    return seq <= 16 and nq // nk >= 2 and (nq // nk) * seq <= 128


def full_attention(qkv, att, rows, seq, causal, nq, nk, hd, maxlen=0, cos_t=None, sin_t=None, kc=None, vc=None):
    """The attention part of one layer of Engine::full (src/model.rs:541-567): rope over positions r % seq,
    kv_write of every row into slot 0 when caches are given, then attention inside the sequences. Small grouped
    sequences without caches (the DiT, the local encoder) take the one-launch rope + attention, which leaves qkv
    unrotated; otherwise q and k are rotated in place first."""
    if cos_t is not None and kc is None and rope_fusable(seq, nq, nk):
        attn_full_rope(qkv, att, cos_t, sin_t, rows, seq, causal, nq, nk, hd, 1.0 / hd ** 0.5)
        return
    if cos_t is not None:
        rope(qkv, cos_t, sin_t, None, rows, seq, nq, nk, hd)
    if kc is not None:
        kv_write(qkv, kc, vc, None, 1, rows, nq, nk, hd, maxlen)
    attn_full(qkv, att, rows, seq, causal, nq, nk, hd, 1.0 / hd ** 0.5)


# ------------------------------------------------------------------------------------------------------------
# Step glue (include/oumu_step.h): the per-row and element-wise kernels between the GEMMs of a step
# ------------------------------------------------------------------------------------------------------------

def rmsnorm(res, w, out, eps, d=None):
    """out = rmsnorm(res) * w; with d, res += d first (add_rmsnorm). res/out [rows][dim], dim 1024 or 2048."""
    _lib.call("oumu_rmsnorm", _p(res), _p(d), _p(w), _p(out), res.shape[0], res.shape[-1], eps, _stream())
    return out


def silu_mul(gu, out):
    """out [rows][F] = bf16(bf16(silu(gate)) * up) of gu = [gate | up] [rows][2F]."""
    _lib.call("oumu_silu_mul", _p(gu), _p(out), gu.shape[0], gu.shape[-1] // 2, _stream())
    return out


def silu_(x):
    _lib.call("oumu_pointwise", _p(x), x.numel(), 0, 1.0, _stream())
    return x


def fsq_(x, scale=9.0):
    _lib.call("oumu_pointwise", _p(x), x.numel(), 1, scale, _stream())
    return x


def build_seq(seq_out, temb, xp, rows, seq, H, mu=None, condp=None, B=0):
    """DiT (seq 11, rows = 2B) or local-encoder (seq 5, temb = the special token) input sequences."""
    _lib.call("oumu_build_seq", _p(seq_out), _p(mu), _p(temb), _p(condp), _p(xp), rows, B, seq, H, _stream())
    return seq_out


def cfg_euler(x, out, B, seq, first, dt, cfg):
    _lib.call("oumu_cfg_euler", _p(x), _p(out), B, seq, first, dt, cfg, _stream())
    return x


def step_end(stop_logits, patch, patches, stop, ctr, lens, B, min_len, max_steps):
    _lib.call("oumu_step_end", _p(stop_logits), _p(patch), _p(patches), _p(stop), _p(ctr), _p(lens), B, min_len,
              max_steps, _stream())


class DecodeLoop:
    """The decoding loop of Engine::decode (src/model.rs:777-796) as one graph launch (oumu_decode_loop_*): the
    step graph `step_graph` (a torch.cuda.CUDAGraph captured with keep_graph=True) repeated inside a CUDA WHILE node
    while ctr[1] < max_steps and some stop[s] < 0, the test made on the device after every step. `status` (int32 [2],
    device) receives the steps run and the iteration-cap flag of each launch."""

    def __init__(self, step_graph, stop, ctr, status, B, max_steps):
        import ctypes
        for t in (stop, ctr, status):
            if t.dtype != torch.int32 or not t.is_cuda or not t.is_contiguous():
                raise ValueError("DecodeLoop: stop, ctr and status are contiguous int32 device tensors")
        if stop.numel() < B or ctr.numel() < 2 or status.numel() < 2:
            raise ValueError("DecodeLoop: stop [B], ctr [>= 2] and status [2]")
        h = ctypes.c_void_p()
        _lib.call("oumu_decode_loop_create", step_graph.raw_cuda_graph(), _p(stop), _p(ctr), _p(status), B,
                  max_steps, ctypes.byref(h))
        self._h = h
        self._keep = (stop, ctr, status)  # the loop's kernels hold these pointers

    def launch(self):
        _lib.call("oumu_decode_loop_launch", self._h, _stream())

    def close(self):
        if self._h is not None and self._h.value:
            _lib.call("oumu_decode_loop_destroy", self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def gemm(x, w, y, bias=None):
    """y[M][N] = bf16(x[M][K] . w[N][K]^T (+ bias)) on the tensor cores; x and y may be row-strided views."""
    M, K = x.shape
    N = w.shape[0]
    if w.shape[1] != K or x.stride(1) != 1 or y.stride(1) != 1 or not w.is_contiguous() or tuple(y.shape) != (M, N):
        raise ValueError("gemm: x [M][K] and y [M][N] with unit column stride, w [N][K] contiguous")
    _lib.call("oumu_gemm", _p(x), x.stride(0), _p(w), _p(y), y.stride(0), _p(bias), M, N, K, _stream())
    return y


def swiglu_interleave(w):
    """The gate|up weight [2F][...] (or bias [2F]) with its rows interleaved in groups of 8, the layout
    oumu_gemm_swiglu reads: rows [16j, 16j + 8) = gate rows [8j, 8j + 8), rows [16j + 8, 16j + 16) = up rows."""
    F = w.shape[0] // 2
    if w.shape[0] != 2 * F or F % 8:
        raise ValueError("swiglu_interleave: 2F rows with F a multiple of 8")
    return w.reshape(2, F // 8, 8, *w.shape[1:]).transpose(0, 1).reshape(w.shape).contiguous()


def swiglu_deinterleave(w_il):
    """The inverse of swiglu_interleave: [gate | up] rows again."""
    F = w_il.shape[0] // 2
    return w_il.reshape(F // 8, 2, 8, *w_il.shape[1:]).transpose(0, 1).reshape(w_il.shape).contiguous()


def gemm_swiglu(x, w_il, act, bias_il=None):
    """act[M][F] = bf16(bf16(silu(gate)) * up) of the gate|up projection x . W^T, one launch (oumu_gemm_swiglu);
    w_il [2F][K] (and bias_il) interleaved by swiglu_interleave. Bit-identical to gemm into [M][2F] + silu_mul."""
    M, K = x.shape
    F = w_il.shape[0] // 2
    if (w_il.shape[1] != K or x.stride(1) != 1 or act.stride(1) != 1 or not w_il.is_contiguous()
            or tuple(act.shape) != (M, F)):
        raise ValueError("gemm_swiglu: x [M][K] and act [M][F] with unit column stride, w_il [2F][K] contiguous")
    _lib.call("oumu_gemm_swiglu", _p(x), x.stride(0), _p(w_il), _p(act), act.stride(0), _p(bias_il), M, F, K,
              _stream())
    return act


def attn_prefill_kv(qkv, out, kc, vc, T, slots, nq, nk, hd, maxlen, scale):
    """Causal prefill of one prompt + its k/v into every take slot, one launch (oumu_attn_prefill_kv): replaces
    kv_write + attn_full (src/model.rs:553-567) and kv_replicate (src/model.rs:705-717)."""
    _lib.call("oumu_attn_prefill_kv", _p(qkv), _p(out), _p(kc), _p(vc), T, slots, nq, nk, hd, maxlen, float(scale),
              _stream())
