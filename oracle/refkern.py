"""TEST INFRASTRUCTURE ONLY — the reference's own kernels on the GPU.

Loads oracle/_ref/voxcpm_ref.fatbin (kernels/voxcpm.cu built as compute_80 PTX, as the reference's build.rs does by
default; the driver JIT-compiles it for the B200) into the current CUDA context with the driver API, and launches
kernels by name with the grids, blocks and shared memory of src/model.rs, like src/gpu.rs:162-176 does.
Buffers are torch CUDA tensors; launches go to the current torch stream.
"""
import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
FATBIN = os.path.join(HERE, "_ref", "voxcpm_ref.fatbin")

_cuda = None
_module = None
_funcs = {}


def available():
    return os.path.exists(FATBIN)


def _drv():
    global _cuda
    if _cuda is None:
        _cuda = ctypes.CDLL("libcuda.so.1")
    return _cuda


def _ck(r, what):
    if r != 0:
        raise RuntimeError(f"{what} failed with CUresult {r}")


def _module_handle():
    global _module
    if _module is None:
        if not available():
            raise RuntimeError(f"{FATBIN} missing: build it with `make -C oracle` where the reference tree exists")
        torch.cuda.init()
        torch.zeros(1, device="cuda")  # make torch's primary context current on this thread
        cu = _drv()
        _ck(cu.cuInit(0), "cuInit")
        ctx = ctypes.c_void_p()
        _ck(cu.cuCtxGetCurrent(ctypes.byref(ctx)), "cuCtxGetCurrent")
        if not ctx.value:
            raise RuntimeError("no current CUDA context")
        data = open(FATBIN, "rb").read()
        buf = ctypes.create_string_buffer(data, len(data))
        mod = ctypes.c_void_p()
        _ck(cu.cuModuleLoadData(ctypes.byref(mod), buf), "cuModuleLoadData")
        _module = mod
    return _module


def _func(name):
    if name not in _funcs:
        f = ctypes.c_void_p()
        _ck(_drv().cuModuleGetFunction(ctypes.byref(f), _module_handle(), name.encode()), f"cuModuleGetFunction {name}")
        _funcs[name] = f
    return _funcs[name]


def P(t):
    """Pointer argument (A::P of src/gpu.rs:54-60); None -> null."""
    return ctypes.c_uint64(0 if t is None else (t if isinstance(t, int) else t.data_ptr()))


def I(v):
    return ctypes.c_int32(int(v))


def F(v):
    return ctypes.c_float(float(v))


def launch(name, grid, block, smem, args):
    """cuLaunchKernel(f, grid, (block,1,1), smem, stream, args) — src/gpu.rs:162-176."""
    f = _func(name)
    vals = list(args)
    arr = (ctypes.c_void_p * len(vals))(*[ctypes.cast(ctypes.pointer(v), ctypes.c_void_p) for v in vals])
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    gx, gy, gz = grid
    _ck(_drv().cuLaunchKernel(f, ctypes.c_uint(gx), ctypes.c_uint(gy), ctypes.c_uint(gz), ctypes.c_uint(block),
                              ctypes.c_uint(1), ctypes.c_uint(1), ctypes.c_uint(smem), stream, arr, None),
        f"cuLaunchKernel {name}")


# ---- the reference's launch sites (src/model.rs) ----

def rope(qkv, cos_t, sin_t, pos, rows, seq, nq, nk, hd):
    """src/model.rs:544-550 (seq > 0, pos null) and :581-587 (seq = 0, pos = ctr)."""
    launch("rope", (rows, nq + nk, 1), 64, 0, [P(qkv), P(cos_t), P(sin_t), P(pos), I(rows), I(seq), I(nq), I(nk),
                                               I(hd)])


def kv_write(qkv, kc, vc, pos, slots, rows, nq, nk, hd, maxlen):
    """src/model.rs:553-559 (prefill, grid (rows,1,nk)) and :590-595 (decode, grid (1,B,nk))."""
    launch("kv_write", (rows, slots, nk), 128, 0, [P(qkv), P(kc), P(vc), P(pos), I(rows), I(nq), I(nk), I(hd),
                                                   I(maxlen)])


def attn_decode(qkv, kc, vc, part, att, pos, B, nq, nk, hd, maxlen, scale):
    """attn_decode grid (B, nq, maxlen/64) then attn_combine grid (B, nq) block hd (src/model.rs:596-615)."""
    nsp = maxlen // 64
    launch("attn_decode", (B, nq, nsp), 128, 0, [P(qkv), P(kc), P(vc), P(part), P(pos), I(nq), I(nk), I(hd),
                                                 I(maxlen), F(scale)])
    launch("attn_combine", (B, nq, 1), hd, 0, [P(part), P(att), I(nq), I(hd), I(nsp)])


_CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES = 8


def _allow_smem(name, smem):
    """Opt the kernel in to more than 48 KB of dynamic shared memory. The reference never does this
    (src/gpu.rs:162-176 launches with the default limit), so its attn_full cannot launch for seq > 12160 at hd 128
    ((hd + seq) * 4 bytes > 48 KB) although src/model.rs:411 accepts prompts of 16384 positions. The harness sets
    the attribute so that the reference's arithmetic can still be compared at those lengths; the kernel is
    unchanged."""
    if smem > 48 * 1024:
        _ck(_drv().cuFuncSetAttribute(_func(name), ctypes.c_int(_CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES),
                                      ctypes.c_int(smem)), f"cuFuncSetAttribute {name}")


def attn_full(qkv, out, rows, seq, causal, nq, nk, hd, scale):
    """src/model.rs:561-567: grid (rows, nq), block 128, dynamic smem (hd + seq) * 4."""
    _allow_smem("attn_full", (hd + seq) * 4)
    launch("attn_full", (rows, nq, 1), 128, (hd + seq) * 4, [P(qkv), P(out), I(seq), I(int(bool(causal))), I(nq),
                                                             I(nk), I(hd), F(scale)])


def kv_replicate(c, B, nk, maxlen, hd, T):
    """src/model.rs:708-714: grid (T, nk, B-1), block 128."""
    if B > 1:
        launch("kv_replicate", (T, nk, B - 1), 128, 0, [P(c), I(B), I(nk), I(maxlen), I(hd), I(T)])


def attn_decode_per_take(qkv, kc, vc, part, att, lens, B, nq, nk, hd, maxlen, scale):
    """Per-take lengths with the reference kernel, which has one shared position: one launch per take with
    slot-offset pointers and that take's own device position L_s - 1 (grid.x = 1)."""
    row = (nq + 2 * nk) * hd
    slot = nk * maxlen * hd
    nsp = maxlen // 64
    pos = torch.tensor([int(L) - 1 for L in lens], dtype=torch.int32, device=qkv.device)
    for s in range(B):
        attn_decode(qkv.data_ptr() + 2 * s * row, kc.data_ptr() + 2 * s * slot, vc.data_ptr() + 2 * s * slot,
                    part.data_ptr() + 4 * s * nq * nsp * (hd + 2), att.data_ptr() + 2 * s * nq * hd,
                    pos.data_ptr() + 4 * s, 1, nq, nk, hd, maxlen, scale)
    torch.cuda.current_stream().synchronize()
    return pos
