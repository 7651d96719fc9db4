"""TEST INFRASTRUCTURE ONLY — numpy/ctypes front end of oracle/attn_ref.c (the fp32 CPU restatement).

All bf16 arrays are numpy uint16 bit patterns. Functions follow the reference kernels they restate
(kernels/voxcpm.cu:100-129,131-185,262-297,407-413 and src/model.rs:337-349).
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
_lib = None
_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float


def build():
    subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(
                os.path.join(HERE, "attn_ref.c")):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.oracle_rotary_tables.argtypes = [_I, _I, _P, _P, _P]
        L.oracle_rope.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, _I]
        L.oracle_kv_write.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I]
        L.oracle_kv_replicate.argtypes = [_P, _I, _I, _I, _I, _I]
        L.oracle_attn_decode.argtypes = [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F]
        L.oracle_attn_full.argtypes = [_P, _P, _I, _I, _I, _I, _I, _I, _F]
        L.oracle_threads.restype = _I
        L.oracle_set_threads.argtypes = [_I]
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dt):
    a = np.ascontiguousarray(a, dtype=dt)
    return a


def threads():
    return int(lib().oracle_threads())


def set_threads(n):
    lib().oracle_set_threads(int(n))


def rotary_tables(maxlen, hd, ext=None):
    cs = np.empty((maxlen, hd // 2), np.float32)
    sn = np.empty_like(cs)
    e = None if ext is None else _c(ext, np.float64)
    lib().oracle_rotary_tables(maxlen, hd, _ptr(e), _ptr(cs), _ptr(sn))
    return cs, sn


def rope(qkv, cos_t, sin_t, pos, rows, seq, nq, nk, hd):
    """In place on qkv (uint16 [rows][(nq+2nk)*hd]); pos: int or None."""
    assert qkv.dtype == np.uint16 and qkv.flags.c_contiguous
    p = None if pos is None else np.array([pos], np.int32)
    lib().oracle_rope(_ptr(qkv), _ptr(_c(cos_t, np.float32)), _ptr(_c(sin_t, np.float32)), _ptr(p), rows, seq, nq,
                      nk, hd)


def kv_write(qkv, kc, vc, pos, slots, rows, nq, nk, hd, maxlen):
    assert kc.dtype == np.uint16 and kc.flags.c_contiguous and vc.flags.c_contiguous
    p = None if pos is None else np.array([pos], np.int32)
    lib().oracle_kv_write(_ptr(_c(qkv, np.uint16)), _ptr(kc), _ptr(vc), _ptr(p), slots, rows, nq, nk, hd, maxlen)


def kv_replicate(c, B, nk, maxlen, hd, T):
    assert c.dtype == np.uint16 and c.flags.c_contiguous
    lib().oracle_kv_replicate(_ptr(c), B, nk, maxlen, hd, T)


def attn_decode(qkv, kc, vc, pos, lens, B, nq, nk, hd, maxlen, scale):
    """Returns out uint16 [B][nq*hd]. pos: int (shared) or None; lens: int array [B] or None."""
    out = np.empty((B, nq * hd), np.uint16)
    p = None if pos is None else np.array([pos], np.int32)
    ln = None if lens is None else _c(lens, np.int32)
    lib().oracle_attn_decode(_ptr(_c(qkv, np.uint16)), _ptr(_c(kc, np.uint16)), _ptr(_c(vc, np.uint16)), _ptr(out),
                             _ptr(p), _ptr(ln), B, nq, nk, hd, maxlen, float(scale))
    return out


def attn_full(qkv, rows, seq, causal, nq, nk, hd, scale):
    out = np.empty((rows, nq * hd), np.uint16)
    lib().oracle_attn_full(_ptr(_c(qkv, np.uint16)), _ptr(out), rows, seq, int(bool(causal)), nq, nk, hd,
                           float(scale))
    return out
