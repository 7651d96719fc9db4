"""The C-ABI library: it loads, exports every entry point include/*.h declares, rejects invalid arguments
on the host before touching the GPU, and builds the rotary tables bit-exactly like the reference (no GPU needed)."""
import ctypes
import os
import re

import numpy as np
import pytest

from oumu_b200 import _lib, build
from oracle import cpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", f) for f in ("oumu_attn.h", "oumu_step.h")]


def declarations():
    text = "\n".join(open(h).read() for h in HEADERS)
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    out = {}
    for m in re.finditer(r"(?:^|\n)\s*(?:const\s+)?[a-z_]+\s*\*?\s*(oumu_[a-z0-9_]+)\s*\(([^;]*?)\)\s*;", text):
        args = m.group(2).strip()
        out[m.group(1)] = 0 if args in ("", "void") else args.count(",") + 1
    return out


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    decl = declarations()
    assert len(decl) >= 12, decl
    for name, nargs in decl.items():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
        assert name in _lib.SIGNATURES, f"{name} missing from the ctypes table"
        assert len(_lib.SIGNATURES[name][1]) == nargs, f"{name}: {nargs} C parameters"
    assert set(_lib.SIGNATURES) <= set(decl)


def test_status_strings(lib):
    assert lib.oumu_status_string(0) == b"ok"
    assert lib.oumu_status_string(3) == b"workspace too small"


def test_invalid_arguments_are_rejected_on_the_host(lib):
    P = ctypes.c_void_p(16 * 1024)  # never dereferenced: validation fails first
    # nq % nk != 0
    assert lib.oumu_attn_full(P, P, 10, 5, 0, 16, 3, 128, 0.1, None) == _lib.ERR_INVALID
    # rows not a multiple of seq
    assert lib.oumu_attn_full(P, P, 11, 5, 0, 16, 2, 128, 0.1, None) == _lib.ERR_INVALID
    # unsupported head dim
    assert lib.oumu_attn_full(P, P, 10, 5, 0, 16, 2, 96, 0.1, None) == _lib.ERR_UNSUPPORTED
    # decode: group of 16 q heads per kv head, null length source, misaligned pointer
    assert lib.oumu_attn_decode(P, P, P, P, P, 1 << 20, P, None, 4, 16, 1, 128, 4096, 0.1, None) == \
        _lib.ERR_UNSUPPORTED
    assert lib.oumu_attn_decode(P, P, P, P, P, 1 << 20, None, None, 4, 16, 2, 128, 4096, 0.1, None) == \
        _lib.ERR_INVALID
    assert lib.oumu_attn_decode(ctypes.c_void_p(16 * 1024 + 2), P, P, P, P, 1 << 20, P, None, 4, 16, 2, 128, 4096,
                                0.1, None) == _lib.ERR_INVALID
    # kv_replicate with T > maxlen, rope decode without pos
    assert lib.oumu_kv_replicate(P, 4, 2, 64, 128, 65, None) == _lib.ERR_INVALID
    assert lib.oumu_rope(P, P, P, None, 4, 0, 16, 2, 128, None) == _lib.ERR_INVALID
    # prefill kv_write past the end of the cache
    assert lib.oumu_kv_write(P, P, P, None, 1, 65, 16, 2, 128, 64, None) == _lib.ERR_INVALID
    # unsupported shapes give a zero workspace size
    assert lib.oumu_attn_decode_workspace(4, 16, 3, 128, 4096) == 0


def test_invalid_arguments_of_the_fused_and_step_entry_points(lib):
    P = ctypes.c_void_p(16 * 1024)  # never dereferenced: validation fails first
    # rope + small attention: no rotary tables; sequences longer than 16; one q head per kv head; a stacked group
    # of more than 128 rows (32 q heads x 5 tokens)
    assert lib.oumu_attn_full_rope(P, P, None, P, 22, 11, 0, 16, 2, 128, 0.1, None) == _lib.ERR_INVALID
    assert lib.oumu_attn_full_rope(P, P, P, P, 34, 17, 0, 16, 2, 128, 0.1, None) == _lib.ERR_UNSUPPORTED
    assert lib.oumu_attn_full_rope(P, P, P, P, 22, 11, 0, 16, 16, 128, 0.1, None) == _lib.ERR_UNSUPPORTED
    assert lib.oumu_attn_full_rope(P, P, P, P, 10, 5, 0, 64, 2, 128, 0.1, None) == _lib.ERR_UNSUPPORTED
    # prefill with the KV epilogue: prompt longer than the slot; no slots; prompts of 16 or fewer (small path)
    assert lib.oumu_attn_prefill_kv(P, P, P, P, 65, 4, 16, 2, 128, 64, 0.1, None) == _lib.ERR_INVALID
    assert lib.oumu_attn_prefill_kv(P, P, P, P, 32, 0, 16, 2, 128, 64, 0.1, None) == _lib.ERR_INVALID
    assert lib.oumu_attn_prefill_kv(P, P, P, P, 16, 4, 16, 2, 128, 64, 0.1, None) == _lib.ERR_UNSUPPORTED
    # step glue: RMS norm width, SwiGLU width, FSQ scale, build_seq shape, cfg_euler token window, step_end steps
    assert lib.oumu_rmsnorm(P, None, P, P, 4, 1536, 1e-5, None) == _lib.ERR_UNSUPPORTED
    assert lib.oumu_silu_mul(P, P, 4, 12, None) == _lib.ERR_INVALID
    assert lib.oumu_pointwise(P, 64, 1, 0.0, None) == _lib.ERR_INVALID
    assert lib.oumu_build_seq(P, P, P, P, P, 6, 2, 11, 1024, None) == _lib.ERR_INVALID  # rows != 2 B for the DiT
    assert lib.oumu_cfg_euler(P, P, 4, 11, 8, 0.1, 2.0, None) == _lib.ERR_INVALID
    assert lib.oumu_step_end(P, P, P, P, P, P, 4, 2, 0, None) == _lib.ERR_INVALID
    # projection GEMM: K not a multiple of its 64-element tile
    assert lib.oumu_gemm(P, 100, P, P, 128, None, 4, 128, 100, None) == _lib.ERR_INVALID
    # decoding loop: no step graph, no status buffer, no takes, no steps; the handle is cleared on failure;
    # launching a null loop is rejected and destroying one is a no-op
    h = ctypes.c_void_p(1234)
    assert lib.oumu_decode_loop_create(None, P, P, P, 4, 8, ctypes.byref(h)) == _lib.ERR_INVALID
    assert h.value is None
    assert lib.oumu_decode_loop_create(P, P, P, None, 4, 8, ctypes.byref(h)) == _lib.ERR_INVALID
    assert lib.oumu_decode_loop_create(P, P, P, P, 0, 8, ctypes.byref(h)) == _lib.ERR_INVALID
    assert lib.oumu_decode_loop_create(P, P, P, P, 4, 0, ctypes.byref(h)) == _lib.ERR_INVALID
    assert lib.oumu_decode_loop_create(P, P, P, P, 4, 8, None) == _lib.ERR_INVALID
    assert lib.oumu_decode_loop_launch(None, None) == _lib.ERR_INVALID
    assert lib.oumu_decode_loop_destroy(None) == _lib.OK


@pytest.mark.parametrize("maxlen,hd,ext", [(4096, 128, None), (64, 64, None), (300, 128, "longrope")])
def test_rotary_tables_bit_exact_with_oracle(lib, maxlen, hd, ext):
    e = None
    if ext:
        e = np.linspace(1.0, 40.0, hd // 2).astype(np.float64)  # LongRoPE-style short factors
    cs = np.empty((maxlen, hd // 2), np.float32)
    sn = np.empty_like(cs)
    ep = None if e is None else e.ctypes.data_as(ctypes.c_void_p)
    assert lib.oumu_rotary_tables(maxlen, hd, ep, cs.ctypes.data_as(ctypes.c_void_p),
                                  sn.ctypes.data_as(ctypes.c_void_p)) == 0
    rc, rs = cpu.rotary_tables(maxlen, hd, e)
    assert (cs.view(np.uint32) == rc.view(np.uint32)).all()
    assert (sn.view(np.uint32) == rs.view(np.uint32)).all()
