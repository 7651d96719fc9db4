"""ctypes binding of the C ABI in include/oumu_attn.h and include/oumu_step.h (liboumu_attn.so, built in-tree by oumu_b200/build.py).

Loading fails loudly when the library is missing: there is no CPU or eager fallback anywhere in this package.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liboumu_attn.so")

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_WORKSPACE, ERR_CUDA, ERR_DEVICE = range(6)

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_Z = ctypes.c_size_t
_L = ctypes.c_long

# name -> (restype, argtypes); the exact declarations of include/oumu_attn.h and include/oumu_step.h
SIGNATURES = {
    "oumu_status_string": (ctypes.c_char_p, [_I]),
    "oumu_last_cuda_error": (ctypes.c_char_p, []),
    "oumu_rotary_tables": (_I, [_I, _I, _P, _P, _P]),
    "oumu_rope": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "oumu_kv_write": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P]),
    "oumu_decode_prologue": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "oumu_attn_decode_workspace": (_Z, [_I, _I, _I, _I, _I]),
    "oumu_attn_decode_reset": (_I, [_P, _Z, _I, _I, _I, _I, _I, _P]),
    "oumu_attn_decode": (_I, [_P, _P, _P, _P, _P, _Z, _P, _P, _I, _I, _I, _I, _I, _F, _P]),
    "oumu_attn_decode_static": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P]),
    "oumu_attn_decode_step": (_I, [_P, _P, _P, _P, _P, _Z, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P]),
    "oumu_attn_full": (_I, [_P, _P, _I, _I, _I, _I, _I, _I, _F, _P]),
    "oumu_attn_full_rope": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _F, _P]),
    "oumu_kv_replicate": (_I, [_P, _I, _I, _I, _I, _I, _P]),
    "oumu_attn_prefill_kv": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _F, _P]),
    "oumu_device_error": (_I, [_I]),
    "oumu_set_pdl": (_I, [_I]),
    "oumu_set_wait_limit_ns": (_I, [ctypes.c_ulonglong]),
    "oumu_test_drop_last_tile": (_I, [_I]),
    "oumu_rmsnorm": (_I, [_P, _P, _P, _P, _I, _I, _F, _P]),
    "oumu_silu_mul": (_I, [_P, _P, _I, _I, _P]),
    "oumu_pointwise": (_I, [_P, _L, _I, _F, _P]),
    "oumu_build_seq": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "oumu_cfg_euler": (_I, [_P, _P, _I, _I, _I, _F, _F, _P]),
    "oumu_step_end": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "oumu_gemm": (_I, [_P, _I, _P, _P, _I, _P, _I, _I, _I, _P]),
    "oumu_gemm_swiglu": (_I, [_P, _I, _P, _P, _I, _P, _I, _I, _I, _P]),
    "oumu_decode_loop_create": (_I, [_P, _P, _P, _P, _I, _I, ctypes.POINTER(_P)]),
    "oumu_decode_loop_launch": (_I, [_P, _P]),
    "oumu_decode_loop_destroy": (_I, [_P]),
}

_lib = None


class OumuError(RuntimeError):
    def __init__(self, fn, status):
        lib = load()
        msg = lib.oumu_status_string(status).decode()
        if status == ERR_CUDA:
            msg += ": " + lib.oumu_last_cuda_error().decode()
        super().__init__(f"{fn} failed: {msg} (status {status})")
        self.status = status


def load():
    """The loaded library (ctypes.CDLL) with every entry point typed."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m oumu_b200.build` (nvcc, sm_100a); "
                "this package has no fallback path")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(lib, name)
            f.restype = res
            f.argtypes = args
        _lib = lib
    return _lib


def check(fn, status):
    if status != OK:
        raise OumuError(fn, status)


# entry-point calls made through call() (each launches at most one kernel); read by the benchmark to count launches
CALLS = [0]


def call(name, *args):
    """Call entry point `name` and raise OumuError on a non-zero status."""
    CALLS[0] += 1
    st = getattr(load(), name)(*args)
    check(name, st)
    return st
