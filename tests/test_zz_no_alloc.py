"""The decode entry point that allocates nothing (oumu_attn_decode_static), for hosts that cannot give this library
device memory for scratch: its split-KV partials and combine counters live in a static device array instead of a
caller workspace. Called through the C ABI, it must give the workspace entry point's result, call after call.

Collected last on purpose, and self-contained: it passes alone in a fresh process and after the other tests."""
import ctypes

import numpy as np
import pytest
import torch

import golden_cases as gc
from oumu_b200 import _lib, ops, synth

pytestmark = pytest.mark.gpu

NQ, NK, HD = 16, 2, 128


def _u16(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def _static(lib, qkv, kc, vc, out, lens, B, nq, nk, hd, maxlen):
    return lib.oumu_attn_decode_static(qkv.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), None,
                                       lens.data_ptr(), B, nq, nk, hd, maxlen, hd ** -0.5,
                                       torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("B,maxlen,nq,nk,hd", [(64, 4096, 16, 2, 128), (5, 320, 8, 2, 64)])
def test_static_scratch_decode_matches_workspace_decode(cuda, B, maxlen, nq, nk, hd):
    lib = _lib.load()
    g = torch.Generator(device="cuda")
    g.manual_seed(4242 + B)
    rnd = lambda *s: torch.randn(s, generator=g, device="cuda").to(torch.bfloat16)  # noqa: E731
    lens = torch.tensor(synth.uniform_int(77 + B, B, 1, maxlen), dtype=torch.int32, device="cuda")
    ws = ops.decode_workspace(B, nq, nk, hd, maxlen)
    for call in range(2):  # two calls in a row on fresh data: the shared array must not carry state across calls
        qkv, kc, vc = rnd(B, (nq + 2 * nk) * hd), rnd(B, nk, maxlen, hd), rnd(B, nk, maxlen, hd)
        ref = torch.zeros((B, nq * hd), dtype=torch.bfloat16, device="cuda")
        got = torch.full((B, nq * hd), float("nan"), dtype=torch.bfloat16, device="cuda")
        ops.attn_decode(qkv, kc, vc, ref, ws, None, lens, B, nq, nk, hd, maxlen, hd ** -0.5)
        st = _static(lib, qkv, kc, vc, got, lens, B, nq, nk, hd, maxlen)
        assert st == 0, lib.oumu_last_cuda_error().decode()
        torch.cuda.synchronize()
        gc.assert_close(_u16(got), _u16(ref), f"call {call}")
    assert ops.device_error() == 0


def test_static_scratch_rejects_shapes_that_do_not_fit(cuda):
    lib = _lib.load()
    P = ctypes.c_void_p(1 << 20)  # never dereferenced: the size check comes first
    st = lib.oumu_attn_decode_static(P, P, P, P, None, P, 4096, 128, 128, 64, 32, 0.125, None)
    assert st == _lib.ERR_WORKSPACE
    assert b"static scratch" in lib.oumu_last_cuda_error()
