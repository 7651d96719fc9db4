"""The decode entry point that allocates nothing (oumu_attn_decode_static), for hosts that cannot give this library
device memory for scratch (a plug-in that only sees the input and output buffers an engine hands it, an engine whose
memory plan owns every device allocation): its split-KV partials and combine counters live in a static device array
instead of a caller workspace. Called through the C ABI, it must match the CPU oracle and give the workspace entry
point's result, call after call, and a call it rejects must queue nothing.

Collected last on purpose, and self-contained: it passes alone in a fresh process and after the other tests."""
import ctypes

import numpy as np
import pytest
import torch

import golden_cases as gc
from oumu_b200 import _lib, ops, synth
from oracle import cpu

pytestmark = pytest.mark.gpu


def _u16(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def _static(lib, qkv, kc, vc, out, lens, B, nq, nk, hd, maxlen, stream=None):
    st = torch.cuda.current_stream().cuda_stream if stream is None else stream
    return lib.oumu_attn_decode_static(qkv.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                       out if isinstance(out, int) else out.data_ptr(), None, lens.data_ptr(), B, nq,
                                       nk, hd, maxlen, hd ** -0.5, st)


@pytest.mark.parametrize("B,maxlen,nq,nk,hd", [(64, 4096, 16, 2, 128), (5, 320, 8, 2, 64)])
def test_static_scratch_decode_matches_oracle_and_workspace_decode(cuda, B, maxlen, nq, nk, hd):
    lib = _lib.load()
    g = torch.Generator(device="cuda")
    g.manual_seed(4242 + B)
    rnd = lambda *s: torch.randn(s, generator=g, device="cuda").to(torch.bfloat16)  # noqa: E731
    lens_h = synth.uniform_int(77 + B, B, 1, maxlen)
    lens = torch.tensor(lens_h, dtype=torch.int32, device="cuda")
    ws = ops.decode_workspace(B, nq, nk, hd, maxlen)
    for call in range(2):  # two calls in a row on fresh data: the shared array must not carry state across calls
        qkv, kc, vc = rnd(B, (nq + 2 * nk) * hd), rnd(B, nk, maxlen, hd), rnd(B, nk, maxlen, hd)
        ref = torch.zeros((B, nq * hd), dtype=torch.bfloat16, device="cuda")
        got = torch.full((B, nq * hd), float("nan"), dtype=torch.bfloat16, device="cuda")
        ops.attn_decode(qkv, kc, vc, ref, ws, None, lens, B, nq, nk, hd, maxlen, hd ** -0.5)
        st = _static(lib, qkv, kc, vc, got, lens, B, nq, nk, hd, maxlen)
        assert st == 0, lib.oumu_last_cuda_error().decode()
        torch.cuda.synchronize()
        orc = cpu.attn_decode(_u16(qkv), _u16(kc), _u16(vc), None, np.asarray(lens_h, np.int32), B, nq, nk, hd,
                              maxlen, hd ** -0.5)
        gc.assert_close(_u16(got), orc, f"call {call} vs oracle")
        gc.assert_close(_u16(got), _u16(ref), f"call {call} vs workspace entry point")
    assert ops.device_error() == 0


def test_static_scratch_rejects_shapes_it_cannot_run(cuda):
    lib = _lib.load()
    P = ctypes.c_void_p(1 << 20)  # never dereferenced: every check comes before any work
    # more (take, kv head) counters than the array holds
    assert lib.oumu_attn_decode_static(P, P, P, P, None, P, 4096, 128, 128, 64, 32, 0.125, None) == _lib.ERR_WORKSPACE
    assert b"static scratch" in lib.oumu_last_cuda_error()
    # the limits oumu_attn_decode has: head size, GQA group, the shared-memory length table (hd 128)
    assert lib.oumu_attn_decode_static(P, P, P, P, None, P, 4, 16, 2, 96, 64, 0.125, None) == _lib.ERR_UNSUPPORTED
    assert lib.oumu_attn_decode_static(P, P, P, P, None, P, 4, 32, 2, 128, 64, 0.125, None) == _lib.ERR_UNSUPPORTED
    assert lib.oumu_attn_decode_static(P, P, P, P, None, P, 1204, 16, 2, 128, 64, 0.125, None) == _lib.ERR_UNSUPPORTED
    # misaligned output
    assert lib.oumu_attn_decode_static(P, P, P, ctypes.c_void_p((1 << 20) + 2), None, P, 4, 16, 2, 128, 64, 0.125,
                                       None) == _lib.ERR_INVALID


def test_rejected_static_call_queues_nothing(cuda):
    # Captured on a stream: a rejected call must add no node to the graph (no memset of the shared array, no
    # launch); an accepted call adds the counter memset and the kernel.
    from cuda.bindings import runtime as rt
    lib = _lib.load()
    B, maxlen, nq, nk, hd = 3, 128, 16, 2, 128
    qkv = torch.zeros((B, (nq + 2 * nk) * hd), dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros((B, nk, maxlen, hd), dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    out = torch.zeros((B, nq * hd), dtype=torch.bfloat16, device="cuda")
    lens = torch.full((B,), 7, dtype=torch.int32, device="cuda")
    # first call outside any capture: the device address of the array is looked up here
    assert _static(lib, qkv, kc, vc, out, lens, B, nq, nk, hd, maxlen) == 0
    torch.cuda.synchronize()
    s = torch.cuda.Stream()

    def captured_nodes(call):
        err, = rt.cudaStreamBeginCapture(s.cuda_stream, rt.cudaStreamCaptureMode.cudaStreamCaptureModeThreadLocal)
        assert err == rt.cudaError_t.cudaSuccess
        rc = call()
        err, graph = rt.cudaStreamEndCapture(s.cuda_stream)
        assert err == rt.cudaError_t.cudaSuccess
        err, _, n = rt.cudaGraphGetNodes(graph, 0)
        assert err == rt.cudaError_t.cudaSuccess
        rt.cudaGraphDestroy(graph)
        return rc, n

    rc, n = captured_nodes(lambda: _static(lib, qkv, kc, vc, out.data_ptr() + 2, lens, B, nq, nk, hd, maxlen,
                                           stream=s.cuda_stream))
    assert rc == _lib.ERR_INVALID and n == 0, (rc, n)
    rc, n = captured_nodes(lambda: _static(lib, qkv, kc, vc, out, lens, B, nq, nk, 96, maxlen, stream=s.cuda_stream))
    assert rc == _lib.ERR_UNSUPPORTED and n == 0, (rc, n)
    rc, n = captured_nodes(lambda: _static(lib, qkv, kc, vc, out, lens, B, nq, nk, hd, maxlen, stream=s.cuda_stream))
    assert rc == 0 and n == 2, (rc, n)
    torch.cuda.synchronize()
