"""Failure detection on the device without a fault: a bounded wait of the decode kernel runs out and is reported.

A test hook leaves the last tile of the first CTA's range unloaded (the producer never issues its copy, so its stage is a
flag that nothing sets); with the wait limit lowered to 10 ms the consumer that owns the tile gives up. The launch
returns normally, the device error word holds OUMU_DEVERR_TIMEOUT, the workspace's combine counters are back at
zero, and the very next call on the same workspace is correct. Nothing traps, faults or waits without a bound."""
import time

import numpy as np
import pytest
import torch

import golden_cases as gc
from oumu_b200 import _lib, ops
from oracle import cpu

pytestmark = pytest.mark.gpu

DEVERR_TIMEOUT = 1
NQ, NK, HD = 16, 2, 128


def _u16(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def _case(B, maxlen, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    rnd = lambda *s: torch.randn(s, generator=g, device="cuda").to(torch.bfloat16)  # noqa: E731
    return rnd(B, (NQ + 2 * NK) * HD), rnd(B, NK, maxlen, HD), rnd(B, NK, maxlen, HD)


@pytest.fixture
def short_waits(cuda):
    lib = _lib.load()
    ops.device_error(reset=True)
    _lib.check("oumu_set_wait_limit_ns", lib.oumu_set_wait_limit_ns(10_000_000))  # 10 ms
    yield lib
    lib.oumu_test_drop_last_tile(0)
    _lib.check("oumu_set_wait_limit_ns", lib.oumu_set_wait_limit_ns(0))  # back to the default (2 s)
    ops.device_error(reset=True)


@pytest.mark.parametrize("fused", [False, True], ids=["attention", "fused_layer"])
def test_wait_that_runs_out_is_reported_and_the_next_call_is_correct(short_waits, fused):
    lib = short_waits
    B, maxlen = 4, 512
    lens = [300, 200, 511, 100]
    ln = torch.tensor(lens, dtype=torch.int32, device="cuda")
    ws = ops.decode_workspace(B, NQ, NK, HD, maxlen)
    cs, sn = (t.cuda() for t in ops.rotary_tables(maxlen, HD))
    out = torch.zeros((B, NQ * HD), dtype=torch.bfloat16, device="cuda")

    def run(qkv, kc, vc):
        if fused:
            ops.attn_decode_step(qkv, kc, vc, out, ws, cs, sn, None, ln, B, NQ, NK, HD, maxlen, HD ** -0.5)
        else:
            ops.attn_decode(qkv, kc, vc, out, ws, None, ln, B, NQ, NK, HD, maxlen, HD ** -0.5)

    # the faulty launch: the last tile of CTA 0's range never arrives
    assert lib.oumu_test_drop_last_tile(1) == 0
    qkv, kc, vc = _case(B, maxlen, 31)
    t0 = time.perf_counter()
    run(qkv, kc, vc)
    torch.cuda.synchronize()
    took = time.perf_counter() - t0
    assert lib.oumu_test_drop_last_tile(0) == 1
    err = ops.device_error(reset=True)
    assert err & DEVERR_TIMEOUT, f"device error word {err}"
    assert took < 1.5, f"the launch took {took:.3f} s with a 10 ms wait limit"
    cnt = ws[: B * NK * 4].view(torch.int32)
    assert int(cnt.abs().sum()) == 0, "combine counters left non-zero by the aborted launch"

    # the same workspace and context, a normal launch: correct against the oracle, no error
    qkv, kc, vc = _case(B, maxlen, 32)
    qkv_h, kc_h, vc_h = _u16(qkv), _u16(kc), _u16(vc)
    run(qkv, kc, vc)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    if fused:  # the oracle's prologue (rope + kv_write at each take's newest position), then attention
        cs_h, sn_h = cpu.rotary_tables(maxlen, HD)
        for s, L in enumerate(lens):
            row = np.ascontiguousarray(qkv_h[s:s + 1])
            cpu.rope(row, cs_h, sn_h, L - 1, 1, 0, NQ, NK, HD)
            kcs, vcs = np.ascontiguousarray(kc_h[s:s + 1]), np.ascontiguousarray(vc_h[s:s + 1])
            cpu.kv_write(row, kcs, vcs, L - 1, 1, 1, NQ, NK, HD, maxlen)
            qkv_h[s], kc_h[s], vc_h[s] = row[0], kcs[0], vcs[0]
    ref = cpu.attn_decode(qkv_h, kc_h, vc_h, None, np.asarray(lens, np.int32), B, NQ, NK, HD, maxlen, HD ** -0.5)
    gc.assert_close(_u16(out), ref, "after a timed-out launch")
    assert int(cnt.abs().sum()) == 0


def test_wait_limit_restores_the_default(cuda):
    lib = _lib.load()
    _lib.check("oumu_set_wait_limit_ns", lib.oumu_set_wait_limit_ns(0))
    assert lib.oumu_test_drop_last_tile(0) == 0  # the hook is off outside the test above
