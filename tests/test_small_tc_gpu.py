"""The tensor-core short-sequence kernel (sq::k_attn_small_tc: TMA boxes per unit, S and O in TMEM), which
oumu_attn_full and oumu_attn_full_rope take for grouped heads once a call has at least 4 units per SM: against the CPU
oracle (kernels/voxcpm.cu:262-297 restated) and, with rope, bit-identical to rope then attention.
Shapes: the DiT's, a causal 128-row stack, hd 64 with a group of 4, the local encoder's at a large batch, and a
group of 16 split into two units per kv head."""
import numpy as np
import pytest
import torch

import golden_cases as gc
from oumu_b200 import ops
from oracle import cpu

pytestmark = pytest.mark.gpu

CASES = [
    # nseq, seq, causal, nq, nk, hd
    (600, 11, 0, 16, 2, 128),
    (600, 16, 1, 16, 2, 128),
    (700, 7, 0, 8, 2, 64),
    (320, 5, 0, 16, 2, 128),
    (300, 11, 0, 32, 2, 128),
]


def _u16(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("nseq,seq,causal,nq,nk,hd", CASES)
def test_small_tc_vs_oracle(cuda, nseq, seq, causal, nq, nk, hd):
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    G = nq // nk
    hs = max(d for d in range(1, G + 1) if G % d == 0 and d * seq <= 128)
    assert nseq * nk * (G // hs) >= 4 * sms, "the case must reach the tensor-core kernel"
    rows, W = nseq * seq, (nq + 2 * nk) * hd
    g = torch.Generator(device="cuda")
    g.manual_seed(nseq + seq)
    qkv = torch.randn((rows, W), generator=g, device="cuda").to(torch.bfloat16)
    out = torch.full((rows, nq * hd), float("nan"), dtype=torch.bfloat16, device="cuda")
    ops.attn_full(qkv, out, rows, seq, causal, nq, nk, hd, hd ** -0.5)
    torch.cuda.synchronize()
    ref = cpu.attn_full(_u16(qkv), rows, seq, causal, nq, nk, hd, hd ** -0.5)
    gc.assert_close(_u16(out), ref, f"{nseq} x {seq}, {nq}q/{nk}kv, hd {hd}, causal {causal}")
    if ops.rope_fusable(seq, nq, nk):
        cs, sn = (t.cuda() for t in ops.rotary_tables(seq, hd))
        fused = torch.full_like(out, float("nan"))
        ops.attn_full_rope(qkv, fused, cs, sn, rows, seq, causal, nq, nk, hd, hd ** -0.5)
        rq = qkv.clone()
        ops.rope(rq, cs, sn, None, rows, seq, nq, nk, hd)
        pair = torch.full_like(out, float("nan"))
        ops.attn_full(rq, pair, rows, seq, causal, nq, nk, hd, hd ** -0.5)
        torch.cuda.synchronize()
        assert torch.equal(fused.view(torch.int16), pair.view(torch.int16)), "rope fused != rope then attention"
        q_h = _u16(qkv).copy()
        cpu.rope(q_h, cs.cpu().numpy(), sn.cpu().numpy(), None, rows, seq, nq, nk, hd)
        gc.assert_close(_u16(fused), cpu.attn_full(q_h, rows, seq, causal, nq, nk, hd, hd ** -0.5), "with rope")
    assert ops.device_error() == 0
