"""Rope + small-sequence attention in one launch (oumu_attn_full_rope): the output is bit-identical to oumu_rope
followed by oumu_attn_full (the launch pair of Engine::full, src/model.rs:541-567), and qkv is left unrotated."""
import pytest
import torch

from oumu_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def rnd(shape, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(shape, generator=g, device="cuda").to(torch.bfloat16)


CASES = [
    # nseq, seq, causal, nq, nk, hd
    (64, 11, 0, 16, 2, 128),   # the DiT (2 CFG branches x 32 takes, 11 tokens)
    (32, 5, 0, 16, 2, 128),    # the local encoder (5 tokens)
    (9, 16, 1, 16, 2, 128),    # 128 stacked rows, causal
    (17, 7, 0, 8, 2, 64),      # hd 64, group of 4
    (3, 1, 0, 4, 2, 128),      # one token
]


@pytest.mark.parametrize("nseq,seq,causal,nq,nk,hd", CASES)
def test_attn_full_rope_matches_rope_then_attention(cuda, nseq, seq, causal, nq, nk, hd):
    rows, W = nseq * seq, (nq + 2 * nk) * hd
    cs, sn = ops.rotary_tables(64, hd)
    cs, sn = cs.cuda(), sn.cuda()
    qkv = rnd((rows, W), 7)
    scale = hd ** -0.5
    ref_qkv = qkv.clone()
    want = torch.empty((rows, nq * hd), dtype=torch.bfloat16, device="cuda")
    ops.rope(ref_qkv, cs, sn, None, rows, seq, nq, nk, hd)
    ops.attn_full(ref_qkv, want, rows, seq, causal, nq, nk, hd, scale)
    got = torch.full((rows, nq * hd), 5.0, dtype=torch.bfloat16, device="cuda")
    before = qkv.clone()
    ops.attn_full_rope(qkv, got, cs, sn, rows, seq, causal, nq, nk, hd, scale)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    assert torch.equal(qkv.view(torch.int16), before.view(torch.int16))
    assert ops.device_error() == 0


def test_full_attention_takes_the_fused_launch(cuda):
    # the engine's call (DiT shape): same output as the explicit two-launch sequence
    rows, seq, nq, nk, hd = 22 * 11, 11, 16, 2, 128
    cs, sn = ops.rotary_tables(64, hd)
    cs, sn = cs.cuda(), sn.cuda()
    qkv = rnd((rows, (nq + 2 * nk) * hd), 8)
    a, b = (torch.empty((rows, nq * hd), dtype=torch.bfloat16, device="cuda") for _ in range(2))
    ref_qkv = qkv.clone()
    ops.rope(ref_qkv, cs, sn, None, rows, seq, nq, nk, hd)
    ops.attn_full(ref_qkv, a, rows, seq, 0, nq, nk, hd, hd ** -0.5)
    ops.full_attention(qkv, b, rows, seq, 0, nq, nk, hd, cos_t=cs, sin_t=sn)
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


@pytest.mark.parametrize("seq,nq,nk", [(17, 16, 2), (11, 16, 16), (16, 32, 2)])
def test_attn_full_rope_rejects_other_shapes(cuda, seq, nq, nk):
    hd = 128
    cs, sn = ops.rotary_tables(64, hd)
    cs, sn = cs.cuda(), sn.cuda()
    qkv = rnd((2 * seq, (nq + 2 * nk) * hd), 9)
    out = torch.empty((2 * seq, nq * hd), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.OumuError):
        ops.attn_full_rope(qkv, out, cs, sn, 2 * seq, seq, 0, nq, nk, hd, hd ** -0.5)
