"""The prefill with its KV epilogue (oumu_attn_prefill_kv): the attention output is bit-identical to oumu_attn_full's,
and every take slot holds, bit for bit, what kv_write into slot 0 followed by kv_replicate leaves there
(src/model.rs:553-567,705-717), with every position past the prompt untouched."""
import pytest
import torch

from oumu_b200 import ops

pytestmark = pytest.mark.gpu


def rnd(shape, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(shape, generator=g, device="cuda").to(torch.bfloat16)


CASES = [
    # T, slots, nq, nk, hd, maxlen
    (1024, 64, 16, 2, 128, 4096),  # config 3
    (200, 5, 16, 2, 128, 256),     # ragged prompt, a few takes
    (17, 3, 16, 2, 128, 64),       # the shortest prompt on the tensor-core path
    (300, 9, 8, 8, 64, 512),       # hd 64, one q head per kv head
    (129, 1, 16, 2, 128, 129),     # one slot, prompt filling the slot, a one-row last tile
]


@pytest.mark.parametrize("T,slots,nq,nk,hd,maxlen", CASES)
def test_prefill_kv_matches_separate_launches(cuda, T, slots, nq, nk, hd, maxlen):
    W = (nq + 2 * nk) * hd
    qkv = rnd((T, W), 1)
    scale = hd ** -0.5
    # reference: attention, then k/v into slot 0 and replicated into the other slots
    want_out = torch.empty((T, nq * hd), dtype=torch.bfloat16, device="cuda")
    ops.attn_full(qkv, want_out, T, T, 1, nq, nk, hd, scale)
    sentinel_k, sentinel_v = rnd((slots, nk, maxlen, hd), 2), rnd((slots, nk, maxlen, hd), 3)
    want_k, want_v = sentinel_k.clone(), sentinel_v.clone()
    ops.kv_write(qkv, want_k, want_v, None, 1, T, nq, nk, hd, maxlen)
    ops.kv_replicate(want_k, slots, nk, maxlen, hd, T)
    ops.kv_replicate(want_v, slots, nk, maxlen, hd, T)
    # one launch
    out = torch.full((T, nq * hd), 3.0, dtype=torch.bfloat16, device="cuda")
    kc, vc = sentinel_k.clone(), sentinel_v.clone()
    ops.attn_prefill_kv(qkv, out, kc, vc, T, slots, nq, nk, hd, maxlen, scale)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), want_out.view(torch.int16))
    assert torch.equal(kc.view(torch.int16), want_k.view(torch.int16))
    assert torch.equal(vc.view(torch.int16), want_v.view(torch.int16))
    assert torch.equal(kc[:, :, T:].view(torch.int16), sentinel_k[:, :, T:].view(torch.int16))
    assert ops.device_error() == 0


def test_prefill_kv_rejects_short_prompts(cuda):
    from oumu_b200 import _lib
    qkv = rnd((16, 20 * 128), 4)
    out = torch.empty((16, 16 * 128), dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros((2, 2, 64, 128), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.OumuError):
        ops.attn_prefill_kv(qkv, out, kc, kc.clone(), 16, 2, 16, 2, 128, 64, 128 ** -0.5)


def test_prefill_kv_config3_repeated(cuda):
    """Config 3 called twelve times on fresh inputs, each output bit-identical to oumu_attn_full's. The planned
    epilogue (copy CTAs, stores spread over the query tiles) changes when the V loads land; a wait for the last P.V
    that could pass on the P.V before it once showed here as a wrong query tile in 2 of 6 calls."""
    T, slots, nq, nk, hd, maxlen = 1024, 64, 16, 2, 128, 4096
    scale = hd ** -0.5
    k = torch.zeros((slots, nk, maxlen, hd), dtype=torch.bfloat16, device="cuda")
    v = torch.zeros_like(k)
    for trial in range(12):
        qkv = rnd((T, (nq + 2 * nk) * hd), 100 + trial)
        want = torch.empty((T, nq * hd), dtype=torch.bfloat16, device="cuda")
        ops.attn_full(qkv, want, T, T, 1, nq, nk, hd, scale)
        got = torch.zeros_like(want)
        ops.attn_prefill_kv(qkv, got, k, v, T, slots, nq, nk, hd, maxlen, scale)
        torch.cuda.synchronize()
        bad = (got != want).view(T // 128, 128, -1).any(dim=2).any(dim=1)
        assert not bad.any(), f"call {trial}: query tiles {bad.nonzero().flatten().tolist()} differ"
        kref = qkv[:, nq * hd:(nq + nk) * hd].view(T, nk, hd).permute(1, 0, 2)
        vref = qkv[:, (nq + nk) * hd:].view(T, nk, hd).permute(1, 0, 2)
        assert torch.equal(k[:, :, :T], kref.expand(slots, -1, -1, -1)), f"call {trial}: k slots"
        assert torch.equal(v[:, :, :T], vref.expand(slots, -1, -1, -1)), f"call {trial}: v slots"


def _sweep_cases(n=16, seed=5):
    import random
    rng = random.Random(seed)
    out = []
    for _ in range(n):
        nq, nk = rng.choice([(16, 2), (8, 8), (32, 4), (16, 16), (8, 1), (24, 3)])
        T = rng.choice([17, 100, 129, 200, 255, 384, 511, 640, 900, 1024, 1100, 1500])
        out.append((T, rng.choice([1, 2, 3, 5, 9, 17, 33, 64, 96]), nq, nk, rng.choice([64, 128]),
                    T + rng.choice([0, 1, 7, 64, 300])))
    return out


@pytest.mark.parametrize("T,slots,nq,nk,hd,maxlen", _sweep_cases())
def test_prefill_kv_random_shapes(cuda, T, slots, nq, nk, hd, maxlen):
    """Seeded random shapes through both KV epilogues (the planned one where the grid and its copy CTAs fit on the
    SMs at once, the mirror scheme elsewhere): bit-identical to attn_full + kv_write + kv_replicate."""
    W = (nq + 2 * nk) * hd
    scale = hd ** -0.5
    qkv = rnd((T, W), T + slots)
    want = torch.empty((T, nq * hd), dtype=torch.bfloat16, device="cuda")
    ops.attn_full(qkv, want, T, T, 1, nq, nk, hd, scale)
    k0, v0 = rnd((slots, nk, maxlen, hd), 7), rnd((slots, nk, maxlen, hd), 8)
    wk, wv = k0.clone(), v0.clone()
    ops.kv_write(qkv, wk, wv, None, 1, T, nq, nk, hd, maxlen)
    ops.kv_replicate(wk, slots, nk, maxlen, hd, T)
    ops.kv_replicate(wv, slots, nk, maxlen, hd, T)
    got, gk, gv = torch.zeros_like(want), k0.clone(), v0.clone()
    ops.attn_prefill_kv(qkv, got, gk, gv, T, slots, nq, nk, hd, maxlen, scale)
    torch.cuda.synchronize()
    assert torch.equal(got, want), "attention output"
    assert torch.equal(gk, wk) and torch.equal(gv, wv), "slots"
