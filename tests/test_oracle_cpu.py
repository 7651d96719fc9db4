"""The CPU oracle against independent float64 numpy formulas, and the bf16 / seeded-input helpers (no GPU)."""
import numpy as np
import pytest

from oumu_b200 import synth
from oracle import cpu
import golden_cases as gc


def test_f2b_rounding_matches_reference_rule():
    # src/gpu.rs:72-78: round to nearest even on the upper 16 bits, NaN -> 0x7fc0
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, np.inf, -np.inf, np.nan, 0.0, -0.0, 3.0e38],
                 np.float32)
    h = synth.f32_to_bf16(x)
    assert h[0] == 0x3F80
    assert h[1] == 0x3F80            # tie -> even
    assert h[2] == 0x3F82            # tie -> even (up)
    assert h[3] == 0xC020
    assert h[4] == 0x7F80 and h[5] == 0xFF80
    assert h[6] == 0x7FC0
    assert h[7] == 0x0000 and h[8] == 0x8000
    assert synth.bf16_to_f32(h[:1])[0] == 1.0


def test_synth_is_deterministic_and_normal():
    a = synth.normal_bf16(7, (1000, 64))
    b = synth.normal_bf16(7, (1000, 64))
    c = synth.normal_bf16(8, (1000, 64))
    assert (a == b).all() and not (a == c).all()
    f = synth.bf16_to_f32(a)
    assert abs(f.mean()) < 0.02 and abs(f.std() - 1.0) < 0.02
    lens = synth.uniform_int(synth.config_seed(1), 64, 330, 4096)
    assert lens.min() >= 330 and lens.max() <= 4096 and len(set(lens.tolist())) > 50


def _attn_np(q, k, v, scale):
    s = (q.astype(np.float64) @ k.astype(np.float64).T) * scale
    s -= s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    return (p @ v.astype(np.float64)) / p.sum(axis=-1, keepdims=True)


@pytest.mark.parametrize("seq,causal,nq,nk,hd", [(11, 0, 16, 2, 128), (12, 0, 16, 16, 64), (37, 1, 4, 2, 128),
                                                 (5, 0, 16, 2, 128)])
def test_oracle_attn_full_vs_float64(seq, causal, nq, nk, hd):
    nseq = 3
    rows, W = nseq * seq, (nq + 2 * nk) * hd
    qkv = synth.normal_bf16(11, (rows, W))
    out = cpu.attn_full(qkv, rows, seq, causal, nq, nk, hd, 1 / np.sqrt(hd))
    f = synth.bf16_to_f32(qkv).reshape(rows, nq + 2 * nk, hd)
    ref = np.zeros((rows, nq, hd))
    for n in range(nseq):
        r0 = n * seq
        for h in range(nq):
            kh = h // (nq // nk)
            q, k, v = f[r0:r0 + seq, h], f[r0:r0 + seq, nq + kh], f[r0:r0 + seq, nq + nk + kh]
            for i in range(seq):
                L = i + 1 if causal else seq
                ref[r0 + i, h] = _attn_np(q[i:i + 1], k[:L], v[:L], 1 / np.sqrt(hd))[0]
    gc.assert_close(out, synth.f32_to_bf16(ref.reshape(rows, -1).astype(np.float32)), "attn_full")


def test_oracle_attn_decode_vs_float64():
    B, nq, nk, hd, maxlen = 3, 16, 2, 128, 256
    lens = np.array([1, 65, 256], np.int32)
    W = (nq + 2 * nk) * hd
    qkv = synth.normal_bf16(21, (B, W))
    kc = synth.normal_bf16(22, (B, nk, maxlen, hd))
    vc = synth.normal_bf16(23, (B, nk, maxlen, hd))
    out = cpu.attn_decode(qkv, kc, vc, None, lens, B, nq, nk, hd, maxlen, 1 / np.sqrt(hd))
    qf = synth.bf16_to_f32(qkv).reshape(B, nq + 2 * nk, hd)
    kf, vf = synth.bf16_to_f32(kc), synth.bf16_to_f32(vc)
    ref = np.zeros((B, nq, hd))
    for s in range(B):
        for h in range(nq):
            kh = h // (nq // nk)
            ref[s, h] = _attn_np(qf[s, h][None], kf[s, kh, :lens[s]], vf[s, kh, :lens[s]], 1 / np.sqrt(hd))[0]
    gc.assert_close(out, synth.f32_to_bf16(ref.reshape(B, -1).astype(np.float32)), "attn_decode")
    # shared position (the reference's *pos): every take uses L = pos + 1
    out2 = cpu.attn_decode(qkv, kc, vc, 99, None, B, nq, nk, hd, maxlen, 1 / np.sqrt(hd))
    out3 = cpu.attn_decode(qkv, kc, vc, None, np.full(B, 100, np.int32), B, nq, nk, hd, maxlen, 1 / np.sqrt(hd))
    gc.assert_exact(out2, out3, "pos vs lens")


def test_oracle_rope_formula():
    rows, nq, nk, hd, seq = 6, 2, 1, 128, 3
    W = (nq + 2 * nk) * hd
    qkv = synth.normal_bf16(31, (rows, W))
    cs, sn = cpu.rotary_tables(seq, hd)
    out = qkv.copy()
    cpu.rope(out, cs, sn, None, rows, seq, nq, nk, hd)
    f = synth.bf16_to_f32(qkv).reshape(rows, nq + 2 * nk, hd).astype(np.float64)
    o = synth.bf16_to_f32(out).reshape(rows, nq + 2 * nk, hd).astype(np.float64)
    half = hd // 2
    for r in range(rows):
        p = r % seq
        c, s = cs[p].astype(np.float64), sn[p].astype(np.float64)
        x1, x2 = f[r, :nq + nk, :half], f[r, :nq + nk, half:]
        assert np.abs(o[r, :nq + nk, :half] - (x1 * c - x2 * s)).max() < 0.02
        assert np.abs(o[r, :nq + nk, half:] - (x2 * c + x1 * s)).max() < 0.02
    # v heads untouched
    assert (out.reshape(rows, -1, hd)[:, nq + nk:] == qkv.reshape(rows, -1, hd)[:, nq + nk:]).all()


def test_oracle_rotary_tables_values():
    cs, sn = cpu.rotary_tables(4096, 128)
    # position 0: cos 1, sin 0; values are bf16-representable
    assert (cs[0] == 1).all() and (sn[0] == 0).all()
    assert (synth.bf16_to_f32(synth.f32_to_bf16(cs)) == cs).all()
    p, i = 1000, 5
    fr = np.float32(p) * np.float32(1.0 / np.float32(10000.0) ** np.float32(2 * i / 128))
    assert abs(cs[p, i] - np.cos(np.float64(fr))) < 4e-3


def test_oracle_kv_write_and_replicate_indexing():
    c = dict(kind="kv_rep", B=4, T=9, nq=4, nk=2, hd=64, maxlen=16, seed=5)
    x = gc.inputs(c)
    res = gc.run_oracle(c, x)
    q = x["qkv"].reshape(c["T"], c["nq"] + 2 * c["nk"], c["hd"])
    for s in range(c["B"]):
        for h in range(c["nk"]):
            assert (res["kc"][s, h, :c["T"]] == q[:, c["nq"] + h]).all()
            assert (res["vc"][s, h, :c["T"]] == q[:, c["nq"] + c["nk"] + h]).all()
            assert (res["kc"][s, h, c["T"]:] == 0).all()
    c2 = dict(kind="kv_write", slots=2, rows=1, pos=7, nq=4, nk=2, hd=64, maxlen=16, seed=6)
    x2 = gc.inputs(c2)
    r2 = gc.run_oracle(c2, x2)
    q2 = x2["qkv"].reshape(2, c2["nq"] + 2 * c2["nk"], c2["hd"])
    assert (r2["kc"][1, 1, 7] == q2[1, c2["nq"] + 1]).all()
    assert (r2["kc"].reshape(2, 2, 16, 64)[:, :, :7] == 0).all()
