"""Parity cases of the attention hot path: seeded inputs, and the same pipeline run by three implementations.

  ref     the reference's own kernels on the GPU (oracle/refkern.py; used by tests/golden/gen_golden.py to write
          the golden outputs under tests/golden/)
  oracle  the fp32 CPU restatement (oracle/cpu.py)
  ours    the sm_100a library through its C ABI (oumu_b200/ops.py)

Inputs are rebuilt from the seed (oumu_b200.synth), so a golden file holds only outputs.
Each case follows the reference's launch sequence for that path (src/model.rs):
  rope      rope on a fused qkv buffer (prefill/DiT positions r % seq, or one decode position)
  kv_write  k/v of rows into cache slots at a position
  kv_rep    kv_write of a T-row prompt into slot 0, then kv_replicate to every slot (src/model.rs:553-559,705-717)
  decode    per take: prompt rows roped at their positions and written to the take's slot, then one decode query
            (the last row) against L_s cached positions (config 1 shape: one take, 512 of 4096 positions)
  full      (optional rope with seq) then attn_full over independent sequences
"""
import numpy as np

from oumu_b200 import synth

CASES = {
    "rope_decode": dict(kind="rope", rows=8, seq=0, pos=1234, nq=16, nk=2, hd=128, maxlen=4096, seed=101),
    "rope_prefill": dict(kind="rope", rows=36, seq=12, pos=None, nq=16, nk=2, hd=128, maxlen=64, seed=102),
    "rope_hd64": dict(kind="rope", rows=24, seq=12, pos=None, nq=16, nk=16, hd=64, maxlen=64, seed=103),
    "kv_write_decode": dict(kind="kv_write", slots=3, rows=1, pos=77, nq=16, nk=2, hd=128, maxlen=128, seed=104),
    "kv_write_prefill": dict(kind="kv_write", slots=1, rows=40, pos=None, nq=16, nk=2, hd=128, maxlen=64, seed=105),
    "kv_rep": dict(kind="kv_rep", B=5, T=70, nq=16, nk=2, hd=128, maxlen=128, seed=106),
    # one take, 16 q / 2 kv heads, hd 128, 512 valid positions of a 4096-position slot
    "decode_c1": dict(kind="decode", lens=[512], maxlen=4096, nq=16, nk=2, hd=128, seed=synth.config_seed(0)),
    "decode_lens": dict(kind="decode", lens=[1, 63, 64, 65, 200, 256], maxlen=256, nq=16, nk=2, hd=128, seed=107),
    "decode_hd64_g4": dict(kind="decode", lens=[5, 129, 100], maxlen=192, nq=8, nk=2, hd=64, seed=108),
    "decode_mha": dict(kind="decode", lens=[77, 300], maxlen=320, nq=4, nk=4, hd=128, seed=109),
    # causal prefill (rope at r % seq), two 128-row tiles with a ragged tail
    "full_prefill": dict(kind="full", nseq=1, seq=160, causal=1, rope=1, nq=16, nk=2, hd=128, seed=110),
    "full_two_seqs": dict(kind="full", nseq=2, seq=40, causal=1, rope=1, nq=16, nk=2, hd=128, seed=111),
    "full_noncausal_64": dict(kind="full", nseq=2, seq=48, causal=0, rope=0, nq=4, nk=1, hd=64, seed=112),
    # LocDiT, reference shape: 11 tokens, 16 q / 2 kv heads, hd 128 (src/model.rs:22, kernels/voxcpm.cu:299-301)
    "full_locdit_ref": dict(kind="full", nseq=8, seq=11, causal=0, rope=1, nq=16, nk=2, hd=128, seed=113),
    # LocDiT, BASELINE config 4 shape: 12 tokens, 16 heads, hd 64, no mask
    "full_locdit_c4": dict(kind="full", nseq=8, seq=12, causal=0, rope=0, nq=16, nk=16, hd=64, seed=synth.config_seed(3)),
    # local encoder: 5 tokens (src/model.rs:21)
    "full_locenc": dict(kind="full", nseq=6, seq=5, causal=0, rope=1, nq=16, nk=2, hd=128, seed=114),
}


def width(c):
    return (c["nq"] + 2 * c["nk"]) * c["hd"]


def inputs(c):
    """Seeded inputs of case c (numpy; bf16 as uint16)."""
    W = width(c)
    k = c["kind"]
    if k == "rope":
        return dict(qkv=synth.normal_bf16(c["seed"], (c["rows"], W)))
    if k == "kv_write":
        return dict(qkv=synth.normal_bf16(c["seed"], (c["slots"] * c["rows"], W)))
    if k == "kv_rep":
        return dict(qkv=synth.normal_bf16(c["seed"], (c["T"], W)))
    if k == "decode":
        return dict(prompts=[synth.normal_bf16(c["seed"] * 1000 + s, (L, W)) for s, L in enumerate(c["lens"])])
    if k == "full":
        return dict(qkv=synth.normal_bf16(c["seed"], (c["nseq"] * c["seq"], W)))
    raise ValueError(k)


def scale(c):
    return 1.0 / float(np.sqrt(c["hd"]))


def cache_shape(c, slots):
    return (slots, c["nk"], c["maxlen"], c["hd"])


# ------------------------------------------------------------------------------------------------------------
# oracle pipeline (CPU)
# ------------------------------------------------------------------------------------------------------------

def run_oracle(c, x=None):
    from oracle import cpu
    x = inputs(c) if x is None else x
    k, nq, nk, hd = c["kind"], c["nq"], c["nk"], c["hd"]
    if k == "rope":
        cs, sn = cpu.rotary_tables(c["maxlen"], hd)
        q = x["qkv"].copy()
        cpu.rope(q, cs, sn, c["pos"], c["rows"], c["seq"], nq, nk, hd)
        return dict(qkv=q)
    if k == "kv_write":
        kc = np.zeros(cache_shape(c, c["slots"]), np.uint16)
        vc = np.zeros_like(kc)
        cpu.kv_write(x["qkv"], kc, vc, c["pos"], c["slots"], c["rows"], nq, nk, hd, c["maxlen"])
        return dict(kc=kc, vc=vc)
    if k == "kv_rep":
        kc = np.zeros(cache_shape(c, c["B"]), np.uint16)
        vc = np.zeros_like(kc)
        cpu.kv_write(x["qkv"], kc, vc, None, 1, c["T"], nq, nk, hd, c["maxlen"])
        cpu.kv_replicate(kc, c["B"], nk, c["maxlen"], hd, c["T"])
        cpu.kv_replicate(vc, c["B"], nk, c["maxlen"], hd, c["T"])
        return dict(kc=kc, vc=vc)
    if k == "decode":
        B, maxlen = len(c["lens"]), c["maxlen"]
        cs, sn = cpu.rotary_tables(maxlen, hd)
        kc = np.zeros(cache_shape(c, B), np.uint16)
        vc = np.zeros_like(kc)
        rows = []
        for s, (L, pr) in enumerate(zip(c["lens"], x["prompts"])):
            q = pr.copy()
            cpu.rope(q, cs, sn, None, L, L, nq, nk, hd)
            kcs, vcs = kc[s:s + 1].copy(), vc[s:s + 1].copy()
            cpu.kv_write(q, kcs, vcs, None, 1, L, nq, nk, hd, maxlen)
            kc[s], vc[s] = kcs[0], vcs[0]
            rows.append(q[L - 1])
        qkv = np.stack(rows)
        out = cpu.attn_decode(qkv, kc, vc, None, np.array(c["lens"], np.int32), B, nq, nk, hd, maxlen, scale(c))
        return dict(out=out)
    if k == "full":
        rows = c["nseq"] * c["seq"]
        q = x["qkv"].copy()
        if c["rope"]:
            cs, sn = cpu.rotary_tables(c["seq"], hd)
            cpu.rope(q, cs, sn, None, rows, c["seq"], nq, nk, hd)
        return dict(out=cpu.attn_full(q, rows, c["seq"], c["causal"], nq, nk, hd, scale(c)))
    raise ValueError(k)


# ------------------------------------------------------------------------------------------------------------
# GPU pipelines: the reference kernels (impl="ref") or this library (impl="ours")
# ------------------------------------------------------------------------------------------------------------

def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda()


def _host(t):
    return t.cpu().numpy().view(np.uint16)


def run_gpu(c, impl, x=None):
    import torch
    x = inputs(c) if x is None else x
    fused = impl == "ours_fused"
    if impl == "ref":
        from oracle import refkern as K
    else:
        from oumu_b200 import ops as K
    from oracle import cpu  # rotary tables for the reference path (the reference builds them on the host too)
    k, nq, nk, hd = c["kind"], c["nq"], c["nk"], c["hd"]

    def tables(maxlen):
        if impl == "ref":
            cs, sn = cpu.rotary_tables(maxlen, hd)
            return torch.from_numpy(cs).cuda(), torch.from_numpy(sn).cuda()
        cs, sn = K.rotary_tables(maxlen, hd)
        return cs.cuda(), sn.cuda()

    def ipos(v):
        return None if v is None else torch.tensor([v], dtype=torch.int32, device="cuda")

    if k == "rope":
        cs, sn = tables(c["maxlen"])
        q = _dev(x["qkv"])
        K.rope(q, cs, sn, ipos(c["pos"]), c["rows"], c["seq"], nq, nk, hd)
        torch.cuda.synchronize()
        return dict(qkv=_host(q))
    if k == "kv_write":
        q = _dev(x["qkv"])
        kc = torch.zeros(cache_shape(c, c["slots"]), dtype=torch.int16, device="cuda")
        vc = torch.zeros_like(kc)
        K.kv_write(q, kc, vc, ipos(c["pos"]), c["slots"], c["rows"], nq, nk, hd, c["maxlen"])
        torch.cuda.synchronize()
        return dict(kc=_host(kc), vc=_host(vc))
    if k == "kv_rep":
        q = _dev(x["qkv"])
        kc = torch.zeros(cache_shape(c, c["B"]), dtype=torch.int16, device="cuda")
        vc = torch.zeros_like(kc)
        K.kv_write(q, kc, vc, None, 1, c["T"], nq, nk, hd, c["maxlen"])
        K.kv_replicate(kc, c["B"], nk, c["maxlen"], hd, c["T"])
        K.kv_replicate(vc, c["B"], nk, c["maxlen"], hd, c["T"])
        torch.cuda.synchronize()
        return dict(kc=_host(kc), vc=_host(vc))
    if k == "decode":
        lens, maxlen = c["lens"], c["maxlen"]
        B = len(lens)
        cs, sn = tables(maxlen)
        kc = torch.zeros(cache_shape(c, B), dtype=torch.int16, device="cuda")
        vc = torch.zeros_like(kc)
        qkv = torch.zeros((B, width(c)), dtype=torch.int16, device="cuda")
        for s, (L, pr) in enumerate(zip(lens, x["prompts"])):
            q = _dev(pr)
            if fused:
                # positions < L-1 as a prefill would leave them; the newest row goes through the fused decode step
                if L > 1:
                    K.rope(q, cs, sn, None, L - 1, L, nq, nk, hd)
                    K.kv_write(q, kc[s:s + 1], vc[s:s + 1], None, 1, L - 1, nq, nk, hd, maxlen)
                qkv[s] = q[L - 1]
                continue
            K.rope(q, cs, sn, None, L, L, nq, nk, hd)
            K.kv_write(q, kc[s:s + 1], vc[s:s + 1], None, 1, L, nq, nk, hd, maxlen)
            qkv[s] = q[L - 1]
        att = torch.zeros((B, nq * hd), dtype=torch.int16, device="cuda")
        if fused:
            ws = K.decode_workspace(B, nq, nk, hd, maxlen)
            ln = torch.tensor(lens, dtype=torch.int32, device="cuda")
            K.attn_decode_step(qkv, kc, vc, att, ws, cs, sn, None, ln, B, nq, nk, hd, maxlen, scale(c))
        elif impl == "ref":
            part = torch.zeros(B * nq * (maxlen // 64) * (hd + 2), dtype=torch.float32, device="cuda")
            K.attn_decode_per_take(qkv, kc, vc, part, att, lens, B, nq, nk, hd, maxlen, scale(c))
        else:
            ws = K.decode_workspace(B, nq, nk, hd, maxlen)
            ln = torch.tensor(lens, dtype=torch.int32, device="cuda")
            K.attn_decode(qkv, kc, vc, att, ws, None, ln, B, nq, nk, hd, maxlen, scale(c))
        torch.cuda.synchronize()
        return dict(out=_host(att))
    if k == "full":
        rows = c["nseq"] * c["seq"]
        q = _dev(x["qkv"])
        if c["rope"]:
            cs, sn = tables(c["seq"])
            K.rope(q, cs, sn, None, rows, c["seq"], nq, nk, hd)
        out = torch.zeros((rows, nq * hd), dtype=torch.int16, device="cuda")
        K.attn_full(q, out, rows, c["seq"], c["causal"], nq, nk, hd, scale(c))
        torch.cuda.synchronize()
        return dict(out=_host(out))
    raise ValueError(k)


# ------------------------------------------------------------------------------------------------------------
# comparison
# ------------------------------------------------------------------------------------------------------------

ATOL = 2e-3   # north_star tolerance on bf16 outputs: max abs error 2e-3 ...
RTOL = 1e-2   # ... and max relative error 1e-2 (element-wise |a - b| <= ATOL + RTOL * |b|)


def _ordered(u):
    """bf16 bit patterns (uint16) mapped to integers that count representable values in order (+0 and -0 both 0), so
    that |ordered(a) - ordered(b)| is the distance of a and b in bf16 ulps."""
    u = np.asarray(u).astype(np.int64)
    mag = u & 0x7FFF
    return np.where(u & 0x8000, -mag, mag)


def compare(got, ref, atol=ATOL, rtol=RTOL):
    """Statistics of got vs ref (uint16 bf16 arrays): max abs error, max relative error over |ref| >= 1e-2,
    count of elements outside |got - ref| <= atol + rtol * |ref|, exact-match fraction, and the elements whose
    |got - ref| exceeds atol split into those exactly one bf16 ulp from ref and those further away."""
    g = synth.bf16_to_f32(got).astype(np.float64)
    r = synth.bf16_to_f32(ref).astype(np.float64)
    d = np.abs(g - r)
    big = np.abs(r) >= 1e-2
    over = d > atol
    ulps = np.abs(_ordered(got) - _ordered(ref))
    return dict(
        max_abs=float(d.max()) if d.size else 0.0,
        max_rel=float((d[big] / np.abs(r[big])).max()) if big.any() else 0.0,
        bad=int((d > atol + rtol * np.abs(r)).sum()),
        exact=float((np.asarray(got) == np.asarray(ref)).mean()) if d.size else 1.0,
        n=int(d.size),
        nonfinite=int((~np.isfinite(g)).sum()),
        over_atol=int(over.sum()),
        over_atol_1ulp=int((over & (ulps == 1)).sum()),
        over_atol_more=int((over & (ulps > 1)).sum()),
        max_ulp_over_atol=int(ulps[over].max()) if over.any() else 0,
    )


# Statistics of every tolerance comparison made in this process, by label (printed at the end of the pytest run by
# tests/conftest.py, and written as JSON to $OUMU_PARITY_STATS when that is set).
STATS = {}


def _label(what):
    import os
    test = os.environ.get("PYTEST_CURRENT_TEST", "").split(" ")[0]
    test = test[len("tests/"):] if test.startswith("tests/") else test
    test = test.replace(".py::", "::")
    return f"{test} {what}".strip()


def assert_close(got, ref, what="", atol=ATOL, rtol=RTOL):
    st = compare(got, ref, atol, rtol)
    STATS[_label(what)] = st
    assert st["nonfinite"] == 0 and st["bad"] == 0, f"{what}: {st}"
    return st


def assert_exact(got, ref, what=""):
    got, ref = np.asarray(got), np.asarray(ref)
    assert got.shape == ref.shape, f"{what}: shape {got.shape} vs {ref.shape}"
    n = int((got != ref).sum())
    assert n == 0, f"{what}: {n} of {got.size} elements differ"
