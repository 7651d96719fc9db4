"""The kernels at the benchmark configurations' full sizes and at the edges the reference handles: per-take lengths
1 .. maxlen, maxlen 65536, ragged prefill lengths, the reference-sized workspace, CUDA-graph replay with positions
read on the device, determinism, and the device error word."""
import numpy as np
import pytest
import torch

import golden_cases as gc
from oumu_b200 import ops, synth
from oracle import cpu

pytestmark = pytest.mark.gpu

NQ, NK, HD = 16, 2, 128


def rand_bf16(shape, seed, device="cuda"):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.randn(shape, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)


def u16(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def decode_case(B, lens, maxlen, nq=NQ, nk=NK, hd=HD, seed=0):
    qkv = rand_bf16((B, (nq + 2 * nk) * hd), seed)
    kc = rand_bf16((B, nk, maxlen, hd), seed + 1)
    vc = rand_bf16((B, nk, maxlen, hd), seed + 2)
    ln = torch.tensor(lens, dtype=torch.int32, device="cuda")
    return qkv, kc, vc, ln


def run_decode(qkv, kc, vc, ln, B, maxlen, nq=NQ, nk=NK, hd=HD, ws=None):
    att = torch.zeros((B, nq * hd), dtype=torch.bfloat16, device="cuda")
    ws = ops.decode_workspace(B, nq, nk, hd, maxlen) if ws is None else ws
    ops.attn_decode(qkv, kc, vc, att, ws, None, ln, B, nq, nk, hd, maxlen, hd ** -0.5)
    torch.cuda.synchronize()
    return att, ws


def oracle_decode(qkv, kc, vc, lens, B, maxlen, nq=NQ, nk=NK, hd=HD):
    return cpu.attn_decode(u16(qkv), u16(kc), u16(vc), None, np.asarray(lens, np.int32), B, nq, nk, hd, maxlen,
                           hd ** -0.5)


def test_decode_config2_layer_vs_oracle(cuda):
    # BASELINE config 2, one layer: 64 takes, slots of 4096, lengths uniform in [330, 4096]
    B, maxlen = 64, 4096
    lens = synth.uniform_int(synth.config_seed(1), B, 330, 4096)
    qkv, kc, vc, ln = decode_case(B, lens, maxlen, seed=10)
    att, ws = run_decode(qkv, kc, vc, ln, B, maxlen)
    gc.assert_close(u16(att), oracle_decode(qkv, kc, vc, lens, B, maxlen), "config 2 layer")
    # the combine counters are left at zero, and a second call is bit-identical
    cnt = ws[: B * NK * 4].view(torch.int32)
    assert int(cnt.abs().sum()) == 0
    att2, _ = run_decode(qkv, kc, vc, ln, B, maxlen, ws=ws)
    assert torch.equal(att.view(torch.int16), att2.view(torch.int16))


def test_decode_config2_layers_back_to_back(cuda):
    # several layers launched back to back on one workspace, as in a step: every output checked
    B, maxlen, layers = 64, 4096, 4
    lens = synth.uniform_int(synth.config_seed(1), B, 330, 4096)
    data = [decode_case(B, lens, maxlen, seed=200 + 10 * l) for l in range(layers)]
    ws = ops.decode_workspace(B, NQ, NK, HD, maxlen)
    outs = [torch.zeros((B, NQ * HD), dtype=torch.bfloat16, device="cuda") for _ in range(layers)]
    for _ in range(3):
        for l, (qkv, kc, vc, ln) in enumerate(data):
            ops.attn_decode(qkv, kc, vc, outs[l], ws, None, ln, B, NQ, NK, HD, maxlen, HD ** -0.5)
    torch.cuda.synchronize()
    for l, (qkv, kc, vc, _) in enumerate(data):
        gc.assert_close(u16(outs[l]), oracle_decode(qkv, kc, vc, lens, B, maxlen), f"layer {l}")
    assert int(ws[: B * NK * 4].view(torch.int32).abs().sum()) == 0


def test_decode_bit_identical_whatever_the_merge_path(cuda):
    # The last contributor of a segment split across CTAs merges from its own registers when the others have
    # published first, else through its own record: which one happens depends on timing. Launches of one layer in a
    # graph of programmatically dependent launches (the timing of a step) all give the bits of one eager launch.
    B, maxlen, reps = 64, 4096, 4
    lens = synth.uniform_int(synth.config_seed(1), B, 330, 4096)
    qkv, kc, vc, ln = decode_case(B, lens, maxlen, seed=33)
    want, ws = run_decode(qkv, kc, vc, ln, B, maxlen)
    outs = [torch.zeros_like(want) for _ in range(reps)]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    prev = ops.set_pdl(True)
    try:
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for o in outs:
                    ops.attn_decode(qkv, kc, vc, o, ws, None, ln, B, NQ, NK, HD, maxlen, HD ** -0.5)
    finally:
        ops.set_pdl(prev)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(16):
        for o in outs:
            o.zero_()
        g.replay()
        torch.cuda.synchronize()
        for o in outs:
            assert torch.equal(o.view(torch.int16), want.view(torch.int16))
    assert int(ws[: B * NK * 4].view(torch.int32).abs().sum()) == 0
    del g


@pytest.mark.parametrize("nq,nk,hd", [(16, 2, 128), (16, 2, 64), (8, 8, 128), (12, 4, 64), (7, 1, 128)])
def test_decode_shapes_and_lengths(cuda, nq, nk, hd):
    maxlen = 640
    lens = [1, 2, 63, 64, 65, 127, 128, 129, 333, 639, 640]
    B = len(lens)
    qkv, kc, vc, ln = decode_case(B, lens, maxlen, nq, nk, hd, seed=20)
    att, _ = run_decode(qkv, kc, vc, ln, B, maxlen, nq, nk, hd)
    gc.assert_close(u16(att), oracle_decode(qkv, kc, vc, lens, B, maxlen, nq, nk, hd), f"{nq}/{nk}/{hd}")


@pytest.mark.parametrize("B,maxlen,fused", [(256, 192, False), (1024, 64, False), (1024, 64, True)])
def test_decode_many_takes(cuda, B, maxlen, fused):
    # the reference's MAX_SLOTS (256, src/model.rs:25) and the engine's 1024 takes per GPU: every CTA range then
    # crosses many short segments (lengths 1 .. maxlen)
    lens = [int(v) for v in synth.uniform_int(1234 + B, B, 1, maxlen)]
    qkv, kc, vc, ln = decode_case(B, lens, maxlen, seed=40)
    if not fused:
        att, _ = run_decode(qkv, kc, vc, ln, B, maxlen)
        gc.assert_close(u16(att), oracle_decode(qkv, kc, vc, lens, B, maxlen), f"{B} takes")
        return
    # fused (no rope): the newest k/v go into each take's slot at lens - 1, then attention over [0, lens)
    qkv_h, kc_h, vc_h = u16(qkv), u16(kc), u16(vc)
    att = torch.zeros((B, NQ * HD), dtype=torch.bfloat16, device="cuda")
    ws = ops.decode_workspace(B, NQ, NK, HD, maxlen)
    ops.step_tf_attention(qkv, kc, vc, att, ws, None, None, None, ln, B, NQ, NK, HD, maxlen, rope_on=False)
    torch.cuda.synchronize()
    for t, L in enumerate(lens):
        kcs, vcs = np.ascontiguousarray(kc_h[t:t + 1]), np.ascontiguousarray(vc_h[t:t + 1])
        cpu.kv_write(np.ascontiguousarray(qkv_h[t:t + 1]), kcs, vcs, L - 1, 1, 1, NQ, NK, HD, maxlen)
        kc_h[t], vc_h[t] = kcs[0], vcs[0]
    assert np.array_equal(u16(kc), kc_h) and np.array_equal(u16(vc), vc_h)
    ref = cpu.attn_decode(qkv_h, kc_h, vc_h, None, np.asarray(lens, np.int32), B, NQ, NK, HD, maxlen, HD ** -0.5)
    gc.assert_close(u16(att), ref, f"{B} takes fused")


@pytest.mark.parametrize("maxlen,hd,fused", [(100, 128, False), (100, 128, True), (72, 64, False)])
def test_decode_slot_length_not_a_multiple_of_the_tile(cuda, maxlen, hd, fused):
    # slots of a length that is not a multiple of the 32-position tile: a segment's last tile reaches into the next
    # take's slot (masked) and, for the last take, past the end of the caches (the tensor map fills zeros)
    lens = [1, 31, 32, 33, maxlen - 1, maxlen, 64, maxlen]
    B = len(lens)
    qkv, kc, vc, ln = decode_case(B, lens, maxlen, hd=hd, seed=50 + maxlen)
    if not fused:
        att, _ = run_decode(qkv, kc, vc, ln, B, maxlen, hd=hd)
        gc.assert_close(u16(att), oracle_decode(qkv, kc, vc, lens, B, maxlen, hd=hd), f"maxlen {maxlen}")
        return
    qkv_h, kc_h, vc_h = u16(qkv), u16(kc), u16(vc)
    att = torch.zeros((B, NQ * hd), dtype=torch.bfloat16, device="cuda")
    ws = ops.decode_workspace(B, NQ, NK, hd, maxlen)
    ops.step_tf_attention(qkv, kc, vc, att, ws, None, None, None, ln, B, NQ, NK, hd, maxlen, rope_on=False)
    torch.cuda.synchronize()
    for t, L in enumerate(lens):
        kcs, vcs = np.ascontiguousarray(kc_h[t:t + 1]), np.ascontiguousarray(vc_h[t:t + 1])
        cpu.kv_write(np.ascontiguousarray(qkv_h[t:t + 1]), kcs, vcs, L - 1, 1, 1, NQ, NK, hd, maxlen)
        kc_h[t], vc_h[t] = kcs[0], vcs[0]
    assert np.array_equal(u16(kc), kc_h) and np.array_equal(u16(vc), vc_h)
    ref = cpu.attn_decode(qkv_h, kc_h, vc_h, None, np.asarray(lens, np.int32), B, NQ, NK, hd, maxlen, hd ** -0.5)
    gc.assert_close(u16(att), ref, f"maxlen {maxlen} fused")


def test_decode_rejects_takes_past_shared_memory(cuda):
    # the per-take tile prefix lives in shared memory: far more takes than the engine's 1024 are refused with
    # OUMU_ERR_UNSUPPORTED before any launch
    from oumu_b200 import _lib
    B, maxlen = 4096, 32
    qkv, kc, vc, ln = decode_case(B, [1] * B, maxlen, seed=41)
    att = torch.zeros((B, NQ * HD), dtype=torch.bfloat16, device="cuda")
    ws = ops.decode_workspace(B, NQ, NK, HD, maxlen)
    with pytest.raises(_lib.OumuError):
        ops.attn_decode(qkv, kc, vc, att, ws, None, ln, B, NQ, NK, HD, maxlen, HD ** -0.5)


def test_decode_shared_position_and_max_length(cuda):
    # the reference's form: one shared *pos for every take; and the longest KV the reference accepts (65536)
    B, maxlen = 2, 65536
    qkv, kc, vc, _ = decode_case(B, [maxlen] * B, maxlen, seed=30)
    att = torch.zeros((B, NQ * HD), dtype=torch.bfloat16, device="cuda")
    ws = ops.decode_workspace(B, NQ, NK, HD, maxlen)
    pos = torch.tensor([maxlen - 1], dtype=torch.int32, device="cuda")
    ops.attn_decode(qkv, kc, vc, att, ws, pos, None, B, NQ, NK, HD, maxlen, HD ** -0.5)
    torch.cuda.synchronize()
    gc.assert_close(u16(att), oracle_decode(qkv, kc, vc, [maxlen] * B, B, maxlen), "maxlen 65536")


def test_decode_reference_sized_workspace(cuda):
    # config 1 (one take, 512 of 4096) with exactly the reference's att_part bytes (src/model.rs:237)
    B, maxlen, lens = 1, 4096, [512]
    qkv, kc, vc, ln = decode_case(B, lens, maxlen, seed=40)
    nbytes = ops.reference_part_bytes(B, NQ, HD, maxlen)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    att, _ = run_decode(qkv, kc, vc, ln, B, maxlen, ws=ws)
    gc.assert_close(u16(att), oracle_decode(qkv, kc, vc, lens, B, maxlen), "reference-sized workspace")
    small = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    with pytest.raises(Exception) as e:
        run_decode(qkv, kc, vc, ln, B, maxlen, ws=small)
    assert "workspace" in str(e.value)


@pytest.mark.parametrize("pdl,fused", [(False, False), (True, False), (False, True), (True, True)])
def test_decode_graph_replay_matches_eager(cuda, pdl, fused):
    # Engine::decode captures one step and replays it, positions advancing on the device (src/model.rs:777-796)
    layers, B, maxlen, start = 3, 8, 512, 200
    W = (NQ + 2 * NK) * HD
    cs, sn = ops.rotary_tables(maxlen, HD)
    cs, sn = cs.cuda(), sn.cuda()

    def make_state():
        torch.manual_seed(0)
        st = dict(qkv=[rand_bf16((B, W), 50 + l) for l in range(layers)],
                  kc=[rand_bf16((B, NK, maxlen, HD), 60 + l) for l in range(layers)],
                  vc=[rand_bf16((B, NK, maxlen, HD), 70 + l) for l in range(layers)],
                  att=[torch.zeros((B, NQ * HD), dtype=torch.bfloat16, device="cuda") for _ in range(layers)],
                  ctr=torch.tensor([start, 0, 0, 0], dtype=torch.int32, device="cuda"),
                  ws=ops.decode_workspace(B, NQ, NK, HD, maxlen))
        return st

    def step(st):
        for l in range(layers):
            ops.step_tf_attention(st["qkv"][l], st["kc"][l], st["vc"][l], st["att"][l], st["ws"], cs, sn,
                                  st["ctr"], None, B, NQ, NK, HD, maxlen, fused=fused)
        st["ctr"][0:1].add_(1)

    eager = make_state()
    graphed = make_state()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    prev = ops.set_pdl(pdl)  # programmatic edges inside the captured step only
    try:
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                step(graphed)
    finally:
        ops.set_pdl(prev)
    torch.cuda.current_stream().wait_stream(s)
    # capture records without running: the graphed state is still the initial one
    for _ in range(5):
        step(eager)
        g.replay()
    torch.cuda.synchronize()
    assert int(graphed["ctr"][0]) == start + 5 == int(eager["ctr"][0])
    for l in range(layers):
        assert torch.equal(eager["att"][l].view(torch.int16), graphed["att"][l].view(torch.int16))
        assert torch.equal(eager["kc"][l].view(torch.int16), graphed["kc"][l].view(torch.int16))
    # and the last step against the oracle (the caches hold the rotated keys of every written position)
    l = layers - 1
    L = start + 5
    q = graphed["qkv"][l].clone()
    if fused:  # the fused launch leaves q unrotated in qkv: rotate it the reference's way for the oracle
        ops.rope(q, cs, sn, graphed["ctr"][0:1] - 1, B, 0, NQ, NK, HD)
        torch.cuda.synchronize()
    ref = oracle_decode(q, graphed["kc"][l], graphed["vc"][l], [L] * B, B, maxlen)
    gc.assert_close(u16(graphed["att"][l]), ref, "graph replay")
    del g


@pytest.mark.parametrize("rope_on", [True, False])
def test_fused_step_equals_prologue_then_attention(cuda, rope_on):
    # config 2 shape: outputs, caches and the k part of qkv bit-identical; q left unrotated by the fused launch
    B, maxlen = 64, 4096
    lens = synth.uniform_int(synth.config_seed(1), B, 330, 4096)
    cs, sn = ops.rotary_tables(maxlen, HD)
    cs, sn = (cs.cuda(), sn.cuda()) if rope_on else (None, None)
    qkv, kc, vc, ln = decode_case(B, lens, maxlen, seed=300)
    a = dict(q=qkv.clone(), k=kc.clone(), v=vc.clone(), o=torch.zeros((B, NQ * HD), dtype=torch.bfloat16,
                                                                        device="cuda"))
    b = {k: v.clone() for k, v in a.items()}
    ws = ops.decode_workspace(B, NQ, NK, HD, maxlen)
    ops.step_tf_attention(a["q"], a["k"], a["v"], a["o"], ws, cs, sn, None, ln, B, NQ, NK, HD, maxlen,
                          rope_on=rope_on, fused=False)
    ops.step_tf_attention(b["q"], b["k"], b["v"], b["o"], ws, cs, sn, None, ln, B, NQ, NK, HD, maxlen,
                          rope_on=rope_on, fused=True)
    torch.cuda.synchronize()
    for key in ("o", "k", "v"):
        assert torch.equal(a[key].view(torch.int16), b[key].view(torch.int16)), key
    W = NQ * HD
    assert torch.equal(a["q"][:, W:].view(torch.int16), b["q"][:, W:].view(torch.int16))
    assert torch.equal(b["q"][:, :W].view(torch.int16), qkv[:, :W].view(torch.int16))


def test_decode_prologue_equals_rope_then_kv_write(cuda):
    B, maxlen = 6, 256
    W = (NQ + 2 * NK) * HD
    cs, sn = ops.rotary_tables(maxlen, HD)
    cs, sn = cs.cuda(), sn.cuda()
    lens = torch.tensor([1, 5, 64, 100, 255, 256], dtype=torch.int32, device="cuda")
    q0 = rand_bf16((B, W), 80)
    a = dict(q=q0.clone(), k=torch.zeros((B, NK, maxlen, HD), dtype=torch.bfloat16, device="cuda"))
    a["v"] = torch.zeros_like(a["k"])
    b = {k: v.clone() for k, v in a.items()}
    ops.decode_prologue(a["q"], a["k"], a["v"], cs, sn, None, lens, B, NQ, NK, HD, maxlen)
    for s in range(B):  # the reference's pair, one take at a time at its own position
        p = torch.tensor([int(lens[s]) - 1], dtype=torch.int32, device="cuda")
        ops.rope(b["q"][s:s + 1], cs, sn, p, 1, 0, NQ, NK, HD)
        ops.kv_write(b["q"][s:s + 1], b["k"][s:s + 1], b["v"][s:s + 1], p, 1, 1, NQ, NK, HD, maxlen)
    torch.cuda.synchronize()
    for key in a:
        assert torch.equal(a[key].view(torch.int16), b[key].view(torch.int16)), key
    # without tables (residual LM, no rope): q untouched, k/v copied
    c = dict(q=q0.clone(), k=torch.zeros_like(a["k"]), v=torch.zeros_like(a["v"]))
    ops.decode_prologue(c["q"], c["k"], c["v"], None, None, None, lens, B, NQ, NK, HD, maxlen)
    torch.cuda.synchronize()
    assert torch.equal(c["q"].view(torch.int16), q0.view(torch.int16))
    row = q0.view(B, NQ + 2 * NK, HD)
    for s in range(B):
        assert torch.equal(c["k"][s, :, int(lens[s]) - 1], row[s, NQ:NQ + NK])


@pytest.mark.parametrize("T,causal,hd,nq,nk", [(1024, 1, 128, 16, 2), (1000, 1, 128, 16, 2), (129, 1, 128, 16, 2),
                                               (17, 1, 128, 16, 2), (300, 0, 64, 8, 2), (256, 0, 128, 4, 4)])
def test_prefill_vs_oracle(cuda, T, causal, hd, nq, nk):
    W = (nq + 2 * nk) * hd
    qkv = rand_bf16((T, W), 90 + T)
    out = torch.zeros((T, nq * hd), dtype=torch.bfloat16, device="cuda")
    ops.attn_full(qkv, out, T, T, causal, nq, nk, hd, hd ** -0.5)
    torch.cuda.synchronize()
    ref = cpu.attn_full(u16(qkv), T, T, causal, nq, nk, hd, hd ** -0.5)
    gc.assert_close(u16(out), ref, f"prefill T={T}")


@pytest.mark.parametrize("causal", [1, 0])
def test_prefill_several_sequences_vs_oracle(cuda, causal):
    # three prompts of 200 tokens in one call: each sequence's ragged last tile reaches into the next one's rows,
    # which the sequence bound masks
    nseq, seq, nq, nk, hd = 3, 200, 16, 2, 128
    rows, W = nseq * seq, (nq + 2 * nk) * hd
    qkv = rand_bf16((rows, W), 95 + causal)
    out = torch.zeros((rows, nq * hd), dtype=torch.bfloat16, device="cuda")
    ops.attn_full(qkv, out, rows, seq, causal, nq, nk, hd, hd ** -0.5)
    torch.cuda.synchronize()
    ref = cpu.attn_full(u16(qkv), rows, seq, causal, nq, nk, hd, hd ** -0.5)
    gc.assert_close(u16(out), ref, f"{nseq} x {seq} causal={causal}")


@pytest.mark.parametrize("nseq,seq,nq,nk,hd", [(512, 12, 16, 16, 64), (512, 11, 16, 2, 128), (256, 5, 16, 2, 128)])
def test_locdit_full_size_vs_oracle(cuda, nseq, seq, nq, nk, hd):
    # config 4 (256 takes x 2 CFG = 512 sequences of 12 tokens, 16 heads, hd 64) and the reference's DiT / LocEnc
    rows, W = nseq * seq, (nq + 2 * nk) * hd
    qkv = rand_bf16((rows, W), 100 + seq)
    out = torch.zeros((rows, nq * hd), dtype=torch.bfloat16, device="cuda")
    ops.attn_full(qkv, out, rows, seq, 0, nq, nk, hd, hd ** -0.5)
    torch.cuda.synchronize()
    gc.assert_close(u16(out), cpu.attn_full(u16(qkv), rows, seq, 0, nq, nk, hd, hd ** -0.5), f"seq {seq}")


def test_kv_replicate_config3(cuda):
    # config 3: the prompt KV (T = 1024) copied into 64 take slots of 4096 positions
    B, maxlen, T = 64, 4096, 1024
    c = torch.zeros((B, NK, maxlen, HD), dtype=torch.bfloat16, device="cuda")
    c[0, :, :T] = rand_bf16((NK, T, HD), 110)
    c[1:, :, T:T + 8] = 1.0  # positions >= T must stay untouched
    ops.kv_replicate(c, B, NK, maxlen, HD, T)
    torch.cuda.synchronize()
    assert torch.equal(c[1:, :, :T].view(torch.int16), c[:1, :, :T].expand(B - 1, -1, -1, -1).view(torch.int16))
    assert bool((c[1:, :, T:T + 8] == 1.0).all())


def test_device_error_word(cuda):
    assert ops.device_error() == 0
    # a length outside [1, maxlen] is clamped by the kernel and recorded (no out-of-range access)
    B, maxlen = 2, 128
    qkv, kc, vc, _ = decode_case(B, [1, 1], maxlen, seed=120)
    ln = torch.tensor([0, maxlen + 5], dtype=torch.int32, device="cuda")
    att, ws = run_decode(qkv, kc, vc, ln, B, maxlen)
    assert bool(torch.isfinite(att.float()).all())
    assert ops.device_error(reset=True) & 2
    assert ops.device_error() == 0


@pytest.mark.parametrize("L", [4096, 16384])
def test_decode_one_long_take(cuda, L):
    # one take decoded alone over a long context: the grid shrinks so that each segment is split over at most ~8
    # CTAs (16 CTAs of 16 tiles at 4096 positions, 64 CTAs of 64 tiles at 16384)
    B, maxlen = 1, L
    qkv, kc, vc, ln = decode_case(B, [L], maxlen, seed=41)
    att, _ = run_decode(qkv, kc, vc, ln, B, maxlen)
    gc.assert_close(u16(att), oracle_decode(qkv, kc, vc, [L], B, maxlen), f"one take, L={L}")


@pytest.mark.parametrize("nseq,seq,causal,hd,nq,nk", [(2, 4100, 1, 64, 2, 1), (1, 4352, 0, 128, 2, 2),
                                                       (1, 4096, 1, 128, 4, 2)])
def test_long_prefill_pairs_vs_oracle(cuda, nseq, seq, causal, hd, nq, nk):
    # sequences of 4096 positions and more take the two-tiles-per-CTA kernel (pp::k_attn_prefill_pp): ragged last
    # tiles reaching into the next sequence's rows, an odd number of query tiles (a CTA with one tile), non-causal
    # rows over every key tile, hd 64 and 128, one and two q heads per kv head
    rows, W = nseq * seq, (nq + 2 * nk) * hd
    qkv = rand_bf16((rows, W), 130 + seq + causal)
    out = torch.zeros((rows, nq * hd), dtype=torch.bfloat16, device="cuda")
    ops.attn_full(qkv, out, rows, seq, causal, nq, nk, hd, hd ** -0.5)
    torch.cuda.synchronize()
    ref = cpu.attn_full(u16(qkv), rows, seq, causal, nq, nk, hd, hd ** -0.5)
    gc.assert_close(u16(out), ref, f"{nseq} x {seq} causal={causal} hd={hd}")
    assert ops.device_error() == 0
