"""Parity at the benchmark configurations' full sizes against the reference's own kernels, run live on the B200
(kernels/voxcpm.cu built as compute_80 PTX the way its build.rs does, JIT-compiled by the driver and launched with the
grids of src/model.rs by oracle/refkern.py), on the same seeded inputs and through the same launch sequences:

  config 2   one decode layer, 64 takes, slots of 4096, lengths U[330, 4096]; the reference has one shared position,
             so it runs once per take with that take's own device position (kernels/voxcpm.cu:131-185,
             src/model.rs:596-615); plus the whole decode layer (rope + kv_write + attention) against the fused launch
  config 3   causal prefill T = 1024 with the prompt's k/v copied into 64 take slots (src/model.rs:541-567,705-717)
  config 4   LocDiT: 512 sequences x 12 tokens (16 heads, hd 64), the reference's DiT shape (512 x 11, 16q/2kv,
             hd 128, with rope) and the local encoder (256 x 5) (kernels/voxcpm.cu:262-297)
  long       causal prefill at T = 4096 and at the reference's prompt limit T = 16384 (src/model.rs:411)

Outputs must be within |a - b| <= 2e-3 + 1e-2 |b| element-wise (bf16); caches and rotated k bit-exact. Every
comparison's error statistics (max abs / rel error, exact fraction, elements beyond 2e-3 split into single-ulp flips
and larger) are printed at the end of the pytest run."""
import numpy as np
import pytest
import torch

import golden_cases as gc
from oumu_b200 import ops, synth

pytestmark = pytest.mark.gpu

NQ, NK, HD = 16, 2, 128


@pytest.fixture(scope="module")
def ref():
    from oracle import refkern
    if not refkern.available():
        pytest.skip("oracle/_ref/voxcpm_ref.fatbin not built (needs the reference tree)")
    return refkern


def _rnd(shape, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(shape, generator=g, device="cuda", dtype=torch.float32).to(torch.bfloat16)


def _u16(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def _tables(maxlen, hd):
    from oracle import cpu  # the reference builds its tables on the host (src/model.rs:337-349)
    cs, sn = cpu.rotary_tables(maxlen, hd)
    return torch.from_numpy(cs).cuda(), torch.from_numpy(sn).cuda()


def _zeros_like_out(rows, nq, hd):
    return torch.zeros((rows, nq * hd), dtype=torch.bfloat16, device="cuda")


def _config2(seed):
    B, maxlen = 64, 4096
    lens = synth.uniform_int(synth.config_seed(1), B, 330, 4096)
    qkv = _rnd((B, (NQ + 2 * NK) * HD), seed)
    kc = _rnd((B, NK, maxlen, HD), seed + 1)
    vc = _rnd((B, NK, maxlen, HD), seed + 2)
    return B, maxlen, lens, qkv, kc, vc


def test_config2_decode_attention_vs_reference_kernels(cuda, ref):
    B, maxlen, lens, qkv, kc, vc = _config2(7001)
    part = torch.zeros(B * NQ * (maxlen // 64) * (HD + 2), dtype=torch.float32, device="cuda")
    want = _zeros_like_out(B, NQ, HD)
    ref.attn_decode_per_take(qkv, kc, vc, part, want, lens, B, NQ, NK, HD, maxlen, HD ** -0.5)
    got = _zeros_like_out(B, NQ, HD)
    ws = ops.decode_workspace(B, NQ, NK, HD, maxlen)
    ln = torch.tensor(lens, dtype=torch.int32, device="cuda")
    ops.attn_decode(qkv, kc, vc, got, ws, None, ln, B, NQ, NK, HD, maxlen, HD ** -0.5)
    torch.cuda.synchronize()
    gc.assert_close(_u16(got), _u16(want), "config 2 layer: attention")
    assert ops.device_error() == 0


def test_config2_fused_decode_layer_vs_reference_kernels(cuda, ref):
    # The step's decode layer: per take, rope of q and k at the take's newest position, k/v written into its slot,
    # then attention over the slot (reference: rope + kv_write + attn_decode + attn_combine per take; ours: one
    # launch for all takes).
    B, maxlen, lens, qkv, kc, vc = _config2(7101)
    cs, sn = _tables(maxlen, HD)
    row, slot = (NQ + 2 * NK) * HD, NK * maxlen * HD
    q_r, k_r, v_r = qkv.clone(), kc.clone(), vc.clone()
    pos = torch.tensor([L - 1 for L in lens], dtype=torch.int32, device="cuda")
    for s in range(B):
        qp, pp = q_r.data_ptr() + 2 * s * row, pos.data_ptr() + 4 * s
        ref.rope(qp, cs, sn, pp, 1, 0, NQ, NK, HD)
        ref.kv_write(qp, k_r.data_ptr() + 2 * s * slot, v_r.data_ptr() + 2 * s * slot, pp, 1, 1, NQ, NK, HD, maxlen)
    part = torch.zeros(B * NQ * (maxlen // 64) * (HD + 2), dtype=torch.float32, device="cuda")
    want = _zeros_like_out(B, NQ, HD)
    ref.attn_decode_per_take(q_r, k_r, v_r, part, want, lens, B, NQ, NK, HD, maxlen, HD ** -0.5)

    q_o, k_o, v_o = qkv.clone(), kc.clone(), vc.clone()
    got = _zeros_like_out(B, NQ, HD)
    ws = ops.decode_workspace(B, NQ, NK, HD, maxlen)
    ln = torch.tensor(lens, dtype=torch.int32, device="cuda")
    ocs, osn = ops.rotary_tables(maxlen, HD)
    ops.attn_decode_step(q_o, k_o, v_o, got, ws, ocs.cuda(), osn.cuda(), None, ln, B, NQ, NK, HD, maxlen,
                         HD ** -0.5)
    torch.cuda.synchronize()
    gc.assert_close(_u16(got), _u16(want), "config 2 fused layer: attention")
    gc.assert_exact(_u16(k_o), _u16(k_r), "config 2 fused layer: K cache")
    gc.assert_exact(_u16(v_o), _u16(v_r), "config 2 fused layer: V cache")
    ks = slice(NQ * HD, (NQ + NK) * HD)  # the rotated k is written back into qkv, as rope does
    gc.assert_exact(_u16(q_o[:, ks]), _u16(q_r[:, ks]), "config 2 fused layer: rotated k in qkv")
    assert ops.device_error() == 0


def test_config3_prefill_with_slot_copies_vs_reference_kernels(cuda, ref):
    # rope, kv_write into slot 0, causal attn_full, kv_replicate of K and V into slots 1..63 (the reference) against
    # rope and one launch of attention + k/v into all 64 slots (ours)
    T, slots, maxlen = 1024, 64, 4096
    qkv = _rnd((T, (NQ + 2 * NK) * HD), 7201)
    cs, sn = _tables(maxlen, HD)
    q_r = qkv.clone()
    k_r = torch.zeros((slots, NK, maxlen, HD), dtype=torch.bfloat16, device="cuda")
    v_r = torch.zeros_like(k_r)
    want = _zeros_like_out(T, NQ, HD)
    ref.rope(q_r, cs, sn, None, T, T, NQ, NK, HD)
    ref.kv_write(q_r, k_r, v_r, None, 1, T, NQ, NK, HD, maxlen)
    ref.attn_full(q_r, want, T, T, 1, NQ, NK, HD, HD ** -0.5)
    ref.kv_replicate(k_r, slots, NK, maxlen, HD, T)
    ref.kv_replicate(v_r, slots, NK, maxlen, HD, T)

    ocs, osn = (t.cuda() for t in ops.rotary_tables(maxlen, HD))
    q_o = qkv.clone()
    k_o, v_o = torch.zeros_like(k_r), torch.zeros_like(v_r)
    got = _zeros_like_out(T, NQ, HD)
    ops.rope(q_o, ocs, osn, None, T, T, NQ, NK, HD)
    ops.attn_prefill_kv(q_o, got, k_o, v_o, T, slots, NQ, NK, HD, maxlen, HD ** -0.5)
    torch.cuda.synchronize()
    gc.assert_close(_u16(got), _u16(want), "config 3 prefill T=1024: attention")
    gc.assert_exact(_u16(q_o), _u16(q_r), "config 3 prefill: rotated qkv")
    gc.assert_exact(_u16(k_o), _u16(k_r), "config 3 prefill: K cache, 64 slots")
    gc.assert_exact(_u16(v_o), _u16(v_r), "config 3 prefill: V cache, 64 slots")


@pytest.mark.parametrize("what,nseq,seq,nq,nk,hd,rope", [
    ("config 4 LocDiT 512 x 12, 16 heads, hd 64", 512, 12, 16, 16, 64, False),
    ("reference DiT shape 512 x 11, 16q/2kv, hd 128, rope", 512, 11, 16, 2, 128, True),
    ("local encoder 256 x 5, 16q/2kv, hd 128, rope", 256, 5, 16, 2, 128, True),
], ids=["config4", "dit_ref_shape", "local_encoder"])
def test_small_sequences_vs_reference_kernels(cuda, ref, what, nseq, seq, nq, nk, hd, rope):
    rows = nseq * seq
    qkv = _rnd((rows, (nq + 2 * nk) * hd), 7301 + seq)
    q_r = qkv.clone()
    want = _zeros_like_out(rows, nq, hd)
    if rope:
        cs, sn = _tables(seq, hd)
        ref.rope(q_r, cs, sn, None, rows, seq, nq, nk, hd)
    ref.attn_full(q_r, want, rows, seq, 0, nq, nk, hd, hd ** -0.5)
    got = _zeros_like_out(rows, nq, hd)
    q_o = qkv.clone()
    if rope:
        ocs, osn = (t.cuda() for t in ops.rotary_tables(seq, hd))
        ops.attn_full_rope(q_o, got, ocs, osn, rows, seq, 0, nq, nk, hd, hd ** -0.5)  # one launch, as the step runs
        got2 = _zeros_like_out(rows, nq, hd)
        ops.rope(q_o, ocs, osn, None, rows, seq, nq, nk, hd)
        ops.attn_full(q_o, got2, rows, seq, 0, nq, nk, hd, hd ** -0.5)
        torch.cuda.synchronize()
        gc.assert_exact(_u16(got2), _u16(got), f"{what}: rope fused == rope then attention")
    else:
        ops.attn_full(q_o, got, rows, seq, 0, nq, nk, hd, hd ** -0.5)
        torch.cuda.synchronize()
    gc.assert_close(_u16(got), _u16(want), what)


@pytest.mark.parametrize("T,nq,nk,slots", [(4096, 16, 2, 3), (16384, 2, 1, 2)])
def test_long_prefill_vs_reference_kernels(cuda, ref, T, nq, nk, slots):
    # the tensor-core prefill at long prompts, up to the reference's limit of 16384 positions (src/model.rs:411);
    # fewer heads at 16384 keep the reference kernel's run (one CTA per query row and head) short
    hd = HD
    qkv = _rnd((T, (nq + 2 * nk) * hd), 7401 + T)
    cs, sn = _tables(T, hd)
    q_r = qkv.clone()
    k_r = torch.zeros((slots, nk, T, hd), dtype=torch.bfloat16, device="cuda")
    v_r = torch.zeros_like(k_r)
    want = _zeros_like_out(T, nq, hd)
    ref.rope(q_r, cs, sn, None, T, T, nq, nk, hd)
    ref.kv_write(q_r, k_r, v_r, None, 1, T, nq, nk, hd, T)
    ref.attn_full(q_r, want, T, T, 1, nq, nk, hd, hd ** -0.5)
    ref.kv_replicate(k_r, slots, nk, T, hd, T)
    ref.kv_replicate(v_r, slots, nk, T, hd, T)
    ocs, osn = (t.cuda() for t in ops.rotary_tables(T, hd))
    q_o = qkv.clone()
    k_o, v_o = torch.zeros_like(k_r), torch.zeros_like(v_r)
    got = _zeros_like_out(T, nq, hd)
    ops.rope(q_o, ocs, osn, None, T, T, nq, nk, hd)
    ops.attn_prefill_kv(q_o, got, k_o, v_o, T, slots, nq, nk, hd, T, hd ** -0.5)
    got2 = _zeros_like_out(T, nq, hd)
    ops.attn_full(q_o, got2, T, T, 1, nq, nk, hd, hd ** -0.5)
    torch.cuda.synchronize()
    gc.assert_close(_u16(got), _u16(want), f"prefill T={T} {nq}q/{nk}kv: attention")
    gc.assert_exact(_u16(got2), _u16(got), f"prefill T={T}: with and without the KV epilogue")
    gc.assert_exact(_u16(k_o), _u16(k_r), f"prefill T={T}: K cache")
    gc.assert_exact(_u16(v_o), _u16(v_r), f"prefill T={T}: V cache")
