"""Whole-step parity: the random-init decoding step (oumu_b200.engine, a restatement of Engine::step,
src/model.rs:725-773) against the same step run through the reference's own kernels (tests/perf_step_ref.py:
rmsnorm, rope, kv_write, attn_decode + attn_combine, attn_full, dit_build, gather_rows, cfg_euler, fsq_act, step_end
... from kernels/voxcpm.cu, launched with the grids of src/model.rs), on the same weights, KV state and diffusion
noise; the reference side's GEMMs are cuBLAS, ours cuBLAS or this library's GEMM for the LM projections.

The reference decodes every take at one shared position (src/model.rs:596-615), so the takes share one length. The
noise is the reference's verification mode (a replayed [step][64][4] table, kernels/voxcpm.cu:347-366) on its side
and the same values as this engine's noise input on ours.

Every step starts both engines from the same state (the reference's: KV caches, hidden states, conditioning patch,
patches, stop flags, counters). A random-init network amplifies one-ulp differences layer after layer (28 + 8 LM
layers, and FSQ rounds hidden values to levels 1/9 apart), so the yardstick is the reference's own sensitivity: a
third engine runs the reference kernels from the same state with its hidden states and conditioning patch moved by
one bf16 ulp in half the elements. Checked per step, by relative L2 error as the reference's own checks do
(src/dev.rs:8-20,232-271):
  - the new patch: within 1e-2 (the reference's published tolerance, README), and
  - the DiT output of the step's first pass, the base LM output before FSQ, the FSQ levels, the base and residual LM
    hidden states and the stop logits: no further from the reference than its one-ulp-perturbed self (x 1.5 + 1e-3);
  - the stop flags and the step counter: identical."""
import pytest
import torch

from oumu_b200 import engine

pytestmark = pytest.mark.gpu

B, MAXLEN, L0, STEPS = 4, 512, 300, 6
PATCH_REL_L2 = 1e-2


def _probe(cls):
    """cls with the output of the first DiT pass of each step kept (dit_hout, all 11 tokens of every row)."""
    class Probe(cls):
        dit0 = None

        def full(self, tf, x, rows, seq, out):
            r = super().full(tf, x, rows, seq, out)
            if tf is self.dit and self.dit0 is None:
                self.dit0 = out.clone()
            return r
    return Probe


def _rel_l2(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def _load_state(dst, src):
    for tf_d, tf_s in ((dst.base, src.base), (dst.res, src.res)):
        for a, b in zip(tf_d.kc + tf_d.vc, tf_s.kc + tf_s.vc):
            a.copy_(b)
    for name in ("lm_h", "res_h", "cond", "patches", "stop"):
        getattr(dst, name).copy_(getattr(src, name))


@pytest.mark.parametrize("lm_tc", [(), ("qkv", "o", "gu", "down"), ("qkv", "o", "gu", "down", "swiglu")],
                         ids=["cublas_gemms", "library_gemms", "library_gemms_fused_swiglu"])
def test_decoding_step_matches_the_reference_kernels(cuda, lm_tc):
    from oracle import refkern
    if not refkern.available():
        pytest.skip("oracle/_ref/voxcpm_ref.fatbin not built (needs the reference tree)")
    import perf_step_ref

    kw = dict(maxlen=MAXLEN, max_steps=16, min_len=2, seed=0)
    ours = _probe(engine.Engine)(B, lm_tc=lm_tc, **kw)
    ref = _probe(perf_step_ref.RefStep)(B, **kw)
    pert = _probe(perf_step_ref.RefStep)(B, **kw)
    ref.prime([L0] * B, seed=1)
    ref.ctr[0] = L0 - 1  # the shared position the reference writes next (ours: lens[s] - 1 per take)

    g = torch.Generator(device="cuda")
    g.manual_seed(77)
    # diffusion noise of every step, bf16-representable so that both sides' roundings are exact
    table = torch.randn((STEPS, 64, 4), generator=g, device="cuda").to(torch.bfloat16).float()
    ref.noise_table = pert.noise_table = table

    worst = {}
    stops = []
    for n in range(STEPS):
        # the same state in all three; ours gets per-take lengths equal to the shared position + 1
        _load_state(ours, ref)
        _load_state(pert, ref)
        ours.set_lens([int(ref.ctr[0]) + 1] * B)
        ours.stop.copy_(ref.stop)
        ours.ctr.copy_(ref.ctr)
        pert.ctr.copy_(ref.ctr)
        for name in ("lm_h", "res_h", "cond"):  # one ulp up in a random half of the elements
            t = getattr(pert, name)
            t.view(torch.int16).add_((torch.rand(t.shape, generator=g, device="cuda") < 0.5).to(torch.int16))
        ours.noise.copy_(table[n].t().reshape(1, engine.PATCH).expand(B, -1))  # [t][c] time-major, every take
        for e in (ours, ref, pert):
            e.dit0 = None
            e.step()
        torch.cuda.synchronize()

        err = _rel_l2(ours.x, ref.x)
        worst["patch"] = max(worst.get("patch", 0.0), err)
        assert err <= PATCH_REL_L2, f"step {n}: patch rel-L2 {err:.3e}"
        for what in ("dit0", "lm_raw", "lm_h", "res_h", "stop_l"):
            e_ours, e_floor = _rel_l2(getattr(ours, what), getattr(ref, what)), _rel_l2(getattr(pert, what),
                                                                                        getattr(ref, what))
            worst[what] = max(worst.get(what, 0.0), e_ours / max(e_floor, 1e-12))
            assert e_ours <= 1.5 * e_floor + 1e-3, f"step {n}: {what} rel-L2 {e_ours:.3e}, reference floor {e_floor:.3e}"
        f_ours = float((ours.q != ref.q).float().mean())
        f_floor = float((pert.q != ref.q).float().mean())
        assert f_ours <= 1.5 * f_floor + 1e-2, f"step {n}: FSQ levels differ in {f_ours:.3f}, floor {f_floor:.3f}"
        assert torch.equal(ours.stop, ref.stop), f"step {n}: stop {ours.stop.tolist()} vs {ref.stop.tolist()}"
        assert int(ours.ctr[1]) == int(ref.ctr[1]) == n + 1
        assert ours.lens.tolist() == [int(ref.ctr[0]) + 1] * B and int(ref.ctr[0]) == L0 + n
        stops.append(ref.stop.tolist())
    assert any(s >= 0 for s in stops[-1]), "no take stopped: the stop path was not exercised"
    print("step parity over", STEPS, "steps: worst patch rel-L2", f"{worst.pop('patch'):.2e};",
          "worst ratio to the reference's one-ulp floor:", {k: f"{v:.2f}" for k, v in worst.items()},
          "stop flags", stops[-1])


def test_fused_swiglu_step_is_bit_identical(cuda):
    """The engine's default LM path (the gate|up GEMM writing the SwiGLU activation itself, oumu_gemm_swiglu) against
    the same engine with the GEMM and silu_mul as two launches: same seed, same state, three steps, every output
    and state bit for bit."""
    kw = dict(maxlen=MAXLEN, max_steps=16, min_len=2, seed=0)
    a = engine.Engine(B, lm_tc=("qkv", "o", "gu", "down", "swiglu"), **kw)
    b = engine.Engine(B, lm_tc=("qkv", "o", "gu", "down"), **kw)
    assert a.base.layers[0]["gu"].swiglu and not b.base.layers[0]["gu"].swiglu
    assert torch.equal(a.base.layers[3]["gu"].standard_weight(), b.base.layers[3]["gu"].w)
    for e in (a, b):
        e.prime([L0, L0 + 17, L0 + 40, L0 + 5], seed=1)
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    for n in range(3):
        noise = torch.randn((B, engine.PATCH), generator=g, device="cuda").to(torch.bfloat16)
        for e in (a, b):
            e.noise.copy_(noise)
            e.step()
        torch.cuda.synchronize()
        for what in ("x", "cond", "lm_h", "res_h", "stop_l", "q", "patches", "stop", "lens", "ctr"):
            assert torch.equal(getattr(a, what), getattr(b, what)), f"step {n}: {what} differs"
