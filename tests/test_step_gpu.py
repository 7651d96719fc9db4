"""The decoding step around the attention: the step-glue kernels (include/oumu_step.h) against plain PyTorch fp32
restatements of the reference kernels they replace, and the whole random-init step (oumu_b200.engine): a captured
CUDA graph replays it bit for bit like the eager calls, at a small size and at the benchmark's 32 takes per GPU."""
import pytest
import torch

from oumu_b200 import engine, ops

pytestmark = pytest.mark.gpu


def rnd(shape, seed, scale=1.0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return (torch.randn(shape, generator=g, device="cuda") * scale).to(torch.bfloat16)


def rb(x):
    return x.to(torch.bfloat16).float()


def assert_ulps(got, want, what, max_frac=0.01):
    """bf16 results whose fp32 intermediates may differ in the last bits (reduction order, exp/tanh): every element
    within one bf16 ulp, and only a small fraction not identical."""
    g, w = got.float(), want.float()
    diff = (g - w).abs()
    assert bool((diff <= w.abs() * 2.0 ** -7 + 1e-30).all()), f"{what}: max diff {diff.max().item()}"
    frac = (diff > 0).float().mean().item()
    assert frac <= max_frac, f"{what}: {frac:.4f} of the elements differ"


@pytest.mark.parametrize("dim,rows", [(1024, 77), (2048, 32), (1024, 1)])
def test_rmsnorm_and_add_rmsnorm(cuda, dim, rows):
    x, d, w = rnd((rows, dim), 1), rnd((rows, dim), 2), rnd((dim,), 3, 0.1) + 1
    out = torch.empty_like(x)
    # rmsnorm (kernels/voxcpm.cu:43-52)
    ops.rmsnorm(x, w, out, 1e-5)
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5)
    assert_ulps(out, rb(rb(xf * r) * w.float()), "rmsnorm")
    # add_rmsnorm (kernels/voxcpm.cu:55-67): the residual update is exact, the norm within an ulp
    res = x.clone()
    ops.rmsnorm(res, w, out, 1e-5, d=d)
    v = rb(xf + d.float())
    assert torch.equal(res.float(), v)
    r = torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + 1e-5)
    assert_ulps(out, rb(rb(v * r) * w.float()), "add_rmsnorm")


def test_silu_mul_silu_fsq(cuda):
    rows, F = 33, 6144
    gu = rnd((rows, 2 * F), 4, 3.0)
    out = torch.empty((rows, F), dtype=torch.bfloat16, device="cuda")
    ops.silu_mul(gu, out)
    g, u = gu[:, :F].float(), gu[:, F:].float()
    assert_ulps(out, rb(rb(g / (1 + torch.exp(-g))) * u), "silu_mul")
    x = rnd((rows, 2048), 5, 3.0)
    y = ops.silu_(x.clone())
    assert_ulps(y, rb(x.float() / (1 + torch.exp(-x.float()))), "silu")
    q = ops.fsq_(x.clone(), 9.0)
    want = rb(torch.round(rb(rb(torch.tanh(x.float())) * 9.0)) / 9.0)
    assert (q.float() != want).float().mean().item() < 1e-3


def test_build_seq_dit_and_encoder_exact(cuda):
    B, H = 5, 1024
    mu, temb, condp, xp = rnd((B, 2 * H), 6), rnd((H,), 7), rnd((B * 4, H), 8), rnd((B * 4, H), 9)
    seq = torch.full((2 * B * 11, H), 7.0, dtype=torch.bfloat16, device="cuda")
    ops.build_seq(seq, temb, xp, 2 * B, 11, H, mu=mu, condp=condp, B=B)
    s = seq.view(2 * B, 11, H)
    # kernels/voxcpm.cu:299-315: [mu0, mu1, t, cond x4, x x4], unconditional rows with mu = 0
    assert torch.equal(s[:B, :2], mu.view(B, 2, H))
    assert torch.equal(s[B:, :2], torch.zeros_like(s[B:, :2]))
    assert torch.equal(s[:, 2], temb.expand(2 * B, H))
    for half in (s[:B], s[B:]):
        assert torch.equal(half[:, 3:7], condp.view(B, 4, H))
        assert torch.equal(half[:, 7:], xp.view(B, 4, H))
    enc = torch.empty((B * 5, H), dtype=torch.bfloat16, device="cuda")
    ops.build_seq(enc, temb, xp, B, 5, H)
    e = enc.view(B, 5, H)
    assert torch.equal(e[:, 0], temb.expand(B, H)) and torch.equal(e[:, 1:], xp.view(B, 4, H))


@pytest.mark.parametrize("seq,first", [(4, 0), (11, 7)])
def test_cfg_euler(cuda, seq, first):
    B, dt, cfg = 6, 0.0986, 2.0
    out = rnd((2 * B * seq, 64), 10)
    x = rnd((B, 256), 11)
    want_x = x.float().clone()
    o = out.view(2 * B, seq, 64)[:, first:first + 4].reshape(2 * B, 256).float()
    pos, neg = o[:B], o[B:]
    # kernels/voxcpm.cu:334-345 (CFG-Zero* + Euler, bf16 roundings)
    dot = rb(rb(pos * neg).sum(-1, keepdim=True))
    nn = rb(rb(rb(neg * neg).sum(-1, keepdim=True)) + 1e-8)
    st = rb(dot / nn)
    a = rb(neg * st)
    d = rb(a + rb(cfg * rb(pos - a)))
    want_x = rb(want_x - rb(dt * d))
    ops.cfg_euler(x, out, B, seq, first, dt, cfg)
    assert_ulps(x, want_x, "cfg_euler", max_frac=0.05)


def test_step_end_exact(cuda):
    B, max_steps = 7, 5
    logits = rnd((B, 2), 12)
    patch = rnd((B, 256), 13)
    patches = torch.zeros((B, max_steps, 256), dtype=torch.bfloat16, device="cuda")
    stop = torch.tensor([-1, -1, 1, -1, -1, -1, -1], dtype=torch.int32, device="cuda")
    ctr = torch.tensor([100, 3, 0, 0], dtype=torch.int32, device="cuda")
    lens = torch.arange(B, dtype=torch.int32, device="cuda") + 50
    ops.step_end(logits, patch, patches, stop, ctr, lens, B, 2, max_steps)
    torch.cuda.synchronize()
    assert torch.equal(patches[:, 3], patch) and int(patches[:, [0, 1, 2, 4]].float().abs().sum()) == 0
    want = logits[:, 1].float() > logits[:, 0].float()
    exp_stop = [(3 if w else -1) if s < 0 else s for w, s in zip(want.tolist(), [-1, -1, 1, -1, -1, -1, -1])]
    assert stop.tolist() == exp_stop
    assert ctr.tolist()[:2] == [101, 4]
    assert lens.tolist() == [51 + i for i in range(B)]
    # past max_steps nothing is recorded, the counters still advance
    ctr.copy_(torch.tensor([0, max_steps, 0, 0], dtype=torch.int32))
    before = patches.clone()
    ops.step_end(logits, patch, patches, stop, ctr, None, B, 2, max_steps)
    torch.cuda.synchronize()
    assert torch.equal(patches, before) and ctr.tolist()[:2] == [1, max_steps + 1]


def _state(e):
    ts = [e.x, e.cond, e.noise, e.lm_h, e.res_h, e.patches, e.lens, e.ctr, e.stop]
    return ts + e.base.kc + e.base.vc + e.res.kc + e.res.vc


def test_engine_graph_replays_the_eager_step(cuda):
    e = engine.Engine(4, maxlen=256, base_layers=2, res_layers=1, enc_layers=1, dit_layers=1, max_steps=8)
    e.prime([10, 50, 100, 200], seed=3)
    s0 = [t.clone() for t in _state(e)]
    e.step()
    e.step()
    torch.cuda.synchronize()
    eager = [t.clone() for t in _state(e)]
    for t, v in zip(_state(e), s0):
        t.copy_(v)
    g = e.capture()  # one eager step, then the capture
    for t, v in zip(_state(e), s0):
        t.copy_(v)
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    for i, (t, v) in enumerate(zip(_state(e), eager)):
        assert torch.equal(t.view(torch.uint8), v.view(torch.uint8)), f"state tensor {i} differs"
    assert e.lens.tolist() == [12, 52, 102, 202] and e.ctr.tolist()[:2] == [2, 2]
    assert bool(torch.isfinite(e.patches[:, :2].float()).all())
    assert ops.device_error() == 0


def test_engine_full_size_step(cuda):
    # the benchmark's per-GPU step: 32 takes, 28 + 8 LM layers, KV slots of 4096
    e = engine.Engine(32)
    e.prime([330 + 100 * i for i in range(32)])
    g = e.capture()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert e.ctr.tolist()[:2] == [4, 4]
    assert e.lens.tolist() == [334 + 100 * i for i in range(32)]
    for t in (e.patches[:, :4], e.lm_h, e.res_h):
        assert bool(torch.isfinite(t.float()).all())
    assert ops.device_error() == 0
