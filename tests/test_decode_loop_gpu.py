"""The decoding loop with the stop test on the device (oumu_decode_loop_*, ops.DecodeLoop, Engine.decode): one graph
launch runs `while ctr[1] < max_steps and some stop[s] < 0: step`, the loop of Engine::decode
(src/model.rs:777-796) whose host reads the stop flags after every step.

Control flow is checked exactly on a step graph of one oumu_step_end (stop logits chosen per take) against a
restatement of the reference's host loop; the whole random-init step is checked bit for bit against the host loop
of the same captured graph; and a step graph that never advances ctr[1] ends at the loop's step cap with the flag
set (the bound that keeps a faulty step from holding the device)."""
import pytest
import torch

from oumu_b200 import engine, ops

pytestmark = pytest.mark.gpu


def host_loop(stop0, n0, want, min_len, max_steps):
    """Engine::decode's loop (src/model.rs:784-793) with step_end's stop rule (kernels/voxcpm.cu:415-433) applied
    per step: the stop flags, ctr[1] and the number of steps at the end."""
    stop, n, steps = list(stop0), n0, 0
    while n < max_steps and any(s < 0 for s in stop):
        for s, w in enumerate(want):
            if w and n > min_len and stop[s] < 0:
                stop[s] = n
        n += 1
        steps += 1
    return stop, n, steps


def logits_for(want):
    """Stop logits [B][2] whose argmax asks to stop exactly for the takes in `want`."""
    lg = torch.zeros((len(want), 2), dtype=torch.float32)
    lg[:, 1] = torch.tensor([1.0 if w else -1.0 for w in want])
    return lg.to(torch.bfloat16).cuda()


def capture(fn):
    g = torch.cuda.CUDAGraph(keep_graph=True)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    g.instantiate()
    return g


CASES = [
    # (B, want stop, stop at launch, ctr[1] at launch, min_len, max_steps)
    (4, "all", None, 0, 3, 10),       # every take stops after min_len: the loop ends early
    (4, "but_last", None, 0, 3, 10),  # one take never stops: max_steps
    (4, "all", [0, 1, 2, 3], 0, 3, 10),  # all stopped at launch: no step
    (4, "none", None, 10, 3, 10),     # max_steps patches at launch: no step
    (6, "odd", [-1, -1, 5, -1, -1, -1], 2, 1, 12),  # resumed mid-decode, one take already stopped
    (300, "all_but_7", None, 0, 2, 9),  # more takes than the test kernel's threads
]


@pytest.mark.parametrize("B,pattern,stop0,n0,min_len,max_steps", CASES)
def test_loop_matches_the_host_loop(cuda, B, pattern, stop0, n0, min_len, max_steps):
    want = {"all": [True] * B, "none": [False] * B, "but_last": [True] * (B - 1) + [False],
            "odd": [s % 2 == 1 for s in range(B)], "all_but_7": [s != 7 for s in range(B)]}[pattern]
    stop0 = stop0 or [-1] * B
    logits = logits_for(want)
    patch = (torch.arange(B * 256, device="cuda") % 97).to(torch.bfloat16).view(B, 256)
    patches = torch.zeros((B, max_steps, 256), dtype=torch.bfloat16, device="cuda")
    stop = torch.tensor(stop0, dtype=torch.int32, device="cuda")
    ctr = torch.tensor([500, n0, 0, 0], dtype=torch.int32, device="cuda")
    status = torch.full((2,), 77, dtype=torch.int32, device="cuda")
    g = capture(lambda: ops.step_end(logits, patch, patches, stop, ctr, None, B, min_len, max_steps))
    loop = ops.DecodeLoop(g, stop, ctr, status, B, max_steps)
    want_stop, want_n, steps = host_loop(stop0, n0, want, min_len, max_steps)
    for launch in range(2):  # a second launch after resetting the state repeats the first
        stop.copy_(torch.tensor(stop0, dtype=torch.int32))
        ctr.copy_(torch.tensor([500, n0, 0, 0], dtype=torch.int32))
        patches.zero_()
        loop.launch()
        torch.cuda.synchronize()
        assert stop.tolist() == want_stop, launch
        assert ctr.tolist()[:2] == [500 + steps, want_n], launch
        assert status.tolist() == [steps, 0], launch
        rec = [n for n in range(n0, want_n) if n < max_steps]
        for n in range(max_steps):
            exp = patch if n in rec else torch.zeros_like(patch)
            assert torch.equal(patches[:, n], exp), (launch, n)
    loop.close()
    assert ops.device_error() == 0


def test_loop_ends_at_its_step_cap(cuda):
    # a step graph that never advances ctr[1]: the loop still ends, after max_steps steps, with status[1] = 1
    B, max_steps = 3, 6
    stop = torch.full((B,), -1, dtype=torch.int32, device="cuda")
    ctr = torch.zeros(4, dtype=torch.int32, device="cuda")
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    ticks = torch.zeros(1, dtype=torch.int32, device="cuda")
    g = capture(lambda: ticks.add_(1))
    loop = ops.DecodeLoop(g, stop, ctr, status, B, max_steps)
    loop.launch()
    torch.cuda.synchronize()
    assert int(ticks) == max_steps and status.tolist() == [max_steps, 1] and ctr.tolist()[1] == 0
    loop.close()


def _state(e):
    ts = [e.x, e.cond, e.noise, e.lm_h, e.res_h, e.patches, e.lens, e.ctr, e.stop]
    return ts + e.base.kc + e.base.vc + e.res.kc + e.res.vc


def test_engine_decode_device_loop_equals_host_loop(cuda):
    e = engine.Engine(6, maxlen=256, base_layers=2, res_layers=1, enc_layers=1, dit_layers=1, max_steps=12,
                      min_len=1)
    e.prime([10, 40, 70, 100, 130, 160], seed=5)
    g = e.capture(keep_graph=True)  # one eager step, then the capture
    s0 = [t.clone() for t in _state(e)]
    host = e.decode(g, device_loop=False)
    torch.cuda.synchronize()
    after_host = [t.clone() for t in _state(e)]
    for t, v in zip(_state(e), s0):
        t.copy_(v)
    dev = e.decode(g, device_loop=True)
    torch.cuda.synchronize()
    assert dev == host
    for i, (t, v) in enumerate(zip(_state(e), after_host)):
        assert torch.equal(t.view(torch.uint8), v.view(torch.uint8)), f"state tensor {i} differs"
    n = int(e.ctr[1])
    assert int(e.loop_status[0]) == n - 1 and int(e.loop_status[1]) == 0  # the capture's eager step ran first
    assert all(1 <= c <= e.max_steps for c in dev)
    assert n == e.max_steps or all(s >= 0 for s in e.stop.tolist())
    assert ops.device_error() == 0
