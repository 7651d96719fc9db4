"""The tensor-core projection GEMM of the decoding step (oumu_gemm, include/oumu_step.h) against an exact (float64)
PyTorch reference of the reference engine's Lin::fwd (x . W^T + bias, one bf16 rounding; src/model.rs:27-45,
src/gpu.rs:186-229): the step's shapes at 32 and 64 takes, the DiT's 704-row shapes, ragged M and N, row-strided
operands, determinism, and a CUDA graph of programmatically dependent launches."""
import pytest
import torch

from oumu_b200 import ops

pytestmark = pytest.mark.gpu


def rnd(shape, seed, scale=1.0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return (torch.randn(shape, generator=g, device="cuda") * scale).to(torch.bfloat16)


def reference(x, w, bias=None):
    """(bf16(x . W^T + bias), sum |x| . |W|^T): the exact product in float64, and the magnitude that bounds the
    rounding error of any fp32 summation order."""
    y = x.double() @ w.double().t()
    if bias is not None:
        y = y + bias.double()
    return y.to(torch.bfloat16), x.float().abs() @ w.float().abs().t()


def assert_gemm_close(got, want, what):
    """fp32 accumulation in another order than the exact sum: within one bf16 ulp of the exact result, or within
    2^-18 of the sum of |terms| where the result cancels to almost nothing; identical to it almost everywhere."""
    ref, mag = want
    g, w = got.float(), ref.float()
    diff = (g - w).abs()
    tol = w.abs() * 2.0 ** -7 + mag * 2.0 ** -18
    bad = diff > tol
    assert not bool(bad.any()), (f"{what}: {int(bad.sum())} outputs off, max diff {diff.max().item()}, "
                                 f"first at {torch.nonzero(bad)[0].tolist()}")
    frac = (diff > 0).float().mean().item()
    assert frac < 0.02, f"{what}: {frac:.4f} of the outputs differ from the exact result"


SHAPES = [
    # the LM projections at 32 takes per GPU (qkv, o, gate|up, down) and the step's heads
    (32, 2560, 2048), (32, 2048, 2048), (32, 12288, 2048), (32, 2048, 6144), (32, 512, 2048), (32, 2048, 512),
    (32, 2048, 4096), (32, 1024, 2048),
    # 64 takes, ragged M and N, tiny shapes
    (64, 2560, 2048), (48, 700, 4096), (4, 300, 128), (1, 64, 64), (32, 2, 2048),
    # DiT-sized token counts (several token tiles)
    (704, 2560, 1024), (704, 1024, 4096), (160, 1024, 1024),
]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_matches_fp32_reference(cuda, M, N, K):
    x, w = rnd((M, K), 1), rnd((N, K), 2, 0.02)
    bias = rnd((N,), 3, 0.1)
    for b in (None, bias):
        y = torch.full((M, N), 9.0, dtype=torch.bfloat16, device="cuda")
        ops.gemm(x, w, y, bias=b)
        torch.cuda.synchronize()
        assert_gemm_close(y, reference(x, w, b), f"M={M} N={N} K={K} bias={b is not None}")


def test_gemm_strided_operands_and_determinism(cuda):
    # x rows 5 * 1024 apart (the local encoder's first tokens), y a column slice of a wider buffer
    M, N, K = 32, 1024, 1024
    big = rnd((M * 5, K), 4)
    x = big.view(M, 5 * K)[:, :K]
    w, bias = rnd((N, K), 5, 0.02), rnd((N,), 6, 0.1)
    out = torch.zeros((M, 2 * N), dtype=torch.bfloat16, device="cuda")
    ops.gemm(x, w, out[:, N:], bias=bias)
    ops.gemm(x, w, out[:, :N])
    torch.cuda.synchronize()
    assert_gemm_close(out[:, N:], reference(x, w, bias), "strided, bias")
    assert_gemm_close(out[:, :N], reference(x, w), "strided")
    # deterministic: the same inputs give the same bits
    again = torch.zeros_like(out)
    ops.gemm(x, w, again[:, N:], bias=bias)
    torch.cuda.synchronize()
    assert torch.equal(again[:, N:], out[:, N:])


def test_gemm_chain_in_graph_with_pdl(cuda):
    # y1 = x W1^T, y2 = y1 W2^T, ...: each launch reads the previous one's output, in a graph with programmatic
    # edges; the results must equal the eager launches bit for bit
    M, D = 32, 2048
    ws_ = [rnd((D, D), 10 + i, 0.03) for i in range(6)]
    x = rnd((M, D), 9)
    ys = [torch.empty((M, D), dtype=torch.bfloat16, device="cuda") for _ in ws_]
    def chain():
        src = x
        for w, y in zip(ws_, ys):
            ops.gemm(src, w, y)
            src = y

    chain()
    torch.cuda.synchronize()
    eager = [y.clone() for y in ys]
    src = x
    for w, y in zip(ws_, eager):
        assert_gemm_close(y, reference(src, w), "chain")
        src = y
    for y in ys:
        y.zero_()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        prev = ops.set_pdl(True)
        try:
            with torch.cuda.graph(g, stream=s):
                chain()
        finally:
            ops.set_pdl(prev)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    for a, b in zip(ys, eager):
        assert torch.equal(a, b)
    assert ops.device_error() == 0


def test_gemm_rejects_bad_shapes(cuda):
    from oumu_b200 import _lib
    x, w = rnd((8, 100), 1), rnd((16, 100), 2)
    y = torch.empty((8, 16), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.OumuError):
        ops.gemm(x, w, y)  # K not a multiple of 64


# (M, F, K): the LM's gate|up at 32 and 64 takes, one-tile and one-K-block shapes, and shapes whose K split is 6 or
# 7 (owner row ranges the SwiGLU form rounds to whole 16-row groups), with 32, 64 and 128-token tiles
SWIGLU_SHAPES = [(32, 6144, 2048), (64, 6144, 2048), (1, 8, 64), (5, 24, 128), (48, 200, 4096), (32, 1280, 2048),
                 (32, 1536, 2048), (100, 1280, 2048), (704, 1024, 1024), (33, 1000, 512)]


@pytest.mark.parametrize("M,F,K", SWIGLU_SHAPES)
def test_gemm_swiglu_bit_identical_to_gemm_then_silu_mul(cuda, M, F, K):
    """oumu_gemm_swiglu (gate|up projection with the SwiGLU activation in its epilogue) against the two launches it
    replaces, oumu_gemm into [gate | up] and oumu_silu_mul (kernels/voxcpm.cu:92-99): bit-identical, with and
    without a bias, into a row-strided output whose padding it leaves alone."""
    x, w = rnd((M, K), 4), rnd((2 * F, K), 5, 0.02)
    bias = rnd((2 * F,), 6, 0.1)
    w_il = ops.swiglu_interleave(w)
    assert torch.equal(ops.swiglu_deinterleave(w_il), w)
    for b in (None, bias):
        gu = torch.empty((M, 2 * F), dtype=torch.bfloat16, device="cuda")
        ops.gemm(x, w, gu, bias=b)
        want = torch.empty((M, F), dtype=torch.bfloat16, device="cuda")
        ops.silu_mul(gu, want)
        buf = torch.full((M, F + 8), 7.0, dtype=torch.bfloat16, device="cuda")
        ops.gemm_swiglu(x, w_il, buf[:, :F], bias_il=None if b is None else ops.swiglu_interleave(b))
        torch.cuda.synchronize()
        assert torch.equal(buf[:, :F], want), (M, F, K, b is not None, float((buf[:, :F].float() - want.float()).abs().max()))
        assert bool((buf[:, F:] == 7.0).all())
    assert ops.device_error() == 0


def test_gemm_swiglu_rejects_bad_shapes(cuda):
    from oumu_b200 import _lib
    x = rnd((8, 128), 1)
    w = rnd((24, 128), 2)  # F = 12: not a multiple of 8
    act = torch.empty((8, 12), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.OumuError):
        _lib.call("oumu_gemm_swiglu", x.data_ptr(), 128, w.data_ptr(), act.data_ptr(), 12, None, 8, 12, 128, None)
    w = rnd((32, 128), 2)
    act = torch.empty((8, 16), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.OumuError):  # output pitch below F
        _lib.call("oumu_gemm_swiglu", x.data_ptr(), 128, w.data_ptr(), act.data_ptr(), 8, None, 8, 16, 128, None)
