"""Parity of the sm_100a library (through its C ABI) with the CPU oracle, with the golden outputs of the reference's
own kernels, and with those kernels run live when their fatbin travelled with the tree."""
import json
import os

import numpy as np
import pytest

import golden_cases as gc

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
EXACT = ("rope", "kv_write", "kv_rep")
NAMES = list(gc.CASES)


def _check(kind, got, ref, what):
    for key in ref:
        if kind in EXACT:
            gc.assert_exact(got[key], ref[key], f"{what}.{key}")
        else:
            gc.assert_close(got[key], ref[key], f"{what}.{key}")


@pytest.mark.gpu
@pytest.mark.parametrize("name", NAMES)
def test_ours_matches_oracle(cuda, name):
    c = gc.CASES[name]
    x = gc.inputs(c)
    _check(c["kind"], gc.run_gpu(c, "ours", x), gc.run_oracle(c, x), name)


@pytest.mark.gpu
@pytest.mark.parametrize("name", NAMES)
def test_ours_matches_reference_golden(cuda, name):
    path = os.path.join(GOLDEN, name + ".npz")
    if not os.path.exists(path):
        pytest.fail(f"golden file {path} missing")
    z = np.load(path)
    c = json.loads(str(z["case"]))
    got = gc.run_gpu(c, "ours")
    _check(c["kind"], got, {k: z[k] for k in got}, name)


@pytest.mark.gpu
@pytest.mark.parametrize("name", NAMES)
def test_ours_matches_reference_kernels_live(cuda, name):
    from oracle import refkern
    if not refkern.available():
        pytest.skip("oracle/_ref/voxcpm_ref.fatbin not built (needs the reference tree)")
    c = gc.CASES[name]
    x = gc.inputs(c)
    _check(c["kind"], gc.run_gpu(c, "ours", x), gc.run_gpu(c, "ref", x), name)


DECODE = [n for n in NAMES if gc.CASES[n]["kind"] == "decode"]


@pytest.mark.gpu
@pytest.mark.parametrize("name", DECODE)
def test_fused_decode_step_matches_golden_and_unfused(cuda, name):
    # the newest position goes through the fused launch (rope + kv_write + attention): the same output as the
    # separate launches, bit for bit, and the reference's output within tolerance
    c = gc.CASES[name]
    x = gc.inputs(c)
    fused = gc.run_gpu(c, "ours_fused", x)
    gc.assert_exact(fused["out"], gc.run_gpu(c, "ours", x)["out"], name)
    path = os.path.join(GOLDEN, name + ".npz")
    gc.assert_close(fused["out"], np.load(path)["out"], name)
