"""Pins the CPU oracle to the reference itself: every golden file under tests/golden/ holds the outputs of the
reference's own kernels (kernels/voxcpm.cu on a B200, written by tests/golden/gen_golden.py). The oracle must
reproduce them within the north_star tolerance, and bit-exactly for the copies and the rotary embedding."""
import glob
import json
import os

import numpy as np
import pytest

import golden_cases as gc

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
FILES = sorted(glob.glob(os.path.join(GOLDEN, "*.npz")))


def test_every_case_has_a_golden_file():
    have = {os.path.basename(f)[:-4] for f in FILES}
    missing = sorted(set(gc.CASES) - have)
    assert not missing, f"no golden output for {missing}: run tests/golden/gen_golden.py on a GPU"


@pytest.mark.parametrize("path", FILES, ids=[os.path.basename(f)[:-4] for f in FILES])
def test_oracle_matches_reference_kernels(path):
    z = np.load(path)
    name = os.path.basename(path)[:-4]
    case = json.loads(str(z["case"]))
    assert case == gc.CASES[name], "case definition changed since the golden file was written"
    got = gc.run_oracle(case)
    for key, val in got.items():
        ref = z[key]
        assert ref.shape == val.shape
        if case["kind"] in ("kv_write", "kv_rep", "rope"):
            gc.assert_exact(val, ref, f"{name}.{key}")
        else:
            gc.assert_close(val, ref, f"{name}.{key}")
