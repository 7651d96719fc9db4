"""Writes the golden outputs of every case in tests/golden_cases.py by running the REFERENCE's own kernels
(kernels/voxcpm.cu, built by `make -C oracle` into oracle/_ref/voxcpm_ref.fatbin as compute_80 PTX and JIT-compiled
by the driver) on a GPU, with the reference's launch shapes (src/model.rs).

    python tests/golden/gen_golden.py [outdir]        (default: tests/golden)

Each case becomes <outdir>/<case>.npz holding the output arrays (uint16 bf16 bit patterns) and the case's
parameters; inputs are not stored, they are rebuilt from the seed.
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, os.path.dirname(HERE))

import golden_cases as gc  # noqa: E402


def main():
    out = sys.argv[1] if len(sys.argv) > 1 else HERE
    os.makedirs(out, exist_ok=True)
    for name, c in gc.CASES.items():
        res = gc.run_gpu(c, "ref")
        np.savez_compressed(os.path.join(out, name + ".npz"), case=json.dumps(c), **res)
        print(name, {k: v.shape for k, v in res.items()}, flush=True)


if __name__ == "__main__":
    main()
