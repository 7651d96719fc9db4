import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    # build on first use if the tree arrived without the library (the product has no fallback path)
    from oumu_b200 import build
    build.build()
    return torch.device("cuda")


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """Per-comparison error statistics of the attention outputs (bf16) against their references: max abs and max
    relative error, exact fraction, and the elements beyond 2e-3 split into single-ulp flips and larger errors."""
    gc = sys.modules.get("golden_cases")
    stats = getattr(gc, "STATS", None) if gc else None
    if not stats:
        return
    path = os.environ.get("OUMU_PARITY_STATS")
    if path:
        import json
        with open(path, "w") as f:
            json.dump(stats, f, indent=1, sort_keys=True)
    tr = terminalreporter
    tr.section("parity statistics (bf16 outputs vs reference)")
    tr.write_line(f"{'n':>9} {'max_abs':>8} {'max_rel':>8} {'exact':>6} {'>2e-3':>6} {'1ulp':>6} {'more':>5}  comparison")
    for k, s in stats.items():
        tr.write_line(f"{s['n']:>9} {s['max_abs']:>8.2e} {s['max_rel']:>8.2e} {s['exact']:>6.3f} {s['over_atol']:>6} "
                      f"{s['over_atol_1ulp']:>6} {s['over_atol_more']:>5}  {k}")
    worst = max(stats.values(), key=lambda s: s["max_abs"])
    more = sum(s["over_atol_more"] for s in stats.values())
    flips = sum(s["over_atol_1ulp"] for s in stats.values())
    n = sum(s["n"] for s in stats.values())
    tr.write_line(f"parity summary: {len(stats)} comparisons, {n} elements, worst max_abs {worst['max_abs']:.3e}, "
                  f"{flips} elements beyond 2e-3 that are single-ulp flips, {more} beyond 2e-3 by more than one ulp")
