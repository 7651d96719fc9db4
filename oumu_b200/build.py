"""Build the sm_100a attention library in-tree: oumu_b200/liboumu_attn.so.

Usage: python -m oumu_b200.build [--force] [--verbose]
Plain nvcc, no torch extension machinery: the library exposes only the C ABI of include/oumu_attn.h and include/oumu_step.h.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "liboumu_attn.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _sources():
    srcs = [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith((".cu", ".cuh", ".h", ".cpp"))]
    inc = os.path.join(ROOT, "include")
    return srcs + [os.path.join(inc, f) for f in sorted(os.listdir(inc)) if f.endswith(".h")]


def stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(s) > t for s in _sources())


def build(force=False, verbose=False, ptxas_info=False):
    if not force and not stale():
        return LIB
    cmd = [NVCC, *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr",
           "-Xcompiler", "-fPIC,-O2", "-shared", "-I", os.path.join(ROOT, "include"),
           "-o", LIB + ".tmp", os.path.join(CSRC, "oumu_attn.cu")]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    if verbose or ptxas_info:
        sys.stdout.write(r.stdout + r.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="--verbose" in sys.argv, ptxas_info="--ptxas" in sys.argv)
    print(LIB)
