"""oumu_b200 — sm_100a (B200) attention hot path of hayatree/oumu behind the reference's kernel ABI.

The product is liboumu_attn.so (C ABI: include/oumu_attn.h). `ops` mirrors the reference's launch interface over
that ABI for torch CUDA tensors; `synth` builds the seeded synthetic inputs of the benchmark configurations.
"""
from . import _lib  # noqa: F401

__all__ = ["ops", "synth", "build"]
