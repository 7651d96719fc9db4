"""Seeded synthetic inputs with the shapes of the benchmark configurations.

The generator is counter-based splitmix64 -> Box-Muller -> bf16 round-to-nearest-even, so every element is a pure
function of (seed, index) and the same arrays can be rebuilt anywhere (tests, fixtures, bench) without storing them.
bf16 values are handled as uint16 bit patterns; `bf16_to_f32` / `f32_to_bf16` convert.
"""
import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(seed, n, offset=0):
    """n consecutive splitmix64 outputs of stream `seed`, starting after `offset` draws."""
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + (np.arange(offset + 1, offset + n + 1, dtype=np.uint64) * _GOLDEN)
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def normal_f32(seed, n):
    """n standard normal draws (float32): Box-Muller on pairs of splitmix64 outputs."""
    m = (n + 1) // 2
    z = splitmix64(seed, 2 * m)
    u1 = ((z[0::2] >> np.uint64(11)).astype(np.float64) + 1.0) * (1.0 / 9007199254740992.0)
    u2 = (z[1::2] >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
    r = np.sqrt(-2.0 * np.log(u1))
    out = np.empty(2 * m, dtype=np.float64)
    out[0::2] = r * np.cos(2.0 * np.pi * u2)
    out[1::2] = r * np.sin(2.0 * np.pi * u2)
    return out[:n].astype(np.float32)


def f32_to_bf16(x):
    """float32 -> bf16 bit patterns (uint16), round-to-nearest-even, NaN -> 0x7fc0."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)).astype(np.uint16)
    r[np.isnan(x)] = 0x7FC0
    return r


def bf16_to_f32(h):
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def normal_bf16(seed, shape, std=1.0):
    n = int(np.prod(shape))
    x = normal_f32(seed, n)
    if std != 1.0:
        x = x * np.float32(std)
    return f32_to_bf16(x).reshape(shape)


def uniform_int(seed, n, lo, hi):
    """n integers uniform in [lo, hi] (inclusive)."""
    z = splitmix64(seed, n)
    return (lo + (z % np.uint64(hi - lo + 1)).astype(np.int64)).astype(np.int32)


def config_seed(config_id):
    """Seed of benchmark configuration `config_id` (0x5EED + id)."""
    return 0x5EED + int(config_id)
