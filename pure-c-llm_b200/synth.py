"""Seeded synthetic inputs: splitmix64 -> Box-Muller normals.

One generator serves the parity tests, the golden fixtures and bench.py so
that every consumer sees the same tensors for the same (seed, stream) pair.
splitmix64 (Steele, Lea & Flood, "Fast splittable pseudorandom number
generators", OOPSLA 2014) gives 64-bit words; the top 53 bits make a uniform
in [0, 1); Box-Muller turns pairs of uniforms into standard normals.
"""
import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(seed: int, n: int, offset: int = 0) -> np.ndarray:
    """Words offset+1 .. offset+n of the splitmix64 sequence started at `seed`."""
    with np.errstate(over="ignore"):
        idx = np.arange(offset + 1, offset + n + 1, dtype=np.uint64)
        z = np.uint64(seed) + idx * _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def uniform(seed: int, n: int, offset: int = 0) -> np.ndarray:
    """Uniform doubles in [0, 1) from the top 53 bits of each word."""
    return (splitmix64(seed, n, offset) >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)


def normal(seed: int, shape, mean: float = 0.0, std: float = 1.0, chunk: int = 1 << 24) -> np.ndarray:
    """float32 array of N(mean, std^2) samples, Box-Muller over uniform pairs."""
    n = int(np.prod(shape)) if len(tuple(np.atleast_1d(shape))) else 1
    out = np.empty(n, dtype=np.float32)
    done = 0
    while done < n:
        m = min(chunk, n - done)
        pairs = (m + 1) // 2
        u = uniform(seed, 2 * pairs, offset=2 * (done // 2))
        u1 = 1.0 - u[0::2]                      # (0, 1]: log is finite
        u2 = u[1::2]
        r = np.sqrt(-2.0 * np.log(u1))
        z = np.empty(2 * pairs, dtype=np.float64)
        z[0::2] = r * np.cos(2.0 * np.pi * u2)
        z[1::2] = r * np.sin(2.0 * np.pi * u2)
        out[done:done + m] = (mean + std * z[:m]).astype(np.float32)
        done += m
    return out.reshape(shape)


def uniform_int(seed: int, n: int, lo: int, hi: int) -> np.ndarray:
    """n integers uniform in [lo, hi] (inclusive), e.g. ragged cache lengths."""
    u = uniform(seed, n)
    return (lo + np.floor(u * (hi - lo + 1))).astype(np.int32)
