"""Seeded synthetic inputs shared by the tests, the smoke check and bench.py.

Generator: splitmix64 -> uniform in (0, 1) -> Box-Muller N(0, 1) in f64 ->
f32 -> f16 (round to nearest even).  Seeds: 1 q, 2 k, 3 v, 4 norm weights,
5 sequence lengths, 6 weights / token ids.  The reference has no input
generator for these shapes (its attention microbench uses the deterministic
pattern of attention_microbench.rs:203-214, which the oracle also provides).
"""
import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(seed: int, n: int, offset: int = 0) -> np.ndarray:
    """Outputs offset .. offset+n-1 of the splitmix64 stream seeded by `seed`."""
    idx = np.arange(offset + 1, offset + n + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + idx * _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        z = z ^ (z >> np.uint64(31))
    return z


def uniform(seed: int, n: int, offset: int = 0) -> np.ndarray:
    z = splitmix64(seed, n, offset)
    return ((z >> np.uint64(11)).astype(np.float64) + 0.5) * (1.0 / 9007199254740992.0)


def normal(seed: int, n: int, dtype=np.float16, chunk: int = 1 << 22) -> np.ndarray:
    """n samples of N(0,1) from `seed`, as `dtype` (default float16)."""
    out = np.empty(n, dtype=dtype)
    npairs = (n + 1) // 2
    done = 0
    while done < npairs:
        c = min(chunk, npairs - done)
        u = uniform(seed, 2 * c, 2 * done)
        u1, u2 = u[0::2], u[1::2]
        r = np.sqrt(-2.0 * np.log(u1))
        t = 2.0 * np.pi * u2
        pair = np.empty(2 * c, dtype=np.float64)
        pair[0::2] = r * np.cos(t)
        pair[1::2] = r * np.sin(t)
        lo = 2 * done
        hi = min(n, lo + 2 * c)
        out[lo:hi] = pair[: hi - lo].astype(np.float32).astype(dtype)
        done += c
    return out


def norm_weight(seed: int, d: int) -> np.ndarray:
    """f16(1 + N(0, 0.02)) per-head RMSNorm weight (Qwen3 q_norm / k_norm)."""
    n = normal(seed, d, dtype=np.float64)
    return (1.0 + 0.02 * n).astype(np.float32).astype(np.float16)


def ragged_lengths(seed: int, count: int, lo: int = 128, hi: int = 8192) -> np.ndarray:
    """count lengths uniform in [lo, hi] (config 4's ragged prefill batch)."""
    z = splitmix64(seed, count)
    return (lo + (z % np.uint64(hi - lo + 1)).astype(np.int64)).astype(np.int32)
