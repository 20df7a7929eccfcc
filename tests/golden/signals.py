"""Portable, seeded test signals for the parity fixtures.

The generator is splitmix64 in numpy uint64 arithmetic followed by Box-Muller,
so the same seed gives bit-identical float32 signals on every machine and numpy
version.  Both the fixture generator and the tests use it, so the fixtures store
only reference outputs, never inputs.
"""
import math

import numpy as np

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _splitmix64(seed, n):
    with np.errstate(over="ignore"):
        s = (np.uint64(seed) * np.uint64(0x9E3779B97F4A7C15)
             + np.arange(1, n + 1, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15))
        z = s
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return z


def uniform(seed, n):
    """n doubles in (0, 1) from the top 53 bits."""
    z = _splitmix64(seed, n) >> np.uint64(11)
    return (z.astype(np.float64) + 0.5) * (1.0 / 9007199254740992.0)


def normal(seed, shape):
    """standard normal float32 array of the given shape (Box-Muller)."""
    n = int(np.prod(shape))
    m = (n + 1) // 2
    u1 = uniform(seed, 2 * m)
    a, b = u1[0::2], u1[1::2]
    r = np.sqrt(-2.0 * np.log(a))
    v = np.concatenate([r * np.cos(2 * math.pi * b), r * np.sin(2 * math.pi * b)])
    return v[:n].reshape(shape).astype(np.float32)


def sinusoids(seed, n=65536, fs=44100.0):
    """8 sinusoids, frequencies log-uniform in 43 Hz..20 kHz, amplitudes
    U(0.1, 1), random phases, plus N(0, 0.01^2) noise -- the B=1 slice of the
    CUDA-graph round-trip workload."""
    u = uniform(seed, 24)
    f = np.exp(math.log(43.0) + u[0:8] * (math.log(20000.0) - math.log(43.0)))
    a = 0.1 + 0.9 * u[8:16]
    ph = 2 * math.pi * u[16:24]
    t = np.arange(n) / fs
    x = (a[:, None] * np.sin(2 * math.pi * f[:, None] * t + ph[:, None])).sum(0)
    x = x + 0.01 * normal(seed + 1000, (n,)).astype(np.float64)
    return x.astype(np.float32)[None]


def chirp(seed, n, fs=44100.0, f0=40.0, f1=18000.0, dur=60.0):
    """logarithmic sweep f0 -> f1 over dur seconds plus N(0, 0.05^2) noise."""
    t = np.arange(n) / fs
    k = math.log(f1 / f0) / dur
    phase = 2 * math.pi * f0 * (np.exp(k * t) - 1.0) / k
    x = np.sin(phase) + 0.05 * normal(seed, (n,)).astype(np.float64)
    return x.astype(np.float32)
