"""Shared loaders for the reference fixtures (see tests/golden/make_golden.py)."""
import functools
import pathlib

import numpy as np

from signals import chirp, normal, sinusoids  # noqa: F401

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "reference_fixtures.npz"
GOLDEN_ALT = pathlib.Path(__file__).resolve().parent / "golden" / "reference_fixtures_alt.npz"
STRIDE = 13
STRIDE_SLICED = 41
N = 65536


@functools.lru_cache(maxsize=1)
def ref():
    with np.load(GOLDEN) as f:
        return {k: f[k] for k in f.files}


@functools.lru_cache(maxsize=1)
def oracle():
    from oracle.cqt_oracle import OctCQTOracle
    return OctCQTOracle()


# other filterbanks (band lengths 32..2048), as in tests/golden/make_golden.py
ALT_CONFIGS = [([4, 4, 1], [8, 16, 32]), ([2, 2, 2, 3], [8, 12, 16, 32]),
               ([3, 4, 2], [8, 64, 64])]
STRIDE_ALT = 37


@functools.lru_cache(maxsize=1)
def ref_alt():
    with np.load(GOLDEN_ALT) as f:
        return {k: f[k] for k in f.files}


@functools.lru_cache(maxsize=4)
def oracle_alt(i):
    from oracle.cqt_oracle import OctCQTOracle
    no, bpo = ALT_CONFIGS[i]
    return OctCQTOracle(no, bpo)


def x_alt():
    return normal(21, (2, N))


def x_noise():
    return normal(0, (2, N))


def gc_seed(ncoef):
    g = normal(11, (2, 2, ncoef))
    return (g[0] + 1j * g[1]).astype(np.complex64)


def gy_seed():
    return normal(12, (2, N))


# 32768-sample slices of the default bank, as in tests/golden/make_golden.py --short
GOLDEN_32K = pathlib.Path(__file__).resolve().parent / "golden" / "reference_fixtures_32k.npz"
N_SHORT = 32768
STRIDE_SHORT = 29


@functools.lru_cache(maxsize=1)
def ref_short():
    with np.load(GOLDEN_32K) as f:
        return {k: f[k] for k in f.files}


@functools.lru_cache(maxsize=1)
def oracle_short():
    from oracle.cqt_oracle import OctCQTOracle
    return OctCQTOracle((3, 4, 2), (8, 16, 32), 44100, N_SHORT)


def x_short():
    return normal(31, (2, N_SHORT))


def gc_short(ncoef):
    g = normal(32, (2, 2, ncoef))
    return (g[0] + 1j * g[1]).astype(np.complex64)


def gy_short():
    return normal(33, (2, N_SHORT))
