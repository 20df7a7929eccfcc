"""Shared loaders for the reference fixtures (see tests/golden/make_golden.py)."""
import functools
import pathlib

import numpy as np

from signals import chirp, normal, sinusoids  # noqa: F401

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "reference_fixtures.npz"
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


def x_noise():
    return normal(0, (2, N))


def gc_seed(ncoef):
    g = normal(11, (2, 2, ncoef))
    return (g[0] + 1j * g[1]).astype(np.complex64)


def gy_seed():
    return normal(12, (2, N))
