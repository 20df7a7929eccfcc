"""CPU checks of the product table builder and of the kernels' dataflow model.

* the product filterbank / heap layout reproduces the oracle (itself pinned to
  the reference);
* ``kernel_model`` (the exact index arithmetic of the CUDA kernels, in numpy
  float64) reproduces numpy's FFTs and, driven by the product tables, the
  oracle's analysis, synthesis and both adjoints.
"""
import numpy as np
import pytest

import kernel_model as km
from fixtures import gc_seed, gy_seed, oracle, x_noise
from flash_cqt_b200.layout import Filterbank, HeapLayout
from flash_cqt_b200.tables import PLANE_STRIDE, build_tables
from oracle.cqt_oracle import snr_db


@pytest.fixture(scope="module")
def heap():
    return HeapLayout(Filterbank([3, 4, 2], [8, 16, 32], 44100, 65536))


@pytest.fixture(scope="module")
def tabs(heap):
    return build_tables(heap)


def test_filterbank_matches_oracle(heap):
    o = oracle()
    bank = heap.bank
    assert bank.oct_bins == o.bank.oct_bins
    assert bank.size_per_oct == o.bank.size_per_oct
    assert (bank.M0, bank.Mnyq, bank.fbins) == (o.bank.M0, o.bank.Mnyq, o.bank.fbins)
    for a, b in zip(bank.ranges, o.bank.wins):
        np.testing.assert_array_equal(a, b)
    for a, b in zip(bank.gd, o.bank.gd):
        np.testing.assert_allclose(a, b, rtol=1e-12, atol=0)
    for (i1, g1, p1, d1, c1), (i2, g2, p2, d2, c2) in zip(
            heap.groups + heap.side_groups, o.all_groups):
        np.testing.assert_array_equal(i1, i2)
        np.testing.assert_array_equal(p1, p2)
        np.testing.assert_array_equal(c1, c2)
        np.testing.assert_allclose(g1, g2, rtol=1e-12, atol=0)
        np.testing.assert_allclose(d1, d2, rtol=1e-12, atol=0)
    assert heap.ncoef == o.ncoef == 132992
    assert len(heap.bands) == 154


def test_plane_assignment(tabs):
    for s, (dest, gre, gim, mask, npl) in tabs["inv"].items():
        live = dest >= 0
        assert np.unique(dest[live]).size == live.sum(), s
        assert npl <= 4
        # every bin of the half spectrum is covered by some window
        assert np.all(mask[:32769] != 0), s
        assert np.all(mask[32769:] == 0)


def test_stockham_schedules_match_fft():
    rng = np.random.default_rng(3)
    for cfg in (km.BAND_CFG_P16, km.BAND_CFG_P32):
        for M, (P, rad) in cfg.items():
            assert np.prod(rad) == M and max(rad) <= P and all(P % r == 0 for r in rad)
            v = rng.standard_normal((2, M)) + 1j * rng.standard_normal((2, M))
            assert snr_db(np.fft.fft(v), km.stockham(v, rad, -1)) > 250
            assert snr_db(np.fft.ifft(v) * M, km.stockham(v, rad, +1)) > 250


def test_packed_spectrum_model():
    v = np.random.default_rng(5).standard_normal((2, 16384)) + 0j
    for rad in (km.SPEC_RADICES_P16, km.SPEC_RADICES_P32):
        assert np.prod(rad) == 16384
        assert snr_db(np.fft.fft(v), km.stockham(v, rad, -1)) > 250
    x = x_noise().astype(np.float64)
    X = km.spectrum_fwd(x)
    assert snr_db(np.fft.rfft(x), X) > 250
    F = np.fft.rfft(x) + 1j * 0.3   # imag on DC / Nyquist must be ignored
    assert snr_db(np.fft.irfft(F, n=65536), km.spectrum_inv(F)) > 250


def test_analysis_model_vs_oracle(heap, tabs):
    o = oracle()
    x = x_noise().astype(np.float64)
    src, gain = tabs["fwd"]["analysis"]
    h = km.bands_fwd(km.spectrum_fwd(x), {"src": src, "gain": gain}, heap.bands)
    assert snr_db(o.heap(o.fwd(x)), h) > 140


def _synth(tabs, heap, s, K):
    dest, gre, gim, mask, npl = tabs["inv"][s]
    E = km.bands_inv(K, {"dest": dest, "gre": gre, "gim": gim}, heap.bands,
                     npl, PLANE_STRIDE)
    return km.spectrum_inv(km.planes_reduce(E, mask, npl, PLANE_STRIDE))


def test_synthesis_model_vs_oracle(heap, tabs):
    o = oracle()
    x = x_noise().astype(np.float64)
    K = o.heap(o.fwd(x))
    y = _synth(tabs, heap, "synth", K)
    assert snr_db(o.bwd(o.unheap(K)), y) > 140
    assert snr_db(x, y) > 140


def test_adjoint_models_vs_oracle(heap, tabs):
    o = oracle()
    gc = gc_seed(o.ncoef).astype(np.complex128)
    gx = _synth(tabs, heap, "adj_an", gc)
    assert snr_db(o.adj_fwd(o.unheap(gc)), gx) > 140
    gy = gy_seed().astype(np.float64)
    src, gain = tabs["fwd"]["adj_synth"]
    gk = km.bands_fwd(km.spectrum_fwd(gy), {"src": src, "gain": gain},
                      heap.bands)
    assert snr_db(o.heap(o.adj_bwd(gy)), gk) > 140


@pytest.mark.parametrize("bank", [([3, 4, 2], [8, 16, 32]), ([4, 4, 1], [8, 16, 32]),
                                  ([2, 2, 2, 3], [8, 12, 16, 32]), ([3, 4, 2], [8, 64, 64])])
def test_pruned_taps_are_dead(bank):
    """The band kernels skip the first-stage inputs r = 6..9 of a block-length
    class (and, at M = 2048, the last-stage outputs 3 and 4 of the
    synthesis) when the closed-form geometry puts taps [6M/16, 10M/16) outside
    every octave band's window (the upload's check).  The per-tap tables must
    agree: no gather and no scatter tap in that range carries a gain."""
    tabs = build_tables(HeapLayout(Filterbank(bank[0], bank[1], 44100, 65536)))
    geom, blen, boff = tabs["band_geom"], tabs["band_len"], tabs["band_off"]
    sets = [tabs["fwd"]["analysis"][1], tabs["fwd"]["adj_synth"][1],
            tabs["inv"]["synth"][1], tabs["inv"]["adj_an"][1]]
    pruned = 0
    for M in sorted(set(blen.tolist())):
        octave = [b for b in range(len(blen)) if blen[b] == M and not geom[b, 3] & 1]
        if not octave:
            continue
        m = np.arange(6 * M // 16, 10 * M // 16)
        # the upload's criterion, from the closed-form geometry alone
        if not all((((m + geom[b, 1]) & (M - 1)) >= geom[b, 2]).all() for b in octave):
            continue
        pruned += 1
        for b in octave:
            for gains in sets:
                assert not gains[boff[b] + m].any(), (M, b)
        if M == 2048:   # last stage radix 8, span 256: outputs 3, 4 = taps 768..1279
            assert 3 * 256 == 6 * M // 16 and 5 * 256 == 10 * M // 16
    assert pruned > 0


# more banks: 16- to 2048-point bands, 162 to 338 bands, 3 colour planes
MORE_BANKS = [([3, 4, 2], [12, 24, 48]), ([2, 3, 4], [8, 16, 24]), ([5, 4], [8, 32]),
              ([1, 2, 3, 3], [8, 12, 16, 32]), ([4, 5], [12, 24]), ([2, 2, 5], [16, 32, 48]),
              ([2, 3, 4], [12, 24, 32]), ([4, 4, 1], [16, 32, 64]), ([3, 6], [8, 24])]


@pytest.mark.parametrize("bank", MORE_BANKS)
def test_more_banks_model_vs_oracle(bank):
    """the product's tables for other banks, driven through the kernels'
    dataflow model, reproduce the oracle's analysis and synthesis"""
    from oracle.cqt_oracle import OctCQTOracle
    heap = HeapLayout(Filterbank(bank[0], bank[1], 44100, 65536))
    tabs = build_tables(heap)
    lens = sorted(set(int(M) for _, M, _ in heap.gspec))
    assert 16 <= lens[0] and lens[-1] <= 2048
    o = OctCQTOracle(bank[0], bank[1], 44100, 65536)
    x = np.random.default_rng(7).standard_normal((1, 65536))
    src, gain = tabs["fwd"]["analysis"]
    h = km.bands_fwd(km.spectrum_fwd(x), {"src": src, "gain": gain}, heap.bands)
    ref = o.heap(o.fwd(x))
    assert snr_db(ref, h) > 140
    dest, gre, gim, mask, npl = tabs["inv"]["synth"]
    E = km.bands_inv(ref, {"dest": dest, "gre": gre, "gim": gim}, heap.bands, npl,
                     PLANE_STRIDE)
    y = km.spectrum_inv(km.planes_reduce(E, mask, npl, PLANE_STRIDE))
    assert snr_db(o.bwd(o.unheap(ref)), y) > 140


@pytest.mark.parametrize("bank", [([3, 3, 3], [16, 16, 16]), ([9], [24])])
def test_unsupported_band_lengths_are_refused(bank):
    """banks that need 4096- or 8-point bands are refused when the tables are
    built, with the lengths named (the upload refuses them as well)"""
    heap = HeapLayout(Filterbank(bank[0], bank[1], 44100, 65536))
    with pytest.raises(ValueError, match="block lengths"):
        build_tables(heap)
