"""The CPU oracle against fixtures produced by the reference itself.

These pin ``oracle/`` before it is trusted as the checker of the CUDA path.
Tolerances: the reference computes in float32 (torch CPU), the oracle in
float64, so agreement is bounded by float32 rounding (~130 dB).
"""
import numpy as np
import pytest

from fixtures import (ALT_CONFIGS, STRIDE, STRIDE_ALT, STRIDE_SLICED, chirp,
                      gc_seed, gy_seed, oracle, oracle_alt, ref, ref_alt, sinusoids,
                      x_alt, x_noise)
from oracle.cqt_oracle import SlicedOracle, snr_db


def test_layout_checksums_exact():
    o, r = oracle(), ref()
    lay = []
    for idx, gv, pos, gdv, conj in o.all_groups:
        b, M = idx.shape
        w = np.arange(1, b * M + 1, dtype=np.int64)
        lay.append([b, M, idx.sum(), (idx.reshape(-1) * w).sum(), pos.sum(),
                    (pos.reshape(-1) * w).sum(), conj.sum(), (gv != 0).sum(),
                    (gdv != 0).sum()])
    np.testing.assert_array_equal(np.array(lay, dtype=np.int64), r["layout"])


def test_windows_and_duals_match():
    o, r = oracle(), ref()
    gv_sum = np.array([g[1].sum() for g in o.all_groups])
    gdv_sum = np.array([g[3].sum() for g in o.all_groups])
    np.testing.assert_allclose(gv_sum, r["gv_sum"], rtol=1e-6)
    np.testing.assert_allclose(gdv_sum, r["gdv_sum"], rtol=1e-6)
    rows = np.concatenate([g[1][0] for g in o.all_groups])
    drows = np.concatenate([g[3][-1] for g in o.all_groups])
    assert snr_db(r["gv_rows"], rows) > 135
    assert snr_db(r["gdv_rows"], drows) > 125
    np.testing.assert_allclose(o.bank.frqs_hz, r["frqs_hz"], rtol=1e-12)


def test_analysis_coefficients():
    o, r = oracle(), ref()
    h = o.heap(o.fwd(x_noise()))
    assert snr_db(r["coef_noise_s"], h.reshape(-1)[::STRIDE]) > 125
    e = np.array([np.sum(np.abs(h[:, off + i * M:off + (i + 1) * M]) ** 2)
                  for b, M, off in o.gspec for i in range(b)])
    np.testing.assert_allclose(e, r["coef_noise_e"], rtol=2e-5)
    hs = o.heap(o.fwd(sinusoids(1)))
    assert snr_db(r["coef_sines_s"], hs.reshape(-1)[::STRIDE]) > 120


def test_round_trip():
    o, r = oracle(), ref()
    x = x_noise()
    y = o.bwd(o.fwd(x))
    assert snr_db(x, y) > 200  # float64 oracle is exact to ~1e-15
    assert snr_db(r["y_noise_s"], y.reshape(-1)[::STRIDE]) > 125
    assert r["rt_noise_db"] > 125


def test_gradients_match_reference_autograd():
    o, r = oracle(), ref()
    gc = gc_seed(o.ncoef)
    gx = o.adj_fwd(o.unheap(gc.astype(np.complex128)))
    assert snr_db(r["gx_an_s"], gx.reshape(-1)[::STRIDE]) > 120
    np.testing.assert_allclose(np.sum(gx ** 2), r["gx_an_norm"], rtol=1e-5)
    gk = o.heap(o.adj_bwd(gy_seed()))
    assert snr_db(r["gk_syn_s"], gk.reshape(-1)[::STRIDE]) > 120


def test_adjoint_identity():
    """<A x, c> == <x, A^T c> for both maps (real inner products)."""
    o = oracle()
    x = x_noise().astype(np.float64)
    c = gc_seed(o.ncoef).astype(np.complex128)
    ax = o.heap(o.fwd(x))
    lhs = np.sum(ax.real * c.real + ax.imag * c.imag)
    rhs = np.sum(x * o.adj_fwd(o.unheap(c)))
    assert abs(lhs - rhs) < 1e-9 * abs(lhs)
    y = o.bwd(o.unheap(c))
    gy = gy_seed().astype(np.float64)
    lhs2 = np.sum(y * gy)
    g = o.heap(o.adj_bwd(gy))
    rhs2 = np.sum(c.real * g.real + c.imag * g.imag)
    assert abs(lhs2 - rhs2) < 1e-9 * abs(lhs2)


@pytest.mark.parametrize("L", [150000])
def test_sliced_matches_reference(L):
    r = ref()
    so = SlicedOracle()
    x = chirp(5, L)[None].astype(np.float64)
    assert so.num_slices(L) == int(r["sliced_S"])
    blocks, side = so.fwd(x)
    bs = np.concatenate([c.reshape(-1)[::STRIDE_SLICED] for c in blocks])
    ss = np.concatenate([c.reshape(-1)[::STRIDE_SLICED] for c in side])
    assert snr_db(r["sliced_blocks_s"], bs) > 120
    # the DC / Nyquist side bands of a chirp hold ~1e-6 of the energy, so the
    # reference's float32 leakage bounds their own relative SNR near 110 dB;
    # measured against the whole coefficient set they are at float32 level
    assert snr_db(r["sliced_side_s"], ss) > 105
    assert snr_db(np.concatenate([r["sliced_blocks_s"], r["sliced_side_s"]]),
                  np.concatenate([bs, ss])) > 120
    y = so.bwd(blocks, side, length=L)
    assert snr_db(r["sliced_y_s"], y.reshape(-1)[::STRIDE_SLICED]) > 125
    assert snr_db(x, y) > 200
    np.testing.assert_allclose(so.tw[::64], r["tukey"], atol=1e-7)


@pytest.mark.parametrize("i", range(len(ALT_CONFIGS)))
def test_other_filterbanks_match_reference(i):
    """layout checksums exact, coefficients and round trip against the
    reference on three other banks (130, 170 and 410 bands)"""
    o, r = oracle_alt(i), ref_alt()
    lay = []
    for idx, gv, pos, gdv, conj in o.all_groups:
        b, M = idx.shape
        w = np.arange(1, b * M + 1, dtype=np.int64)
        lay.append([b, M, idx.sum(), (idx.reshape(-1) * w).sum(), pos.sum(), conj.sum(),
                    (gv != 0).sum()])
    np.testing.assert_array_equal(np.array(lay, dtype=np.int64), r[f"alt{i}_layout"])
    x = x_alt()
    h = o.heap(o.fwd(x))
    assert snr_db(r[f"alt{i}_coef_s"], h.reshape(-1)[::STRIDE_ALT]) >= 120
    y = o.bwd(o.fwd(x))
    assert snr_db(r[f"alt{i}_y_s"], y.reshape(-1)[::STRIDE_ALT]) >= 125


def test_oracle_pinned_at_32768_sample_slices():
    """the oracle at audio_len / sl_len 32768 against the reference's own
    outputs (tests/golden/make_golden.py --short): layout exact, coefficients,
    round trip, both gradients and the sliced transform"""
    from fixtures import (N_SHORT, STRIDE_SHORT, gc_short, gy_short, oracle_short,
                          ref_short, x_short, STRIDE_SLICED, chirp)
    from oracle.cqt_oracle import SlicedOracle
    o, r = oracle_short(), ref_short()
    lay = []
    for idx, gv, pos, gdv, conj in o.all_groups:
        b, M = idx.shape
        w = np.arange(1, b * M + 1, dtype=np.int64)
        lay.append([b, M, int(idx.reshape(-1).sum()), int((idx.reshape(-1) * w).sum()),
                    int(pos.reshape(-1).sum()), int(conj.sum()), int((gv != 0).sum())])
    np.testing.assert_array_equal(np.array(lay, dtype=np.int64), r["layout"])
    x = x_short().astype(np.float64)
    h = o.heap(o.fwd(x))
    assert snr_db(r["coef_s"], h.reshape(-1)[::STRIDE_SHORT]) >= 120
    y = o.bwd(o.fwd(x))
    assert snr_db(r["y_s"], y.reshape(-1)[::STRIDE_SHORT]) >= 125
    gx = o.adj_fwd(o.unheap(gc_short(o.ncoef).astype(np.complex128)))
    assert snr_db(r["gx_an_s"], gx.reshape(-1)[::STRIDE_SHORT]) >= 120
    gk = o.heap(o.adj_bwd(gy_short().astype(np.float64)))
    assert snr_db(r["gk_syn_s"], gk.reshape(-1)[::STRIDE_SHORT]) >= 120
    so = SlicedOracle(sl_len=N_SHORT)
    L = 100000
    xc = chirp(35, L)[None].astype(np.float64)
    assert so.num_slices(L) == int(r["sliced_S"])
    bl, sd = so.fwd(xc)
    bs = np.concatenate([c.reshape(-1)[::STRIDE_SLICED] for c in bl])
    assert snr_db(r["sliced_blocks_s"], bs) >= 120
    ys = so.bwd(bl, sd, length=L)
    assert snr_db(r["sliced_y_s"], ys.reshape(-1)[::STRIDE_SLICED]) >= 125
