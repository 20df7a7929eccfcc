"""numpy model of the CUDA kernels' dataflow and index arithmetic.

Each function mirrors one kernel of ``flash_cqt_b200/csrc`` step for step
(same stage radices, same Stockham read/write indices, same per-CTA split of
the packed FFT, same untangle/retangle quads), but runs vectorised over the
butterfly index.  The CPU tests compare it with numpy's FFT and with the
oracle, so an index error shows up here before any GPU time is spent.
"""
import numpy as np

N = 65536
L = N // 2          # packed complex length
HALFL = L // 2      # per-CTA sub-transform length (16384)


def W(base, e, sign=-1):
    return np.exp(sign * 2j * np.pi * np.asarray(e, dtype=np.float64) / base)


def stockham(u, radices, sign):
    """Stockham autosort FFT of u (last axis) with the given stage radices.

    Stage with radix R and span NS: butterfly j reads u[j + r * M / R],
    multiplies by W_{NS R}^{r k} (k = j mod NS), runs a length-R DFT and
    writes element r to (j // NS) * NS * R + k + r * NS."""
    M = u.shape[-1]
    ns = 1
    for R in radices:
        nb = M // R
        j = np.arange(nb)
        k = j % ns
        r = np.arange(R)
        v = u[..., j[:, None] + r[None, :] * (M // R)]          # [.., nb, R]
        if ns > 1:
            v = v * W(ns * R, r[None, :] * k[:, None], sign)
        v = np.fft.fft(v, axis=-1) if sign < 0 else np.fft.ifft(v, axis=-1) * R
        out = np.empty_like(u)
        dst = (j // ns)[:, None] * ns * R + k[:, None] + r[None, :] * ns
        out[..., dst] = v
        u = out
        ns *= R
    assert ns == M
    return u


SPEC_RADICES_P32 = (32, 32, 16)
SPEC_RADICES_P16 = (16, 16, 16, 4)
SPEC_RADICES = SPEC_RADICES_P16


def spectrum_fwd(x):
    """x [B, N] real -> X [B, N/2 + 1] = rfft(x), the way the two CTAs of a
    slice compute it: CTA h forms the radix-2 DIF half u_h, runs the 16384
    point Stockham FFT, then untangles the (q, L - q) pairs of its parity."""
    z = x[..., 0::2] + 1j * x[..., 1::2]
    n = np.arange(HALFL)
    X = np.zeros(x.shape[:-1] + (L + 1,), np.complex128)
    for h in (0, 1):
        if h == 0:
            u = z[..., :HALFL] + z[..., HALFL:]
        else:
            u = (z[..., :HALFL] - z[..., HALFL:]) * W(L, n)
        U = stockham(u, SPEC_RADICES, -1)       # U[k'] = Z[2k' + h]
        if h == 0:
            kp = np.arange(0, HALFL // 2 + 1)        # pairs k' <-> (16384 - k') % 16384
            kq = (HALFL - kp) % HALFL
        else:
            kp = np.arange(0, HALFL // 2)            # pairs k' <-> 16383 - k'
            kq = HALFL - 1 - kp
        q = 2 * kp + h
        qb = L - q                                  # partner bin (L for q = 0)
        zq, zb = U[..., kp], U[..., kq]
        w = W(N, q)
        X[..., q] = 0.5 * (zq + np.conj(zb)) - 0.5j * w * (zq - np.conj(zb))
        X[..., qb] = 0.5 * (zb + np.conj(zq)) + 0.5j * np.conj(w) * (zb - np.conj(zq))
    return X


def spectrum_inv(F):
    """F [B, N/2 + 1] half spectrum -> irfft(F) [B, N] (imaginary parts of the
    DC and Nyquist bins ignored, as irfft does), the way the two CTAs of a
    slice compute it: each CTA retangles the quads {n, 16384 - n, n + 16384,
    32768 - n} into its DIF half u_h, runs the inverse 16384 point Stockham
    FFT and stores the outputs z[2m + h] de-interleaved."""
    F = F.copy()
    F[..., 0] = F[..., 0].real
    F[..., L] = F[..., L].real
    y = np.zeros(F.shape[:-1] + (N,))

    def zs(q):
        # packed spectrum Zs[q] from F[q], F[L - q]  (q in [0, L))
        a, b = F[..., q], np.conj(F[..., L - q])
        return 0.5 * (a + b) + 1j * 0.5 * (a - b) * W(N, q, +1)

    for h in (0, 1):
        n = np.arange(0, HALFL // 2 + 1)           # quad leaders
        m = (HALFL - n) % HALFL
        u = np.zeros(F.shape[:-1] + (HALFL,), np.complex128)
        for idx in (n, m):
            a, b = zs(idx), zs(idx + HALFL)
            u[..., idx] = (a + b) if h == 0 else (a - b) * W(L, idx, +1)
        out = stockham(u, SPEC_RADICES, +1) / L     # z[2m + h]
        y[..., 2 * (2 * np.arange(HALFL) + h)] = out.real
        y[..., 2 * (2 * np.arange(HALFL) + h) + 1] = out.imag
    return y


# band FFT configurations: (points per thread P, stage radices), for the two
# register budgets the band kernels compile for (FCQT_BAND_P = 32 or 16)
BAND_CFG_P32 = {32: (32, (32,)), 64: (32, (32, 2)), 128: (32, (32, 4)),
                256: (32, (32, 8)), 512: (32, (32, 16)), 1024: (32, (32, 32)),
                2048: (32, (32, 32, 2))}
BAND_CFG_P16 = {16: (16, (16,)), 32: (16, (16, 2)), 64: (16, (16, 4)), 128: (16, (16, 8)),
                256: (16, (16, 16)), 512: (16, (16, 16, 2)),
                1024: (16, (16, 16, 4)), 2048: (16, (16, 16, 8))}
BAND_CFG = BAND_CFG_P16


def bands_fwd(X, tab, bands):
    """X [B, N/2+1] -> coefficient heap [B, ncoef]: gather g * X[k] (conj on
    flagged taps) per band, unnormalised inverse DFT via the band's Stockham
    schedule (the 1/M lives in the gain table)."""
    B = X.shape[0]
    out = np.zeros((B, tab["src"].size), np.complex128)
    for M, off in bands:
        s = tab["src"][off:off + M].astype(np.int64)
        g = tab["gain"][off:off + M].astype(np.float64)
        live = s >= 0
        k = np.where(live, s & 0xFFFF, 0)
        v = X[:, k]
        v = np.where((s & 0x10000).astype(bool) & live, np.conj(v), v) * g * live
        out[:, off:off + M] = stockham(v, BAND_CFG[M][1], +1)
    return out


def bands_inv(K, tab, bands, nplanes, es):
    """coefficient heap -> colour planes E [B, nplanes * es]: forward DFT per
    band, per-tap gains (re, im), store at the tap's plane/bin."""
    B = K.shape[0]
    E = np.full((B, nplanes * es), np.nan, np.complex128)
    for M, off in bands:
        d = tab["dest"][off:off + M].astype(np.int64)
        v = stockham(K[:, off:off + M], BAND_CFG[M][1], -1)
        v = v.real * tab["gre"][off:off + M] + 1j * v.imag * tab["gim"][off:off + M]
        live = d >= 0
        assert np.all(np.isnan(E[:, d[live]])), "plane collision"
        E[:, d[live]] = v[:, live]
    return E


def planes_reduce(E, mask, nplanes, es):
    """F[q] = sum of the planes flagged in mask[q], in plane order."""
    B = E.shape[0]
    F = np.zeros((B, L + 1), np.complex128)
    for p in range(nplanes):
        sel = (mask[:L + 1] >> p) & 1 == 1
        F[:, sel] += E[:, p * es + np.nonzero(sel)[0]]
    assert not np.isnan(F).any(), "read of an unwritten plane slot"
    return F
