"""CPU oracle for the factored constant-Q transform -- TEST INFRASTRUCTURE ONLY.

This module is the parity checker for the CUDA product path.  Only files under
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import it; the product package never does.

It restates, in float64 numpy, the reference algorithm of Flash-CQT:

* the filterbank (windows, window ranges, canonical dual windows) of
  ``flash_cqt/ref_util.py:16-52`` and ``flash_cqt/filterbank.py:26-122``;
* the per-group gather/window/scatter layout of ``flash_cqt/oct_cqt.py:36-70``
  (octave groups, then the DC and Nyquist side groups, ``oct_cqt.py:72-82``);
* ``OctCQT.fwd`` (``oct_cqt.py:84-96``): rfft, gather x window, ifft per group,
  conjugate-masked side blocks;
* ``OctCQT.bwd`` (``oct_cqt.py:98-117``): fft x dual, flat index_add into the
  half spectrum, irfft;
* the exact adjoints (transposes, in torch's complex-gradient convention
  grad = dL/dRe + i dL/dIm) of both maps, which is what torch autograd through
  ``OctCQT`` computes (the reference proves the same constants, N/2 and 2/N, in
  ``bench/autograd_check.py:63-138``).

Parity is pinned against fixtures produced by the reference itself
(``tests/golden/make_golden.py`` imports the reference read-only and runs it);
``tests/test_oracle.py`` checks this module against them.
"""
import math

import numpy as np


# ---------------------------------------------------------------- filterbank
def hann(length):
    """Zero-phase periodic Hann window, peak at index 0 (ref_util.py:16-22)."""
    r = np.arange(length, dtype=np.float64) * (2.0 * np.pi / length)
    return 0.5 * (np.cos(r) + 1.0)


def window_ranges(lengths, centres, total):
    """Absolute spectrum bins covered by each window (ref_util.py:25-40).

    Window ``i`` of length ``Lg`` is centred on the cumulative shift position
    and spans ``[-(Lg // 2), Lg - Lg // 2)`` around it, modulo ``total``."""
    shift = np.concatenate(([np.mod(-centres[-1], total)],
                            centres[1:] - centres[:-1]))
    pos = np.cumsum(shift)
    nn = int(pos[-1])
    pos = pos - shift[0]
    out = []
    for lg, p in zip(lengths, pos):
        out.append(np.mod(np.arange(-(lg // 2) + p, lg - lg // 2 + p,
                                    dtype=np.int64), nn))
    return out, nn


def canonical_duals(windows, ranges, nn, block_sizes):
    """Painless-case canonical dual windows (ref_util.py:43-52): divide each
    window by the diagonal of the frame operator sum_i M_i |g_i|^2."""
    diag = np.zeros(nn, dtype=np.float64)
    for g, m, rg in zip(windows, block_sizes, ranges):
        np.add.at(diag, rg, np.fft.fftshift(g) ** 2 * m)
    return [g / np.fft.ifftshift(diag[rg]) for g, rg in zip(windows, ranges)]


def _next_pow2(v):
    return 1 if v == 0 else 2 ** math.ceil(math.log2(v))


class Bank:
    """FlexOctBank restated (filterbank.py:26-122), float64 throughout."""

    def __init__(self, num_octs, bins_per_oct, fs, audio_len, min_win=4):
        num_octs = [num_octs] if isinstance(num_octs, int) else list(num_octs)
        bins_per_oct = ([bins_per_oct] if isinstance(bins_per_oct, int)
                        else list(bins_per_oct))
        nyq = fs / 2.0
        scale = float(audio_len) / fs
        K = len(num_octs)
        # top frequency of each group (filterbank.py:51-52)
        tops = [fs * 2.0 ** (-1 - sum(num_octs[j + 1:])) for j in range(K)]
        freqs, lens = [], []
        for j in range(K):
            n, b = num_octs[j], bins_per_oct[j]
            # groups below Nyquist are built with one extra octave that is
            # dropped again (filterbank.py:58-66)
            if tops[j] < nyq:
                fmax, ng = 2.0 * tops[j] - 1e-6, n + 1
            else:
                fmax, ng = tops[j] - 1e-6, n
            fmin = fmax / 2.0 ** ng
            nb = ng * b
            p = 2.0 ** ((math.log2(fmax) - math.log2(fmin)) / (nb - 1))
            q = math.sqrt(p) / (p - 1.0) / 2.0
            f = fmin * p ** np.arange(nb + 1)
            f[-1] = min(f[-1], nyq)
            f = f * scale
            keep = n * b
            m = np.zeros(keep)
            m[0] = np.round(f[0] / q)
            m[1:] = np.round(f[2:keep + 1] - f[0:keep - 1])
            freqs.extend(f[:keep])
            lens.extend(m)
        nbins = len(freqs)
        freqs = np.array(freqs)
        lens = np.array(lens)
        m_dc = np.round(2.0 * freqs[0])
        m_nyq = np.round(nyq * scale - freqs[-2])
        # centre bins, last bin moved midway to Nyquist (filterbank.py:90-94)
        c = np.concatenate(([0.0], freqs, [nyq * scale]))
        c = np.concatenate((c, audio_len - c[-2:0:-1]))
        c[nbins] = 0.5 * (c[nbins - 1] + c[nbins + 1])
        c[nbins + 2] = audio_len - c[nbins]
        centres = np.round(c).astype(np.int64)
        raw = np.concatenate(([m_dc], lens, [m_nyq], lens[::-1]))
        raw = np.clip(raw, min_win, None)
        # per-octave pow2 block sizes, mirrored (filterbank.py:104-112)
        self.oct_bins = [b for n, b in zip(num_octs, bins_per_oct)
                         for _ in range(n)]
        self.size_per_oct = []
        blk = raw.copy()
        i = 1
        for b in self.oct_bins:
            v = _next_pow2(raw[i:i + b].max())
            self.size_per_oct.append(int(v))
            blk[i:i + b] = v
            blk[len(blk) - i - b:len(blk) - i] = v
            i += b
        self.M = blk.astype(np.int64)
        self.g = [hann(int(m)) for m in raw]
        self.wins, self.nn = window_ranges([len(g) for g in self.g], centres,
                                           audio_len)
        assert self.nn == audio_len
        self.gd = canonical_duals(self.g, self.wins, self.nn, self.M)
        self.fbins = nbins
        self.frqs_hz = freqs / scale
        self.M0 = int(self.M[0])
        self.Mnyq = int(self.M[nbins + 1])


# ------------------------------------------------------------------ transform
class OctCQTOracle:
    """OctCQT restated (oct_cqt.py:18-117) in float64 numpy, plus adjoints."""

    def __init__(self, num_octs=(3, 4, 2), bins_per_oct=(8, 16, 32), fs=44100,
                 audio_len=65536):
        self.bank = bank = Bank(num_octs, bins_per_oct, fs, audio_len)
        self.nn = nn = bank.nn
        self.Ls = audio_len
        self.oct_bins = bank.oct_bins
        self.size_per_oct = bank.size_per_oct
        half = nn // 2

        def layout(band_ids, Lo):
            # oct_cqt.py:36-70: first half of the support at [0, r), wrapped
            # tail at [Lo - l, Lo), zeros between
            nb = len(band_ids)
            idx = np.zeros((nb, Lo), np.int64)
            gv = np.zeros((nb, Lo))
            pos = np.zeros((nb, Lo), np.int64)
            gdv = np.zeros((nb, Lo))
            for r_, bi in enumerate(band_ids):
                wr = bank.wins[bi]
                lg = len(wr)
                r, l = (lg + 1) // 2, lg // 2
                gs = np.fft.fftshift(bank.g[bi])
                idx[r_, :r] = wr[l:]
                idx[r_, Lo - l:] = wr[:l]
                gv[r_, :r] = gs[l:]
                gv[r_, Lo - l:] = gs[:l]
                gd = bank.gd[bi] * Lo
                gdv[r_, :r] = gd[:r]
                gdv[r_, Lo - l:] = gd[r:]
                pos[r_, :r] = wr[l:]
                pos[r_, Lo - l:] = wr[:l]
            conj = idx > half
            idx = np.where(conj, nn - idx, idx)
            valid = pos <= half
            gdv = gdv * valid
            pos = np.where(valid, pos, 0)
            return idx, gv, pos, gdv, conj

        self.groups = []
        start = 1
        for i, b in enumerate(self.oct_bins):
            self.groups.append(layout(range(start, start + b),
                                      self.size_per_oct[i]))
            start += b
        self.side_groups = [layout([0], bank.M0),
                            layout([bank.fbins + 1], bank.Mnyq)]
        self.all_groups = self.groups + self.side_groups
        self.gspec = []
        off = 0
        for idx, *_ in self.all_groups:
            b, M = idx.shape
            self.gspec.append((b, M, off))
            off += b * M
        self.ncoef = off

    # forward / inverse -----------------------------------------------------
    def fwd(self, x):
        """x [B, N] real -> list of complex [B, b, M] (octave groups + DC +
        Nyquist), float64."""
        x = np.asarray(x, dtype=np.float64)
        X = np.fft.rfft(x, axis=-1)
        out = []
        for idx, gv, pos, gdv, conj in self.all_groups:
            a = X[..., idx]
            a = np.where(conj, np.conj(a), a) * gv
            out.append(np.fft.ifft(a, axis=-1))
        return out

    def bwd(self, blocks):
        """inverse of fwd (all groups, side included)."""
        B = blocks[0].shape[0]
        F = np.zeros((B, self.nn // 2 + 1), np.complex128)
        for c, (idx, gv, pos, gdv, conj) in zip(blocks, self.all_groups):
            s = np.fft.fft(c, axis=-1) * gdv
            for b in range(B):
                np.add.at(F[b], pos.reshape(-1), s[b].reshape(-1))
        return np.fft.irfft(F, n=self.nn, axis=-1)

    # adjoints (torch complex-gradient convention) --------------------------
    def adj_fwd(self, gblocks):
        """transpose of fwd: coefficient gradients -> gradient w.r.t. x."""
        B = gblocks[0].shape[0]
        N = self.nn
        half = N // 2
        G = np.zeros((B, half + 1), np.complex128)
        for gc, (idx, gv, pos, gdv, conj) in zip(gblocks, self.all_groups):
            M = idx.shape[1]
            gvv = np.fft.fft(gc, axis=-1) / M * gv
            gvv = np.where(conj, np.conj(gvv), gvv)
            for b in range(B):
                np.add.at(G[b], idx.reshape(-1), gvv[b].reshape(-1))
        # rfft transpose: G_x = (N/2) irfft(G') with the DC / Nyquist bins
        # doubled (their imaginary parts carry no gradient)
        G[:, 0] *= 2.0
        G[:, half] *= 2.0
        return (N / 2.0) * np.fft.irfft(G, n=N, axis=-1)

    def adj_bwd(self, gy):
        """transpose of bwd: gradient w.r.t. y -> coefficient gradients."""
        gy = np.asarray(gy, dtype=np.float64)
        N = self.nn
        half = N // 2
        GF = (2.0 / N) * np.fft.rfft(gy, axis=-1)
        GF[:, 0] = 0.5 * GF[:, 0].real
        GF[:, half] = 0.5 * GF[:, half].real
        out = []
        for idx, gv, pos, gdv, conj in self.all_groups:
            M = idx.shape[1]
            gs = GF[:, pos] * gdv
            out.append(np.fft.ifft(gs, axis=-1) * M)
        return out

    # helpers ---------------------------------------------------------------
    def heap(self, blocks):
        """concatenate per-group blocks into one [B, ncoef] complex heap."""
        B = blocks[0].shape[0]
        return np.concatenate([c.reshape(B, -1) for c in blocks], axis=-1)

    def unheap(self, h):
        B = h.shape[0]
        return [h[:, off:off + b * M].reshape(B, b, M)
                for b, M, off in self.gspec]


def snr_db(ref, test):
    """10 log10(|ref|^2 / |ref - test|^2), complex or real, float64."""
    ref = np.asarray(ref)
    test = np.asarray(test)
    if np.iscomplexobj(ref) or np.iscomplexobj(test):
        ref = np.concatenate([np.real(ref).ravel(), np.imag(ref).ravel()])
        test = np.concatenate([np.real(test).ravel(), np.imag(test).ravel()])
    ref = ref.astype(np.float64).ravel()
    test = test.astype(np.float64).ravel()
    e = np.sum((ref - test) ** 2)
    p = np.sum(ref ** 2)
    return float("inf") if e == 0 else float(10.0 * np.log10(p / e))


# ------------------------------------------------------------------ sliced
def tukey(sl_len, tr_area):
    """slice window of sliced.py:26-38 (flat top, Hann transitions)."""
    hhop = sl_len // 4
    htr = tr_area // 2
    w = hann(2 * tr_area)
    tw = np.zeros(sl_len)
    tw[hhop - htr:hhop + htr] = w[tr_area:]
    tw[hhop + htr:3 * hhop - htr] = 1.0
    tw[3 * hhop - htr:3 * hhop + htr] = w[:tr_area]
    return tw


class SlicedOracle:
    """SlicedCQT restated (sliced.py:41-167): 50%-overlap Tukey slicing with
    alternating quarter rolls, per-slice OctCQT, coefficient re-roll and
    overlap-add."""

    def __init__(self, num_octs=(3, 4, 2), bins_per_oct=(8, 16, 32),
                 fs=44100, sl_len=65536, tr_area=None):
        tr_area = sl_len // 4 if tr_area is None else tr_area
        self.sl_len = sl_len
        self.H = sl_len // 4
        self.cqt = OctCQTOracle(num_octs, bins_per_oct, fs, sl_len)
        self.tw = tukey(sl_len, tr_area)
        self.rolls = [m // 4 for m in self.cqt.size_per_oct]

    def num_slices(self, L):
        nb = -(-L // self.H)
        return (nb + 1) // 2 + 1

    def slices(self, x):
        """x [B, L] -> windowed, rolled slices [B, S, sl_len]."""
        B, L = x.shape
        H = self.H
        S = self.num_slices(L)
        nb = -(-L // H)
        xp = np.concatenate([np.zeros((B, 2 * H)), x,
                             np.zeros((B, nb * H - L + 3 * H))], axis=-1)
        sl = np.stack([xp[:, 2 * H * s:2 * H * s + 4 * H] for s in range(S)],
                      axis=1) * self.tw
        out = np.empty_like(sl)
        out[:, 0::2] = np.roll(sl[:, 0::2], -H, axis=-1)
        out[:, 1::2] = np.roll(sl[:, 1::2], H, axis=-1)
        return out

    def fwd(self, x):
        """x [B, L] -> (blocks [B, b, S*M] per octave, side [B, S, 1, M])."""
        x = np.asarray(x, dtype=np.float64)
        B = x.shape[0]
        sl = self.slices(x)
        S = sl.shape[1]
        coef = self.cqt.fwd(sl.reshape(B * S, -1))
        nO = len(self.cqt.groups)
        blocks = []
        for c, r in zip(coef[:nO], self.rolls):
            _, b, M = c.shape
            c = c.reshape(B, S, b, M)
            c2 = np.empty_like(c)
            c2[:, 0::2] = np.roll(c[:, 0::2], r, axis=-1)
            c2[:, 1::2] = np.roll(c[:, 1::2], -r, axis=-1)
            blocks.append(c2.transpose(0, 2, 1, 3).reshape(B, b, S * M))
        side = [c.reshape(B, S, 1, -1) for c in coef[nO:]]
        return blocks, side

    def bwd(self, blocks, side, length=None):
        B = blocks[0].shape[0]
        m0 = self.cqt.size_per_oct[0]
        S = blocks[0].shape[-1] // m0
        per = []
        for c, r in zip(blocks, self.rolls):
            b = c.shape[1]
            M = c.shape[-1] // S
            c = c.reshape(B, b, S, M).transpose(0, 2, 1, 3)
            c2 = np.empty_like(c)
            c2[:, 0::2] = np.roll(c[:, 0::2], -r, axis=-1)
            c2[:, 1::2] = np.roll(c[:, 1::2], r, axis=-1)
            per.append(c2.reshape(B * S, b, M))
        for c in side:
            per.append(c.reshape(B * S, 1, -1))
        y = self.cqt.bwd(per).reshape(B, S, -1)
        H = self.H
        y2 = np.empty_like(y)
        y2[:, 0::2] = np.roll(y[:, 0::2], H, axis=-1)
        y2[:, 1::2] = np.roll(y[:, 1::2], -H, axis=-1)
        out = np.zeros((B, (S + 1) * 2 * H))
        out[:, :S * 2 * H] += y2[:, :, :2 * H].reshape(B, -1)
        out[:, 2 * H:] += y2[:, :, 2 * H:].reshape(B, -1)
        out = out[:, 2 * H:]
        return out if length is None else out[:, :length]
