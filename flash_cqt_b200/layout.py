"""Filterbank and coefficient-heap layout (host side, built once per plan).

The maths is the reference's invertible "oct mode" nonstationary-Gabor bank:
Hann windows centred on a per-group log-spaced frequency grid, window lengths
from the neighbour spacing, per-octave power-of-two block sizes and the
painless-case canonical duals.  It restates

* ``flash_cqt/ref_util.py:16-52``   (Hann window, window ranges, duals),
* ``flash_cqt/filterbank.py:26-122`` (``FlexOctBank`` group rule, DC/Nyquist
  windows, centre bins, block sizes),
* ``flash_cqt/oct_cqt.py:36-82``     (gather / window / scatter layout of one
  block: support start at ``[0, r)``, wrapped tail at ``[M - l, M)``).

Everything is computed in float64 numpy and rounded to float32 only when the
kernel tables are emitted, so the float32 tables are within half an ulp of the
exact values (the reference rounds the windows to float32 before forming the
duals; the difference is ~1e-7 relative, far below the parity tolerances).
"""
import math

import numpy as np


def periodic_hann(n):
    t = np.arange(n, dtype=np.float64) * (2.0 * math.pi / n)
    return 0.5 + 0.5 * np.cos(t)


class Filterbank:
    """Windows, dual windows and per-octave block layout for one slice length."""

    def __init__(self, num_octs, bins_per_oct, fs, audio_len, min_win=4):
        if isinstance(num_octs, int):
            num_octs = [num_octs]
        if isinstance(bins_per_oct, int):
            bins_per_oct = [bins_per_oct]
        if len(num_octs) != len(bins_per_oct):
            raise ValueError("num_octs and bins_per_oct differ in length")
        self.num_octs = list(num_octs)
        self.bins_per_oct = list(bins_per_oct)
        self.fs = fs
        self.Ls = audio_len
        nyq = 0.5 * fs
        to_bins = float(audio_len) / fs

        # per group: top frequency of the group; groups below Nyquist get one
        # extra (dropped) octave so that their spacing matches a standalone
        # CQT of that group
        centre_f, length = [], []
        ngroups = len(self.num_octs)
        for j in range(ngroups):
            top = fs * 2.0 ** (-1 - sum(self.num_octs[j + 1:]))
            n, b = self.num_octs[j], self.bins_per_oct[j]
            extra = top < nyq
            hi = (2.0 * top if extra else top) - 1e-6
            noct = n + (1 if extra else 0)
            lo = hi / 2.0 ** noct
            nb = noct * b
            ratio = 2.0 ** ((math.log2(hi) - math.log2(lo)) / (nb - 1))
            qfac = math.sqrt(ratio) / (ratio - 1.0) / 2.0
            f = lo * ratio ** np.arange(nb + 1)
            f[-1] = min(f[-1], nyq)
            f = f * to_bins
            kept = n * b
            m = np.empty(kept)
            m[0] = np.round(f[0] / qfac)
            m[1:] = np.round(f[2:kept + 1] - f[:kept - 1])
            centre_f.append(f[:kept])
            length.append(m)
        freqs = np.concatenate(centre_f)
        lens = np.concatenate(length)
        nb = freqs.size
        m_dc = np.round(2.0 * freqs[0])
        m_nyq = np.round(nyq * to_bins - freqs[-2])

        # centre bins of all 2 nb + 2 windows (positive half, Nyquist, mirror)
        c = np.concatenate(([0.0], freqs, [nyq * to_bins]))
        c = np.concatenate((c, audio_len - c[-2:0:-1]))
        c[nb] = 0.5 * (c[nb - 1] + c[nb + 1])
        c[nb + 2] = audio_len - c[nb]
        centres = np.round(c).astype(np.int64)

        raw = np.concatenate(([m_dc], lens, [m_nyq], lens[::-1]))
        raw = np.maximum(raw, min_win)

        self.oct_bins = [b for n, b in zip(self.num_octs, self.bins_per_oct)
                         for _ in range(n)]
        self.size_per_oct = []
        blk = raw.copy()
        pos = 1
        for b in self.oct_bins:
            p2 = int(2 ** math.ceil(math.log2(raw[pos:pos + b].max())))
            self.size_per_oct.append(p2)
            blk[pos:pos + b] = p2
            blk[blk.size - pos - b:blk.size - pos] = p2
            pos += b
        self.block = blk.astype(np.int64)

        # windows and their absolute bin ranges
        self.g = [periodic_hann(int(m)) for m in raw]
        # window i sits at the running sum of the centre steps, the walk
        # starting from the wrap-around step of the last centre
        first = np.mod(-centres[-1], audio_len)
        steps = np.concatenate(([first], np.diff(centres)))
        nn = int(np.sum(steps))
        walk = np.cumsum(steps) - first
        if nn != audio_len:
            raise ValueError("window centres do not close the circle")
        self.nn = nn
        self.ranges = []
        for g, p in zip(self.g, walk):
            lg = g.size
            self.ranges.append(np.mod(np.arange(p - lg // 2, p + lg - lg // 2,
                                                dtype=np.int64), nn))
        # painless canonical duals: g_i / sum_j M_j |g_j|^2 on the supports
        frame = np.zeros(nn)
        for g, mb, rg in zip(self.g, self.block, self.ranges):
            np.add.at(frame, rg, np.fft.fftshift(g) ** 2 * mb)
        self.gd = [g / np.fft.ifftshift(frame[rg])
                   for g, rg in zip(self.g, self.ranges)]

        self.fbins = nb
        self.frqs_hz = freqs / to_bins
        self.M0 = int(self.block[0])
        self.Mnyq = int(self.block[nb + 1])


def block_layout(bank, band_ids, Lo):
    """Per-tap arrays of one block of bands sharing block length Lo.

    Returns (idx, gv, pos, gdv, conj) as numpy arrays of shape [b, Lo]:
    the analysis gather bin (mirrored into [0, nn/2], conj set for mirrored
    taps), the window, the synthesis scatter bin (0 where dropped), the dual
    window times Lo (0 where dropped: only bins <= nn/2 are scattered, the
    rest follows from Hermitian symmetry), and the conjugation mask."""
    nn = bank.nn
    half = nn // 2
    b = len(band_ids)
    idx = np.zeros((b, Lo), np.int64)
    gv = np.zeros((b, Lo))
    pos = np.zeros((b, Lo), np.int64)
    gdv = np.zeros((b, Lo))
    for row, bi in enumerate(band_ids):
        rg = bank.ranges[bi]
        lg = rg.size
        r, l = (lg + 1) // 2, lg // 2
        g = np.fft.fftshift(bank.g[bi])
        gd = bank.gd[bi] * Lo
        idx[row, :r], idx[row, Lo - l:] = rg[l:], rg[:l]
        pos[row, :r], pos[row, Lo - l:] = rg[l:], rg[:l]
        gv[row, :r], gv[row, Lo - l:] = g[l:], g[:l]
        gdv[row, :r], gdv[row, Lo - l:] = gd[:r], gd[r:]
    conj = idx > half
    idx = np.where(conj, nn - idx, idx)
    keep = pos <= half
    return idx, gv, np.where(keep, pos, 0), gdv * keep, conj


class HeapLayout:
    """Group and band order of the coefficient heap: the octave groups
    (lowest first), then the DC and the Nyquist side blocks."""

    def __init__(self, bank):
        self.bank = bank
        self.groups = []
        start = 1
        for i, b in enumerate(bank.oct_bins):
            self.groups.append(block_layout(bank, range(start, start + b),
                                            bank.size_per_oct[i]))
            start += b
        self.side_groups = [block_layout(bank, [0], bank.M0),
                            block_layout(bank, [bank.fbins + 1], bank.Mnyq)]
        self.gspec = []
        self.bands = []   # (M, heap offset) per band, heap order
        off = 0
        for idx, *_ in self.groups + self.side_groups:
            b, M = idx.shape
            self.gspec.append((b, M, off))
            for r in range(b):
                self.bands.append((M, off + r * M))
            off += b * M
        self.ncoef = off
