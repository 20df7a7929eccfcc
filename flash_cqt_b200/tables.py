"""Kernel tables for the two engines (analysis engine, synthesis engine).

Analysis engine (``bands_fwd`` over the untangled half spectrum X = rfft(x)):
    coef[band, n] = sum_m gain[m] * X~[src[m]] * exp(+2 pi i m n / M)
with X~ = X or conj(X) per tap.  One table set per use:

* ``analysis``  src = window gather bin (``oct_cqt.py:84-96``; mirrored taps
  conjugated), gain = window / M  (the ifft's 1/M folded in);
* ``adj_synth`` the transpose of the synthesis (``fused.py:466-474`` proves
  the constants): src = scatter bin, gain = dual * (2/N), halved on the DC
  and Nyquist bins.

Synthesis engine (``bands_inv`` into colour planes, then ``spectrum_inv``):
    E[plane, bin] = (Re S[m] * gre[m], Im S[m] * gim[m]),  S = DFT_M(coef)
    y = irfft(sum over the planes flagged in mask[bin])

* ``synth``   dest = scatter bin of live dual taps (``oct_cqt.py:98-117``),
  gre = gim = dual * M;
* ``adj_an``  the transpose of the analysis (``fused.py:452-464``): dest =
  analysis gather bin, gre = window / M * N/2 (doubled on DC / Nyquist), gim
  = +-gre (sign = conjugation, zero on DC / Nyquist).

Colour planes replace the reference's atomic scatter (``radix_impl.cuh:100-
129``): every live tap gets a (plane, bin) slot of its own, chosen greedily per
band run, so the reduction in ``spectrum_inv`` reads each slot exactly once in
a fixed plane order -- deterministic, no zeroing, no atomics.
"""
import math

import numpy as np

N_SLICE = 65536
SLICE_LENS = (65536, 32768)   # slice lengths the CUDA engines are built for
HALF = N_SLICE // 2
PLANE_STRIDE = HALF + 8   # complex elements per colour plane (64-B multiple)
MAX_PLANES = 4


def plane_stride(n):
    """complex elements per spectrum row / colour plane for n-sample slices
    (n / 2 + 8: every row a 64-byte multiple)"""
    return n // 2 + 8
FWD_SETS = ("analysis", "adj_synth")
INV_SETS = ("synth", "adj_an")
BAND_ORDER = (2048, 1024, 512, 256, 128, 64, 32, 16)   # scheduling classes


def _assign_planes(runs, nbins):
    """Greedy colouring of tap runs: each run (array of bins, distinct within
    the run) gets the lowest plane where none of its bins is taken."""
    used = np.zeros((MAX_PLANES, nbins), bool)
    plane = []
    for bins in runs:
        for p in range(MAX_PLANES):
            if not used[p, bins].any():
                used[p, bins] = True
                plane.append(p)
                break
        else:
            raise RuntimeError("scatter overlap exceeds %d planes" % MAX_PLANES)
    mask = np.zeros(nbins, np.uint8)
    for p in range(MAX_PLANES):
        mask |= (used[p].astype(np.uint8) << p)
    nplanes = int(max(plane) + 1) if plane else 1
    return plane, mask, nplanes


def build_tables(heap):
    """All host tables for one HeapLayout (numpy, float32 / int32)."""
    bank = heap.bank
    N = bank.nn
    if N not in SLICE_LENS:
        raise ValueError("the CUDA engines are built for 65536- and 32768-sample "
                         "slices, got %d" % N)
    lens = sorted({int(M) for _, M, _ in heap.gspec})
    bad = [M for M in lens if M not in BAND_ORDER]
    if bad:
        raise ValueError("the band kernels take block lengths that are powers of two in "
                         "16..2048; this filterbank needs %s" % bad)
    half = N // 2
    stride = plane_stride(N)
    nc = heap.ncoef
    groups = heap.groups + heap.side_groups
    src_an = np.full(nc, -1, np.int32)
    gain_an = np.zeros(nc, np.float64)
    src_as = np.full(nc, -1, np.int32)
    gain_as = np.zeros(nc, np.float64)
    dest_bins = {s: np.full(nc, -1, np.int64) for s in INV_SETS}
    gre = {s: np.zeros(nc, np.float64) for s in INV_SETS}
    gim = {s: np.zeros(nc, np.float64) for s in INV_SETS}
    runs = {s: [] for s in INV_SETS}     # (tap indices) per run
    for (b, M, off), (idx, gv, pos, gdv, conj) in zip(heap.gspec, groups):
        for r in range(b):
            o = off + r * M
            sl = slice(o, o + M)
            live_a = gv[r] != 0
            live_s = gdv[r] != 0
            k = idx[r]
            cj = conj[r]
            # analysis gather
            src_an[sl] = np.where(live_a, k | (cj.astype(np.int64) << 16), -1)
            gain_an[sl] = np.where(live_a, gv[r] / M, 0.0)
            # transpose of the synthesis: gather at the scatter bins
            edge_s = (pos[r] == 0) | (pos[r] == half)
            src_as[sl] = np.where(live_s, pos[r], -1)
            gain_as[sl] = np.where(live_s, gdv[r] * (2.0 / N)
                                   * np.where(edge_s, 0.5, 1.0), 0.0)
            # synthesis scatter
            dest_bins["synth"][sl] = np.where(live_s, pos[r], -1)
            gre["synth"][sl] = gim["synth"][sl] = np.where(live_s, gdv[r], 0.0)
            taps = np.arange(o, o + M)
            runs["synth"].append(taps[live_s])
            # transpose of the analysis: scatter at the gather bins
            edge_a = (k == 0) | (k == half)
            ga = gv[r] / M * (N / 2.0)
            dest_bins["adj_an"][sl] = np.where(live_a, k, -1)
            gre["adj_an"][sl] = np.where(live_a, ga * np.where(edge_a, 2.0, 1.0), 0.0)
            gim["adj_an"][sl] = np.where(live_a & ~edge_a,
                                         ga * np.where(cj, -1.0, 1.0), 0.0)
            # mirrored and direct taps of a side band may hit the same bin:
            # they form separate runs
            runs["adj_an"].append(taps[live_a & ~cj])
            if (live_a & cj).any():
                runs["adj_an"].append(taps[live_a & cj])

    t = {}
    t["fwd"] = {
        "analysis": (src_an, gain_an.astype(np.float32)),
        "adj_synth": (src_as, gain_as.astype(np.float32)),
    }
    # per band: the contiguous half-spectrum segment [lo, lo + n) holding all
    # live gather bins of the band (staged into shared memory by bands_fwd)
    t["seg"] = {}
    for nm, (src, _) in t["fwd"].items():
        seg = np.zeros((len(heap.bands), 2), np.int32)
        for i, (M, o) in enumerate(heap.bands):
            s_ = src[o:o + M]
            bins = (s_[s_ >= 0] & 0xFFFF).astype(np.int64)
            if bins.size:
                lo, hi = int(bins.min()), int(bins.max())
                if hi - lo + 1 > M:
                    raise RuntimeError("band %d gathers from more than M bins" % i)
                seg[i] = (lo, hi - lo + 1)
        t["seg"][nm] = seg
    t["inv"] = {}
    for s in INV_SETS:
        rr = [rn for rn in runs[s] if rn.size]
        plane, mask, nplanes = _assign_planes(
            [dest_bins[s][rn] for rn in rr], half + 1)
        dest = np.full(nc, -1, np.int64)
        for rn, p in zip(rr, plane):
            dest[rn] = p * stride + dest_bins[s][rn]
        maskp = np.zeros(stride, np.uint8)
        maskp[:half + 1] = mask
        t["inv"][s] = (dest.astype(np.int32), gre[s].astype(np.float32),
                       gim[s].astype(np.float32), maskp, nplanes)
    t["nplanes"] = max(v[4] for v in t["inv"].values())

    # per band geometry for the closed-form octave path: lo, l, Lg, flags.
    # A band takes the closed form only where it reproduces every per-tap
    # table entry exactly; the DC / Nyquist side bands, and octave bands that
    # touch an edge bin or a mirrored (conjugated) bin, take the table path
    # (flags bit 0).
    geom = np.zeros((len(heap.bands), 4), np.int32)
    nocts = sum(g[0].shape[0] for g in heap.groups)
    for i, (M, o) in enumerate(heap.bands):
        if i >= nocts:
            geom[i] = (0, 0, 0, 1)              # side band: table path
            continue
        rg = bank.ranges[i + 1]                 # octave bands are windows 1..nb
        lg = rg.size
        g = _octave_geometry(t, o, M, int(rg[0]), lg // 2, lg, stride)
        geom[i] = g if g is not None else (0, 0, 0, 1)
    t["band_geom"] = geom
    # coefficient groups in heap order (octave groups roll in the sliced
    # layout, the DC and Nyquist side groups do not)
    t["group_count"] = np.array([g[0] for g in heap.gspec], np.int32)
    t["group_roll"] = np.array([1] * len(heap.groups) + [0] * len(heap.side_groups),
                               np.int32)

    # band scheduling classes, largest block length first
    bands = heap.bands
    cls = []
    order = []
    for M in BAND_ORDER:
        ids = [i for i, (m, _) in enumerate(bands) if m == M]
        if ids:
            cls.append((M, len(ids), len(order)))
            order.extend(ids)
    t["classes"] = cls
    t["band_list"] = np.array(order, np.int32)
    t["band_off"] = np.array([o for _, o in bands], np.int32)
    t["band_len"] = np.array([m for m, _ in bands], np.int32)

    # twiddles: W_2048^e for the band FFTs, two-level W_65536 for the packed
    # FFT engine (W^e = hi[e >> 8] * lo[e & 255]); float64 maths, one rounding
    e = np.arange(2048)
    t["tw2048"] = _cplx32(np.exp(-2j * math.pi * e / 2048))
    e = np.arange(256)
    t["tw_hi"] = _cplx32(np.exp(-2j * math.pi * (256 * e) / 65536))
    t["tw_lo"] = _cplx32(np.exp(-2j * math.pi * e / 65536))
    t["slice_len"] = N
    return t


def _octave_geometry(t, o, M, lo, l, lg, stride=PLANE_STRIDE):
    """(lo, l, Lg, flags) when tap m of the band at heap offset o maps to bin
    lo + ((m + l) mod M) inside the window support (live iff that index is
    below Lg) in every gather and scatter table, with one colour plane per
    inverse set and equal real / imaginary scatter gains; else None"""
    m = np.arange(M)
    ii = (m + l) % M
    live = ii < lg
    bins = lo + ii
    for src, gain in t["fwd"].values():
        s_, g_ = src[o:o + M], gain[o:o + M]
        ok = np.where(s_ >= 0, live & (s_ == bins), g_ == 0)
        if not ok.all():
            return None
    flags = 0
    for w, s in enumerate(INV_SETS):
        dest, gr, gi = (a[o:o + M] for a in t["inv"][s][:3])
        writes = live & (gr != 0)
        if ((dest >= 0) != writes).any() or (gi[writes] != gr[writes]).any():
            return None
        planes = np.unique(dest[writes] // stride)
        if planes.size != 1 or (dest[writes] % stride != bins[writes]).any():
            return None
        flags |= int(planes[0]) << (4 + 4 * w)
    return (lo, l, lg, flags)


def _cplx32(z):
    out = np.empty(z.shape + (2,), np.float32)
    out[..., 0] = z.real
    out[..., 1] = z.imag
    return out


# ---------------------------------------------------------------- C export
# Field order of the binary table file: the pointer fields of
# cqt_host_tables (include/flash_cqt_b200.h) in declaration order, with the
# two plane counts as one-element int32 arrays after their masks.
HOST_FIELDS = [
    ("band_off", np.int32), ("band_list", np.int32), ("band_geom", np.int32),
    ("group_count", np.int32), ("group_roll", np.int32),
    ("class_len", np.int32), ("class_count", np.int32), ("class_first", np.int32),
    ("an_src", np.int32), ("an_gain", np.float32), ("an_seg", np.int32),
    ("as_src", np.int32), ("as_gain", np.float32), ("as_seg", np.int32),
    ("sy_dest", np.int32), ("sy_gre", np.float32), ("sy_gim", np.float32),
    ("sy_mask", np.uint8), ("sy_nplanes", np.int32),
    ("aa_dest", np.int32), ("aa_gre", np.float32), ("aa_gim", np.float32),
    ("aa_mask", np.uint8), ("aa_nplanes", np.int32),
    ("tw2048", np.float32), ("tw_hi", np.float32), ("tw_lo", np.float32),
]


def host_arrays(tabs):
    """the cqt_host_tables arrays of `tabs` by field name"""
    cls = tabs["classes"]
    a = {
        "band_off": tabs["band_off"], "band_list": tabs["band_list"],
        "band_geom": tabs["band_geom"], "group_count": tabs["group_count"],
        "group_roll": tabs["group_roll"],
        "class_len": [c[0] for c in cls], "class_count": [c[1] for c in cls],
        "class_first": [c[2] for c in cls],
        "an_src": tabs["fwd"]["analysis"][0], "an_gain": tabs["fwd"]["analysis"][1],
        "an_seg": tabs["seg"]["analysis"],
        "as_src": tabs["fwd"]["adj_synth"][0], "as_gain": tabs["fwd"]["adj_synth"][1],
        "as_seg": tabs["seg"]["adj_synth"],
        "tw2048": tabs["tw2048"], "tw_hi": tabs["tw_hi"], "tw_lo": tabs["tw_lo"],
    }
    for pre, key in (("sy", "synth"), ("aa", "adj_an")):
        d, gr, gi, mk, npl = tabs["inv"][key]
        a.update({pre + "_dest": d, pre + "_gre": gr, pre + "_gim": gi,
                  pre + "_mask": mk, pre + "_nplanes": [npl]})
    return {k: np.ascontiguousarray(np.asarray(v), dtype=dt).reshape(-1)
            for (k, dt), v in ((f, a[f[0]]) for f in HOST_FIELDS)}


def save_host_tables(tabs, path):
    """Write the host tables for C consumers of the library: for every field
    of HOST_FIELDS in order, an int64 element count and the raw
    little-endian elements.  nbands, ncoef, ngroups and nclasses are the
    counts of band_off, an_src, group_count and class_len."""
    arrs = host_arrays(tabs)
    with open(path, "wb") as f:
        for name, _ in HOST_FIELDS:
            a = arrs[name]
            f.write(np.int64(a.size).tobytes())
            f.write(a.tobytes())
