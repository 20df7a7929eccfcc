"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run once, in a container where the reference checkout is mounted read-only::

    python tests/golden/make_golden.py /path/to/Flash-CQT          # default bank
    python tests/golden/make_golden.py /path/to/Flash-CQT --alt    # other banks
    python tests/golden/make_golden.py /path/to/Flash-CQT --short  # 32768-sample slices

It imports the reference package (``flash_cqt``) and runs its own public API
(``OctCQT.fwd/bwd``, torch autograd through them, ``SlicedCQT.fwd/bwd``) on
seeded inputs, then stores small samples and checksums in
``tests/golden/reference_fixtures.npz``.  The tests never import the reference;
they compare ``oracle/`` (and, on a GPU, the CUDA path) with these numbers.

Inputs come from ``signals.py`` (splitmix64 + Box-Muller, bit-reproducible on
every machine), so the fixtures hold reference outputs only.
"""
import pathlib
import sys

import numpy as np

sys.path.insert(0, str(pathlib.Path(__file__).resolve().parent))
from signals import chirp, normal, sinusoids  # noqa: E402

HERE = pathlib.Path(__file__).resolve().parent
STRIDE = 13  # prime sampling stride over flattened coefficient heaps
STRIDE_SLICED = 41


def main(ref_root):
    sys.path.insert(0, str(ref_root))
    import torch
    from flash_cqt import OctCQT, SlicedCQT

    torch.set_num_threads(8)
    N = 65536
    cqt = OctCQT([3, 4, 2], [8, 16, 32], fs=44100, audio_len=N)
    groups = list(cqt.groups) + list(cqt.side_groups)
    out = {}

    # ---- layout checksums (oct_cqt.py:36-82)
    lay = []
    for idx, gv, pos, gdv, conj in groups:
        b, M = idx.shape
        w = torch.arange(1, b * M + 1, dtype=torch.int64)
        lay.append([b, M,
                    int(idx.reshape(-1).sum()), int((idx.reshape(-1) * w).sum()),
                    int(pos.reshape(-1).sum()), int((pos.reshape(-1) * w).sum()),
                    int(conj.sum()), int((gv != 0).sum()), int((gdv != 0).sum())])
        out.setdefault("gv_rows", []).append(gv[0].double().numpy())
        out.setdefault("gdv_rows", []).append(gdv[-1].double().numpy())
    out["layout"] = np.array(lay, dtype=np.int64)
    out["gv_sum"] = np.array([float(g[1].double().sum()) for g in groups])
    out["gv_sq"] = np.array([float(g[1].double().square().sum()) for g in groups])
    out["gdv_sum"] = np.array([float(g[3].double().sum()) for g in groups])
    out["gdv_sq"] = np.array([float(g[3].double().square().sum())
                              for g in groups])
    out["gv_rows"] = np.concatenate(out["gv_rows"])
    out["gdv_rows"] = np.concatenate(out["gdv_rows"])
    out["frqs_hz"] = np.asarray(cqt.frqs_hz, dtype=np.float64)

    def heap(blocks, side):
        allb = list(blocks) + list(side)
        B = allb[0].shape[0]
        return torch.cat([c.reshape(B, -1) for c in allb], -1)

    def band_stats(h):
        # per band energy and complex sum, band = one row of one group
        e, s = [], []
        off = 0
        for idx, *_ in groups:
            b, M = idx.shape
            for r in range(b):
                seg = h[:, off + r * M: off + (r + 1) * M].to(torch.complex128)
                e.append(float(seg.abs().square().sum()))
                s.append(complex(seg.sum()))
            off += b * M
        return np.array(e), np.array(s)

    # ---- config 1: N(0,1) slices, coefficients and round trip
    x = normal(0, (2, N))
    xt = torch.from_numpy(x)
    blocks, side = cqt.fwd(xt)
    h = heap(blocks, side)
    y = cqt.bwd(blocks, side)
    out["coef_noise_s"] = h.reshape(-1)[::STRIDE].numpy()
    out["coef_noise_e"], out["coef_noise_sum"] = band_stats(h)
    out["y_noise_s"] = y.reshape(-1)[::STRIDE].numpy()
    d = (y.double() - xt.double())
    out["rt_noise_db"] = float(10 * torch.log10(xt.double().square().sum()
                                                 / d.square().sum()))

    # ---- config 2 input: sinusoids
    xs = sinusoids(1)
    bs, ss = cqt.fwd(torch.from_numpy(xs))
    hs = heap(bs, ss)
    ys = cqt.bwd(bs, ss)
    out["coef_sines_s"] = hs.reshape(-1)[::STRIDE].numpy()
    out["coef_sines_e"], _ = band_stats(hs)
    out["y_sines_s"] = ys.reshape(-1)[::STRIDE].numpy()

    # ---- gradients through torch autograd (bench/autograd_gpu.py:58-101)
    gcr = normal(11, (2, 2, h.shape[1]))
    gc = (gcr[0] + 1j * gcr[1]).astype(np.complex64)
    xg = xt.clone().requires_grad_(True)
    bl, sd = cqt.fwd(xg)
    hh = heap(bl, sd)
    loss = (torch.view_as_real(hh) * torch.view_as_real(torch.from_numpy(gc))).sum()
    loss.backward()
    out["gx_an_s"] = xg.grad.reshape(-1)[::STRIDE].numpy()
    out["gx_an_norm"] = float(xg.grad.double().square().sum())
    gy = normal(12, (2, N))
    leaves = [c.detach().clone().requires_grad_(True)
              for c in list(blocks) + list(side)]
    ng = len(cqt.groups)
    yy = cqt.bwd(leaves[:ng], leaves[ng:])
    (yy * torch.from_numpy(gy)).sum().backward()
    gk = torch.cat([lv.grad.reshape(2, -1) for lv in leaves], -1)
    out["gk_syn_s"] = gk.reshape(-1)[::STRIDE].numpy()
    out["gk_syn_e"], _ = band_stats(gk)

    # ---- sliced transform on a short chirp (sliced.py:134-167)
    sl = SlicedCQT([3, 4, 2], [8, 16, 32], fs=44100, sl_len=N)
    L = 150000
    xc = chirp(5, L)[None, None]
    sb, sside = sl.fwd(torch.from_numpy(xc))
    sy = sl.bwd(sb, sside, length=L)
    out["sliced_S"] = int(sl._num_slices(L))
    out["sliced_blocks_s"] = np.concatenate(
        [c.reshape(-1)[::STRIDE_SLICED].numpy() for c in sb])
    out["sliced_side_s"] = np.concatenate(
        [c.reshape(-1)[::STRIDE_SLICED].numpy() for c in sside])
    out["sliced_y_s"] = sy.reshape(-1)[::STRIDE_SLICED].numpy()
    xd = torch.from_numpy(xc).double()
    out["sliced_rt_db"] = float(10 * torch.log10(
        xd.square().sum() / (sy.double() - xd).square().sum()))
    out["tukey"] = sl.tw.double().numpy()[::64]

    np.savez_compressed(HERE / "reference_fixtures.npz", **out)
    for k, v in out.items():
        v = np.asarray(v)
        print(f"{k:18s} {str(v.dtype):10s} {v.shape}")
    print("round trip (noise)", out["rt_noise_db"], "sliced", out["sliced_rt_db"])


# Filterbanks other than the default, all with band lengths 32..2048 (the
# range of the reference's fused kernels, radix_impl.cuh:435-441): one inside
# the default's band count, two above it.
ALT_CONFIGS = [([4, 4, 1], [8, 16, 32]), ([2, 2, 2, 3], [8, 12, 16, 32]),
               ([3, 4, 2], [8, 64, 64])]
STRIDE_ALT = 37


def main_alt(ref_root):
    """reference_fixtures_alt.npz: per alternative filterbank, the layout
    checksums, strided coefficient samples and the round trip of two N(0,1)
    slices through the reference OctCQT"""
    sys.path.insert(0, str(ref_root))
    import torch
    from flash_cqt import OctCQT

    torch.set_num_threads(8)
    N = 65536
    out = {}
    x = normal(21, (2, N))
    xt = torch.from_numpy(x)
    for i, (no, bpo) in enumerate(ALT_CONFIGS):
        cqt = OctCQT(no, bpo, fs=44100, audio_len=N)
        groups = list(cqt.groups) + list(cqt.side_groups)
        lay = []
        for idx, gv, pos, gdv, conj in groups:
            b, M = idx.shape
            w = torch.arange(1, b * M + 1, dtype=torch.int64)
            lay.append([b, M, int(idx.reshape(-1).sum()), int((idx.reshape(-1) * w).sum()),
                        int(pos.reshape(-1).sum()), int(conj.sum()), int((gv != 0).sum())])
        blocks, side = cqt.fwd(xt)
        h = torch.cat([c.reshape(2, -1) for c in list(blocks) + list(side)], -1)
        y = cqt.bwd(blocks, side)
        out[f"alt{i}_layout"] = np.array(lay, dtype=np.int64)
        out[f"alt{i}_coef_s"] = h.reshape(-1)[::STRIDE_ALT].numpy()
        out[f"alt{i}_y_s"] = y.reshape(-1)[::STRIDE_ALT].numpy()
        print(no, bpo, "bands", sum(g[0].shape[0] for g in groups), "ncoef", h.shape[1])
    np.savez_compressed(HERE / "reference_fixtures_alt.npz", **out)


# 32768-sample slices of the default bank (band lengths 16..1024)
N_SHORT = 32768
STRIDE_SHORT = 29


def main_short(ref_root):
    """reference_fixtures_32k.npz: the default bank at audio_len / sl_len
    32768 -- layout checksums, strided coefficients and round trip of two
    N(0,1) slices, the gradients of both transforms through torch autograd,
    and the sliced transform of a short chirp"""
    sys.path.insert(0, str(ref_root))
    import torch
    from flash_cqt import OctCQT, SlicedCQT

    torch.set_num_threads(8)
    N = N_SHORT
    cqt = OctCQT([3, 4, 2], [8, 16, 32], fs=44100, audio_len=N)
    groups = list(cqt.groups) + list(cqt.side_groups)
    out = {}
    lay = []
    for idx, gv, pos, gdv, conj in groups:
        b, M = idx.shape
        w = torch.arange(1, b * M + 1, dtype=torch.int64)
        lay.append([b, M, int(idx.reshape(-1).sum()), int((idx.reshape(-1) * w).sum()),
                    int(pos.reshape(-1).sum()), int(conj.sum()), int((gv != 0).sum())])
    out["layout"] = np.array(lay, dtype=np.int64)
    x = normal(31, (2, N))
    xt = torch.from_numpy(x)
    blocks, side = cqt.fwd(xt)
    h = torch.cat([c.reshape(2, -1) for c in list(blocks) + list(side)], -1)
    y = cqt.bwd(blocks, side)
    out["coef_s"] = h.reshape(-1)[::STRIDE_SHORT].numpy()
    out["y_s"] = y.reshape(-1)[::STRIDE_SHORT].numpy()
    gcr = normal(32, (2, 2, h.shape[1]))
    gc = (gcr[0] + 1j * gcr[1]).astype(np.complex64)
    xg = xt.clone().requires_grad_(True)
    bl, sd = cqt.fwd(xg)
    hh = torch.cat([c.reshape(2, -1) for c in list(bl) + list(sd)], -1)
    (torch.view_as_real(hh) * torch.view_as_real(torch.from_numpy(gc))).sum().backward()
    out["gx_an_s"] = xg.grad.reshape(-1)[::STRIDE_SHORT].numpy()
    gy = normal(33, (2, N))
    leaves = [c.detach().clone().requires_grad_(True) for c in list(blocks) + list(side)]
    ng = len(cqt.groups)
    (cqt.bwd(leaves[:ng], leaves[ng:]) * torch.from_numpy(gy)).sum().backward()
    gk = torch.cat([lv.grad.reshape(2, -1) for lv in leaves], -1)
    out["gk_syn_s"] = gk.reshape(-1)[::STRIDE_SHORT].numpy()
    sl = SlicedCQT([3, 4, 2], [8, 16, 32], fs=44100, sl_len=N)
    L = 100000
    xc = chirp(35, L)[None, None]
    sb, sside = sl.fwd(torch.from_numpy(xc))
    sy = sl.bwd(sb, sside, length=L)
    out["sliced_S"] = int(sl._num_slices(L))
    out["sliced_blocks_s"] = np.concatenate([c.reshape(-1)[::STRIDE_SLICED].numpy()
                                             for c in sb])
    out["sliced_y_s"] = sy.reshape(-1)[::STRIDE_SLICED].numpy()
    np.savez_compressed(HERE / "reference_fixtures_32k.npz", **out)
    print("bands", sum(g[0].shape[0] for g in groups), "ncoef", h.shape[1],
          "sliced S", out["sliced_S"])


if __name__ == "__main__":
    if len(sys.argv) not in (2, 3) or (len(sys.argv) == 3
                                       and sys.argv[2] not in ("--alt", "--short")):
        raise SystemExit("usage: make_golden.py <reference checkout> [--alt | --short]")
    if len(sys.argv) == 3 and sys.argv[2] == "--alt":
        main_alt(pathlib.Path(sys.argv[1]))
    elif len(sys.argv) == 3:
        main_short(pathlib.Path(sys.argv[1]))
    else:
        main(pathlib.Path(sys.argv[1]))
