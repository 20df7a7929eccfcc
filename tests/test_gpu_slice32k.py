"""32768-sample slices: the same engines with the 8192-point spectrum CTAs and
band lengths 16..1024, against the oracle (pinned to the reference at this
length by test_oracle.py) and the reference's own outputs.

Tolerances as everywhere: coefficients >= 120 dB (every band >= 110 dB),
reconstruction >= 125 dB, gradients >= 120 dB; the sliced stream and its
streaming form bit for bit as at 65536.
"""
import numpy as np
import pytest
import torch

from fixtures import (N_SHORT, STRIDE_SHORT, STRIDE_SLICED, chirp, gc_short, gy_short,
                      oracle_short, ref_short, x_short)
from oracle.cqt_oracle import snr_db

pytestmark = pytest.mark.gpu

N = N_SHORT


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(scope="module")
def t(dev):
    from flash_cqt_b200 import OctCQT, TrainableCQT
    return TrainableCQT(OctCQT([3, 4, 2], [8, 16, 32], fs=44100, audio_len=N, device=dev), dev)


def _np(a):
    return a.detach().cpu().numpy()


def test_analysis_matches_oracle_and_reference(t, dev):
    o, r = oracle_short(), ref_short()
    assert t.eng.tables.slice_len == N
    x = x_short()
    h = _np(t.eng.analysis(torch.from_numpy(x).to(dev)))
    want = o.heap(o.fwd(x.astype(np.float64)))
    assert snr_db(want, h) >= 120
    assert snr_db(r["coef_s"], h.reshape(-1)[::STRIDE_SHORT]) >= 120
    for b, M, off in o.gspec:
        for i in range(b):
            s = slice(off + i * M, off + (i + 1) * M)
            assert snr_db(want[:, s], h[:, s]) >= 110, (M, off, i)


@pytest.mark.parametrize("B", [1, 3, 17, 64])
def test_round_trip(t, dev, B):
    g = torch.Generator(device="cpu").manual_seed(300 + B)
    x = torch.randn(B, N, generator=g).to(dev)
    y = t.eng.synthesis(t.eng.analysis(x))
    xs, ys = _np(x).astype(np.float64), _np(y).astype(np.float64)
    for b in range(B):
        assert snr_db(xs[b], ys[b]) >= 125, b


def test_adjoints_match_oracle_and_reference_autograd(t, dev):
    o, r = oracle_short(), ref_short()
    gc = gc_short(o.ncoef)
    gx = _np(t.eng.adj_analysis(torch.from_numpy(gc).to(dev)))
    assert snr_db(o.adj_fwd(o.unheap(gc.astype(np.complex128))), gx) >= 120
    assert snr_db(r["gx_an_s"], gx.reshape(-1)[::STRIDE_SHORT]) >= 120
    gy = gy_short()
    gk = _np(t.eng.adj_synthesis(torch.from_numpy(gy).to(dev)))
    assert snr_db(o.heap(o.adj_bwd(gy.astype(np.float64))), gk) >= 120
    assert snr_db(r["gk_syn_s"], gk.reshape(-1)[::STRIDE_SHORT]) >= 120


def test_train_step_gradient_and_fused_loss(t, dev):
    o = oracle_short()
    x0, tg0 = x_short(), gy_short()
    tgt = torch.from_numpy(tg0).to(dev)
    xe = torch.from_numpy(x0).to(dev).requires_grad_(True)
    ((t.bwd(*t.fwd(xe)) - tgt) ** 2).mean().backward()
    xf = torch.from_numpy(x0).to(dev).requires_grad_(True)
    loss, y = t.mse_loss(*t.fwd(xf), tgt, return_output=True)
    loss.backward()
    yo = o.bwd(o.fwd(x0.astype(np.float64)))
    want = o.adj_fwd(o.adj_bwd(2.0 * (yo - tg0) / yo.size))
    assert snr_db(want, _np(xe.grad).astype(np.float64)) >= 120
    assert snr_db(want, _np(xf.grad).astype(np.float64)) >= 120
    ref_loss = float(((y.double() - tgt.double()) ** 2).mean())
    assert abs(float(loss.detach()) - ref_loss) <= 1e-5 * ref_loss


def test_fused_planar_api(dev):
    from flash_cqt_b200 import FusedOctCQT, OctCQT
    f = FusedOctCQT(OctCQT([3, 4, 2], [8, 16, 32], fs=44100, audio_len=N, device=dev), dev)
    x = torch.from_numpy(x_short()).to(dev)
    kr, ki = f.fwd(x)
    y = f.bwd(kr, ki)
    assert snr_db(_np(x).astype(np.float64), _np(y).astype(np.float64)) >= 125


def test_sliced_matches_oracle_and_reference(dev):
    from flash_cqt_b200 import SlicedCQT
    from oracle.cqt_oracle import SlicedOracle
    r = ref_short()
    L = 100000
    xc = chirp(35, L)
    sl = SlicedCQT([3, 4, 2], [8, 16, 32], fs=44100, sl_len=N, device=dev)
    assert sl._fused(dev) is not None        # the fused sliced kernels, not the generic path
    blocks, side = sl.fwd(torch.from_numpy(xc).to(dev).view(1, 1, L))
    so = SlicedOracle(sl_len=N)
    ob, _ = so.fwd(xc[None].astype(np.float64))
    got = np.concatenate([_np(c).reshape(-1) for c in blocks])
    want = np.concatenate([c.reshape(-1) for c in ob])
    assert snr_db(want, got) >= 120
    bs = np.concatenate([_np(c).reshape(-1)[::STRIDE_SLICED] for c in blocks])
    assert snr_db(r["sliced_blocks_s"], bs) >= 120
    y = sl.bwd(blocks, side, length=L)
    assert snr_db(xc.astype(np.float64), _np(y).reshape(-1).astype(np.float64)) >= 125
    assert snr_db(r["sliced_y_s"], _np(y).reshape(-1)[::STRIDE_SLICED]) >= 125


def test_sliced_stream_matches_whole_buffer(dev):
    from flash_cqt_b200 import SlicedCQT
    sl = SlicedCQT([3, 4, 2], [8, 16, 32], fs=44100, sl_len=N, device=dev)
    hop = sl.hop
    n = 5
    x = torch.randn(2, 1, n * hop, generator=torch.Generator(device="cpu").manual_seed(9)).to(dev)
    wb, ws = sl.fwd(x)
    out = list(sl.stream_fwd(iter([x[..., i * hop:(i + 1) * hop] for i in range(n)])))
    for k, (bl, sd) in enumerate(out):
        for c, blk, m in zip(bl, wb, sl.size_per_oct):
            assert torch.equal(c, blk[..., k * m:(k + 1) * m])
    ys = torch.cat(list(sl.stream_bwd(iter(out))), dim=-1)
    assert torch.equal(ys, sl.bwd(wb, ws)[..., :n * hop])
