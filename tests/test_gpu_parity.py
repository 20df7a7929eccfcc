"""Parity of the CUDA path (through the C ABI) with the CPU oracle.

Tolerances (from the north star): coefficients >= 120 dB relative SNR against
the oracle, reconstruction >= 125 dB, gradients >= 120 dB against the oracle's
exact adjoints (which are pinned to torch autograd through the reference).
"""
import pathlib

import numpy as np
import pytest
import torch

from fixtures import STRIDE, gc_seed, gy_seed, oracle, ref, sinusoids, x_noise
from oracle.cqt_oracle import snr_db

pytestmark = pytest.mark.gpu

COEF_DB = 120.0
RT_DB = 125.0
GRAD_DB = 120.0


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(scope="module")
def eng(dev):
    from flash_cqt_b200.engine import Engine
    return Engine.from_params([3, 4, 2], [8, 16, 32], 44100, 65536, dev)


def _np(t):
    return t.detach().cpu().numpy()


def test_analysis_matches_oracle_and_reference(eng, dev):
    o, r = oracle(), ref()
    x = x_noise()
    h = _np(eng.analysis(torch.from_numpy(x).to(dev)))
    want = o.heap(o.fwd(x.astype(np.float64)))
    assert snr_db(want, h) >= COEF_DB
    assert snr_db(r["coef_noise_s"], h.reshape(-1)[::STRIDE]) >= COEF_DB
    # every band on its own, not just the aggregate
    for b, M, off in o.gspec:
        for i in range(b):
            s = slice(off + i * M, off + (i + 1) * M)
            assert snr_db(want[:, s], h[:, s]) >= 110, (M, off, i)


def test_analysis_sinusoids(eng, dev):
    o, r = oracle(), ref()
    x = sinusoids(1)
    h = _np(eng.analysis(torch.from_numpy(x).to(dev)))
    assert snr_db(o.heap(o.fwd(x.astype(np.float64))), h) >= COEF_DB
    assert snr_db(r["coef_sines_s"], h.reshape(-1)[::STRIDE]) >= COEF_DB


def test_synthesis_matches_oracle(eng, dev):
    o = oracle()
    x = x_noise()
    want = o.heap(o.fwd(x.astype(np.float64)))
    c = torch.from_numpy(want.astype(np.complex64)).to(dev)
    y = _np(eng.synthesis(c))
    assert snr_db(o.bwd(o.unheap(want)), y) >= RT_DB
    assert snr_db(x, y) >= RT_DB


@pytest.mark.parametrize("B", [1, 3, 5, 17, 64])
def test_round_trip_batches(eng, dev, B):
    g = torch.Generator(device="cpu").manual_seed(100 + B)
    x = torch.randn(B, 65536, generator=g).to(dev)
    y = eng.synthesis(eng.analysis(x))
    xs, ys = _np(x).astype(np.float64), _np(y).astype(np.float64)
    for b in range(B):
        assert snr_db(xs[b], ys[b]) >= RT_DB, b


def test_adjoints_match_oracle(eng, dev):
    o = oracle()
    gc = gc_seed(o.ncoef)
    gx = _np(eng.adj_analysis(torch.from_numpy(gc).to(dev)))
    assert snr_db(o.adj_fwd(o.unheap(gc.astype(np.complex128))), gx) >= GRAD_DB
    gy = gy_seed()
    gk = _np(eng.adj_synthesis(torch.from_numpy(gy).to(dev)))
    assert snr_db(o.heap(o.adj_bwd(gy.astype(np.float64))), gk) >= GRAD_DB


def test_adjoints_match_reference_autograd_fixtures(eng, dev):
    r = ref()
    o = oracle()
    gx = _np(eng.adj_analysis(torch.from_numpy(gc_seed(o.ncoef)).to(dev)))
    assert snr_db(r["gx_an_s"], gx.reshape(-1)[::STRIDE]) >= GRAD_DB
    gk = _np(eng.adj_synthesis(torch.from_numpy(gy_seed()).to(dev)))
    assert snr_db(r["gk_syn_s"], gk.reshape(-1)[::STRIDE]) >= GRAD_DB


def test_trainable_gradients(dev):
    """TrainableCQT through torch autograd vs the oracle's exact transposes."""
    from flash_cqt_b200 import OctCQT, TrainableCQT
    o = oracle()
    cqt = OctCQT([3, 4, 2], [8, 16, 32], fs=44100, audio_len=65536, device=dev)
    t = TrainableCQT(cqt, dev)
    x = torch.from_numpy(x_noise()).to(dev).requires_grad_(True)
    gc = torch.from_numpy(gc_seed(o.ncoef)).to(dev)
    blocks, side = t.fwd(x)
    h = torch.cat([c.reshape(2, -1) for c in list(blocks) + list(side)], -1)
    (torch.view_as_real(h) * torch.view_as_real(gc)).sum().backward()
    want = o.adj_fwd(o.unheap(gc_seed(o.ncoef).astype(np.complex128)))
    assert snr_db(want, _np(x.grad)) >= GRAD_DB
    # synthesis gradient w.r.t. leaf blocks
    leaves = [c.detach().clone().requires_grad_(True) for c in list(blocks) + list(side)]
    gy = torch.from_numpy(gy_seed()).to(dev)
    (t.bwd(leaves[:9], leaves[9:]) * gy).sum().backward()
    gk = torch.cat([lv.grad.reshape(2, -1) for lv in leaves], -1)
    assert snr_db(o.heap(o.adj_bwd(gy_seed().astype(np.float64))), _np(gk)) >= GRAD_DB


def test_train_step_chain_gradient(dev):
    """analysis -> synthesis -> MSE -> backward vs the oracle chain rule."""
    from flash_cqt_b200 import OctCQT, TrainableCQT
    o = oracle()
    t = TrainableCQT(OctCQT([3, 4, 2], [8, 16, 32], fs=44100, audio_len=65536,
                            device=dev), dev)
    x0 = x_noise()
    tgt = gy_seed()
    x = torch.from_numpy(x0).to(dev).requires_grad_(True)
    y = t.bwd(*t.fwd(x))
    loss = (y - torch.from_numpy(tgt).to(dev)).square().mean()
    loss.backward()
    yo = o.bwd(o.fwd(x0.astype(np.float64)))
    gy = 2.0 * (yo - tgt) / yo.size
    want = o.adj_fwd(o.adj_bwd(gy))
    assert snr_db(want, _np(x.grad)) >= GRAD_DB


def test_planar_and_interleaved_agree_bitwise(dev):
    from flash_cqt_b200 import FusedOctCQT, OctCQT
    cqt = OctCQT([3, 4, 2], [8, 16, 32], fs=44100, audio_len=65536, device=dev)
    f = FusedOctCQT(cqt, dev)
    x = torch.from_numpy(x_noise()).to(dev)
    KR, KI = f.fwd(x)
    h = f.eng.analysis(x)
    assert torch.equal(KR, h.real) and torch.equal(KI, h.imag)
    XO = f.bwd(KR, KI)
    assert torch.equal(XO, f.eng.synthesis(h))
    bl = f.blocks_view(KR, KI)
    assert [tuple(b.shape[1:]) for b in bl] == [(b, M) for b, M, _ in f.gspec]


def _offset_view(shape, dtype, dev, elems):
    """a contiguous view whose data pointer sits `elems` elements past an
    allocation's (256-byte aligned) start"""
    n = int(np.prod(shape))
    return torch.empty(n + elems, dtype=dtype, device=dev)[elems:].view(*shape)


def test_unaligned_buffers_agree_bitwise(eng, dev):
    """buffers that are 8- (complex, signals) or 4-byte (planar) aligned take
    the per-element copies instead of the TMA bulk / float4 ones: same bits"""
    from flash_cqt_b200 import _native
    B = 3
    x = torch.from_numpy(np.stack([x_noise()[0]] * B)).to(dev)
    a = eng.analysis(x)
    c8 = _offset_view((B, eng.ncoef), torch.complex64, dev, 1)
    assert c8.data_ptr() % 16 == 8
    assert torch.equal(eng.analysis(x, out=c8), a)
    kr = _offset_view((B, eng.ncoef), torch.float32, dev, 1)
    ki = _offset_view((B, eng.ncoef), torch.float32, dev, 3)
    eng.analysis_planar(x, kr, ki)
    assert torch.equal(kr, a.real) and torch.equal(ki, a.imag)
    y = eng.synthesis(a)
    y8 = _offset_view((B, 65536), torch.float32, dev, 2)
    assert torch.equal(eng.synthesis(c8, out=y8), y)
    y16 = _offset_view((B, 65536), torch.float32, dev, 4)
    assert torch.equal(eng.synthesis_planar(kr, ki, y16), y)
    # a 4-byte aligned signal is refused at the C ABI
    x4 = _offset_view((B, 65536), torch.float32, dev, 1)
    x4.copy_(x)
    ws = eng.workspace(B)
    with pytest.raises(RuntimeError, match="aligned"):
        eng.tables.call("cqt_analysis", x4.data_ptr(), a.data_ptr(), None,
                        _native.CQT_LAYOUT_COMPLEX, B, ws.data_ptr(), ws.numel(),
                        int(torch.cuda.current_stream(dev).cuda_stream))
    # through the Python engine the same tensor is realigned, not refused
    assert torch.equal(eng.analysis(x4), a)


def test_deterministic(eng, dev):
    x = torch.from_numpy(x_noise()).to(dev)
    a1 = eng.analysis(x)
    a2 = eng.analysis(x)
    assert torch.equal(a1, a2)
    y1 = eng.synthesis(a1)
    y2 = eng.synthesis(a1)
    assert torch.equal(y1, y2)


def test_linearity_large_batch(eng, dev):
    """size-independent property at a large batch: A(x1 + 2 x2) = A x1 + 2 A x2"""
    g = torch.Generator(device="cpu").manual_seed(7)
    x1 = torch.randn(256, 65536, generator=g).to(dev)
    x2 = torch.randn(256, 65536, generator=g).to(dev)
    a = eng.analysis(x1 + 2 * x2)
    b = eng.analysis(x1) + 2 * eng.analysis(x2)
    assert snr_db(_np(a), _np(b)) >= 120
    y = eng.synthesis(a)
    assert snr_db(_np(x1 + 2 * x2).astype(np.float64), _np(y)) >= RT_DB


def test_graph_replay_rebuilds_outputs(eng, dev):
    from flash_cqt_b200 import Graphed
    x = torch.from_numpy(sinusoids(1)).to(dev)

    def rt(inp):
        return eng.synthesis(eng.analysis(inp))

    g = Graphed(rt, x)
    eager = rt(x)
    g._out.fill_(1e9)   # poison the static output, the replay must rebuild it
    y = g(x)
    assert torch.equal(y, eager)
    assert snr_db(_np(x).astype(np.float64), _np(y)) >= RT_DB


def test_zero_and_impulse(eng, dev):
    z = torch.zeros(2, 65536, device=dev)
    assert torch.count_nonzero(eng.analysis(z)) == 0
    imp = torch.zeros(1, 65536, device=dev)
    imp[0, 12345] = 1.0
    o = oracle()
    assert snr_db(o.heap(o.fwd(_np(imp).astype(np.float64))),
                  _np(eng.analysis(imp))) >= COEF_DB


def test_bad_inputs_raise(eng, dev):
    with pytest.raises(TypeError):
        eng.analysis(torch.zeros(1, 65536, device=dev, dtype=torch.float64))
    with pytest.raises(ValueError):
        eng.analysis(torch.zeros(1, 4096, device=dev))
    with pytest.raises(ValueError):
        eng.analysis(torch.zeros(1, 65536))
    with pytest.raises(ValueError):
        eng.synthesis(torch.zeros(1, 100, dtype=torch.complex64, device=dev))
    # outputs written in place must match the batch exactly (no short buffers)
    x2 = torch.zeros(2, 65536, device=dev)
    kr = torch.zeros(1, eng.ncoef, device=dev)
    with pytest.raises(ValueError):
        eng.analysis_planar(x2, kr, kr.clone())
    with pytest.raises(ValueError):
        eng.synthesis_planar(kr, kr.clone(), torch.zeros(1, 4096, device=dev))
    with pytest.raises(ValueError):
        eng.analysis(x2, out=torch.zeros(1, eng.ncoef, dtype=torch.complex64, device=dev))


def test_oversized_batch_refused(eng, dev):
    """batches past the exact (band, slice) split are refused before any
    buffer is touched"""
    from flash_cqt_b200 import _native
    with pytest.raises(RuntimeError, match="too many slices"):
        eng.tables.call("cqt_analysis", 0, 0, None, _native.CQT_LAYOUT_COMPLEX, 1 << 24,
                        0, 0, 0)


def test_sliced_matches_oracle(dev):
    from flash_cqt_b200 import SlicedCQT
    from fixtures import STRIDE_SLICED, chirp
    from oracle.cqt_oracle import SlicedOracle
    r = ref()
    L = 150000
    x = chirp(5, L)
    sl = SlicedCQT([3, 4, 2], [8, 16, 32], fs=44100, sl_len=65536, device=dev)
    xt = torch.from_numpy(x).to(dev).view(1, 1, L)
    blocks, side = sl.fwd(xt)
    so = SlicedOracle()
    ob, os_ = so.fwd(x[None].astype(np.float64))
    got = np.concatenate([_np(c).reshape(-1) for c in blocks])
    want = np.concatenate([c.reshape(-1) for c in ob])
    assert snr_db(want, got) >= COEF_DB
    bs = np.concatenate([_np(c).reshape(-1)[::STRIDE_SLICED] for c in blocks])
    assert snr_db(r["sliced_blocks_s"], bs) >= COEF_DB
    y = sl.bwd(blocks, side, length=L)
    assert snr_db(x.astype(np.float64), _np(y).reshape(-1)) >= RT_DB


class _PluginEngine:
    """An OctCQT-shaped engine swapped into SlicedCQT.cqt (the reference's
    plugin point, used by bench/scoreboard.py): forces the generic path."""

    def __init__(self, cqt):
        self.inner = cqt

    def fwd(self, x):
        return self.inner.fwd(x)

    def bwd(self, blocks, side=None):
        return self.inner.bwd(blocks, side)


def _flat(blocks, side):
    return torch.cat([c.reshape(-1) for c in list(blocks) + list(side)])


@pytest.mark.parametrize("shape", [(1, 1, 150000), (2, 2, 65537), (1, 3, 262144),
                                   (1, 1, 1000), (2, 1, 32768)])
def test_sliced_fused_equals_generic_path(dev, shape):
    from flash_cqt_b200 import SlicedCQT
    g = torch.Generator(device="cpu").manual_seed(sum(shape))
    x = torch.randn(*shape, generator=g).to(dev)
    fused = SlicedCQT([3, 4, 2], [8, 16, 32], fs=44100, sl_len=65536, device=dev)
    gen = SlicedCQT([3, 4, 2], [8, 16, 32], fs=44100, sl_len=65536, device=dev)
    gen.cqt = _PluginEngine(gen.cqt)
    fb, fs_ = fused.fwd(x)
    gb, gs = gen.fwd(x)
    for a, b in zip(list(fb) + list(fs_), list(gb) + list(gs)):
        assert a.shape == b.shape
    assert snr_db(_np(_flat(gb, gs)), _np(_flat(fb, fs_))) >= COEF_DB
    L = shape[-1]
    yf = fused.bwd(fb, fs_, length=L)
    yg = gen.bwd(gb, gs, length=L)
    assert snr_db(_np(yg).astype(np.float64), _np(yf)) >= RT_DB
    assert snr_db(_np(x).astype(np.float64), _np(yf)) >= RT_DB
    # blocks handed back untouched are used in place; a copy takes the packing path
    yc = fused.bwd([c.clone() for c in fb], [c.clone() for c in fs_], length=L)
    assert torch.equal(yc, yf)
    yd = fused.bwd(fb, fs_)
    assert yd.shape[-1] == fused._num_slices(L) * 2 * fused.H


def test_sliced_gradients_match_generic_autograd(dev):
    from flash_cqt_b200 import SlicedCQT
    g = torch.Generator(device="cpu").manual_seed(99)
    L = 120000
    x0 = torch.randn(1, 2, L, generator=g).to(dev)
    fused = SlicedCQT([3, 4, 2], [8, 16, 32], fs=44100, sl_len=65536, device=dev)
    gen = SlicedCQT([3, 4, 2], [8, 16, 32], fs=44100, sl_len=65536, device=dev)
    gen.cqt = _PluginEngine(gen.cqt)
    # analysis gradient
    grads = []
    for sl in (fused, gen):
        x = x0.clone().requires_grad_(True)
        b, s = sl.fwd(x)
        w = torch.randn(_flat(b, s).shape, dtype=torch.complex64,
                        generator=torch.Generator(device="cpu").manual_seed(5)).to(dev)
        (torch.view_as_real(_flat(b, s)) * torch.view_as_real(w)).sum().backward()
        grads.append(_np(x.grad))
    assert snr_db(grads[1].astype(np.float64), grads[0]) >= GRAD_DB
    # synthesis gradient w.r.t. leaf blocks, and the chain
    b0, s0 = fused.fwd(x0)
    u = torch.randn(1, 2, L, generator=torch.Generator(device="cpu").manual_seed(6)).to(dev)
    sg = []
    for sl in (fused, gen):
        leaves = [c.detach().clone().requires_grad_(True) for c in list(b0) + list(s0)]
        y = sl.bwd(leaves[:9], leaves[9:], length=L)
        (y * u).sum().backward()
        sg.append(_np(torch.cat([lv.grad.reshape(-1) for lv in leaves])))
    assert snr_db(sg[1], sg[0]) >= GRAD_DB


@pytest.mark.parametrize("fused", [True, False])
def test_sliced_stream_matches_whole_buffer(dev, fused):
    """streaming with one half slice of state == whole-buffer transform
    (the reference's own check, bench/sliced.py:112-135).  The fused path
    keeps its state on the device and is bit-identical to the whole buffer;
    the generic path (a swapped-in engine) agrees to the parity tolerances."""
    from flash_cqt_b200 import SlicedCQT
    sl = SlicedCQT([3, 4, 2], [8, 16, 32], fs=44100, sl_len=65536, device=dev)
    if not fused:
        sl.cqt = _PluginEngine(sl.cqt)
    hop = sl.hop
    n = 4
    x = torch.randn(2, 1, n * hop, generator=torch.Generator(device="cpu").manual_seed(8)).to(dev)
    wb, ws = sl.fwd(x)
    chunks = [x[..., i * hop:(i + 1) * hop] for i in range(n)]
    out = list(sl.stream_fwd(iter(chunks)))
    assert len(out) == sl._num_slices(n * hop)
    for k, (bl, sd) in enumerate(out):
        for c, blk, m in zip(bl, wb, sl.size_per_oct):
            ref = blk[..., k * m:(k + 1) * m]
            if fused:
                assert torch.equal(c, ref)
            else:
                assert snr_db(_np(ref), _np(c)) >= COEF_DB - 5 or \
                    float(ref.abs().max()) < 1e-6
        for c, whole in zip(sd, ws):
            if fused:
                assert torch.equal(c, whole[:, :, k])
    ys = torch.cat(list(sl.stream_bwd(iter(out))), dim=-1)
    yw = sl.bwd(wb, ws)
    assert ys.shape[-1] == n * hop
    if fused:
        assert torch.equal(ys, yw[..., :n * hop])
    else:
        assert snr_db(_np(yw[..., :n * hop]).astype(np.float64), _np(ys)) >= RT_DB


def test_graphed_streamer_matches_whole_buffer(dev):
    """one CUDA graph replay per chunk (SliceStream) == whole-buffer
    transform bit for bit, across two streams on one streamer"""
    from flash_cqt_b200 import SlicedCQT
    sl = SlicedCQT([3, 4, 2], [8, 16, 32], fs=44100, sl_len=65536, device=dev)
    hop, n = sl.hop, 5
    st = sl.streamer((2, 1))
    g = torch.Generator(device="cpu").manual_seed(14)
    for _ in range(2):
        x = torch.randn(2, 1, n * hop, generator=g).to(dev)
        wb, ws = sl.fwd(x)
        yw = sl.bwd(wb, ws)
        st.reset()
        outs = [st.fwd(x[..., i * hop:(i + 1) * hop]) for i in range(n)] + [st.flush()]
        for k, (bl, sd) in enumerate(outs):
            for c, blk, m in zip(bl, wb, sl.size_per_oct):
                assert torch.equal(c, blk[..., k * m:(k + 1) * m])
            for c, whole in zip(sd, ws):
                assert torch.equal(c, whole[:, :, k])
        ys = [st.bwd(bl, sd) for bl, sd in outs]
        assert ys[0] is None
        assert torch.equal(torch.cat(ys[1:], dim=-1), yw[..., :n * hop])


def test_sliced_stream_gradient(dev):
    """gradients through the device-state streaming path equal the
    whole-buffer transform's"""
    from flash_cqt_b200 import SlicedCQT
    sl = SlicedCQT([3, 4, 2], [8, 16, 32], fs=44100, sl_len=65536, device=dev)
    hop, n = sl.hop, 3
    g = torch.Generator(device="cpu").manual_seed(9)
    x = torch.randn(1, 2, n * hop, generator=g).to(dev)
    u = torch.randn(1, 2, n * hop, generator=g).to(dev)
    grads = []
    for streamed in (True, False):
        xl = x.clone().requires_grad_(True)
        if streamed:
            chunks = [xl[..., i * hop:(i + 1) * hop] for i in range(n)]
            y = torch.cat(list(sl.stream_bwd(sl.stream_fwd(iter(chunks)))), dim=-1)
        else:
            b, sd = sl.fwd(xl)
            y = sl.bwd(b, sd)[..., :n * hop]
        (y * u).sum().backward()
        grads.append(xl.grad)
    assert snr_db(_np(grads[1]).astype(np.float64), _np(grads[0])) >= GRAD_DB


@pytest.mark.parametrize("i", range(3))
def test_other_filterbanks(dev, i):
    """banks of 130, 170 and 410 bands (band lengths 32..2048): analysis and
    round trip against the oracle and the reference's fixtures, both
    transposes against the oracle"""
    from fixtures import ALT_CONFIGS, STRIDE_ALT, oracle_alt, ref_alt, x_alt
    from flash_cqt_b200.engine import Engine
    no, bpo = ALT_CONFIGS[i]
    e = Engine.from_params(no, bpo, 44100, 65536, dev)
    o, r = oracle_alt(i), ref_alt()
    x = x_alt()
    h = e.analysis(torch.from_numpy(x).float().to(dev))
    want = o.heap(o.fwd(x))
    assert snr_db(want, _np(h)) >= COEF_DB
    assert snr_db(r[f"alt{i}_coef_s"], _np(h).reshape(-1)[::STRIDE_ALT]) >= COEF_DB
    y = e.synthesis(h)
    assert snr_db(x, _np(y)) >= RT_DB
    assert snr_db(r[f"alt{i}_y_s"], _np(y).reshape(-1)[::STRIDE_ALT]) >= RT_DB
    g = np.random.default_rng(i).standard_normal((2, 2, e.ncoef))
    gc = (g[0] + 1j * g[1]).astype(np.complex64)
    gx = e.adj_analysis(torch.from_numpy(gc).to(dev))
    assert snr_db(o.adj_fwd(o.unheap(gc.astype(np.complex128))), _np(gx)) >= GRAD_DB
    gy = np.random.default_rng(10 + i).standard_normal((2, 65536))
    gk = e.adj_synthesis(torch.from_numpy(gy).float().to(dev))
    assert snr_db(o.heap(o.adj_bwd(gy)), _np(gk)) >= GRAD_DB


@pytest.mark.parametrize("bank", [([3, 4, 2], [12, 24, 48]), ([2, 2, 5], [16, 32, 48]),
                                  ([5, 4], [8, 32])])
def test_more_filterbanks_against_oracle(dev, bank):
    """banks the reference's fixtures do not cover: 16-point bands at
    65536-sample slices (230 bands), 338 bands (descriptors in device memory)
    and an 8/32 two-group bank; analysis, round trip and both transposes
    against the oracle"""
    from flash_cqt_b200.engine import Engine
    from oracle.cqt_oracle import OctCQTOracle
    e = Engine.from_params(bank[0], bank[1], 44100, 65536, dev)
    o = OctCQTOracle(bank[0], bank[1], 44100, 65536)
    x = np.random.default_rng(41).standard_normal((2, 65536))
    h = e.analysis(torch.from_numpy(x).float().to(dev))
    want = o.heap(o.fwd(x))
    assert snr_db(want, _np(h)) >= COEF_DB
    for b in range(2):
        assert snr_db(want[b], _np(h)[b]) >= COEF_DB, b
    y = e.synthesis(h)
    assert snr_db(x, _np(y)) >= RT_DB
    g = np.random.default_rng(42).standard_normal((2, 2, e.ncoef))
    gc = (g[0] + 1j * g[1]).astype(np.complex64)
    gx = e.adj_analysis(torch.from_numpy(gc).to(dev))
    assert snr_db(o.adj_fwd(o.unheap(gc.astype(np.complex128))), _np(gx)) >= GRAD_DB
    gy = np.random.default_rng(43).standard_normal((2, 65536))
    gk = e.adj_synthesis(torch.from_numpy(gy).float().to(dev))
    assert snr_db(o.heap(o.adj_bwd(gy)), _np(gk)) >= GRAD_DB




def test_host_pipeline_equals_device_round_trip(dev):
    """chunks through the overlapped host pipeline == one device round trip,
    bit for bit, with a ragged last chunk and slot reuse across calls"""
    from flash_cqt_b200 import FusedOctCQT, HostPipeline, OctCQT
    f = FusedOctCQT(OctCQT([3, 4, 2], [8, 16, 32], fs=44100, audio_len=65536, device=dev), dev)
    pipe = HostPipeline(lambda x: f.bwd(*f.fwd(x)), chunk=16, device=dev)
    g = torch.Generator(device="cpu").manual_seed(13)
    for B in (37, 50):
        xh = torch.randn(B, 65536, generator=g).pin_memory()
        yh = pipe(xh)
        want = f.bwd(*f.fwd(xh.to(dev))).cpu()
        assert torch.equal(yh, want)


def test_no_bounded_wait_expired(eng, dev):
    """every bounded wait on a TMA completion in the kernels run so far ended
    by completion, not by its poll limit"""
    from flash_cqt_b200._native import wait_timeouts
    torch.cuda.synchronize()
    assert wait_timeouts() == 0


_TRAIN_STEP = r"""
import sys, torch
sys.path.insert(0, sys.argv[2])
from flash_cqt_b200 import OctCQT, TrainableCQT, _native
dev = torch.device("cuda:0")
cqt = OctCQT([3, 4, 2], [8, 16, 32], fs=44100, audio_len=65536, device=dev)
t = TrainableCQT(cqt, dev)
g = torch.Generator(device="cpu").manual_seed(11)
x = torch.randn(3, 65536, generator=g).to(dev).requires_grad_(True)
tgt = torch.randn(3, 65536, generator=g).to(dev)
blocks, side = t.fwd(x)
y = t.bwd(blocks, side)
((y - tgt) ** 2).mean().backward()
from flash_cqt_b200 import FusedOctCQT
f = FusedOctCQT(cqt, dev)
kr, ki = f.fwd(x.detach())
kr, ki = kr.clone(), ki.clone()
yf = f.bwd(kr, ki).clone()
torch.save({"fast": _native.torch_ops() is not None, "y": y.detach().cpu(),
            "b0": blocks[0].detach().cpu(), "gx": x.grad.cpu(), "kr": kr.cpu(),
            "ki": ki.cpu(), "yf": yf.cpu()}, sys.argv[1])
"""


def test_torch_fast_path_matches_ctypes_path(tmp_path):
    """TrainableCQT and FusedOctCQT through the C++ fast path and through the
    Python autograd functions / launchers over ctypes run the same kernels:
    bit-identical outputs and gradients"""
    import os
    import subprocess
    import sys
    root = str(pathlib.Path(__file__).resolve().parents[1])
    script = tmp_path / "step.py"
    script.write_text(_TRAIN_STEP)
    out = {}
    for flag in ("1", "0"):
        f = tmp_path / f"r{flag}.pt"
        env = dict(os.environ, FLASH_CQT_B200_TORCH_OPS=flag)
        subprocess.run([sys.executable, str(script), str(f), root], check=True, env=env,
                       timeout=600)
        out[flag] = torch.load(f)
    if not out["1"]["fast"]:
        pytest.skip("torch fast path not built")
    assert not out["0"]["fast"]
    for k in ("y", "b0", "gx", "kr", "ki", "yf"):
        assert torch.equal(out["1"][k], out["0"][k]), k


def test_empty_batch(eng, dev):
    """a batch of zero slices launches nothing and returns empty results of
    the right shapes on every entry point"""
    from flash_cqt_b200 import FusedOctCQT, OctCQT, TrainableCQT
    x0 = torch.zeros(0, 65536, device=dev)
    h = eng.analysis(x0)
    assert h.shape == (0, eng.ncoef) and h.dtype == torch.complex64
    assert eng.synthesis(h).shape == (0, 65536)
    assert eng.adj_analysis(h).shape == (0, 65536)
    assert eng.adj_synthesis(x0).shape == (0, eng.ncoef)
    cqt = OctCQT([3, 4, 2], [8, 16, 32], fs=44100, audio_len=65536, device=dev)
    t = TrainableCQT(cqt, dev)
    blocks, side = t.fwd(x0)
    assert all(c.shape[0] == 0 for c in list(blocks) + list(side))
    assert t.bwd(blocks, side).shape == (0, 65536)
    f = FusedOctCQT(cqt, dev)
    kr, ki = f.fwd(x0)
    assert kr.shape == (0, eng.ncoef) and f.bwd(kr, ki).shape == (0, 65536)
