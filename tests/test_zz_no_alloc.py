"""The allocation-free analysis entry point against the workspace one.

``cqt_analysis_noalloc`` exists for callers that cannot allocate device
memory -- typically a real-time audio callback, where a cudaMalloc can block
and synchronise the device and so cause dropouts.  It must give the same
coefficients as ``cqt_analysis`` (which takes a caller-allocated workspace):
same kernels, same tables, only the scratch rows live in a static device array
inside the library.  Two calls in a row check that the shared scratch, which
keeps the previous call's contents, does not leak into the next result.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test; it also passes on its own in a
fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle.cqt_oracle import snr_db

pytestmark = pytest.mark.gpu

COEF_DB = 120.0   # the coefficient tolerance of the parity tests


@pytest.fixture(scope="module")
def eng():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from flash_cqt_b200.engine import Engine
    return Engine.from_params([3, 4, 2], [8, 16, 32], 44100, 65536,
                              torch.device("cuda:0"))


def _noalloc(eng, x, out, out_im=None, layout=None):
    from flash_cqt_b200 import _native
    L = _native.lib()
    if layout is None:
        layout = _native.CQT_LAYOUT_COMPLEX
    im = ctypes.c_void_p(out_im.data_ptr()) if out_im is not None else None
    rc = L.cqt_analysis_noalloc(eng.tables.handle, ctypes.c_void_p(x.data_ptr()),
                                ctypes.c_void_p(out.data_ptr()), im, layout, x.shape[0],
                                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc, L.cqt_last_error().decode()


def test_noalloc_matches_workspace_entry_point_twice(eng):
    g = torch.Generator(device="cpu").manual_seed(2024)
    for batch in (8, 3):   # a full scratch, then a smaller call over stale rows
        x = torch.randn(batch, 65536, generator=g).to(eng.dev)
        want = eng.analysis(x)                       # cqt_analysis, workspace
        got = torch.full_like(want, float("nan"))
        rc, msg = _noalloc(eng, x, got)
        assert rc == 0, msg
        torch.cuda.synchronize()
        w, h = want.cpu().numpy(), got.cpu().numpy()
        assert np.isfinite(h).all()
        assert snr_db(w, h) >= COEF_DB
        for b in range(batch):
            assert snr_db(w[b], h[b]) >= COEF_DB, b


def test_noalloc_stale_nan_scratch_does_not_leak(eng):
    """a call on NaN input leaves NaN in every scratch row; the next call, on
    finite input and fewer slices, must still be finite and exact"""
    nan_x = torch.full((8, 65536), float("nan"), device=eng.dev)
    junk = torch.empty(8, eng.ncoef, dtype=torch.complex64, device=eng.dev)
    rc, msg = _noalloc(eng, nan_x, junk)
    assert rc == 0, msg
    g = torch.Generator(device="cpu").manual_seed(7)
    x = torch.randn(3, 65536, generator=g).to(eng.dev)
    got = torch.full((3, eng.ncoef), float("nan"), dtype=torch.complex64, device=eng.dev)
    rc, msg = _noalloc(eng, x, got)
    assert rc == 0, msg
    want = eng.analysis(x)
    torch.cuda.synchronize()
    h = got.cpu().numpy()
    assert np.isfinite(h).all()
    assert snr_db(want.cpu().numpy(), h) >= COEF_DB


def test_noalloc_planar_layout(eng):
    from flash_cqt_b200 import _native
    g = torch.Generator(device="cpu").manual_seed(11)
    x = torch.randn(5, 65536, generator=g).to(eng.dev)
    kr = torch.full((5, eng.ncoef), float("nan"), device=eng.dev)
    ki = torch.full((5, eng.ncoef), float("nan"), device=eng.dev)
    rc, msg = _noalloc(eng, x, kr, ki, _native.CQT_LAYOUT_PLANAR)
    assert rc == 0, msg
    want = eng.analysis(x)
    torch.cuda.synchronize()
    got = torch.complex(kr, ki).cpu().numpy()
    assert np.isfinite(got).all()
    assert snr_db(want.cpu().numpy(), got) >= COEF_DB


def test_noalloc_allocates_nothing_after_warmup(eng):
    """after the warm-up call (batch 0: address lookup only), a call leaves
    the device's free memory unchanged -- nothing is allocated for it"""
    x = torch.randn(8, 65536, device=eng.dev)
    out = torch.empty(8, eng.ncoef, dtype=torch.complex64, device=eng.dev)
    rc, msg = _noalloc(eng, x[:0], out[:0])
    assert rc == 0, msg
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(eng.dev)
    for _ in range(3):
        rc, msg = _noalloc(eng, x, out)
        assert rc == 0, msg
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(eng.dev)
    assert free1 == free0, (free0, free1)


def test_noalloc_rejects_batches_above_its_scratch(eng):
    x = torch.zeros(9, 65536, device=eng.dev)
    out = torch.empty(9, eng.ncoef, dtype=torch.complex64, device=eng.dev)
    rc, msg = _noalloc(eng, x, out)
    assert rc == -1
    assert "at most 8 slices" in msg


def test_noalloc_32768_sample_slices():
    """the same scratch serves the 8192-point spectrum rows of 32768-sample
    slices (shorter rows, the same static array)"""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from flash_cqt_b200.engine import Engine
    e32 = Engine.from_params([3, 4, 2], [8, 16, 32], 44100, 32768, torch.device("cuda:0"))
    g = torch.Generator(device="cpu").manual_seed(32)
    for batch in (8, 5):
        x = torch.randn(batch, 32768, generator=g).to(e32.dev)
        want = e32.analysis(x)
        got = torch.full_like(want, float("nan"))
        rc, msg = _noalloc(e32, x, got)
        assert rc == 0, msg
        torch.cuda.synchronize()
        w, h = want.cpu().numpy(), got.cpu().numpy()
        assert np.isfinite(h).all()
        for b in range(batch):
            assert snr_db(w[b], h[b]) >= COEF_DB, b
