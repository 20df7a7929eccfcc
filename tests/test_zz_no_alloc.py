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


def _noalloc(eng, x, out):
    from flash_cqt_b200 import _native
    L = _native.lib()
    rc = L.cqt_analysis_noalloc(eng.tables.handle, ctypes.c_void_p(x.data_ptr()),
                                ctypes.c_void_p(out.data_ptr()), None,
                                _native.CQT_LAYOUT_COMPLEX, x.shape[0],
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


def test_noalloc_rejects_batches_above_its_scratch(eng):
    x = torch.zeros(9, 65536, device=eng.dev)
    out = torch.empty(9, eng.ncoef, dtype=torch.complex64, device=eng.dev)
    rc, msg = _noalloc(eng, x, out)
    assert rc == -1
    assert "at most 8 slices" in msg
