"""CPU checks of the C ABI library: it loads, exports every function the
header declares, and rejects bad arguments before touching a GPU."""
import ctypes
import pathlib
import re

import numpy as np
import pytest
import torch

from flash_cqt_b200 import _native
from flash_cqt_b200.layout import Filterbank, HeapLayout
from flash_cqt_b200.tables import build_tables

HEADER = pathlib.Path(__file__).resolve().parents[1] / "include" / "flash_cqt_b200.h"


def declared_functions():
    txt = HEADER.read_text()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]*?\b(cqt_\w+)\s*\(",
                                 txt, flags=re.M)))


def test_library_exports_header_symbols():
    L = _native.lib()
    names = declared_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(_native.exported_symbols())
    assert L.cqt_version() == 101


def test_bad_arguments_rejected_without_gpu():
    L = _native.lib()
    h = _native.HostTables()
    out = ctypes.c_void_p()
    assert L.cqt_tables_upload(ctypes.byref(h), 0, ctypes.byref(out)) == -1
    assert b"class count" in L.cqt_last_error()
    assert L.cqt_workspace_bytes(None, 4) == 0
    assert L.cqt_analysis(None, None, None, None, 0, 1, None, 0, None) == -1


def test_out_of_range_tables_rejected():
    """the upload bounds-checks every gather and scatter index on the host"""
    tabs = build_tables(HeapLayout(Filterbank([3, 4, 2], [8, 16, 32], 44100, 65536)))
    src, gain = tabs["fwd"]["analysis"]
    bad = src.copy()
    bad[5] = 40000
    tabs["fwd"]["analysis"] = (bad, gain)
    with pytest.raises(RuntimeError, match="gather bin (out of range|outside)"):
        _native.DeviceTables(tabs, 0)


def test_engine_refuses_cpu():
    from flash_cqt_b200.engine import Engine
    with pytest.raises(RuntimeError):
        Engine.from_params([3, 4, 2], [8, 16, 32], 44100, 65536, device="cpu")
    if not torch.cuda.is_available():
        from flash_cqt_b200 import OctCQT
        cqt = OctCQT([3, 4, 2], [8, 16, 32], fs=44100, audio_len=65536)
        with pytest.raises(RuntimeError):
            cqt.fwd(torch.zeros(1, 65536))


@pytest.mark.parametrize("bank", [([3, 4, 2], [8, 16, 32]), ([4, 4, 1], [8, 16, 32]),
                                  ([2, 2, 2, 3], [8, 12, 16, 32]), ([3, 4, 2], [8, 64, 64])])
def test_valid_tables_pass_host_validation(bank):
    """Without a GPU the upload gets past every host-side check and fails only
    at the first CUDA call, so the product tables satisfy the ABI contract
    (closed-form octave geometry == per-tap tables, every index in range),
    for the default bank and for banks of 130, 170 and 410 bands."""
    if torch.cuda.is_available():
        pytest.skip("covered by the GPU tests when a device is present")
    tabs = build_tables(HeapLayout(Filterbank(bank[0], bank[1], 44100, 65536)))
    with pytest.raises(RuntimeError, match=r"cqt_tables_upload failed \(-2\)"):
        _native.DeviceTables(tabs, 0)


def test_inconsistent_geometry_rejected():
    tabs = build_tables(HeapLayout(Filterbank([3, 4, 2], [8, 16, 32], 44100, 65536)))
    g = tabs["band_geom"].copy()
    g[40, 1] += 1          # shift one octave band's window phase
    tabs["band_geom"] = g
    with pytest.raises(RuntimeError, match="disagrees with geometry"):
        _native.DeviceTables(tabs, 0)


def test_torch_fast_path_loads():
    """the host C++ torch fast path (built beside the library) imports and
    exposes its handle; it holds no device code of its own"""
    from flash_cqt_b200 import build
    if not build.torch_ops_path().exists():
        pytest.skip("torch fast path not built")
    mod = _native.torch_ops()
    assert mod is not None
    for m in ("analysis", "synthesis", "adj_analysis", "adj_synthesis", "analysis_planar",
              "synthesis_planar", "analysis_heap", "synthesis_heap", "fwd", "last_heap",
              "workspace"):
        assert hasattr(mod.Handle, m), m
    for n in ("cqt_analysis", "cqt_synthesis", "cqt_adj_analysis", "cqt_adj_synthesis",
              "cqt_workspace_bytes", "cqt_last_error"):
        assert _native.fn_address(n)


def test_torch_fast_path_raises_python_errors():
    """argument errors from the C++ fast path arrive as Python exceptions
    (ValueError here: tensors not on the handle's device), before any entry
    point is called -- the pointers handed over below are never used"""
    from flash_cqt_b200 import build
    if not build.torch_ops_path().exists():
        pytest.skip("torch fast path not built")
    mod = _native.torch_ops()

    class Owner:
        pass

    h = mod.Handle(0, 0, 10, 1, 1, 1, 1, 1, _native.fn_address("cqt_last_error"), 1, 1,
                   Owner(), [2, 2], [3, 2], 1)
    cases = ((h.analysis, torch.zeros(1, 65536)),
             (h.synthesis, torch.zeros(1, 10, dtype=torch.complex64)),
             (h.adj_analysis, torch.zeros(1, 10, dtype=torch.complex64)),
             (h.adj_synthesis, torch.zeros(2, 65536)))
    for fn, t in cases:
        with pytest.raises(ValueError, match="must be a tensor on cuda:0"):
            fn(t)
    with pytest.raises(ValueError, match="must be a tensor on cuda:0"):
        h.mse(torch.zeros(1, 10, dtype=torch.complex64), torch.zeros(1, 65536))
    p = torch.zeros(1, 10)
    with pytest.raises(ValueError, match="must be a tensor on cuda:0"):
        h.analysis_planar(torch.zeros(1, 65536), p, p)
    with pytest.raises(ValueError, match="must be float32 on cuda:0"):
        h.synthesis_planar(p, p, torch.zeros(1, 65536))
