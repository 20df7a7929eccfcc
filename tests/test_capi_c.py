"""The C ABI used from plain C (tests/capi_roundtrip.c): host tables exported
with ``save_host_tables``, one analysis -> synthesis round trip on the GPU,
reconstruction >= 125 dB.  The build half runs without a GPU."""
import os
import pathlib
import shutil
import subprocess

import pytest
import torch

from flash_cqt_b200 import _native
from flash_cqt_b200.layout import Filterbank, HeapLayout
from flash_cqt_b200.tables import save_host_tables, build_tables

ROOT = pathlib.Path(__file__).resolve().parents[1]
CUDA = pathlib.Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def _build(tmp_path):
    if shutil.which("gcc") is None or not (CUDA / "include" / "cuda_runtime_api.h").exists():
        pytest.skip("gcc or the CUDA headers are missing")
    exe = tmp_path / "capi_roundtrip"
    libdir = _native.LIB_PATH.parent
    subprocess.run(["gcc", "-O2", "-std=c11", str(ROOT / "tests" / "capi_roundtrip.c"),
                    "-I", str(ROOT / "include"), "-I", str(CUDA / "include"),
                    "-L", str(libdir), "-lflashcqt_b200", "-L", str(CUDA / "lib64"),
                    "-lcudart", "-lm", f"-Wl,-rpath,{libdir}",
                    f"-Wl,-rpath,{CUDA / 'lib64'}", "-o", str(exe)], check=True)
    tabs = tmp_path / "tables.bin"
    save_host_tables(build_tables(HeapLayout(Filterbank([3, 4, 2], [8, 16, 32], 44100, 65536))),
                     tabs)
    return exe, tabs


def test_c_program_builds(tmp_path):
    _build(tmp_path)


@pytest.mark.gpu
def test_c_program_round_trip(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    exe, tabs = _build(tmp_path)
    out = subprocess.run([str(exe), str(tabs), "3"], capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr
    snr = float(out.stdout.split()[1])
    assert snr >= 125.0, out.stdout
