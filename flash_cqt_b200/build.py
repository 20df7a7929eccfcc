"""Build the sm_100a shared library ``_lib/libflashcqt_b200.so`` in-tree.

    python -m flash_cqt_b200.build [--force] [--verbose]

nvcc compiles each ``csrc/*.cu`` for ``-gencode arch=compute_100a,code=sm_100a``
(B200 only, no PTX fallback for other GPUs) and links one shared object with
the CUDA runtime linked statically, so the library depends on nothing but the
driver.  Rebuilds only what changed.
"""
import argparse
import os
import pathlib
import shutil
import subprocess
import sys

PKG = pathlib.Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "_lib" / "libflashcqt_b200.so"
INCLUDE = PKG.parent / "include"
SOURCES = ["spectrum.cu", "bands.cu", "halo.cu", "capi.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-O3", "-I", str(INCLUDE)]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"),
                 "/usr/local/cuda/bin/nvcc"):
        if cand and pathlib.Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build")


def _deps():
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
                  + list(INCLUDE.glob("*.h")))


def build(force=False, verbose=False, ptxas_info=False, defines=(), lib=None,
          build_dir=None):
    """Compile and link; `defines` (e.g. ["FCQT_BAND_P=16"]) and an alternative
    `lib` / `build_dir` produce variant builds of the same ABI."""
    global BUILD, LIB
    if lib is not None:
        LIB = pathlib.Path(lib)
        BUILD = pathlib.Path(build_dir) if build_dir else LIB.parent / "_build"
    BUILD.mkdir(parents=True, exist_ok=True)
    LIB.parent.mkdir(parents=True, exist_ok=True)
    cc = nvcc()
    hdr_time = max(p.stat().st_mtime for p in _deps())
    objs = []
    for src in SOURCES:
        s = CSRC / src
        o = BUILD / (src + ".o")
        objs.append(o)
        if (not force and o.exists()
                and o.stat().st_mtime >= max(s.stat().st_mtime, hdr_time)):
            continue
        cmd = [cc, *ARCH, *FLAGS, *["-D" + d for d in defines], "-c", str(s), "-o", str(o)]
        if ptxas_info:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    if force or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [cc, *ARCH, "-shared", "-o", str(LIB), *map(str, objs),
               "-Xcompiler", "-fPIC", "-cudart", "static"]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    return LIB


TORCH_OPS_SRC = CSRC / "torch_ops.cpp"


def torch_ops_path():
    import sysconfig
    return PKG / "_lib" / ("_torchops" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_torch_ops(force=False, verbose=False):
    """Compile the torch fast path (``csrc/torch_ops.cpp``, host C++ only)
    against the installed torch; it calls the CUDA library through function
    pointers, so it links nothing of ours."""
    import sysconfig
    import torch
    from torch.utils import cpp_extension as ce
    out = torch_ops_path()
    out.parent.mkdir(parents=True, exist_ok=True)
    if not force and out.exists() and out.stat().st_mtime >= TORCH_OPS_SRC.stat().st_mtime:
        return out
    inc = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"]]
    libdirs = ce.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    # the system g++ (not $CXX): exceptions thrown here unwind through torch's
    # libraries and must share their C++ runtime
    cxx = shutil.which("g++", path="/usr/bin:/bin") or "g++"
    cmd = [cxx, "-O3", "-std=c++17", "-fPIC", "-shared",
           "-DTORCH_EXTENSION_NAME=_torchops", "-DTORCH_API_INCLUDE_EXTENSION_H",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}",   # default visibility: c10 exception types must match
           *[f"-I{d}" for d in inc], str(TORCH_OPS_SRC), "-o", str(out),
           *[f"-L{d}" for d in libdirs], *[f"-Wl,-rpath,{d}" for d in libdirs[:1]],
           "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_python"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("-D", dest="defines", action="append", default=[])
    ap.add_argument("--lib", default=None)
    ap.add_argument("--no-torch-ops", action="store_true",
                    help="skip the torch fast path (host C++)")
    a = ap.parse_args(argv)
    print(build(a.force, a.verbose, a.ptxas_info, a.defines, a.lib))
    if not a.no_torch_ops and a.lib is None:
        print(build_torch_ops(a.force, a.verbose))


if __name__ == "__main__":
    sys.exit(main())
