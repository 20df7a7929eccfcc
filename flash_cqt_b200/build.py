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
SOURCES = ["spectrum.cu", "bands.cu", "capi.cu"]
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


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("-D", dest="defines", action="append", default=[])
    ap.add_argument("--lib", default=None)
    a = ap.parse_args(argv)
    print(build(a.force, a.verbose, a.ptxas_info, a.defines, a.lib))


if __name__ == "__main__":
    sys.exit(main())
