"""Build the reference's own code for the checker and bench.py's reference
arms -- TEST / BENCH INFRASTRUCTURE, never part of the product path.

    python oracle/build_ref.py [--ref DIR]      (default: the checkout named by
                                                  FLASH_CQT_REFERENCE, else the
                                                  ``reference_path`` of BASELINE.json)

Everything is built from the sources where they lie in the read-only reference
checkout; every output goes under ``oracle/_ref/`` (git-ignored, so it stays
out of history, and not excluded from the snapshot that runs on the GPU box,
so it travels there like the product's own built libraries).  No reference source file is copied:

* ``flash_cqt/*.py`` (the pure-torch ``OctCQT`` / ``FusedOctCQT`` /
  ``TrainableCQT`` package, ``oct_cqt.py:18-117``, ``trainable.py:28-191``)
  is byte-compiled, and the code objects are marshalled into one bundle,
  ``oracle/_ref/flash_cqt.bundle`` (a dict module name -> code, what a
  ``.pyc`` holds after its header; one file because the GPU box snapshot does
  not carry ``.pyc`` files), which ``oracle/ref_loader.py`` imports unchanged;
* ``flash_cqt/csrc/{packedfft,radix,persist2}.cu`` (the factored path's CUDA
  extensions, ``fused.py:63-132``) are compiled by
  ``torch.utils.cpp_extension`` for sm_100a into
  ``oracle/_ref/ext/<name>/<name>.so``.

``oracle/ref_loader.py`` imports the result.  When the reference checkout is
absent (the GPU box) there is nothing to build and the existing outputs are
used.
"""
import argparse
import os
import pathlib
import marshal
import shutil
import sys

HERE = pathlib.Path(__file__).resolve().parent
OUT = HERE / "_ref"


def _default_ref():
    """the reference checkout: FLASH_CQT_REFERENCE, else the ``reference_path``
    recorded in the repository's BASELINE.json (None when neither names one)"""
    env = os.environ.get("FLASH_CQT_REFERENCE")
    if env:
        return env
    try:
        import json
        return json.loads((HERE.parent / "BASELINE.json").read_text()).get("reference_path")
    except (OSError, ValueError):
        return None


DEFAULT_REF = _default_ref()
PY_MODULES = ["__init__", "ref_util", "filterbank", "oct_cqt", "sliced", "graphed",
              "fused", "trainable"]
# name the reference's loaders give each extension (fused.py:63-132)
EXTENSIONS = {"packedfft": "flash_cqt_packedfft", "radix": "flash_cqt_radix",
              "persist2": "flash_cqt_persist2"}
ARCH = ["-gencode=arch=compute_100a,code=sm_100a"]


BUNDLE = OUT / "flash_cqt.bundle"


def build_python(ref):
    src = pathlib.Path(ref) / "flash_cqt"
    OUT.mkdir(parents=True, exist_ok=True)
    codes = {}
    for m in PY_MODULES:
        text = (src / f"{m}.py").read_text()
        name = "flash_cqt" if m == "__init__" else f"flash_cqt.{m}"
        codes[name] = marshal.dumps(compile(text, f"flash_cqt/{m}.py", "exec", dont_inherit=True))
    BUNDLE.write_bytes(marshal.dumps({"python": sys.version_info[:2], "modules": codes}))
    return BUNDLE


def build_extensions(ref, verbose=False, force=False):
    """compile the extensions that are missing (all with force); about ten
    minutes for the three from scratch"""
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    from torch.utils import cpp_extension as ce
    built = {}
    for stem, name in EXTENSIONS.items():
        bdir = OUT / "ext" / name
        so = bdir / f"{name}.so"
        if force or not so.exists():
            bdir.mkdir(parents=True, exist_ok=True)
            src = pathlib.Path(ref) / "flash_cqt" / "csrc" / f"{stem}.cu"
            ce.load(name=name, sources=[str(src)], build_directory=str(bdir),
                    extra_cuda_cflags=ARCH + ["-O3"], verbose=verbose)
        built[name] = so
    return built


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=DEFAULT_REF)
    ap.add_argument("--no-cuda", action="store_true", help="byte-compile the package only")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true", help="rebuild the CUDA extensions")
    a = ap.parse_args(argv)
    ref = pathlib.Path(a.ref) if a.ref else None
    if ref is None or not (ref / "flash_cqt" / "oct_cqt.py").exists():
        print(f"no reference checkout at {ref}; nothing to build", file=sys.stderr)
        return 0
    print(build_python(ref))
    if not a.no_cuda:
        for name, so in build_extensions(ref, a.verbose, a.force).items():
            print(name, so, so.exists())
    return 0


def clean():
    if OUT.exists():
        shutil.rmtree(OUT)


if __name__ == "__main__":
    sys.exit(main())
