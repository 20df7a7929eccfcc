"""Import the reference's own code built by ``oracle/build_ref.py`` -- TEST /
BENCH INFRASTRUCTURE, never part of the product path.

``package()`` imports the byte-compiled reference package (the code bundle
``oracle/_ref/flash_cqt.bundle``) unmodified, through a meta-path finder
that serves ``flash_cqt`` and its submodules from it; ``package(cuda=True)`` also loads the
reference's CUDA extensions built for sm_100a and hands them to the
package's own extension caches (``fused.py:63-132`` keep each loaded module
in a module global and build it only while that global is None), so its
``TrainableCQT`` and resident pair run the reference kernels without a
compiler or the reference sources on the machine.
"""
import importlib
import importlib.abc
import importlib.util
import marshal
import pathlib
import sys

REF = pathlib.Path(__file__).resolve().parent / "_ref"
BUNDLE = REF / "flash_cqt.bundle"


class _BundleImporter(importlib.abc.MetaPathFinder, importlib.abc.Loader):
    """imports ``flash_cqt`` and ``flash_cqt.*`` from the marshalled code objects"""

    def __init__(self, codes):
        self.codes = codes

    def find_spec(self, fullname, path=None, target=None):
        if fullname not in self.codes:
            return None
        return importlib.util.spec_from_loader(fullname, self, origin=str(BUNDLE),
                                               is_package=fullname == "flash_cqt")

    def create_module(self, spec):
        return None

    def exec_module(self, module):
        stem = "__init__" if module.__name__ == "flash_cqt" else module.__name__.split(".")[-1]
        module.__file__ = str(REF / "flash_cqt" / f"{stem}.py")   # never read
        exec(marshal.loads(self.codes[module.__name__]), module.__dict__)
EXT_CACHES = (("_FEXT", "flash_cqt_packedfft"), ("_XEXT", "flash_cqt_radix"),
              ("_P2EXT", "flash_cqt_persist2"))


def available(cuda=False):
    ok = BUNDLE.exists()
    if cuda:
        ok = ok and all((REF / "ext" / n / f"{n}.so").exists() for _, n in EXT_CACHES)
    return ok


def package(cuda=False):
    if not available(cuda):
        raise RuntimeError("the reference is not built here (python oracle/build_ref.py)")
    if not any(isinstance(f, _BundleImporter) for f in sys.meta_path):
        b = marshal.loads(BUNDLE.read_bytes())
        if tuple(b["python"]) != tuple(sys.version_info[:2]):
            raise RuntimeError(f"reference bundle built for Python {b['python']}")
        sys.meta_path.insert(0, _BundleImporter(b["modules"]))
    # the reference imports Triton only if it can (fused.py:149-154) and its
    # factored CUDA path does not use it; Triton's @jit needs source text,
    # which compiled code does not carry, so Triton is hidden while the
    # reference modules load (a None entry in sys.modules makes the import fail)
    saved = {k: sys.modules[k] for k in list(sys.modules)
             if k == "triton" or k.startswith("triton.")}
    sys.modules["triton"] = None
    sys.modules["triton.language"] = None
    try:
        pkg = importlib.import_module("flash_cqt")
        importlib.import_module("flash_cqt.fused")
        importlib.import_module("flash_cqt.trainable")
    finally:
        for k in ("triton", "triton.language"):
            sys.modules.pop(k, None)
        sys.modules.update(saved)
    if cuda:
        import torch  # noqa: F401  (the extensions link against its libraries)
        fused = importlib.import_module("flash_cqt.fused")
        for var, name in EXT_CACHES:
            if getattr(fused, var) in (None, False):
                so = REF / "ext" / name / f"{name}.so"
                spec = importlib.util.spec_from_file_location(name, str(so))
                mod = importlib.util.module_from_spec(spec)
                spec.loader.exec_module(mod)
                setattr(fused, var, mod)
    return pkg
