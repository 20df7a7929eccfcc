"""ctypes binding of ``libflashcqt_b200.so`` (C ABI in include/flash_cqt_b200.h).

The shared library is built in-tree by ``flash_cqt_b200.build`` (or by
``__graft_entry__.build()``); ``FLASH_CQT_B200_LIB`` may point at another
build of the same ABI.  There is no fallback: if the library is missing
or a call fails, a ``RuntimeError`` carrying the library's own message is
raised.
"""
import ctypes
import os
import pathlib
import threading

import numpy as np

LIB_PATH = pathlib.Path(os.environ.get(
    "FLASH_CQT_B200_LIB",
    pathlib.Path(__file__).resolve().parent / "_lib" / "libflashcqt_b200.so"))

CQT_LAYOUT_PLANAR = 0
CQT_LAYOUT_COMPLEX = 1

_i32p = ctypes.POINTER(ctypes.c_int32)
_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)


class HostTables(ctypes.Structure):
    _fields_ = [
        ("nbands", ctypes.c_int32), ("ncoef", ctypes.c_int32),
        ("band_off", _i32p), ("band_list", _i32p), ("band_geom", _i32p),
        ("ngroups", ctypes.c_int32), ("group_count", _i32p), ("group_roll", _i32p),
        ("nclasses", ctypes.c_int32),
        ("class_len", _i32p), ("class_count", _i32p), ("class_first", _i32p),
        ("an_src", _i32p), ("an_gain", _f32p), ("an_seg", _i32p),
        ("as_src", _i32p), ("as_gain", _f32p), ("as_seg", _i32p),
        ("sy_dest", _i32p), ("sy_gre", _f32p), ("sy_gim", _f32p),
        ("sy_mask", _u8p), ("sy_nplanes", ctypes.c_int32),
        ("aa_dest", _i32p), ("aa_gre", _f32p), ("aa_gim", _f32p),
        ("aa_mask", _u8p), ("aa_nplanes", ctypes.c_int32),
        ("tw2048", _f32p), ("tw_hi", _f32p), ("tw_lo", _f32p),
        ("slice_len", ctypes.c_int32),
    ]


class CqtSignal(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("ld", ctypes.c_int64),
                ("sample0", ctypes.c_int64), ("count", ctypes.c_int64),
                ("length", ctypes.c_int64)]


class CqtSlices(ctypes.Structure):
    _fields_ = [("rows", ctypes.c_int32), ("slice0", ctypes.c_int32),
                ("slices", ctypes.c_int32), ("window", ctypes.c_void_p)]


_lib = None
_lock = threading.Lock()


def lib():
    """Load the shared library once; raise if it has not been built."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is not built; run `python -m "
                    "flash_cqt_b200.build` (needs nvcc) -- there is no CPU "
                    "fallback for the CUDA transform")
            L = ctypes.CDLL(str(LIB_PATH))
            vp, sz, ci = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int
            L.cqt_version.restype = ci
            L.cqt_last_error.restype = ctypes.c_char_p
            L.cqt_wait_timeouts.argtypes = [ctypes.POINTER(ctypes.c_uint)]
            L.cqt_wait_timeouts.restype = ci
            L.cqt_tables_upload.argtypes = [ctypes.POINTER(HostTables), ci,
                                            ctypes.POINTER(vp)]
            L.cqt_tables_upload.restype = ci
            L.cqt_tables_free.argtypes = [vp]
            L.cqt_tables_free.restype = ci
            L.cqt_ncoef.argtypes = [vp]
            L.cqt_ncoef.restype = ctypes.c_int32
            L.cqt_slice_len.argtypes = [vp]
            L.cqt_slice_len.restype = ctypes.c_int32
            L.cqt_workspace_bytes.argtypes = [vp, ci]
            L.cqt_workspace_bytes.restype = sz
            for name in ("cqt_analysis", "cqt_synthesis", "cqt_adj_analysis",
                         "cqt_adj_synthesis"):
                fn = getattr(L, name)
                if name in ("cqt_analysis", "cqt_adj_synthesis"):
                    fn.argtypes = [vp, vp, vp, vp, ci, ci, vp, sz, vp]
                else:
                    fn.argtypes = [vp, vp, vp, ci, vp, ci, vp, sz, vp]
                fn.restype = ci
            fl = ctypes.c_float
            L.cqt_synthesis_sqerr.argtypes = [vp, vp, vp, ci, vp, vp, vp, fl, ci, vp, sz, vp]
            L.cqt_synthesis_sqerr.restype = ci
            L.cqt_adj_synthesis_sqerr.argtypes = [vp, vp, vp, fl, vp, vp, vp, ci, ci, vp, sz, vp]
            L.cqt_adj_synthesis_sqerr.restype = ci
            i64_ = ctypes.c_int64
            L.cqt_halo_create.argtypes = [ci, ci, i64_, ci, ctypes.POINTER(vp), vp]
            L.cqt_halo_connect.argtypes = [vp, vp, vp]
            L.cqt_halo_send.argtypes = [vp, vp, i64_, i64_, vp]
            L.cqt_halo_recv_add.argtypes = [vp, vp, i64_, i64_, vp]
            L.cqt_halo_waits.argtypes = [vp, ctypes.POINTER(ctypes.c_uint), ci]
            L.cqt_halo_free.argtypes = [vp]
            for nm in ("cqt_halo_create", "cqt_halo_connect", "cqt_halo_send",
                       "cqt_halo_recv_add", "cqt_halo_waits", "cqt_halo_free"):
                getattr(L, nm).restype = ci
            L.cqt_workspace_waits.argtypes = [vp, sz, ctypes.POINTER(ctypes.c_uint), ci]
            L.cqt_workspace_waits.restype = ci
            L.cqt_debug_expire_waits.argtypes = [ci]
            L.cqt_debug_expire_waits.restype = ci
            L.cqt_launch_stage.argtypes = [vp, ci, vp, vp, vp, vp, ci, ci, vp, sz, vp]
            L.cqt_launch_stage.restype = ci
            L.cqt_analysis_noalloc.argtypes = [vp, vp, vp, vp, ci, ci, vp]
            L.cqt_analysis_noalloc.restype = ci
            i64 = ctypes.c_int64
            L.cqt_sliced_count.argtypes = [i64]
            L.cqt_sliced_count.restype = ci
            sigp, slp = ctypes.POINTER(CqtSignal), ctypes.POINTER(CqtSlices)
            L.cqt_sliced_analysis.argtypes = [vp, sigp, slp, vp, vp, sz, vp]
            L.cqt_sliced_adj_synthesis.argtypes = [vp, sigp, slp, vp, vp, sz, vp]
            L.cqt_sliced_synthesis.argtypes = [vp, vp, slp, sigp, vp, sz, vp]
            L.cqt_sliced_adj_analysis.argtypes = [vp, vp, slp, sigp, vp, sz, vp]
            for nm in ("cqt_sliced_analysis", "cqt_sliced_adj_synthesis",
                       "cqt_sliced_synthesis", "cqt_sliced_adj_analysis"):
                getattr(L, nm).restype = ci
            _lib = L
    return _lib


def exported_symbols():
    """Names the C header declares (checked by the CPU tests)."""
    return ["cqt_tables_upload", "cqt_tables_free", "cqt_ncoef", "cqt_slice_len",
            "cqt_workspace_bytes", "cqt_analysis", "cqt_synthesis",
            "cqt_adj_analysis", "cqt_adj_synthesis", "cqt_synthesis_sqerr",
            "cqt_adj_synthesis_sqerr", "cqt_launch_stage",
            "cqt_analysis_noalloc", "cqt_sliced_count", "cqt_sliced_analysis",
            "cqt_sliced_synthesis", "cqt_sliced_adj_analysis",
            "cqt_sliced_adj_synthesis", "cqt_halo_create", "cqt_halo_connect",
            "cqt_halo_send", "cqt_halo_recv_add", "cqt_halo_waits", "cqt_halo_free",
            "cqt_wait_timeouts", "cqt_workspace_waits",
            "cqt_debug_expire_waits", "cqt_last_error", "cqt_version"]


WS_HEADER = 256   # bytes at the front of a workspace: the wait-status word


def workspace_waits(ws, clear=True):
    """expired bounded waits recorded in the workspace tensor `ws` by the calls
    that used it since its header was last cleared (synchronous)"""
    n = ctypes.c_uint(0)
    _check(lib().cqt_workspace_waits(ws.data_ptr(), ws.numel() * ws.element_size(),
                                     ctypes.byref(n), 1 if clear else 0),
           "cqt_workspace_waits")
    return int(n.value)


def check_waits_enabled():
    """FLASH_CQT_B200_CHECK_WAITS=1: every engine call reads its workspace's
    wait status afterwards (synchronising) and raises if a wait ran out"""
    return os.environ.get("FLASH_CQT_B200_CHECK_WAITS", "0") not in ("", "0")


def wait_timeouts():
    """Bounded kernel waits that gave up on the current device (0 when healthy)."""
    n = ctypes.c_uint(0)
    _check(lib().cqt_wait_timeouts(ctypes.byref(n)), "cqt_wait_timeouts")
    return int(n.value)


_torchops = None
_torchops_tried = False


def torch_ops():
    """The torch fast path (``_lib/_torchops*.so``, built from
    ``csrc/torch_ops.cpp`` by ``flash_cqt_b200.build``): the whole-slice entry
    points and TrainableCQT's autograd functions in C++, calling this
    library's entry points.  None when it is not built or
    ``FLASH_CQT_B200_TORCH_OPS=0``; the ctypes path then serves every call
    (the same CUDA kernels either way)."""
    global _torchops, _torchops_tried
    if _torchops_tried:
        return _torchops
    with _lock:
        if not _torchops_tried:
            _torchops_tried = True
            if os.environ.get("FLASH_CQT_B200_TORCH_OPS", "1") != "0":
                import importlib.util
                import sysconfig
                import torch  # noqa: F401  (its libraries resolve the module's)
                path = LIB_PATH.parent / ("_torchops" + sysconfig.get_config_var("EXT_SUFFIX"))
                if path.exists():
                    spec = importlib.util.spec_from_file_location("flash_cqt_b200._torchops",
                                                                  str(path))
                    mod = importlib.util.module_from_spec(spec)
                    spec.loader.exec_module(mod)
                    _torchops = mod
    return _torchops


def fn_address(name):
    """address of an exported entry point of the library"""
    return ctypes.cast(getattr(lib(), name), ctypes.c_void_p).value


def _check(rc, what):
    if rc != 0:
        msg = lib().cqt_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed ({rc}): {msg}")


def _ptr(a, ctype):
    return a.ctypes.data_as(ctypes.POINTER(ctype))


class DeviceTables:
    """Device-resident copy of the host tables (owns the cqt_tables handle)."""

    def __init__(self, tabs, device_index):
        L = lib()
        keep = []

        def arr(a, dt, ct):
            a = np.ascontiguousarray(a, dtype=dt)
            keep.append(a)
            return _ptr(a, ct)

        cls = tabs["classes"]
        h = HostTables()
        h.nbands = len(tabs["band_off"])
        h.ncoef = len(tabs["fwd"]["analysis"][0])
        h.band_off = arr(tabs["band_off"], np.int32, ctypes.c_int32)
        h.band_list = arr(tabs["band_list"], np.int32, ctypes.c_int32)
        h.band_geom = arr(tabs["band_geom"], np.int32, ctypes.c_int32)
        h.ngroups = len(tabs["group_count"])
        h.group_count = arr(tabs["group_count"], np.int32, ctypes.c_int32)
        h.group_roll = arr(tabs["group_roll"], np.int32, ctypes.c_int32)
        h.nclasses = len(cls)
        h.class_len = arr([c[0] for c in cls], np.int32, ctypes.c_int32)
        h.class_count = arr([c[1] for c in cls], np.int32, ctypes.c_int32)
        h.class_first = arr([c[2] for c in cls], np.int32, ctypes.c_int32)
        src, gain = tabs["fwd"]["analysis"]
        h.an_src = arr(src, np.int32, ctypes.c_int32)
        h.an_gain = arr(gain, np.float32, ctypes.c_float)
        h.an_seg = arr(tabs["seg"]["analysis"], np.int32, ctypes.c_int32)
        src, gain = tabs["fwd"]["adj_synth"]
        h.as_src = arr(src, np.int32, ctypes.c_int32)
        h.as_gain = arr(gain, np.float32, ctypes.c_float)
        h.as_seg = arr(tabs["seg"]["adj_synth"], np.int32, ctypes.c_int32)
        d, gr, gi, mk, npl = tabs["inv"]["synth"]
        h.sy_dest = arr(d, np.int32, ctypes.c_int32)
        h.sy_gre = arr(gr, np.float32, ctypes.c_float)
        h.sy_gim = arr(gi, np.float32, ctypes.c_float)
        h.sy_mask = arr(mk, np.uint8, ctypes.c_uint8)
        h.sy_nplanes = npl
        d, gr, gi, mk, npl = tabs["inv"]["adj_an"]
        h.aa_dest = arr(d, np.int32, ctypes.c_int32)
        h.aa_gre = arr(gr, np.float32, ctypes.c_float)
        h.aa_gim = arr(gi, np.float32, ctypes.c_float)
        h.aa_mask = arr(mk, np.uint8, ctypes.c_uint8)
        h.aa_nplanes = npl
        h.tw2048 = arr(tabs["tw2048"], np.float32, ctypes.c_float)
        h.tw_hi = arr(tabs["tw_hi"], np.float32, ctypes.c_float)
        h.tw_lo = arr(tabs["tw_lo"], np.float32, ctypes.c_float)
        h.slice_len = int(tabs.get("slice_len", 65536))
        handle = ctypes.c_void_p()
        _check(L.cqt_tables_upload(ctypes.byref(h), int(device_index),
                                   ctypes.byref(handle)), "cqt_tables_upload")
        self.handle = handle
        self.device_index = int(device_index)
        self.ncoef = int(L.cqt_ncoef(handle))
        self.slice_len = int(L.cqt_slice_len(handle))

    def workspace_bytes(self, batch):
        return int(lib().cqt_workspace_bytes(self.handle, int(batch)))

    _SIG_FIRST = ("cqt_analysis", "cqt_adj_synthesis")

    def call(self, name, a, b, c, layout, batch, ws, ws_bytes, stream):
        fns = self.__dict__.get("_fns")
        if fns is None:   # bound once: no library lock on the per-call path
            L = lib()
            fns = self._fns = {n: getattr(L, n) for n in
                               ("cqt_analysis", "cqt_synthesis", "cqt_adj_analysis",
                                "cqt_adj_synthesis")}
        fn = fns[name]
        if name in self._SIG_FIRST:
            rc = fn(self.handle, a, b, c, layout, int(batch), ws, ws_bytes, stream)
        else:
            rc = fn(self.handle, a, b, layout, c, int(batch), ws, ws_bytes, stream)
        if rc != 0:
            _check(rc, name)

    def stage(self, stage, sig_in, sig_out, c_re, c_im, layout, batch, ws,
              ws_bytes, stream):
        _check(lib().cqt_launch_stage(self.handle, int(stage), sig_in, sig_out,
                                      c_re, c_im, layout, int(batch), ws,
                                      ws_bytes, stream), "cqt_launch_stage")

    def sliced(self, name, *args):
        fns = self.__dict__.get("_sfns")
        if fns is None:   # bound once: no library lock on the per-call path
            L = lib()
            fns = self._sfns = {n: getattr(L, n) for n in
                                ("cqt_sliced_analysis", "cqt_sliced_synthesis",
                                 "cqt_sliced_adj_analysis", "cqt_sliced_adj_synthesis")}
        rc = fns[name](self.handle, *args)
        if rc != 0:
            _check(rc, name)

    def __del__(self):
        h = getattr(self, "handle", None)
        if h is not None and _lib is not None:
            try:
                _lib.cqt_tables_free(h)
            except Exception:
                pass
            self.handle = None
