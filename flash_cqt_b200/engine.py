"""Torch-facing wrapper of the CUDA engines for one filterbank on one device.

PyTorch only provides device memory and the current stream here; every
transform runs in the sm_100a kernels of ``libflashcqt_b200.so``.
"""
import ctypes

import torch

from . import _native
from .layout import Filterbank, HeapLayout
from .tables import build_tables


def _cuda_device(device):
    dev = torch.device(device) if device is not None else torch.device("cuda")
    if dev.type != "cuda":
        raise RuntimeError(f"the CQT engines run on CUDA devices only, got {dev}")
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is not available: the B200 CQT engines need a GPU "
                           "(there is no CPU fallback)")
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    return dev


class Engine:
    """Device tables + workspace; analysis, synthesis and both transposes.

    Coefficients are complex64 [B, ncoef] (interleaved) or a pair of float32
    [B, ncoef] planes.  Calls on one Engine must be ordered on one stream at a
    time: the workspace is shared (the reference reuses its scratch the same
    way, trainable.py:65-73)."""

    def __init__(self, heap, device=None):
        self.dev = _cuda_device(device)
        self.heap = heap
        self.ncoef = heap.ncoef
        self.N = heap.bank.nn   # samples per slice (65536 or 32768)
        self.host_tables = build_tables(heap)
        self.tables = _native.DeviceTables(self.host_tables, self.dev.index)
        assert self.tables.ncoef == self.ncoef
        self._ws = None
        self._ws_retired = []   # outgrown workspaces, kept alive (see workspace())
        self._ws_need = {}      # batch -> bytes
        # the C++ fast path over the same entry points (None: ctypes only);
        # it owns the workspace and keeps the tables alive
        self._ops = None
        mod = _native.torch_ops()
        if mod is not None:
            ngo = len(heap.groups)
            self._ops = mod.Handle(
                self.tables.handle.value, self.dev.index, self.ncoef,
                *[_native.fn_address(n) for n in (
                    "cqt_analysis", "cqt_synthesis", "cqt_adj_analysis",
                    "cqt_adj_synthesis", "cqt_workspace_bytes", "cqt_last_error",
                    "cqt_synthesis_sqerr", "cqt_adj_synthesis_sqerr")],
                self.tables, [b for b, _, _ in heap.gspec], [M for _, M, _ in heap.gspec],
                ngo)
            self._ops.set_slice_len(self.N)

    @classmethod
    def from_params(cls, num_octs, bins_per_oct, fs, audio_len, device=None):
        return cls(HeapLayout(Filterbank(num_octs, bins_per_oct, fs, audio_len)),
                   device)

    # ---------------------------------------------------------------- plumbing
    def workspace(self, batch):
        """grow-only scratch shared by the calls on this engine.  An outgrown
        buffer is retired, not freed: a CUDA graph captured earlier may still
        address it (Graphed, HostPipeline, the streaming graphs)."""
        if self._ops is not None:
            return self._ops.workspace(batch)
        need = self._ws_need.get(batch)
        if need is None:
            need = self._ws_need[batch] = self.tables.workspace_bytes(batch)
        if self._ws is None or self._ws.numel() < need:
            if self._ws is not None:
                self._ws_retired.append(self._ws)
            self._ws = torch.empty(max(need, _native.WS_HEADER), dtype=torch.uint8,
                                   device=self.dev)
            self._ws[:_native.WS_HEADER].zero_()   # the wait-status header
        return self._ws

    def wait_status(self, clear=True):
        """bounded kernel waits that gave up in the calls on this engine's
        workspace since the last check (synchronous; 0 when healthy)"""
        ws = self.workspace(0)
        return _native.workspace_waits(ws, clear)

    def _check_waits(self, what):
        n = self.wait_status()
        if n:
            raise RuntimeError(f"{what}: {n} bounded wait(s) in the kernels gave up; "
                               "the results of this call are not trustworthy")

    def _stream(self):
        return ctypes_stream(torch.cuda.current_stream(self.dev))

    def _signal(self, t, name):
        if not torch.is_tensor(t) or t.device != self.dev:
            raise ValueError(f"{name} must be a tensor on {self.dev}")
        if t.dtype != torch.float32:
            raise TypeError(f"{name} must be float32, got {t.dtype}")
        if t.dim() != 2 or t.shape[-1] != self.N:
            raise ValueError(f"{name} must be [B, {self.N}], got {tuple(t.shape)}")
        t = t.contiguous()
        # the engines move signals as float2 / float4 vectors
        return t if t.data_ptr() % 16 == 0 else t.clone()

    def _coef(self, c, name):
        if not torch.is_tensor(c) or c.device != self.dev:
            raise ValueError(f"{name} must be a tensor on {self.dev}")
        if c.dtype != torch.complex64:
            raise TypeError(f"{name} must be complex64, got {c.dtype}")
        if c.dim() != 2 or c.shape[-1] != self.ncoef:
            raise ValueError(f"{name} must be [B, {self.ncoef}], got {tuple(c.shape)}")
        return c.resolve_conj().contiguous()

    def _out(self, t, shape, dtype, name):
        """a caller-supplied output: written in place, so it must match exactly"""
        if (not torch.is_tensor(t) or t.device != self.dev or t.dtype != dtype
                or tuple(t.shape) != tuple(shape) or not t.is_contiguous()):
            raise ValueError(f"{name} must be a contiguous {dtype} tensor of shape "
                             f"{tuple(shape)} on {self.dev}")
        return t

    def _planes(self, re, im):
        for t, nm in ((re, "re"), (im, "im")):
            if not torch.is_tensor(t) or t.device != self.dev or t.dtype != torch.float32:
                raise ValueError(f"coefficient plane {nm} must be float32 on {self.dev}")
            if t.dim() != 2 or t.shape[-1] != self.ncoef:
                raise ValueError(f"coefficient plane {nm} must be [B, {self.ncoef}]")
        if re.shape != im.shape:
            raise ValueError("coefficient planes differ in shape")
        return re.contiguous(), im.contiguous()

    def _run(self, name, a, b, c, layout, batch):
        if torch.cuda.current_device() != self.dev.index:
            with torch.cuda.device(self.dev):
                return self._run(name, a, b, c, layout, batch)
        ws = self.workspace(batch)
        self.tables.call(name, a, b, c, layout, batch, ws.data_ptr(), ws.numel(),
                         _raw_stream_of(self.dev.index))
        if _native.check_waits_enabled():
            self._check_waits(name)

    # ----------------------------------------------------------------- complex
    def analysis(self, x, out=None):
        """x [B, N] float32 (N samples per slice) -> coefficient heap complex64 [B, ncoef]."""
        if out is None and self._ops is not None:
            return self._ops.analysis(x)
        x = self._signal(x, "x")
        B = x.shape[0]
        if out is None:
            out = torch.empty(B, self.ncoef, dtype=torch.complex64, device=self.dev)
        self._out(out, (B, self.ncoef), torch.complex64, "out")
        self._run("cqt_analysis", x.data_ptr(), out.data_ptr(), None,
                  _native.CQT_LAYOUT_COMPLEX, B)
        return out

    def synthesis(self, c, out=None):
        """coefficient heap complex64 [B, ncoef] -> y [B, N] float32."""
        if out is None and self._ops is not None:
            return self._ops.synthesis(c)
        c = self._coef(c, "coefficients")
        B = c.shape[0]
        if out is None:
            out = torch.empty(B, self.N, dtype=torch.float32, device=self.dev)
        self._out(out, (B, self.N), torch.float32, "out")
        self._run("cqt_synthesis", c.data_ptr(), None, out.data_ptr(),
                  _native.CQT_LAYOUT_COMPLEX, B)
        return out

    def adj_analysis(self, g, out=None):
        """transpose of analysis: complex64 grads [B, ncoef] -> [B, N]."""
        if out is None and self._ops is not None:
            return self._ops.adj_analysis(g)
        g = self._coef(g, "coefficient gradient")
        B = g.shape[0]
        if out is None:
            out = torch.empty(B, self.N, dtype=torch.float32, device=self.dev)
        self._out(out, (B, self.N), torch.float32, "out")
        self._run("cqt_adj_analysis", g.data_ptr(), None, out.data_ptr(),
                  _native.CQT_LAYOUT_COMPLEX, B)
        return out

    def adj_synthesis(self, gy, out=None):
        """transpose of synthesis: [B, N] -> complex64 grads [B, ncoef]."""
        if out is None and self._ops is not None:
            return self._ops.adj_synthesis(gy)
        gy = self._signal(gy, "signal gradient")
        B = gy.shape[0]
        if out is None:
            out = torch.empty(B, self.ncoef, dtype=torch.complex64, device=self.dev)
        self._out(out, (B, self.ncoef), torch.complex64, "out")
        self._run("cqt_adj_synthesis", gy.data_ptr(), out.data_ptr(), None,
                  _native.CQT_LAYOUT_COMPLEX, B)
        return out

    # -------------------------------------------------------- squared error
    def synthesis_sqerr(self, c, target):
        """coefficient heap [B, ncoef] and target [B, N] -> (loss, y):
        y = synthesis(c), loss = mean((y - target)^2) as a 0-dim float32
        tensor, summed in a fixed order inside the engines."""
        c = self._coef(c, "coefficients")
        B = c.shape[0]
        target = self._signal(target, "target")
        if target.shape[0] != B:
            raise ValueError(f"target must be [{B}, {self.N}], got {tuple(target.shape)}")
        y = torch.empty(B, self.N, dtype=torch.float32, device=self.dev)
        loss = torch.empty((), dtype=torch.float32, device=self.dev)
        self._run_sqerr(c.data_ptr(), y.data_ptr(), target.data_ptr(), loss.data_ptr(),
                        1.0 / (B * self.N) if B else 0.0, B)
        return loss, y, target

    def adj_synthesis_sqerr(self, y, target, scale, g):
        """transpose of the synthesis applied to scale * g * (y - target), y and
        target [B, N] float32, g a device float32 scalar tensor (e.g. dL/dloss)"""
        y = self._signal(y, "y")
        target = self._signal(target, "target")
        B = y.shape[0]
        if target.shape[0] != B:
            raise ValueError(f"target must be [{B}, {self.N}], got {tuple(target.shape)}")
        if (not torch.is_tensor(g) or g.device != self.dev or g.dtype != torch.float32
                or g.numel() != 1):
            raise ValueError(f"g must be a float32 scalar tensor on {self.dev}")
        g = g.contiguous()
        if torch.cuda.current_device() != self.dev.index:
            with torch.cuda.device(self.dev):
                return self.adj_synthesis_sqerr(y, target, scale, g)
        out = torch.empty(B, self.ncoef, dtype=torch.complex64, device=self.dev)
        ws = self.workspace(B)
        rc = _native.lib().cqt_adj_synthesis_sqerr(
            self.tables.handle, y.data_ptr(), target.data_ptr(), float(scale), g.data_ptr(),
            out.data_ptr(), None, _native.CQT_LAYOUT_COMPLEX, B, ws.data_ptr(), ws.numel(),
            _raw_stream_of(self.dev.index))
        _native._check(rc, "cqt_adj_synthesis_sqerr")
        if _native.check_waits_enabled():
            self._check_waits("cqt_adj_synthesis_sqerr")
        return out

    def _run_sqerr(self, c, y, target, loss, scale, B):
        if torch.cuda.current_device() != self.dev.index:
            with torch.cuda.device(self.dev):
                return self._run_sqerr(c, y, target, loss, scale, B)
        ws = self.workspace(B)
        rc = _native.lib().cqt_synthesis_sqerr(
            self.tables.handle, c, None, _native.CQT_LAYOUT_COMPLEX, y, target, loss,
            float(scale), B, ws.data_ptr(), ws.numel(), _raw_stream_of(self.dev.index))
        _native._check(rc, "cqt_synthesis_sqerr")
        if _native.check_waits_enabled():
            self._check_waits("cqt_synthesis_sqerr")

    # ------------------------------------------------------------------ planar
    def analysis_planar(self, x, kr, ki):
        """x [B, N] -> the planes kr, ki [B, ncoef] (written in place)"""
        if self._ops is not None:
            self._ops.analysis_planar(x, kr, ki)
            return kr, ki
        x = self._signal(x, "x")
        B = x.shape[0]
        self._out(kr, (B, self.ncoef), torch.float32, "coefficient plane re")
        self._out(ki, (B, self.ncoef), torch.float32, "coefficient plane im")
        self._run("cqt_analysis", x.data_ptr(), kr.data_ptr(), ki.data_ptr(),
                  _native.CQT_LAYOUT_PLANAR, B)
        return kr, ki

    def synthesis_planar(self, kr, ki, y):
        """planes kr, ki [B, ncoef] -> y [B, N] (written in place)"""
        if self._ops is not None:
            self._ops.synthesis_planar(kr, ki, y)
            return y
        kr, ki = self._planes(kr, ki)
        self._out(y, (kr.shape[0], self.N), torch.float32, "y")
        self._run("cqt_synthesis", kr.data_ptr(), ki.data_ptr(), y.data_ptr(),
                  _native.CQT_LAYOUT_PLANAR, kr.shape[0])
        return y


def ctypes_stream(stream):
    return int(stream.cuda_stream)


def _raw_stream_of(index):
    """cudaStream_t of the current stream on device `index` (the fast torch
    accessor where present)"""
    return torch.cuda.current_stream(index).cuda_stream


_raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
if _raw is not None:
    _raw_stream_of = _raw   # noqa: F811 -- same result, without a Stream object


class SlicedEngine:
    """The sliced streaming transform on one Engine (cqt_sliced_* entry points).

    Signals are float32 [rows, length] (any row stride with unit element
    stride); coefficients live in one complex64 buffer of rows * S * ncoef
    values, group after group: octave groups as [rows, b, S*M], side groups as
    [rows, S, M] (the layout of ``SlicedCQT.fwd``'s blocks).  ``ws`` overrides
    the engine's shared workspace with a caller-owned uint8 device buffer of
    at least ``eng.tables.workspace_bytes(rows * S)`` bytes."""

    def __init__(self, eng, window):
        from . import _native
        self.eng = eng
        self._nat = _native
        if window.numel() != eng.N:
            raise ValueError(f"the slice window must have {eng.N} samples")
        self.window = window.to(device=eng.dev, dtype=torch.float32).contiguous()
        self.gspec = eng.heap.gspec

    def count(self, length):
        """slices of a stream of `length` samples (sliced.py:102-104)"""
        if length <= 0:
            return 1
        H = self.eng.N // 4
        return (-(-int(length) // H) + 1) // 2 + 1

    def coef_numel(self, rows, S):
        return rows * S * self.eng.ncoef

    def group_views(self, buf, lead, S):
        """split the coefficient buffer into per-group views with leading dims
        `lead` (rows = prod(lead)): octave [*lead, b, S*M], side [*lead, S, 1, M]"""
        rows = 1
        for d in lead:
            rows *= d
        ngo = len(self.eng.heap.groups)
        sizes = [rows * S * b * M for b, M, _ in self.gspec]
        out = [v.view(*lead, b, S * M) if gi < ngo else v.view(*lead, S, 1, M)
               for gi, (v, (b, M, _)) in enumerate(zip(buf.split(sizes), self.gspec))]
        return out[:ngo], out[ngo:]

    def _sig(self, x, name):
        if x.device != self.eng.dev or x.dtype != torch.float32 or x.dim() != 2:
            raise ValueError(f"{name} must be float32 [rows, samples] on {self.eng.dev}")
        if x.stride(-1) != 1:
            x = x.contiguous()
        return x

    def _call(self, name, *args):
        if torch.cuda.current_device() != self.eng.dev.index:
            with torch.cuda.device(self.eng.dev):
                return self.eng.tables.sliced(name, *args)
        self.eng.tables.sliced(name, *args)

    def _slices(self, rows, slice0, S, window):
        return self._nat.CqtSlices(rows, slice0, S, window.data_ptr() if window is not None else None)

    def _signal(self, t, sample0, length):
        return self._nat.CqtSignal(t.data_ptr(), t.stride(0), int(sample0), t.shape[1],
                                int(length))

    def analysis(self, x, S=None, out=None, adjoint_of_synthesis=False, slice0=0,
                 sample0=0, length=None, ws=None):
        """x [rows, count] holding global samples [sample0, sample0 + count)
        of signals of global length `length` (default sample0 + count) ->
        coefficients of global slices [slice0, slice0 + S), complex64
        [rows * S * ncoef].  The transpose of the synthesis uses no window."""
        x = self._sig(x, "signal")
        rows, count = x.shape
        length = sample0 + count if length is None else int(length)
        S = self.count(length) - slice0 if S is None else int(S)
        if out is None:
            out = torch.empty(self.coef_numel(rows, S), dtype=torch.complex64,
                              device=self.eng.dev)
        elif (not torch.is_tensor(out) or out.device != self.eng.dev
              or out.dtype != torch.complex64 or not out.is_contiguous()
              or out.numel() != self.coef_numel(rows, S)):
            raise ValueError("out must be a contiguous complex64 buffer of rows * S * ncoef "
                             f"values on {self.eng.dev}")
        if ws is None:
            ws = self.eng.workspace(rows * S)
        stream = _raw_stream_of(self.eng.dev.index)
        sig = self._signal(x, sample0, length)
        if adjoint_of_synthesis:
            sl = self._slices(rows, slice0, S, None)
            self._call("cqt_sliced_adj_synthesis", ctypes.byref(sig), ctypes.byref(sl),
                       out.data_ptr(), ws.data_ptr(), ws.numel(), stream)
        else:
            sl = self._slices(rows, slice0, S, self.window)
            self._call("cqt_sliced_analysis", ctypes.byref(sig), ctypes.byref(sl),
                       out.data_ptr(), ws.data_ptr(), ws.numel(), stream)
        return out

    def synthesis(self, coef, rows, S, length, out=None, adjoint_of_analysis=False,
                  slice0=0, sample0=0, count=None, ws=None):
        """coefficients of global slices [slice0, slice0 + S) -> overlap-added
        output [rows, count] holding global samples [sample0, sample0 + count)
        (default: the whole signal [0, length)).  The transpose of the
        analysis applies the window."""
        if coef.dtype != torch.complex64 or coef.device != self.eng.dev:
            raise ValueError("coefficients must be complex64 on the engine's device")
        coef = coef.resolve_conj().contiguous()
        if coef.numel() != self.coef_numel(rows, S):
            raise ValueError("coefficient buffer does not match rows * S * ncoef")
        count = int(length) - sample0 if count is None else int(count)
        if out is None:
            out = torch.empty(rows, count, dtype=torch.float32, device=self.eng.dev)
        elif (not torch.is_tensor(out) or out.device != self.eng.dev
              or out.dtype != torch.float32 or tuple(out.shape) != (rows, count)
              or out.stride(-1) != 1):
            # written in place: no copy may stand in for it
            raise ValueError(f"out must be float32 [rows, count] = [{rows}, {count}] with "
                             f"unit sample stride on {self.eng.dev}")
        if ws is None:
            ws = self.eng.workspace(rows * S)
        stream = _raw_stream_of(self.eng.dev.index)
        sig = self._signal(out, sample0, length)
        if adjoint_of_analysis:
            sl = self._slices(rows, slice0, S, self.window)
            self._call("cqt_sliced_adj_analysis", coef.data_ptr(), ctypes.byref(sl),
                       ctypes.byref(sig), ws.data_ptr(), ws.numel(), stream)
        else:
            sl = self._slices(rows, slice0, S, None)
            self._call("cqt_sliced_synthesis", coef.data_ptr(), ctypes.byref(sl),
                       ctypes.byref(sig), ws.data_ptr(), ws.numel(), stream)
        return out
