"""Torch-facing wrapper of the CUDA engines for one filterbank on one device.

PyTorch only provides device memory and the current stream here; every
transform runs in the sm_100a kernels of ``libflashcqt_b200.so``.
"""
import torch

from . import _native
from .layout import Filterbank, HeapLayout
from .tables import build_tables

N = 65536


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
        self.host_tables = build_tables(heap)
        self.tables = _native.DeviceTables(self.host_tables, self.dev.index)
        assert self.tables.ncoef == self.ncoef
        self._ws = None

    @classmethod
    def from_params(cls, num_octs, bins_per_oct, fs, audio_len, device=None):
        return cls(HeapLayout(Filterbank(num_octs, bins_per_oct, fs, audio_len)),
                   device)

    # ---------------------------------------------------------------- plumbing
    def workspace(self, batch):
        need = self.tables.workspace_bytes(batch)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(max(need, 16), dtype=torch.uint8, device=self.dev)
        return self._ws

    def _stream(self):
        return ctypes_stream(torch.cuda.current_stream(self.dev))

    def _signal(self, t, name):
        if not torch.is_tensor(t) or t.device != self.dev:
            raise ValueError(f"{name} must be a tensor on {self.dev}")
        if t.dtype != torch.float32:
            raise TypeError(f"{name} must be float32, got {t.dtype}")
        if t.dim() != 2 or t.shape[-1] != N:
            raise ValueError(f"{name} must be [B, {N}], got {tuple(t.shape)}")
        return t.contiguous()

    def _coef(self, c, name):
        if not torch.is_tensor(c) or c.device != self.dev:
            raise ValueError(f"{name} must be a tensor on {self.dev}")
        if c.dtype != torch.complex64:
            raise TypeError(f"{name} must be complex64, got {c.dtype}")
        if c.dim() != 2 or c.shape[-1] != self.ncoef:
            raise ValueError(f"{name} must be [B, {self.ncoef}], got {tuple(c.shape)}")
        return c.resolve_conj().contiguous()

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
        with torch.cuda.device(self.dev):
            ws = self.workspace(batch)
            self.tables.call(name, a, b, c, layout, batch, ws.data_ptr(), ws.numel(),
                             self._stream())

    # ----------------------------------------------------------------- complex
    def analysis(self, x, out=None):
        """x [B, 65536] float32 -> coefficient heap complex64 [B, ncoef]."""
        x = self._signal(x, "x")
        B = x.shape[0]
        if out is None:
            out = torch.empty(B, self.ncoef, dtype=torch.complex64, device=self.dev)
        self._run("cqt_analysis", x.data_ptr(), out.data_ptr(), None,
                  _native.CQT_LAYOUT_COMPLEX, B)
        return out

    def synthesis(self, c, out=None):
        """coefficient heap complex64 [B, ncoef] -> y [B, 65536] float32."""
        c = self._coef(c, "coefficients")
        B = c.shape[0]
        if out is None:
            out = torch.empty(B, N, dtype=torch.float32, device=self.dev)
        self._run("cqt_synthesis", c.data_ptr(), None, out.data_ptr(),
                  _native.CQT_LAYOUT_COMPLEX, B)
        return out

    def adj_analysis(self, g, out=None):
        """transpose of analysis: complex64 grads [B, ncoef] -> [B, 65536]."""
        g = self._coef(g, "coefficient gradient")
        B = g.shape[0]
        if out is None:
            out = torch.empty(B, N, dtype=torch.float32, device=self.dev)
        self._run("cqt_adj_analysis", g.data_ptr(), None, out.data_ptr(),
                  _native.CQT_LAYOUT_COMPLEX, B)
        return out

    def adj_synthesis(self, gy, out=None):
        """transpose of synthesis: [B, 65536] -> complex64 grads [B, ncoef]."""
        gy = self._signal(gy, "signal gradient")
        B = gy.shape[0]
        if out is None:
            out = torch.empty(B, self.ncoef, dtype=torch.complex64, device=self.dev)
        self._run("cqt_adj_synthesis", gy.data_ptr(), out.data_ptr(), None,
                  _native.CQT_LAYOUT_COMPLEX, B)
        return out

    # ------------------------------------------------------------------ planar
    def analysis_planar(self, x, kr, ki):
        x = self._signal(x, "x")
        kr, ki = self._planes(kr, ki)
        self._run("cqt_analysis", x.data_ptr(), kr.data_ptr(), ki.data_ptr(),
                  _native.CQT_LAYOUT_PLANAR, x.shape[0])
        return kr, ki

    def synthesis_planar(self, kr, ki, y):
        kr, ki = self._planes(kr, ki)
        self._run("cqt_synthesis", kr.data_ptr(), ki.data_ptr(), y.data_ptr(),
                  _native.CQT_LAYOUT_PLANAR, kr.shape[0])
        return y


def ctypes_stream(stream):
    return int(stream.cuda_stream)
