"""``OctCQT``: the invertible oct-mode CQT of one 65536- or 32768-sample slice.

Drop-in for ``flash_cqt/oct_cqt.py:18-117``: same constructor, same
attributes (``bank``, ``nn``, ``oct_bins``, ``size_per_oct``, ``frqs_hz``,
``groups``, ``side_groups``, ``pos_flat``), same ``fwd`` / ``bwd`` contract --
but ``fwd`` / ``bwd`` run on the B200 engines (differentiable through the
transposed engines), not as eager torch ops.  The layout attributes are built
on the host and live on ``device`` as in the reference; the transform itself
needs a CUDA device and a 65536- or 32768-sample slice and raises otherwise
(there is no CPU path).
"""
import torch

from .layout import Filterbank, HeapLayout


class OctCQT:
    def __init__(self, num_octs, bins_per_oct, fs=44100, audio_len=44100,
                 device="cpu", dtype=torch.float32):
        self.bank = Filterbank(num_octs, bins_per_oct, fs, audio_len)
        self.heap = HeapLayout(self.bank)
        self.Ls = audio_len
        self.nn = self.bank.nn
        self.device = torch.device(device)
        self.dtype = dtype
        self.oct_bins = self.bank.oct_bins
        self.numocts = len(self.oct_bins)
        self.size_per_oct = self.bank.size_per_oct
        self.frqs_hz = self.bank.frqs_hz

        def as_torch(grp):
            idx, gv, pos, gdv, conj = grp
            return (torch.as_tensor(idx, device=self.device),
                    torch.as_tensor(gv, dtype=dtype, device=self.device),
                    torch.as_tensor(pos, device=self.device),
                    torch.as_tensor(gdv, dtype=dtype, device=self.device),
                    torch.as_tensor(conj, device=self.device))

        self.groups = [as_torch(g) for g in self.heap.groups]
        self.side_groups = [as_torch(g) for g in self.heap.side_groups]
        self.pos_flat = torch.cat([g[2].reshape(-1) for g in self.groups]
                                  + [g[2].reshape(-1) for g in self.side_groups])
        self._t = None

    def _trainable(self, device):
        from .trainable import TrainableCQT
        from .tables import SLICE_LENS
        if self.nn not in SLICE_LENS:
            raise NotImplementedError(
                f"the B200 engines are built for slices of {SLICE_LENS} samples "
                f"(this bank has audio_len {self.nn})")
        if self._t is None or self._t.dev != device:
            self._t = TrainableCQT(self, device)
        return self._t

    def fwd(self, x):
        """x [..., Ls] real, returns (blocks, side); blocks[i] is
        [..., oct_bins[i], size_per_oct[i]] complex, side is (dc, nyq), each
        [..., 1, M] complex"""
        if x.shape[-1] != self.Ls:
            raise ValueError(f"last dimension must be {self.Ls}")
        return self._trainable(x.device).fwd(x)

    def bwd(self, blocks, side=None):
        """inverse of fwd, side may be None to discard the DC and Nyquist bands"""
        return self._trainable(blocks[0].device).bwd(blocks, side)
