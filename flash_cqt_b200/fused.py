"""``FusedOctCQT``: the planar, workspace-returning launcher API.

Drop-in for the launcher surface of ``flash_cqt/fused.py:226`` --
``FusedOctCQT(cqt, device)``, ``.fwd(x) -> (KR, KI)``, ``.bwd(KR, KI) -> XO``,
``.blocks_view``, ``.ncoef``, ``.gspec``, ``._workspace(B)`` -- with the
reference's contract that ``fwd`` / ``bwd`` return internal workspace tensors
that the next call of the same batch size overwrites (fused.py:517-523,
787-793).  The kernels are the B200 engines (one packed-spectrum kernel and one
band kernel per direction); the reference's Triton / cuBLAS / tf32 paths and
its ``sim_*`` matmul simulator are not part of this build.  ``prec`` is kept
as an attribute for compatibility and only "ieee" (fp32) exists.
"""
import torch

from .trainable import _engine_for


class FusedOctCQT:
    """kernel tables and launchers for one OctCQT at audio_len 65536 (or 32768)"""

    def __init__(self, cqt, device=None):
        from .tables import SLICE_LENS
        assert cqt.nn in SLICE_LENS, f"fused path is built for sl_len in {SLICE_LENS}"
        dev = torch.device(device) if device is not None else cqt.device
        self.cqt = cqt
        self.eng = _engine_for(cqt, dev)
        self.dev = self.eng.dev
        self.gspec = list(cqt.heap.gspec)
        self.ncoef = cqt.heap.ncoef
        self.prec = "ieee"
        self._ws = {}
        # host copies of the kernel tables, for inspection (torch, CPU)
        t = self.eng.host_tables
        self.radix = {
            "band_off": torch.as_tensor(t["band_off"]),
            "band_len": torch.as_tensor(t["band_len"]),
            "an_src": torch.as_tensor(t["fwd"]["analysis"][0]),
            "an_gain": torch.as_tensor(t["fwd"]["analysis"][1]),
            "as_src": torch.as_tensor(t["fwd"]["adj_synth"][0]),
            "as_gain": torch.as_tensor(t["fwd"]["adj_synth"][1]),
            "sy_dest": torch.as_tensor(t["inv"]["synth"][0]),
            "sy_gain": torch.as_tensor(t["inv"]["synth"][1]),
            "aa_dest": torch.as_tensor(t["inv"]["adj_an"][0]),
        }

    def _workspace(self, B):
        if B not in self._ws:
            z = lambda *s: torch.zeros(*s, dtype=torch.float32, device=self.dev)
            self._ws[B] = dict(KR=z(B, self.ncoef), KI=z(B, self.ncoef), XO=z(B, self.eng.N))
        return self._ws[B]

    def _check_prec(self):
        if getattr(self, "prec", "ieee") != "ieee":
            raise NotImplementedError("only fp32 ('ieee') kernels exist in this build")

    def fwd(self, x):
        """x [B, N] (N = audio_len) -> (KR, KI) planar [B, ncoef] workspace tensors"""
        self._check_prec()
        B = x.shape[0]
        w = self._workspace(B)
        self.eng.analysis_planar(x, w["KR"], w["KI"])
        return w["KR"], w["KI"]

    def bwd(self, KR, KI):
        """(KR, KI) planar -> XO [B, N] workspace tensor"""
        self._check_prec()
        B = KR.shape[0]
        w = self._workspace(B)
        self.eng.synthesis_planar(KR, KI, w["XO"])
        return w["XO"]

    def blocks_view(self, KR, KI):
        """complex per group views of the flat coefficient planes"""
        return [torch.complex(KR[:, off:off + b * M], KI[:, off:off + b * M])
                .view(-1, b, M) for b, M, off in self.gspec]
