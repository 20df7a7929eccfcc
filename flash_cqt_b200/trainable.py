"""Differentiable constant-Q transform on the B200 engines.

Drop-in for ``flash_cqt/trainable.py:28-191`` (``TrainableCQT``): the
transform is linear, so the backward of the analysis is the transpose of the
analysis (synthesis engine with the analysis window, ``cqt_adj_analysis``) and
the backward of the synthesis is the transpose of the synthesis (analysis
engine with the dual window, ``cqt_adj_synthesis``).  Nothing is saved for
backward.

When the torch fast path (``csrc/torch_ops.cpp``) is built, ``fwd`` / ``bwd``
and the two autograd functions run in C++ (same kernels, same results, no
Python in the backward); the Python classes below serve otherwise.

Differences from the reference, all in the data path, none in the interface:
the coefficients come out of the kernel already interleaved, so the blocks
returned by ``fwd`` are zero-copy views of one complex64 heap (the reference
builds them with ``torch.complex`` copies, trainable.py:146-152), and ``bwd``
hands such views back to the kernel without a ``torch.cat`` when they are
still laid out as ``fwd`` produced them.
"""
import weakref

import torch

from .engine import Engine


class _Analysis(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, eng):
        ctx.eng = eng
        return eng.analysis(x)

    @staticmethod
    def backward(ctx, g):
        return ctx.eng.adj_analysis(g.contiguous()), None


class _Synthesis(torch.autograd.Function):
    @staticmethod
    def forward(ctx, c, eng):
        ctx.eng = eng
        return eng.synthesis(c)

    @staticmethod
    def backward(ctx, gy):
        return ctx.eng.adj_synthesis(gy.contiguous()), None


class _SynthesisMSE(torch.autograd.Function):
    """synthesis + mean squared error: (loss, y), y not differentiable; the
    backward folds dL/dy = 2 dL/dloss (y - target) / n into the load of the
    transposed synthesis (cqt_adj_synthesis_sqerr)"""

    @staticmethod
    def forward(ctx, c, target, eng):
        ctx.eng = eng
        loss, y, t = eng.synthesis_sqerr(c, target)
        ctx.y, ctx.t = y, t
        ctx.mark_non_differentiable(y)
        ctx.set_materialize_grads(False)   # no zero gradient is built for y
        return loss, y

    @staticmethod
    def backward(ctx, gl, _gy):
        if gl is None:
            return None, None, None
        y, t = ctx.y, ctx.t
        scale = 2.0 / y.numel() if y.numel() else 0.0
        gl = gl.to(device=y.device, dtype=torch.float32).contiguous()
        gc = ctx.eng.adj_synthesis_sqerr(y, t, scale, gl)
        gt = (y - t) * (gl * -scale) if ctx.needs_input_grad[1] else None
        return gc, gt, None


def _engine_for(cqt, device):
    """One Engine per (filterbank, device), cached on the OctCQT object."""
    dev = torch.device(device) if device is not None else None
    cache = cqt.__dict__.setdefault("_b200_engines", {})
    key = str(dev)
    if key not in cache:
        cache[key] = Engine(cqt.heap, dev)
    return cache[key]


class TrainableCQT:
    """OctCQT-shaped ``fwd`` / ``bwd`` on the CUDA engines, with gradients.

        cqt = OctCQT([3, 4, 2], [8, 16, 32], fs=44100, audio_len=65536,
                     device="cuda")
        t = TrainableCQT(cqt)
        blocks, side = t.fwd(x)       # x [..., 65536] float32
        y = t.bwd(blocks, side)       # gradients flow both ways
    """

    def __init__(self, cqt, device="cuda"):
        from .tables import SLICE_LENS
        if cqt.nn not in SLICE_LENS:
            raise ValueError(f"the CUDA engines are built for slices of {SLICE_LENS} samples, "
                             f"got {cqt.nn}")
        self.cqt = cqt
        self.N = cqt.nn
        self.eng = _engine_for(cqt, device)
        self.dev = self.eng.dev
        self.gspec = cqt.heap.gspec
        self.ncoef = cqt.heap.ncoef
        self.ngroups = len(cqt.heap.groups)
        self._sizes = [b * M for b, M, _ in self.gspec]

    def split(self, h, lead):
        """heap [B, ncoef] complex -> (blocks, side) views with leading dims."""
        vs = [p.view(*lead, b, M)
              for p, (b, M, _) in zip(h.split(self._sizes, dim=1), self.gspec)]
        # remembered (weakly: no tensor is kept alive) so that heap_of can
        # recognise them by identity
        self._last = (weakref.ref(h), tuple(weakref.ref(v) for v in vs))
        return vs[:self.ngroups], vs[self.ngroups:]

    def fwd(self, x):
        """x [..., N] real (N = audio_len) -> (blocks, side), complex64, gradients flow."""
        ops = self.eng._ops
        if ops is not None:   # the same, from C++ (autograd nodes included)
            return ops.fwd(x)
        lead = x.shape[:-1]
        B = 1
        for d in lead:   # explicit: reshape cannot infer -1 for an empty batch
            B *= d
        h = _Analysis.apply(x.reshape(B, self.N).contiguous(), self.eng)
        return self.split(h, lead)

    def heap_of(self, blocks, side=None):
        """(blocks, side) -> one [B, ncoef] complex64 heap (zero-copy when the
        blocks are untouched views of one heap, as ``fwd`` returns them)."""
        allb = list(blocks) + list(side if side is not None else [])
        last = self.__dict__.get("_last")
        if last is not None and len(allb) == len(last[1]) and \
                all(a is r() for a, r in zip(allb, last[1])):
            h = last[0]()
            if h is not None:
                return h   # the very views the last fwd returned
        lead = allb[0].shape[:-2]
        B = 1
        for d in lead:
            B *= d
        base = allb[0]._base
        if (side is not None and len(allb) == len(self.gspec) and base is not None
                and base.dim() == 2 and base.shape == (B, self.ncoef)
                and base.dtype == torch.complex64 and base.is_contiguous()
                and all(c._base is base for c in allb)
                and all(c.storage_offset() - base.storage_offset() == off
                        and c.stride()[-1] == 1 and c.stride()[-2] == M
                        for c, (b, M, off) in zip(allb, self.gspec))):
            return base
        parts = [c.reshape(B, c.shape[-2] * c.shape[-1]).to(torch.complex64) for c in allb]
        if side is None:
            nside = sum(b * M for b, M, _ in self.gspec[self.ngroups:])
            parts.append(torch.zeros(B, nside, dtype=torch.complex64,
                                     device=parts[0].device))
        return torch.cat(parts, dim=-1)

    def bwd(self, blocks, side=None):
        """inverse of fwd (side None drops the DC and Nyquist bands)."""
        lead = blocks[0].shape[:-2]
        ops = self.eng._ops
        if ops is not None:
            h = ops.last_heap(list(blocks) + list(side)) if side is not None else None
            if h is None:
                h = self.heap_of(blocks, side)
            y = ops.synthesis_heap(h)
            # a one-dimensional lead is the heap's batch already: no view node
            return y if len(lead) == 1 else y.reshape(*lead, self.N)
        h = self.heap_of(blocks, side)
        return _Synthesis.apply(h, self.eng).reshape(*lead, self.N)

    def mse_loss(self, blocks, side, target, return_output=False):
        """``((self.bwd(blocks, side) - target) ** 2).mean()`` -- the loss of the
        reference's train step -- with the loss and its gradient folded into
        the engines: the synthesis sums the squared error as it stores y, and
        the backward forms 2 (y - target) / n inside the transposed
        synthesis' load (no elementwise kernels in between).  target
        [..., N] float32 like the output; returns the 0-dim loss, or
        (loss, y) with ``return_output`` (y carries no gradient)."""
        ops = self.eng._ops
        if ops is not None and side is not None:
            # the views of the last fwd: one call into C++ (ValueError on a bad target)
            r = ops.mse_views(blocks + side if type(blocks) is list and type(side) is list
                              else list(blocks) + list(side), target)
            if r is not None:
                return r if return_output else r[0]
        lead = blocks[0].shape[:-2]
        B = 1
        for d in lead:
            B *= d
        if tuple(target.shape) != (*lead, self.N):
            raise ValueError(f"target must be {(*lead, self.N)}, got {tuple(target.shape)}")
        h = None
        if ops is not None and side is not None:
            h = ops.last_heap(list(blocks) + list(side))
        if h is None:
            h = self.heap_of(blocks, side)
        t2 = target if target.dim() == 2 else target.reshape(B, self.N)
        if ops is not None:
            loss, y = ops.mse(h, t2)
        else:
            loss, y = _SynthesisMSE.apply(h, t2, self.eng)
        if return_output:
            return loss, (y if len(lead) == 1 else y.reshape(*lead, self.N))
        return loss

    # flat-heap entry points (no per-group views), used by the fused sliced path
    def analysis_heap(self, x):
        ops = self.eng._ops
        return ops.analysis_heap(x) if ops is not None else _Analysis.apply(x, self.eng)

    def synthesis_heap(self, h):
        ops = self.eng._ops
        return ops.synthesis_heap(h) if ops is not None else _Synthesis.apply(h, self.eng)
