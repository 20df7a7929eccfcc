"""Streamable sliced CQT: 50%-overlap Tukey slices through the per-slice engine.

Drop-in for ``flash_cqt/sliced.py:41-209`` (``SlicedCQT``): same constructor,
``fwd`` / ``bwd`` / ``stream_fwd`` / ``stream_bwd`` and latency helpers, and
the same plugin point -- ``self.cqt`` is any object with OctCQT-shaped
``fwd(sl[..., sl_len]) -> (blocks, side)`` and ``bwd(blocks, side)``.  The
default engine is this package's ``OctCQT``, i.e. the B200 kernels.

Slicing (sliced.py:102-117): pad 2H in front, cut 4H windows every 2H, apply
the Tukey window, roll even slices by -H and odd ones by +H.  The coefficient
arrangement (sliced.py:119-146) rolls each octave block by +-M/4 per parity
and lays slices out along the time axis; ``bwd`` undoes both and overlap-adds
(sliced.py:148-167).

With the default engine all of that is fused into the CUDA kernels (the
cqt_sliced_* entry points): the analysis front end reads the slices straight
out of the signal with window and roll applied, the band kernels write the
rolled block layout directly (blocks are zero-copy views of one buffer), and
the synthesis back end un-rolls and overlap-adds in its store.  Gradients flow
through the transposed kernels.  A swapped-in ``self.cqt`` takes the generic
path (eager slicing around the engine's own fwd / bwd).
"""
import math

import torch

from .engine import SlicedEngine
from .layout import periodic_hann
from .oct_cqt import OctCQT
from .tables import SLICE_LENS


class _SlicedAnalysis(torch.autograd.Function):
    """x2 [rows, count] holds global samples [sample0, sample0 + count) of
    signals of global length `length`; -> coefficients of slices
    [slice0, slice0 + S)"""

    @staticmethod
    def forward(ctx, x2, se, S, slice0=0, sample0=0, length=None):
        length = sample0 + x2.shape[1] if length is None else length
        ctx.se, ctx.rows, ctx.count, ctx.S = se, x2.shape[0], x2.shape[1], S
        ctx.map = (slice0, sample0, length)
        return se.analysis(x2, S, slice0=slice0, sample0=sample0, length=length)

    @staticmethod
    def backward(ctx, g):
        slice0, sample0, length = ctx.map
        gx = ctx.se.synthesis(g.contiguous(), ctx.rows, ctx.S, length,
                              adjoint_of_analysis=True, slice0=slice0,
                              sample0=sample0, count=ctx.count)
        return gx, None, None, None, None, None


class _SlicedSynthesis(torch.autograd.Function):
    """coefficients of slices [slice0, slice0 + S) -> overlap-added output
    holding global samples [sample0, sample0 + count)"""

    @staticmethod
    def forward(ctx, buf, se, rows, S, length, slice0=0, sample0=0, count=None):
        ctx.se, ctx.S = se, S
        ctx.map = (slice0, sample0, length)
        return se.synthesis(buf, rows, S, length, slice0=slice0, sample0=sample0,
                            count=count)

    @staticmethod
    def backward(ctx, gy):
        slice0, sample0, length = ctx.map
        g = ctx.se.analysis(gy.contiguous(), ctx.S, adjoint_of_synthesis=True,
                            slice0=slice0, sample0=sample0, length=length)
        return g, None, None, None, None, None, None, None


def makewnd(sl_len, tr_area, device="cpu", dtype=torch.float32):
    """Tukey slice window: zero, Hann rise centred at sl_len/4, flat top, Hann
    fall centred at 3 sl_len/4, zero (sliced.py:26-38)."""
    hhop = sl_len // 4
    htr = tr_area // 2
    w = torch.as_tensor(periodic_hann(2 * tr_area))
    tw = torch.zeros(sl_len, dtype=torch.float64)
    tw[hhop - htr:hhop + htr] = w[tr_area:]
    tw[hhop + htr:3 * hhop - htr] = 1.0
    tw[3 * hhop - htr:3 * hhop + htr] = w[:tr_area]
    return tw.to(dtype).to(device)


class SlicedCQT:
    def __init__(self, num_octs=[3, 4, 2], bins_per_oct=[8, 16, 32], fs=44100,
                 sl_len=65536, tr_area=None, device="cuda", dtype=torch.float32):
        if sl_len % 4:
            raise ValueError("sl_len must be a multiple of 4")
        if tr_area is None:
            tr_area = sl_len // 4
        if tr_area % 2 or not 0 < 2 * tr_area <= sl_len:
            raise ValueError("tr_area must be even and 0 < 2 tr_area <= sl_len")
        self.fs = fs
        self.sl_len = sl_len
        self.tr_area = tr_area
        self.H = sl_len // 4
        self.hop = sl_len // 2
        self.device = torch.device(device)
        self.dtype = dtype
        self.cqt = OctCQT(num_octs, bins_per_oct, fs=fs, audio_len=sl_len,
                          device=device, dtype=dtype)
        self.oct_bins = self.cqt.oct_bins
        self.size_per_oct = self.cqt.size_per_oct
        self.frqs_hz = self.cqt.frqs_hz
        self.tw = makewnd(sl_len, tr_area, device=device, dtype=dtype)
        self._roll = [m // 4 for m in self.size_per_oct]
        self._fused_cqt = self.cqt
        self._se = None

    # the fused kernels serve the default engine on a CUDA device
    def _fused(self, device):
        if (self.cqt is not self._fused_cqt or self.sl_len not in SLICE_LENS
                or device.type != "cuda"):
            return None
        if self._se is None or self._se.eng.dev != device:
            eng = self.cqt._trainable(device).eng
            self._se = SlicedEngine(eng, self.tw)
        return self._se

    # latency helpers (sliced.py:71-98)
    def latency_ms(self, sl_len=None):
        return 1000.0 * (sl_len if sl_len is not None else self.sl_len) / self.fs

    def lowest_fmin(self, sl_len=None):
        sl = sl_len if sl_len is not None else self.sl_len
        n0 = 1
        while n0 < len(self.oct_bins) and self.oct_bins[n0] == self.oct_bins[0]:
            n0 += 1
        b0 = self.oct_bins[0]
        ratio = 2.0 ** ((n0 + 1) / ((n0 + 1) * b0 - 1))
        q0 = math.sqrt(ratio) / (ratio - 1.0) / 2.0
        return 8.0 * self.fs * q0 / sl

    def latency_table(self, sl_lens=(8192, 16384, 32768, 65536, 131072)):
        need = float(self.frqs_hz[0])
        lines = [f"{'sl_len':>8} {'latency_ms':>11} {'lowest_fmin_hz':>15}   "
                 f"covers fmin {need:.1f} hz"]
        for sl in sl_lens:
            fmin = self.lowest_fmin(sl)
            lines.append(f"{sl:>8} {self.latency_ms(sl):>11.1f} {fmin:>15.1f}   "
                         f"{'yes' if fmin <= need else 'no'}")
        return "\n".join(lines)

    # slicing
    def _num_slices(self, L):
        nb = -(-L // self.H)
        return (nb + 1) // 2 + 1

    def _slice(self, x):
        B, C, L = x.shape
        H = self.H
        S = self._num_slices(L)
        nb = -(-L // H)
        xp = torch.nn.functional.pad(x, (2 * H, nb * H - L + 3 * H))
        sl = xp.unfold(-1, 4 * H, 2 * H)[:, :, :S, :] * self.tw
        even = (torch.arange(S, device=x.device) % 2 == 0).view(1, 1, -1, 1)
        return torch.where(even, torch.roll(sl, -H, -1), torch.roll(sl, H, -1))

    def _arrange(self, blocks, S, fwd):
        out = []
        even = (torch.arange(S, device=blocks[0].device) % 2 == 0).view(1, 1, -1, 1, 1)
        s = 1 if fwd else -1
        for c, r in zip(blocks, self._roll):
            out.append(torch.where(even, torch.roll(c, s * r, -1),
                                   torch.roll(c, -s * r, -1)))
        return out

    # whole-buffer API
    def fwd(self, x):
        """x [B, C, L] real -> (blocks, side); blocks[i] is
        [B, C, oct_bins[i], S * size_per_oct[i]] complex (slices in time
        order), side is (dc, nyq) kept per slice, [B, C, S, 1, M]"""
        B, C, L = x.shape
        se = self._fused(x.device)
        if se is not None:
            S = self._num_slices(L)
            buf = _SlicedAnalysis.apply(x.reshape(B * C, L), se, S)
            return se.group_views(buf, (B, C), S)
        sl = self._slice(x)
        S = sl.shape[2]
        blocks, side = self.cqt.fwd(sl)
        blocks = self._arrange(blocks, S, fwd=True)
        blocks = [c.permute(0, 1, 3, 2, 4).reshape(B, C, b, S * m)
                  for c, b, m in zip(blocks, self.oct_bins, self.size_per_oct)]
        return blocks, side

    def _fused_buffer(self, se, blocks, side, rows, S):
        """the coefficient buffer behind (blocks, side): zero-copy when they
        are untouched views of one buffer, else packed in group order"""
        allb = list(blocks) + list(side if side is not None else [])
        base = allb[0]._base
        if side is not None and base is not None and base.dim() == 1 \
                and base.numel() == se.coef_numel(rows, S) \
                and all(c._base is base and c.is_contiguous() for c in allb):
            offs, off = [], 0
            for b, M, _ in se.gspec:
                offs.append(off)
                off += rows * S * b * M
            if all(c.storage_offset() - base.storage_offset() == o
                   for c, o in zip(allb, offs)):
                return base
        parts = [c.reshape(-1).to(torch.complex64) for c in allb]
        if side is None:
            nside = sum(rows * S * b * M for b, M, _ in se.gspec[len(blocks):])
            parts.append(torch.zeros(nside, dtype=torch.complex64, device=parts[0].device))
        return torch.cat(parts)

    def bwd(self, blocks, side=None, length=None):
        """inverse of fwd; length trims the tail padding"""
        B, C = blocks[0].shape[:2]
        S = blocks[0].shape[-1] // self.size_per_oct[0]
        se = self._fused(blocks[0].device)
        if se is not None:
            L = S * 2 * self.H if length is None else int(length)
            buf = self._fused_buffer(se, blocks, side, B * C, S)
            return _SlicedSynthesis.apply(buf, se, B * C, S, L).view(B, C, L)
        blocks = [c.reshape(B, C, b, S, m).permute(0, 1, 3, 2, 4)
                  for c, b, m in zip(blocks, self.oct_bins, self.size_per_oct)]
        blocks = self._arrange(blocks, S, fwd=False)
        y = self.cqt.bwd(blocks, side)
        H = self.H
        even = (torch.arange(S, device=y.device) % 2 == 0).view(1, 1, -1, 1)
        y = torch.where(even, torch.roll(y, H, -1), torch.roll(y, -H, -1))
        out = torch.zeros(B, C, (S + 1) * 2 * H, dtype=y.dtype, device=y.device)
        out[..., :S * 2 * H] += y[..., :2 * H].reshape(B, C, -1)
        out[..., 2 * H:] += y[..., 2 * H:].reshape(B, C, -1)
        out = out[..., 2 * H:]
        return out if length is None else out[..., :length]

    def streamer(self, lead, device=None):
        """a SliceStream (one CUDA graph replay per chunk) for chunks of
        shape [*lead, hop]"""
        return SliceStream(self, lead, device)

    # streaming API, state of one half slice (sliced.py:171-209)
    #
    # With the default engine the state stays on the device: stream_fwd keeps
    # the previous hop in a [rows, 2 hops] window buffer and runs the fused
    # sliced analysis on that window as global slice k (global samples
    # [hop (k - 1), hop (k + 1)), the +-H / +-M/4 rolls by the parity of k);
    # stream_bwd runs the fused synthesis of slice k into a [rows, 2 hops]
    # buffer and adds the tail kept from slice k - 1.  Coefficients and output
    # are bit-identical to the whole-buffer fwd / bwd (each output sample is
    # the same sum of two terms).
    def stream_fwd(self, chunks):
        """chunks yields [B, C, hop] pieces (pad the last one); yields one
        (blocks, side) per slice, blocks[i] [B, C, oct_bins[i], M_i]"""
        prev = None
        win = None
        k = 0
        hop = self.hop

        def one_generic(prev, chunk, k):
            sl = torch.cat([prev, chunk], dim=-1) * self.tw
            sl = torch.roll(sl, -self.H if k % 2 == 0 else self.H, -1)
            blocks, side = self.cqt.fwd(sl.unsqueeze(2))
            blocks = self._arrange(blocks, 1, fwd=(k % 2 == 0))
            return [c[:, :, 0] for c in blocks], [c[:, :, 0] for c in side]

        def one_fused(se, win, lead, k):
            buf = _SlicedAnalysis.apply(win, se, 1, k, hop * (k - 1), hop * (k + 1))
            blocks, side = se.group_views(buf, lead, 1)
            return blocks, [c[:, :, 0] for c in side]

        se = None
        for chunk in chunks:
            if prev is None:
                prev = torch.zeros_like(chunk)
                se = self._fused(chunk.device) if chunk.shape[-1] == hop else None
            if se is None:
                yield one_generic(prev, chunk, k)
            else:
                B, C, _ = chunk.shape
                if win is None or chunk.requires_grad:   # fresh buffer under autograd
                    win = chunk.new_zeros(B * C, 2 * hop)
                win[:, :hop] = prev.reshape(B * C, hop)
                win[:, hop:] = chunk.reshape(B * C, hop)
                yield one_fused(se, win, (B, C), k)
            prev = chunk
            k += 1
        if prev is not None:
            if se is None:
                yield one_generic(prev, torch.zeros_like(prev), k)
            else:
                B, C, _ = prev.shape
                win = prev.new_zeros(B * C, 2 * hop)
                win[:, :hop] = prev.reshape(B * C, hop)
                yield one_fused(se, win, (B, C), k)

    def stream_bwd(self, slice_coeffs):
        """slice_coeffs yields (blocks, side) per slice as stream_fwd emits;
        yields [B, C, hop] output pieces, one slice behind the input"""
        tail = None
        k = 0
        hop = self.hop
        for blocks, side in slice_coeffs:
            B, C = blocks[0].shape[:2]
            se = self._fused(blocks[0].device)
            if se is not None and blocks[0].shape[-1] == self.size_per_oct[0]:
                sd = [c.unsqueeze(2) for c in side] if side is not None else None
                buf = self._fused_buffer(se, blocks, sd, B * C, 1)
                y = _SlicedSynthesis.apply(buf, se, B * C, 1, hop * (k + 1), k,
                                           hop * (k - 1), 2 * hop).view(B, C, 2 * hop)
            else:
                blocks = [c.unsqueeze(2) for c in blocks]
                side = [c.unsqueeze(2) for c in side] if side is not None else None
                blocks = self._arrange(blocks, 1, fwd=not (k % 2 == 0))
                y = self.cqt.bwd(blocks, side)[:, :, 0]
                y = torch.roll(y, self.H if k % 2 == 0 else -self.H, -1)
            if tail is not None:
                yield tail + y[..., :hop]
            tail = y[..., hop:]
            k += 1


class SliceStream:
    """The streaming transform as one CUDA graph replay per chunk.

        st = sliced.streamer((B, C))
        blocks, side = st.fwd(chunk)      # chunk [B, C, hop]; one slice per call
        blocks, side = st.flush()         # the last slice (zeros after the end)
        y = st.bwd(blocks, side)          # [B, C, hop], one slice behind; None first

    State on the device: the two-hop input window, the overlap-add tail.
    Slices map onto the window the same way for every k but the boundary
    clip, so three graphs per direction cover the stream: k = 0 (samples
    before the start read as zeros, mapped as global slice 0), odd k (as
    slice 1) and even k >= 2 (as slice 2); the rolls follow the parity.
    Results are bit-identical to ``stream_fwd`` / ``stream_bwd`` and to the
    whole-buffer transform.  Inference only (graphs record no autograd);
    returned tensors are fresh copies."""

    def __init__(self, sliced, lead, device=None):
        dev = torch.device(device) if device is not None else sliced.device
        se = sliced._fused(dev)
        if se is None:
            raise RuntimeError("the graphed stream needs the default engine on a CUDA device")
        self.sl, self.se, self.lead = sliced, se, tuple(lead)
        rows = 1
        for d in self.lead:
            rows *= d
        self.rows, self.hop = rows, sliced.hop
        hop = self.hop
        z = lambda *s_, dt=torch.float32: torch.zeros(*s_, dtype=dt, device=dev)
        self.win = z(rows, 2 * hop)
        self.chunk = z(rows, hop)
        self.coef = z(se.coef_numel(rows, 1), dt=torch.complex64)
        self.cin = z(se.coef_numel(rows, 1), dt=torch.complex64)
        self.ybuf = z(rows, 2 * hop)
        self.tail = z(rows, hop)
        self.out = z(rows, hop)
        self.ws = torch.zeros(max(se.eng.tables.workspace_bytes(rows), 256), dtype=torch.uint8,
                              device=dev)   # zeroed: the header holds the wait status
        self.kf = self.kb = 0

        def fwd_body(s0):
            self.win[:, :hop].copy_(self.win[:, hop:])
            self.win[:, hop:].copy_(self.chunk)
            se.analysis(self.win, 1, out=self.coef, slice0=s0, sample0=hop * (s0 - 1),
                        length=hop * (s0 + 1), ws=self.ws)

        def bwd_body(s0):
            se.synthesis(self.cin, rows, 1, hop * (s0 + 1), out=self.ybuf, slice0=s0,
                         sample0=hop * (s0 - 1), count=2 * hop, ws=self.ws)
            torch.add(self.tail, self.ybuf[:, :hop], out=self.out)
            self.tail.copy_(self.ybuf[:, hop:])

        with torch.cuda.device(dev):
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side), torch.no_grad():
                for s0 in (0, 1, 2):   # warm-up outside the captures
                    fwd_body(s0)
                    bwd_body(s0)
            torch.cuda.current_stream(dev).wait_stream(side)
            self.gf, self.gb = [], []
            for s0 in (0, 1, 2):
                for body, lst in ((fwd_body, self.gf), (bwd_body, self.gb)):
                    g = torch.cuda.CUDAGraph()
                    with torch.no_grad(), torch.cuda.graph(g):
                        body(s0)
                    lst.append(g)
        self.reset()

    def reset(self):
        """start a new stream (the state buffers are cleared)"""
        self.win.zero_()
        self.tail.zero_()
        self.kf = self.kb = 0

    @staticmethod
    def _variant(k):
        return 0 if k == 0 else (1 if k % 2 else 2)

    @torch.no_grad()
    def fwd(self, chunk):
        """chunk [*lead, hop] -> (blocks, side) of the next slice"""
        if tuple(chunk.shape) != self.lead + (self.hop,):
            raise ValueError(f"chunk must be {self.lead + (self.hop,)}, got {tuple(chunk.shape)}")
        self.chunk.copy_(chunk.reshape(self.rows, self.hop))
        return self._run_fwd()

    @torch.no_grad()
    def flush(self):
        """the final slice: the hop after the last chunk reads as zeros"""
        self.chunk.zero_()
        return self._run_fwd()

    def _run_fwd(self):
        self.gf[self._variant(self.kf)].replay()
        self.kf += 1
        blocks, side = self.se.group_views(self.coef.clone(), self.lead, 1)
        return blocks, [c[:, :, 0] for c in side]

    @torch.no_grad()
    def bwd(self, blocks, side):
        """(blocks, side) of the next slice -> the finished hop one slice
        behind ([*lead, hop]), or None after the first slice"""
        sd = [c.unsqueeze(2) for c in side] if side is not None else None
        buf = self.sl._fused_buffer(self.se, blocks, sd, self.rows, 1)
        self.cin.copy_(buf)
        self.gb[self._variant(self.kb)].replay()
        self.kb += 1
        if self.kb == 1:
            return None
        return self.out.clone().view(*self.lead, self.hop)
