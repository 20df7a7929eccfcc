"""Slice-range partitioning of the sliced transform over several GPUs.

One process per GPU (``torch.distributed``, NCCL for CUDA tensors).  A long
stream of S slices (SlicedCQT, 50 % overlap, hop 2H = 32768 samples) is cut
into contiguous slice ranges, rank r owning slices [s0, s1) and the output
samples [2H s0, 2H s1):

* analysis needs no communication -- slice g reads global samples
  [2H (g - 1), 2H (g + 1)), so a rank reads its range plus one hop of input
  halo at each end (``input_window``), from a replicated signal or from the
  chunk it was handed;
* synthesis overlap-adds inside the rank; output hop q receives slices q and
  q + 1, so the only hop a rank cannot finish alone is its last one, which
  also gets the first-half contribution of the next rank's first slice.  Each
  rank r > 0 therefore sends one hop (2H samples per row) to rank r - 1, which
  adds it in; nothing else crosses NVLink.  On GPUs under NCCL the hop moves
  through this build's peer-memory kernels (``PeerHalo``: plain NVLink stores
  into the neighbour's IPC-mapped buffer, a flag, an acknowledgement, bounded
  waits); otherwise -- and on CPU ranks -- through torch.distributed send /
  receive (``exchange_halo``).

The partition is pure bookkeeping on slice indices; the transform itself is
the fused sliced kernels (``SlicedEngine``) on each rank's device.
"""
import torch
import torch.distributed as dist


def slice_ranges(S, world):
    """Balanced contiguous slice ranges [(s0, s1)] for `world` ranks."""
    base, extra = divmod(S, world)
    out, s = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((s, s + n))
        s += n
    return out


class Partition:
    """Geometry of one rank's share of a stream of `length` samples."""

    def __init__(self, length, S, rank, world, hop=32768):
        self.length, self.S, self.rank, self.world, self.hop = length, S, rank, world, hop
        ranges = slice_ranges(S, world)
        self.s0, self.s1 = ranges[rank]
        self.nslices = self.s1 - self.s0
        # with fewer slices than ranks the trailing ranks own nothing; the
        # halo exchange pairs a rank with its right neighbour only when that
        # neighbour has slices (it alone sends), so both sides agree
        self.right_nslices = (ranges[rank + 1][1] - ranges[rank + 1][0]
                              if rank + 1 < world else 0)

    def input_window(self):
        """global input samples the rank's slices read: [start, stop)"""
        return self.hop * (self.s0 - 1), self.hop * (self.s1 + 1)

    def synthesis_window(self):
        """global samples the rank's slices overlap-add into: one hop before
        the owned range (sent to the left neighbour) plus the owned range"""
        return self.hop * (self.s0 - 1), self.hop * self.s1

    def owned(self):
        """global output samples the rank owns after the halo exchange
        (empty, at the signal's end, for a rank whose slices start past it)"""
        lo = min(self.hop * self.s0, self.length)
        hi = min(self.hop * self.s1, self.length)
        return lo, max(lo, hi)


def exchange_halo(local, part, group=None):
    """local [rows, 2H + owned...]: the rank's overlap-added synthesis over
    ``part.synthesis_window()``.  Sends the first hop to rank - 1, adds the
    hop received from rank + 1 into the last owned hop, and returns the owned
    part (a view of `local`).  Every rank makes the same calls in the same
    order.  A rank sends only if it owns slices, and receives only from a right
    neighbour that owns slices, so a stream of fewer slices than ranks leaves
    no receive without its send (the trailing ranks own nothing and take no
    part)."""
    H2 = part.hop
    ops = []
    recv = None
    if part.rank > 0 and part.nslices > 0:
        ops.append(dist.P2POp(dist.isend, local[:, :H2].contiguous(), part.rank - 1,
                              group=group))
    if part.right_nslices > 0:
        recv = torch.empty(local.shape[0], H2, dtype=local.dtype, device=local.device)
        ops.append(dist.P2POp(dist.irecv, recv, part.rank + 1, group=group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    if recv is not None and part.nslices > 0:
        local[:, -H2:] += recv
    lo, hi = part.owned()
    start = lo - part.synthesis_window()[0]
    return local[:, start:start + (hi - lo)]


class PeerHalo:
    """The overlap-add halo over peer memory (``cqt_halo_*``): this build's own
    kernels store rank r's first hop straight into rank r - 1's receive buffer
    over NVLink (plain peer stores, CUDA IPC mapping, no multicast) and raise
    a flag; rank r - 1 waits (bounded, 10 s), adds it into its last owned hop
    and acknowledges.  Stream-ordered, no host synchronisation; an expired
    wait is counted on the device and raised by ``check``.

    Set up in two local steps -- ``PeerHalo(...)`` allocates and exports the
    receive buffer (``handle``), ``connect`` maps the neighbours' buffers --
    so that the ranks can exchange handles and agree on success between
    them (``PartitionedSlicedCQT`` does)."""

    HANDLE = 64

    def __init__(self, rows, hop, device, wait_ms=10000):
        import ctypes
        from . import _native
        self._n = _native
        self._c = ctypes
        self.rows, self.hop, self.device = rows, hop, device
        self.h = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * self.HANDLE)()
        _native._check(_native.lib().cqt_halo_create(device.index, rows, hop, int(wait_ms),
                                                     ctypes.byref(self.h), handle),
                       "cqt_halo_create")
        self.handle = bytes(handle)
        self.epoch = 0

    def connect(self, left=None, right=None):
        """map the receive buffers of the left / right neighbour (their
        ``handle`` bytes, None for no neighbour on that side)"""
        buf = lambda b: ((self._c.c_ubyte * self.HANDLE).from_buffer_copy(b)
                         if b is not None else None)
        self._n._check(self._n.lib().cqt_halo_connect(self.h, buf(left), buf(right)),
                       "cqt_halo_connect")

    def exchange(self, local, send, recv):
        """local [rows, window] float32 on the device: send local[:, :hop]
        to the left neighbour and/or add the right neighbour's hop into
        local[:, -hop:] (the calls every rank makes in the same order)"""
        from .engine import _raw_stream_of
        L = self._n.lib()
        self.epoch += 1
        stream = _raw_stream_of(self.device.index)
        if local.stride(-1) != 1:
            raise ValueError("the overlap-add window must have unit sample stride")
        ld = local.stride(0)
        if send:
            self._n._check(L.cqt_halo_send(self.h, local.data_ptr(), ld, self.epoch, stream),
                           "cqt_halo_send")
        if recv:
            dst = local[:, local.shape[1] - self.hop:]
            self._n._check(L.cqt_halo_recv_add(self.h, dst.data_ptr(), ld, self.epoch, stream),
                           "cqt_halo_recv_add")

    def check(self):
        """synchronous: raise if any wait of this exchange gave up"""
        n = self._c.c_uint(0)
        self._n._check(self._n.lib().cqt_halo_waits(self.h, self._c.byref(n), 1),
                       "cqt_halo_waits")
        if n.value:
            raise RuntimeError(f"overlap-add halo: {n.value} bounded wait(s) on a neighbour "
                               "gave up (a rank stopped or fell too far behind)")

    def __del__(self):
        h = getattr(self, "h", None)
        if h is not None and h.value and self._n._lib is not None:
            try:
                self._n.lib().cqt_halo_free(h)
            except Exception:
                pass


class PartitionedSlicedCQT:
    """A SlicedCQT whose slices are spread over the ranks of a process group.

        part = PartitionedSlicedCQT(SlicedCQT(..., device=f"cuda:{rank}"), rank, world)
        blocks, side = part.fwd(x_chunk, length, sample0)   # this rank's slices
        y_owned = part.bwd(blocks, side, length)           # owned samples only
    """

    def __init__(self, sliced, rank, world, group=None, halo="auto", halo_wait_ms=10000):
        """halo: "peer" (this build's peer-memory kernels), "collective"
        (torch.distributed send / receive), or "auto" -- peer memory for CUDA
        tensors under an NCCL group, the collective otherwise; halo_wait_ms
        bounds every peer-memory wait on a neighbour"""
        self.sl = sliced
        self.rank, self.world, self.group = rank, world, group
        self.halo = halo
        self.halo_wait_ms = halo_wait_ms
        self._peer = {}

    def partition(self, length):
        return Partition(length, self.sl._num_slices(length), self.rank, self.world,
                         self.sl.hop)

    def fwd(self, x, length, sample0=0):
        """x [B, C, count]: global samples [sample0, sample0 + count) of the
        signals (the rank's input window, or the whole replicated signal).
        Returns the blocks of the rank's slices in SlicedCQT.fwd's layout."""
        B, C, _ = x.shape
        p = self.partition(length)
        se = self.sl._fused(x.device)
        if se is None:
            raise RuntimeError("the partitioned transform needs the default CUDA engine")
        if p.nslices == 0:   # a trailing rank of a stream shorter than the world
            buf = torch.empty(0, dtype=torch.complex64, device=x.device)
        else:
            buf = se.analysis(x.reshape(B * C, -1), p.nslices, slice0=p.s0,
                              sample0=sample0, length=length)
        return se.group_views(buf, (B, C), p.nslices)

    def bwd(self, blocks, side, length):
        """synthesis of the rank's slices + halo exchange -> the rank's owned
        output samples [B, C, owned]"""
        B, C = blocks[0].shape[:2]
        p = self.partition(length)
        lo, hi = p.synthesis_window()
        if p.nslices == 0:   # nothing to synthesise; still takes its (empty) part
            local = torch.zeros(B * C, hi - lo, device=blocks[0].device)
        else:
            se = self.sl._fused(blocks[0].device)
            buf = self.sl._fused_buffer(se, blocks, side, B * C, p.nslices)
            local = se.synthesis(buf, B * C, p.nslices, length, slice0=p.s0, sample0=lo,
                                 count=hi - lo)
        halo = self._peer_halo(B * C, p, local.device) if self._use_peer(local) else None
        if halo is not None:
            halo.exchange(local, send=p.rank > 0 and p.nslices > 0, recv=p.right_nslices > 0)
            lo_, hi_ = p.owned()
            start = lo_ - p.synthesis_window()[0]
            own = local[:, start:start + (hi_ - lo_)]
        else:
            own = exchange_halo(local, p, self.group)
        return own.reshape(B, C, -1)

    def _use_peer(self, t):
        if self.halo == "collective" or self.world == 1:
            return False
        if self.halo == "peer":
            return True
        return t.is_cuda and dist.get_backend(self.group) == "nccl"

    def _peer_halo(self, rows, p, device):
        """one exchange per (rows, left, right) shape; created collectively on
        first use (every rank takes the same bwd calls in the same order, and
        every rank makes the same collectives here whatever fails locally)"""
        key = (rows, p.rank > 0 and p.nslices > 0, p.right_nslices > 0)
        if key not in self._peer:
            h, err = None, None
            try:
                h = PeerHalo(rows, p.hop, device, wait_ms=self.halo_wait_ms)
            except RuntimeError as e:   # e.g. no memory for the receive buffer
                err = str(e)
            got = [None] * p.world
            dist.all_gather_object(got, (h.handle if h is not None else None, err),
                                   group=self.group)
            bad = [e for _, e in got if e]
            if not bad:
                try:
                    h.connect(left=got[p.rank - 1][0] if key[1] else None,
                              right=got[p.rank + 1][0] if key[2] else None)
                except RuntimeError as e:   # e.g. no peer access between these devices
                    err = str(e)
                errs = [None] * p.world
                dist.all_gather_object(errs, err, group=self.group)
                bad = [e for e in errs if e]
            # every rank takes the same transport
            if bad:
                del h
                if self.halo == "peer":
                    raise RuntimeError(f"peer-memory halo unavailable: {bad[0]}")
                self.halo = "collective"   # auto: torch.distributed on every rank
                return None
            self._peer[key] = h
        return self._peer[key]

    def check_halo(self):
        """synchronous: raise if a peer-memory halo wait gave up"""
        for h in self._peer.values():
            h.check()
