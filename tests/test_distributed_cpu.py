"""Slice-range partitioning and the overlap-add halo exchange, on CPU ranks.

world_size 2 and 3 ``gloo`` process groups run ``flash_cqt_b200.distributed``'s
bookkeeping and ``exchange_halo`` on per-rank overlap-add buffers built from
the oracle's per-slice synthesis; the owned output ranges, gathered, must equal
the oracle's whole-buffer inverse.  This is the host-side logic of the
multi-GPU sliced path; on GPUs the same functions run on the fused kernels'
outputs over NCCL.  Failures are made on the host: a rank that leaves without
sending, and a stand-in for the peer-memory set-up that fails on one rank
(every rank must then take the same transport).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flash_cqt_b200.distributed import Partition, exchange_halo, slice_ranges

H = 16384
L = 150000


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _local_synthesis(so, coef_per_slice, part, L=L):
    """the rank's overlap-add over part.synthesis_window() from the oracle's
    per-slice inverses (un-rolled by +-H by slice parity)"""
    lo, hi = part.synthesis_window()
    out = np.zeros((1, hi - lo))
    for g in range(part.s0, part.s1):
        y = so.cqt.bwd(coef_per_slice[g])[0]
        y = np.roll(y, H if g % 2 == 0 else -H)
        p = 2 * H * (g - 1) + np.arange(4 * H)
        keep = (p >= 0) & (p < L) & (p >= lo) & (p < hi)
        out[0, p[keep] - lo] += y[keep]
    return out


def _worker(rank, world, port, q, L=L):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        import pathlib
        root = pathlib.Path(__file__).resolve().parents[1]
        sys.path.insert(0, str(root))
        sys.path.insert(0, str(root / "tests" / "golden"))
        from oracle.cqt_oracle import SlicedOracle
        from signals import chirp
        so = SlicedOracle()
        x = chirp(5, L)[None].astype(np.float64)
        S = so.num_slices(L)
        sl = so.slices(x)[0]                       # [S, 65536]
        coef = [[c[None] for c in so.cqt.fwd(sl[g][None])] for g in range(S)]
        coef = [[c[0] for c in cs] for cs in coef]
        part = Partition(L, S, rank, world)
        local = torch.from_numpy(_local_synthesis(so, coef, part, L))
        own = exchange_halo(local, part)
        lo, hi = part.owned()
        q.put((rank, lo, hi, own.numpy().copy()))
    finally:
        dist.destroy_process_group()


# (3, 30000) and (4, 30000): a 2-slice stream on more ranks than slices, so
# the trailing ranks own nothing and must not be waited for
@pytest.mark.parametrize("world,L", [(2, L), (3, L), (3, 30000), (4, 30000)])
def test_partitioned_overlap_add_equals_whole_buffer(world, L):
    from oracle.cqt_oracle import SlicedOracle
    from signals import chirp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, L)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    got.sort()
    y = np.concatenate([g[3] for g in got], axis=-1)
    assert [g[1] for g in got] == sorted(g[1] for g in got)
    assert got[0][1] == 0 and got[-1][2] == L
    so = SlicedOracle()
    x = chirp(5, L)[None].astype(np.float64)
    want = so.bwd(*so.fwd(x), length=L)
    np.testing.assert_allclose(y, want, rtol=0, atol=1e-9)


def test_slice_ranges_cover_and_balance():
    for S in (1, 5, 82, 83):
        for world in (1, 2, 4, 8):
            r = slice_ranges(S, world)
            assert r[0][0] == 0 and r[-1][1] == S
            assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
            n = [b - a for a, b in r]
            assert max(n) - min(n) <= 1


def _dropping_worker(rank, world, port, q):
    """rank 1 fails before the halo exchange (it never sends); rank 0 must
    get an error from its bounded wait, not hang"""
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    part = Partition(4 * 32768, 4, rank, world)
    lo, hi = part.synthesis_window()
    local = torch.zeros(2, hi - lo)
    try:
        if rank == 1:
            q.put((rank, "dropped"))
            return                      # leaves without sending its first hop
        try:
            exchange_halo(local, part)
            q.put((rank, "no error"))
        except Exception as e:          # the bounded wait gave up
            q.put((rank, type(e).__name__))
    finally:
        if rank == 0:
            dist.destroy_process_group()


def test_dropped_halo_times_out():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dropping_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert got[1] == "dropped"
    assert got[0] not in ("no error",), got
    assert all(p.exitcode is not None for p in procs)


def _agreement_worker(rank, world, port, q, fail_rank, fail_at, mode):
    """PartitionedSlicedCQT's peer-memory halo set-up with a stand-in for the
    CUDA IPC exchange: one rank's create or connect fails, and every rank must
    take the same transport (or all raise), with no collective left unmatched"""
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        import flash_cqt_b200.distributed as D

        class FakeHalo:
            def __init__(self, rows, hop, device, wait_ms=10000):
                if rank == fail_rank and fail_at == "create":
                    raise RuntimeError("no memory for the receive buffer")
                self.handle = bytes([rank]) * 64
                self.left = self.right = None

            def connect(self, left=None, right=None):
                if rank == fail_rank and fail_at == "connect":
                    raise RuntimeError("no peer access")
                self.left, self.right = left, right

        D.PeerHalo = FakeHalo
        part = D.PartitionedSlicedCQT(None, rank, world, halo=mode)
        p = D.Partition(6 * 32768, 6, rank, world)
        try:
            h = part._peer_halo(2, p, torch.device("cpu"))
            res = ("none" if h is None else "peer", part.halo,
                   None if h is None else (h.left, h.right))
        except RuntimeError:
            res = ("raised", part.halo, None)
        dist.barrier()   # every rank is still in step after the set-up
        q.put((rank,) + res)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fail_rank,fail_at,mode", [
    (None, None, "auto"), (1, "create", "auto"), (2, "connect", "auto"),
    (0, "connect", "peer")])
def test_peer_halo_setup_agrees(fail_rank, fail_at, mode):
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_agreement_worker,
                         args=(r, world, port, q, fail_rank, fail_at, mode))
             for r in range(world)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    outcomes = {g[1] for g in got}
    if fail_rank is None:
        assert outcomes == {"peer"} and all(g[2] == "auto" for g in got)
        for r, _, _, (left, right) in got:   # the neighbours' handles, where they exist
            assert left == (bytes([r - 1]) * 64 if r > 0 else None)
            assert right == (bytes([r + 1]) * 64 if r < world - 1 else None)
    elif mode == "auto":
        assert outcomes == {"none"} and all(g[2] == "collective" for g in got)
    else:
        assert outcomes == {"raised"}
