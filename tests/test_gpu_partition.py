"""The slice-range partitioned sliced transform on the GPU.

Ranks are emulated in one process on one GPU (the halo added by hand) and, when
two to four GPUs are present, run as NCCL processes with either halo transport
(this build's peer-memory kernels, or torch.distributed send / receive), over
several consecutive calls.  All must reproduce the whole-stream SlicedCQT bit
for bit: every slice is computed by the same kernel arithmetic, and every
output sample is the same two-term sum.  A send dropped on the host must make
the neighbour's bounded wait give up and be reported.
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

L = 300001          # 10 slices, ragged tail


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


def _signal(dev):
    g = torch.Generator(device="cpu").manual_seed(31)
    return torch.randn(2, 1, L, generator=g).to(dev)


@pytest.mark.parametrize("world", [1, 3, 4])
def test_emulated_ranks_match_whole_stream(dev, world):
    from flash_cqt_b200 import SlicedCQT
    from flash_cqt_b200.distributed import PartitionedSlicedCQT
    x = _signal(dev)
    sl = SlicedCQT([3, 4, 2], [8, 16, 32], fs=44100, sl_len=65536, device=dev)
    wb, ws = sl.fwd(x)
    y_whole = sl.bwd(wb, ws, length=L)
    parts = [PartitionedSlicedCQT(sl, r, world) for r in range(world)]
    locals_, owned = [], []
    for r, pc in enumerate(parts):
        p = pc.partition(L)
        # input window only (one hop of halo each side), not the whole signal
        a, b = p.input_window()
        a0, b0 = max(a, 0), min(b, L)
        blocks, side = pc.fwd(x[..., a0:b0], L, sample0=a0)
        for c, full, m in zip(blocks, wb, sl.size_per_oct):
            assert torch.equal(c, full[..., p.s0 * m:p.s1 * m])
        for c, full in zip(side, ws):
            assert torch.equal(c, full[:, :, p.s0:p.s1])
        se = sl._fused(dev)
        buf = sl._fused_buffer(se, blocks, side, 2, p.nslices)
        lo, hi = p.synthesis_window()
        locals_.append((p, se.synthesis(buf, 2, p.nslices, L, slice0=p.s0, sample0=lo,
                                        count=hi - lo)))
    # the halo: rank r + 1's first hop is added into rank r's last hop
    H2 = sl.hop
    for r in range(world - 1):
        locals_[r][1][:, -H2:] += locals_[r + 1][1][:, :H2]
    for p, loc in locals_:
        lo, hi = p.owned()
        start = lo - p.synthesis_window()[0]
        owned.append(loc[:, start:start + hi - lo])
    y = torch.cat(owned, dim=-1).view(2, 1, L)
    assert torch.equal(y, y_whole)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, q, halo="auto", steps=3, drop=False):
    """one rank of the partitioned stream under NCCL: `steps` fwd + bwd
    calls (the peer-memory halo's flags and acknowledgements advance one
    epoch per call); with `drop`, a last exchange in which rank 1 does not
    send, so rank 0's bounded wait must run out and be reported"""
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        from flash_cqt_b200 import SlicedCQT
        from flash_cqt_b200.distributed import PartitionedSlicedCQT
        dev = torch.device("cuda", rank)
        x = _signal(dev)
        sl = SlicedCQT([3, 4, 2], [8, 16, 32], fs=44100, sl_len=65536, device=dev)
        pc = PartitionedSlicedCQT(sl, rank, world, halo=halo, halo_wait_ms=1500)
        outs = []
        for _ in range(steps):
            blocks, side = pc.fwd(x, L)
            outs.append(pc.bwd(blocks, side, L).cpu().numpy())
        torch.cuda.synchronize()
        pc.check_halo()
        dropped = None
        if drop:
            h = next(iter(pc._peer.values()))
            p = pc.partition(L)
            lo, hi = p.synthesis_window()
            local = torch.zeros(2, hi - lo, device=dev)
            h.exchange(local, send=False, recv=rank == 0)   # rank 1 drops its hop
            torch.cuda.synchronize()
            try:
                pc.check_halo()
                dropped = "no error"
            except RuntimeError as e:
                dropped = "raised" if "gave up" in str(e) else repr(e)
            # the context is still usable after the expired wait
            xs = x[..., :70000].contiguous()
            assert torch.isfinite(sl.bwd(*sl.fwd(xs), length=70000)).all()
        lo, hi = pc.partition(L).owned()
        q.put((rank, lo, hi, outs, dropped))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _run_ranks(world, **kw):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, q), kwargs=kw)
             for r in range(world)]
    for p in procs:
        p.start()
    got = sorted((q.get(timeout=300) for _ in range(world)), key=lambda g: g[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return got


@pytest.mark.parametrize("halo", ["peer", "collective"])
@pytest.mark.parametrize("world", [2, 3, 4])
def test_nccl_ranks_match_whole_stream(dev, halo, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from flash_cqt_b200 import SlicedCQT
    got = _run_ranks(world, halo=halo, steps=3)
    sl = SlicedCQT([3, 4, 2], [8, 16, 32], fs=44100, sl_len=65536, device=dev)
    x = _signal(dev)
    want = sl.bwd(*sl.fwd(x), length=L).cpu().numpy()
    for step in range(3):
        y = np.concatenate([g[3][step] for g in got], axis=-1)
        np.testing.assert_array_equal(y, want)


def test_peer_halo_dropped_send_is_reported(dev):
    """rank 1 skips one send (a failure made on the host, between steps):
    rank 0's bounded wait gives up after 1.5 s, check_halo raises, and the
    context stays usable; nothing faults or hangs"""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    got = _run_ranks(2, halo="peer", steps=1, drop=True)
    assert got[0][4] == "raised", got[0][4]
    assert got[1][4] == "no error"


def test_unaligned_rows_and_offsets_agree_bitwise(dev):
    """Rows whose global sample 0 is not 8-byte aligned (odd sample0, odd row
    stride, odd element offset) take the scalar loads and single-lane atomics;
    aligned rows take float2 loads and two-lane atomics.  Both must give the
    same bits for the same slices."""
    from flash_cqt_b200 import SlicedCQT
    sl = SlicedCQT([3, 4, 2], [8, 16, 32], fs=44100, sl_len=65536, device=dev)
    se = sl._fused(dev)
    H2 = sl.hop
    x = _signal(dev).view(2, L)
    S = se.count(L)
    ref = se.analysis(x, S)
    rb, rs = se.group_views(ref, (2,), S)
    s0, n = 3, 4
    a, b = H2 * (s0 - 1) - 1, H2 * (s0 + n + 1) + 1      # odd first sample
    ld = (b - a) + 3                                       # odd row stride
    store = torch.zeros(2 * ld + 4, device=dev)
    xw = store[1:1 + 2 * ld].view(2, ld)[:, :b - a]        # row 0 misaligned, row 1 not
    xw.copy_(x[:, a:b])
    buf = se.analysis(xw, n, slice0=s0, sample0=a, length=L)
    bb, bs = se.group_views(buf, (2,), n)
    for c, full, m in zip(bb, rb, sl.size_per_oct):
        assert torch.equal(c, full[..., s0 * m:(s0 + n) * m])
    for c, full in zip(bs, rs):
        assert torch.equal(c, full[:, s0:s0 + n])
    # synthesis and the windowed adjoint into aligned and misaligned rows
    lo, hi = H2 * (s0 - 1), H2 * (s0 + n)
    for adj in (False, True):
        ya = se.synthesis(buf, 2, n, L, slice0=s0, sample0=lo, count=hi - lo,
                          adjoint_of_analysis=adj)
        outs = torch.full((2 * ld + 4,), 7.0, device=dev)
        yu = outs[1:1 + 2 * ld].view(2, ld)[:, :hi - lo + 2]
        se.synthesis(buf, 2, n, L, out=yu, slice0=s0, sample0=lo - 1,
                     count=hi - lo + 2, adjoint_of_analysis=adj)
        assert torch.equal(yu[:, 1:1 + hi - lo], ya)
        assert torch.all(yu[:, 0] == 0) and torch.all(yu[:, -1] == 0)
