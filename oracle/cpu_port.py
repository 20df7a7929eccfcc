"""CPU baseline port of the reference transform -- TEST / BENCH INFRASTRUCTURE.

The reference path is Python (torch CPU ops), so it cannot be compiled into
``oracle/_ref`` and it does not travel to the GPU box; this module restates its
exact op sequence in torch float32 on the host cores, which is what
``bench.py``'s CPU baseline and ``--impl reference`` arm time:

* analysis  ``oct_cqt.py:84-96``:  one ``rfft``; per group a gather x window
  and one ``ifft``; the side groups gather with the conjugation mask;
* synthesis ``oct_cqt.py:98-117``: per group ``fft`` x dual window; one flat
  ``index_add_`` into the half spectrum; one ``irfft``.

The layout (gather indices, windows, scatter positions, duals) comes from
``oracle.cqt_oracle.OctCQTOracle``, whose float64 values are rounded to
float32 once, as the reference stores them.
"""
import os

import numpy as np
import torch

from .cqt_oracle import OctCQTOracle


class CPUPort:
    def __init__(self, threads=None):
        self.threads = int(threads or os.cpu_count() or 1)
        torch.set_num_threads(self.threads)
        o = OctCQTOracle()
        self.nn = o.nn
        self.groups = []
        for idx, gv, pos, gdv, conj in o.all_groups:
            self.groups.append((torch.from_numpy(idx), torch.from_numpy(gv).float(),
                                torch.from_numpy(pos), torch.from_numpy(gdv).float(),
                                torch.from_numpy(conj)))
        self.pos_flat = torch.cat([g[2].reshape(-1) for g in self.groups])

    @torch.no_grad()
    def fwd(self, x):
        ft = torch.fft.rfft(x)
        out = []
        for idx, gv, pos, gdv, conj in self.groups:
            a = ft[..., idx]
            if bool(conj.any()):
                a = torch.where(conj, a.conj(), a)
            out.append(torch.fft.ifft(a * gv))
        return out

    @torch.no_grad()
    def bwd(self, blocks):
        B = blocks[0].shape[0]
        src = torch.cat([(torch.fft.fft(c) * g[3]).reshape(B, -1)
                         for c, g in zip(blocks, self.groups)], dim=-1)
        fr = torch.zeros(B, self.nn // 2 + 1, dtype=src.dtype)
        torch.view_as_real(fr).index_add_(1, self.pos_flat, torch.view_as_real(src))
        return torch.fft.irfft(fr, n=self.nn)

    def round_trip(self, x):
        return self.bwd(self.fwd(x))


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def time_round_trips(batch=16, seconds=10.0, threads=None, warmup=2):
    """Median round trips/s of the CPU port over ~`seconds` of work."""
    import time
    port = CPUPort(threads)
    g = torch.Generator().manual_seed(4)
    x = torch.randn(batch, port.nn, generator=g)
    for _ in range(warmup):
        port.round_trip(x)
    ts = []
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end or len(ts) < 3:
        t0 = time.perf_counter()
        y = port.round_trip(x)
        ts.append(time.perf_counter() - t0)
    err = float(((y.double() - x.double()) ** 2).sum() / (x.double() ** 2).sum())
    ts.sort()
    med = ts[len(ts) // 2]
    return {"round_trips_per_s": batch / med, "ms_per_call": 1e3 * med,
            "batch": batch, "calls": len(ts), "threads": port.threads,
            "snr_db": float(-10 * np.log10(err)), "cpu": cpu_model()}
