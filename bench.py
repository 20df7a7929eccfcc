#!/usr/bin/env python
"""Benchmark: 65536-sample CQT round trips/s on 1..8 B200 (+ train step ms).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B]
    python bench.py --impl reference ...      # the reference's own CPU path

One step = one analysis + synthesis round trip of B slices per GPU (default
1024, inputs larger than L2) through the sm_100a engines, replayed as one CUDA
graph.  Under torchrun every rank runs its own batch (weak scaling, no
collective on the data path); the time is the max over ranks.  Rank 0 prints
one JSON line.
"""
import argparse
import json
import math
import os
import pathlib
import statistics
import subprocess
import sys
import threading
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N = 65536
METRIC = "65536-sample CQT round trips/s"
# algorithmic bytes per slice (x in, coefficients out, coefficients in, y out)
RT_BYTES = 262144 + 1063936 + 1063936 + 262144
# train step per sample: round trip + target in + y re-read + coefficient
# gradients out and in + dL/dx out
TRAIN_BYTES = RT_BYTES + 262144 + 262144 + 1063936 + 1063936 + 262144


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1024, help="slices per GPU per step")
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the batch sweep, train step, e2e and CPU baseline")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--halo", choices=["auto", "peer", "collective"], default="auto",
                    help="transport of the config-5 overlap-add halo at N > 1: this build's "
                         "peer-memory kernels, torch.distributed send / receive, or auto "
                         "(peer memory under NCCL)")
    ap.add_argument("--reference-gpu-only", action="store_true",
                    help="run only the same-box GPU baseline of the reference's own "
                         "kernels and print it")
    ap.add_argument("--train-only", action="store_true",
                    help="run only the B = 16 train step measurements and print them "
                         "(for profiling its launches)")
    ap.add_argument("--sliced-only", action="store_true",
                    help="run only the config-5 long-stream measurement and print its "
                         "result (for profiling the sliced kernels)")
    return ap.parse_args()


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples (every 20 ms) of SM clock and throttle reasons,
    read on a thread as they arrive.  Entering waits (up to 3 s) for the first
    sample, so a short timed region still has samples: the first is taken
    right before it, with the GPU still at load clocks from the warm-up."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []
        self._first = threading.Event()

    def _read(self):
        for ln in self.proc.stdout:
            if ln.strip():
                self.lines.append(ln)
                self._first.set()

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self
        self._thread = threading.Thread(target=self._read, daemon=True)
        self._thread.start()
        self._first.wait(timeout=3.0)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.03)   # one more sample at the end of the region
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait()
            self._thread.join(timeout=5)

    def summary(self):
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                 "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            p = [s.strip() for s in ln.split(",")]
            if len(p) < 7:
                continue
            try:
                sm.append(float(p[0]))
                smax = float(p[1])
            except ValueError:
                continue
            for nm, v in zip(names, p[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------- reference arm
REF_ARM_SECONDS = 150.0   # bound on the whole --impl reference run


def reference_round_trip():
    """(round_trip(x), describe) of the reference's own CPU path: the unmodified
    ``OctCQT.fwd`` -> ``.bwd`` (oct_cqt.py:84-117) imported from the build in
    oracle/_ref when present, else the torch restatement in oracle/cpu_port.py"""
    import torch
    from oracle import ref_loader
    from oracle.cpu_port import cpu_model
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    if ref_loader.available():
        fc = ref_loader.package()
        cqt = fc.OctCQT([3, 4, 2], [8, 16, 32], fs=44100, audio_len=N)

        @torch.no_grad()
        def rt(x):
            return cqt.bwd(*cqt.fwd(x))
        return rt, "reference", threads, ("the reference's unmodified OctCQT.fwd -> .bwd "
                                          "(byte-compiled from its sources, oracle/build_ref.py) "
                                          f"on {cpu_model()}")
    from oracle.cpu_port import CPUPort
    port = CPUPort(threads)
    return port.round_trip, "port", threads, ("torch CPU float32 restatement of "
                                              f"OctCQT.fwd/bwd (oracle/cpu_port.py) on {cpu_model()}")


def run_reference(args, rank):
    if rank != 0:
        return
    import torch
    rt, kind, cores, what = reference_round_trip()
    g = torch.Generator().manual_seed(4)
    # per-slice cost from a small warm-up, then the largest per-step batch (up
    # to the GPU arm's) that keeps the whole run inside REF_ARM_SECONDS
    probe = torch.randn(16, N, generator=g)
    rt(probe)
    t0 = time.perf_counter()
    rt(probe)
    per_slice = (time.perf_counter() - t0) / 16
    B = args.batch
    budget = REF_ARM_SECONDS / max(1, args.steps + args.warmup)
    while B > 16 and B * per_slice > budget:
        B //= 2
    x = torch.randn(B, N, generator=g)
    for _ in range(max(args.warmup, 1)):
        rt(x)
    ts = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        y = rt(x)
        ts.append(time.perf_counter() - t0)
    err = float(((y.double() - x.double()) ** 2).sum() / (x.double() ** 2).sum())
    tot = sum(ts)
    value = B * args.steps / tot
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "round_trips/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * tot / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "FusedOctCQT round trip (analysis + synthesis), "
                               "OctCQT([3,4,2],[8,16,32]) fs 44100, 65536-sample N(0,1) "
                               "slices (config 4)",
                   "global_batch": B, "per_gpu_batch": args.batch if B == args.batch else B,
                   "seq_len": N, "parallelism": "cpu, rank 0 only",
                   "same_batch_as_gpu_arm": B == args.batch,
                   "note": "per-step batch lowered only to keep the run within "
                           f"{REF_ARM_SECONDS:.0f} s; per-slice CPU throughput is flat "
                           "above ~64 slices"},
        "round_trip_snr_db": -10 * math.log10(err),
        "cpu_baseline": {"value": value, "unit": "round_trips/s", "cores": cores,
                         "kind": kind,
                         "sample": f"{args.steps} round trips of {B} slices, {what}"},
        "e2e": {"value": value, "unit": "round_trips/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline(seconds):
    """the reference's CPU path timed on the host for ~`seconds` (bounded
    sample: 64-slice round trips) -- the cpu_baseline object of the GPU arm"""
    import torch
    rt, kind, cores, what = reference_round_trip()
    B = 64
    x = torch.randn(B, N, generator=torch.Generator().manual_seed(4))
    rt(x)
    calls, t0 = 0, time.perf_counter()
    while True:
        y = rt(x)
        calls += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    err = float(((y.double() - x.double()) ** 2).sum() / (x.double() ** 2).sum())
    return {"value": B * calls / el, "unit": "round_trips/s", "cores": cores, "kind": kind,
            "sample": "%d calls of a %d-slice round trip (%.0f s), %s, %.1f dB"
                      % (calls, B, el, what, -10 * math.log10(err))}


def cpu_configs():
    """configs 1, 3 and 5 through the reference's own CPU code (the package
    built from its sources in oracle/_ref), on all host cores: medians after
    warm-ups, with the GPU rows' seeds (config 5's noise comes from the CPU
    generator, the GPU row's from the CUDA one).  None when the reference is
    not built here."""
    import statistics
    import torch
    from oracle import ref_loader
    from oracle.cpu_port import cpu_model
    if not ref_loader.available():
        return None
    fc = ref_loader.package()
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)

    def median_ms(fn, warm, reps):
        for _ in range(warm):
            fn()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return 1e3 * statistics.median(ts)

    def snr(a, b):
        a, b = a.double(), b.double()
        return float(10 * torch.log10((a ** 2).sum() / ((b - a) ** 2).sum()))

    out = {"kind": "reference", "cores": threads, "cpu": cpu_model(),
           "what": "the reference's unmodified OctCQT / SlicedCQT (oracle/build_ref.py)"}
    cqt = fc.OctCQT([3, 4, 2], [8, 16, 32], fs=44100, audio_len=N)
    # config 1: 4 slices of N(0, 1), seed 0, fwd -> bwd
    x1 = torch.randn(4, N, generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        ms1 = median_ms(lambda: cqt.bwd(*cqt.fwd(x1)), 2, 10)
        y1 = cqt.bwd(*cqt.fwd(x1))
    out["config1_b4_round_trip"] = {"ms": ms1, "snr_db": snr(x1, y1), "runs": "median of 10"}
    # config 3: B = 16 train step through torch autograd on OctCQT
    x3 = torch.randn(16, N, generator=torch.Generator().manual_seed(2))
    t3 = torch.randn(16, N, generator=torch.Generator().manual_seed(3))

    def step():
        xg = x3.detach().requires_grad_(True)
        ((cqt.bwd(*cqt.fwd(xg)) - t3) ** 2).mean().backward()
    out["config3_train_step_b16"] = {"ms": median_ms(step, 2, 10), "runs": "median of 10"}
    # config 5: SlicedCQT fwd + bwd on 8 x 60 s of chirp + noise
    sl = fc.SlicedCQT([3, 4, 2], [8, 16, 32], fs=44100, sl_len=N, device="cpu")
    tt = torch.arange(SLICED_LEN, dtype=torch.float64) / 44100.0
    k = math.log(18000.0 / 40.0) / 60.0
    phase = 2 * math.pi * 40.0 * (torch.exp(k * tt) - 1.0) / k
    x5 = (torch.sin(phase).float().expand(SLICED_SIGNALS, SLICED_LEN)
          + 0.05 * torch.randn(SLICED_SIGNALS, SLICED_LEN,
                               generator=torch.Generator().manual_seed(5)))
    x5 = x5.reshape(SLICED_SIGNALS, 1, SLICED_LEN).contiguous()
    with torch.no_grad():
        ms5 = median_ms(lambda: sl.bwd(*sl.fwd(x5), length=SLICED_LEN), 1, 3)
        y5 = sl.bwd(*sl.fwd(x5), length=SLICED_LEN)
    out["config5_sliced_stream"] = {"ms": ms5, "snr_db": snr(x5, y5), "runs": "median of 3",
                                    "signals": SLICED_SIGNALS, "samples": SLICED_LEN}
    return out


def reference_gpu(dev, batches=(1, 64, 256, 1024), reps=20):
    """Same-box GPU baseline of the reference's own CUDA kernels (built from
    its sources for sm_100a by oracle/build_ref.py): its TrainableCQT factored
    round trip (fft3 + radix bands, trainable.py:75-109) under CUDA-graph
    replay, and its factored resident pair (persist2.cu fwd2 + inv2, one
    cooperative launch per direction, driven as bench/resident2.py does).
    Reported beside this build's own graphed round trip; never part of the
    timed product path."""
    import torch
    from oracle import ref_loader
    if not ref_loader.available(cuda=True):
        return {"unavailable": "reference not built here (python oracle/build_ref.py)"}
    fc = ref_loader.package(cuda=True)
    from flash_cqt.trainable import TrainableCQT as RefTrainable
    import flash_cqt.fused as rfused
    cqt = fc.OctCQT([3, 4, 2], [8, 16, 32], fs=44100, audio_len=N, device=dev)
    rt_ = RefTrainable(cqt, dev)
    f, rx = rt_.f, rt_.f.radix
    p2 = rfused._P2EXT
    w32r, w32i = rt_.FR[1].contiguous(), rt_.FI[1].contiguous()
    out = {}

    def graphed(fn):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):
                fn()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            res = fn()
        return g, res

    def timed(run):
        for _ in range(3):
            run()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            run()
        b.record()
        b.synchronize()
        return a.elapsed_time(b) / reps

    def snr(x, y):
        return float(10 * torch.log10((x.double() ** 2).sum() / ((y.double() - x.double()) ** 2).sum()))

    for B in batches:
        x = torch.randn(B, N, device=dev, generator=torch.Generator(device=dev).manual_seed(4))
        with torch.no_grad():
            g, y = graphed(lambda: rt_._synthesis(*rt_._analysis(x)))
            ms_f = timed(g.replay)
            s_f = snr(x, y)
            del g
            w = f._workspace(B)
            pl = [torch.empty(B, N // 2, device=dev) for _ in range(4)]
            args = (x, w["KR"], w["KI"], w["FR"], w["FI"], w["XO"], *pl, w32r, w32i,
                    rt_.WLR, rt_.WLI, rt_.WKR, rt_.WKI, rt_.WNR, rt_.WNI,
                    rx["desc"], rx["route"], rx["gdv"], rx["pos"], rx["rr"], rx["ri"],
                    f.ncoef, B)

            def resident():
                p2.fwd2(*args)
                p2.inv2(*args)
            ms_r = timed(resident)
            s_r = snr(x, w["XO"])
        out[str(B)] = {"trainable_factored_graphed": {"ms": ms_f, "round_trips_per_s": B / (ms_f / 1e3),
                                                       "snr_db": s_f},
                       "resident_pair_persist2": {"ms": ms_r, "round_trips_per_s": B / (ms_r / 1e3),
                                                  "snr_db": s_r}}
        del w, pl, args
        f._ws.clear()
        rt_.scr.clear()
        torch.cuda.empty_cache()
    out["what"] = ("the reference's own kernels (packedfft.cu, radix.cu, persist2.cu) "
                   "built for sm_100a from its sources, run on this GPU")
    return out


# -------------------------------------------------------------------- b200
def load_traffic():
    p = ROOT / "profiles" / "ncu_traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except ValueError:
            return None
    return None


def main():
    args = parse()
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta
        if args.impl == "b200":
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                    device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo", timeout=timedelta(seconds=300))
        if rank == 0:
            print(f"process group: backend {dist.get_backend()}, "
                  f"{dist.get_world_size()} ranks", file=sys.stderr, flush=True)
    if args.impl == "reference":
        run_reference(args, rank)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return

    import numpy as np
    from flash_cqt_b200 import FusedOctCQT, Graphed, OctCQT, TrainableCQT
    from flash_cqt_b200 import _native

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if args.reference_gpu_only:
        if rank == 0:
            print(json.dumps({"reference_gpu": reference_gpu(dev)}), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.train_only:
        pk = ROOT / "MEASURED_PEAKS.json"
        hbm = (json.loads(pk.read_text()).get("hbm_gbs") if pk.exists() else None) or 6650.0
        cqt = OctCQT([3, 4, 2], [8, 16, 32], fs=44100, audio_len=N, device=dev)
        r = train_step(TrainableCQT(cqt, dev), dev, max(args.warmup, 3), args.steps, hbm)
        if rank == 0:
            print(json.dumps(r), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.sliced_only:
        pk = ROOT / "MEASURED_PEAKS.json"
        hbm = (json.loads(pk.read_text()).get("hbm_gbs") if pk.exists() else None) or 6650.0
        r = sliced_stream(dev, world, rank, max(args.warmup, 3), args.steps, hbm, args.halo)
        if rank == 0:
            print(json.dumps({"sliced_stream": r}), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    B = args.batch
    W = max(args.warmup, 3)
    K = args.steps
    cqt = OctCQT([3, 4, 2], [8, 16, 32], fs=44100, audio_len=N, device=dev)
    t = TrainableCQT(cqt, dev)
    eng = t.eng
    g = torch.Generator(device=dev).manual_seed(4 + rank)
    x = torch.randn(B, N, device=dev, generator=g)
    coef = torch.empty(B, eng.ncoef, dtype=torch.complex64, device=dev)
    y = torch.empty(B, N, device=dev)

    def round_trip():
        eng.analysis(x, out=coef)
        eng.synthesis(coef, out=y)

    # correctness guard on the benchmarked buffers
    round_trip()
    torch.cuda.synchronize()
    err = ((y.double() - x.double()) ** 2).sum() / (x.double() ** 2).sum()
    rt_db = float(-10 * torch.log10(err))

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(W):
            round_trip()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        round_trip()
    for _ in range(W):
        graph.replay()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with ClockSampler(local) as clk:
        ev0.record()
        for _ in range(K):
            graph.replay()
        ev1.record()
        barrier()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        tt = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    ms_step = ms / K
    value = world * B * K / (ms / 1e3)

    # ---- per-kernel CUDA-event timing (eager launches of each stage)
    stream = torch.cuda.current_stream()
    ws = eng.workspace(B)
    sp = int(stream.cuda_stream)
    names = ["spectrum_fwd", "bands_fwd", "bands_inv", "spectrum_inv"]
    kev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in range(4)] for _ in range(K)]

    def stage(s):
        eng.tables.stage(s, x.data_ptr(), y.data_ptr(), coef.data_ptr(), None,
                         _native.CQT_LAYOUT_COMPLEX, B, ws.data_ptr(), ws.numel(), sp)

    for _ in range(W):
        for s in range(4):
            stage(s)
    torch.cuda.synchronize()
    for k in range(K):
        for s in range(4):
            kev[k][s][0].record()
            stage(s)
            kev[k][s][1].record()
    torch.cuda.synchronize()
    kms = [statistics.mean(kev[k][s][0].elapsed_time(kev[k][s][1]) for k in range(K))
           for s in range(4)]
    tabs = eng.host_tables
    live_syn = int((tabs["inv"]["synth"][0] >= 0).sum())
    spec_bytes = 32769 * 8
    kbytes = [262144 + spec_bytes, spec_bytes + 1063936,
              1063936 + live_syn * 8, live_syn * 8 + 262144]
    dom = max(range(4), key=lambda i: kms[i])
    peaks = {}
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        peaks = json.loads(pk.read_text())
    hbm = peaks.get("hbm_gbs")
    peak_src = "measured" if hbm else "fallback"
    hbm = hbm or 6650.0
    ach = kbytes[dom] * B / (kms[dom] / 1e3) / 1e9
    traffic = None
    tr = load_traffic()
    if tr and names[dom] in tr.get("dram_bytes_per_slice", {}):
        traffic = tr["dram_bytes_per_slice"][names[dom]] * B
    roofline = {"bound": "hbm", "kernel": names[dom], "achieved": ach, "peak": hbm,
                "unit": "GB/s", "frac": ach / hbm, "traffic": traffic,
                "peak_source": peak_src,
                "algorithmic_bytes_per_launch": kbytes[dom] * B}
    rt_ach = RT_BYTES * B / (ms_step / 1e3) / 1e9
    pipeline = {"achieved": rt_ach, "peak": hbm, "unit": "GB/s", "frac": rt_ach / hbm,
                "algorithmic_bytes_per_step": RT_BYTES * B}
    kernels = {nm: {"ms": kms[i], "share": kms[i] / sum(kms),
                    "algorithmic_gbs": kbytes[i] * B / (kms[i] / 1e3) / 1e9}
               for i, nm in enumerate(names)}

    line = {
        "metric": METRIC, "value": value, "unit": "round_trips/s", "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "FusedOctCQT round trip (analysis + synthesis), "
                               "OctCQT([3,4,2],[8,16,32]) fs 44100, 65536-sample "
                               "N(0,1) slices, CUDA-graph replay (config 4)",
                   "global_batch": B * world, "per_gpu_batch": B, "seq_len": N,
                   "parallelism": f"batch-sharded x{world}, no communication",
                   "l2": "inputs larger than L2 (x %d MiB, coefficients %d MiB per GPU)"
                         % (B * N * 4 >> 20, B * eng.ncoef * 8 >> 20)},
        "round_trip_snr_db": rt_db,
        "comm": ({"backend": dist.get_backend(), "nranks": dist.get_world_size(),
                  "data_path_collectives": 0,
                  "note": "one NCCL communicator of all ranks; used only for the barrier "
                          "and the max-over-ranks timing reduction"}
                 if world > 1 else {"backend": None, "nranks": 1}),
        "gpu_launches": 4 * K,
        "roofline": roofline,
        "pipeline_roofline": pipeline,
        "kernels": kernels,
        "clocks": clk.summary(),
    }

    if not args.no_extras:
        line.update(extras(args, eng, t, dev, world, rank, barrier, W, K, hbm))
        if world == 1 and rank == 0:
            line["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
            cfg = cpu_configs()
            if cfg is not None:
                line["cpu_baseline"]["configs"] = cfg
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# config 5: 8 signals x 60 s at 44.1 kHz, slices range-partitioned over ranks
SLICED_SIGNALS = 8
SLICED_LEN = 2646000
# algorithmic bytes per signal: input + 82 slices x coefficients w + r + output
SLICED_BYTES = 10584000 + 82 * 2127872 + 10584000


def sliced_stream(dev, world, rank, W, K, hbm, halo="auto"):
    """SlicedCQT fwd + bwd (fused kernels) on the config-5 stream; at N > 1
    the slices are range-partitioned and only the overlap-add halo crosses
    NVLink.  Strong scaling: the whole stream is fixed, time is max over ranks."""
    import math
    import torch
    import torch.distributed as dist
    from flash_cqt_b200 import SlicedCQT
    from flash_cqt_b200.distributed import PartitionedSlicedCQT
    sl = SlicedCQT([3, 4, 2], [8, 16, 32], fs=44100, sl_len=65536, device=dev)
    # seeded log sweep 40 Hz -> 18 kHz over 60 s plus N(0, 0.05^2) noise
    tt = torch.arange(SLICED_LEN, device=dev, dtype=torch.float64) / 44100.0
    k = math.log(18000.0 / 40.0) / 60.0
    phase = 2 * math.pi * 40.0 * (torch.exp(k * tt) - 1.0) / k
    g = torch.Generator(device=dev).manual_seed(5)
    x = (torch.sin(phase).float().expand(SLICED_SIGNALS, SLICED_LEN)
         + 0.05 * torch.randn(SLICED_SIGNALS, SLICED_LEN, device=dev, generator=g))
    x = x.reshape(SLICED_SIGNALS, 1, SLICED_LEN).contiguous()
    pc = PartitionedSlicedCQT(sl, rank, world, halo=halo)

    def step():
        if world == 1:
            b, s_ = sl.fwd(x)
            return sl.bwd(b, s_, length=SLICED_LEN)
        b, s_ = pc.fwd(x, SLICED_LEN)
        return pc.bwd(b, s_, SLICED_LEN)

    y = step()
    torch.cuda.synchronize()
    lo, hi = pc.partition(SLICED_LEN).owned()
    ref = x[..., lo:hi].double() if world > 1 else x.double()
    snr = float(10 * torch.log10((ref ** 2).sum() / ((y.double() - ref) ** 2).sum()))
    for _ in range(W):
        step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(3, min(K, 20))
    e0.record()
    for _ in range(reps):
        step()
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / reps
    if world > 1:
        pc.check_halo()   # raises if a bounded wait on a neighbour gave up
        tt_ = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tt_, op=dist.ReduceOp.MAX)
        ms = float(tt_.item())
    gbs = SLICED_SIGNALS * SLICED_BYTES / (ms / 1e3) / 1e9
    return {"workload": "SlicedCQT fwd + bwd, 8 x 2,646,000-sample chirp + noise, 82 "
                        "slices per signal, fused sliced kernels, slices range-partitioned "
                        "over ranks with an NVLink overlap-add halo (strong scaling)",
            "ms_per_step": ms, "signals_per_s": SLICED_SIGNALS / (ms / 1e3),
            "slices_per_s": SLICED_SIGNALS * 82 / (ms / 1e3),
            "achieved_gbs": gbs, "frac_of_hbm": gbs / (hbm * world),
            "snr_db": snr, "scaling": "strong", "n_gpus": world,
            "halo": ("this build's peer-memory kernels (CUDA IPC, plain NVLink stores, "
                     "flag + acknowledgement, bounded waits)" if world > 1 and pc._use_peer(y)
                     else "torch.distributed send / receive" if world > 1 else None)}


def slice32k_round_trip(dev, hbm, B=2048, reps=10):
    """round trips/s of 32768-sample slices (default bank), graph replay,
    B slices per step; algorithmic bytes per slice: x in, coefficients out
    and in, y out"""
    import torch
    from flash_cqt_b200 import OctCQT, TrainableCQT
    n = 32768
    e32 = TrainableCQT(OctCQT([3, 4, 2], [8, 16, 32], fs=44100, audio_len=n, device=dev),
                       dev).eng
    xs = torch.randn(B, n, device=dev, generator=torch.Generator(device=dev).manual_seed(6))
    cs = torch.empty(B, e32.ncoef, dtype=torch.complex64, device=dev)
    ys = torch.empty(B, n, device=dev)

    def rt():
        e32.analysis(xs, out=cs)
        e32.synthesis(cs, out=ys)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            rt()
    torch.cuda.current_stream().wait_stream(s)
    gg = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gg):
        rt()
    for _ in range(3):
        gg.replay()
    ts = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        gg.replay()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b))
    med = statistics.median(ts)
    err = float(((ys.double() - xs.double()) ** 2).sum() / (xs.double() ** 2).sum())
    per_slice = 2 * n * 4 + 2 * e32.ncoef * 8
    gbs = B * per_slice / (med / 1e3) / 1e9
    del gg
    return {"batch": B, "ms": med, "round_trips_per_s": B / (med / 1e3),
            "algorithmic_bytes_per_slice": per_slice, "achieved_gbs": gbs,
            "frac_of_hbm": gbs / hbm, "round_trip_snr_db": -10 * math.log10(err)}


def extras(args, eng, t, dev, world, rank, barrier, W, K, hbm=6549.1):
    """e2e through the public API, the batch sweep, the train step and the
    sliced stream."""
    import torch
    from flash_cqt_b200 import FusedOctCQT, Graphed, HostPipeline
    out = {}
    out["sliced_stream"] = sliced_stream(dev, world, rank, W, K, hbm, args.halo)
    B = args.batch
    # ---- e2e through the public host API: pinned host x -> HostPipeline
    # (H2D, graphed FusedOctCQT fwd -> bwd, D2H, overlapped chunk by chunk)
    # -> pinned host y; every copy inside the timed region
    f = FusedOctCQT(t.cqt, dev)
    xh = torch.randn(B, N).pin_memory()
    yh = torch.empty(B, N).pin_memory()
    pipe = HostPipeline(lambda inp: f.bwd(*f.fwd(inp)), chunk=128, device=dev)
    for _ in range(W):
        pipe(xh, yh, sync=False)
    pipe.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K):
        pipe(xh, yh, sync=False)
    pipe.join()
    e1.record()
    barrier()
    ms = e0.elapsed_time(e1)
    if world > 1:
        import torch.distributed as dist
        tt = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    err = float(((yh.double() - xh.double()) ** 2).sum() / (xh.double() ** 2).sum())
    out["e2e"] = {"value": world * B * K / (ms / 1e3), "unit": "round_trips/s",
                  "h2d_bytes_per_step": B * N * 4, "d2h_bytes_per_step": B * N * 4,
                  "api": "HostPipeline(FusedOctCQT.fwd -> .bwd, chunk 128) with pinned host x / y",
                  "round_trip_snr_db": -10 * math.log10(err)}
    del pipe
    # the same without overlap: one H2D, one graphed round trip, one D2H per step
    xd = torch.empty(B, N, device=dev)
    gr = Graphed(lambda inp: f.bwd(*f.fwd(inp)), xd)
    xin = gr.static_inputs[0]
    for _ in range(W):
        xin.copy_(xh, non_blocking=True)
        yh.copy_(gr.run(), non_blocking=True)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K):
        xin.copy_(xh, non_blocking=True)
        yh.copy_(gr.run(), non_blocking=True)
    e1.record()
    barrier()
    ms = e0.elapsed_time(e1)
    if world > 1:
        import torch.distributed as dist
        tt = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    out["e2e_unpipelined"] = {"value": world * B * K / (ms / 1e3), "unit": "round_trips/s",
                              "api": "Graphed(FusedOctCQT.fwd -> .bwd), copies not overlapped"}
    del gr, f
    # ---- batch sweep (config 2 is B = 1), graphed, per GPU
    sweep = {}
    for Bs in (1, 4, 16, 64, 256, 1024):
        xs = torch.randn(Bs, N, device=dev)
        cs = torch.empty(Bs, eng.ncoef, dtype=torch.complex64, device=dev)
        ys = torch.empty(Bs, N, device=dev)

        def rt():
            eng.analysis(xs, out=cs)
            eng.synthesis(cs, out=ys)

        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):
                rt()
        torch.cuda.current_stream().wait_stream(s)
        gg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gg):
            rt()
        reps = 50 if Bs <= 64 else 10
        ts = []
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            gg.replay()
            b.record()
            b.synchronize()
            ts.append(a.elapsed_time(b))
        med = statistics.median(ts)
        sweep[str(Bs)] = {"ms": med, "round_trips_per_s": Bs / (med / 1e3)}
        del gg
    out["sweep_per_gpu"] = sweep
    # 32768-sample slices (the same engines, 8192-point spectrum CTAs): 2048
    # slices per step move the bytes of the 1024-slice headline step
    out["slice_32768"] = slice32k_round_trip(dev, hbm)
    # same-box GPU baseline: the reference's own factored kernels and its
    # resident pair, built from its sources (oracle/build_ref.py)
    if world == 1:
        try:
            rg = reference_gpu(dev)
        except Exception as e:   # a missing build or a failure here must not hide the run
            rg = {"unavailable": f"{type(e).__name__}: {e}"}
        for Bs, r in list(rg.items()):
            if isinstance(r, dict) and Bs in sweep:
                best = max(v["round_trips_per_s"] for v in r.values())
                r["this_build_round_trips_per_s"] = sweep[Bs]["round_trips_per_s"]
                r["this_build_over_best_reference"] = sweep[Bs]["round_trips_per_s"] / best
        out["reference_gpu"] = rg
    # ---- config 2: one slice of 8 seeded sinusoids (log-uniform 43 Hz - 20 kHz,
    # amplitudes U(0.1, 1), phases U(0, 2 pi)) + N(0, 0.01^2) noise, graphed
    # round trip and its reconstruction SNR
    g1 = torch.Generator().manual_seed(1)
    fr = torch.exp(torch.empty(8, dtype=torch.float64).uniform_(math.log(43.0),
                                                                 math.log(20000.0),
                                                                 generator=g1))
    am = torch.empty(8, dtype=torch.float64).uniform_(0.1, 1.0, generator=g1)
    ph = torch.empty(8, dtype=torch.float64).uniform_(0.0, 2 * math.pi, generator=g1)
    tt = torch.arange(N, dtype=torch.float64) / 44100.0
    x1 = (am[:, None] * torch.sin(2 * math.pi * fr[:, None] * tt + ph[:, None])).sum(0)
    x1 = x1 + 0.01 * torch.randn(N, dtype=torch.float64, generator=g1)
    x1 = x1.float().view(1, N).to(dev)
    c1 = torch.empty(1, eng.ncoef, dtype=torch.complex64, device=dev)
    y1 = torch.empty(1, N, device=dev)

    def rt1():
        eng.analysis(x1, out=c1)
        eng.synthesis(c1, out=y1)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            rt1()
    torch.cuda.current_stream().wait_stream(s)
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2):
        rt1()
    ts = []
    for _ in range(50):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g2.replay()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b))
    xd, yd = x1.double(), y1.double()
    out["config2_b1_sinusoids"] = {
        "ms": statistics.median(ts),
        "snr_db": float(10 * torch.log10((xd ** 2).sum() / ((yd - xd) ** 2).sum())),
        "input": "8 seeded sinusoids + N(0, 0.01^2), seed 1, graph replay"}
    del g2
    out.update(train_step(t, dev, W, K, hbm))
    return out


def train_step(t, dev, W, K, hbm):
    """config 3: B = 16 train step (analysis -> synthesis -> MSE vs a seeded
    target -> backward), eager as the reference writes it, with the loss
    folded into the engines, and the latter's device time under graph replay"""
    import torch
    out = {}
    Bt = 16
    gx = torch.Generator(device=dev).manual_seed(2)
    xt = torch.randn(Bt, N, device=dev, generator=gx)
    tgt = torch.randn(Bt, N, device=dev, generator=torch.Generator(device=dev).manual_seed(3))

    # every step starts from a fresh leaf on the resident input (no copy)
    def step():
        xg = xt.detach().requires_grad_(True)
        yy = t.bwd(*t.fwd(xg))
        ((yy - tgt) ** 2).mean().backward()
        return xg.grad

    for _ in range(W):
        step()
    torch.cuda.synchronize()
    ts = []
    for _ in range(max(K, 50)):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        step()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b))
    ref_form_ms = statistics.median(ts)
    # the same step with the loss folded into the engines (TrainableCQT.mse_loss:
    # squared-error sum in the synthesis epilogue, 2 (y - t) / n formed in the
    # transposed synthesis' load)
    def step_fused(xg):
        t.mse_loss(*t.fwd(xg), tgt).backward()

    def fused_eager():
        xg = xt.detach().requires_grad_(True)
        step_fused(xg)
        return xg.grad

    for _ in range(W):
        fused_eager()
    torch.cuda.synchronize()
    ts = []
    for _ in range(max(K, 50)):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fused_eager()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b))
    fused_ms = statistics.median(ts)
    # device time of the fused step alone: forward and backward captured in one
    # CUDA graph (static input, gradient in the graph's pool) and replayed
    xs = xt.clone().requires_grad_(True)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            xs.grad = None
            step_fused(xs)
    torch.cuda.current_stream().wait_stream(s)
    xs.grad = None
    gstep = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gstep):
        step_fused(xs)
    for _ in range(3):
        gstep.replay()
    torch.cuda.synchronize()
    reps = max(K, 50)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        gstep.replay()
    b.record()
    b.synchronize()
    gpu_ms = a.elapsed_time(b) / reps
    del gstep
    step_bytes = TRAIN_BYTES * Bt
    out["train_step_ms_b16"] = fused_ms
    out["train_step"] = {
        "batch": Bt, "ms": fused_ms,
        "ms_is": "median of 50 eager steps (CUDA events) of the fused-loss form",
        "fused_loss_eager_ms": fused_ms, "reference_form_eager_ms": ref_form_ms,
        "fused_loss_gpu_ms": gpu_ms,
        "roofline": {"bound": "hbm", "algorithmic_bytes_per_step": step_bytes,
                     "achieved": step_bytes / (gpu_ms / 1e3) / 1e9, "peak": hbm,
                     "unit": "GB/s", "frac": step_bytes / (gpu_ms / 1e3) / 1e9 / hbm,
                     "time": "fused_loss_gpu_ms (device time of the graph-replayed step)"},
        "eager_frac_of_hbm": step_bytes / (fused_ms / 1e3) / 1e9 / hbm,
        "what": "analysis -> synthesis -> MSE vs a seeded target -> backward, B = 16 "
                "(x seed 2, target seed 3); fused_loss = "
                "TrainableCQT.mse_loss(*fwd(x), t).backward() (the same loss, folded into "
                "the engines); reference_form = the reference's "
                "((bwd(*fwd(x)) - t) ** 2).mean().backward() on this build's TrainableCQT"}
    return out


if __name__ == "__main__":
    main()
