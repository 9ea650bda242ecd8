#!/usr/bin/env python3
"""Benchmark: fused rANS decode + dequant + GEMV on B200.

Workload (one GPU): the Llama-7B layer-shape GEMV sweep at batch 1 --
[4096x4096], [11008x4096], [4096x11008] -- with discrete-Laplace (b = 0.5)
4-bit symbols, group-128 fp16 scales U(0.01, 0.03), zero-point 8 and
x ~ N(0, 1) fp16 (seeded synthetic inputs of the reference's benchmark
shapes). Each matrix is encoded into the packed format (8x512 / 8x256 tiles,
32 interleaved rANS streams per tile, one table per matrix). To keep every
step's weights out of L2 (126 MB), REPLICAS copies of the three matrices
(~180 MB compressed in total) sit in HBM and one step runs the sweep over
all of them: 3 * REPLICAS fused GEMV launches, captured in a CUDA graph.

Metric: effective 4-bit weight GB/s = (M*K/2 bytes per matrix) / time, the
reference's "fused decode + GEMV" throughput view. The JSON line also
carries the compressed-byte HBM view (roofline), symbols/s, an end-to-end
figure through the public API with host buffers, and the reference CPU path
(the oracle's restatement) timed on this host.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ecq|reference]

With N > 1 (torchrun, one rank per GPU) every rank runs the same sweep on
its own GPU (weak scaling; the tiles are independent, no collective).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

SHAPES = [(4096, 4096), (11008, 4096), (4096, 11008)]
GROUP = 128
LAPLACE_B = 0.5
WORKLOAD = "llama7b_gemv_sweep_b1"
L2_BYTES = 126 * 1000 * 1000  # B200 L2, as the bench line states it


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ecq", "reference"], default="ecq")
    ap.add_argument("--replicas", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-llama", action="store_true", help="skip the 7B tensor-parallel decode step")
    ap.add_argument("--llama-steps", type=int, default=20)
    ap.add_argument("--no-batched", action="store_true", help="skip the 70B-MLP batched-token config")
    ap.add_argument("--no-sweep", action="store_true", help="skip the 8192x8192 entropy sweep")
    ap.add_argument("--no-sharded", action="store_true", help="skip the column-sharded sweep (N > 1)")
    return ap.parse_args()


def make_inputs():
    """Symbols, scales and x of the three shapes (seeded), plus their packed encodings."""
    import ecq_b200 as ecq
    from ecq_b200 import synthetic as syn

    out = []
    for i, (M, K) in enumerate(SHAPES):
        sym = syn.laplace_symbols(M, K, b=LAPLACE_B, seed=10 * i)
        sc = syn.group_scales(M, K, GROUP, seed=10 * i + 1)
        x = syn.activations(1, K, seed=10 * i + 2)
        enc = ecq.encode_matrix(sym, group_size=GROUP)
        out.append(dict(M=M, K=K, sym=sym, scales=sc, x=x, enc=enc))
    return out


def algorithmic_bytes(enc, M, K, B=1):
    """Bytes the fused GEMV must move: tile streams + per-tile offsets +
    per-stream lengths + decode table (64 KB) + fp16 scales + x + y."""
    ng = (K + GROUP - 1) // GROUP
    return (enc.compressed_bytes + 4 * (enc.n_tiles + 1) + 2 * 32 * enc.n_tiles + 4 * 16384
            + 2 * M * ng + 2 * B * K + 2 * B * M)


def issue_roofline(symbols_per_s, shapes, inst_executed, sm_count, sm_mhz):
    """Symbols/s against the integer-issue ceiling of the decode.

    Each SM has 4 schedulers, each issuing at most one warp instruction per
    cycle, and one warp instruction advances 32 lanes (32 streams). The
    decode's cost is the warp instructions one launch executes
    (`inst_executed`, ncu `smsp__inst_executed.sum` per shape "MxK"), so
    ceiling = sm_count * 4 * clock * 32 / (instructions per 32 symbols),
    with the instructions per 32 symbols weighted over the sweep's shapes.
    Returns None when a shape has no instruction count."""
    if not inst_executed or any(f"{M}x{K}" not in inst_executed for M, K in shapes):
        return None
    inst = sum(float(inst_executed[f"{M}x{K}"]) for M, K in shapes)
    sym = sum(M * K for M, K in shapes)
    per32 = inst / (sym / 32.0)
    ceiling = sm_count * 4 * sm_mhz * 1e6 * 32.0 / per32
    return {"inst_per_32_symbols": round(per32, 2), "sm_count": sm_count, "sm_mhz": sm_mhz,
            "ceiling_symbols_per_s": round(ceiling, 1), "frac": round(symbols_per_s / ceiling, 4)}


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "50", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.15)
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [v.strip() for v in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_baseline(inputs, threads, repeats=2, min_seconds=0.0):
    """The reference's CPU path (oracle restatement): per tile decode +
    dequant + matvec, over all three matrices, on `threads` host threads.
    Runs the sweep at least `repeats` times and until `min_seconds` of wall
    time have passed; returns (effective GB/s over all sweeps, seconds, sweeps)."""
    from oracle import oracle

    n, total = 0, 0.0
    while n < repeats or total < min_seconds:
        t0 = time.perf_counter()
        for d in inputs:
            e = d["enc"]
            y, bad = oracle.gemv_packed(e.data, e.tile_offset, e.stream_len, d["M"], d["K"], 8, e.tile_cols,
                                        e.table.freq, d["scales"].astype(np.float32), GROUP,
                                        d["x"].astype(np.float32), threads=threads)
            assert bad == 0
        total += time.perf_counter() - t0
        n += 1
    eff = sum(d["M"] * d["K"] / 2 for d in inputs)
    return eff * n / total / 1e9, total, n


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle

    inputs = make_inputs()
    threads = oracle.cpu_count()
    eff = sum(d["M"] * d["K"] / 2 for d in inputs)
    # each step: the full sweep once (bounded: ~0.2-1 s on a many-core host)
    for _ in range(max(args.warmup, 1)):
        cpu_baseline(inputs, threads, repeats=1)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_baseline(inputs, threads, repeats=1)
    dt = time.perf_counter() - t0
    value = eff * args.steps / dt / 1e9
    line = {
        "impl": "reference", "metric": "fused decode+GEMV effective 4-bit weight GB/s", "value": round(value, 3),
        "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * dt / args.steps, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": WORKLOAD, "shapes": SHAPES, "laplace_b": LAPLACE_B, "group_size": GROUP,
                   "batch": 1, "replicas": 1},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": "one full sweep (3 matrices, 107M symbols) per step: oracle C restatement of "
                                   "interleaved_rans_decode per tile + dequant + matvec, threads over row slabs"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ecq(args):
    import torch
    import torch.distributed as dist

    import ecq_b200 as ecq

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    inputs = make_inputs()
    R = args.replicas
    sets = []
    for r in range(R):
        mats = []
        for d in inputs:
            m = ecq.DeviceMatrix.from_encoded(d["enc"], group_size=GROUP, device=dev)
            mats.append(dict(m=m, sc=torch.from_numpy(d["scales"]).to(dev), x=torch.from_numpy(d["x"]).to(dev),
                             y=torch.empty(1, d["M"], dtype=torch.float16, device=dev)))
        sets.append(mats)
    torch.cuda.synchronize()

    # correctness gate before timing: every shape once against the oracle
    from oracle import oracle

    for d, e in zip(inputs, sets[0]):
        y = e["m"].gemv(e["x"], e["sc"], out=e["y"])
        e["m"].check()
        yr = oracle.dequant_gemv(d["sym"], d["scales"].astype(np.float32), GROUP, d["x"].astype(np.float32))
        err = float(np.max(np.abs(y.float().cpu().numpy()[0] - yr)) / np.max(np.abs(yr)))
        assert err <= 2e-3, f"parity gate failed: {err}"

    stream = torch.cuda.Stream(device=dev)
    # one graph per step (the whole ring) and one graph per launch (for per-kernel timing)
    step_graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        for mats in sets:  # warm the launch path (attributes) before capture
            for e in mats:
                e["m"].gemv(e["x"], e["sc"], out=e["y"])
        stream.synchronize()
        with torch.cuda.graph(step_graph, stream=stream):
            for mats in sets:
                for e in mats:
                    e["m"].gemv(e["x"], e["sc"], out=e["y"])
        launch_graphs = []
        for mats in sets:
            row = []
            for e in mats:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    e["m"].gemv(e["x"], e["sc"], out=e["y"])
                row.append(g)
            launch_graphs.append(row)
    launches_per_step = 3 * R

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step_graph.replay()
    stream.synchronize()
    barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(args.steps):
                step_graph.replay()
            ev1.record(stream)
        ev1.synchronize()
    torch.cuda.synchronize()
    barrier()
    ms = ev0.elapsed_time(ev1)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    eff_per_step = R * sum(d["M"] * d["K"] / 2 for d in inputs)
    sym_per_step = R * sum(d["M"] * d["K"] for d in inputs)
    value = world * eff_per_step * args.steps / (ms_max / 1e3) / 1e9

    # per-launch durations (events around each single-launch graph, same ring order)
    per_shape_ms = [[] for _ in SHAPES]
    with torch.cuda.stream(stream):
        evs = []
        n_rounds = max(3, min(args.steps // 4, 50))
        for _ in range(n_rounds):
            for row in launch_graphs:
                for i, g in enumerate(row):
                    a = torch.cuda.Event(enable_timing=True)
                    b = torch.cuda.Event(enable_timing=True)
                    a.record(stream)
                    g.replay()
                    b.record(stream)
                    evs.append((i, a, b))
    stream.synchronize()
    for i, a, b in evs:
        per_shape_ms[i].append(a.elapsed_time(b))
    avg_ms = [statistics.mean(v) for v in per_shape_ms]
    share = [a * 1 for a in avg_ms]
    dom = int(np.argmax(share))
    d = inputs[dom]
    alg = algorithmic_bytes(d["enc"], d["M"], d["K"])
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    achieved = alg / (avg_ms[dom] / 1e3) / 1e9
    traffic = None
    tf = ROOT / "profiles" / "gemv_dram_traffic.json"
    if tf.exists():
        try:
            traffic = json.loads(tf.read_text()).get(f"{d['M']}x{d['K']}")
        except Exception:
            traffic = None

    # end to end through the public API: x from pinned host, fused GEMVs, y back to pinned host
    e2e = None
    if not args.no_e2e:
        # every GEMV of the step gets its own x and y; all x of a step arrive in
        # one pinned host->device copy and all y leave in one device->host copy
        Ks = [d0["K"] for d0 in inputs]
        Ms = [d0["M"] for d0 in inputs]
        hx = torch.cat([torch.from_numpy(d0["x"]).reshape(-1) for _ in sets for d0 in inputs]).pin_memory()
        hy = torch.empty(R * sum(Ms), dtype=torch.float16).pin_memory()
        dx = torch.empty_like(hx, device=dev)
        dy = torch.empty_like(hy, device=dev)
        views, ox, oy = [], 0, 0
        for si in range(R):
            for i in range(len(inputs)):
                views.append((si, i, dx[ox:ox + Ks[i]].view(1, Ks[i]), dy[oy:oy + Ms[i]].view(1, Ms[i])))
                ox += Ks[i]
                oy += Ms[i]
        e2e_graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(e2e_graph, stream=stream):
                dx.copy_(hx, non_blocking=True)
                for si, i, xv, yv in views:
                    e = sets[si][i]
                    e["m"].gemv(xv, e["sc"], out=yv)
                hy.copy_(dy, non_blocking=True)
        e2e_steps = max(1, args.steps // 2)
        with torch.cuda.stream(stream):
            for _ in range(max(args.warmup, 3)):
                e2e_graph.replay()
                stream.synchronize()
            barrier()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            t0 = time.perf_counter()
            a.record(stream)
            for _ in range(e2e_steps):
                e2e_graph.replay()
                stream.synchronize()  # the host reads every step's results
                _ = float(hy[0])
            b.record(stream)
            b.synchronize()
            wall = time.perf_counter() - t0
        te = torch.tensor([max(a.elapsed_time(b), wall * 1e3)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e_ms = float(te.item())
        h2d = R * sum(2 * d0["K"] for d0 in inputs)
        d2h = R * sum(2 * d0["M"] for d0 in inputs)
        e2e = {"value": round(world * eff_per_step * e2e_steps / (e_ms / 1e3) / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "path": "DeviceMatrix.gemv (libecq C ABI) in a CUDA graph: every GEMV's x in one pinned-host copy, "
                       "every y back in one; the host reads y after every step"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as _o

        threads = _o.cpu_count()
        v, secs, sweeps = cpu_baseline(inputs, threads, repeats=2, min_seconds=1.5)
        cpu = {"value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"{sweeps} full sweeps (3 matrices, {sum(d0['M'] * d0['K'] for d0 in inputs) / 1e6:.0f}M "
                         f"symbols each) in {secs:.2f} s on {threads} threads (~{secs * threads:.0f} CPU-s): oracle "
                         f"C restatement of interleaved_rans_decode per tile + dequant + matvec, threads over row "
                         f"slabs"}

    batched = None
    if not args.no_batched:
        batched = run_batched(dev, world, rank, barrier)

    sweep = None
    if not args.no_sweep and world == 1:
        sweep = run_entropy_sweep(dev)

    sharded = None
    if world > 1 and not args.no_sharded:
        sharded = run_sharded_sweep(inputs, dev, world, rank, barrier,
                                    {f"{M}x{K}": round(v * 1e3, 2) for (M, K), v in zip(SHAPES, avg_ms)})

    llama = None
    if not args.no_llama:
        del step_graph, launch_graphs
        if not args.no_e2e:
            del e2e_graph
        sets.clear()
        torch.cuda.empty_cache()
        llama = run_llama(args, world, rank, local, dev, barrier)
        step_graph = launch_graphs = None

    comp_bytes_step = R * sum(algorithmic_bytes(d0["enc"], d0["M"], d0["K"]) for d0 in inputs)
    ms_step = ms_max / args.steps
    clk = clocks.summary()
    issue = None
    try:
        inst = json.loads((ROOT / "profiles" / "gemv_issue.json").read_text()).get("inst_executed")
        issue = issue_roofline(sym_per_step / (ms_step / 1e3), SHAPES, inst,
                               torch.cuda.get_device_properties(dev).multi_processor_count,
                               float(clk.get("sm_mhz") or peaks.get("sm_max_mhz", 1965.0)))
    except (OSError, ValueError):
        issue = None
    line = {
        "metric": "fused decode+GEMV effective 4-bit weight GB/s", "value": round(value, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": WORKLOAD, "shapes": SHAPES, "laplace_b": LAPLACE_B, "group_size": GROUP,
                   "batch": 1, "tile": "8x512 (K=4096) / 8x256 (K=11008), 32 streams",
                   "replicas": R,
                   "l2": (f"inputs larger than L2: {R} replica sets, {comp_bytes_step / 1e6:.0f} MB per step > 126 MB"
                          if comp_bytes_step > L2_BYTES else
                          f"inputs fit in L2 ({R} replica sets, {comp_bytes_step / 1e6:.0f} MB per step <= 126 MB): "
                          f"not a valid HBM measurement, raise --replicas"),
                   "bits_per_symbol": [round(d0["enc"].bits_per_symbol, 4) for d0 in inputs],
                   "parallelism": f"replicas{world}"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "traffic": traffic,
                     "kernel": f"matrix_kernel gemv {d['M']}x{d['K']}",
                     "avg_launch_us": round(avg_ms[dom] * 1e3, 2), "algorithmic_bytes": alg,
                     "per_shape_us": {f"{M}x{K}": round(v * 1e3, 2) for (M, K), v in zip(SHAPES, avg_ms)}},
        "views": {
            "effective_4bit_gbs": round(value / world, 2),
            "compressed_gbs": round(comp_bytes_step / (ms_step / 1e3) / 1e9, 2),
            "symbols_per_s": round(sym_per_step / (ms_step / 1e3), 1),
            "plain_4bit_roofline_gbs": hbm_peak,
            "issue_roofline": issue,
        },
        "e2e": e2e,
        "cpu_baseline": cpu,
        "llama7b_decode": llama,
        "batched_70b_mlp": batched,
        "entropy_sweep_8192": sweep,
        "column_sharded_sweep": sharded,
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        del step_graph, launch_graphs
        dist.destroy_process_group()


def _median_ms(fn, flush, reps=10, warm=3, barrier=None):
    """Median CUDA-event time of fn() over `reps` calls, each preceded by a
    write of `flush` (larger than L2) so that no call finds its inputs in L2."""
    import torch

    for _ in range(warm):
        fn()
    times = []
    for _ in range(reps):
        flush.zero_()
        if barrier is not None:
            barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b))
    return statistics.median(times)


def _device_laplace(M, K, b, dev, seed):
    import torch

    from ecq_b200 import synthetic as syn

    g = torch.Generator(device=dev).manual_seed(seed)
    p = torch.tensor(syn.laplace_probs(b), device=dev, dtype=torch.float32)
    return torch.multinomial(p, M * K, replacement=True, generator=g).to(torch.uint8).reshape(M, K).cpu().numpy()


def run_batched(dev, world=1, rank=0, barrier=None):
    """70B-MLP-shaped 28672 x 8192 matrix (Laplace b = 0.5, group-128 scales,
    8x256 tiles) at token batches 1, 8, 32, 128: batch 1 runs the fused GEMV,
    larger batches the tcgen05 kernel that decodes each tile straight into the
    tensor core's shared-memory operand (no decoded weight in HBM). As a
    control, the same encoding decoded to fp16 in HBM + a cuBLAS GEMM. With
    several ranks the matrix is column-sharded: each rank holds an even share
    of the K-tiles (same encoding), computes a partial y and an NCCL
    all-reduce sums them. CUDA events, max over ranks; 3 warm-up and 10 timed
    calls, each preceded by a 256 MB write that flushes L2."""
    import torch
    import torch.distributed as dist

    import ecq_b200 as ecq
    from ecq_b200 import synthetic as syn
    from ecq_b200.codec import slice_matrix, split_even

    M, K, TC = 28672, 8192, 256
    sym = _device_laplace(M, K, LAPLACE_B, dev, 0)
    enc = ecq.encode_matrix(sym, tile_cols=TC, group_size=GROUP)
    sc_all = syn.group_scales(M, K, GROUP, seed=1)
    nk = K // enc.tile_cols
    kt0, kt1 = split_even(nk, world)[rank]
    if world > 1:
        enc = slice_matrix(enc, 0, (M + 7) // 8, kt0, kt1)
    c0, c1 = kt0 * enc.tile_cols, kt1 * enc.tile_cols
    m = ecq.DeviceMatrix.from_encoded(enc, group_size=GROUP, device=dev)
    sc = torch.from_numpy(np.ascontiguousarray(sc_all[:, c0 // GROUP:c1 // GROUP])).to(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    gx = torch.Generator(device=dev).manual_seed(5)
    out = {"shape": [M, K], "tile": f"8x{TC}", "bits_per_symbol": round(enc.bits_per_symbol, 4), "n_gpus": world,
           "shard": f"K-tiles [{kt0}, {kt1}) of {nk} per rank" if world > 1 else "whole matrix",
           "batches": {}}

    def timed(fn):
        ms = _median_ms(fn, flush, barrier=barrier)
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    for B in (1, 8, 32, 128):
        x = torch.randn(B, K, device=dev, dtype=torch.float16, generator=gx)[:, c0:c1].contiguous()

        def fused():
            y = m.matmul(x, sc)
            if world > 1:
                dist.all_reduce(y)
            return y

        def control():
            y = torch.mm(x, m.dequantize(sc).t(), out_dtype=torch.float32).to(torch.float16)
            if world > 1:
                dist.all_reduce(y)
            return y

        ms = timed(fused)
        row = {"ms": round(ms, 4), "tokens_per_s": round(B * 1000.0 / ms, 1),
               "effective_4bit_gbs": round(M * K / 2 / (ms / 1e3) / 1e9, 1),
               "symbols_per_s": round(M * K / (ms / 1e3), 1),
               "useful_tflops": round(2.0 * B * M * K / (ms / 1e3) / 1e12, 2),
               "path": ("fused GEMV" if B == 1 else "fused decode + tcgen05 MMA (x in TMEM, W tile in SMEM)")
               + (" + NCCL all-reduce" if world > 1 else "")}
        if B > 1:
            cms = timed(control)
            row["control_decode_fp16_cublas_ms"] = round(cms, 4)
        out["batches"][str(B)] = row
    m.check()
    return out


def run_sharded_sweep(inputs, dev, world, rank, barrier, per_shape_us):
    """The sweep's three shapes split over the ranks, each whole matrix once
    per call: K-split (every rank a share of the K-tiles) summed over the
    ranks by the fused peer exchange (GEMV push + sum kernel) and, for
    comparison, by an NCCL all-reduce; and row-split (every rank a share of
    the row slabs) followed by an NCCL all-gather. CUDA events, max over
    ranks, median of 10 calls each preceded by a 256 MB L2 flush. The fused
    K-split result is checked against the unsharded GEMV first."""
    import torch
    import torch.distributed as dist

    import ecq_b200 as ecq
    from ecq_b200.codec import slice_matrix, split_even
    from ecq_b200.comm import PeerExchange

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    xch = PeerExchange(n_max=max(d["M"] for d in inputs), device=dev)
    out = {}

    def timed(fn):
        ms = _median_ms(fn, flush, barrier=barrier)
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    try:
        for (M, K), d in zip(SHAPES, inputs):
            enc = d["enc"]
            nk, ns = K // enc.tile_cols, (M + 7) // 8
            kt0, kt1 = split_even(nk, world)[rank]
            s0, s1 = split_even(ns, world)[rank]
            c0, c1 = kt0 * enc.tile_cols, kt1 * enc.tile_cols
            mk = ecq.DeviceMatrix.from_encoded(slice_matrix(enc, 0, ns, kt0, kt1), group_size=GROUP, device=dev)
            sk = torch.from_numpy(np.ascontiguousarray(d["scales"][:, c0 // GROUP:c1 // GROUP])).to(dev)
            xk = torch.from_numpy(np.ascontiguousarray(d["x"][:, c0:c1])).to(dev)
            mr = ecq.DeviceMatrix.from_encoded(slice_matrix(enc, s0, s1, 0, nk), group_size=GROUP, device=dev)
            sr = torch.from_numpy(np.ascontiguousarray(d["scales"][s0 * 8:min(s1 * 8, M)])).to(dev)
            x = torch.from_numpy(d["x"]).to(dev)
            rows_max = max(min(b * 8, M) - a * 8 for a, b in split_even(ns, world))
            yr = torch.zeros(1, rows_max, dtype=torch.float16, device=dev)
            yg = torch.empty(world, rows_max, dtype=torch.float16, device=dev)
            yk = torch.empty(M, dtype=torch.float16, device=dev)

            def fused():
                xch.gemv_push(mk, xk, sk)
                return xch.sum(M, out=yk)

            def nccl():
                y = mk.gemv(xk, sk)
                dist.all_reduce(y)
                return y

            def rows():
                mr.gemv(x, sr, out=yr[:, : mr.rows])
                dist.all_gather_into_tensor(yg, yr)
                return yg

            y_full = ecq.DeviceMatrix.from_encoded(enc, group_size=GROUP, device=dev).gemv(
                x, torch.from_numpy(d["scales"]).to(dev))
            y_f = fused().clone()
            torch.cuda.synchronize()
            xch.check()
            err = float((y_f.float() - y_full[0].float()).abs().max() / y_full.float().abs().max())
            assert err <= 2e-3, f"sharded parity gate failed for {M}x{K}: {err}"
            res = {"k_split_fused_us": round(1e3 * timed(fused), 2), "k_split_nccl_us": round(1e3 * timed(nccl), 2),
                   "row_split_allgather_us": round(1e3 * timed(rows), 2),
                   "one_gpu_us": per_shape_us.get(f"{M}x{K}"), "max_rel_err": round(err, 6)}
            res["effective_4bit_gbs_fused"] = round(M * K / 2 / (res["k_split_fused_us"] / 1e6) / 1e9, 1)
            out[f"{M}x{K}"] = res
            mk.check()
            mr.check()
    finally:
        xch.close()
    return {"n_gpus": world, "shapes": out,
            "split": "K-tiles (fused exchange or NCCL all-reduce) / row slabs (NCCL all-gather)"}


def run_entropy_sweep(dev):
    """8192 x 8192 at batch 1 over Laplace scales b in {0.3, 0.5, 1, 2, 100}
    and group sizes 64 and 128: the fused GEMV's time against the compressed
    size, mapping where decode (symbols/s) rather than HBM bytes bounds it.
    Median of 10 CUDA-event timed calls, each after a 256 MB L2 flush."""
    import torch

    import ecq_b200 as ecq
    from ecq_b200 import synthetic as syn

    M = K = 8192
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    x = torch.from_numpy(syn.activations(1, K, seed=2)).to(dev)
    y = torch.empty(1, M, dtype=torch.float16, device=dev)
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    rows = []
    for i, b in enumerate((0.3, 0.5, 1.0, 2.0, 100.0)):
        sym = _device_laplace(M, K, b, dev, 100 + i)
        for g in (64, 128):
            enc = ecq.encode_matrix(sym, group_size=g)
            m = ecq.DeviceMatrix.from_encoded(enc, group_size=g, device=dev)
            sc = torch.from_numpy(syn.group_scales(M, K, g, seed=1)).to(dev)
            ms = _median_ms(lambda: m.gemv(x, sc, out=y), flush)
            m.check()
            comp = enc.compressed_bytes + 4 * (enc.n_tiles + 1) + 64 * enc.n_tiles + 4 * 16384 + 2 * M * (K // g) \
                + 2 * K + 2 * M
            rows.append({"laplace_b": b, "group_size": g, "entropy_bits": round(syn.entropy_bits(syn.laplace_probs(b)), 3),
                         "bits_per_symbol": round(enc.bits_per_symbol, 4), "tile": f"8x{enc.tile_cols}",
                         "us": round(ms * 1e3, 2), "effective_4bit_gbs": round(M * K / 2 / (ms / 1e3) / 1e9, 1),
                         "compressed_gbs": round(comp / (ms / 1e3) / 1e9, 1),
                         "hbm_frac": round(comp / (ms / 1e3) / 1e9 / hbm, 4),
                         "symbols_per_s": round(M * K / (ms / 1e3), 1)})
            del m
    return {"shape": [M, K], "batch": 1, "cases": rows}


def run_llama(args, world, rank, local, dev, barrier):
    """Synthetic Llama-7B batch-1 decode step, tensor-parallel over the ranks,
    captured in one CUDA graph. With several ranks the row-parallel layers'
    all-reduces run fused into the GEMV and the next add + RMSNorm over NVLink
    peer memory; the same weights are also timed with NCCL all-reduces
    (`tokens_per_s_nccl`). Returns the summary."""
    import torch
    import torch.distributed as dist

    from ecq_b200.model import Llama7BDecoder

    t0 = time.perf_counter()
    dec = Llama7BDecoder(tp=world, rank=rank, device=dev, group=None, exchange="peer")
    build_s = time.perf_counter() - t0
    tok = torch.tensor([1], device=dev)
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())

    def timed(use_peer):
        dec.use_peer = use_peer
        with torch.cuda.stream(s):
            for _ in range(2):
                dec.step(tok)
            s.synchronize()
            dec.check()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                out = dec.step(tok)
            for _ in range(3):
                g.replay()
            s.synchronize()
        barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            a.record(s)
            for _ in range(args.llama_steps):
                g.replay()
            b.record(s)
        b.synchronize()
        ms = a.elapsed_time(b) / args.llama_steps
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dec.check()
        nxt = int(out.item())
        del g
        return float(t.item()), nxt

    ms, nxt = timed(True)
    res = {"tokens_per_s": round(1000.0 / ms, 2), "ms_per_token": round(ms, 3), "tp": world,
           "exchange": "fused peer-memory all-reduce (GEMV push + add/RMSNorm sum)" if world > 1 else "none",
           "steps": args.llama_steps, "symbols_per_token_per_rank": dec.symbols,
           "compressed_bytes_per_rank": dec.compressed_bytes, "build_s": round(build_s, 1), "next_token": nxt,
           "config": "32 layers, hidden 4096, 32 heads x 128, MLP 11008, vocab 32000, 2048-token fp16 KV cache; "
                     "Student-t(4)*0.02 weights, group-128 symmetric 4-bit, rANS per matrix; batch 1; CUDA graph"}
    if world > 1:
        ms_n, nxt_n = timed(False)
        res["tokens_per_s_nccl"] = round(1000.0 / ms_n, 2)
        res["ms_per_token_nccl"] = round(ms_n, 3)
        res["next_token_nccl"] = nxt_n
    dec.close()
    return res


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ecq(args)


if __name__ == "__main__":
    main()
