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

With N > 1 (torchrun, one rank per GPU) every matrix is column-sharded
(K-split) over the N GPUs: each rank decodes its share of the columns of
every matrix and pushes its fp32 partial y to every rank over NVLink peer
memory; a sum kernel on each rank closes the all-reduce (strong scaling of
each GEMV; the value is the whole matrices' effective bytes over the time,
max over ranks). Before timing, the sharded result is checked against the
oracle (tp_parity), and the 7B decode step's TP-N logits against TP-1.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
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
    ap.add_argument("--replicas", type=int, default=0,
                    help="replica sets of the three matrices (0: 8 on one GPU, 5 per GPU on several)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-llama", action="store_true", help="skip the 7B tensor-parallel decode step")
    ap.add_argument("--llama-steps", type=int, default=20)
    ap.add_argument("--no-batched", action="store_true", help="skip the 70B-MLP batched-token config")
    ap.add_argument("--no-sweep", action="store_true", help="skip the 8192x8192 entropy sweep")
    ap.add_argument("--no-sharded", action="store_true", help="skip the column-sharded sweep (N > 1)")
    ap.add_argument("--no-control", action="store_true", help="skip the plain 4-bit GEMV control")
    ap.add_argument("--compression-table", action="store_true",
                    help="print bits/symbol per tile shape against the entropy (host only, no GPU) and exit")
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


class OracleEncoded:
    """A packed matrix encoded by the oracle's C restatement of the reference
    encoder (the fields cpu_baseline reads): the reference arm encodes its
    inputs this way, so it runs without libecq."""

    def __init__(self, sym, tile_cols):
        from oracle import oracle

        freq, _ = oracle.table_for(np.bincount(sym.reshape(-1), minlength=16))
        tiles = oracle.encode_matrix_tiles(sym, freq, 8, tile_cols)
        self.tile_cols = tile_cols
        self.table = type("Table", (), {"freq": freq})()
        self.data = np.concatenate([t[0] for t in tiles])
        self.tile_offset = np.zeros(len(tiles) + 1, dtype=np.uint32)
        self.tile_offset[1:] = np.cumsum([t[0].size for t in tiles])
        self.stream_len = np.concatenate([t[1] for t in tiles]).astype(np.uint16)


def make_reference_inputs():
    """make_inputs' symbols, scales and x, encoded by the oracle (8x512 tiles
    for K = 4096, 8x256 for K = 11008, as the GPU arm's encoding)."""
    from ecq_b200 import synthetic as syn

    out = []
    for i, (M, K) in enumerate(SHAPES):
        sym = syn.laplace_symbols(M, K, b=LAPLACE_B, seed=10 * i)
        out.append(dict(M=M, K=K, sym=sym, scales=syn.group_scales(M, K, GROUP, seed=10 * i + 1),
                        x=syn.activations(1, K, seed=10 * i + 2), enc=OracleEncoded(sym, 512 if K % 512 == 0 else 256)))
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
    """SM clock and clock-event (throttle) reasons of this rank's GPU during
    the timed region, read every 2 ms on a host thread through NVML, the
    library nvidia-smi queries (read-only calls). The timed regions last
    tens of milliseconds, shorter than nvidia-smi's sampling start-up."""

    def __init__(self, device, period_s: float = 0.002):
        self.device = device
        self.period = period_s
        self.samples: list = []
        self.max_mhz = None
        self.nvml = None
        self.handle = None

    def _open(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        self.nvml = pynvml
        prop = torch.cuda.get_device_properties(self.device)
        try:
            bus = f"{prop.pci_domain_id:08X}:{prop.pci_bus_id:02X}:{prop.pci_device_id:02X}.0"
            self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(self.device.index or 0)
        self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)

    def _run(self):
        nv, h = self.nvml, self.handle
        reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while True:
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM), reasons(h)))
            except Exception:
                return
            if self.stop.wait(self.period):
                return

    def __enter__(self):
        import threading

        self.stop = threading.Event()
        self.thread = None
        try:
            self._open()
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        except Exception:
            self.handle = None
        return self

    def __exit__(self, *a):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)
        if self.nvml is not None:
            try:
                self.nvml.nvmlShutdown()
            except Exception:
                pass

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        nv = self.nvml
        masks = {"hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
                 "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
                 "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
                 "sw_power_cap": "nvmlClocksEventReasonSwPowerCap"}
        reasons = set()
        for name, attr in masks.items():
            bit = getattr(nv, attr, None)
            if bit is not None and any(r & bit for _, r in self.samples):
                reasons.add(name)
        return {"sm_mhz": statistics.median(c for c, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(self.samples), "source": "NVML every 2 ms"}


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

    inputs = make_reference_inputs()
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
        "ms_per_step": round(1e3 * dt / args.steps, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": WORKLOAD, "shapes": SHAPES, "laplace_b": LAPLACE_B, "group_size": GROUP,
                   "batch": 1, "replicas": 1},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": "one full sweep (3 matrices, 107M symbols) per step: oracle C restatement of "
                                   "interleaved_rans_decode per tile + dequant + matvec, threads over row slabs"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


class Unit:
    """One GEMV of a step: a whole matrix (one GPU) or this rank's K-split
    shard of it (several GPUs), its group scales, its slice of x and the full
    y [1, M] it produces."""

    def __init__(self, i, M, m, sc, x, y, c0, c1, enc):
        self.i, self.M, self.m, self.sc, self.x, self.y = i, M, m, sc, x, y
        self.c0, self.c1, self.enc = c0, c1, enc


def _shard_cols(K, world, rank):
    """This rank's group-aligned column range [c0, c1) of a K-split."""
    from ecq_b200.codec import split_even

    g0, g1 = split_even(K // GROUP, world)[rank]
    return g0 * GROUP, g1 * GROUP


def build_units(inputs, R, dev, world, rank):
    """R replica sets of the three shapes. One GPU: each matrix whole, in the
    standard encoding (8x512 / 8x256 tiles). N GPUs: each rank encodes its
    K-split shard (same symbols, scales and table) with the widest tile that
    still gives the shard >= 2048 tiles, so a shard keeps the GPU's warps busy
    (ecq_b200.model.shard_tile_cols)."""
    import torch

    import ecq_b200 as ecq
    from ecq_b200.model import shard_tile_cols

    encs = []
    for d in inputs:
        if world == 1:
            encs.append((d["enc"], 0, d["K"]))
        else:
            c0, c1 = _shard_cols(d["K"], world, rank)
            enc = ecq.encode_matrix(np.ascontiguousarray(d["sym"][:, c0:c1]), d["enc"].table,
                                    tile_cols=shard_tile_cols(d["M"], c1 - c0), group_size=GROUP)
            encs.append((enc, c0, c1))
    units = []
    for _ in range(R):
        for i, (d, (enc, c0, c1)) in enumerate(zip(inputs, encs)):
            units.append(Unit(i, d["M"], ecq.DeviceMatrix.from_encoded(enc, group_size=GROUP, device=dev),
                              torch.from_numpy(np.ascontiguousarray(d["scales"][:, c0 // GROUP:c1 // GROUP])).to(dev),
                              torch.from_numpy(np.ascontiguousarray(d["x"][:, c0:c1])).to(dev),
                              torch.empty(1, d["M"], dtype=torch.float16, device=dev), c0, c1, enc))
    return units


def launch(u, xch, x=None, y=None):
    """One unit: the fused GEMV (one GPU), or this rank's shard GEMV pushing
    its fp32 partials to every rank followed by the sum consumer (the
    column-sharded GEMV with its all-reduce fused in)."""
    x = u.x if x is None else x
    y = u.y if y is None else y
    if xch is None:
        u.m.gemv(x, u.sc, out=y)
    else:
        xch.gemv_push(u.m, x, u.sc)
        xch.sum(u.M, out=y.view(-1))


def run_ecq(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=600))

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_ranks(v):
        t = torch.tensor([float(v)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))

    inputs = make_inputs()
    R = args.replicas or (8 if world == 1 else 5 * world)
    xch = None
    if world > 1:
        from ecq_b200.comm import PeerExchange

        xch = PeerExchange(n_max=max(d["M"] for d in inputs), device=dev)
    units = build_units(inputs, R, dev, world, rank)
    torch.cuda.synchronize()

    # correctness gate before timing: every shape once against the oracle; at
    # N > 1 this is the column-sharded GEMV (K-split + fused exchange) checked
    # against the oracle's whole-matrix dequant + matvec on every rank
    from oracle import oracle

    y_refs = [oracle.dequant_gemv(d["sym"], d["scales"].astype(np.float32), GROUP, d["x"].astype(np.float32))[0]
              for d in inputs]
    errs = []
    for u in units[:3]:
        launch(u, xch)
        torch.cuda.synchronize()
        u.m.check()
        if xch is not None:
            xch.check()
        yr = y_refs[u.i]
        errs.append(float(np.max(np.abs(u.y.float().cpu().numpy()[0] - yr)) / np.max(np.abs(yr))))
    gate_err = max_ranks(max(errs))
    assert gate_err <= 2e-3, f"parity gate failed: {gate_err}"
    tp_parity = None
    if world > 1:
        tp_parity = {"exchange_rel_err": round(gate_err, 6),
                     "exchange_vs": "oracle fp64 dequant + matvec of each whole sweep matrix, max over shapes and ranks"}
        tp_parity.update(rmsnorm_parity(inputs[0], units[0], xch, y_refs[0], dev, max_ranks))

    stream = torch.cuda.Stream(device=dev)
    step_graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        for u in units:  # warm the launch path (attributes) before capture
            launch(u, xch)
        stream.synchronize()
        with torch.cuda.graph(step_graph, stream=stream):
            for u in units:
                launch(u, xch)
    kernels_per_unit = 1 if world == 1 else 2
    shard_tiles = {f"{d['M']}x{d['K']}": f"8x{u.enc.tile_cols}" for d, u in zip(inputs, units[:3])}

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step_graph.replay()
    stream.synchronize()
    barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clocks:
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(args.steps):
                step_graph.replay()
            ev1.record(stream)
        ev1.synchronize()
    torch.cuda.synchronize()
    barrier()
    ms_max = max_ranks(ev0.elapsed_time(ev1))
    if xch is not None:
        xch.check()
    eff_per_step = R * sum(d["M"] * d["K"] / 2 for d in inputs)
    sym_per_step = R * sum(d["M"] * d["K"] for d in inputs)
    value = eff_per_step * args.steps / (ms_max / 1e3) / 1e9
    ms_step = ms_max / args.steps

    split = None
    if world == 1:
        # per-launch durations: events around one-launch graphs, cycling the ring
        graphs = []
        with torch.cuda.stream(stream):
            for u in units:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    launch(u, None)
                graphs.append((u.i, g))
        per_shape_ms = [[] for _ in SHAPES]
        with torch.cuda.stream(stream):
            evs = []
            for _ in range(max(3, min(args.steps // 4, 50))):
                for i, g in graphs:
                    a = torch.cuda.Event(enable_timing=True)
                    b = torch.cuda.Event(enable_timing=True)
                    a.record(stream)
                    g.replay()
                    b.record(stream)
                    evs.append((i, a, b))
        stream.synchronize()
        for i, a, b in evs:
            per_shape_ms[i].append(a.elapsed_time(b))
        kern_ms = [statistics.mean(v) for v in per_shape_ms]
        del graphs
    else:
        split = exchange_split(units, xch, stream, max_ranks)
        kern_ms = [split[f"{M}x{K}"]["gemv_push_us"] / 1e3 for M, K in SHAPES]
    dom = int(np.argmax(kern_ms))
    du = units[dom]
    alg = algorithmic_bytes(du.enc, du.M, du.c1 - du.c0)
    if world > 1:  # the shard's partials go to every rank as 8-byte words instead of an fp16 y
        alg += du.M * (8 * world - 2)
    achieved = alg / (kern_ms[dom] / 1e3) / 1e9
    traffic, traffic_src = None, None
    tf = ROOT / "profiles" / "gemv_dram_traffic.json"
    if world == 1 and tf.exists():
        try:
            traffic = json.loads(tf.read_text()).get(f"{du.M}x{du.c1 - du.c0}")
            traffic_src = ("committed ncu capture (profiles/gemv_dram_traffic.json, dram__bytes_read.sum + "
                           "dram__bytes_write.sum of this shape's launch), not measured in this run")
        except Exception:
            traffic = None

    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(units, xch, stream, args, eff_per_step, barrier, max_ranks)

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

    control = None
    if world == 1 and not args.no_control:
        control = run_plain4_control(inputs, R, stream, kern_ms, value, hbm_peak)

    batched = None
    if not args.no_batched:
        batched = run_batched(dev, world, rank, barrier)

    sweep = None
    if not args.no_sweep and world == 1:
        sweep = run_entropy_sweep(dev)

    sharded = None
    if world > 1 and not args.no_sharded:
        sharded = run_sharded_sweep(inputs, units, xch, dev, world, rank, barrier, max_ranks)
        sharded["gemv_push_and_consumer_split_us"] = split

    comp_bytes_step = sum(algorithmic_bytes(u.enc, u.M, u.c1 - u.c0) for u in units)
    del step_graph
    llama = None
    if not args.no_llama:
        units.clear()
        torch.cuda.empty_cache()
        llama = run_llama(args, world, rank, local, dev, barrier, max_ranks)
        if llama is not None and world > 1:
            tp_parity = dict(tp_parity or {}, **llama.pop("tp_parity", {}))

    clk = clocks.summary()
    issue = None
    if world == 1:
        try:
            inst = json.loads((ROOT / "profiles" / "gemv_issue.json").read_text()).get("inst_executed")
            issue = issue_roofline(sym_per_step / (ms_step / 1e3), SHAPES, inst,
                                   torch.cuda.get_device_properties(dev).multi_processor_count,
                                   float(clk.get("sm_mhz") or peaks.get("sm_max_mhz", 1965.0)))
            if issue is not None:
                issue["inst_source"] = ("committed ncu capture (profiles/gemv_issue.json, smsp__inst_executed.sum "
                                        "per shape), not measured in this run")
        except (OSError, ValueError):
            issue = None
    if world == 1:
        tiles = "8x512 (K=4096) / 8x256 (K=11008), 32 streams"
        par = "one GPU, whole matrices"
    else:
        tiles = shard_tiles
        par = (f"K-split column shard over {world} GPUs: each rank decodes its share of every matrix's columns and "
               f"pushes fp32 partials to every rank over NVLink peer memory, a sum kernel closes the all-reduce")
    line = {
        "metric": "fused decode+GEMV effective 4-bit weight GB/s", "value": round(value, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": WORKLOAD, "shapes": SHAPES, "laplace_b": LAPLACE_B, "group_size": GROUP,
                   "batch": 1, "tile": tiles, "replicas": R,
                   "l2": (f"inputs larger than L2: {R} replica sets, {comp_bytes_step / 1e6:.0f} MB per GPU per step "
                          f"> 126 MB" if comp_bytes_step > L2_BYTES else
                          f"inputs fit in L2 ({R} replica sets, {comp_bytes_step / 1e6:.0f} MB per GPU per step <= "
                          f"126 MB): not a valid HBM measurement, raise --replicas"),
                   "bits_per_symbol": [round(d0["enc"].bits_per_symbol, 4) for d0 in inputs],
                   "parallelism": par},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "traffic": traffic, "traffic_source": traffic_src,
                     "kernel": (f"matrix_kernel gemv {du.M}x{du.c1 - du.c0}" if world == 1 else
                                f"matrix_kernel gemv + push, shard {du.M}x{du.c1 - du.c0}"),
                     "avg_launch_us": round(kern_ms[dom] * 1e3, 2), "algorithmic_bytes": alg,
                     "per_shape_us": {f"{M}x{K}": round(v * 1e3, 2) for (M, K), v in zip(SHAPES, kern_ms)}},
        "views": {
            "effective_4bit_gbs": round(value / world, 2),
            "compressed_gbs": round(comp_bytes_step * world / (ms_step / 1e3) / 1e9, 2),
            "symbols_per_s": round(sym_per_step / (ms_step / 1e3), 1),
            "plain_4bit_roofline_gbs": hbm_peak,
            "issue_roofline": issue,
            "plain_4bit_control": control,
        },
        "e2e": e2e,
        "cpu_baseline": cpu,
        "batched_70b_mlp": batched,
        "entropy_sweep_8192": sweep,
        "column_sharded_sweep": sharded,
        "llama7b_decode": llama,
        "tp_parity": tp_parity,
        "gpu_launches": kernels_per_unit * len(inputs) * R * args.steps,
        "clocks": clk,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if xch is not None:
        xch.close()
    if world > 1:
        dist.destroy_process_group()


def rmsnorm_parity(d, u, xch, y_ref, dev, max_ranks):
    """The row-parallel exchange with its residual add + RMSNorm consumer
    (gemv push -> ecq_tp_add_rmsnorm_f16) on one sweep shape, against the
    oracle's dequant + matvec followed by a numpy residual add and RMSNorm
    (fp16 roundings where the kernel rounds). Returns the max relative errors
    over ranks."""
    import torch

    M = d["M"]
    rng = np.random.default_rng(123)
    h0 = rng.standard_normal(M).astype(np.float16)
    w = (1.0 + 0.1 * rng.standard_normal(M)).astype(np.float16)
    h = torch.from_numpy(h0).to(dev)
    wt = torch.from_numpy(w).to(dev)
    xch.gemv_push(u.m, u.x, u.sc)
    y = xch.add_rmsnorm(h, wt, 1e-5)
    torch.cuda.synchronize()
    u.m.check()
    xch.check()
    h_ref = (h0.astype(np.float32) + y_ref.astype(np.float16).astype(np.float32)).astype(np.float16)
    hf = h_ref.astype(np.float32)
    y_ref2 = (hf / np.sqrt(np.mean(hf * hf) + 1e-5)).astype(np.float16).astype(np.float32) * w.astype(np.float32)
    eh = float(np.max(np.abs(h.float().cpu().numpy() - hf)) / np.max(np.abs(hf)))
    ey = float(np.max(np.abs(y.float().cpu().numpy() - y_ref2)) / np.max(np.abs(y_ref2)))
    return {"residual_rel_err": round(max_ranks(eh), 6), "rmsnorm_rel_err": round(max_ranks(ey), 6),
            "rmsnorm_shape": f"{M}x{d['K']}"}


def exchange_split(units, xch, stream, max_ranks):
    """Device time of the two kernels of each column-sharded GEMV: the shard
    GEMV with its push, and the sum consumer (which includes waiting for the
    slowest rank's push). CUDA events between the launches of an eager run
    over the whole ring, queued behind a device-side sleep so that host
    launch gaps do not enter the intervals; median per shape, max over ranks."""
    import torch

    torch.cuda.synchronize()
    marks = []
    with torch.cuda.stream(stream):
        torch.cuda._sleep(50_000_000)
        for u in units:
            e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            e0.record(stream)
            xch.gemv_push(u.m, u.x, u.sc)
            e1.record(stream)
            xch.sum(u.M, out=u.y.view(-1))
            e2.record(stream)
            marks.append((u.i, e0, e1, e2))
    stream.synchronize()
    xch.check()
    out = {}
    for i, (M, K) in enumerate(SHAPES):
        g = [a.elapsed_time(b) * 1e3 for j, a, b, _ in marks if j == i]
        c = [b.elapsed_time(e) * 1e3 for j, _, b, e in marks if j == i]
        out[f"{M}x{K}"] = {"gemv_push_us": round(max_ranks(statistics.median(g)), 2),
                           "consumer_us": round(max_ranks(statistics.median(c)), 2)}
    return out


def run_e2e(units, xch, stream, args, eff_per_step, barrier, max_ranks):
    """The same step through the public API with host buffers: every unit's x
    (this rank's slice) arrives in one pinned host->device copy and every y
    leaves in one device->host copy, inside the timed region; the host reads y
    after every step. Max over ranks."""
    import torch

    dev = units[0].y.device
    hx = torch.cat([u.x.reshape(-1).cpu() for u in units]).pin_memory()
    hy = torch.empty(sum(u.M for u in units), dtype=torch.float16).pin_memory()
    dx = torch.empty_like(hx, device=dev)
    dy = torch.empty_like(hy, device=dev)
    views, ox, oy = [], 0, 0
    for u in units:
        kx = u.x.numel()
        views.append((u, dx[ox:ox + kx].view(1, kx), dy[oy:oy + u.M].view(1, u.M)))
        ox += kx
        oy += u.M
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(g, stream=stream):
            dx.copy_(hx, non_blocking=True)
            for u, xv, yv in views:
                launch(u, xch, xv, yv)
            hy.copy_(dy, non_blocking=True)
    steps = max(1, args.steps // 2)
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            g.replay()
            stream.synchronize()
        barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        a.record(stream)
        for _ in range(steps):
            g.replay()
            stream.synchronize()  # the host reads every step's results
            _ = float(hy[0])
        b.record(stream)
        b.synchronize()
        wall = time.perf_counter() - t0
    e_ms = max_ranks(max(a.elapsed_time(b), wall * 1e3))
    del g
    return {"value": round(eff_per_step * steps / (e_ms / 1e3) / 1e9, 3), "unit": "GB/s",
            "h2d_bytes_per_step": int(hx.numel() * 2), "d2h_bytes_per_step": int(hy.numel() * 2),
            "path": "DeviceMatrix.gemv / PeerExchange (libecq C ABI) in a CUDA graph: every GEMV's x in one "
                    "pinned-host copy, every y back in one; the host reads y after every step"}


def run_plain4_control(inputs, R, stream, rans_ms, rans_eff_gbs, hbm_peak):
    """The in-run control: the same three shapes, scales and x with the
    symbols stored as plain packed 4-bit (no entropy coding), multiplied by
    the hand-written plain 4-bit GEMV (ecq_plain4_gemv). R replica sets keep
    the weights out of L2 exactly as for the rANS sweep; one step is the
    sweep over all of them in one CUDA graph, timed with CUDA events over 20
    replays after 3 warm-up replays, plus per-launch times from one-launch
    graphs cycling over the ring. Returns effective 4-bit GB/s, the HBM fraction of the bytes it
    moves (weights + scales + x + y) and the rANS/plain time ratio."""
    import torch

    from ecq_b200.device import Packed4Matrix

    dev = torch.device("cuda", torch.cuda.current_device())
    sets = []
    for _ in range(R):
        row = []
        for d in inputs:
            row.append(dict(p=Packed4Matrix.from_symbols(d["sym"], GROUP, device=dev),
                            sc=torch.from_numpy(d["scales"]).to(dev), x=torch.from_numpy(d["x"]).to(dev),
                            y=torch.empty(1, d["M"], dtype=torch.float16, device=dev)))
        sets.append(row)
    from oracle import oracle

    for d, e in zip(inputs, sets[0]):
        y = e["p"].gemv(e["x"], e["sc"], out=e["y"])
        yr = oracle.dequant_gemv(d["sym"], d["scales"].astype(np.float32), GROUP, d["x"].astype(np.float32))
        err = float(np.max(np.abs(y.float().cpu().numpy()[0] - yr)) / np.max(np.abs(yr)))
        assert err <= 2e-3, f"plain 4-bit parity gate failed: {err}"
    g = torch.cuda.CUDAGraph()
    singles = []
    with torch.cuda.stream(stream):
        with torch.cuda.graph(g, stream=stream):
            for row in sets:
                for e in row:
                    e["p"].gemv(e["x"], e["sc"], out=e["y"])
        for row in sets:  # one-launch graphs over the whole ring, so no launch finds its weights in L2
            for i, e in enumerate(row):
                gg = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gg, stream=stream):
                    e["p"].gemv(e["x"], e["sc"], out=e["y"])
                singles.append((i, gg))
        for _ in range(3):
            g.replay()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        steps = 20
        a.record(stream)
        for _ in range(steps):
            g.replay()
        b.record(stream)
        b.synchronize()
        ms = a.elapsed_time(b) / steps
        per = [[] for _ in inputs]
        evs = []
        for _ in range(10):
            for i, gg in singles:
                x0 = torch.cuda.Event(enable_timing=True)
                x1 = torch.cuda.Event(enable_timing=True)
                x0.record(stream)
                gg.replay()
                x1.record(stream)
                evs.append((i, x0, x1))
        stream.synchronize()
    for i, x0, x1 in evs:
        per[i].append(x0.elapsed_time(x1))
    per_us = [statistics.median(v) * 1e3 for v in per]
    eff = R * sum(d["M"] * d["K"] / 2 for d in inputs)
    moved = R * sum(d["M"] * d["K"] / 2 + 2 * d["M"] * ((d["K"] + GROUP - 1) // GROUP) + 2 * d["K"] + 2 * d["M"]
                    for d in inputs)
    eff_gbs = eff / (ms / 1e3) / 1e9
    del g, singles
    return {"kernel": "plain4_gemv_kernel (ecq_plain4_gemv), packed nibbles + group-128 fp16 scales",
            "effective_4bit_gbs": round(eff_gbs, 2),
            "hbm_gbs": round(moved / (ms / 1e3) / 1e9, 2), "hbm_frac": round(moved / (ms / 1e3) / 1e9 / hbm_peak, 4),
            "ms_per_sweep": round(ms, 4), "replicas": R,
            "per_shape_us": {f"{d['M']}x{d['K']}": round(u, 2) for d, u in zip(inputs, per_us)},
            "rans_over_plain_time": round(eff_gbs / rans_eff_gbs, 3) if rans_eff_gbs else None,
            "rans_per_shape_us": {f"{d['M']}x{d['K']}": round(v * 1e3, 2) for d, v in zip(inputs, rans_ms)}}


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
    """70B-MLP-shaped 28672 x 8192 matrix (Laplace b = 0.5, group-128 scales)
    at token batches 1, 8, 32, 128 through DeviceMatrix.matmul, the one
    dispatch of the batched entry points: up to 4 tokens the fused GEMV that
    decodes each tile once for the whole batch, more the tcgen05 kernel that
    decodes each tile straight into the tensor core's shared-memory operand
    (8x256 tiles); no decoded weight goes to HBM on either. Also: B = 8 on the
    batched fused GEMV (8x512 and 8x256 encodings), and, as a control, the
    8x256 encoding decoded to fp16 in HBM + a cuBLAS GEMM.
    With several ranks the matrix is column-sharded: each rank holds an even
    share of the K-tiles (same encoding), computes a partial y and an NCCL
    all-reduce sums them. CUDA events, max over ranks; 3 warm-up and 10 timed
    calls, each preceded by a 256 MB write that flushes L2."""
    import torch
    import torch.distributed as dist

    import ecq_b200 as ecq
    from ecq_b200 import synthetic as syn
    from ecq_b200.codec import slice_matrix, split_even

    M, K = 28672, 8192
    sym = _device_laplace(M, K, LAPLACE_B, dev, 0)
    sc_all = syn.group_scales(M, K, GROUP, seed=1)
    mats = {}
    for TC in (256, 512):
        enc = ecq.encode_matrix(sym, tile_cols=TC, group_size=GROUP)
        nk = K // TC
        # the same column range on both encodings: shards of 512 columns
        kt0, kt1 = split_even(K // 512, world)[rank]
        kt0, kt1 = kt0 * (512 // TC), kt1 * (512 // TC)
        if world > 1:
            enc = slice_matrix(enc, 0, (M + 7) // 8, kt0, kt1)
        mats[TC] = (ecq.DeviceMatrix.from_encoded(enc, group_size=GROUP, device=dev), enc, kt0 * TC, kt1 * TC, nk)
    m, enc, c0, c1, nk = mats[256]
    m512 = mats[512][0]
    sc = torch.from_numpy(np.ascontiguousarray(sc_all[:, c0 // GROUP:c1 // GROUP])).to(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    gx = torch.Generator(device=dev).manual_seed(5)
    out = {"shape": [M, K], "tile": "8x256 (8x512 where stated)", "bits_per_symbol": round(enc.bits_per_symbol, 4),
           "bits_per_symbol_8x512": round(mats[512][1].bits_per_symbol, 4), "n_gpus": world,
           "shard": f"columns [{c0}, {c1}) of {K} per rank" if world > 1 else "whole matrix", "batches": {}}

    def timed(fn):
        ms = _median_ms(fn, flush, barrier=barrier)
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    def reduce(y):
        if world > 1:
            dist.all_reduce(y)
        return y

    def row_of(B, ms, path):
        return {"ms": round(ms, 4), "tokens_per_s": round(B * 1000.0 / ms, 1),
                "effective_4bit_gbs": round(M * K / 2 / (ms / 1e3) / 1e9, 1),
                "symbols_per_s": round(M * K / (ms / 1e3), 1),
                "useful_tflops": round(2.0 * B * M * K / (ms / 1e3) / 1e12, 2),
                "path": path + (" + NCCL all-reduce" if world > 1 else "")}

    for B in (1, 8, 32, 128):
        x = torch.randn(B, K, device=dev, dtype=torch.float16, generator=gx)[:, c0:c1].contiguous()
        m.ensure_workspace(min(B, 8))
        m512.ensure_workspace(min(B, 8))
        ms = timed(lambda: reduce(m.matmul(x, sc)))
        from ecq_b200.device import GEMV_MAX_BATCH, TENSOR_CORE_MAX_BATCH

        path = ("fused GEMV" if B == 1 else
                "fused GEMV, each tile decoded once for the batch" if B <= GEMV_MAX_BATCH else
                "fused decode + tcgen05 MMA (x in TMEM, W tile in SMEM)" if B <= TENSOR_CORE_MAX_BATCH else
                "W decoded once to fp16 (matrix_kernel) + cuBLAS GEMM")
        row = row_of(B, ms, path + " [8x256 tiles]")
        if B > TENSOR_CORE_MAX_BATCH:
            row["tcgen05_ms"] = round(timed(lambda: reduce(m.matmul_tc(x, sc))), 4)
        if B > 1:
            row["control_decode_fp16_cublas_ms"] = round(
                timed(lambda: reduce(torch.mm(x, m.dequantize(sc).t(), out_dtype=torch.float32).to(torch.float16))), 4)
        if B in (1, 8):
            row["gemv_8x512_ms"] = round(timed(lambda: reduce(m512.gemv(x, sc))), 4)
        if B == 8:
            row["gemv_8x256_batched_ms"] = round(timed(lambda: reduce(m.gemv(x, sc))), 4)
            # the dispatch on the default GEMV encoding (8x512: no tcgen05 kernel)
            row["dispatch_8x512_ms"] = round(timed(lambda: reduce(m512.matmul(x, sc))), 4)
        out["batches"][str(B)] = row
    b1, b8 = out["batches"]["1"], out["batches"]["8"]
    out["b8_over_b1_time_8x512"] = round(b8["gemv_8x512_ms"] / b1["gemv_8x512_ms"], 3)
    out["b8_dispatch_over_b1_time_8x512"] = round(b8["dispatch_8x512_ms"] / b1["gemv_8x512_ms"], 3)
    m.check()
    m512.check()
    return out


def run_sharded_sweep(inputs, units, xch, dev, world, rank, barrier, max_ranks):
    """Each sweep shape split over the ranks, one whole matrix per call (median
    of 10 calls, each after a 256 MB L2 flush and a barrier; CUDA events, max
    over ranks): the K-split shard GEMV closed by the fused peer exchange (the
    headline's unit), the same shard GEMV closed by an NCCL all-reduce, and a
    row split (every rank a share of the row slabs, whole K, standard
    encoding) followed by an NCCL all-gather."""
    import torch
    import torch.distributed as dist

    import ecq_b200 as ecq
    from ecq_b200.codec import slice_matrix, split_even

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    out = {}
    for d, u in zip(inputs, units[:3]):
        M, K = d["M"], d["K"]
        enc = d["enc"]
        ns, nk = (M + 7) // 8, K // enc.tile_cols
        s0, s1 = split_even(ns, world)[rank]
        mr = ecq.DeviceMatrix.from_encoded(slice_matrix(enc, s0, s1, 0, nk), group_size=GROUP, device=dev)
        sr = torch.from_numpy(np.ascontiguousarray(d["scales"][s0 * 8:min(s1 * 8, M)])).to(dev)
        x = torch.from_numpy(d["x"]).to(dev)
        rows_max = max(min(hi * 8, M) - lo * 8 for lo, hi in split_even(ns, world))
        yr = torch.zeros(1, rows_max, dtype=torch.float16, device=dev)
        yg = torch.empty(world, rows_max, dtype=torch.float16, device=dev)

        def fused():
            launch(u, xch)

        def nccl():
            y = u.m.gemv(u.x, u.sc)
            dist.all_reduce(y)

        def rows():
            mr.gemv(x, sr, out=yr[:, : mr.rows])
            dist.all_gather_into_tensor(yg, yr)

        res = {"shard_tile": f"8x{u.enc.tile_cols}", "shard_bits_per_symbol": round(u.enc.bits_per_symbol, 4),
               "k_split_fused_us": round(1e3 * max_ranks(_median_ms(fused, flush, barrier=barrier)), 2),
               "k_split_nccl_us": round(1e3 * max_ranks(_median_ms(nccl, flush, barrier=barrier)), 2),
               "row_split_allgather_us": round(1e3 * max_ranks(_median_ms(rows, flush, barrier=barrier)), 2)}
        res["effective_4bit_gbs_fused"] = round(M * K / 2 / (res["k_split_fused_us"] / 1e6) / 1e9, 1)
        out[f"{M}x{K}"] = res
        u.m.check()
        mr.check()
        xch.check()
    return {"n_gpus": world, "shapes": out,
            "split": "K-split shards (fused exchange or NCCL all-reduce) / row slabs (NCCL all-gather)"}


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


def run_llama(args, world, rank, local, dev, barrier, max_ranks):
    """Synthetic Llama-7B batch-1 decode step, tensor-parallel over the ranks,
    captured in one CUDA graph. With several ranks the row-parallel layers'
    all-reduces run fused into the GEMV and the next add + RMSNorm over NVLink
    peer memory; the same weights are also timed with NCCL all-reduces
    (`tokens_per_s_nccl`). Also: the step's device time split by kernel kind
    (rank 0, one eager step), and at N > 1 the TP-N logits against a TP-1
    decoder of the same weights and KV cache built on rank 0 (tp_parity).
    Returns the summary."""
    import torch

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
        ms = max_ranks(a.elapsed_time(b) / args.llama_steps)
        dec.check()
        nxt = int(out.item())
        del g
        return ms, nxt

    ms, nxt = timed(True)
    with torch.cuda.stream(s):
        breakdown = dec.step_breakdown(tok)
        logits = dec.step_logits(tok).float().cpu()
    res = {"tokens_per_s": round(1000.0 / ms, 2), "ms_per_token": round(ms, 3), "tp": world,
           "exchange": "fused peer-memory all-reduce (GEMV push + add/RMSNorm sum)" if world > 1 else "none",
           "steps": args.llama_steps, "symbols_per_token_per_rank": dec.symbols,
           "compressed_bytes_per_rank": dec.compressed_bytes, "build_s": round(build_s, 1), "next_token": nxt,
           "breakdown_us_rank0": breakdown,
           "config": "32 layers, hidden 4096, 32 heads x 128, MLP 11008, vocab 32000, 2048-token fp16 KV cache; "
                     "Student-t(4)*0.02 weights, group-128 symmetric 4-bit, rANS per matrix; batch 1; CUDA graph"}
    if world > 1:
        ms_n, nxt_n = timed(False)
        res["tokens_per_s_nccl"] = round(1000.0 / ms_n, 2)
        res["ms_per_token_nccl"] = round(ms_n, 3)
        res["next_token_nccl"] = nxt_n
    dec.close()
    del dec
    torch.cuda.empty_cache()
    if world > 1:
        par = {}
        if rank == 0:
            ref = Llama7BDecoder(tp=1, rank=0, device=dev)
            with torch.cuda.stream(s):
                l1 = ref.step_logits(tok).float().cpu()
            s.synchronize()
            ref.check()
            par = {"logits_rel_err_vs_tp1": round(float((logits - l1).abs().max() / l1.abs().max()), 6),
                   "same_next_token": bool(int(torch.argmax(logits)) == int(torch.argmax(l1)) == nxt),
                   "next_token_tp1": int(torch.argmax(l1)),
                   "logits_vs": "TP-1 decoder of the same weights and KV cache on rank 0 (its own exchange-free "
                                "path), 7B config"}
            del ref
            torch.cuda.empty_cache()
        barrier()
        res["tp_parity"] = par
    return res


def compression_table(M=4096, K=4096):
    """Bits per symbol of the packed format against the symbols' entropy, per
    tile shape: the kernels' 8-row tiles of 128, 256 and 512 columns (32
    streams of tile_cols/4 symbols), and taller or wider tiles the format
    allows but the kernels do not take (16x512, 8x1024, 32x512: 256-512
    symbols per stream). The excess over the entropy is each stream's 4-byte
    flush plus the padding of every stream to its tile's longest. Inputs: the
    sweep's Laplace symbols at b = 0.3, 0.5, 1, 2 and Student-t(4) weights
    quantised per group of 128, M x K each."""
    from ecq_b200 import synthetic as syn
    from ecq_b200.codec import RANSTable
    from oracle import oracle

    cases = [(f"laplace b={b}", syn.laplace_symbols(M, K, b=b, seed=1)) for b in (0.3, 0.5, 1.0, 2.0)]
    cases.append(("student-t(4) group-128", syn.quantize_symmetric_groups(
        syn.student_t_weights(M, K, seed=2).astype(np.float32), 128)[0]))
    rows = []
    for name, sym in cases:
        p_ = np.bincount(sym.reshape(-1), minlength=16) / sym.size
        ent = float(-(p_[p_ > 0] * np.log2(p_[p_ > 0])).sum())
        table = RANSTable.from_symbols(sym)
        row = {"symbols": name, "entropy_bits": round(ent, 3)}
        for tr, tc in ((8, 128), (8, 256), (8, 512), (16, 512), (8, 1024), (32, 512)):
            nbytes = 0
            for r0 in range(0, M, tr):
                for c0 in range(0, K, tc):
                    data, _, _ = oracle.encode_interleaved(sym[r0:r0 + tr, c0:c0 + tc].reshape(-1), table.freq, 32)
                    nbytes += data.size
            row[f"{tr}x{tc}"] = round(8.0 * nbytes / sym.size, 4)
        rows.append(row)
    return {"shape": [M, K], "streams_per_tile": 32, "bits_per_symbol": rows,
            "kernels_take": ["8x128", "8x256", "8x512"]}


def main():
    args = parse()
    if args.compression_table:
        print(json.dumps(compression_table()), flush=True)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ecq(args)


if __name__ == "__main__":
    main()
