"""Benchmark of the dendritic matrix tick (one JSON line on stdout).

Workload (BASELINE.json metric): N=166,000 neurons, M=24,988,875 edges
(``random_topology(166000, 25_000_000, seed=0)``, the reference generator's
stream), B=1, fp32 weights, constant drives 0.2 / 0.1.  A step is one tick.

* ``value``     synapse-updates/s = M*B / tick time, inputs resident in HBM.
                B = 1: all K ticks run in ONE persistent cooperative launch of the
                tiled kernel (the multi-tick path); other batches replay a
                captured CUDA graph of 64 ticks.
* ``e2e``       the same metric through the public API: calls of
                ``NativeDendriticMatrixRuntime.stream`` over min(K, 512) ticks,
                each of which for every tick copies its drive [B,N] from pinned
                host memory to the device, runs the tick and copies the new
                state back to pinned host memory (the median of five calls).
                At B = 1 the ticks run in rollout launches of up to 32 ticks
                (each tick reads its own drive row and writes its own state
                row); the copies of neighbouring chunks overlap the running
                chunk on two copy streams.  The calls reuse the same pinned
                buffers, so from the second warm-up call on stream() replays
                one CUDA graph of its copies and launches.
* ``roofline``  HBM roofline of the tick kernel: algorithmic bytes
                M*(w+4) + 4*(N+1) + 24*B*N per tick over the measured tick
                time, against MEASURED_PEAKS.json's hbm_gbs.  The tiled layout
                stores 2-byte column indices, so it streams fewer bytes than
                the algorithmic count (``streamed_bytes_per_tick``).
* ``cpu_baseline``  the reference's own CPU ``DendriticMatrixRuntime`` (fp32,
                ``torch.sparse.mm``) from its offline install under baseline/_ref,
                on all host cores and on one thread, with the CPU model and
                torch version; beside it the C port of the tick (oracle/, OpenMP
                over all host cores).  Each on a bounded sample of the same ticks.

``--impl reference`` times the reference's own CPU runtime alone on all host
cores (the C port when the install is absent).

``--gpus N`` (under torchrun, one rank per GPU) row-shards the graph over the
ranks; the soma vector is exchanged every tick by peer stores inside the tick
kernel over NVLink (B = 1, the tiled path), else by an NCCL all-gather.  Its
``e2e`` goes through ``ShardedDendriticMatrixRuntime.stream`` (every rank
uploads its rows' drive and downloads its rows' state every tick).  With the default
workload the graph grows with N -- N*166,000 neurons and N*25M candidate
edges, i.e. a fixed 166k-row, ~25M-edge share per GPU ("scaling": "weak"; at
N = 8 this is the 1.33M / 200M graph).  An explicit ``--workload`` is split
over the N GPUs as it is ("scaling": "strong").
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from neurosim_gpu_b200 import (DendriticDynamics, Dynamics,  # noqa: E402
                               NativeDendriticMatrixRuntime, random_topology)
from neurosim_gpu_b200.native import _outputs  # noqa: E402

WORKLOADS = {
    # name: (neurons, candidate edges, batch, precision)
    "matrix_n166k_m25M_b1_fp32": (166_000, 25_000_000, 1, "fp32"),
    "matrix_n166k_m25M_b1_nvfp4": (166_000, 25_000_000, 1, "nvfp4"),
    "matrix_n166k_m10M_b1_fp32": (166_000, 10_000_000, 1, "fp32"),
    "matrix_n166k_m10M_b1_fp16": (166_000, 10_000_000, 1, "fp16"),
    "matrix_n166k_m10M_b1_fp8": (166_000, 10_000_000, 1, "fp8"),
    "matrix_n166k_m10M_b1_nvfp4": (166_000, 10_000_000, 1, "nvfp4"),
    "matrix_n166k_m25M_b8_fp32": (166_000, 25_000_000, 8, "fp32"),
    "matrix_n50k_m1M_b8_fp32": (50_000, 1_000_000, 8, "fp32"),
    "matrix_n4096_m65k_b1_fp32": (4096, 65_536, 1, "fp32"),
    "matrix_n1000_m20k_b1_fp32": (1000, 20_000, 1, "fp32"),
    "matrix_n1330k_m200M_b1_fp32": (1_330_000, 200_000_000, 1, "fp32"),
    # PELS (event) ticks, theta = 0.02 (166k / 25M for the
    # reference's published PELS number)
    "pels_n50k_m1M_b1_t0.02": (50_000, 1_000_000, 1, "fp32"),
    "pels_n50k_m1M_b8_t0.02": (50_000, 1_000_000, 8, "fp32"),
    "pels_n166k_m25M_b1_t0.02": (166_000, 25_000_000, 1, "fp32"),
}
PELS_THETA = 0.02
DEFAULT_WORKLOAD = "matrix_n166k_m25M_b1_fp32"
WEIGHT_BYTES = {"fp32": 4.0, "fp16": 2.0, "fp8": 1.0, "nvfp4": 0.5 + 1.0 / 16.0}
FALLBACK_HBM_GBS = 6650.0
L2_FLUSH_BYTES = 256 << 20  # twice the B200's 126 MB L2
E2E_CALLS = 5  # stream() calls timed for the single-GPU e2e figure (median reported)


def algorithmic_bytes(neurons: int, edges: int, batch: int, precision: str) -> float:
    """M*(w + 4) + 4*(N+1) + 24*B*N (+4 B of global scale for fp8 / nvfp4)."""
    extra = 4 if precision in ("fp8", "nvfp4") else 0
    return edges * (WEIGHT_BYTES[precision] + 4) + 4 * (neurons + 1) + 24 * batch * neurons + extra


def hbm_peak() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    except (OSError, ValueError, KeyError):
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(workload: str) -> float | None:
    """DRAM bytes per launch recorded from an ncu capture (profiles/traffic.txt)."""
    path = ROOT / "profiles" / "traffic.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 2 and parts[0] == workload and not line.startswith("#"):
            return float(parts[1])
    return None


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while the GPU works."""

    QUERY = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int) -> None:
        self.index = index
        self.samples: list[list[str]] = []
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.index}",
                                      f"--query-gpu={self.QUERY}",
                                      "--format=csv,noheader,nounits"],
                                     capture_output=True, text=True, timeout=5).stdout
                row = [v.strip() for v in out.strip().split(",")]
                if len(row) == 7:
                    self.samples.append(row)
            except (OSError, subprocess.SubprocessError):
                pass
            self._stop.wait(0.1)

    def __enter__(self):
        self._thread.start()
        return self

    def __exit__(self, *exc) -> None:
        self._stop.set()
        self._thread.join()

    def summary(self) -> dict:
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[0]) for r in self.samples if r[0].replace(".", "").isdigit()]
        reasons = sorted({names[i] for r in self.samples for i in range(4)
                          if r[3 + i].lower() in ("active", "1")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(self.samples[0][1]) if self.samples[0][1].isdigit() else None,
                "reasons": reasons, "samples": len(self.samples)}


def bench_model(neurons: int, device) -> DendriticDynamics:
    soma = Dynamics(torch.full((neurons,), 0.72, device=device),
                    torch.full((neurons,), 0.8, device=device))
    return DendriticDynamics.from_time_constants(soma, dt=1.0, tau_dendrite=4.0,
                                                 tau_adaptation=25.0, coupling=0.5,
                                                 adaptation_strength=0.2)


def cpu_oracle_rate(graph, batch: int, seconds: float, max_ticks: int | None = None):
    """Synapse-updates/s of the C oracle tick over all host cores, bounded by time."""
    import numpy as np

    import oracle
    n = graph.n_neurons
    csr = oracle.CSR.make(n, graph.in_rowptr.cpu().numpy(), graph.in_col.cpu().numpy(),
                          graph.in_weight.detach().cpu().numpy())
    model = bench_model(n, "cpu")
    params = [p.numpy() for p in model.parameters()]
    s = np.zeros((batch, n), np.float32)
    d, a = np.zeros_like(s), np.zeros_like(s)
    u, v = np.full_like(s, 0.2), np.full_like(s, 0.1)
    s, d, a = oracle.matrix_tick(csr, s, d, a, params, u, v)  # warm caches / threads
    ticks, start = 0, time.perf_counter()
    while True:
        s, d, a = oracle.matrix_tick(csr, s, d, a, params, u, v)
        ticks += 1
        elapsed = time.perf_counter() - start
        if elapsed >= seconds or (max_ticks is not None and ticks >= max_ticks):
            break
    per_tick = elapsed / ticks
    return graph.n_edges * batch / per_tick, per_tick, ticks, oracle.max_threads()


REFERENCE_INSTALL = ROOT / "baseline" / "_ref"
TOPOLOGY_FIELDS = ("src", "dst", "weight", "out_rowptr", "in_rowptr", "in_col",
                   "out_weight_index", "in_weight")


def host_identity() -> dict:
    """CPU model, usable cores and torch version of the host that runs the CPU leg."""
    model = None
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    return {"cpu_model": model, "host_cores": cores, "torch": torch.__version__}


def reference_runtime_rate(graph, batch: int, seconds: float, max_ticks: int | None = None
                           ) -> dict | None:
    """The reference's own CPU ``DendriticMatrixRuntime`` (fp32, ``torch.sparse.mm``;
    compartmental.py:274-293), from its offline install under baseline/_ref, on the
    same graph: all host cores, then one thread, under ``inference_mode`` with 5
    warm-up ticks, the median of timed blocks of ticks.  None when the install is
    absent.  The graph is handed over as the reference's own ``SparseTopology``
    dataclass holding this run's arrays (equal, array for array, to the
    reference generator's: tests/test_topology_golden.py).
    """
    if not (REFERENCE_INSTALL / "neurosim_gpu" / "__init__.py").exists():
        return None
    if str(REFERENCE_INSTALL) not in sys.path:
        sys.path.insert(0, str(REFERENCE_INSTALL))
    import neurosim_gpu as ref

    n = graph.n_neurons
    topology = ref.SparseTopology(n_neurons=n, **{f: getattr(graph, f).detach().cpu()
                                                  for f in TOPOLOGY_FIELDS})
    soma = ref.Dynamics(torch.full((n,), 0.72), torch.full((n,), 0.8))
    model = ref.DendriticDynamics.from_time_constants(soma, dt=1.0, tau_dendrite=4.0,
                                                      tau_adaptation=25.0, coupling=0.5,
                                                      adaptation_strength=0.2)
    identity = host_identity()
    threads_before = torch.get_num_threads()
    result = {"kind": "reference", "runtime": "neurosim_gpu.DendriticMatrixRuntime (fp32)",
              "reference_version": getattr(ref, "__version__", None), **identity, "runs": []}
    try:
        for threads in (identity["host_cores"], 1):
            torch.set_num_threads(threads)
            runtime = ref.DendriticMatrixRuntime(topology, model, torch.zeros(batch, n))
            with torch.inference_mode():
                for _ in range(5):
                    runtime.step(0.2, dendritic_drive=0.1)
                blocks, ticks, start = [], 0, time.perf_counter()
                while True:
                    t0 = time.perf_counter()
                    for _ in range(4):
                        runtime.step(0.2, dendritic_drive=0.1)
                    blocks.append((time.perf_counter() - t0) / 4)
                    ticks += 4
                    if time.perf_counter() - start >= seconds or (
                            max_ticks is not None and ticks >= max_ticks):
                        break
            per_tick = statistics.median(blocks)
            result["runs"].append({"threads": threads, "ms_per_tick": per_tick * 1e3,
                                   "value": graph.n_edges * batch / per_tick, "ticks": ticks})
    finally:
        torch.set_num_threads(threads_before)
    return result


def build_graph(neurons: int, edges: int, device):
    # CPU draws (the reference's random stream), canonicalised on the GPU.
    return random_topology(neurons, edges, device="cpu", seed=0, build_device=device)


def run_reference(args, workload: str, explicit_workload: bool, world: int) -> dict:
    """The reference arm: the reference's own CPU DendriticMatrixRuntime on all host
    cores (the baseline/_ref install), each step one full tick of the same graph; the
    C port of the tick (oracle/) when the install is absent."""
    neurons, edges, batch, precision = WORKLOADS[workload]
    name = workload
    if world > 1 and not explicit_workload:
        neurons, edges = neurons * world, edges * world
        name = f"matrix_weak_n{neurons}_m{edges}_b{batch}_{precision}"
    graph = random_topology(neurons, edges, device="cpu", seed=0)
    steps = max(args.steps, 1)
    reference = reference_runtime_rate(graph, batch, seconds=30.0, max_ticks=steps)
    # The C port (oracle/, OpenMP over all host cores), reported beside it.
    port_rate, port_tick, port_ticks, port_cores = cpu_oracle_rate(graph, batch, seconds=10.0,
                                                                   max_ticks=steps)
    port = {"value": port_rate, "unit": "synapse-updates/s", "cores": port_cores, "kind": "port",
            "ms_per_tick": port_tick * 1e3, "sample": f"{port_ticks} ticks of the full graph"}
    if reference is not None:
        full = reference["runs"][0]
        rate, per_tick = full["value"], full["ms_per_tick"] * 1e-3
        baseline = {"value": rate, "unit": "synapse-updates/s", "cores": full["threads"],
                    "kind": "reference",
                    "sample": f"{full['ticks']} ticks of the full graph (median of 4-tick blocks)",
                    **{k: v for k, v in reference.items() if k != "kind"}, "port": port}
    else:
        rate, per_tick = port_rate, port_tick
        baseline = {**port, "reason": "the reference install (baseline/_ref) is absent"}
    return {
        "metric": "synapse-updates/s (M*B/tick)", "value": rate, "unit": "synapse-updates/s",
        "impl": "reference", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": per_tick * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (reference random_topology stream, seed 0)",
        "config": {"workload": name, "neurons": neurons, "edges": graph.n_edges,
                   "batch": batch, "weights": "fp32"},
        "cpu_baseline": baseline,
        "e2e": {"value": rate, "unit": "synapse-updates/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def run_pels(args, workload: str) -> dict:
    """PELS ticks (advance + emit, active-edge scatter) replayed from a CUDA graph."""
    from neurosim_gpu_b200 import NativeDendriticPELSRuntime

    neurons, edges, batch, _ = WORKLOADS[workload]
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    graph = build_graph(neurons, edges, device)
    model = bench_model(neurons, device)
    # The reference's PELS benchmark drive, 0.2 + 0.1 sin(0.11 t) (benchmarks/compartmental.py),
    # as a 64-tick cycle; at B = 8 each batch row adds its own offset drawn U[0, 0.4] - 0.2.
    chunk = 64
    offset = 0.0 if batch == 1 else ((torch.rand(batch, 1, generator=torch.Generator()
                                                 .manual_seed(0)) * 0.4 - 0.2).to(device))
    drive = [offset + 0.2 + 0.1 * math.sin(0.11 * t) for t in range(chunk)]
    runtime = NativeDendriticPELSRuntime(graph, model, torch.zeros(batch, neurons, device=device),
                                         theta=PELS_THETA, propagation=args.propagation)
    steps = max(args.steps - args.steps % chunk, chunk)
    with torch.inference_mode():
        runtime.run(max(args.warmup, chunk), drive, dendritic_drive=0.1, graph_ticks=chunk)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        runtime.run(steps, drive, dendritic_drive=0.1, graph_ticks=chunk)
        e1.record()
        e1.synchronize()
        tick_ms = e0.elapsed_time(e1) / steps
        # Activity over one drive cycle after the timed ticks (eager, with statistics).
        active_neurons = active_edges = 0
        for t in range(chunk):
            _, stats = runtime.step(drive[t], dendritic_drive=0.1, collect_stats=True)
            active_neurons += stats.active_neurons
            active_edges += stats.active_edges
        active_neurons, active_edges = active_neurons / chunk, active_edges / chunk
    m = graph.n_edges
    # Bytes of one event tick: the advance reads s, d, a, emitted, current and
    # writes s, d, a, emitted (36 B per pair); the scatter reads dst and weight
    # and read-modify-writes the current for every active edge (16 B).
    algo = 36 * batch * neurons + 16 * active_edges
    peak, peak_kind = hbm_peak()
    achieved = algo / (tick_ms * 1e-3) / 1e9
    return {
        "metric": "synapse-updates/s (M*B/tick)", "value": m * batch / (tick_ms * 1e-3),
        "unit": "synapse-updates/s", "n_gpus": 1, "steps": steps, "warmup": args.warmup,
        "ms_per_step": tick_ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (reference random_topology stream, seed 0; drive 0.2 + 0.1 sin(0.11 t) "
                "over a 64-tick cycle, dendritic 0.1)",
        "config": {"workload": workload, "neurons": neurons, "edges": m, "batch": batch,
                   "theta": PELS_THETA, "active_neurons_per_tick": active_neurons,
                   "active_edges_per_tick": active_edges,
                   "active_edge_fraction": active_edges / max(m * batch, 1),
                   "kernel_path": "pels-" + runtime.propagation_path, "ticks_per_graph": chunk},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": None,
                     "algorithmic_bytes_per_launch": algo, "peak_source": peak_kind,
                     "kernel": "event_advance_kernel + event_scatter_kernel"
                     + (" + tiled_tick_kernel (gated)" if runtime.propagation_path == "hybrid" else ""),
                     "per": "tick"},
        "gpu_launches": (3 if runtime.propagation_path == "hybrid" else 2) * steps,
    }


def run_native(args, workload: str) -> dict:
    if workload.startswith("pels_"):
        return run_pels(args, workload)
    neurons, edges, batch, precision = WORKLOADS[workload]
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    graph = build_graph(neurons, edges, device)
    model = bench_model(neurons, device)
    runtime = NativeDendriticMatrixRuntime(graph, model, torch.zeros(batch, neurons, device=device),
                                           precision=precision, kernel=args.kernel)
    chunk = 64
    path = runtime.kernel_path
    tiled = path in ("tiled", "cluster")  # one launch runs every tick
    with torch.inference_mode():
        # Warm-up (includes graph capture or the layout build, and weight packing).
        runtime.run(max(args.warmup, 1) * 1, 0.2, dendritic_drive=0.1, graph_ticks=chunk)
        # B = 1 (tiled / cluster): one launch runs all K ticks; other
        # batches replay a CUDA graph of `chunk` ticks.
        steps = max(args.steps, 1) if tiled else max(args.steps - args.steps % chunk, chunk)
        runtime.run(chunk, 0.2, dendritic_drive=0.1, graph_ticks=chunk)
        torch.cuda.synchronize()
        timed_launch = None
        if tiled:
            # The timed launch is prepared (validated, its arguments packed)
            # before the timed region, so the region holds device work only.
            u, us = runtime._drive(0.2)
            v, vs = runtime._drive(0.1, "dendritic_drive")
            _, views = _outputs(3, runtime.state)
            timed_launch = runtime._prepare(runtime.state, runtime.dendritic_state,
                                            runtime.adaptation_state, u, us, v, vs, views,
                                            ticks=steps)
        flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
        sampler = ClockSampler(torch.cuda.current_device())
        with sampler:
            # Busy pre-roll so the first samples already see the loaded clock.
            pre = time.perf_counter()
            while time.perf_counter() - pre < 0.3:
                runtime.run(chunk * 4, 0.2, dendritic_drive=0.1, graph_ticks=chunk)
                torch.cuda.synchronize()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            # An L2 flush (a write of twice the L2) before the start event: no
            # edge bytes of earlier launches stay in L2, and the device is busy
            # while the host enqueues the timed work.
            flush.zero_()
            start.record()
            if timed_launch is not None:
                timed_launch()
            else:
                runtime.run(steps, 0.2, dendritic_drive=0.1, graph_ticks=chunk)
            end.record()
            end.synchronize()
            if timed_launch is not None:
                runtime.state, runtime.dendritic_state, runtime.adaptation_state = views
            post = time.perf_counter()
            while time.perf_counter() - post < 0.3:
                runtime.run(chunk * 4, 0.2, dendritic_drive=0.1, graph_ticks=chunk)
                torch.cuda.synchronize()
        total_ms = start.elapsed_time(end)
        tick_ms = total_ms / steps

        # Launch durations bracketed one by one (eager ticks).
        events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(50)]
        for e0, e1 in events:
            e0.record()
            runtime.step(0.2, dendritic_drive=0.1)
            e1.record()
        torch.cuda.synchronize()
        launch_ms = statistics.median(e0.elapsed_time(e1) for e0, e1 in events)

        # End to end through the public API with host buffers: stream() uploads
        # every tick's drive from pinned host memory and downloads every tick's
        # state, the copies overlapping the ticks.
        e2e_steps = min(steps, 512)
        host_drives = torch.full((e2e_steps, batch, neurons), 0.2).pin_memory()
        host_states = torch.empty((e2e_steps, batch, neurons)).pin_memory()
        # Two warm-up calls with the same buffers: the first builds the rollout
        # plan (rings, streams, prepared launches), the second captures the
        # call's copies and launches into the CUDA graph the timed calls replay.
        for _ in range(2):
            runtime.stream(host_drives, host_states, dendritic_drive=0.1)
        torch.cuda.synchronize()
        calls = []  # E2E_CALLS timed calls; the median call is reported
        for _ in range(E2E_CALLS):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            wall = time.perf_counter()
            e0.record()
            runtime.stream(host_drives, host_states, dendritic_drive=0.1)
            e1.record()
            e1.synchronize()
            wall = time.perf_counter() - wall
            calls.append(max(e0.elapsed_time(e1), wall * 1e3))
        e2e_ms = statistics.median(calls) / e2e_steps

    m = graph.n_edges
    layout = runtime._tiled_layout()
    rate = m * batch / (tick_ms * 1e-3)
    peak, peak_kind = hbm_peak()
    algo = algorithmic_bytes(neurons, m, batch, precision)
    achieved = algo / (tick_ms * 1e-3) / 1e9
    result = {
        "metric": "synapse-updates/s (M*B/tick)", "value": rate, "unit": "synapse-updates/s",
        "n_gpus": 1, "steps": steps, "warmup": args.warmup, "ms_per_step": tick_ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (reference random_topology stream, seed 0; drives 0.2/0.1)",
        "config": {"workload": workload, "neurons": neurons, "edges": m, "batch": batch,
                   "weights": precision, "parallelism": "single GPU",
                   "l2": "inputs larger than L2 (edge stream %.0f MB vs 126 MB); L2 flushed "
                         "(256 MB write) before the timed launch" % (algo / 1e6),
                   **({"ticks_per_launch": steps} if tiled else {"ticks_per_graph": chunk}),
                   "kernel_path": runtime.kernel_path,
                   "column_blocks": layout.blocks if layout is not None else None,
                   "padding_fraction": round(layout.padding_fraction, 4) if layout is not None
                   else None},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": ncu_traffic(workload),
                     "algorithmic_bytes_per_launch": algo, "peak_source": peak_kind,
                     "kernel": {"tiled": "tiled_tick_kernel", "cluster": "cluster_tick_kernel"}
                     .get(path, "csr_batch_kernel" if batch > 1 else "csr_tick_kernel"),
                     "per": "tick",
                     "streamed_bytes_per_tick": (layout.stream_bytes() + 28 * batch * neurons
                                                 + 8 * layout.blocks * layout.splits * neurons
                                                 if layout is not None else None),
                     "tick_ms": tick_ms, "single_tick_launch_ms_median": launch_ms},
        "e2e": {"value": m * batch / (e2e_ms * 1e-3), "unit": "synapse-updates/s",
                "h2d_bytes_per_step": 4 * batch * neurons, "d2h_bytes_per_step": 4 * batch * neurons,
                "ms_per_step": e2e_ms, "api": "NativeDendriticMatrixRuntime.stream",
                "steps": e2e_steps, "calls": E2E_CALLS,
                "timing": "median of the calls, each timed alone (device events or wall "
                          "clock, whichever is longer)"},
        "gpu_launches": 1 if tiled else steps,
        "clocks": sampler.summary(),
    }
    if not args.skip_strong and workload == DEFAULT_WORKLOAD:
        # The multi-GPU configuration's graph on this one GPU: the T(1) of the
        # strong-scaling curve that the --gpus N lines continue.
        cpu_graph_arrays = {f: getattr(graph, f).detach().cpu() for f in TOPOLOGY_FIELDS}
        del runtime, graph
        torch.cuda.empty_cache()
        result["strong_scaling"] = strong_scaling_record(args, 1, 0, device)
        from neurosim_gpu_b200 import SparseTopology
        graph = SparseTopology(n_neurons=neurons, **cpu_graph_arrays)
    if not args.skip_cpu_baseline:
        rate_cpu, per_tick, ticks, cores = cpu_oracle_rate(graph, batch, seconds=args.cpu_seconds)
        port = {"value": rate_cpu, "unit": "synapse-updates/s", "cores": cores, "kind": "port",
                "sample": f"{ticks} ticks of the full graph ({per_tick * 1e3:.2f} ms/tick)"}
        reference = reference_runtime_rate(graph, batch, seconds=args.cpu_seconds)
        if reference is not None:
            full = reference["runs"][0]
            result["cpu_baseline"] = {
                "value": full["value"], "unit": "synapse-updates/s", "cores": full["threads"],
                "kind": "reference",
                "sample": f"{full['ticks']} ticks of the full graph ({full['ms_per_tick']:.2f} "
                          "ms/tick, median of 4-tick blocks)",
                **{k: v for k, v in reference.items() if k != "kind"}, "port": port}
        else:
            result["cpu_baseline"] = {**port, **host_identity(),
                                      "reason": "the reference install (baseline/_ref) is absent"}
    return result


def run_sharded_pels(args) -> dict:
    """Row-sharded PELS ticks on every rank of the torchrun job (strong scaling)."""
    import datetime

    import torch.distributed as dist

    from neurosim_gpu_b200.sharded import broadcast_graph
    from neurosim_gpu_b200.sharded_pels import ShardedDendriticPELSRuntime

    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=300))
    rank, world = dist.get_rank(), dist.get_world_size()
    neurons, edges, batch, _ = WORKLOADS[args.workload]
    graph = broadcast_graph(neurons, edges, seed=0, device=device)
    m = int(graph[1].numel())
    model = bench_model(neurons, device)
    chunk = 64
    offset = 0.0 if batch == 1 else ((torch.rand(batch, 1, generator=torch.Generator()
                                                 .manual_seed(0)) * 0.4 - 0.2).to(device))
    drive = [offset + 0.2 + 0.1 * math.sin(0.11 * t) for t in range(chunk)]
    runtime = ShardedDendriticPELSRuntime(graph, model, torch.zeros(batch, neurons, device=device),
                                          theta=PELS_THETA, exchange=args.exchange,
                                          propagation=args.propagation)
    steps = max(args.steps - args.steps % chunk, chunk)

    def timed(fn) -> float:
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dist.all_reduce(torch.zeros(1, device=device))  # ranks lined up on the device
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1)], device=device)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return float(ms.item())

    with torch.inference_mode():
        runtime.run(max(args.warmup - args.warmup % chunk, chunk), drive, dendritic_drive=0.1,
                    graph_ticks=chunk)
        torch.cuda.synchronize()
        sampler = ClockSampler(local_rank) if rank == 0 else None
        if sampler:
            sampler.__enter__()
        total_ms = timed(lambda: runtime.run(steps, drive, dendritic_drive=0.1, graph_ticks=chunk))
        if sampler:
            sampler.__exit__(None, None, None)
        tick_ms = total_ms / steps
        rows = runtime.shard.rows
        host_drive = torch.full((batch, rows), 0.2).pin_memory()
        host_state = torch.empty((batch, rows)).pin_memory()
        dev_drive = torch.zeros((batch, neurons), device=device)
        lo, hi = runtime.shard.lo, runtime.shard.hi
        e2e_steps = min(steps, 256)

        def e2e():
            for _ in range(e2e_steps):
                dev_drive[:, lo:hi].copy_(host_drive, non_blocking=True)
                host_state.copy_(runtime.step(dev_drive, dendritic_drive=0.1), non_blocking=True)

        e2e()
        e2e_ms = timed(e2e) / e2e_steps
    runtime.check_status()
    result = {
        "metric": "synapse-updates/s (M*B/tick)", "value": m * batch / (tick_ms * 1e-3),
        "unit": "synapse-updates/s", "n_gpus": world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": tick_ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (reference random_topology stream, seed 0; drive 0.2 + 0.1 sin(0.11 t) "
                "over a 64-tick cycle, dendritic 0.1)",
        "config": {"workload": args.workload, "neurons": neurons, "edges": m, "batch": batch,
                   "theta": PELS_THETA,
                   "parallelism": f"row-sharded x{world}, " + (
                       "deltas exchanged by peer stores inside the advance kernel (NVLink)"
                       if runtime.exchange == "peer" else "NCCL all-gather of deltas"),
                   "kernel_path": "pels-rows-" + runtime.propagation, "ticks_per_graph": chunk},
        "roofline": {"bound": "hbm", "achieved": None, "peak": hbm_peak()[0], "unit": "GB/s",
                     "frac": None, "traffic": None, "per_gpu": True,
                     "kernel": "event_rows_kernel + event_scatter_rows_kernel"
                     + (" + tiled_tick_kernel (gated)" if runtime.propagation == "hybrid" else "")},
        "e2e": {"value": m * batch / (e2e_ms * 1e-3), "unit": "synapse-updates/s",
                "h2d_bytes_per_step": 4 * batch * neurons,
                "d2h_bytes_per_step": 4 * batch * neurons, "ms_per_step": e2e_ms},
        "gpu_launches": (3 if runtime.propagation == "hybrid" else 2) * steps * world,
        "clocks": sampler.summary() if sampler else None,
    }
    runtime.release_graphs()
    runtime.close()
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()
    return result if rank == 0 else None


STRONG_GRAPH = (1_330_000, 200_000_000)  # the scaled graph of the multi-GPU configuration


def strong_scaling_record(args, world: int, rank: int, device) -> dict | None:
    """The 1.33M / 200M graph (fp32, B = 1) on this run's ``world`` GPUs, so that
    every line of a 1 -> N curve carries the same graph: ms/tick, synapse-updates/s
    and the per-GPU HBM fraction.  One GPU: the single-GPU runtime; N GPUs: rows
    split over the ranks with the fused peer exchange.  ``--steps`` ticks in one
    persistent launch per rank, timed on the device (max over ranks), after an
    L2 flush and a warm-up launch of the same length.  Rank 0 returns the record."""
    import torch.distributed as dist

    neurons, edges = STRONG_GRAPH
    ticks = max(args.steps, 1)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world == 1:
        graph = build_graph(neurons, edges, device)
        m = graph.n_edges
        runtime = NativeDendriticMatrixRuntime(graph, bench_model(neurons, device),
                                               torch.zeros(1, neurons, device=device))
        with torch.inference_mode():
            runtime.run(ticks, 0.2, dendritic_drive=0.1)  # warm-up (builds the layout)
            u, us = runtime._drive(0.2)
            v, vs = runtime._drive(0.1, "dendritic_drive")
            _, views = _outputs(3, runtime.state)
            launch = runtime._prepare(runtime.state, runtime.dendritic_state,
                                      runtime.adaptation_state, u, us, v, vs, views, ticks=ticks)
            torch.cuda.synchronize()
            flush.zero_()
            e0.record()
            launch()
            e1.record()
            e1.synchronize()
            runtime.check_status()
        tick_ms = e0.elapsed_time(e1) / ticks
        rows, local_edges = neurons, m
        layout = runtime._tiled_layout()
        blocks = layout.blocks if layout is not None else None
        path = runtime.kernel_path
        del runtime, graph
    else:
        from neurosim_gpu_b200.sharded import ShardedDendriticMatrixRuntime, broadcast_graph
        graph = broadcast_graph(neurons, edges, seed=0, device=device)
        m = int(graph[1].numel())
        runtime = ShardedDendriticMatrixRuntime(graph, bench_model(neurons, device),
                                                torch.zeros(1, neurons, device=device))
        with torch.inference_mode():
            runtime.run(ticks, 0.2, dendritic_drive=0.1)  # warm-up (same launch length)
            launch = (runtime.prepare_run(ticks, 0.2, dendritic_drive=0.1)
                      if runtime.exchange == "peer" else None)
            torch.cuda.synchronize()
            dist.barrier()
            dist.all_reduce(torch.zeros(1, device=device))  # ranks lined up on the device
            flush.zero_()
            e0.record()
            if launch is not None:
                launch()
            else:
                runtime.run(ticks, 0.2, dendritic_drive=0.1)
            e1.record()
            e1.synchronize()
            runtime.check_status()
        elapsed = torch.tensor([e0.elapsed_time(e1)], device=device)
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
        tick_ms = float(elapsed.item()) / ticks
        rows, local_edges = runtime.shard.rows, runtime.local_edges
        blocks = runtime.layout.blocks if runtime.layout is not None else None
        path = f"{runtime.kernel_path}, {runtime.exchange} exchange"
        runtime.release_graphs()
        runtime.close()
        del runtime, graph
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    peak, peak_kind = hbm_peak()
    per_gpu = algorithmic_bytes(rows, local_edges, 1, "fp32")
    return {"graph": "matrix_n1330k_m200M_b1_fp32", "neurons": neurons, "edges": m,
            "n_gpus": world, "ticks": ticks, "ms_per_tick": tick_ms,
            "value": m / (tick_ms * 1e-3), "unit": "synapse-updates/s",
            "kernel_path": path, "column_blocks": blocks,
            "rank0_rows": rows, "rank0_edges": local_edges,
            "hbm_frac_per_gpu": per_gpu / (tick_ms * 1e-3) / 1e9 / peak,
            "peak_source": peak_kind,
            "note": "strong scaling: the same graph at every N; T(1) / T(N) is the speed-up"}


def run_sharded(args, explicit_workload: bool) -> dict:
    """Row-sharded ticks on every rank of the torchrun job; rank 0 reports."""
    import datetime

    import torch.distributed as dist

    from neurosim_gpu_b200.sharded import ShardedDendriticMatrixRuntime, broadcast_graph

    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", device_id=device,
                            timeout=datetime.timedelta(seconds=300))
    rank, world = dist.get_rank(), dist.get_world_size()
    neurons, edges, batch, precision = WORKLOADS[args.workload]
    if explicit_workload:
        scaling, name = "strong", args.workload
    else:
        neurons, edges = neurons * world, edges * world
        scaling = "weak"
        name = f"matrix_weak_n{neurons}_m{edges}_b{batch}_{precision}"
    graph = broadcast_graph(neurons, edges, seed=0, device=device)
    m = int(graph[1].numel())
    model = bench_model(neurons, device)
    runtime = ShardedDendriticMatrixRuntime(graph, model, torch.zeros(batch, neurons, device=device),
                                            precision=precision, exchange=args.exchange)
    chunk = 32
    steps = max(args.steps, 1)  # exactly K ticks are timed
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)

    align = torch.zeros(1, device=device)

    def timed(fn, flush_first: bool = False) -> float:
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        # A one-float all-reduce on the stream lines the ranks' streams up on
        # the device (the host barrier releases the ranks tens of us apart); the
        # flush behind it takes equally long everywhere and gives the host the
        # time to enqueue the timed work before the stream reaches it.
        dist.all_reduce(align)
        if flush_first:
            flush.zero_()
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1)], device=device)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return float(ms.item())

    with torch.inference_mode():
        runtime.run(max(args.warmup, chunk), 0.2, dendritic_drive=0.1, graph_ticks=chunk)
        runtime.run(steps, 0.2, dendritic_drive=0.1, graph_ticks=chunk)  # same length, untimed
        torch.cuda.synchronize()
        sampler = ClockSampler(local_rank) if rank == 0 else None
        if sampler:
            sampler.__enter__()
        if runtime.exchange == "peer":
            # The persistent launch is prepared (a cross-rank barrier, argument
            # checks) before the timed region; an L2 flush precedes it.
            launch = runtime.prepare_run(steps, 0.2, dendritic_drive=0.1)
            total_ms = timed(launch, flush_first=True)
        else:
            total_ms = timed(lambda: runtime.run(steps, 0.2, dendritic_drive=0.1,
                                                 graph_ticks=chunk), flush_first=True)
        if sampler:
            sampler.__exit__(None, None, None)
        tick_ms = total_ms / steps
        # End to end through the public stream(): every step, every rank copies its
        # rows' drive in from pinned host memory and its rows' new state back out
        # (peer exchange: rollout launches of up to 32 ticks, the copies overlapping
        # them; NCCL exchange: one step() per tick).
        rows = runtime.shard.rows
        e2e_steps = min(steps, 512)
        host_drives = torch.full((e2e_steps, batch, rows), 0.2).pin_memory()
        host_states = torch.empty((e2e_steps, batch, rows)).pin_memory()
        runtime.stream(host_drives[:8], host_states[:8], dendritic_drive=0.1)
        e2e_ms = timed(lambda: runtime.stream(host_drives, host_states,
                                              dendritic_drive=0.1)) / e2e_steps
    runtime.check_status()
    layout = runtime.layout
    local_algo = algorithmic_bytes(rows, runtime.local_edges, batch, precision)
    peak, peak_kind = hbm_peak()
    achieved = local_algo / (tick_ms * 1e-3) / 1e9
    result = {
        "metric": "synapse-updates/s (M*B/tick)", "value": m * batch / (tick_ms * 1e-3),
        "unit": "synapse-updates/s", "n_gpus": world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": tick_ms, "higher_is_better": True, "scaling": scaling,
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (reference random_topology stream, seed 0; drives 0.2/0.1)",
        "config": {"workload": name, "neurons": neurons, "edges": m, "batch": batch,
                   "weights": precision,
                   "parallelism": f"row-sharded x{world}, " + (
                       "soma exchange by peer stores inside the tick kernel (NVLink)"
                       if runtime.exchange == "peer" else "NCCL all-gather"),
                   "l2": "inputs larger than L2", "kernel_path": runtime.kernel_path,
                   "column_blocks": layout.blocks if layout is not None else None,
                   "ticks_per_graph": chunk},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": None, "per_gpu": True,
                     "algorithmic_bytes_per_launch": local_algo, "peak_source": peak_kind,
                     "kernel": "tiled_tick_kernel" if layout is not None else "csr_tick_kernel"},
        "e2e": {"value": m * batch / (e2e_ms * 1e-3), "unit": "synapse-updates/s",
                "h2d_bytes_per_step": 4 * batch * neurons, "d2h_bytes_per_step": 4 * batch * neurons,
                "ms_per_step": e2e_ms, "api": "ShardedDendriticMatrixRuntime.stream",
                "steps": e2e_steps},
        "gpu_launches": world if runtime.exchange == "peer" else steps * world,
        "clocks": sampler.summary() if sampler else None,
    }
    runtime.release_graphs()
    runtime.close()
    del runtime, graph
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    if not args.skip_strong:
        strong = strong_scaling_record(args, world, rank, device)
        if strong is not None:
            result["strong_scaling"] = strong
    dist.barrier()
    dist.destroy_process_group()
    return result


def run_profile(args, workload: str) -> None:
    """Eager launches only (no graph, no copies, no CPU leg): the command ncu captures.

    ``--warmup`` launches run first, then ``--steps`` launches; each launch is one
    tick, or ``--launch-ticks`` ticks of the persistent tiled kernel, so
    ``ncu -s <warmup> -c <n>`` selects launches.
    """
    neurons, edges, batch, precision = WORKLOADS[workload]
    device = torch.device("cuda", 0)
    if args.profile_shard:
        run_profile_shard(args, workload, device)
        return
    graph = build_graph(neurons, edges, device)
    runtime = NativeDendriticMatrixRuntime(graph, bench_model(neurons, device),
                                           torch.zeros(batch, neurons, device=device),
                                           precision=precision)
    with torch.inference_mode():
        runtime._weights()  # pack reduced-precision weights before the counted launches
        runtime._tiled_layout()
        torch.cuda.synchronize()
        for _ in range(args.warmup + args.steps):
            if args.launch_ticks > 1:
                runtime.run(args.launch_ticks, 0.2, dendritic_drive=0.1)
            else:
                runtime.step(0.2, dendritic_drive=0.1)
    torch.cuda.synchronize()
    print(json.dumps({"profile": workload, "ticks": args.warmup + args.steps,
                      "state_mean": float(runtime.state.mean())}))


def run_profile_shard(args, workload: str, device) -> None:
    """``--profile-shard R/W``: rank R's share of a W-way row split of the
    workload's graph, built and launched on one GPU.  With ``--launch-ticks``
    above 1, persistent launches with the in-kernel exchange over a world of
    one (what each rank of a W-GPU run launches, minus the stores to and the
    wait for the other ranks); else one-tick launches of the rank's kernel
    without an exchange.  Only the rank's destination CSR and layout stay on
    the device."""
    from neurosim_gpu_b200.sharded import ShardedDendriticMatrixRuntime

    rank, world = (int(v) for v in args.profile_shard.split("/"))
    neurons, edges, batch, precision = WORKLOADS[workload]
    graph = build_graph(neurons, edges, device)
    csr = (graph.in_rowptr.to(device), graph.in_col.to(device), graph.in_weight.to(device))
    del graph
    runtime = ShardedDendriticMatrixRuntime(csr, bench_model(neurons, device),
                                            torch.zeros(batch, neurons, device=device),
                                            precision=precision, rank=rank, world=world)
    del csr
    torch.cuda.synchronize()
    torch.cuda.empty_cache()  # release the graph build's blocks before the captured launches
    with torch.inference_mode():
        if args.launch_ticks > 1:
            us_per_tick = _profile_shard_runs(args, runtime)
        else:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            for i in range(args.warmup + args.steps):
                if i == args.warmup:
                    e0.record()
                runtime.finish(runtime.local_step(0.2, dendritic_drive=0.1))
            e1.record()
            e1.synchronize()
            us_per_tick = e0.elapsed_time(e1) * 1e3 / max(args.steps, 1)
    torch.cuda.synchronize()
    runtime.check_status()
    layout = runtime.layout
    print(json.dumps({"profile": workload, "shard": args.profile_shard,
                      "rows": runtime.shard.rows, "edges": runtime.local_edges,
                      "kernel_path": runtime.kernel_path,
                      "column_blocks": layout.blocks if layout is not None else None,
                      "splits": layout.splits if layout is not None else None,
                      "slots": layout.n_slots if layout is not None else None,
                      "padding_fraction": layout.padding_fraction if layout is not None else None,
                      "tasks": layout.n_tasks if layout is not None else None,
                      "ticks_per_launch": args.launch_ticks,
                      "us_per_tick_diagnostic": us_per_tick,
                      "launches": args.warmup + args.steps,
                      "state_mean": float(runtime.state.mean())}))


def _profile_shard_runs(args, runtime) -> float:
    """Persistent launches of ``--launch-ticks`` ticks of one rank's share with
    the in-kernel exchange over a world of one: the rank stores its rows' new
    state into its own gathered buffer only and its end-of-tick barrier counts
    its own arrivals, so every other step of an N-GPU rank's launch runs as it
    does there (the stores to N - 1 peers and the wait for them excepted)."""
    from neurosim_gpu_b200.native import _PeerExchange

    shard = runtime.shard
    counter = torch.zeros(32, dtype=torch.int64, device=shard.device)
    u, us, v, vs = runtime._drives(0.2, 0.1)
    epoch = 0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for i in range(args.warmup + args.steps):
        if i == args.warmup:
            e0.record()
        x = _PeerExchange()
        x.world, x.rank, x.row_offset = 1, 0, shard.lo
        cur = shard.current
        x.gathered[0][0] = shard.buffers[cur].data_ptr()
        x.gathered[0][1] = shard.buffers[1 - cur].data_ptr()
        x.counters[0] = counter.data_ptr()
        x.epoch = epoch
        s_rows = shard.own(cur)
        out_d = torch.empty_like(runtime.dendritic_state)
        out_a = torch.empty_like(runtime.adaptation_state)
        runtime.extension.prepare_run_tiled_peers(
            s_rows, runtime.dendritic_state, runtime.adaptation_state, runtime.params,
            runtime.layout, u, us, v, vs, out=(s_rows, out_d, out_a), ticks=args.launch_ticks,
            exchange=x, status=runtime.status)()
        runtime.dendritic_state, runtime.adaptation_state = out_d, out_a
        shard.current = (cur + args.launch_ticks) % 2
        epoch += args.launch_ticks
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) * 1e3 / max(args.steps * args.launch_ticks, 1)


def run_profile_suite(args) -> None:
    """Two launches of each kernel that is not the headline's, on small cases, in
    a fixed order; the second launch of each runs inside an NVTX range named
    ``measure`` (``ncu --nvtx --nvtx-include measure/`` captures just those):

    1. cluster_tick_kernel: config 1 (4,096 / 65k), 64 ticks per launch;
    2. event_advance_kernel + event_scatter_kernel: PELS at 50k / 1M, theta 0.02,
       the reference's sinusoidal drive (a warmed-up, active state);
    3. event_rows_kernel + event_scatter_rows_kernel: the row-sharded PELS tick
       of one rank holding all rows (no exchange), same graph and drive;
    4. amax_kernel + fp8_kernel, amax_kernel + nvfp4_kernel: the weight
       encoders on 40M weights (160 MB, larger than L2).
    """
    from neurosim_gpu_b200 import NativeDendriticPELSRuntime, encode_sparse_weights
    from neurosim_gpu_b200.sharded_pels import ShardedDendriticPELSRuntime

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    drive = [0.2 + 0.1 * math.sin(0.11 * t) for t in range(64)]
    with torch.inference_mode():
        small = build_graph(4096, 65_536, device)
        cluster = NativeDendriticMatrixRuntime(small, bench_model(4096, device),
                                               torch.zeros(1, 4096, device=device))
        assert cluster.kernel_path == "cluster"
        nvtx = torch.cuda.nvtx

        def measured(fn):
            torch.cuda.synchronize()
            nvtx.range_push("measure")
            fn()
            torch.cuda.synchronize()
            nvtx.range_pop()

        cluster.run(64, 0.2, dendritic_drive=0.1)  # builds the plan (one launch)
        cluster.run(64, 0.2, dendritic_drive=0.1)
        measured(lambda: cluster.run(64, 0.2, dendritic_drive=0.1))
        graph = build_graph(50_000, 1_000_000, device)
        model = bench_model(50_000, device)
        zero = torch.zeros(1, 50_000, device=device)
        pels = NativeDendriticPELSRuntime(graph, model, zero.clone(), theta=PELS_THETA)
        rows = ShardedDendriticPELSRuntime((graph.in_rowptr, graph.in_col, graph.in_weight), model,
                                           zero.clone(), theta=PELS_THETA, rank=0, world=1)
        for t in range(100):  # warm the dynamics up to the cycle's active phase, eagerly
            pels.step(drive[t % 64], dendritic_drive=0.1)
            rows.step(drive[t % 64], dendritic_drive=0.1)
        torch.cuda.synchronize()
        pels.step(drive[100 % 64], dendritic_drive=0.1)
        measured(lambda: pels.step(drive[101 % 64], dendritic_drive=0.1))
        rows.step(drive[100 % 64], dendritic_drive=0.1)
        measured(lambda: rows.step(drive[101 % 64], dendritic_drive=0.1))
        weights = torch.randn(40_000_000, device=device, generator=torch.Generator(device)
                              .manual_seed(0)) * 0.02
        for fmt in ("fp8", "nvfp4"):
            encode_sparse_weights(weights, fmt)
            measured(lambda: encode_sparse_weights(weights, fmt))
        torch.cuda.synchronize()
        marks = {"cluster_state_mean": float(cluster.state.mean()),
                 "pels_state_mean": float(pels.state.mean()),
                 "rows_state_mean": float(rows.state.mean())}
    print(json.dumps({"profile": "suite", **marks}))


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=4096)
    parser.add_argument("--warmup", type=int, default=64)
    parser.add_argument("--impl", choices=("native", "reference"), default="native")
    parser.add_argument("--workload", choices=sorted(WORKLOADS), default=None)
    parser.add_argument("--cpu-seconds", type=float, default=10.0)
    parser.add_argument("--skip-cpu-baseline", action="store_true")
    parser.add_argument("--skip-strong", action="store_true",
                        help="leave out the 1.33M / 200M strong-scaling record")
    parser.add_argument("--kernel", choices=("auto", "csr", "tiled", "cluster"), default="auto",
                        help="matrix tick path (auto: cluster for small graphs, tiled at B = 1)")
    parser.add_argument("--exchange", choices=("auto", "nccl", "peer"), default="auto",
                        help="row-sharded runs: soma / delta exchange (auto: peer stores)")
    parser.add_argument("--propagation", choices=("auto", "event", "hybrid"), default="auto",
                        help="PELS workloads: propagation of the emitted deltas (auto: the "
                             "hybrid tick at B = 1 for graphs of >= 2^20 edges)")
    parser.add_argument("--profile", action="store_true",
                        help="eager launches only, for ncu captures (prints no bench line)")
    parser.add_argument("--profile-suite", action="store_true",
                        help="two launches of each non-headline kernel on small cases, for ncu")
    parser.add_argument("--profile-shard", default=None, metavar="R/W",
                        help="with --profile: rank R's share of a W-way row split, on one GPU")
    parser.add_argument("--launch-ticks", type=int, default=1,
                        help="with --profile: ticks per launch of the persistent tiled kernel")
    args = parser.parse_args()
    explicit_workload = args.workload is not None
    if args.workload is None:
        args.workload = DEFAULT_WORKLOAD
    if args.profile_suite:
        run_profile_suite(args)
        return
    if args.profile:
        run_profile(args, args.workload)
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args, args.workload, explicit_workload,
                                           max(world, args.gpus))))
        return
    if world > 1 or args.gpus > 1:
        if args.workload.startswith("pels_"):
            result = run_sharded_pels(args)
        else:
            result = run_sharded(args, explicit_workload)
        if rank == 0:
            print(json.dumps(result))
        return
    print(json.dumps(run_native(args, args.workload)))


if __name__ == "__main__":
    main()
