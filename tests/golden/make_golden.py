"""Generate the golden fixtures in this folder from the reference implementation.

This script imports the reference package (``neurosim_gpu``) from a source
checkout given by ``--reference`` (its ``src`` directory is put on
``sys.path``) and records what the reference itself computes:

* ``topology_checksums.json`` -- SHA-256 of every array of
  ``random_topology(N, M, seed)`` built on CPU (topology.py:213-247), for the
  benchmark configurations and the small test graphs;
* ``trajectories.npz`` -- DendriticMatrixRuntime states (compartmental.py:274-293)
  along rollouts of the benchmark configurations;
* ``small_matrix.npz`` -- the strided / broadcast-drive rollout of the
  reference's own native test (tests/test_native_compartmental.py:40-57);
* ``small_pels.npz`` -- DendriticPELSRuntime (theta=0.02) snapshots, one per
  tick, for teacher-forced emit-mask checks (runtime.py:225-253);
* ``precision.npz`` -- encode_sparse_weights / quantize_dequantize outputs
  (precision.py:45-112) for a set of weight vectors, plus the E4M3 cast of a
  dense value sweep.

Run (only where the reference checkout exists):
    python tests/golden/make_golden.py --reference <path-to-reference-checkout>
The fixtures are committed; nothing at test time reads the reference.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

BENCH_GRAPHS = [  # (neurons, candidate edges, seed)
    (1000, 20000, 0),
    (4096, 65536, 0),
    (50000, 1000000, 0),
    (166000, 10000000, 0),
    (166000, 25000000, 0),
]
TOPOLOGY_FIELDS = ("src", "dst", "weight", "out_rowptr", "in_rowptr", "in_col",
                   "out_weight_index", "in_weight")


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().cpu().contiguous().numpy().tobytes()).hexdigest()


def model_for(ns, n, *, alpha=0.72, gain=0.8, tau_d=4.0, tau_a=25.0, c=0.5, k=0.2):
    soma = ns.Dynamics(torch.full((n,), alpha), torch.full((n,), gain))
    return ns.DendriticDynamics.from_time_constants(
        soma, dt=1.0, tau_dendrite=tau_d, tau_adaptation=tau_a, coupling=c,
        adaptation_strength=k)


def checksums(ns, out):
    graphs = list(BENCH_GRAPHS) + [(97, 600, 83), (65, 4000, 83), (1024, 16000, 83)]
    for n, m, seed in graphs:
        g = ns.random_topology(n, m, device="cpu", seed=seed)
        out[f"{n}_{m}_{seed}"] = {"n_neurons": n, "n_edges": g.n_edges,
                                  **{f: sha(getattr(g, f)) for f in TOPOLOGY_FIELDS}}
        print("checksum", n, m, g.n_edges, flush=True)


def trajectories(ns):
    arrays = {}
    # config 0 / config 1: constant drives, zero initial state.
    for n, m, ticks, keep in ((1000, 20000, 1000, (1, 10, 100, 1000)),
                              (4096, 65536, 1000, (1, 1000))):
        g = ns.random_topology(n, m, device="cpu", seed=0)
        rt = ns.DendriticMatrixRuntime(g, model_for(ns, n), torch.zeros(1, n))
        with torch.inference_mode():
            for t in range(1, ticks + 1):
                rt.step(0.2, dendritic_drive=0.1)
                if t in keep:
                    for name in ("state", "dendritic_state", "adaptation_state"):
                        arrays[f"n{n}_t{t}_{name}"] = getattr(rt, name).numpy().copy()
        print("trajectory", n, flush=True)
    # config 2: N=50k, B=1 and B=8 (per-batch drive U[0,0.4] from seed 0).
    n = 50000
    g = ns.random_topology(n, 1000000, device="cpu", seed=0)
    sample = np.arange(0, n, 50)
    for batch in (1, 8):
        drive = torch.rand((batch, 1), generator=torch.Generator().manual_seed(0)) * 0.4
        rt = ns.DendriticMatrixRuntime(g, model_for(ns, n), torch.zeros(batch, n))
        with torch.inference_mode():
            for t in range(1, 1001):
                rt.step(drive, dendritic_drive=0.1)
        arrays[f"n50000_b{batch}_drive"] = drive.numpy()
        for name in ("state", "dendritic_state", "adaptation_state"):
            value = getattr(rt, name).numpy()
            arrays[f"n50000_b{batch}_t1000_{name}_sample"] = value[:, sample].copy()
            arrays[f"n50000_b{batch}_t1000_{name}_mean"] = value.astype(np.float64).mean(axis=1)
        print("trajectory 50k", batch, flush=True)
    arrays["n50000_sample_index"] = sample
    np.savez_compressed(HERE / "trajectories.npz", **arrays)


def small_graph(ns, n=97, batch=3, edges=600):
    # tests/test_native_compartmental.py:25-33, on CPU.
    graph = ns.random_topology(n, edges, device="cpu", seed=83)
    soma = ns.Dynamics(torch.linspace(0.4, 0.95, n), torch.full((n,), 0.8))
    model = ns.DendriticDynamics.from_time_constants(
        soma, dt=1, tau_dendrite=torch.linspace(2, 8, n), tau_adaptation=25,
        coupling=0.6, adaptation_strength=0.3)
    state = torch.full((batch, n), 0.2)
    return graph, model, state


def params_of(model):
    return np.stack([model.soma.alpha.numpy(), model.soma.gain.numpy(),
                     model.dendrite_decay.numpy(), model.adaptation_decay.numpy(),
                     model.coupling.numpy(), model.adaptation_strength.numpy()])


def small_matrix(ns):
    from dataclasses import replace
    graph, model, state = small_graph(ns)
    model = replace(model, coupling=torch.ones(194)[::2] * 0.6)
    rt = ns.DendriticMatrixRuntime(graph, model, state.clone())
    drives = [0.2, torch.tensor(0.2), torch.tensor([[0.1], [0.3], [0.5]]),
              torch.linspace(0.1, 0.3, 194)[::2]]
    arrays = {"params": params_of(model), "in_rowptr": graph.in_rowptr.numpy(),
              "in_col": graph.in_col.numpy(), "in_weight": graph.in_weight.numpy(),
              "initial": state.numpy()}
    with torch.inference_mode():
        for i, value in enumerate(drives):
            for _ in range(8):
                rt.step(value, dendritic_drive=-0.1)
            for name in ("state", "dendritic_state", "adaptation_state"):
                arrays[f"block{i}_{name}"] = getattr(rt, name).numpy().copy()
    arrays["drive2"] = drives[2].numpy()
    arrays["drive3"] = drives[3].numpy()
    np.savez_compressed(HERE / "small_matrix.npz", **arrays)


def small_pels(ns):
    graph, model, state = small_graph(ns)
    rt = ns.DendriticPELSRuntime(graph, model, state.clone(), theta=0.02, propagation="matrix")
    arrays = {"params": params_of(model), "in_rowptr": graph.in_rowptr.numpy(),
              "in_col": graph.in_col.numpy(), "weight_before": graph.in_weight.numpy().copy()}
    names = ("state", "dendritic_state", "adaptation_state", "emitted_state",
             "persistent_current")
    snaps = {name: [] for name in names}
    with torch.inference_mode():
        for t in range(51):
            if t == 25:
                graph.apply_source_weights_(graph.weight * 0.7)
            rt._refresh_current()          # snapshot the refreshed current the tick uses
            for name in names:
                snaps[name].append(getattr(rt, name).numpy().copy())
            if t < 50:
                rt.step(0.3, dendritic_drive=0.1)
    arrays["weight_after"] = graph.in_weight.numpy().copy()
    for name in names:
        arrays[name] = np.stack(snaps[name])
    np.savez_compressed(HERE / "small_pels.npz", **arrays)


def precision(ns):
    from neurosim_gpu.precision import encode_sparse_weights, quantize_dequantize
    gen = torch.Generator().manual_seed(5)
    vectors = {
        "config0": ns.random_topology(1000, 20000, device="cpu", seed=0).in_weight,
        "linspace77": torch.linspace(-3, 3, 77),
        "zeros19": torch.zeros(19),
        "one": torch.tensor([0.37]),
        "empty": torch.zeros(0),
        "normal15": torch.randn(15, generator=gen),
        "normal16": torch.randn(16, generator=gen),
        "normal17": torch.randn(17, generator=gen),
        "normal605": torch.randn(605, generator=gen) * 0.05,
        "normal4097": torch.randn(4097, generator=gen) * 3.0,
        "quarters": (torch.randint(-24, 25, (256,), generator=gen) * 0.25).float(),
        "signed_zero": torch.tensor([0.0, -0.0, 1.0, -0.0, -2.0, 0.0, 0.5, -0.25]),
        "wide_range": torch.randn(512, generator=gen) * torch.logspace(-30, 3, 512),
        "tiny": torch.full((33,), 1e-39),
    }
    arrays = {}
    for name, value in vectors.items():
        value = value.float().contiguous()
        arrays[f"{name}_value"] = value.numpy()
        for fmt in ("fp8", "nvfp4"):
            codes, scales, scale = encode_sparse_weights(value, fmt)
            arrays[f"{name}_{fmt}_codes"] = codes.numpy()
            if scales is not None:
                arrays[f"{name}_{fmt}_scales"] = scales.numpy()
            arrays[f"{name}_{fmt}_scale"] = scale.reshape(1).numpy()
        for fmt in ("fp16", "fp8", "nvfp4"):
            arrays[f"{name}_{fmt}_decoded"] = quantize_dequantize(value, fmt).numpy()
    # The E4M3 cast itself: all 256 codes, and a dense sweep with exact midpoints.
    codes = torch.arange(256, dtype=torch.uint8)
    arrays["e4m3_decode"] = codes.view(torch.float8_e4m3fn).float().numpy()
    finite = arrays["e4m3_decode"][np.isfinite(arrays["e4m3_decode"])]
    levels = np.unique(finite.astype(np.float32))
    mids = ((levels[1:].astype(np.float64) + levels[:-1]) / 2).astype(np.float32)
    sweep = np.concatenate([levels, mids, np.nextafter(mids, np.float32(np.inf)),
                            np.nextafter(mids, np.float32(-np.inf)),
                            np.linspace(-448, 448, 20001, dtype=np.float32),
                            np.float32(2.0) ** np.arange(-12, 9, dtype=np.float32)])
    sweep = sweep[np.abs(sweep) <= 448].astype(np.float32)
    arrays["e4m3_sweep"] = sweep
    arrays["e4m3_sweep_codes"] = torch.from_numpy(sweep).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.savez_compressed(HERE / "precision.npz", **arrays)


def main():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", required=True, type=Path)
    parser.add_argument("--skip-large", action="store_true")
    parser.add_argument("--huge", action="store_true",
                        help="also checksum the N=1.33M, M=200M graph (about 20 GB of host memory)")
    args = parser.parse_args()
    sys.path.insert(0, str(args.reference / "src"))
    import neurosim_gpu as ns  # noqa: E402  (reference package)
    torch.set_num_threads(8)
    if not args.huge:
        precision(ns)
        small_matrix(ns)
        small_pels(ns)
        trajectories(ns)
    path = HERE / "topology_checksums.json"
    if not args.skip_large:
        sums = {}
        checksums(ns, sums)
        path.write_text(json.dumps(sums, indent=1) + "\n")
    if args.huge:
        sums = json.loads(path.read_text())
        n, m = 1330000, 200000000
        g = ns.random_topology(n, m, device="cpu", seed=0)
        sums[f"{n}_{m}_0"] = {"n_neurons": n, "n_edges": g.n_edges,
                              **{f: sha(getattr(g, f)) for f in TOPOLOGY_FIELDS}}
        path.write_text(json.dumps(sums, indent=1) + "\n")


if __name__ == "__main__":
    main()
