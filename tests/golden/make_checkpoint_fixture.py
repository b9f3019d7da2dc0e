"""Write runtime checkpoints with the reference's own checkpoint module.

The reference package (``neurosim_gpu``) is imported from the checkout given by
``--reference``.  A DendriticMatrixRuntime and a DendriticPELSRuntime (theta
0.02) on ``random_topology(200, 1500, seed=3)`` run 6 ticks and are captured
with the reference's ``capture_runtime`` (src/neurosim_gpu/checkpoint.py:121-155).
tests/test_checkpoint.py checks this package's signature and payload layout
against them and restores them.

Run (only where the reference checkout exists):
    python tests/golden/make_checkpoint_fixture.py --reference <path-to-reference-checkout>
The files are committed; nothing at test time reads the reference.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", required=True)
    args = parser.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "src"))
    from neurosim_gpu.checkpoint import capture_runtime
    from neurosim_gpu.compartmental import (DendriticDynamics, DendriticMatrixRuntime,
                                            DendriticPELSRuntime)
    from neurosim_gpu.dynamics import Dynamics
    from neurosim_gpu.topology import random_topology

    n = 200
    graph = random_topology(n, 1500, device="cpu", seed=3)
    soma = Dynamics(torch.linspace(0.5, 0.9, n), torch.full((n,), 0.8))
    model = DendriticDynamics.from_time_constants(soma, dt=1.0, tau_dendrite=4.0,
                                                  tau_adaptation=25.0, coupling=0.5,
                                                  adaptation_strength=0.2)
    state = torch.full((2, n), 0.1)
    matrix = DendriticMatrixRuntime(graph, model, state.clone())
    pels = DendriticPELSRuntime(graph, model, state.clone(), theta=0.02)
    for _ in range(6):
        matrix.step(0.2, dendritic_drive=0.1)
        pels.step(0.2, dendritic_drive=0.1)
    torch.save(capture_runtime(matrix), HERE / "checkpoint_ref_matrix.pt")
    torch.save(capture_runtime(pels), HERE / "checkpoint_ref_pels.pt")
    print("wrote", HERE / "checkpoint_ref_matrix.pt", HERE / "checkpoint_ref_pels.pt")


if __name__ == "__main__":
    main()
