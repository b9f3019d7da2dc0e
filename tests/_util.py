"""Helpers shared by the tests: model builders and oracle adapters."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

import oracle
from neurosim_gpu_b200 import DendriticDynamics, Dynamics, random_topology

GOLDEN = Path(__file__).resolve().parent / "golden"


def make(n=97, batch=3, edges=600, device="cuda", seed=83):
    """The reference test fixture (tests/test_native_compartmental.py:25-33)."""
    graph = random_topology(n, edges, device="cpu", seed=seed).to(device)
    soma = Dynamics(torch.linspace(0.4, 0.95, n, device=device),
                    torch.full((n,), 0.8, device=device))
    model = DendriticDynamics.from_time_constants(
        soma, dt=1, tau_dendrite=torch.linspace(2, 8, n), tau_adaptation=25,
        coupling=0.6, adaptation_strength=0.3)
    state = torch.full((batch, n), 0.2, device=device)
    return graph, model, state


def bench_model(n, device="cuda", alpha=0.72, gain=0.8, tau_d=4.0, tau_a=25.0, c=0.5, k=0.2):
    """The benchmark parameters (simulate.py:36-42, 67-73)."""
    soma = Dynamics(torch.full((n,), alpha, device=device), torch.full((n,), gain, device=device))
    return DendriticDynamics.from_time_constants(soma, dt=1.0, tau_dendrite=tau_d,
                                                 tau_adaptation=tau_a, coupling=c,
                                                 adaptation_strength=k)


def npy(value) -> np.ndarray:
    """A CPU numpy copy; floating tensors become float32, integer tensors keep their dtype."""
    if isinstance(value, torch.Tensor):
        value = value.detach()
        if value.is_floating_point():
            value = value.float()
        return value.cpu().numpy()
    return np.asarray(value, dtype=np.float32)


def csr_of(graph, weight=None) -> oracle.CSR:
    w = graph.in_weight if weight is None else weight
    return oracle.CSR.make(graph.n_neurons, npy(graph.in_rowptr).astype(np.int32),
                           npy(graph.in_col).astype(np.int32), npy(w))


def params_of(model) -> list[np.ndarray]:
    return [npy(p) for p in model.parameters()]


def drive_np(value, shape):
    if isinstance(value, torch.Tensor):
        return np.ascontiguousarray(np.broadcast_to(npy(value), shape))
    return np.full(shape, np.float32(value), dtype=np.float32)


class OracleMatrix:
    """The oracle stepped like a runtime (matrix tick)."""

    def __init__(self, graph, model, state, weight=None):
        self.csr = csr_of(graph, weight)
        self.params = params_of(model)
        self.s = npy(state).copy()
        self.d = np.zeros_like(self.s)
        self.a = np.zeros_like(self.s)

    def step(self, drive=0.0, dendritic_drive=0.0):
        shape = self.s.shape
        self.s, self.d, self.a = oracle.matrix_tick(self.csr, self.s, self.d, self.a, self.params,
                                                    drive_np(drive, shape),
                                                    drive_np(dendritic_drive, shape))
        return self.s


def assert_states(native, expected_s, expected_d, expected_a, atol=2e-6, rtol=2e-4):
    for name, value in (("state", expected_s), ("dendritic_state", expected_d),
                        ("adaptation_state", expected_a)):
        np.testing.assert_allclose(npy(getattr(native, name)), value, atol=atol, rtol=rtol,
                                   err_msg=name)


def assert_same_as(native, other, atol=2e-6, rtol=2e-4):
    assert_states(native, npy(other.state if hasattr(other, "state") else other.s),
                  npy(other.dendritic_state if hasattr(other, "dendritic_state") else other.d),
                  npy(other.adaptation_state if hasattr(other, "adaptation_state") else other.a),
                  atol=atol, rtol=rtol)
