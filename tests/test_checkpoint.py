"""Runtime checkpoints: the reference's format and signature, restore round trips.

tests/golden/checkpoint_ref_*.pt were written by the reference's own
``capture_runtime`` (tests/golden/make_checkpoint_fixture.py) for its CPU
dendritic runtimes; the checks follow src/neurosim_gpu/checkpoint.py:121-245.
"""

from __future__ import annotations

from pathlib import Path

import pytest
import torch

from neurosim_gpu_b200 import DendriticDynamics, Dynamics, random_topology
from neurosim_gpu_b200.checkpoint import (capture_runtime, restore_runtime, runtime_signature,
                                          load_runtime_checkpoint, save_runtime_checkpoint)
from neurosim_gpu_b200.runtime import validate_emission_threshold

GOLDEN = Path(__file__).resolve().parent / "golden"


def _model(n, device="cpu"):
    soma = Dynamics(torch.linspace(0.5, 0.9, n, device=device), torch.full((n,), 0.8, device=device))
    return DendriticDynamics.from_time_constants(soma, dt=1.0, tau_dendrite=4.0,
                                                 tau_adaptation=25.0, coupling=0.5,
                                                 adaptation_strength=0.2)


def _stub(type_name, pels):
    """A CPU object with a runtime's checkpointed attributes, named like the reference's."""
    graph = random_topology(200, 1500, device="cpu", seed=3)
    model = _model(200)
    cls = type(type_name, (), {})
    rt = cls()
    rt.topology, rt.compartment_dynamics, rt.dynamics = graph, model, model.soma
    rt.checkpoint_precision = "fp32"
    rt.state = torch.zeros(2, 200)
    rt.dendritic_state = torch.zeros(2, 200)
    rt.adaptation_state = torch.zeros(2, 200)
    if pels:
        rt.theta = validate_emission_threshold(torch.tensor(0.02), graph)
        rt.emitted_state = torch.zeros(2, 200)
        rt.persistent_current = torch.zeros(2, 200)
        rt._tick, rt._weight_version = 0, graph.weight_version
    return rt


@pytest.mark.parametrize("kind,type_name", [("matrix", "DendriticMatrixRuntime"),
                                            ("pels", "DendriticPELSRuntime")])
def test_signature_and_layout_match_the_reference(kind, type_name):
    ref = torch.load(GOLDEN / f"checkpoint_ref_{kind}.pt", weights_only=True)
    rt = _stub(type_name, kind == "pels")
    assert runtime_signature(rt) == ref["runtime_signature"]
    ours = capture_runtime(rt)
    assert set(ours) == set(ref)
    assert set(ours["tensors"]) == set(ref["tensors"])
    assert set(ours["scalars"]) == set(ref["scalars"])
    assert ours["topology"].keys() == ref["topology"].keys()
    for key in ("format", "version", "runtime_type", "precision"):
        assert ours[key] == ref[key]


@pytest.mark.parametrize("kind,type_name", [("matrix", "DendriticMatrixRuntime"),
                                            ("pels", "DendriticPELSRuntime")])
def test_restores_reference_checkpoints(kind, type_name):
    ref = torch.load(GOLDEN / f"checkpoint_ref_{kind}.pt", weights_only=True)
    rt = _stub(type_name, kind == "pels")
    restore_runtime(rt, ref)
    for name, value in ref["tensors"].items():
        assert torch.equal(getattr(rt, name), value), name
    if kind == "pels":
        assert rt._tick == 6


def _altered(change):
    ref = torch.load(GOLDEN / "checkpoint_ref_matrix.pt", weights_only=True)
    change(ref)
    return ref


@pytest.mark.parametrize("change,message", [
    (lambda p: p.update(format="x"), "format"),
    (lambda p: p.update(precision="fp8"), "precision"),
    (lambda p: p.update(runtime_type="Other"), "runtime type"),
    (lambda p: p.update(runtime_signature="0" * 64), "parameters differ"),
    (lambda p: p["tensors"].update(state=torch.zeros(3, 200)), "shape"),
    (lambda p: p["topology"]["in_col"].__setitem__(0, p["topology"]["in_col"][0] + 1), "in_col|structure"),
])
def test_rejects_incompatible_checkpoints(change, message):
    with pytest.raises(ValueError, match=message):
        restore_runtime(_stub("DendriticMatrixRuntime", False), _altered(change))


@pytest.mark.gpu
@pytest.mark.parametrize("batch", [1, 3])
def test_native_matrix_checkpoint_round_trip(tmp_path, batch):
    from neurosim_gpu_b200 import NativeDendriticMatrixRuntime
    graph = random_topology(3000, 90000, device="cpu", seed=12).to("cuda")
    model = _model(3000, "cuda")
    a = NativeDendriticMatrixRuntime(graph, model, torch.full((batch, 3000), 0.1, device="cuda"))
    with torch.inference_mode():
        a.run(7, 0.2, dendritic_drive=0.1)
    save_runtime_checkpoint(a, tmp_path / "c.pt")
    b = NativeDendriticMatrixRuntime(graph, model, torch.zeros(batch, 3000, device="cuda"))
    load_runtime_checkpoint(tmp_path / "c.pt", b)
    with torch.inference_mode():
        a.run(13, 0.2, dendritic_drive=0.1)
        b.run(13, 0.2, dendritic_drive=0.1)
    for name in ("state", "dendritic_state", "adaptation_state"):
        assert torch.equal(getattr(a, name), getattr(b, name)), name


@pytest.mark.gpu
def test_native_pels_checkpoint_round_trip(tmp_path):
    from neurosim_gpu_b200 import NativeDendriticPELSRuntime
    graph = random_topology(3000, 90000, device="cpu", seed=12).to("cuda")
    model = _model(3000, "cuda")
    a = NativeDendriticPELSRuntime(graph, model, torch.full((2, 3000), 0.1, device="cuda"),
                                   theta=0.02)
    with torch.inference_mode():
        for _ in range(7):
            a.step(0.2, dendritic_drive=0.1)
    save_runtime_checkpoint(a, tmp_path / "p.pt")
    b = NativeDendriticPELSRuntime(graph, model, torch.zeros(2, 3000, device="cuda"), theta=0.02)
    load_runtime_checkpoint(tmp_path / "p.pt", b)
    assert b._tick == a._tick
    for name in ("state", "emitted_state", "persistent_current"):
        assert torch.equal(getattr(a, name), getattr(b, name)), name
    with torch.inference_mode():
        for _ in range(5):
            a.step(0.2, dendritic_drive=0.1)
            b.step(0.2, dendritic_drive=0.1)
    # The scatter adds with float atomics, so later ticks agree to rounding only.
    torch.testing.assert_close(a.state, b.state, atol=1e-5, rtol=0)
