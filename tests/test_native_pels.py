"""Native PELS tick vs the CPU oracle (reference tests/test_native_compartmental.py:99-178)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from _util import GOLDEN, OracleMatrix, assert_same_as, bench_model, csr_of, drive_np, make, npy, params_of
from neurosim_gpu_b200 import (NativeDendriticPELSRuntime, load_native_extension,
                               random_topology)

pytestmark = pytest.mark.gpu

EPSILON = 1e-6  # emit decisions may differ only this close to the threshold


@pytest.fixture(scope="module")
def ext():
    return load_native_extension()


# test_native_compartmental.py:99-110
def test_theta_zero_long_rollout_matches_matrix(ext):
    graph, model, state = make(1024, 2, 16000)
    native = NativeDendriticPELSRuntime(graph, model, state.clone(), theta=0, extension=ext)
    reference = OracleMatrix(graph, model, state)
    with torch.inference_mode():
        for t in range(500):
            value = 0.2 if t % 70 < 35 else 0.05
            native.step(value, dendritic_drive=0.1)
            reference.step(value, 0.1)
    assert_same_as(native, reference, atol=8e-6)
    torch.testing.assert_close(native.persistent_current,
                               native._propagate(native.emitted_state), rtol=2e-4, atol=1e-5)


def _snapshot(rt):
    return {name: npy(getattr(rt, name)).copy() for name in
            ("state", "dendritic_state", "adaptation_state", "emitted_state",
             "persistent_current")}


def _teacher_forced_tick(ext, native, theta, drive, dendritic_drive, csr, params):
    """Step native once and check it against one oracle tick from the same pre-state."""
    pre = _snapshot(native)
    shape = pre["state"].shape
    with torch.inference_mode():
        native.step(drive, dendritic_drive=dendritic_drive)
    s, d, a, e, cur, active = oracle.event_tick(
        csr, pre["state"], pre["dendritic_state"], pre["adaptation_state"], params,
        pre["persistent_current"], pre["emitted_state"], np.full(shape[1], theta, np.float32),
        drive_np(drive, shape), drive_np(dendritic_drive, shape))
    ns, ne = npy(native.state), npy(native.emitted_state)
    np.testing.assert_allclose(ns, s, atol=1e-6, rtol=0)
    np.testing.assert_allclose(npy(native.dendritic_state), d, atol=1e-6, rtol=0)
    np.testing.assert_allclose(npy(native.adaptation_state), a, atol=1e-6, rtol=0)
    native_active = (ne == ns) & (ns != pre["emitted_state"])
    residual = np.abs(s - pre["emitted_state"])
    differ = native_active != active
    assert np.all(np.abs(residual[differ] - theta) <= EPSILON), "emit mask disagrees"
    if not differ.any():
        np.testing.assert_allclose(ne, e, atol=1e-6, rtol=0)
        np.testing.assert_allclose(npy(native.persistent_current), cur, atol=2e-6, rtol=0)
    return int(active.sum()), int(differ.sum())


# test_native_compartmental.py:142-164, teacher-forced tick by tick
def test_nonzero_threshold_emit_mask_agrees_tick_by_tick(ext):
    graph, model, state = make()
    native = NativeDendriticPELSRuntime(graph, model, state.clone(), theta=0.02, extension=ext)
    params = params_of(model)
    flips = 0
    for t in range(50):
        if t == 25:
            graph.apply_source_weights_(graph.weight * 0.7)
            native._refresh_current()
        _, differ = _teacher_forced_tick(ext, native, 0.02, 0.3, 0.1, csr_of(graph), params)
        flips += differ
        assert float((native.state - native.emitted_state).abs().max()) < 0.020001
        torch.testing.assert_close(native.persistent_current,
                                   native._propagate(native.emitted_state), rtol=2e-4, atol=2e-6)
    assert flips <= 2


def test_nonzero_threshold_free_run_against_reference_golden(ext):
    """The reference's own DendriticPELSRuntime(theta=0.02) trajectory (small_pels.npz)."""
    golden = np.load(GOLDEN / "small_pels.npz")
    graph, model, state = make()
    native = NativeDendriticPELSRuntime(graph, model, state.clone(), theta=0.02, extension=ext)
    with torch.inference_mode():
        for t in range(50):
            if t == 25:
                graph.apply_source_weights_(graph.weight * 0.7)
            native.step(0.3, dendritic_drive=0.1)
    for name in ("state", "dendritic_state", "adaptation_state", "emitted_state"):
        np.testing.assert_allclose(npy(getattr(native, name)), golden[name][50], atol=2e-6,
                                   rtol=2e-4, err_msg=name)


def test_statistics_are_counted_natively(ext):
    graph, model, state = make()
    native = NativeDendriticPELSRuntime(graph, model, state.clone(), theta=0.02, extension=ext)
    degree = npy(graph.out_degree)
    for _ in range(6):
        before = npy(native.emitted_state).copy()
        with torch.inference_mode():
            _, stats = native.step(0.3, collect_stats=True)
        after = npy(native.emitted_state)
        active = after != before
        assert native.last_backend == "native-stats"
        assert stats.active_neurons == int(active.sum())
        assert stats.active_edges == int((active * degree[None, :]).sum())
        assert stats.path == ("event" if stats.active_neurons else "idle")


# test_native_compartmental.py:166-178
def test_idle_updates_traces_and_retains_returned_state(ext):
    graph, model, state = make()
    native = NativeDendriticPELSRuntime(graph, model, state.clone(), theta=2, extension=ext)
    with torch.inference_mode():
        previous = native.step(0.5)
        saved = previous.clone()
        current = native.persistent_current.clone()
        first_adaptation = native.adaptation_state.clone()
        for _ in range(10):
            native.step(0.5)
    assert torch.equal(previous, saved)
    assert torch.equal(native.persistent_current, current)
    assert not torch.equal(first_adaptation, native.adaptation_state)
    _, stats = native.step(0.5, collect_stats=True)
    assert stats.path == "idle" and stats.active_edges == 0


def test_reference_call_form_with_weight_index(ext):
    """dendritic_event with (out_weight_index, in_weight), as the reference runtime calls it."""
    graph, model, state = make(300, 4, 6000)
    a = NativeDendriticPELSRuntime(graph, model, state.clone(), theta=0.0, extension=ext)
    b = NativeDendriticPELSRuntime(graph, model, state.clone(), theta=0.0, extension=ext)
    with torch.inference_mode():
        for _ in range(10):
            a.step(0.25, dendritic_drive=0.05)
            s, d, ad, e = ext.dendritic_event(
                b.state, b.dendritic_state, b.adaptation_state, b._parameters(),
                b.persistent_current, b.emitted_state, b.theta, graph.out_rowptr, graph.dst,
                graph.out_weight_index, graph.in_weight, None, 0.25, None, 0.05)
            b.state, b.dendritic_state, b.adaptation_state, b.emitted_state = s, d, ad, e
    assert_same_as(a, b, atol=1e-6)
    torch.testing.assert_close(a.persistent_current, b.persistent_current, atol=1e-6, rtol=0)


def test_theta_validation():
    graph, model, state = make()
    with pytest.raises(ValueError):
        NativeDendriticPELSRuntime(graph, model, state.clone(), theta=-1.0)
    with pytest.raises(ValueError, match="infinite"):
        NativeDendriticPELSRuntime(graph, model, state.clone(), theta=float("inf"))
    with pytest.raises(ValueError, match="FP32"):
        NativeDendriticPELSRuntime(graph, model, state.clone(), theta=0.0, precision="fp8")


@pytest.mark.parametrize("batch", [1, 8])
def test_config2_theta_zero_1000_ticks_matches_reference_matrix(ext, batch):
    """N=50k, M=1M: PELS at theta=0 against the reference matrix trajectory."""
    golden = np.load(GOLDEN / "trajectories.npz")
    n = 50000
    graph = random_topology(n, 1000000, device="cpu", seed=0).to("cuda")
    drive = torch.from_numpy(golden[f"n50000_b{batch}_drive"]).cuda()
    native = NativeDendriticPELSRuntime(graph, bench_model(n),
                                        torch.zeros(batch, n, device="cuda"), theta=0.0,
                                        extension=ext)
    with torch.inference_mode():
        for _ in range(1000):
            native.step(drive, dendritic_drive=0.1)
    sample = golden["n50000_sample_index"]
    for name in ("state", "dendritic_state", "adaptation_state"):
        got = npy(getattr(native, name))[:, sample]
        np.testing.assert_allclose(got, golden[f"n50000_b{batch}_t1000_{name}_sample"],
                                   atol=1e-5, rtol=0, err_msg=name)


def test_config2_theta_002_teacher_forced(ext):
    n, batch = 50000, 8
    graph = random_topology(n, 1000000, device="cpu", seed=0).to("cuda")
    model = bench_model(n)
    drive = torch.rand((batch, 1), generator=torch.Generator().manual_seed(0)).cuda() * 0.4
    native = NativeDendriticPELSRuntime(graph, model, torch.zeros(batch, n, device="cuda"),
                                        theta=0.02, extension=ext)
    csr, params = csr_of(graph), params_of(model)
    with torch.inference_mode():
        for _ in range(30):
            native.step(drive, dendritic_drive=0.1)
    total_flips = 0
    for _ in range(5):
        active, flips = _teacher_forced_tick(ext, native, 0.02, drive, 0.1, csr, params)
        assert active > 0
        total_flips += flips
    assert total_flips <= 10


@pytest.mark.parametrize("batch", [1, 4])
def test_run_graph_equals_steps(ext, batch):
    """PELS run() (a CUDA graph of event ticks) against step(): equal up to the
    rounding of the scatter's float atomics; at theta = 0 equal to the matrix path."""
    from neurosim_gpu_b200 import NativeDendriticMatrixRuntime
    graph, model, state = make(2000, batch, 60000)
    stepped = NativeDendriticPELSRuntime(graph, model, state.clone(), theta=0.02)
    replayed = NativeDendriticPELSRuntime(graph, model, state.clone(), theta=0.02)
    exact = NativeDendriticPELSRuntime(graph, model, state.clone(), theta=0.0)
    matrix = NativeDendriticMatrixRuntime(graph, model, state.clone())
    with torch.inference_mode():
        for _ in range(70):
            stepped.step(0.2, dendritic_drive=0.1)
        replayed.run(70, 0.2, dendritic_drive=0.1, graph_ticks=16)
        exact.run(70, 0.2, dendritic_drive=0.1, graph_ticks=16)
        matrix.run(70, 0.2, dendritic_drive=0.1)
    assert replayed._tick == 70
    torch.testing.assert_close(replayed.state, stepped.state, atol=1e-5, rtol=0)
    torch.testing.assert_close(replayed.emitted_state, stepped.emitted_state, atol=1e-5, rtol=0)
    torch.testing.assert_close(exact.state, matrix.state, atol=2e-5, rtol=0)


def test_run_with_a_drive_cycle_equals_steps(ext):
    """A periodic drive: run() replays the cycle; step() with the same drives agrees."""
    import math
    graph, model, state = make(2000, 2, 60000)
    cycle = [0.2 + 0.1 * math.sin(0.11 * t) for t in range(16)]
    stepped = NativeDendriticPELSRuntime(graph, model, state.clone(), theta=0.02)
    replayed = NativeDendriticPELSRuntime(graph, model, state.clone(), theta=0.02)
    with torch.inference_mode():
        for t in range(48):
            stepped.step(cycle[t % 16], dendritic_drive=0.1)
        replayed.run(48, cycle, dendritic_drive=0.1, graph_ticks=16)
    torch.testing.assert_close(replayed.state, stepped.state, atol=1e-5, rtol=0)
    with pytest.raises(ValueError, match="cycle"):
        replayed.run(20, cycle, dendritic_drive=0.1, graph_ticks=16)


# --- hybrid propagation (B = 1): scatter below the gate, tiled W @ delta above it ---

def test_hybrid_theta_zero_through_the_tiled_propagation_equals_the_matrix_tick(ext):
    """theta = 0: every neuron emits, so every tick is above any gate below M and
    the deltas are propagated by the tiled kernel; the tick equals the matrix tick."""
    n = 20000
    graph = random_topology(n, 400000, device="cpu", seed=8).to("cuda")
    model = bench_model(n)
    initial = torch.rand(1, n, generator=torch.Generator().manual_seed(2)).cuda()
    pels = NativeDendriticPELSRuntime(graph, model, initial.clone(), theta=0.0,
                                      propagation="hybrid", hybrid_gate=0.5)
    assert pels.propagation_path == "hybrid"
    reference = OracleMatrix(graph, model, initial)
    with torch.inference_mode():
        for _ in range(40):
            pels.step(0.2, dendritic_drive=0.1)
            reference.step(0.2, 0.1)
        pels.run(64, 0.2, dendritic_drive=0.1, graph_ticks=32)
    for _ in range(64):
        reference.step(0.2, 0.1)
    assert_same_as(pels, reference, atol=8e-6, rtol=0)
    pels.check_status()


@pytest.mark.parametrize("gate", [1e-6, 0.05, 1.0])
def test_hybrid_theta_nonzero_matches_the_event_path(ext, gate):
    """theta = 0.02 under the reference's sinusoidal drive: light ticks take the
    scatter and heavy ones the tiled kernel (gate 0.05); all tiled (1e-6) or all
    scatter (1.0).  Equal to the event path for the first ticks; afterwards the
    persistent current stays W @ emitted."""
    import math
    n = 20000
    graph = random_topology(n, 400000, device="cpu", seed=8).to("cuda")
    model = bench_model(n)
    initial = torch.rand(1, n, generator=torch.Generator().manual_seed(4)).cuda()
    hybrid = NativeDendriticPELSRuntime(graph, model, initial.clone(), theta=0.02,
                                        propagation="hybrid", hybrid_gate=gate)
    event = NativeDendriticPELSRuntime(graph, model, initial.clone(), theta=0.02,
                                       propagation="event")
    assert event.propagation_path == "event"
    drive = [0.2 + 0.1 * math.sin(0.11 * t) for t in range(32)]
    with torch.inference_mode():
        for t in range(4):
            hybrid.step(drive[t], dendritic_drive=0.1)
            event.step(drive[t], dendritic_drive=0.1)
    for name in ("state", "dendritic_state", "adaptation_state", "emitted_state",
                 "persistent_current"):
        torch.testing.assert_close(getattr(hybrid, name), getattr(event, name), atol=2e-6,
                                   rtol=0, msg=name)
    with torch.inference_mode():
        hybrid.run(64, drive, dendritic_drive=0.1, graph_ticks=32)
    want = oracle.spmv(csr_of(graph), npy(hybrid.emitted_state))
    np.testing.assert_allclose(npy(hybrid.persistent_current), want, atol=2e-5, rtol=0)
    hybrid.check_status()


def test_hybrid_is_for_single_batches(ext):
    graph, model, state = make(500, 2, 5000)
    with pytest.raises(ValueError, match="B = 1"):
        NativeDendriticPELSRuntime(graph, model, state, theta=0.02,
                                   propagation="hybrid").step(0.2)
    with pytest.raises(ValueError, match="propagation"):
        NativeDendriticPELSRuntime(graph, model, state, theta=0.02, propagation="matrix")
    auto = NativeDendriticPELSRuntime(graph, model, state[:1].clone(), theta=0.02)
    assert auto.propagation_path == "event"  # below 2^20 edges the scatter does every tick
