"""Native matrix tick vs the CPU oracle and the reference's golden trajectories.

Mirrors tests/test_native_compartmental.py of the reference (file:line cited
per test), with the CPU oracle (oracle/) as the checker in place of the
PyTorch reference runtime.  All tests here run the CUDA library.
"""

from __future__ import annotations

from dataclasses import replace

import numpy as np
import pytest
import torch

import oracle
from _util import (GOLDEN, OracleMatrix, assert_same_as, assert_states, bench_model, make,
                   npy)
from neurosim_gpu_b200 import (NativeDendriticMatrixRuntime, NativeDendriticPELSRuntime,
                               SparseTopology, load_native_extension, quantize_dequantize,
                               random_topology)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ext():
    return load_native_extension()


# test_native_compartmental.py:40-57
@pytest.mark.parametrize("width", [8, 16, 32])
def test_matrix_widths_and_strided_broadcast_inputs(ext, width):
    graph, model, state = make()
    state = state.T.contiguous().T                      # column-major state
    model = replace(model, coupling=torch.ones(194, device="cuda")[::2] * 0.6)  # strided
    native = NativeDendriticMatrixRuntime(graph, model, state.clone(), threads_per_row=width,
                                          extension=ext)
    reference = OracleMatrix(graph, model, state)
    golden = np.load(GOLDEN / "small_matrix.npz")
    drives = [0.2, torch.tensor(0.2, device="cuda"),
              torch.tensor([[0.1], [0.3], [0.5]], device="cuda"),
              torch.linspace(0.1, 0.3, 194, device="cuda")[::2]]
    with torch.inference_mode():
        for block, value in enumerate(drives):
            for _ in range(8):
                native.step(value, dendritic_drive=-0.1)
                reference.step(value, dendritic_drive=-0.1)
            assert_same_as(native, reference)
            # The reference's own trajectory for the same inputs.
            assert_states(native, golden[f"block{block}_state"],
                          golden[f"block{block}_dendritic_state"],
                          golden[f"block{block}_adaptation_state"])
    assert native.last_backend == "native"


@pytest.mark.parametrize("width", [4, 8, 16, 32])
def test_lane_width_of_the_c_abi(ext, width):
    graph, model, state = make(300, 5, 9000)
    native = NativeDendriticMatrixRuntime(graph, model, state.clone(), extension=ext)
    reference = OracleMatrix(graph, model, state)
    with torch.inference_mode():
        for _ in range(5):
            views = ext.dendritic_step(native.state, native.dendritic_state,
                                       native.adaptation_state, native._parameters(),
                                       graph.in_rowptr, graph.in_col, graph.in_weight, None, 0.25,
                                       None, 0.05, width)
            native.state, native.dendritic_state, native.adaptation_state = views
            reference.step(0.25, 0.05)
    assert_same_as(native, reference)


# test_native_compartmental.py:59-69
@pytest.mark.parametrize("n,batch,edges", [(1, 2, 0), (9, 0, 20), (65, 3, 4000)])
def test_empty_edges_empty_batch_and_large_degree(ext, n, batch, edges):
    graph, model, state = make(n, batch, edges)
    for kind, kwargs in ((NativeDendriticMatrixRuntime, {}),
                         (NativeDendriticPELSRuntime, {"theta": 0.0})):
        native = kind(graph, model, state.clone(), extension=ext, **kwargs)
        reference = OracleMatrix(graph, model, state)
        with torch.inference_mode():
            for _ in range(8):
                native.step(0.2)
                reference.step(0.2)
        assert_same_as(native, reference)
        assert native.state.shape == (batch, n)


# test_native_compartmental.py:71-97
@pytest.mark.parametrize("width", [8, 16, 32])
def test_fp16_weight_storage_matches_rounded_fp32_and_refreshes(ext, width):
    graph, model, state = make()
    rounded = SparseTopology.from_edges(graph.n_neurons, graph.src, graph.dst,
                                        graph.weight.half().float())
    native = NativeDendriticMatrixRuntime(graph, model, state.clone(), extension=ext,
                                          threads_per_row=width, weight_dtype=torch.float16)
    reference = NativeDendriticMatrixRuntime(rounded, model, state.clone(), extension=ext,
                                             threads_per_row=width)
    with torch.inference_mode():
        for tick in range(12):
            if tick == 6:
                graph.apply_source_weights_(graph.weight * 0.7)
                rounded.apply_source_weights_(graph.weight.half().float())
            native.step(0.2, dendritic_drive=0.1)
            reference.step(0.2, dendritic_drive=0.1)
            for field in ("state", "dendritic_state", "adaptation_state"):
                assert torch.equal(getattr(native, field), getattr(reference, field)), field
    assert native.last_backend == "native-fp16-weight"


def test_reduced_precision_is_inference_only(ext):
    graph, model, state = make()
    native = NativeDendriticMatrixRuntime(graph, model, state.clone(), extension=ext,
                                          weight_dtype=torch.float16)
    drive = torch.tensor(0.3, device="cuda", requires_grad=True)
    with pytest.raises(RuntimeError, match="inference-only"):
        native.step(drive)
    assert torch.equal(native.state, state)


# test_native_compartmental.py:112-140
@pytest.mark.parametrize("fmt", ["fp8", "nvfp4"])
@pytest.mark.parametrize("edge_count", [0, 605])
@pytest.mark.parametrize("width", [8, 16, 32])
def test_packed_weights_match_decoded_fp32(ext, fmt, edge_count, width):
    graph, model, state = make(edges=edge_count)
    if edge_count and graph.n_edges % 2 == 0:  # odd edge count: a half-filled last byte
        graph = SparseTopology.from_edges(graph.n_neurons, graph.src[:-1], graph.dst[:-1],
                                          graph.weight[:-1])
    decoded = SparseTopology.from_edges(graph.n_neurons, graph.src, graph.dst, graph.weight)
    native = NativeDendriticMatrixRuntime(graph, model, state.clone(), extension=ext,
                                          threads_per_row=width, weight_format=fmt)
    reference = NativeDendriticMatrixRuntime(decoded, model, state.clone(), extension=ext,
                                             threads_per_row=width)
    with torch.inference_mode():
        for tick in range(6):
            if tick == 3:
                graph.apply_source_weights_(graph.weight * 0.7)
            if tick in (0, 3):
                csr = quantize_dequantize(graph.in_weight, fmt)
                decoded.apply_source_weights_(csr[graph.out_weight_index.long()])
            native.step(0.2, dendritic_drive=0.1)
            reference.step(0.2, dendritic_drive=0.1)
            assert_same_as(native, reference, atol=2e-7)
    assert native.last_backend == f"native-{fmt}-weight"
    assert native.weight_storage_bytes == sum(
        v.numel() * v.element_size() for v in native._packed_weight if v is not None)


@pytest.mark.parametrize("fmt", ["fp16", "fp8", "nvfp4"])
def test_in_kernel_decode_is_bit_exact(ext, fmt):
    """One edge per row and a source of ones: the product is the decoded weight."""
    golden = np.load(GOLDEN / "precision.npz")
    for name in ("config0", "normal4097", "quarters", "signed_zero", "wide_range", "normal17"):
        value = torch.from_numpy(golden[f"{name}_value"]).cuda()
        m = value.numel()
        rowptr = torch.arange(m + 1, dtype=torch.int32, device="cuda")
        col = (torch.arange(m, dtype=torch.int32, device="cuda") * 7) % m
        ones = torch.ones(1, m, device="cuda")
        if fmt == "fp16":
            args = (value.half(),)
        else:
            from neurosim_gpu_b200 import encode_sparse_weights
            args = encode_sparse_weights(value, fmt)
        weight, scales, scale = (args + (None, None))[:3]
        got = ext.csr_propagate(rowptr, col, weight, ones, scales, scale)
        expected = golden[f"{name}_{fmt}_decoded"]
        assert np.array_equal(npy(got)[0].view(np.uint32), expected.view(np.uint32)), name


# test_native_compartmental.py:218-229
def test_parameters_remain_live_and_no_grad_can_accelerate(ext):
    graph, model, state = make()
    model = replace(model, coupling=model.coupling.clone().requires_grad_())
    native = NativeDendriticMatrixRuntime(graph, model, state.clone(), extension=ext)
    reference = OracleMatrix(graph, model, state)
    with torch.no_grad():
        for _ in range(6):
            model.coupling.mul_(0.9)
            native.step(0.2)
            reference.params = [npy(p) for p in model.parameters()]
            reference.step(0.2)
    assert_same_as(native, reference)
    assert native.last_backend == "native"


# test_native_compartmental.py:166-178 (matrix form)
def test_returned_states_are_fresh_allocations(ext):
    graph, model, state = make()
    native = NativeDendriticMatrixRuntime(graph, model, state.clone(), extension=ext)
    with torch.inference_mode():
        first = native.step(0.3)
        saved = first.clone()
        for _ in range(5):
            native.step(0.3)
    assert torch.equal(first, saved)


# test_native_compartmental.py:254-266
def test_invalid_inputs_fail_before_state_mutation(ext):
    graph, model, state = make()
    native = NativeDendriticMatrixRuntime(graph, model, state.clone(), extension=ext)
    for value in (torch.zeros(3, 3, 97, device="cuda"), torch.zeros(97),
                  torch.zeros(97, device="cuda", dtype=torch.float64)):
        with pytest.raises(ValueError):
            native.step(value)
        assert torch.equal(native.state, state)
    with pytest.raises(ValueError, match="threads_per_row"):
        NativeDendriticMatrixRuntime(graph, model, state, threads_per_row=7)
    with pytest.raises(RuntimeError, match="parameter"):
        ext.dendritic_step(state, state, state, [state], graph.in_rowptr, graph.in_col,
                           graph.in_weight, None, 0., None, 0., 32)
    with pytest.raises(RuntimeError, match="CSR"):
        ext.dendritic_step(state, state, state, native._parameters(), graph.in_rowptr[:-1],
                           graph.in_col, graph.in_weight, None, 0., None, 0., 32)
    with pytest.raises(RuntimeError, match="width"):
        ext.dendritic_step(state, state, state, native._parameters(), graph.in_rowptr,
                           graph.in_col, graph.in_weight, None, 0., None, 0., 7)


def test_run_graph_equals_steps(ext):
    graph, model, state = make(500, 2, 12000)
    stepped = NativeDendriticMatrixRuntime(graph, model, state.clone(), extension=ext)
    replayed = NativeDendriticMatrixRuntime(graph, model, state.clone(), extension=ext)
    drive = torch.tensor([[0.1], [0.3]], device="cuda")
    with torch.inference_mode():
        for _ in range(37):
            stepped.step(drive, dendritic_drive=0.05)
        replayed.run(37, drive, dendritic_drive=0.05, graph_ticks=8)
    for field in ("state", "dendritic_state", "adaptation_state"):
        assert torch.equal(getattr(stepped, field), getattr(replayed, field)), field


def test_autograd_requests_use_the_differentiable_tick(ext):
    """test_native_compartmental.py:180-216: gradients flow, labelled reference-autograd."""
    graph, model, state = make(17, 2, 80)
    weights = graph.weight.detach().clone().requires_grad_()
    graph = SparseTopology.from_edges(17, graph.src, graph.dst, weights)
    drive = torch.full_like(state, 0.3, requires_grad=True)
    native = NativeDendriticMatrixRuntime(graph, model, state.clone(), extension=ext)
    s, d, a = state.clone(), torch.zeros_like(state), torch.zeros_like(state)
    dense = graph.dense_matrix()
    for _ in range(4):
        native.step(drive, dendritic_drive=0.2)
        s, d, a = model.advance(s, d, a, s @ dense.T, drive, dendritic_drive=0.2)
    got = torch.autograd.grad(native.state.sum(), (weights, drive), retain_graph=True)
    want = torch.autograd.grad(s.sum(), (weights, drive))
    for g, w in zip(got, want):
        torch.testing.assert_close(g, w, atol=2e-5, rtol=2e-4)
        assert float(g.abs().sum()) > 0
    assert native.last_backend == "reference-autograd"


# --- benchmark configurations, long rollouts ---------------------------------

def _golden_rollout(ext, n, m, ticks, use_run):
    graph = random_topology(n, m, device="cpu", seed=0).to("cuda")
    native = NativeDendriticMatrixRuntime(graph, bench_model(n), torch.zeros(1, n, device="cuda"),
                                          extension=ext)
    with torch.inference_mode():
        if use_run:
            native.run(ticks, 0.2, dendritic_drive=0.1)
        else:
            for _ in range(ticks):
                native.step(0.2, dendritic_drive=0.1)
    return native


def test_config0_1000_ticks_against_reference_golden(ext):
    golden = np.load(GOLDEN / "trajectories.npz")
    native = _golden_rollout(ext, 1000, 20000, 1000, use_run=False)
    assert_states(native, golden["n1000_t1000_state"], golden["n1000_t1000_dendritic_state"],
                  golden["n1000_t1000_adaptation_state"], atol=1e-5, rtol=0)


def test_config1_1000_ticks_graph_replay_against_reference_golden(ext):
    golden = np.load(GOLDEN / "trajectories.npz")
    native = _golden_rollout(ext, 4096, 65536, 1000, use_run=True)
    assert_states(native, golden["n4096_t1000_state"], golden["n4096_t1000_dendritic_state"],
                  golden["n4096_t1000_adaptation_state"], atol=1e-5, rtol=0)


@pytest.mark.parametrize("batch", [1, 8])
def test_config2_1000_ticks_against_reference_golden(ext, batch):
    golden = np.load(GOLDEN / "trajectories.npz")
    n = 50000
    graph = random_topology(n, 1000000, device="cpu", seed=0).to("cuda")
    drive = torch.from_numpy(golden[f"n50000_b{batch}_drive"]).cuda()
    native = NativeDendriticMatrixRuntime(graph, bench_model(n),
                                          torch.zeros(batch, n, device="cuda"), extension=ext)
    with torch.inference_mode():
        native.run(1000, drive, dendritic_drive=0.1)
    sample = golden["n50000_sample_index"]
    for name in ("state", "dendritic_state", "adaptation_state"):
        got = npy(getattr(native, name))
        np.testing.assert_allclose(got[:, sample], golden[f"n50000_b{batch}_t1000_{name}_sample"],
                                   atol=1e-5, rtol=0, err_msg=name)
        np.testing.assert_allclose(got.astype(np.float64).mean(axis=1),
                                   golden[f"n50000_b{batch}_t1000_{name}_mean"], atol=1e-6)


@pytest.mark.parametrize("fmt", ["fp32", "fp16", "fp8", "nvfp4"])
def test_config3_quantized_1000_ticks_against_oracle(ext, fmt):
    """N=166k, M=10M: state within 1e-5 of the same-precision fp32 path on decoded weights."""
    n = 166000
    graph = random_topology(n, 10_000_000, device="cpu", seed=0, build_device="cuda")
    model = bench_model(n)
    native = NativeDendriticMatrixRuntime(graph, model, torch.zeros(1, n, device="cuda"),
                                          extension=ext, precision=fmt)
    decoded = quantize_dequantize(graph.in_weight, fmt)
    reference = OracleMatrix(graph, model, torch.zeros(1, n), weight=decoded)
    with torch.inference_mode():
        native.run(1000, 0.2, dendritic_drive=0.1)
    for _ in range(1000):
        reference.step(0.2, 0.1)
    assert_same_as(native, reference, atol=1e-5, rtol=0)


def test_config4_1000_ticks_against_oracle(ext):
    """N=166k, M=25M, fp32: within 1e-5 max-abs of the CPU oracle after 1,000 ticks."""
    n = 166000
    graph = random_topology(n, 25_000_000, device="cpu", seed=0, build_device="cuda")
    model = bench_model(n)
    native = NativeDendriticMatrixRuntime(graph, model, torch.zeros(1, n, device="cuda"),
                                          extension=ext)
    reference = OracleMatrix(graph, model, torch.zeros(1, n))
    with torch.inference_mode():
        native.run(1000, 0.2, dendritic_drive=0.1)
    for _ in range(1000):
        reference.step(0.2, 0.1)
    assert_same_as(native, reference, atol=1e-5, rtol=0)


@pytest.mark.parametrize("kernel,batch,n,m,ticks", [
    ("tiled", 1, 6000, 150000, 9), ("tiled", 1, 6000, 150000, 70), ("cluster", 1, 1000, 20000, 9),
    ("cluster", 1, 1000, 20000, 300), ("csr", 2, 3000, 60000, 9)])
def test_stream_equals_steps_with_the_same_drives(ext, kernel, batch, n, m, ticks):
    """stream(): host drives in, every tick's state out, copies overlapping the
    ticks (tiled and cluster: rollout launches of 4, 8, 16, ... ticks); equal
    bit for bit to step() with the same drives."""
    graph = random_topology(n, m, device="cpu", seed=5).to("cuda")
    model = bench_model(n)
    initial = torch.rand(batch, n, generator=torch.Generator().manual_seed(1)).cuda()
    drives = torch.rand(ticks, batch, n, generator=torch.Generator().manual_seed(2)) * 0.4
    if ticks > 9:
        drives = drives[:, 0]  # [T, N] drives, one row per tick
    drives = drives.pin_memory()
    stepped = NativeDendriticMatrixRuntime(graph, model, initial.clone(), kernel=kernel)
    streamed = NativeDendriticMatrixRuntime(graph, model, initial.clone(), kernel=kernel)
    assert streamed.kernel_path == kernel
    states = []
    with torch.inference_mode():
        for t in range(ticks):
            states.append(stepped.step(drives[t].cuda(), dendritic_drive=0.1).clone())
        out = streamed.stream(drives, dendritic_drive=0.1)
    torch.cuda.synchronize()
    assert out.device.type == "cpu" and out.is_pinned()
    for t in range(ticks):
        assert torch.equal(out[t], states[t].cpu()), t
    streamed.check_status()
    for name in ("state", "dendritic_state", "adaptation_state"):
        assert torch.equal(getattr(streamed, name), getattr(stepped, name)), name


@pytest.mark.parametrize("kernel,n,m", [("tiled", 6000, 150000), ("cluster", 1000, 20000)])
def test_stream_calls_reuse_their_plan(ext, kernel, n, m):
    """Consecutive stream() calls of different lengths, with step() and run() in
    between, reuse one rollout plan (rings, copy streams, prepared launches) and
    still equal step() bit for bit; states handed out earlier stay unchanged."""
    graph = random_topology(n, m, device="cpu", seed=6).to("cuda")
    model = bench_model(n)
    initial = torch.rand(1, n, generator=torch.Generator().manual_seed(3)).cuda()
    drives = (torch.rand(60, 1, n, generator=torch.Generator().manual_seed(4)) * 0.4).pin_memory()
    stepped = NativeDendriticMatrixRuntime(graph, model, initial.clone(), kernel=kernel)
    streamed = NativeDendriticMatrixRuntime(graph, model, initial.clone(), kernel=kernel)
    with torch.inference_mode():
        first = streamed.stream(drives[:20], dendritic_drive=0.1)
        kept = streamed.state
        kept_copy = kept.clone()
        plan = streamed._rollout_plan
        streamed.step(0.3, dendritic_drive=0.1)
        streamed.run(3, 0.25, dendritic_drive=0.1)
        second = streamed.stream(drives[20:], dendritic_drive=0.1)
        assert streamed._rollout_plan is plan
        states = []
        for t in range(20):
            states.append(stepped.step(drives[t].cuda(), dendritic_drive=0.1).clone())
        stepped.step(0.3, dendritic_drive=0.1)
        for _ in range(3):
            stepped.step(0.25, dendritic_drive=0.1)
        for t in range(20, 60):
            states.append(stepped.step(drives[t].cuda(), dendritic_drive=0.1).clone())
    torch.cuda.synchronize()
    assert torch.equal(kept, kept_copy)
    for t in range(60):
        got = first[t] if t < 20 else second[t - 20]
        assert torch.equal(got, states[t].cpu()), t
    for name in ("state", "dendritic_state", "adaptation_state"):
        assert torch.equal(getattr(streamed, name), getattr(stepped, name)), name
    streamed.check_status()


@pytest.mark.parametrize("kernel,n,m", [("tiled", 6000, 150000), ("cluster", 1000, 20000)])
def test_stream_replays_a_graph_for_repeated_host_buffers(ext, kernel, n, m):
    """stream() calls that reuse the same pinned drive and output buffers (refilled
    in place) replay one captured CUDA graph from the second such call on; a
    call with other buffers in between runs without it.  Every call equals
    step() bit for bit."""
    graph = random_topology(n, m, device="cpu", seed=7).to("cuda")
    model = bench_model(n)
    initial = torch.rand(1, n, generator=torch.Generator().manual_seed(5)).cuda()
    ticks = 20
    gen = torch.Generator().manual_seed(6)
    drives = torch.empty(ticks, 1, n).pin_memory()
    out = torch.empty(ticks, 1, n).pin_memory()
    stepped = NativeDendriticMatrixRuntime(graph, model, initial.clone(), kernel=kernel)
    streamed = NativeDendriticMatrixRuntime(graph, model, initial.clone(), kernel=kernel)
    captured = None
    with torch.inference_mode():
        for call in range(5):
            fresh = call == 3  # other buffers: no graph for this call
            values = torch.rand(ticks, 1, n, generator=gen) * 0.4
            if fresh:
                result = streamed.stream(values.pin_memory(), dendritic_drive=0.1)
            else:
                drives.copy_(values)
                result = streamed.stream(drives, out, dendritic_drive=0.1)
            torch.cuda.synchronize()
            plan = streamed._rollout_plan
            if call == 0:
                assert plan.graph is None
            elif call >= 1:
                assert plan.graph is not None
                captured = plan.graph if captured is None else captured
                assert plan.graph is captured  # captured once, then replayed
            got = result.clone()
            for t in range(ticks):
                want = stepped.step(values[t].cuda(), dendritic_drive=0.1)
                assert torch.equal(got[t], want.cpu()), (call, t)
            if call == 2:  # step() and run() between calls
                streamed.step(0.3, dendritic_drive=0.1)
                stepped.step(0.3, dendritic_drive=0.1)
    for name in ("state", "dendritic_state", "adaptation_state"):
        assert torch.equal(getattr(streamed, name), getattr(stepped, name)), name
    streamed.check_status()
