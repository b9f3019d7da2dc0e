"""The small-graph cluster tick (nsb_dendritic_run_cluster) against the oracle.

One thread-block cluster of 8 CTAs runs T ticks with the state in shared
memory; every case below is checked against the CPU oracle's T ticks
(``oracle.matrix_tick``) on the same seeded inputs.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import oracle
from _util import (OracleMatrix, assert_same_as, bench_model, csr_of, drive_np, make, npy,
                   params_of)
from neurosim_gpu_b200 import (NativeDendriticMatrixRuntime, encode_sparse_weights,
                               load_native_extension, quantize_dequantize, random_topology)
from neurosim_gpu_b200 import native

CTAS = 8


def _slots_py(rowptr: np.ndarray) -> int:
    """The interleaved slot count of the widest CTA, restated in numpy."""
    n = rowptr.size - 1
    rows = -(-n // CTAS)
    rows = -(-rows // 32) * 32
    degree = np.diff(rowptr.astype(np.int64))
    degree = np.concatenate([degree, np.zeros(CTAS * rows - n, np.int64)])
    widest = degree.reshape(-1, 32).max(axis=1) * 32
    return int(widest.reshape(CTAS, -1).sum(axis=1).max())


@pytest.mark.parametrize("n,m", [(1000, 20000), (4096, 65536), (97, 600), (50, 300), (1, 0),
                                 (300, 0), (5000, 30000)])
def test_cluster_slot_count_cpu(n, m):
    """nsb_cluster_slots / nsb_cluster_smem_bytes are host functions (no GPU)."""
    lib = native.load_library()
    graph = random_topology(n, m, device="cpu", seed=0)
    rowptr = graph.in_rowptr.to(torch.int32).contiguous()
    slots = int(lib.nsb_cluster_slots(n, rowptr.data_ptr()))
    assert slots == _slots_py(rowptr.numpy())
    assert slots >= -(-m // CTAS)
    rows = -(-(-(-n // CTAS)) // 32) * 32
    head = CTAS * 8 + ((rows // 32 + 4) & ~3) * 4
    n_pad = (n + 3) & ~3
    assert lib.nsb_cluster_smem_bytes(n, slots) == head + 8 * n_pad + 44 * rows + 8 * slots
    assert lib.nsb_cluster_slots(0, rowptr.data_ptr()) == -1
    assert lib.nsb_cluster_smem_bytes(n, -1) == 0


def test_cluster_entry_point_rejects_bad_arguments_cpu():
    lib = native.load_library()
    assert lib.nsb_dendritic_run_cluster(None, None, 0, 1, None, None, None) != 0
    assert b"tick" in lib.nsb_last_error()


def _packed(graph, fmt):
    if fmt == "fp32":
        return graph.in_weight, None, None, graph.in_weight
    if fmt == "fp16":
        return graph.in_weight.half(), None, None, graph.in_weight.half().float()
    codes, scales, scale = encode_sparse_weights(graph.in_weight, fmt)
    return codes, scales, scale, quantize_dequantize(graph.in_weight, fmt)


def _oracle_ticks(graph, decoded, model, s, d, a, ticks, drive, dendritic_drive):
    csr = csr_of(graph, decoded)
    params = params_of(model)
    s, d, a = npy(s), npy(d), npy(a)
    u = drive_np(drive, s.shape)
    v = drive_np(dendritic_drive, s.shape)
    for _ in range(ticks):
        s, d, a = oracle.matrix_tick(csr, s, d, a, params, u, v)
    return s, d, a


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["fp32", "fp16", "fp8", "nvfp4"])
@pytest.mark.parametrize("n,m,ticks", [(1000, 20000, 100), (4096, 65536, 40), (97, 600, 7),
                                       (50, 300, 3), (2000, 0, 5), (777, 9000, 1)])
def test_cluster_ticks_match_oracle(fmt, n, m, ticks):
    ext = load_native_extension()
    graph = random_topology(n, m, device="cpu", seed=0).to("cuda")
    weight, scales, scale, decoded = _packed(graph, fmt)
    model = bench_model(n)
    gen = torch.Generator().manual_seed(2)
    s0 = torch.rand(1, n, generator=gen).cuda()
    d0 = (torch.rand(1, n, generator=gen) - 0.5).cuda()
    a0 = torch.rand(1, n, generator=gen).cuda()
    drive = (torch.rand(1, n, generator=gen) * 0.4).cuda()
    slots, smem = ext.cluster_plan(graph.in_rowptr)
    out = [torch.full_like(s0, float("nan")) for _ in range(3)]
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ext.prepare_run_cluster(s0, d0, a0, model.parameters(), graph.in_rowptr, graph.in_col,
                            weight, drive, 0.0, None, 0.1, scales, scale, out=out, ticks=ticks,
                            max_slots=slots, status=status)()
    want = _oracle_ticks(graph, decoded, model, s0, d0, a0, ticks, drive, 0.1)
    for got, exp in zip(out, want):
        np.testing.assert_allclose(npy(got), exp, atol=1e-5, rtol=0)
    assert int(status.item()) == 0


@pytest.mark.gpu
def test_cluster_writes_strided_outputs_and_reads_strided_state():
    ext = load_native_extension()
    n = 1000
    graph = random_topology(n, 20000, device="cpu", seed=0).to("cuda")
    model = bench_model(n)
    base = torch.rand(n, 3, generator=torch.Generator().manual_seed(6)).cuda()
    s0, d0, a0 = base[:, 0].reshape(1, n), base[:, 1].reshape(1, n), base[:, 2].reshape(1, n)
    assert s0.stride(1) == 3
    wide = torch.zeros(1, 2 * n, device="cuda")
    out = [wide[:, ::2], torch.empty(1, n, device="cuda"), torch.empty(1, n, device="cuda")]
    slots, _ = ext.cluster_plan(graph.in_rowptr)
    ext.prepare_run_cluster(s0, d0, a0, model.parameters(), graph.in_rowptr, graph.in_col,
                            graph.in_weight, None, 0.2, None, 0.1, out=out, ticks=10,
                            max_slots=slots)()
    want = _oracle_ticks(graph, graph.in_weight, model, s0, d0, a0, 10, 0.2, 0.1)
    for got, exp in zip(out, want):
        np.testing.assert_allclose(npy(got), exp, atol=1e-5, rtol=0)
    assert bool((wide[:, 1::2] == 0).all())


@pytest.mark.gpu
def test_cluster_too_few_slots_sets_status_and_writes_nothing():
    ext = load_native_extension()
    n = 1000
    graph = random_topology(n, 20000, device="cpu", seed=0).to("cuda")
    model = bench_model(n)
    s0 = torch.rand(1, n, generator=torch.Generator().manual_seed(2)).cuda()
    slots, _ = ext.cluster_plan(graph.in_rowptr)
    out = [torch.full_like(s0, 7.0) for _ in range(3)]
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ext.prepare_run_cluster(s0, s0, s0, model.parameters(), graph.in_rowptr, graph.in_col,
                            graph.in_weight, None, 0.2, None, 0.1, out=out, ticks=5,
                            max_slots=slots - 32, status=status)()
    assert int(status.item()) == 7
    for view in out:
        assert bool((view == 7.0).all())


@pytest.mark.gpu
def test_cluster_rejects_batches_and_graphs_that_do_not_fit():
    ext = load_native_extension()
    graph, model, state = make(97, 2, 600)
    slots, _ = ext.cluster_plan(graph.in_rowptr)
    out = [torch.empty_like(state) for _ in range(3)]
    with pytest.raises(RuntimeError, match="B = 1"):
        ext.prepare_run_cluster(state, state, state, model.parameters(), graph.in_rowptr,
                                graph.in_col, graph.in_weight, None, 0., None, 0., out=out,
                                ticks=1, max_slots=slots)()
    big = random_topology(60000, 600000, device="cpu", seed=0).to("cuda")
    slots, smem = ext.cluster_plan(big.in_rowptr)
    assert smem > 232448
    one = torch.zeros(1, 60000, device="cuda")
    out = [torch.empty_like(one) for _ in range(3)]
    with pytest.raises(RuntimeError, match="does not fit"):
        ext.prepare_run_cluster(one, one, one, bench_model(60000).parameters(), big.in_rowptr,
                                big.in_col, big.in_weight, None, 0., None, 0., out=out,
                                ticks=1, max_slots=slots)()
    rt = NativeDendriticMatrixRuntime(big, bench_model(60000), one.clone())
    assert rt.kernel_path == "tiled"
    with pytest.raises(ValueError, match="does not fit"):
        NativeDendriticMatrixRuntime(big, bench_model(60000), one.clone(),
                                     kernel="cluster").kernel_path


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["fp32", "nvfp4"])
def test_runtime_picks_cluster_for_small_graphs(fmt):
    """Config 1 (4,096 / 65,536): run(T) == T x step() bitwise, both == oracle."""
    n = 4096
    graph = random_topology(n, 65536, device="cpu", seed=0).to("cuda")
    model = bench_model(n)
    state = torch.zeros(1, n, device="cuda")
    stepped = NativeDendriticMatrixRuntime(graph, model, state.clone(), precision=fmt)
    ran = NativeDendriticMatrixRuntime(graph, model, state.clone(), precision=fmt)
    assert ran.kernel_path == "cluster"
    reference = OracleMatrix(graph, model, state,
                             weight=quantize_dequantize(graph.in_weight, fmt))
    with torch.inference_mode():
        for _ in range(30):
            stepped.step(0.2, dendritic_drive=0.1)
            reference.step(0.2, 0.1)
        ran.run(30, 0.2, dendritic_drive=0.1)
    torch.cuda.synchronize()
    for name in ("state", "dendritic_state", "adaptation_state"):
        assert torch.equal(getattr(ran, name), getattr(stepped, name)), name
    assert_same_as(ran, reference, atol=1e-5)
    ran.check_status()
    tiled = NativeDendriticMatrixRuntime(graph, model, state.clone(), precision=fmt,
                                         kernel="tiled")
    with torch.inference_mode():
        tiled.run(30, 0.2, dendritic_drive=0.1)
    assert tiled.kernel_path == "tiled"
    assert_same_as(ran, tiled, atol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["fp32", "nvfp4"])
def test_cluster_rollout_per_tick_drives_and_history(fmt):
    """nsb_dendritic_rollout_cluster: tick k reads drive row k (rows 3 floats
    apart beyond N) and writes history row k; equal to single-tick launches
    with those drives, and to the oracle."""
    ext = load_native_extension()
    n, ticks = 1000, 11
    graph = random_topology(n, 20000, device="cpu", seed=3).to("cuda")
    weight, scales, scale, decoded = _packed(graph, fmt)
    model = bench_model(n)
    gen = torch.Generator().manual_seed(5)
    s0 = torch.rand(1, n, generator=gen).cuda()
    d0 = (torch.rand(1, n, generator=gen) - 0.5).cuda()
    a0 = torch.rand(1, n, generator=gen).cuda()
    stride = n + 3
    drives = (torch.rand(ticks * stride, generator=gen) * 0.4).cuda()
    row = [drives[k * stride: k * stride + n].view(1, n) for k in range(ticks)]
    slots, _ = ext.cluster_plan(graph.in_rowptr)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    state = (s0, d0, a0)
    singles = []
    for k in range(ticks):
        nxt = [torch.empty_like(s0) for _ in range(3)]
        ext.prepare_run_cluster(*state, model.parameters(), graph.in_rowptr, graph.in_col, weight,
                                row[k], 0.0, None, 0.1, scales, scale, out=nxt, ticks=1,
                                max_slots=slots, status=status)()
        state = nxt
        singles.append(nxt[0])
    out = [torch.empty_like(s0) for _ in range(3)]
    history = torch.full((ticks, 1, n), float("nan"), device="cuda")
    ext.prepare_run_cluster(s0, d0, a0, model.parameters(), graph.in_rowptr, graph.in_col, weight,
                            row[0], 0.0, None, 0.1, scales, scale, out=out, ticks=ticks,
                            max_slots=slots, status=status, rollout=(stride, history))()
    torch.cuda.synchronize()
    for got, want in zip(out, state):
        assert torch.equal(got, want)
    for k in range(ticks):
        assert torch.equal(history[k], singles[k]), k
    assert int(status.item()) == 0
    csr, params = csr_of(graph, decoded), params_of(model)
    s, d, a = npy(s0), npy(d0), npy(a0)
    for k in range(ticks):
        s, d, a = oracle.matrix_tick(csr, s, d, a, params, npy(row[k]), np.full_like(s, 0.1))
        np.testing.assert_allclose(npy(history[k]), s, atol=1e-5, rtol=0)
