"""Row-sharded PELS: the filtered out-CSR and the delta exchange on CPU (gloo),
the per-rank kernels on one GPU with the exchange done by copies."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from _util import OracleMatrix, bench_model, csr_of, npy, params_of
from neurosim_gpu_b200 import NativeDendriticPELSRuntime, random_topology
from neurosim_gpu_b200.sharded import RowShard
from neurosim_gpu_b200.sharded_pels import ShardedDendriticPELSRuntime, filtered_out_csr


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("n,m,world", [(300, 6000, 2), (1000, 20000, 3), (97, 600, 8),
                                       (5, 0, 2)])
def test_filtered_out_csr_scatters_like_the_full_product_cpu(n, m, world):
    graph = random_topology(n, m, device="cpu", seed=4)
    delta = torch.from_numpy(np.random.default_rng(2).standard_normal(n)) \
        .where(torch.rand(n, generator=torch.Generator().manual_seed(1)) < 0.3,
               torch.zeros(n, dtype=torch.float64))
    dense = torch.zeros(n, n, dtype=torch.float64)
    rows = torch.repeat_interleave(torch.arange(n), graph.in_rowptr.long().diff())
    dense[rows, graph.in_col.long()] = graph.in_weight.double()
    want = dense @ delta
    seen = 0
    for rank in range(world):
        shard = RowShard(n, 1, rank, world, torch.device("cpu"))
        rowptr, dst, weight = filtered_out_csr(graph.in_rowptr, graph.in_col, graph.in_weight,
                                               shard.lo, shard.hi, n)
        assert rowptr.dtype == dst.dtype == torch.int32 and rowptr.numel() == n + 1
        assert int(rowptr[-1]) == dst.numel() == weight.numel()
        seen += dst.numel()
        if dst.numel():
            assert int(dst.min()) >= 0 and int(dst.max()) < shard.rows
        src = torch.repeat_interleave(torch.arange(n), rowptr.long().diff())
        got = torch.zeros(shard.rows, dtype=torch.float64)
        got.index_add_(0, dst.long(), delta[src] * weight.double())
        np.testing.assert_allclose(got.numpy(), want[shard.lo: shard.hi].numpy(), atol=1e-12)
        # Within a source, destinations ascend (the reference's source-major order).
        for s in range(0, n, max(1, n // 7)):
            seg = dst[int(rowptr[s]): int(rowptr[s + 1])]
            assert bool((seg[1:] > seg[:-1]).all())
    assert seen == graph.n_edges


def _gloo_worker(rank, world, port, n, batch, theta, queue):
    """The sharded PELS algorithm with numpy kernels; the exchange over gloo."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        graph = random_topology(n, 20 * n, device="cpu", seed=5)
        csr, params = csr_of(graph), params_of(bench_model(n, device="cpu"))
        full = np.random.default_rng(1).random((batch, n)).astype(np.float32)
        shard = RowShard(n, batch, rank, world, torch.device("cpu"))
        lo, hi = shard.lo, shard.hi
        rowptr, dst, weight = (x.numpy() for x in filtered_out_csr(
            graph.in_rowptr, graph.in_col, graph.in_weight, lo, hi, n))
        s = full[:, lo:hi].copy()
        e = s.copy()
        d = np.zeros_like(s)
        a = np.zeros_like(s)
        cur = oracle.spmv(csr, full)[:, lo:hi].copy()
        rows_params = [p[lo:hi] for p in params]
        for _ in range(6):
            s, d, a = oracle.advance(cur, s, d, a, rows_params, 0.2, 0.1)
            residual = s - e
            active = np.abs(residual) >= np.float32(theta)
            delta = np.where(active, residual, np.float32(0))
            e = np.where(active, s, e)
            shard.own(0).copy_(torch.from_numpy(delta))
            shard.exchange(0)
            gathered = npy(shard.buffers[0])[:n]  # [N, B]
            for src in np.nonzero(np.any(gathered != 0, axis=1))[0]:
                span = slice(rowptr[src], rowptr[src + 1])
                for b in range(batch):
                    np.add.at(cur[b], dst[span], gathered[src, b] * weight[span])
        queue.put((rank, lo, hi, s, d, a, e, cur))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n,batch,theta", [(2, 301, 1, 0.02), (3, 500, 2, 0.0),
                                                 (2, 400, 3, 0.05)])
def test_sharded_pels_over_gloo_matches_the_oracle_event_tick(world, n, batch, theta):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, n, batch, theta, queue))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    graph = random_topology(n, 20 * n, device="cpu", seed=5)
    csr, params = csr_of(graph), params_of(bench_model(n, device="cpu"))
    s = np.random.default_rng(1).random((batch, n)).astype(np.float32)
    e = s.copy()
    d, a = np.zeros_like(s), np.zeros_like(s)
    cur = oracle.spmv(csr, s)
    thetas = np.full(n, theta, np.float32)
    for _ in range(6):
        s, d, a, e, cur, _ = oracle.event_tick(csr, s, d, a, params, cur, e, thetas, 0.2, 0.1)
    for rank, lo, hi, rs, rd, ra, re, rc in results:
        for got, want in ((rs, s), (rd, d), (ra, a), (re, e), (rc, cur)):
            np.testing.assert_allclose(got, want[:, lo:hi], atol=2e-6, rtol=0, err_msg=str(rank))


# --- one GPU: every rank's kernels, deltas moved by copies ------------------------

def _emulated(graph, model, initial, theta, world):
    return [ShardedDendriticPELSRuntime(graph, model, initial, theta=theta, rank=r, world=world)
            for r in range(world)]


def _emulated_tick(ranks, drive=0.2, dendritic=0.1):
    pending = [rt.local_advance(drive, dendritic_drive=dendritic) for rt in ranks]
    for rt in ranks:
        for other in ranks:
            lo, hi = other.shard.lo, other.shard.hi
            rt.shard.buffers[0][lo:hi] = other.shard.buffers[0][lo:hi]
    for rt, (outputs, scatter) in zip(ranks, pending):
        scatter()
        rt.adopt(outputs)


def _full(ranks, name):
    return torch.cat([getattr(rt, name) for rt in ranks], dim=1)


@pytest.mark.gpu
@pytest.mark.parametrize("world,batch", [(2, 1), (3, 2), (4, 1)])
def test_sharded_pels_theta0_equals_the_matrix_tick(world, batch):
    """theta = 0: every row emits every tick, so PELS is the matrix tick
    (the reference's test_native_compartmental.py:99-110 bound, 8e-6)."""
    n = 3001
    graph = random_topology(n, 60000, device="cpu", seed=9).to("cuda")
    model = bench_model(n)
    initial = torch.rand(batch, n, generator=torch.Generator().manual_seed(2)).cuda()
    ranks = _emulated(graph, model, initial, 0.0, world)
    reference = OracleMatrix(graph, model, initial)
    with torch.inference_mode():
        for _ in range(60):
            _emulated_tick(ranks)
            reference.step(0.2, 0.1)
    torch.cuda.synchronize()
    for name, want in (("state", reference.s), ("dendritic_state", reference.d),
                       ("adaptation_state", reference.a)):
        np.testing.assert_allclose(npy(_full(ranks, name)), want, atol=8e-6, rtol=0,
                                   err_msg=name)


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 3])
def test_sharded_pels_matches_one_gpu_and_keeps_the_current_consistent(world):
    n, batch = 5000, 2
    graph = random_topology(n, 150000, device="cpu", seed=3).to("cuda")
    model = bench_model(n)
    initial = torch.rand(batch, n, generator=torch.Generator().manual_seed(6)).cuda()
    ranks = _emulated(graph, model, initial, 0.02, world)
    single = NativeDendriticPELSRuntime(graph, model, initial.clone(), theta=0.02)
    with torch.inference_mode():
        for _ in range(4):
            _emulated_tick(ranks)
            single.step(0.2, dendritic_drive=0.1)
    torch.cuda.synchronize()
    for name in ("state", "dendritic_state", "adaptation_state", "emitted_state",
                 "persistent_current"):
        np.testing.assert_allclose(npy(_full(ranks, name)), npy(getattr(single, name)),
                                   atol=2e-6, rtol=0, err_msg=name)
    with torch.inference_mode():
        for _ in range(40):
            _emulated_tick(ranks)
    # The invariant of the persistent current: current == W @ emitted.
    emitted = _full(ranks, "emitted_state")
    want = oracle.spmv(csr_of(graph), npy(emitted))
    np.testing.assert_allclose(npy(_full(ranks, "persistent_current")), want, atol=2e-5, rtol=0)
    for rt in ranks:
        rt.check_status()


@pytest.mark.gpu
@pytest.mark.parametrize("gate", [1e-6, 0.15, 1.0])
def test_hybrid_row_tick_on_a_one_rank_group_matches_one_gpu(gate):
    """The hybrid row tick (gated scatter or tiled propagate, chosen on the
    device from the activity counted over all ranks) with the peer exchange,
    on a process group of one rank: it tracks the single-GPU event tick and
    keeps current == W @ emitted, through step() and through run()'s graph.
    gate 1e-6: every tick propagates; 1.0: every tick scatters; 0.15: both."""
    n = 6000
    graph = random_topology(n, 200000, device="cpu", seed=8).to("cuda")
    model = bench_model(n)
    initial = torch.rand(1, n, generator=torch.Generator().manual_seed(5)).cuda()
    single = NativeDendriticPELSRuntime(graph, model, initial.clone(), theta=0.02,
                                        propagation="event")
    dist.init_process_group("gloo", store=dist.HashStore(), rank=0, world_size=1)
    try:
        rt = ShardedDendriticPELSRuntime(graph, model, initial.clone(), theta=0.02,
                                         exchange="peer", propagation="hybrid",
                                         hybrid_gate=gate)
        assert rt.exchange == "peer" and rt.propagation == "hybrid"
        drives = [0.2 + 0.1 * np.sin(0.3 * t) for t in range(4)]
        taken = []
        with torch.inference_mode():
            for t in range(4):
                rt.step(drives[t], dendritic_drive=0.1)
                single.step(drives[t], dendritic_drive=0.1)
                counts = rt.workspace[16:40].view(torch.int64)  # count, gate_count, gate_source
                taken.append(int(counts[1]) >= rt._hybrid[2])
        torch.cuda.synchronize()
        if gate == 1e-6:
            assert all(taken)
        if gate == 1.0:
            assert not any(taken)
        for name in ("state", "dendritic_state", "adaptation_state", "emitted_state",
                     "persistent_current"):
            np.testing.assert_allclose(npy(getattr(rt, name)), npy(getattr(single, name)),
                                       atol=2e-6, rtol=0, err_msg=name)
        with torch.inference_mode():
            for _ in range(10):
                rt.step(0.25, dendritic_drive=0.1)
            rt.run(32, 0.25, dendritic_drive=0.1, graph_ticks=16)
        want = oracle.spmv(csr_of(graph), npy(rt.emitted_state))
        np.testing.assert_allclose(npy(rt.persistent_current), want, atol=2e-5, rtol=0)
        rt.check_status()
        rt.release_graphs()
        rt.close()
    finally:
        dist.destroy_process_group()
