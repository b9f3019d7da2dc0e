"""Row sharding: host-side exchange over gloo (CPU) and the per-rank kernels (GPU)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from _util import bench_model, csr_of, npy, params_of
from neurosim_gpu_b200 import NativeDendriticMatrixRuntime, SparseTopology, random_topology
from neurosim_gpu_b200.sharded import RowShard, ShardedDendriticMatrixRuntime, row_bounds


def skewed_topology(n: int, edges: int, seed: int = 3) -> SparseTopology:
    """A graph whose in-degree falls off with the row (row r draws ~(1 - r/n)^2
    of the edges): equal row ranges would give the first rank most of them."""
    g = torch.Generator().manual_seed(seed)
    dst = (n * torch.rand(edges, generator=g) ** 3).long().clamp(max=n - 1)
    src = torch.randint(n, (edges,), generator=g)
    weight = torch.randn(edges, generator=g) * 0.02
    return SparseTopology.from_edges(n, src, dst, weight)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_worker(rank, world, port, n, batch, queue, skewed=False):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        graph = (skewed_topology(n, 20 * n) if skewed
                 else random_topology(n, 20 * n, device="cpu", seed=5))
        csr, params = csr_of(graph), params_of(bench_model(n, device="cpu"))
        full = np.random.default_rng(1).random((batch, n)).astype(np.float32)
        bounds = row_bounds(n, world, graph.in_rowptr) if skewed else None
        shard = RowShard(n, batch, rank, world, torch.device("cpu"), bounds)
        assert shard.in_place != skewed
        shard.load(torch.from_numpy(full))
        d = np.zeros((batch, n), np.float32)
        a = np.zeros((batch, n), np.float32)
        for _ in range(5):
            # Each rank computes only its rows (from the full gathered state).
            s_full = npy(shard.state())
            s2, d2, a2 = oracle.matrix_tick(csr, s_full, d, a, params, 0.2, 0.1)
            dst = 1 - shard.current
            shard.own(dst).copy_(torch.from_numpy(s2[:, shard.lo: shard.hi]))
            shard.exchange(dst)
            shard.current = dst
            d, a = d2, a2
        queue.put((rank, npy(shard.state())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n,batch,skewed", [(2, 301, 1, False), (2, 300, 3, False),
                                                  (3, 1000, 2, False), (3, 1000, 2, True),
                                                  (2, 301, 1, True)])
def test_row_shard_exchange_reassembles_full_state_over_gloo(world, n, batch, skewed):
    """Equal slices gathered in place; edge-balanced (unequal) slices through
    the staging buffer: every rank holds the oracle's full state after 5 ticks."""
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, n, batch, queue, skewed))
             for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    graph = (skewed_topology(n, 20 * n) if skewed
             else random_topology(n, 20 * n, device="cpu", seed=5))
    csr, params = csr_of(graph), params_of(bench_model(n, device="cpu"))
    s = np.random.default_rng(1).random((batch, n)).astype(np.float32)
    d, a = np.zeros_like(s), np.zeros_like(s)
    for _ in range(5):
        s, d, a = oracle.matrix_tick(csr, s, d, a, params, 0.2, 0.1)
    for rank in range(world):
        assert np.array_equal(results[rank], s), rank


def test_row_partition_covers_every_row_once():
    for n, world in ((10, 3), (166000, 8), (7, 8), (1330000, 8)):
        seen = []
        for r in range(world):
            sh = RowShard(n, 1, r, world, torch.device("cpu"))
            assert sh.cols == world * sh.rows_per_rank >= n and sh.in_place
            seen += list(range(sh.lo, sh.hi))
        assert seen == list(range(n))


@pytest.mark.parametrize("n,world", [(20000, 2), (20000, 3), (20000, 8), (4001, 5), (9, 4)])
def test_edge_partition_balances_a_skewed_graph(n, world):
    """Row ranges cut at equal shares of the edges: on a graph whose first rows
    hold most edges every rank gets the same edges to within 4 rows' worth,
    every rank but the last starts on a multiple of 4, and every row is owned
    once.  Equal row ranges would give rank 0 several times its share."""
    graph = skewed_topology(n, 30 * n)
    rowptr = graph.in_rowptr.long()
    bounds = row_bounds(n, world, graph.in_rowptr)
    assert bounds[0] == 0 and bounds[-1] == n and bounds == sorted(bounds)
    seen = []
    for r in range(world):
        sh = RowShard(n, 1, r, world, torch.device("cpu"), bounds)
        assert sh.lo % 4 == 0 or sh.lo == n
        seen += list(range(sh.lo, sh.hi))
    assert seen == list(range(n))
    edges = [int(rowptr[b] - rowptr[a]) for a, b in zip(bounds, bounds[1:])]
    share = int(rowptr[-1]) / world
    degree = rowptr[1:] - rowptr[:-1]
    slack = 2 * 4 * int(degree.max())  # each bound moves by at most 2 rows to a multiple of 4
    assert max(edges) - share <= slack and share - min(edges) <= slack
    if n >= 4000:
        equal = row_bounds(n, world)
        equal_edges = [int(rowptr[b] - rowptr[a]) for a, b in zip(equal, equal[1:])]
        assert max(equal_edges) > 1.5 * share > 1.2 * max(edges)


@pytest.mark.parametrize("smem_limit", [232448, 16384])
def test_row_blocks_of_a_skewed_graph_take_the_whole_graphs_split(smem_limit):
    """A row block of a skewed graph, left to itself, would split its long
    pieces (or not) differently from the whole graph, and so sum its rows in
    another order; graph_split gives every block the whole graph's split."""
    from neurosim_gpu_b200 import native, tiled

    n = 6001
    graph = skewed_topology(n, 180000)
    smem_bytes = lambda cols, bufs: cols * 4 * bufs + 1024  # noqa: E731
    geometry = dict(ctas=148, smem_limit=smem_limit, smem_bytes=smem_bytes)
    whole = tiled.build_tiled_layout(graph.in_rowptr, graph.in_col, graph.in_weight,
                                     neurons=n, **geometry)
    split = tiled.graph_split(graph.in_rowptr, graph.in_col, native.F32, neurons=n, cols=n,
                              **geometry)
    rowptr = graph.in_rowptr.long()
    bounds = row_bounds(n, 3, graph.in_rowptr)
    own, given = [], []
    for lo, hi in zip(bounds, bounds[1:]):
        e0, e1 = int(rowptr[lo]), int(rowptr[hi])
        block = ((rowptr[lo: hi + 1] - e0).int(), graph.in_col[e0:e1].contiguous(),
                 graph.in_weight[e0:e1].contiguous())
        own.append(tiled.build_tiled_layout(*block, neurons=hi - lo, cols=n, **geometry))
        given.append(tiled.build_tiled_layout(*block, neurons=hi - lo, cols=n, split=split,
                                              **geometry))
    assert whole.splits == 1 and split == 0  # the whole graph is too sparse to split
    assert any(layout.splits > 1 for layout in own)
    assert all(layout.splits == 1 for layout in given)


@pytest.mark.gpu
@pytest.mark.parametrize("precision", ["fp32", "nvfp4"])
@pytest.mark.parametrize("batch,world,skewed", [(1, 2, False), (1, 3, False), (4, 2, False),
                                                (1, 3, True), (4, 3, True)])
def test_sharded_ranks_emulated_on_one_gpu_match_single_gpu(precision, batch, world, skewed):
    """All ranks' kernels on one GPU, exchange by copies: bit-identical to one GPU
    (on the skewed graph the ranks' row ranges are balanced by edges, not rows)."""
    n = 6001
    graph = (skewed_topology(n, 180000) if skewed
             else random_topology(n, 180000, device="cpu", seed=9)).to("cuda")
    model = bench_model(n)
    initial = torch.rand(batch, n, generator=torch.Generator().manual_seed(2)).cuda()
    ranks = [ShardedDendriticMatrixRuntime(graph, model, initial, precision=precision,
                                           rank=r, world=world) for r in range(world)]
    if skewed:  # the edge partition differs from equal row ranges here
        assert [rt.shard.lo for rt in ranks] != row_bounds(n, world)[:-1]
    single = NativeDendriticMatrixRuntime(graph, model, initial.clone(), precision=precision,
                                          kernel="tiled")
    with torch.inference_mode():
        for _ in range(12):
            dsts = [rt.local_step(0.2, dendritic_drive=0.1) for rt in ranks]
            for rt, dst in zip(ranks, dsts):
                for other in ranks:
                    lo, hi = other.shard.lo, other.shard.hi
                    rt.shard.buffers[dst][lo:hi] = other.shard.buffers[dst][lo:hi]
                rt.finish(dst)
            single.step(0.2, dendritic_drive=0.1)
    torch.cuda.synchronize()
    for rt in ranks:
        assert rt.kernel_path == single.kernel_path
        assert torch.equal(rt.state, single.state)
        lo, hi = rt.shard.lo, rt.shard.hi
        assert torch.equal(rt.dendritic_state, single.dendritic_state[:, lo:hi])
        assert torch.equal(rt.adaptation_state, single.adaptation_state[:, lo:hi])
        rt.check_status()
