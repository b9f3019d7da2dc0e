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
from neurosim_gpu_b200 import NativeDendriticMatrixRuntime, random_topology
from neurosim_gpu_b200.sharded import RowShard, ShardedDendriticMatrixRuntime


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_worker(rank, world, port, n, batch, queue):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        graph = random_topology(n, 20 * n, device="cpu", seed=5)
        csr, params = csr_of(graph), params_of(bench_model(n, device="cpu"))
        full = np.random.default_rng(1).random((batch, n)).astype(np.float32)
        shard = RowShard(n, batch, rank, world, torch.device("cpu"))
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


@pytest.mark.parametrize("world,n,batch", [(2, 301, 1), (2, 300, 3), (3, 1000, 2)])
def test_row_shard_exchange_reassembles_full_state_over_gloo(world, n, batch):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, n, batch, queue))
             for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    graph = random_topology(n, 20 * n, device="cpu", seed=5)
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
            assert sh.cols == world * sh.rows_per_rank >= n
            seen += list(range(sh.lo, sh.hi))
        assert seen == list(range(n))


@pytest.mark.gpu
@pytest.mark.parametrize("precision", ["fp32", "nvfp4"])
@pytest.mark.parametrize("batch,world", [(1, 2), (1, 3), (4, 2)])
def test_sharded_ranks_emulated_on_one_gpu_match_single_gpu(precision, batch, world):
    """All ranks' kernels on one GPU, exchange by copies: bit-identical to one GPU."""
    n = 6001
    graph = random_topology(n, 180000, device="cpu", seed=9).to("cuda")
    model = bench_model(n)
    initial = torch.rand(batch, n, generator=torch.Generator().manual_seed(2)).cuda()
    ranks = [ShardedDendriticMatrixRuntime(graph, model, initial, precision=precision,
                                           rank=r, world=world) for r in range(world)]
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
