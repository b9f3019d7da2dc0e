"""The scaled graph of the multi-GPU configuration: N = 1.33M, M = 200M (fp32, B = 1).

``random_topology(1_330_000, 200_000_000, seed=0)`` row-sharded
over 1 / 2 / 4 / 8 GPUs.  Its arrays equal the reference's (SHA-256 checked in
test_topology_golden.py).  Here, on one GPU:

* the single-GPU tick (23 column blocks) against the CPU oracle after 200 ticks;
* the 8-rank row split (each rank: 166k rows x 1.33M gathered columns, its own
  tiled layout), the ranks emulated on one GPU with the soma exchange done by
  copies: bit-identical to the single-GPU tick, as the fused exchange is on
  8 GPUs.
"""

from __future__ import annotations

import pytest
import torch

from _util import OracleMatrix, assert_same_as, bench_model
from neurosim_gpu_b200 import NativeDendriticMatrixRuntime, random_topology
from neurosim_gpu_b200.sharded import ShardedDendriticMatrixRuntime

pytestmark = pytest.mark.gpu

N, M = 1_330_000, 200_000_000


@pytest.fixture(scope="module")
def scaled():
    graph = random_topology(N, M, device="cpu", seed=0, build_device="cuda")
    yield graph, bench_model(N)
    del graph
    torch.cuda.empty_cache()


def test_scaled_graph_200_ticks_against_oracle(scaled):
    graph, model = scaled
    native = NativeDendriticMatrixRuntime(graph, model, torch.zeros(1, N, device="cuda"))
    assert native.kernel_path == "tiled" and native._tiled_layout().blocks == 23
    reference = OracleMatrix(graph, model, torch.zeros(1, N))
    with torch.inference_mode():
        native.run(200, 0.2, dendritic_drive=0.1)
    for _ in range(200):
        reference.step(0.2, 0.1)
    native.check_status()
    assert_same_as(native, reference, atol=1e-5, rtol=0)


def test_scaled_graph_eight_ranks_bit_identical_to_one_gpu(scaled):
    graph, model = scaled
    initial = torch.rand(1, N, generator=torch.Generator().manual_seed(8)).cuda()
    csr = (graph.in_rowptr, graph.in_col, graph.in_weight)
    ranks = [ShardedDendriticMatrixRuntime(csr, model, initial, rank=r, world=8)
             for r in range(8)]
    single = NativeDendriticMatrixRuntime(graph, model, initial.clone(), kernel="tiled")
    with torch.inference_mode():
        for _ in range(6):
            dsts = [rt.local_step(0.2, dendritic_drive=0.1) for rt in ranks]
            for rt, dst in zip(ranks, dsts):
                for other in ranks:
                    lo, hi = other.shard.lo, other.shard.hi
                    rt.shard.buffers[dst][lo:hi] = other.shard.buffers[dst][lo:hi]
                rt.finish(dst)
            single.step(0.2, dendritic_drive=0.1)
    torch.cuda.synchronize()
    for rt in ranks:
        assert rt.kernel_path == "tiled" and rt.layout.blocks == 23
        assert torch.equal(rt.state, single.state)
        lo, hi = rt.shard.lo, rt.shard.hi
        assert torch.equal(rt.dendritic_state, single.dendritic_state[:, lo:hi])
        assert torch.equal(rt.adaptation_state, single.adaptation_state[:, lo:hi])
        rt.check_status()
