"""Runtime checkpoints: the reference's format and signature, restore round trips.

tests/golden/checkpoint_ref_*.pt were written by the reference's own
``capture_runtime`` (tests/golden/make_checkpoint_fixture.py) for its CPU
dendritic runtimes; the checks follow src/neurosim_gpu/checkpoint.py:121-245.
"""

from __future__ import annotations

import io
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


# -- row-sharded runs (checkpoint.py:121-282 of the reference: capture / restore of
# the _TENSOR_FIELDS; a sharded run is captured as one whole-graph payload) -----


class _RankStub:
    """The attributes a row-sharded runtime's capture reads, on the CPU."""

    def __init__(self, rank, world, full_d, full_a, state, model, group=None):
        from neurosim_gpu_b200.sharded import RowShard
        batch, n = state.shape
        self.rank, self.world, self.group = rank, world, group
        self.batch, self.neurons, self.precision, self._tick = batch, n, "fp32", 9
        self.shard = RowShard(n, batch, rank, world, torch.device("cpu"))
        self.shard.load(state)
        self.state = self.shard.state()
        self.compartment_dynamics = model
        self.dendritic_state = full_d[:, self.shard.lo:self.shard.hi].clone()
        self.adaptation_state = full_a[:, self.shard.lo:self.shard.hi].clone()

    def gather(self, name):
        from neurosim_gpu_b200.sharded import ShardedDendriticMatrixRuntime
        return ShardedDendriticMatrixRuntime.gather(self, name)


def _sharded_case(n=301, batch=2):
    g = torch.Generator().manual_seed(4)
    return (torch.rand(batch, n, generator=g), torch.rand(batch, n, generator=g),
            torch.rand(batch, n, generator=g))


def _gloo_capture(rank, world, port, queue):
    import io
    import os

    import torch.distributed as dist

    from neurosim_gpu_b200.checkpoint import capture_sharded_runtime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        state, d, a = _sharded_case()
        graph = random_topology(301, 3000, device="cpu", seed=3)
        stub = _RankStub(rank, world, d, a, state, _model(301))
        payload = capture_sharded_runtime(stub, graph if rank == 0 else None)
        blob = None
        if payload is not None:  # serialised: shared tensor storage dies with the child
            buffer = io.BytesIO()
            torch.save(payload, buffer)
            blob = buffer.getvalue()
        queue.put((rank, blob))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_capture_gathers_every_rank_over_gloo(world):
    """The collective capture (gloo ranks on the CPU) gathers the rows of every rank
    into one payload, equal to the in-process capture of the same ranks."""
    import socket

    import torch.multiprocessing as mp

    from neurosim_gpu_b200.checkpoint import capture_sharded_ranks
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_gloo_capture, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(results[r] is None for r in range(1, world))
    payload = torch.load(io.BytesIO(results[0]), weights_only=True)
    state, d, a = _sharded_case()
    for name, want in (("state", state), ("dendritic_state", d), ("adaptation_state", a)):
        assert torch.equal(payload["tensors"][name], want), name
    assert payload["runtime_type"] == "NativeDendriticMatrixRuntime"
    assert payload["scalars"]["_tick"] == 9
    graph = random_topology(301, 3000, device="cpu", seed=3)
    model = _model(301)
    local = capture_sharded_ranks([_RankStub(r, world, d, a, state, model) for r in range(world)],
                                  graph)
    assert local["runtime_signature"] == payload["runtime_signature"]
    for name in ("state", "dendritic_state", "adaptation_state"):
        assert torch.equal(local["tensors"][name], payload["tensors"][name]), name


def test_in_process_capture_rejects_incomplete_ranks():
    from neurosim_gpu_b200.checkpoint import capture_sharded_ranks
    state, d, a = _sharded_case()
    graph = random_topology(301, 3000, device="cpu", seed=3)
    ranks = [_RankStub(r, 3, d, a, state, _model(301)) for r in range(3)]
    with pytest.raises(ValueError, match="every rank"):
        capture_sharded_ranks(ranks[:2], graph)
    ranks[1]._tick = 10
    with pytest.raises(ValueError, match="same tick"):
        capture_sharded_ranks(ranks, graph)


def _emulated_ticks(ranks, ticks, drive=0.2):
    """``ticks`` ticks of ranks that share one GPU; the exchange is a copy."""
    for _ in range(ticks):
        dsts = [rt.local_step(drive, dendritic_drive=0.1) for rt in ranks]
        for rt, dst in zip(ranks, dsts):
            for other in ranks:
                lo, hi = other.shard.lo, other.shard.hi
                rt.shard.buffers[dst][lo:hi] = other.shard.buffers[dst][lo:hi]
            rt.finish(dst)


@pytest.mark.gpu
@pytest.mark.parametrize("precision", ["fp32", "nvfp4"])
def test_sharded_checkpoint_restores_on_one_gpu_and_on_another_world(precision):
    """A world-2 run (ranks emulated on one GPU) is captured, restored into a
    single-GPU runtime and into a world-3 run, and all three continue bit for bit."""
    from neurosim_gpu_b200 import NativeDendriticMatrixRuntime
    from neurosim_gpu_b200.checkpoint import capture_sharded_ranks, restore_sharded_runtime
    from neurosim_gpu_b200.sharded import ShardedDendriticMatrixRuntime
    n = 6001
    graph = random_topology(n, 180000, device="cpu", seed=9).to("cuda")
    model = _model(n, "cuda")
    initial = torch.rand(1, n, generator=torch.Generator().manual_seed(2)).cuda()

    def world_of(size, start):
        return [ShardedDendriticMatrixRuntime(graph, model, start, precision=precision,
                                              rank=r, world=size) for r in range(size)]

    two = world_of(2, initial)
    with torch.inference_mode():
        _emulated_ticks(two, 10)
        payload = capture_sharded_ranks(two, graph)
        _emulated_ticks(two, 6)
    assert payload["scalars"]["_tick"] == 10
    single = NativeDendriticMatrixRuntime(graph, model, torch.zeros(1, n, device="cuda"),
                                          precision=precision, kernel="tiled")
    restore_runtime(single, payload)
    three = world_of(3, torch.zeros(1, n, device="cuda"))
    for rt in three:
        restore_sharded_runtime(rt, payload)
        assert rt._tick == 10
    with torch.inference_mode():
        for _ in range(6):
            single.step(0.2, dendritic_drive=0.1)
        _emulated_ticks(three, 6)
    torch.cuda.synchronize()
    assert torch.equal(single.state, two[0].state)
    for rt in three:
        assert torch.equal(rt.state, two[0].state)
        lo, hi = rt.shard.lo, rt.shard.hi
        assert torch.equal(rt.dendritic_state, single.dendritic_state[:, lo:hi])
        assert torch.equal(rt.adaptation_state, single.adaptation_state[:, lo:hi])
        rt.check_status()
    for rt in two:
        lo, hi = rt.shard.lo, rt.shard.hi
        assert torch.equal(rt.dendritic_state, single.dendritic_state[:, lo:hi])
