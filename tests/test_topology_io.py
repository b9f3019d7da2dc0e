"""Topology files: interchange with the reference's serializer and the loader's checks.

The fixtures tests/golden/topology_ref_*.pt were written by the reference's own
``save_topology`` (tests/golden/make_topology_fixture.py); the checks follow the
reference's contract (src/neurosim_gpu/topology_io.py:56-218).
"""

from __future__ import annotations

import io
from pathlib import Path

import pytest
import torch

from neurosim_gpu_b200 import random_topology
from neurosim_gpu_b200.topology_io import (FORMAT, SCHEMA_VERSION, load_topology, save_topology,
                                           topology_from_dict, topology_to_dict)

GOLDEN = Path(__file__).resolve().parent / "golden"
FIELDS = ("src", "dst", "weight", "out_rowptr", "in_rowptr", "in_col", "out_weight_index",
          "in_weight")


def _same(a, b):
    assert a.n_neurons == b.n_neurons
    for name in FIELDS:
        x, y = getattr(a, name), getattr(b, name)
        assert x.dtype == y.dtype and torch.equal(x.cpu(), y.cpu()), name


@pytest.mark.parametrize("name", ["topology_ref_plain.pt", "topology_ref_with_in_weight.pt"])
def test_reads_files_written_by_the_reference(name):
    loaded = load_topology(GOLDEN / name)
    _same(loaded, random_topology(300, 3000, device="cpu", seed=2))
    assert loaded.weight_version == 0


def test_writes_the_reference_schema():
    want = torch.load(GOLDEN / "topology_ref_with_in_weight.pt", weights_only=True)
    got = topology_to_dict(random_topology(300, 3000, device="cpu", seed=2),
                           include_destination_weights=True)
    assert set(got) == set(want)
    for key, value in want.items():
        if isinstance(value, torch.Tensor):
            assert got[key].dtype == value.dtype and torch.equal(got[key], value), key
        else:
            assert got[key] == value, key
    assert got["format"] == FORMAT and got["version"] == SCHEMA_VERSION


@pytest.mark.parametrize("n,m,dest", [(1, 0, False), (7, 30, True), (2000, 40000, False)])
def test_round_trip(tmp_path, n, m, dest):
    graph = random_topology(n, m, device="cpu", seed=11)
    path = tmp_path / "g.pt"
    save_topology(graph, path, include_destination_weights=dest)
    _same(load_topology(path), graph)
    buffer = io.BytesIO()
    save_topology(graph, buffer)
    buffer.seek(0)
    _same(load_topology(buffer), graph)


def test_weight_version_is_kept_on_request():
    payload = topology_to_dict(random_topology(50, 400, device="cpu", seed=1))
    payload["weight_version"] = 7
    assert topology_from_dict(payload).weight_version == 0
    assert topology_from_dict(payload, reset_weight_version=False).weight_version == 7


def _corrupt(change):
    payload = topology_to_dict(random_topology(60, 600, device="cpu", seed=5),
                               include_destination_weights=True)
    payload = {k: (v.clone() if isinstance(v, torch.Tensor) else v) for k, v in payload.items()}
    change(payload)
    return payload


def _swap(tensor, i, j):
    tensor[i], tensor[j] = tensor[j].clone(), tensor[i].clone()


@pytest.mark.parametrize("change,message", [
    (lambda p: p.update(format="other"), "format"),
    (lambda p: p.update(version=2), "schema version"),
    (lambda p: p.update(n_neurons=0), "positive"),
    (lambda p: p.update(n_neurons=True), "integer"),
    (lambda p: p.pop("in_col"), "missing"),
    (lambda p: p.update(src=p["src"].long()), "int32"),
    (lambda p: p["weight"].__setitem__(3, float("inf")), "finite"),
    (lambda p: p["out_rowptr"].__setitem__(5, 0), "out_rowptr"),
    (lambda p: p["dst"].__setitem__(0, 99), "out of range"),
    (lambda p: _swap(p["dst"], 0, 1), "ordered|in_rowptr|out_weight_index"),
    (lambda p: p["out_weight_index"].__setitem__(0, p["out_weight_index"][1]), "permutation"),
    (lambda p: _swap(p["in_col"], 0, 1), "in_col|ordered"),
    (lambda p: p["in_weight"].__setitem__(0, 1.5), "in_weight"),
])
def test_rejects_inconsistent_payloads(change, message):
    with pytest.raises(ValueError, match=message):
        topology_from_dict(_corrupt(change))


@pytest.mark.gpu
def test_loads_onto_the_gpu_and_ticks_like_the_generated_graph(tmp_path):
    from neurosim_gpu_b200 import NativeDendriticMatrixRuntime
    from _util import bench_model
    graph = random_topology(3000, 90000, device="cpu", seed=8)
    path = tmp_path / "g.pt"
    save_topology(graph, path)
    loaded = load_topology(path, device="cuda")
    assert loaded.in_col.is_cuda
    model = bench_model(3000)
    state = torch.full((1, 3000), 0.1, device="cuda")
    a = NativeDendriticMatrixRuntime(loaded, model, state.clone())
    b = NativeDendriticMatrixRuntime(graph.to("cuda"), model, state.clone())
    with torch.inference_mode():
        a.run(20, 0.2, dendritic_drive=0.1)
        b.run(20, 0.2, dendritic_drive=0.1)
    assert torch.equal(a.state, b.state)
