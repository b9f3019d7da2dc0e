"""Graph identity against the reference generator.

``tests/golden/topology_checksums.json`` holds the SHA-256 of every array of
the reference's ``random_topology(N, M, seed)`` (src/neurosim_gpu/topology.py:
213-247, canonicalised by ``SparseTopology.from_edges``, topology.py:31-115),
written by ``tests/golden/make_golden.py`` from the reference package itself.
These tests build the same graphs with this package and compare every array:

* on the CPU (``build_device`` left at the generator's device) for every
  fixture graph up to 166k / 25M edges;
* with CUDA canonicalisation (CPU draws, ``build_device="cuda"``: the path the
  benchmark and the large parity tests take) for 166k / 10M, 166k / 25M and
  the 1.33M / 200M graph of the multi-GPU configuration.
"""

from __future__ import annotations

import concurrent.futures
import hashlib
import json

import pytest
import torch

from _util import GOLDEN
from neurosim_gpu_b200 import random_topology

FIELDS = ("src", "dst", "weight", "out_rowptr", "in_rowptr", "in_col", "out_weight_index",
          "in_weight")
CHECKSUMS = json.loads((GOLDEN / "topology_checksums.json").read_text())
CPU_GRAPHS = [key for key in CHECKSUMS if key != "1330000_200000000_0"]
CUDA_GRAPHS = ["166000_10000000_0", "166000_25000000_0", "1330000_200000000_0"]


def _sha(array: torch.Tensor) -> str:
    return hashlib.sha256(array.detach().cpu().contiguous().numpy().tobytes()).hexdigest()


def _digests(graph) -> dict[str, str]:
    # hashlib releases the GIL on large buffers: hash the eight arrays in parallel.
    with concurrent.futures.ThreadPoolExecutor(len(FIELDS)) as pool:
        futures = {f: pool.submit(_sha, getattr(graph, f)) for f in FIELDS}
        return {f: futures[f].result() for f in FIELDS}


def _check(key: str, graph) -> None:
    want = CHECKSUMS[key]
    assert graph.n_edges == want["n_edges"]
    got = _digests(graph)
    mismatched = [f for f in FIELDS if got[f] != want[f]]
    assert not mismatched, f"{key}: arrays differ from the reference graph: {mismatched}"


def _parse(key: str) -> tuple[int, int, int]:
    n, m, seed = (int(v) for v in key.split("_"))
    return n, m, seed


def test_every_fixture_graph_is_listed():
    assert set(CPU_GRAPHS) | set(CUDA_GRAPHS) == set(CHECKSUMS)
    for key, entry in CHECKSUMS.items():
        assert set(FIELDS) <= set(entry), key


@pytest.mark.parametrize("key", CPU_GRAPHS)
def test_cpu_graph_equals_reference(key):
    n, m, seed = _parse(key)
    _check(key, random_topology(n, m, device="cpu", seed=seed))


def test_a_changed_weight_is_detected():
    """The digests are sensitive: one flipped weight bit fails the comparison."""
    n, m, seed = _parse("97_600_83")
    graph = random_topology(n, m, device="cpu", seed=seed)
    graph.weight.view(torch.int32)[5] ^= 1
    with pytest.raises(AssertionError, match="weight"):
        _check("97_600_83", graph)


@pytest.mark.gpu
@pytest.mark.parametrize("key", CUDA_GRAPHS)
def test_cuda_canonicalisation_equals_reference(key):
    n, m, seed = _parse(key)
    graph = random_topology(n, m, device="cpu", seed=seed, build_device="cuda")
    assert graph.device.type == "cuda"
    _check(key, graph)
    del graph
    torch.cuda.empty_cache()
