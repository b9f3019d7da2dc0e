"""On-disk topology files, interchangeable with NeuroSim-GPU's ``topology_io``.

A file is a ``torch.save`` mapping in the reference's schema
``neurosim_gpu.sparse_topology`` version 1 (``src/neurosim_gpu/topology_io.py:28-38,
236-270``): the canonical source-major edges ``src`` / ``dst`` / ``weight``, the
row pointers ``out_rowptr`` / ``in_rowptr``, the destination CSR columns
``in_col`` and the permutation ``out_weight_index`` (all indices int32), the
neuron count, the weight version and, optionally, the redundant destination
weights ``in_weight``.  Files written here load in the reference and the other
way round: the field names, dtypes and the ordering contract are the format.

The loader is built for 200M-edge graphs:

* ``torch.load(..., mmap=True)`` maps the file instead of reading it into a
  second host copy;
* the arrays move to the target device once, and every consistency check
  (ordering, uniqueness, row pointers, the permutation and its inverse) runs
  there as a handful of vectorised passes, with no sort and no N x N object;
* the destination weights are rebuilt as ``weight[inverse(out_weight_index)]``.

Nothing here is on the tick's hot path; the runtimes take the resulting
:class:`SparseTopology` as they take one from ``random_topology``.
"""

from __future__ import annotations

from pathlib import Path
from typing import Any, BinaryIO, Mapping

import torch

from .topology import SparseTopology

FORMAT = "neurosim_gpu.sparse_topology"
SCHEMA_VERSION = 1
INDEX_FIELDS = ("src", "dst", "out_rowptr", "in_rowptr", "in_col", "out_weight_index")
TENSOR_FIELDS = INDEX_FIELDS + ("weight",)


def _int(value: Any, name: str) -> int:
    if isinstance(value, bool) or not isinstance(value, int):
        raise ValueError(f"{name} must be a Python integer")
    return int(value)


def _fail_unless(ok: bool, message: str) -> None:
    if not ok:
        raise ValueError(message)


def _check_header(payload: Mapping[str, Any]) -> tuple[int, int]:
    """Format, schema version, neuron count and weight version (topology_io.py:119-140)."""
    _fail_unless(isinstance(payload, Mapping), "topology payload must be a mapping")
    _fail_unless(payload.get("format") == FORMAT, "unsupported topology payload format")
    versions = [_int(payload[key], key) for key in ("version", "schema_version") if key in payload]
    _fail_unless(bool(versions) and all(v == SCHEMA_VERSION for v in versions),
                 f"unsupported topology schema version (expected {SCHEMA_VERSION})")
    n = _int(payload.get("n_neurons"), "n_neurons")
    _fail_unless(n > 0, "n_neurons must be positive")
    _fail_unless(n < 2**31, "n_neurons must be less than 2^31")
    weight_version = _int(payload.get("weight_version", 0), "weight_version")
    _fail_unless(weight_version >= 0, "weight_version must be non-negative")
    for name in TENSOR_FIELDS:
        _fail_unless(name in payload, f"topology payload is missing {name!r}")
        _fail_unless(isinstance(payload[name], torch.Tensor),
                     f"topology payload field {name!r} must be a tensor")
        _fail_unless(payload[name].ndim == 1, f"topology payload field {name!r} must be rank-1")
    for name in INDEX_FIELDS:
        _fail_unless(payload[name].dtype == torch.int32,
                     f"topology payload field {name!r} must use torch.int32")
    _fail_unless(payload["weight"].is_floating_point(),
                 "topology weights must use a floating-point dtype")
    return n, weight_version


def _check_arrays(n: int, t: Mapping[str, torch.Tensor]) -> torch.Tensor:
    """The ordering and consistency contract (topology_io.py:56-218), checked on
    the arrays' device.  Returns the inverse permutation (destination position ->
    canonical edge)."""
    weight = t["weight"]
    m = weight.numel()
    dev = weight.device
    _fail_unless(m < 2**31, "this compact topology supports fewer than 2^31 edges")
    _fail_unless(len({x.device for x in t.values()}) == 1,
                 "topology payload tensors must share one device")
    for name in ("src", "dst", "in_col", "out_weight_index"):
        _fail_unless(t[name].numel() == m, f"{name} length does not match weight length")
    if m:
        _fail_unless(bool(torch.isfinite(weight).all()), "topology weights must be finite")
    src = t["src"].long()
    dst = t["dst"].long()
    for name, rows in (("out_rowptr", src), ("in_rowptr", dst)):
        rowptr = t[name]
        _fail_unless(rowptr.shape == (n + 1,), f"{name} must have shape [{n + 1}]")
        expected = torch.zeros(n + 1, dtype=torch.int64, device=dev)
        if m:
            _fail_unless(bool(((rows >= 0) & (rows < n)).all()), "edge index out of range")
            torch.cumsum(torch.bincount(rows, minlength=n), 0, out=expected[1:])
        _fail_unless(torch.equal(rowptr.long(), expected),
                     f"{name} does not match the edges' "
                     + ("source-major order" if name == "out_rowptr" else "destination counts"))
    inverse = torch.empty(m, dtype=torch.int64, device=dev)
    if not m:
        return inverse
    key = src * n + dst
    step = key[1:] - key[:-1]
    _fail_unless(bool((step >= 0).all()), "source/destination edges are not source-major ordered")
    _fail_unless(bool((step != 0).all()), "duplicate source/destination edge")
    index = t["out_weight_index"].long()
    _fail_unless(bool(((index >= 0) & (index < m)).all()), "out_weight_index is out of range")
    seen = torch.zeros(m, dtype=torch.int32, device=dev)
    seen.index_add_(0, index, torch.ones_like(seen))
    _fail_unless(bool((seen == 1).all()), "out_weight_index must be a permutation")
    inverse[index] = torch.arange(m, device=dev)
    row_of_position = torch.repeat_interleave(torch.arange(n, device=dev),
                                              t["in_rowptr"].long().diff())
    _fail_unless(torch.equal(dst[inverse], row_of_position),
                 "out_weight_index does not match in_rowptr")
    col = t["in_col"].long()
    _fail_unless(torch.equal(col, src[inverse]), "in_col does not match out_weight_index")
    dkey = row_of_position * n + col
    _fail_unless(bool((dkey[1:] >= dkey[:-1]).all()),
                 "destination CSR view is not destination-major ordered")
    return inverse


def topology_to_dict(topology: SparseTopology, *, include_destination_weights: bool = False
                     ) -> dict[str, Any]:
    """A CPU mapping in the file schema (checked before it is returned)."""
    if not isinstance(topology, SparseTopology):
        raise ValueError("topology must be a SparseTopology")
    cpu = lambda x: x.detach().to("cpu").contiguous()  # noqa: E731
    payload: dict[str, Any] = {
        "format": FORMAT, "version": SCHEMA_VERSION, "schema_version": SCHEMA_VERSION,
        "n_neurons": int(topology.n_neurons),
        "weight_version": int(topology.weight_version),
        "weight_version_reset_on_load": True,
    }
    for name in TENSOR_FIELDS:
        payload[name] = cpu(getattr(topology, name))
    if include_destination_weights:
        payload["in_weight"] = cpu(topology.in_weight)
    n, _ = _check_header(payload)
    inverse = _check_arrays(n, {k: payload[k] for k in TENSOR_FIELDS})
    if include_destination_weights:
        _fail_unless(torch.equal(payload["in_weight"], payload["weight"][inverse]),
                     "in_weight does not match weight and out_weight_index")
    return payload


def topology_from_dict(payload: Mapping[str, Any], *, device: torch.device | str | None = None,
                       reset_weight_version: bool = True) -> SparseTopology:
    """The topology of a payload, its arrays on ``device`` (default CPU)."""
    n, saved_version = _check_header(payload)
    target = torch.device("cpu" if device is None else device)
    t = {name: payload[name].detach().to(target).contiguous() for name in TENSOR_FIELDS}
    inverse = _check_arrays(n, t)
    in_weight = t["weight"][inverse]
    if "in_weight" in payload:
        stored = payload["in_weight"]
        _fail_unless(isinstance(stored, torch.Tensor) and stored.ndim == 1,
                     "in_weight must be a rank-1 tensor")
        _fail_unless(stored.dtype == in_weight.dtype and stored.numel() == in_weight.numel(),
                     "in_weight must match weight dtype and length")
        _fail_unless(torch.equal(stored.to(target), in_weight),
                     "in_weight does not match weight and out_weight_index")
    return SparseTopology(n_neurons=n, src=t["src"], dst=t["dst"], weight=t["weight"],
                          out_rowptr=t["out_rowptr"], in_rowptr=t["in_rowptr"],
                          in_col=t["in_col"], out_weight_index=t["out_weight_index"],
                          in_weight=in_weight,
                          weight_version=0 if reset_weight_version else saved_version)


def save_topology(topology: SparseTopology, destination: str | Path | BinaryIO, *,
                  include_destination_weights: bool = False) -> None:
    """Write ``topology`` as a schema-v1 file (``torch.save``)."""
    torch.save(topology_to_dict(topology, include_destination_weights=include_destination_weights),
               destination)


def load_topology(source: str | Path | BinaryIO, *, device: torch.device | str | None = None,
                  reset_weight_version: bool = True) -> SparseTopology:
    """Read a schema-v1 file; a path is memory-mapped, the checks run on ``device``."""
    if isinstance(source, (str, Path)):
        payload = torch.load(source, map_location="cpu", weights_only=True, mmap=True)
    else:
        payload = torch.load(source, map_location="cpu", weights_only=True)
    _fail_unless(isinstance(payload, Mapping), "serialized topology must contain a mapping")
    return topology_from_dict(payload, device=device, reset_weight_version=reset_weight_version)


__all__ = ["FORMAT", "SCHEMA_VERSION", "topology_to_dict", "topology_from_dict",
           "save_topology", "load_topology"]
