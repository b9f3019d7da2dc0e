"""Runtime checkpoints in NeuroSim-GPU's format, for single-GPU and row-sharded runs.

A checkpoint is a ``torch.save`` mapping in the reference's schema
``neurosim_gpu.runtime_checkpoint`` version 1 (``src/neurosim_gpu/checkpoint.py:23-50,
121-155``): the runtime type, the weight precision, a SHA-256 signature of the
runtime's fixed parameters, the topology (the ``neurosim_gpu.sparse_topology``
payload of :mod:`neurosim_gpu_b200.topology_io`) and the runtime's state:

* tensors ``state``, ``dendritic_state``, ``adaptation_state`` and, for the PELS
  runtime, ``emitted_state``, ``persistent_current`` and ``theta``;
* scalars ``_tick`` and ``_weight_version``.

The signature is computed the way the reference computes it
(``checkpoint.py:61-118``: dtype, shape and raw bytes of every parameter
tensor of ``dynamics`` and ``compartment_dynamics``, then ``theta``, then the
precision when it is not fp32), so a checkpoint written by the reference's
dendritic runtimes restores here and the other way round.

A row-sharded run (:class:`~neurosim_gpu_b200.sharded.ShardedDendriticMatrixRuntime`)
is captured as ONE payload of the whole graph (its rows gathered to rank 0),
typed ``NativeDendriticMatrixRuntime``, so it restores into a single-GPU
runtime or into a sharded runtime over any number of ranks.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path
from typing import Any, BinaryIO, Mapping, Sequence

import torch

from .topology import SparseTopology
from .topology_io import topology_from_dict, topology_to_dict

FORMAT = "neurosim_gpu.runtime_checkpoint"
VERSION = 1
TENSOR_FIELDS = ("state", "dendritic_state", "adaptation_state", "emitted_state",
                 "persistent_current", "theta")
SCALAR_FIELDS = ("_tick", "_weight_version")
_STATE_FIELDS = ("state", "dendritic_state", "adaptation_state")
_STRUCTURE = ("src", "dst", "out_rowptr", "in_rowptr", "in_col", "out_weight_index")


def _precision(runtime: Any) -> str:
    return getattr(runtime, "checkpoint_precision", getattr(runtime, "precision", "fp32"))


def runtime_signature(runtime: Any) -> str:
    """SHA-256 of the runtime's fixed parameters (the reference's signature)."""
    digest = hashlib.sha256()

    def add(value: Any) -> None:
        if isinstance(value, torch.Tensor):
            cpu = value.detach().to("cpu").contiguous().clone()
            digest.update(str(cpu.dtype).encode())
            digest.update(repr(tuple(cpu.shape)).encode())
            digest.update(bytes(cpu.untyped_storage()))
        elif value is None or isinstance(value, (str, int, float, bool)):
            digest.update(json.dumps(value, sort_keys=True).encode())
        elif isinstance(value, (tuple, list)):
            for item in value:
                add(item)
        elif hasattr(value, "__dataclass_fields__"):
            for name in value.__dataclass_fields__:
                digest.update(name.encode())
                add(getattr(value, name))

    soma = getattr(runtime, "dynamics", None)
    if soma is not None:
        add(soma.alpha)
        add(soma.gain)
    if hasattr(runtime, "compartment_dynamics"):
        add(runtime.compartment_dynamics)
    if hasattr(runtime, "theta"):
        add(runtime.theta)
    precision = _precision(runtime)
    if precision != "fp32":
        digest.update(f"precision={precision}".encode())
    return digest.hexdigest()


def _header(runtime_type: str, precision: str, signature: str,
            topology: SparseTopology) -> dict[str, Any]:
    return {"format": FORMAT, "version": VERSION, "runtime_type": runtime_type,
            "precision": precision, "runtime_signature": signature,
            "topology": topology_to_dict(topology), "tensors": {}, "scalars": {}}


def capture_runtime(runtime: Any) -> dict[str, Any]:
    """A CPU payload of a single-GPU runtime (``NativeDendriticMatrixRuntime`` / PELS)."""
    topology = getattr(runtime, "topology", None)
    if not isinstance(topology, SparseTopology):
        raise ValueError("runtime must own a SparseTopology")
    payload = _header(type(runtime).__name__, _precision(runtime), runtime_signature(runtime),
                      topology)
    for name in TENSOR_FIELDS:
        value = getattr(runtime, name, None)
        if isinstance(value, torch.Tensor):
            payload["tensors"][name] = value.detach().to("cpu").clone()
    for name in SCALAR_FIELDS:
        value = getattr(runtime, name, None)
        if isinstance(value, (bool, int, float)):
            payload["scalars"][name] = value
    return payload


def _check_payload(payload: Mapping[str, Any]) -> None:
    if payload.get("format") != FORMAT or payload.get("version") != VERSION:
        raise ValueError("unsupported runtime checkpoint format or version")
    for key in ("topology", "tensors", "scalars"):
        if not isinstance(payload.get(key), Mapping):
            raise ValueError(f"checkpoint is missing its {key} payload")


def _check_compatible(payload: Mapping[str, Any], runtime_type: str, precision: str,
                      signature: str, shapes: Mapping[str, tuple]) -> SparseTopology:
    """The reference's restore checks (checkpoint.py:196-245); the saved topology."""
    _check_payload(payload)
    if payload.get("precision", "fp32") != precision:
        raise ValueError("checkpoint precision does not match target runtime")
    if payload.get("runtime_type") != runtime_type:
        raise ValueError("compartment checkpoint runtime type must match target runtime")
    for name, shape in shapes.items():
        value = payload["tensors"].get(name)
        if not isinstance(value, torch.Tensor):
            raise ValueError(f"checkpoint is missing tensor {name}")
        if tuple(value.shape) != shape or value.dtype != torch.float32:
            raise ValueError(f"checkpoint tensor {name} shape or dtype mismatch")
    saved = payload.get("runtime_signature")
    if saved is not None and saved != signature:
        raise ValueError("checkpoint runtime parameters differ from target runtime")
    return topology_from_dict(payload["topology"], device="cpu", reset_weight_version=False)


def _check_structure(saved: SparseTopology, target: SparseTopology) -> None:
    if saved.n_neurons != target.n_neurons or saved.n_edges != target.n_edges:
        raise ValueError("checkpoint topology shape does not match runtime")
    for name in _STRUCTURE:
        if not torch.equal(getattr(saved, name).cpu(), getattr(target, name).cpu()):
            raise ValueError(f"checkpoint topology structure differs in {name}")


def restore_runtime(runtime: Any, payload: Mapping[str, Any]) -> None:
    """Restore a payload into an already-constructed single-GPU runtime.

    The topology structure must match; saved weights are applied through the
    topology's mutation API (so cached packed weights and layouts rebuild).
    """
    target = getattr(runtime, "topology", None)
    if not isinstance(target, SparseTopology):
        raise ValueError("runtime must own a SparseTopology")
    shapes = {name: tuple(getattr(runtime, name).shape) for name in _STATE_FIELDS}
    saved = _check_compatible(payload, type(runtime).__name__, _precision(runtime),
                              runtime_signature(runtime), shapes)
    _check_structure(saved, target)
    weight = saved.weight.to(target.weight.device)
    if weight.dtype != target.weight.dtype:
        raise ValueError("checkpoint topology weight dtype does not match runtime")
    if not torch.equal(target.weight, weight):
        target.apply_source_weights_(weight)
    invalidate = getattr(runtime, "_invalidate_precision_cache", None)
    if invalidate is not None:
        invalidate()
    with torch.no_grad():
        for name, value in payload["tensors"].items():
            current = getattr(runtime, name, None)
            if not isinstance(current, torch.Tensor):
                raise ValueError(f"runtime does not expose checkpoint tensor {name}")
            if current.shape != value.shape or current.dtype != value.dtype:
                raise ValueError(f"checkpoint tensor {name} does not match the runtime's")
            setattr(runtime, name, value.to(current.device).clone())
    for name, value in payload["scalars"].items():
        if hasattr(runtime, name):
            if name == "_weight_version":  # keep a saved stale current stale
                value = target.weight_version - int(value != saved.weight_version)
            setattr(runtime, name, value)


def capture_sharded_runtime(runtime: Any, topology: SparseTopology | None) -> dict | None:
    """One payload of a row-sharded run (collective: every rank calls it).

    Rank 0 passes the full :class:`SparseTopology` of the run (any device) and
    receives the payload, typed ``NativeDendriticMatrixRuntime``; the other
    ranks may pass None and receive None.
    """
    state = runtime.state.detach().to("cpu").clone()
    dendrite = runtime.gather("dendritic_state").detach().to("cpu").clone()
    adaptation = runtime.gather("adaptation_state").detach().to("cpu").clone()
    if runtime.rank != 0:
        return None
    return _sharded_payload(runtime, topology, state, dendrite, adaptation)


def capture_sharded_ranks(ranks: Sequence[Any], topology: SparseTopology) -> dict:
    """One payload of a row-sharded run whose ranks all live in this process.

    ``ranks`` are the per-rank runtimes built with explicit ``rank`` / ``world``
    and no process group (the caller exchanges the soma vector between them);
    their rows are concatenated in rank order, which is what the collective
    :func:`capture_sharded_runtime` gathers to rank 0.  The payload is the same.
    """
    if not ranks:
        raise ValueError("no ranks given")
    world = ranks[0].world
    if sorted(r.rank for r in ranks) != list(range(world)) or any(r.world != world for r in ranks):
        raise ValueError("ranks must be every rank 0..world-1 of one run")
    ordered = sorted(ranks, key=lambda r: r.rank)
    if len({(r._tick, r.shard.current) for r in ordered}) != 1:
        raise ValueError("the ranks are not at the same tick")
    state = ordered[0].state.detach().to("cpu").clone()
    dendrite = torch.cat([r.dendritic_state.detach().to("cpu") for r in ordered], dim=1)
    adaptation = torch.cat([r.adaptation_state.detach().to("cpu") for r in ordered], dim=1)
    return _sharded_payload(ordered[0], topology, state, dendrite, adaptation)


def _sharded_payload(runtime: Any, topology: SparseTopology | None, state: torch.Tensor,
                     dendrite: torch.Tensor, adaptation: torch.Tensor) -> dict:
    if not isinstance(topology, SparseTopology) or topology.n_neurons != runtime.neurons:
        raise ValueError("rank 0 must pass the run's full SparseTopology")
    shape = (runtime.batch, runtime.neurons)
    if any(tuple(t.shape) != shape for t in (state, dendrite, adaptation)):
        raise ValueError("the gathered states do not cover every neuron of the run")
    payload = _header("NativeDendriticMatrixRuntime", runtime.precision,
                      runtime_signature(_SignatureView(runtime)), topology)
    payload["tensors"].update(state=state, dendritic_state=dendrite, adaptation_state=adaptation)
    payload["scalars"].update(_tick=int(runtime._tick))
    return payload


def restore_sharded_runtime(runtime: Any, payload: Mapping[str, Any]) -> None:
    """Restore a whole-graph payload into a row-sharded run (every rank calls it
    with the same payload); each rank takes its rows.  The run's weights are
    fixed at construction, so the saved weights must equal them."""
    shapes = {name: (runtime.batch, runtime.neurons) for name in _STATE_FIELDS}
    saved = _check_compatible(payload, "NativeDendriticMatrixRuntime", runtime.precision,
                              runtime_signature(_SignatureView(runtime)), shapes)
    if saved.n_neurons != runtime.neurons or saved.n_edges != runtime.n_edges:
        raise ValueError("checkpoint topology shape does not match runtime")
    if not runtime.same_weights(saved.in_rowptr, saved.in_col, saved.in_weight):
        raise ValueError("checkpoint weights differ from the sharded run's")
    tensors = payload["tensors"]
    lo, hi = runtime.shard.lo, runtime.shard.hi
    device = runtime.shard.device
    runtime.shard.load(tensors["state"].to(device))
    runtime.dendritic_state = tensors["dendritic_state"][:, lo:hi].to(device).contiguous()
    runtime.adaptation_state = tensors["adaptation_state"][:, lo:hi].to(device).contiguous()
    runtime._tick = int(payload["scalars"].get("_tick", 0))


class _SignatureView:
    """The attributes the signature reads, for a sharded run (full dynamics)."""

    def __init__(self, runtime: Any) -> None:
        self.compartment_dynamics = runtime.compartment_dynamics
        self.dynamics = runtime.compartment_dynamics.soma
        self.checkpoint_precision = runtime.precision


def save_runtime_checkpoint(runtime: Any, destination: str | Path | BinaryIO) -> None:
    torch.save(capture_runtime(runtime), destination)


def load_runtime_checkpoint(source: str | Path | BinaryIO, runtime: Any) -> None:
    payload = torch.load(source, map_location="cpu", weights_only=True)
    if not isinstance(payload, Mapping):
        raise ValueError("runtime checkpoint must contain a mapping")
    restore_runtime(runtime, payload)


__all__ = ["FORMAT", "VERSION", "runtime_signature", "capture_runtime", "restore_runtime",
           "capture_sharded_runtime", "capture_sharded_ranks", "restore_sharded_runtime",
           "save_runtime_checkpoint", "load_runtime_checkpoint"]
