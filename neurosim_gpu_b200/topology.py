"""Sparse graph data model: canonical source-major edges plus a destination CSR.

Mirrors the reference ``SparseTopology`` (src/neurosim_gpu/topology.py:16-210)
and ``random_topology`` (topology.py:213-247) field for field, so the arrays
the CUDA tick consumes are the ones the reference builds:

* canonical edges are unique ``(src, dst)`` pairs sorted source-major; parallel
  edges are coalesced by summing their weights in input order (topology.py:62-83);
* ``in_rowptr / in_col / in_weight`` is the destination-major CSR ``W[dst, src]``
  (rows sorted by source within each destination, topology.py:85-93);
* ``out_rowptr / dst / weight`` is the source-major CSR of the same edges;
* ``out_weight_index[e]`` is the position of canonical edge ``e`` in the
  destination CSR (topology.py:94-103);
* ``weight_version`` counts in-place weight mutations.

``random_topology`` draws exactly the reference's random stream (``randint``
for sources, ``randint`` for destinations, ``randn`` for weights, one
``torch.Generator`` seeded with ``seed``), so a graph built here equals the
reference graph bit for bit: tests/test_topology_golden.py compares the SHA-256
of every array with the reference's digests, for CPU and CUDA
canonicalisation up to the 1.33M-neuron, 200M-edge graph.  A
``build_device`` may differ from the generator device: the random draws stay
on the generator device and the sort / coalesce runs on ``build_device``
(for example CPU draws, CUDA canonicalisation of a 200M-edge graph).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


def _row_pointer(rows: torch.Tensor, n_rows: int) -> torch.Tensor:
    counts = torch.bincount(rows, minlength=n_rows)
    rowptr = torch.zeros(n_rows + 1, dtype=torch.int64, device=rows.device)
    torch.cumsum(counts, dim=0, out=rowptr[1:])
    return rowptr


def _segment_sum_in_order(values: torch.Tensor, group: torch.Tensor, n_groups: int) -> torch.Tensor:
    """Sum ``values`` per ``group`` (groups are contiguous runs), left to right.

    A run of length k is summed as ((v0 + v1) + v2) + ..., the order of an
    in-order ``index_add`` into zeros.  Runs longer than one are rare in random
    graphs, so the loop runs over the run position, not over the elements.
    """
    out = torch.zeros(n_groups, dtype=values.dtype, device=values.device)
    if values.numel() == 0:
        return out
    first = torch.ones_like(group, dtype=torch.bool)
    first[1:] = group[1:] != group[:-1]
    start = torch.nonzero(first).flatten()
    out += values[start]  # 0 + v, as an index_add into zeros would round a -0.0
    position = torch.arange(values.numel(), device=values.device) - start[group]
    longest = int(position.max())
    for k in range(1, longest + 1):
        pick = position == k
        out.index_put_((group[pick],), out[group[pick]] + values[pick])
    return out


@dataclass(frozen=True)
class SparseTopology:
    """A fixed graph with source-major canonical edges and a destination CSR view."""

    n_neurons: int
    src: torch.Tensor
    dst: torch.Tensor
    weight: torch.Tensor
    out_rowptr: torch.Tensor
    in_rowptr: torch.Tensor
    in_col: torch.Tensor
    out_weight_index: torch.Tensor
    in_weight: torch.Tensor
    weight_version: int = 0

    @classmethod
    def from_edges(cls, n_neurons: int, src: torch.Tensor, dst: torch.Tensor,
                   weight: torch.Tensor, *, build_device: torch.device | str | None = None
                   ) -> "SparseTopology":
        if src.ndim != 1 or dst.ndim != 1 or weight.ndim != 1:
            raise ValueError("src, dst and weight must be rank-1 tensors")
        if not (src.numel() == dst.numel() == weight.numel()):
            raise ValueError("src, dst and weight must have equal length")
        if src.dtype not in (torch.int32, torch.int64) or dst.dtype not in (torch.int32, torch.int64):
            raise ValueError("edge indices must use torch.int32 or torch.int64")
        if src.device != dst.device or src.device != weight.device:
            raise ValueError("all edge tensors must be on the same device")
        if n_neurons <= 0:
            raise ValueError("n_neurons must be positive")
        device = torch.device(build_device) if build_device is not None else src.device
        s64 = src.to(device=device, dtype=torch.int64)
        d64 = dst.to(device=device, dtype=torch.int64)
        if s64.numel() and (int(s64.min()) < 0 or int(d64.min()) < 0
                            or int(s64.max()) >= n_neurons or int(d64.max()) >= n_neurons):
            raise ValueError("edge index out of range")
        if s64.numel() >= 2**31:
            raise ValueError("this compact topology supports fewer than 2^31 edges")
        w = weight.to(device=device)
        # Source-major order; a stable sort keeps parallel edges in input order.
        key = s64 * n_neurons + d64
        order = torch.sort(key, stable=True).indices
        key = key[order]
        unique_key, group = torch.unique_consecutive(key, return_inverse=True)
        if w.requires_grad:
            # Differentiable coalescing for trainable weights (index_add keeps the graph).
            canonical = torch.zeros(unique_key.numel(), dtype=w.dtype, device=device
                                    ).index_add(0, group, w[order])
        else:
            canonical = _segment_sum_in_order(w[order], group, unique_key.numel())
        csrc = torch.div(unique_key, n_neurons, rounding_mode="floor")
        cdst = unique_key - csrc * n_neurons
        out_rowptr = _row_pointer(csrc, n_neurons).to(torch.int32)
        # Destination-major CSR of the same edges (sources ascending in a row).
        in_order = torch.sort(cdst * n_neurons + csrc).indices
        in_rowptr = _row_pointer(cdst[in_order], n_neurons).to(torch.int32)
        in_col = csrc[in_order].to(torch.int32)
        in_weight = canonical[in_order]
        out_weight_index = torch.empty(canonical.numel(), dtype=torch.int32, device=device)
        out_weight_index[in_order] = torch.arange(canonical.numel(), dtype=torch.int32,
                                                  device=device)
        return cls(n_neurons=n_neurons, src=csrc.to(torch.int32), dst=cdst.to(torch.int32),
                   weight=canonical, out_rowptr=out_rowptr, in_rowptr=in_rowptr,
                   in_col=in_col, out_weight_index=out_weight_index, in_weight=in_weight)

    @property
    def n_edges(self) -> int:
        return self.weight.numel()

    @property
    def out_degree(self) -> torch.Tensor:
        return self.out_rowptr[1:] - self.out_rowptr[:-1]

    @property
    def in_degree(self) -> torch.Tensor:
        return self.in_rowptr[1:] - self.in_rowptr[:-1]

    @property
    def device(self) -> torch.device:
        return self.weight.device

    def to(self, device: torch.device | str) -> "SparseTopology":
        """A copy of every array on ``device`` (same weight_version)."""
        fields = {name: getattr(self, name).to(device) for name in
                  ("src", "dst", "weight", "out_rowptr", "in_rowptr", "in_col",
                   "out_weight_index", "in_weight")}
        return SparseTopology(n_neurons=self.n_neurons, weight_version=self.weight_version,
                              **fields)

    def sparse_matrix(self) -> torch.Tensor:
        """Destination-major CSR tensor (used by the differentiable autograd path)."""
        return torch.sparse_csr_tensor(self.in_rowptr, self.in_col, self.in_weight,
                                       size=(self.n_neurons, self.n_neurons),
                                       dtype=self.weight.dtype, device=self.weight.device,
                                       check_invariants=False)

    def dense_matrix(self) -> torch.Tensor:
        matrix = torch.zeros((self.n_neurons, self.n_neurons), dtype=self.weight.dtype,
                             device=self.weight.device)
        matrix.index_put_((self.dst.long(), self.src.long()), self.weight, accumulate=True)
        return matrix

    def storage_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (
            self.src, self.dst, self.weight, self.out_rowptr, self.in_rowptr, self.in_col,
            self.out_weight_index, self.in_weight))

    def native_storage_bytes(self) -> int:
        """Arrays the native matrix and event kernels read (topology.py:176-191)."""
        return sum(t.numel() * t.element_size() for t in (
            self.dst, self.out_weight_index, self.out_rowptr, self.in_rowptr, self.in_col,
            self.in_weight))

    @torch.no_grad()
    def apply_source_weights_(self, source_major_weight: torch.Tensor) -> None:
        """Update both weight views from one source-major vector and bump the version."""
        if source_major_weight.shape != self.weight.shape:
            raise ValueError("source_major_weight shape does not match topology")
        if source_major_weight.device != self.weight.device:
            raise ValueError("source_major_weight must be on the topology device")
        if source_major_weight.dtype != self.weight.dtype:
            raise ValueError("source_major_weight dtype does not match topology")
        self.weight.copy_(source_major_weight)
        self.in_weight[self.out_weight_index.to(torch.int64)] = source_major_weight
        self.mark_weights_mutated_()

    def mark_weights_mutated_(self) -> None:
        """Invalidate persistent-current and packed-weight caches after a mutation."""
        object.__setattr__(self, "weight_version", self.weight_version + 1)


def random_topology(n_neurons: int, n_edges: int, *, device: torch.device | str,
                    dtype: torch.dtype = torch.float32, seed: int = 0,
                    weight_scale: float = 0.15,
                    build_device: torch.device | str | None = None) -> SparseTopology:
    """Uniform random graph: the reference generator's exact random stream.

    ``device`` hosts the generator (as in the reference); ``build_device``
    (default: ``device``) is where the arrays are canonicalised and kept.
    """
    if n_neurons <= 0 or n_edges < 0:
        raise ValueError("n_neurons must be positive and n_edges non-negative")
    generator = torch.Generator(device=device)
    generator.manual_seed(seed)
    src = torch.randint(n_neurons, (n_edges,), dtype=torch.int64, device=device,
                        generator=generator)
    dst = torch.randint(n_neurons, (n_edges,), dtype=torch.int64, device=device,
                        generator=generator)
    mean_degree = max(n_edges / n_neurons, 1.0)
    weight = torch.randn(n_edges, dtype=dtype, device=device, generator=generator) * (
        weight_scale / mean_degree ** 0.5)
    return SparseTopology.from_edges(n_neurons, src, dst, weight,
                                     build_device=build_device)
