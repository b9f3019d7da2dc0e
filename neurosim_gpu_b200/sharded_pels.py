"""Row-sharded PELS (event) ticks across the GPUs of one node (one process per GPU).

The reference's PELS runtime (``native_compartmental.py:134-177``,
``csrc/compartmental.cu:142-173``) runs on one GPU.  Here destination rows are
cut into ``world`` contiguous ranges as for the sharded matrix tick
(:class:`~neurosim_gpu_b200.sharded.RowShard`, by default balanced by edges):
rank r owns rows ``[lo_r, hi_r)`` and, for them, the soma / dendrite /
adaptation / emitted state, theta and the persistent current.  Every tick
each rank

1. advances its rows with j = its current and applies the emit rule; each row's
   delta (the residual where it emits, else 0) goes into the gathered delta
   buffer (global row order) at its global row;
2. exchanges the deltas: an NCCL all-gather of the rows' slices
   (``exchange="nccl"``), or peer stores of every delta into every rank's
   buffer inside the advance kernel with a bounded cross-GPU wait at the start
   of the scatter (``exchange="peer"``, CUDA IPC mappings);
3. scatters every nonzero delta of all N sources over its out-edges whose
   destination is one of the rank's rows (the source-major out-CSR filtered
   to those rows, built once) into its current.

No rank holds a full state vector; :meth:`gather` assembles one.  As on one GPU
the scatter's float atomics leave the summation order of the current
nondeterministic.  The weights are fixed at construction.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import native as _native
from . import tiled as _tiled
from .dynamics import DendriticDynamics
from .sharded import RowShard, row_bounds


def filtered_out_csr(in_rowptr: torch.Tensor, in_col: torch.Tensor, in_weight: torch.Tensor,
                     lo: int, hi: int, neurons: int):
    """The source-major CSR of the edges whose destination lies in ``[lo, hi)``.

    Returns ``(rowptr [N+1] int32, dst int32 rebased to [0, hi-lo), weight f32)``.
    Within a source the edges keep the destination order of the CSR, which is
    the reference topology's source-major order (``topology.py:16-210``).
    """
    rowptr = in_rowptr.to(torch.int64)
    e0, e1 = int(rowptr[lo]), int(rowptr[hi])
    device = in_col.device
    src = in_col[e0:e1].to(torch.int64)
    dst = torch.repeat_interleave(torch.arange(hi - lo, device=device),
                                  (rowptr[lo + 1: hi + 1] - rowptr[lo:hi]))
    order = torch.sort(src, stable=True).indices
    counts = torch.bincount(src, minlength=neurons)
    out_rowptr = torch.zeros(neurons + 1, dtype=torch.int64, device=device)
    torch.cumsum(counts, 0, out=out_rowptr[1:])
    return (out_rowptr.to(torch.int32), dst[order].to(torch.int32).contiguous(),
            in_weight[e0:e1].detach()[order].to(torch.float32).contiguous())


class ShardedDendriticPELSRuntime:
    """PELS ticks of one graph, rows split over the ranks of ``group``.

    ``graph`` is a :class:`~neurosim_gpu_b200.topology.SparseTopology` or the
    full destination CSR ``(in_rowptr, in_col, in_weight)`` on this rank's
    device; ``dynamics``, ``initial_state`` ([B, N]) and ``theta`` (scalar or
    [N]) are the full ones.  ``state``, ``dendritic_state``, ``adaptation_state``,
    ``emitted_state`` and ``persistent_current`` are this rank's rows
    ([B, rows]).  ``rank`` / ``world`` may be given to build one rank's share
    without a process group (the caller then moves the deltas).

    ``propagation``: ``'event'`` scatters every tick's emitted deltas;
    ``'hybrid'`` (B = 1, peer exchange) propagates a tick whose emitting
    sources have at least ``hybrid_gate`` x M out-edges over ALL ranks with the
    tiled kernel over the rank's rows (W[rows, :] @ deltas, no atomics) and
    scatters the others, chosen on the device every tick as the single-GPU
    hybrid tick does; ``'auto'`` is the hybrid at B = 1 with the peer exchange
    for graphs of at least 2^20 edges, else the event tick.
    """

    def __init__(self, graph, dynamics: DendriticDynamics, initial_state: torch.Tensor, *,
                 theta, group=None, extension=None, rank: int | None = None,
                 world: int | None = None, exchange: str = "auto",
                 partition: str = "edges", propagation: str = "auto",
                 hybrid_gate: float = 0.15) -> None:
        if isinstance(graph, tuple):
            in_rowptr, in_col, in_weight = graph
        else:
            in_rowptr, in_col, in_weight = graph.in_rowptr, graph.in_col, graph.in_weight
        if initial_state.device.type != "cuda" or initial_state.dtype != torch.float32:
            raise ValueError("native compartment runtime requires CUDA float32")
        if exchange not in ("auto", "nccl", "peer"):
            raise ValueError("exchange must be 'auto', 'nccl' or 'peer'")
        if partition not in ("edges", "rows"):
            raise ValueError("partition must be 'edges' or 'rows'")
        if propagation not in ("auto", "event", "hybrid"):
            raise ValueError("propagation must be 'auto', 'event' or 'hybrid'")
        if not 0.0 < hybrid_gate <= 1.0:
            raise ValueError("hybrid_gate must be in (0, 1]")
        self.group = group
        self.rank = dist.get_rank(group) if rank is None else rank
        self.world = dist.get_world_size(group) if world is None else world
        device = initial_state.device
        batch, neurons = initial_state.shape
        self.batch, self.neurons = batch, neurons
        self.extension = extension if extension is not None else _native.load_native_extension()
        self.shard = RowShard(neurons, batch, self.rank, self.world, device,
                              row_bounds(neurons, self.world,
                                         in_rowptr if partition == "edges" else None))
        lo, hi = self.shard.lo, self.shard.hi
        self.compartment_dynamics = dynamics
        self.params = [p[lo:hi] for p in dynamics.parameters()]
        self.theta = self._validate_theta(theta, in_col, neurons, device)[lo:hi].contiguous()
        self.state = initial_state[:, lo:hi].clone()
        self.emitted_state = initial_state[:, lo:hi].clone()
        self.dendritic_state = torch.zeros_like(self.state)
        self.adaptation_state = torch.zeros_like(self.state)
        # The current of the rank's rows: (W @ emitted) restricted to them.
        full = self.extension.csr_propagate(in_rowptr, in_col, in_weight.detach(),
                                            initial_state.contiguous())
        self.persistent_current = full[:, lo:hi].contiguous()
        self.csr = filtered_out_csr(in_rowptr, in_col, in_weight, lo, hi, neurons)
        self.n_edges = int(in_rowptr[-1])
        self.local_edges = int(self.csr[1].numel())
        self.workspace = torch.zeros(_native.EVENT_ROWS_WORKSPACE, dtype=torch.uint8,
                                     device=device)
        self.status = _tiled.status_word(device)
        self._graphs: dict = {}
        self._tick = 0
        self._peer = None
        self._peer_bases: list[int] = []
        wants_peer = exchange == "peer" or (exchange == "auto" and rank is None)
        # exchange="peer" also runs on a process group of one rank (the fused
        # kernels with the rank's own buffers: tests of the peer path on one GPU).
        if (wants_peer and dist.is_initialized() and self.world <= _native.MAX_PEERS
                and (self.world > 1 or exchange == "peer")):
            self._setup_peer_exchange()
        elif exchange == "peer":
            raise ValueError("the peer exchange needs <= 8 ranks and a process group")
        # Hybrid ticks: the rows' tiled layout over all N columns and the rows'
        # out-degrees (whose emitting sum over all ranks sets the gate).
        self._hybrid = None
        wanted = propagation == "hybrid" or (propagation == "auto" and self.n_edges >= (1 << 20))
        if propagation == "hybrid" and (batch != 1 or self._peer is None):
            raise ValueError("the hybrid row tick takes B = 1 and the peer exchange")
        if wanted and batch == 1 and self._peer is not None and hi > lo:
            rowptr = in_rowptr.to(torch.int64)
            e0, e1 = int(rowptr[lo]), int(rowptr[hi])
            layout = _tiled.build_tiled_layout(
                (rowptr[lo: hi + 1] - e0).to(torch.int32), in_col[e0:e1].contiguous(),
                in_weight.detach()[e0:e1].float().contiguous(), neurons=hi - lo, cols=neurons,
                ctas=_tiled.sm_count(device), smem_limit=_tiled.smem_limit(device))
            out_degree = torch.bincount(in_col.to(torch.int64), minlength=neurons)[lo:hi]
            gate = max(1, int(hybrid_gate * self.n_edges))
            self._hybrid = (layout, out_degree.to(torch.int32).contiguous(), gate)

    @staticmethod
    def _validate_theta(theta, in_col, neurons, device) -> torch.Tensor:
        """The reference's threshold rules (runtime.py:15-34) on the full [N]."""
        theta = torch.as_tensor(theta, dtype=torch.float32, device=device)
        if theta.ndim == 0:
            theta = theta.expand(neurons)
        if theta.shape != (neurons,):
            raise ValueError("theta must be scalar or have one value per neuron")
        if bool(torch.any(theta < 0)) or bool(torch.any(torch.isnan(theta))):
            raise ValueError("theta must be non-negative and finite, except +inf for "
                             "zero-outdegree neurons")
        out_degree = torch.bincount(in_col.to(torch.int64), minlength=neurons)
        if bool(torch.any(torch.isposinf(theta) & (out_degree > 0))):
            raise ValueError("infinite theta is allowed only for zero-outdegree neurons")
        return theta

    # -- exchange ---------------------------------------------------------------
    def _setup_peer_exchange(self) -> None:
        """Map the other ranks' delta buffers and counters (collective)."""
        device = self.shard.device
        self._counters = torch.zeros(32, dtype=torch.int64, device=device)  # [0] is the counter
        mine = [_native.ipc_export(t) for t in (*self.shard.buffers, self._counters)]
        table = [None] * self.world
        dist.all_gather_object(table, (self.rank, torch.cuda.current_device(), mine),
                               group=self.group)
        if len({entry[1] for entry in table}) != self.world:
            raise RuntimeError("the peer exchange needs one GPU per rank")
        x = _native._DeltaExchange()
        x.world, x.rank = self.world, self.rank
        for rank, _, handles in table:
            if rank == self.rank:
                pointers = [t.data_ptr() for t in (*self.shard.buffers, self._counters)]
            else:
                pointers = []
                for handle, offset in handles:
                    base = _native.ipc_import(handle, device)
                    self._peer_bases.append(base)
                    pointers.append(base + offset)
            x.delta[rank][0], x.delta[rank][1], x.counters[rank] = pointers
        self._peer = x
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)

    @property
    def propagation(self) -> str:
        """'hybrid' (scatter or tiled propagate, chosen per tick on the device) or 'event'."""
        return "hybrid" if self._hybrid is not None else "event"

    @property
    def exchange(self) -> str:
        """'peer' (deltas exchanged inside the kernels), 'nccl' or 'none' (one rank)."""
        if self._peer is not None:
            return "peer"
        return "nccl" if self.world > 1 else "none"

    def close(self) -> None:
        """Unmap the other ranks' buffers (collective: every rank calls it)."""
        if self._peer is not None:
            torch.cuda.synchronize(self.shard.device)
            dist.barrier(group=self.group)
            for base in self._peer_bases:
                _native.ipc_release(base, self.shard.device)
            self._peer_bases, self._peer = [], None
            dist.barrier(group=self.group)

    def check_status(self) -> None:
        code = int(self.status.item())
        if code:
            raise RuntimeError(f"cross-GPU delta exchange timeout (code {code})")

    # -- ticks ------------------------------------------------------------------
    def _drives(self, drive, dendritic_drive):
        def split(value):
            value = self.shard.local(value)
            return (None, float(value)) if not isinstance(value, torch.Tensor) else (value, 0.0)
        return split(drive) + split(dendritic_drive)

    def _tick_calls(self, inputs, outputs, u, us, v, vs):
        """(advance, exchange or None, scatter) callables of one tick."""
        s, d, a, e = inputs
        peer = self._peer
        delta = None if peer is not None else self.shard.buffers[0].view(-1)
        hybrid = self._hybrid
        advance = self.extension.prepare_event_rows(
            s, d, a, self.params, self.persistent_current, e, self.theta, u, us, v, vs,
            row_offset=self.shard.lo, cols=self.shard.cols, delta=delta, exchange=peer,
            out=outputs, workspace=self.workspace,
            out_degree=hybrid[1] if hybrid is not None else None)
        rowptr, dst, weight = self.csr
        scatter = self.extension.prepare_scatter_rows(
            self.batch, self.neurons, self.shard.rows, delta, rowptr, dst, weight,
            self.persistent_current, exchange=peer, workspace=self.workspace,
            status=self.status, gate_edges=hybrid[2] if hybrid is not None else 0)
        if hybrid is not None:
            propagate = self.extension.prepare_propagate_rows_gated(
                hybrid[0], self.persistent_current, hybrid[2], workspace=self.workspace,
                status=self.status)
            gated_scatter = scatter

            def scatter() -> None:  # below the gate the first returns, else the second
                gated_scatter()
                propagate()
        exchange = None
        if peer is None and self.world > 1:
            exchange = lambda: self.shard.exchange(0, self.group)  # noqa: E731
        return advance, exchange, scatter

    def local_advance(self, drive=0.0, *, dendritic_drive=0.0):
        """The advance half of a tick (no exchange): returns (outputs, scatter callable).

        For callers that move the deltas themselves (``rank`` / ``world`` given
        without a process group): fill every rank's ``shard.buffers[0]`` with all
        ranks' rows, then call the scatter and adopt the outputs with
        :meth:`adopt`.
        """
        u, us, v, vs = self._drives(drive, dendritic_drive)
        outputs = tuple(torch.empty_like(self.state) for _ in range(4))
        advance, _, scatter = self._tick_calls(
            (self.state, self.dendritic_state, self.adaptation_state, self.emitted_state),
            outputs, u, us, v, vs)
        advance()
        return outputs, scatter

    def adopt(self, outputs) -> None:
        self.state, self.dendritic_state, self.adaptation_state, self.emitted_state = outputs
        self._tick += 1

    def step(self, drive=0.0, *, dendritic_drive=0.0) -> torch.Tensor:
        """One tick on every rank (all ranks call it); returns this rank's rows."""
        u, us, v, vs = self._drives(drive, dendritic_drive)
        outputs = tuple(torch.empty_like(self.state) for _ in range(4))
        advance, exchange, scatter = self._tick_calls(
            (self.state, self.dendritic_state, self.adaptation_state, self.emitted_state),
            outputs, u, us, v, vs)
        advance()
        if exchange is not None:
            exchange()
        scatter()
        self.adopt(outputs)
        return self.state

    def run(self, ticks: int, drive=0.0, *, dendritic_drive=0.0, graph_ticks: int = 32
            ) -> torch.Tensor:
        """``ticks`` ticks (every rank calls it); returns this rank's rows.

        A CUDA graph of ``graph_ticks`` ticks (advance, exchange, scatter) over
        two sets of static state buffers is captured once and replayed.
        ``drive`` is a float, a tensor broadcastable to [B, N], or a list of
        ``graph_ticks`` such drives (tick t of every replay uses
        ``drive[t % graph_ticks]``: a periodic drive; ``ticks`` must then be a
        multiple of ``graph_ticks``, which must be even).
        """
        if ticks < 0:
            raise ValueError("ticks must be non-negative")
        cycle = list(drive) if isinstance(drive, (list, tuple)) else None
        if cycle is not None:
            if len(cycle) != graph_ticks or graph_ticks % 2 or ticks % graph_ticks:
                raise ValueError("a drive cycle needs an even graph_ticks drives and ticks a "
                                 "multiple of graph_ticks")
        graph_ticks = max(2, min(graph_ticks, ticks) // 2 * 2)
        if ticks < graph_ticks:
            for _ in range(ticks):
                self.step(drive, dendritic_drive=dendritic_drive)
            return self.state
        key = (graph_ticks, repr(drive), repr(dendritic_drive))
        entry = self._graphs.get(key)
        if entry is None:
            self._graphs = {}
            entry = self._graphs[key] = self._capture(graph_ticks, drive, dendritic_drive)
        graph, buffers = entry
        for buffer, value in zip(buffers[0], (self.state, self.dendritic_state,
                                              self.adaptation_state, self.emitted_state)):
            buffer.copy_(value)
        for _ in range(ticks // graph_ticks):
            graph.replay()
        self.state, self.dendritic_state, self.adaptation_state, self.emitted_state = (
            b.clone() for b in buffers[0])
        self._tick += ticks // graph_ticks * graph_ticks
        for _ in range(ticks % graph_ticks):
            self.step(drive, dendritic_drive=dendritic_drive)
        return self.state

    def _capture(self, ticks: int, drive, dendritic_drive):
        cycle = list(drive) if isinstance(drive, (list, tuple)) else [drive]
        drives = [self._drives(x, dendritic_drive) for x in cycle]
        buffers = [tuple(torch.empty_like(self.state) for _ in range(4)) for _ in range(2)]
        calls = [self._tick_calls(buffers[k % 2], buffers[(k + 1) % 2], *drives[k % len(drives)])
                 for k in range(ticks)]
        # Warm-up of one tick outside capture (NCCL and kernel set-up); it must
        # not advance the simulation, so the current is put back.  Every rank
        # runs it, so the peer counters stay in step.
        for buffer, value in zip(buffers[0], (self.state, self.dendritic_state,
                                              self.adaptation_state, self.emitted_state)):
            buffer.copy_(value)
        saved = self.persistent_current.clone()
        stream = torch.cuda.Stream(device=self.shard.device)
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for call in calls[0]:
                if call is not None:
                    call()
        torch.cuda.current_stream().wait_stream(stream)
        torch.cuda.synchronize()
        self.persistent_current.copy_(saved)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for advance, exchange, scatter in calls:
                advance()
                if exchange is not None:
                    exchange()
                scatter()
        return graph, buffers

    def release_graphs(self) -> None:
        """Drop captured graphs (do this before destroying the process group)."""
        self._graphs = {}

    def gather(self, name: str) -> torch.Tensor:
        """The full [B, N] value of a per-row attribute (an all-gather)."""
        return self.shard.gather_rows(getattr(self, name), self.group)


__all__ = ["ShardedDendriticPELSRuntime", "filtered_out_csr"]
