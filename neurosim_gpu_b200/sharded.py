"""Row-sharded matrix tick across the GPUs of one node (one process per GPU).

Destination rows are cut into ``world`` contiguous ranges (:func:`row_bounds`):
by default where the prefix sum of ``in_rowptr`` reaches equal shares of the
edges, each range starting on a multiple of 4 rows.  Every tick each rank

1. runs the native tick on its own rows, gathering from the full soma vector
   ``x`` (all N neurons in global row order, so neuron n sits at row n on
   every rank) and writing its new soma values straight into its own rows of
   the next buffer;
2. exchanges the rows: stores into every other rank's buffer inside the tick
   kernel (the fused exchange), or an NCCL all-gather (``N*B*4`` bytes per
   tick; in place when the ranges are equal slices, else through a staging
   buffer of equal slices and one index_select back into row order).

Per-row sums are the same as on one GPU with the same kernel, so sharded
states are bit-identical to the single-GPU runtime's, whatever the partition.
Each rank keeps its own dendrite / adaptation slices and parameter views.
``run`` captures ticks and collectives together in one CUDA graph.

The partition and exchange logic lives in :class:`RowShard`, which runs on any
device and backend (the CPU tests drive it over gloo with the oracle tick).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import native as _native
from . import tiled as _tiled
from .dynamics import DendriticDynamics
from .precision import encode_sparse_weights


def row_bounds(neurons: int, world: int, rowptr: torch.Tensor | None = None) -> list[int]:
    """First rows of the ranks' row ranges (``world + 1`` bounds, 0 and N last).

    With ``rowptr`` (the destination CSR's ``in_rowptr``) the ranges hold
    about equal numbers of edges: bound r is the row where the prefix sum of
    edges reaches r / world of them, rounded to a multiple of 4.  Without it
    they hold equal numbers of rows (a multiple of 4 per rank).  A multiple of
    4 keeps every rank's first row, and with it its slices of the state,
    16-byte aligned (bulk copies in the tick kernel).
    """
    per = 4 * math.ceil(neurons / world / 4)
    if rowptr is None or world == 1:
        return [min(neurons, r * per) for r in range(world)] + [neurons]
    prefix = rowptr.to(torch.int64)
    edges = int(prefix[-1])
    targets = torch.tensor([r * edges // world for r in range(1, world)], dtype=torch.int64,
                           device=prefix.device)
    rows = torch.searchsorted(prefix, targets).tolist()
    bounds = [0]
    for row in rows:
        bounds.append(min(max(4 * ((row + 2) // 4), bounds[-1]), 4 * (neurons // 4)))
    return bounds + [neurons]


@dataclass
class RowShard:
    """Rows of one rank and the double-buffered full soma vector.

    ``bounds`` (from :func:`row_bounds`) are every rank's row ranges; the
    gathered buffers hold the soma vector in global row order, so rank r's
    rows sit at ``bounds[r]`` in every rank's buffer whatever the partition.
    """

    neurons: int
    batch: int
    rank: int
    world: int
    device: torch.device
    bounds: list[int] | None = None

    def __post_init__(self) -> None:
        if self.bounds is None:
            self.bounds = row_bounds(self.neurons, self.world)
        if (len(self.bounds) != self.world + 1 or self.bounds[0] != 0
                or self.bounds[-1] != self.neurons
                or any(a > b for a, b in zip(self.bounds, self.bounds[1:]))
                or any(b % 4 and b != self.neurons for b in self.bounds[:-1])):
            raise ValueError("row bounds must rise from 0 to N in multiples of 4")
        self.lo, self.hi = self.bounds[self.rank], self.bounds[self.rank + 1]
        sizes = [b - a for a, b in zip(self.bounds, self.bounds[1:])]
        # The NCCL exchange gathers slices of rows_per_rank rows from every rank.
        self.rows_per_rank = 4 * math.ceil(max(sizes) / 4)
        # Equal slices at r * rows_per_rank: the buffer itself is gathered in place.
        self.in_place = all(self.bounds[r] == min(self.neurons, r * self.rows_per_rank)
                            for r in range(self.world))
        self.cols = (self.world * self.rows_per_rank if self.in_place
                     else 4 * math.ceil(self.neurons / 4))
        shape = (self.cols, self.batch)
        self.buffers = [torch.zeros(shape, device=self.device) for _ in range(2)]
        self.current = 0
        self._staging = self._pad = self._order = None

    @property
    def rows(self) -> int:
        return self.hi - self.lo

    def load(self, full_state: torch.Tensor) -> None:
        """Set the soma vector from a full [B, N] state."""
        self.buffers[self.current][: self.neurons].copy_(full_state.T)

    def source(self, index: int | None = None) -> torch.Tensor:
        """The full gathered soma vector [B, cols] (strides (1, B))."""
        return self.buffers[self.current if index is None else index].t()

    def own(self, index: int) -> torch.Tensor:
        """This rank's rows of buffer ``index`` as a [B, rows] view."""
        return self.buffers[index][self.lo: self.hi].t()

    def exchange(self, index: int, group=None) -> None:
        """All-gather every rank's slice of buffer ``index`` in place.

        Unequal slices go through a staging buffer of ``world`` equal slices
        (this rank's rows padded to ``rows_per_rank``) and are put back in
        global row order by one index_select.
        """
        chunk = self.rows_per_rank * self.batch
        if self.in_place:
            flat = self.buffers[index].view(-1)
            dist.all_gather_into_tensor(flat, flat[self.rank * chunk: (self.rank + 1) * chunk],
                                        group=group)
            return
        if self._staging is None:
            self._staging = torch.zeros((self.world * self.rows_per_rank, self.batch),
                                        device=self.device)
            self._pad = torch.zeros((self.rows_per_rank, self.batch), device=self.device)
            self._order = torch.cat([torch.arange(r * self.rows_per_rank,
                                                  r * self.rows_per_rank + b - a)
                                     for r, (a, b) in enumerate(zip(self.bounds, self.bounds[1:]))]
                                    ).to(self.device)
        self._pad[: self.rows].copy_(self.buffers[index][self.lo: self.hi])
        dist.all_gather_into_tensor(self._staging.view(-1), self._pad.view(-1), group=group)
        torch.index_select(self._staging, 0, self._order, out=self.buffers[index][: self.neurons])

    def gather_rows(self, local: torch.Tensor, group=None) -> torch.Tensor:
        """Every rank's [B, rows] values assembled into the full [B, N] (an all-gather)."""
        padded = torch.zeros(self.batch, self.rows_per_rank, device=local.device)
        padded[:, : local.shape[1]] = local
        parts = [torch.empty_like(padded) for _ in range(self.world)]
        dist.all_gather(parts, padded.contiguous(), group=group)
        sizes = [b - a for a, b in zip(self.bounds, self.bounds[1:])]
        return torch.cat([part[:, :size] for part, size in zip(parts, sizes)], dim=1)

    def state(self) -> torch.Tensor:
        """The full soma state [B, N] (a view of the current buffer)."""
        return self.source()[:, : self.neurons]

    def local(self, value):
        """A drive (scalar or broadcastable to [B, N]) restricted to this rank's rows."""
        if not isinstance(value, torch.Tensor):
            return value
        return value.expand(self.batch, self.neurons)[:, self.lo: self.hi]


def _unpack_nibbles(packed: torch.Tensor, count: int) -> torch.Tensor:
    return torch.stack((packed & 15, packed >> 4), dim=1).flatten()[:count]


def _pack_nibbles(codes: torch.Tensor) -> torch.Tensor:
    if codes.numel() % 2:
        codes = torch.cat([codes, codes.new_zeros(1)])
    return (codes[0::2] | (codes[1::2] << 4)).contiguous()


class ShardedDendriticMatrixRuntime:
    """The matrix tick of one graph, rows split over the ranks of ``group``.

    ``graph`` is a :class:`~neurosim_gpu_b200.topology.SparseTopology` or a tuple
    ``(in_rowptr, in_col, in_weight)`` of the full destination CSR on this
    rank's device; ``dynamics`` and ``initial_state`` ([B, N]) are the full ones.
    ``state`` is the full soma state on every rank; ``dendritic_state`` and
    ``adaptation_state`` are this rank's rows.  ``partition="edges"`` (the
    default) cuts the rows where the prefix sum of ``in_rowptr`` reaches equal
    shares of the edges, so a degree-skewed graph still gives every rank the
    same work per tick; ``"rows"`` gives every rank the same number of rows.
    The states do not depend on the partition (bit for bit).
    """

    def __init__(self, graph, dynamics: DendriticDynamics, initial_state: torch.Tensor, *,
                 group=None, precision: str = "fp32", kernel: str = "auto",
                 threads_per_row: int | None = None, extension=None,
                 rank: int | None = None, world: int | None = None,
                 exchange: str = "auto", partition: str = "edges") -> None:
        if isinstance(graph, tuple):
            in_rowptr, in_col, in_weight = graph
        else:
            in_rowptr, in_col, in_weight = graph.in_rowptr, graph.in_col, graph.in_weight
        if initial_state.device.type != "cuda" or initial_state.dtype != torch.float32:
            raise ValueError("native compartment runtime requires CUDA float32")
        if kernel not in ("auto", "csr", "tiled"):
            raise ValueError("kernel must be 'auto', 'csr' or 'tiled'")
        if exchange not in ("auto", "nccl", "peer"):
            raise ValueError("exchange must be 'auto', 'nccl' or 'peer'")
        if partition not in ("edges", "rows"):
            raise ValueError("partition must be 'edges' or 'rows'")
        self.group = group
        # rank / world may be given explicitly to build one rank's share without a
        # process group (the exchange is then up to the caller).
        self.rank = dist.get_rank(group) if rank is None else rank
        self.world = dist.get_world_size(group) if world is None else world
        device = initial_state.device
        batch, neurons = initial_state.shape
        self.neurons, self.batch = neurons, batch
        self.extension = extension if extension is not None else _native.load_native_extension()
        self.shard = RowShard(neurons, batch, self.rank, self.world, device,
                              row_bounds(neurons, self.world,
                                         in_rowptr if partition == "edges" else None))
        lo, hi = self.shard.lo, self.shard.hi
        self.compartment_dynamics = dynamics
        self._source_csr = (in_rowptr, in_col, in_weight.detach())
        self.params = [p[lo:hi] for p in dynamics.parameters()]
        self.shard.load(initial_state)
        self.dendritic_state = torch.zeros(batch, hi - lo, device=device)
        self.adaptation_state = torch.zeros(batch, hi - lo, device=device)
        self.precision = precision
        self.status = _tiled.status_word(device)
        self._graphs: dict = {}
        self._rollout_plan = None
        self._tick = 0

        rowptr = in_rowptr.to(torch.int64)
        e0, e1 = int(rowptr[lo]), int(rowptr[hi])
        self.n_edges = int(rowptr[-1])
        self.local_edges = e1 - e0
        # Weights in the storage format, encoded over the WHOLE graph (global scales).
        if precision == "fp32":
            full, scales, scale = in_weight.detach(), None, None
        elif precision == "fp16":
            full, scales, scale = in_weight.detach().half(), None, None
        else:
            full, scales, scale = encode_sparse_weights(in_weight.detach(), precision)
        self.layout = None
        if batch == 1 and kernel != "csr" and self.local_edges > 0:
            fmt = {"fp32": _native.F32, "fp16": _native.F16, "fp8": _native.E4M3,
                   "nvfp4": _native.NVFP4}[precision]
            split = _tiled.graph_split(in_rowptr, in_col, fmt, neurons=neurons, cols=neurons,
                                       ctas=_tiled.sm_count(device),
                                       smem_limit=_tiled.smem_limit(device))
            if precision == "nvfp4":
                local = _pack_nibbles(_unpack_nibbles(full, self.n_edges)[e0:e1])
            else:
                local = full[e0:e1]
            self.layout = _tiled.build_tiled_layout(
                (rowptr[lo: hi + 1] - e0).to(torch.int32), in_col[e0:e1].contiguous(),
                local.contiguous(), neurons=hi - lo, cols=neurons,
                ctas=_tiled.sm_count(device), smem_limit=_tiled.smem_limit(device),
                block_scales=scales, global_scale=scale, scale_offset=e0, split=split)
        # Row-block CSR for the general kernel: the rows' offsets into the full arrays.
        self.csr = (in_rowptr[lo: hi + 1].contiguous(), in_col, full, scales, scale)
        degree = self.n_edges / max(neurons, 1)
        self.threads_per_row = threads_per_row or (8 if degree <= 16 else 16 if degree <= 48
                                                   else 32)
        # B >= 2: the batch kernel's lanes per row as the single-GPU runtime's
        # kernel picks them from the WHOLE graph's mean degree (a row block's
        # own degree may differ, and the lanes fix a row's summation order).
        self._batch_width = threads_per_row or (8 if degree <= 24 else 16 if degree <= 64
                                                else 32)
        # In-kernel peer exchange (run() at B = 1): every rank maps every other
        # rank's gathered buffers and arrival counter through CUDA IPC.
        self._peer = None
        self._peer_epoch = 0
        self._peer_bases: list[int] = []
        wants_peer = exchange == "peer" or (exchange == "auto" and rank is None)
        if (wants_peer and self.world > 1 and self.world <= _native.MAX_PEERS
                and self.layout is not None and dist.is_initialized()):
            self._setup_peer_exchange()
        elif exchange == "peer" and self.world > 1:
            raise ValueError("the peer exchange needs B = 1, the tiled path, <= 8 ranks and "
                             "a process group")

    def _setup_peer_exchange(self) -> None:
        """Map the other ranks' gathered buffers and counters (collective)."""
        device = self.shard.device
        self._counters = torch.zeros(32, dtype=torch.int64, device=device)  # [0] is the counter
        mine = [_native.ipc_export(t) for t in (*self.shard.buffers, self._counters)]
        table = [None] * self.world
        dist.all_gather_object(table, (self.rank, torch.cuda.current_device(), mine),
                               group=self.group)
        if len({entry[1] for entry in table}) != self.world:
            raise RuntimeError("the peer exchange needs one GPU per rank")
        pointers = [[0, 0, 0] for _ in range(self.world)]
        for rank, _, handles in table:
            if rank == self.rank:
                pointers[rank] = [t.data_ptr() for t in (*self.shard.buffers, self._counters)]
                continue
            for i, (handle, offset) in enumerate(handles):
                base = _native.ipc_import(handle, device)
                self._peer_bases.append(base)
                pointers[rank][i] = base + offset
        self._peer = pointers
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)

    def _exchange(self) -> "_native._PeerExchange":
        x = _native._PeerExchange()
        x.world, x.rank, x.row_offset = self.world, self.rank, self.shard.lo
        cur = self.shard.current
        for p, (b0, b1, counter) in enumerate(self._peer):
            x.gathered[p][0], x.gathered[p][1] = (b0, b1) if cur == 0 else (b1, b0)
            x.counters[p] = counter
        x.epoch = self._peer_epoch
        return x

    def same_weights(self, in_rowptr: torch.Tensor, in_col: torch.Tensor,
                     in_weight: torch.Tensor) -> bool:
        """Whether a destination CSR equals the one this run was built from."""
        mine = self._source_csr
        return all(a.numel() == b.numel() and torch.equal(a.to(b.device), b)
                   for a, b in zip((in_rowptr, in_col, in_weight), mine))

    @property
    def exchange(self) -> str:
        """'peer' (soma exchange inside the tick kernel) or 'nccl' (all-gather)."""
        return "peer" if self._peer is not None else "nccl"

    def close(self) -> None:
        """Unmap the other ranks' buffers (collective: every rank calls it)."""
        self._rollout_plan = None  # its argument blocks point into the peers' buffers
        if self._peer is not None:
            torch.cuda.synchronize(self.shard.device)
            dist.barrier(group=self.group)
            for base in self._peer_bases:
                _native.ipc_release(base, self.shard.device)
            self._peer_bases, self._peer = [], None
            dist.barrier(group=self.group)

    @property
    def kernel_path(self) -> str:
        return "tiled" if self.layout is not None else "csr"

    @property
    def state(self) -> torch.Tensor:
        return self.shard.state()

    def check_status(self) -> None:
        code = int(self.status.item())
        if code:
            raise RuntimeError(f"tiled tick pipeline timeout (code {code})")

    def _prepare(self, src: int, dst: int, d, a, u, us, v, vs, out_d, out_a):
        shard = self.shard
        s_rows = shard.own(src)
        out = (shard.own(dst), out_d, out_a)
        if self.layout is not None:
            return self.extension.prepare_step_tiled(
                s_rows, d, a, self.params, self.layout, u, us, v, vs, out=out,
                status=self.status, source=shard.buffers[src].view(-1)[: self.neurons])
        rowptr, col, weight, scales, scale = self.csr
        return self.extension.prepare_step_rows(
            s_rows, d, a, self.params, rowptr, col, weight, u, us, v, vs,
            self.threads_per_row if self.batch == 1 else self._batch_width,
            scales, scale, source=shard.source(src), out=out)

    def _drives(self, drive, dendritic_drive):
        def split(value):
            value = self.shard.local(value)
            return (None, float(value)) if not isinstance(value, torch.Tensor) else (value, 0.0)
        return split(drive) + split(dendritic_drive)

    def local_step(self, drive=0.0, *, dendritic_drive=0.0) -> int:
        """The kernel half of a tick: this rank's rows into the next buffer.

        Returns the index of the buffer written; :meth:`finish` adopts it after
        the exchange.
        """
        u, us, v, vs = self._drives(drive, dendritic_drive)
        src = self.shard.current
        dst = 1 - src
        out_d = torch.empty_like(self.dendritic_state)
        out_a = torch.empty_like(self.adaptation_state)
        self._prepare(src, dst, self.dendritic_state, self.adaptation_state, u, us, v, vs,
                      out_d, out_a)()
        self.dendritic_state, self.adaptation_state = out_d, out_a
        return dst

    def finish(self, dst: int) -> None:
        self.shard.current = dst
        self._tick += 1

    def step(self, drive=0.0, *, dendritic_drive=0.0) -> torch.Tensor:
        """One tick on every rank (all ranks must call it); returns the full state."""
        dst = self.local_step(drive, dendritic_drive=dendritic_drive)
        self.shard.exchange(dst, self.group)
        self.finish(dst)
        return self.state

    def run(self, ticks: int, drive=0.0, *, dendritic_drive=0.0, graph_ticks: int = 32
            ) -> torch.Tensor:
        """``ticks`` ticks with fixed drives (every rank calls it); the full state.

        With the peer exchange, one persistent kernel per rank runs all ticks;
        otherwise a CUDA graph of ``graph_ticks`` ticks + NCCL all-gathers is
        replayed.  Either way the result equals ``ticks`` calls of :meth:`step`.
        """
        if self._peer is not None and ticks > 0:
            return self._run_peer(ticks, drive, dendritic_drive)
        return self._run_graph(ticks, drive, dendritic_drive, graph_ticks)

    def _run_peer(self, ticks: int, drive, dendritic_drive) -> torch.Tensor:
        """All ``ticks`` ticks in one cooperative launch per rank, exchanging the
        soma vector inside the kernel (peer stores + a cross-GPU barrier)."""
        self.prepare_run(ticks, drive, dendritic_drive=dendritic_drive)()
        return self.state

    def prepare_run(self, ticks: int, drive=0.0, *, dendritic_drive=0.0):
        """A callable that enqueues :meth:`run`'s single persistent launch of
        ``ticks`` ticks (peer exchange only; every rank prepares and calls it).

        The preparation -- a synchronisation with every rank's earlier work on
        the gathered buffers, a barrier, argument checks -- happens here, so
        the callable itself only launches.  The runtime's state advances when
        the callable is called.
        """
        if self._peer is None or ticks < 1:
            raise ValueError("prepare_run needs the peer exchange and ticks >= 1")
        u, us, v, vs = self._drives(drive, dendritic_drive)
        # Every rank's earlier work on the gathered buffers (NCCL exchanges of
        # step()) must be finished before any rank's kernel writes into them.
        torch.cuda.current_stream(self.shard.device).synchronize()
        dist.barrier(group=self.group)
        s_rows = self.shard.own(self.shard.current)
        out_d = torch.empty_like(self.dendritic_state)
        out_a = torch.empty_like(self.adaptation_state)
        launch = self.extension.prepare_run_tiled_peers(
            s_rows, self.dendritic_state, self.adaptation_state, self.params, self.layout,
            u, us, v, vs, out=(s_rows, out_d, out_a), ticks=ticks, exchange=self._exchange(),
            status=self.status)

        def run() -> None:
            launch()
            self.dendritic_state, self.adaptation_state = out_d, out_a
            self.shard.current = (self.shard.current + ticks) % 2
            self._peer_epoch += ticks
            self._tick += ticks

        return run

    def stream(self, drives: torch.Tensor, out: torch.Tensor | None = None, *,
               dendritic_drive=0.0) -> torch.Tensor:
        """Advance ``len(drives)`` ticks (every rank calls it with the same count);
        tick t drives THIS rank's rows with ``drives[t]`` and copies the rows' new
        soma state into ``out[t]``.

        ``drives`` is [T, rows] or [T, B, rows] (the rank's rows only) and ``out``
        [T, B, rows], on the host (pinned, so the copies overlap the ticks) or on
        the device.  With the peer exchange (B = 1) the ticks run in rollout
        launches of up to 32 ticks per rank (``nsb_dendritic_rollout_tiled_peers``:
        tick k reads drive row k and writes history row k); the next launch's
        drives are uploaded and the previous launch's states downloaded on two
        copy streams while a launch runs.  Otherwise every tick is a
        :meth:`step` with its drive copied in and the rows' state copied out.
        Equal to ``len(drives)`` calls of :meth:`step` with those drives on the
        rows.  Returns ``out`` (allocated pinned if not given and ``drives`` is on
        the host).
        """
        ticks = drives.shape[0]
        rows, batch = self.shard.rows, self.batch
        if drives.dim() == 2:
            drives = drives.unsqueeze(1)
        if drives.dim() != 3 or drives.shape[-1] != rows or drives.shape[1] not in (1, batch):
            raise ValueError("drives must be [T, rows] or [T, B, rows] (this rank's rows)")
        if out is None:
            on_host = drives.device.type == "cpu"
            out = torch.empty((ticks, batch, rows), pin_memory=on_host,
                              device="cpu" if on_host else drives.device)
        if tuple(out.shape) != (ticks, batch, rows) or out.dtype != torch.float32:
            raise ValueError("out must be [T, B, rows] float32")
        if ticks == 0:
            return out
        with torch.inference_mode():
            if self._peer is not None:
                self._stream_peer(drives, out, dendritic_drive)
            else:
                device = self.shard.device
                drive = torch.zeros((batch, self.neurons), device=device)
                lo, hi = self.shard.lo, self.shard.hi
                for t in range(ticks):
                    drive[:, lo:hi].copy_(drives[t], non_blocking=True)
                    self.step(drive, dendritic_drive=dendritic_drive)
                    out[t].copy_(self.shard.own(self.shard.current), non_blocking=True)
        return out

    def _stream_peer(self, drives, out, dendritic_drive) -> None:
        _, _, v, vs = self._drives(0.0, dendritic_drive)
        # As in prepare_run: earlier NCCL exchanges end on every rank first.
        torch.cuda.current_stream(self.shard.device).synchronize()
        dist.barrier(group=self.group)
        chunks = _tiled.rollout_chunks(drives.shape[0])
        key = (None if v is None else (v.data_ptr(), v.stride()), vs)
        plan = self._rollout_plan
        if plan is None or plan.key != key or plan.capacity < max(chunks):
            plan = self._rollout_plan = _ShardedRolloutPlan(
                self, key, max(_tiled.ROLLOUT_CAP, *chunks), v, vs)
        self.dendritic_state, self.adaptation_state = plan.run(self, drives, out, chunks)

    def _run_graph(self, ticks: int, drive, dendritic_drive, graph_ticks: int) -> torch.Tensor:
        """``ticks`` ticks with fixed drives, replaying a CUDA graph of ticks + all-gathers."""
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
        graph, (d0, a0), final = entry
        d0.copy_(self.dendritic_state)
        a0.copy_(self.adaptation_state)
        if self.shard.current != 0:
            self.shard.buffers[0].copy_(self.shard.buffers[1])
            self.shard.current = 0
        for _ in range(ticks // graph_ticks):
            graph.replay()
        self.dendritic_state, self.adaptation_state = final[0].clone(), final[1].clone()
        self._tick += ticks // graph_ticks * graph_ticks
        for _ in range(ticks % graph_ticks):
            self.step(drive, dendritic_drive=dendritic_drive)
        return self.state

    def _capture(self, ticks: int, drive, dendritic_drive):
        u, us, v, vs = self._drives(drive, dendritic_drive)
        d_buf = [torch.empty_like(self.dendritic_state) for _ in range(2)]
        a_buf = [torch.empty_like(self.adaptation_state) for _ in range(2)]
        calls = []
        for k in range(ticks):
            src, dst = k % 2, (k + 1) % 2
            calls.append((self._prepare(src, dst, d_buf[src], a_buf[src], u, us, v, vs,
                                        d_buf[dst], a_buf[dst]), dst))
        saved = [b.clone() for b in self.shard.buffers]
        stream = torch.cuda.Stream(device=self.shard.device)
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):  # warm-up of the exact calls, outside capture
            for call, dst in calls[:2]:
                call()
                self.shard.exchange(dst, self.group)
        torch.cuda.current_stream().wait_stream(stream)
        torch.cuda.synchronize()
        for buffer, value in zip(self.shard.buffers, saved):  # the warm-up must not advance
            buffer.copy_(value)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for call, dst in calls:
                call()
                self.shard.exchange(dst, self.group)
        return graph, (d_buf[0], a_buf[0]), (d_buf[0], a_buf[0])

    def release_graphs(self) -> None:
        """Drop captured graphs (do this before destroying the process group)."""
        self._graphs = {}

    def gather(self, name: str) -> torch.Tensor:
        """The full [B, N] dendrite or adaptation state (an all-gather)."""
        return self.shard.gather_rows(getattr(self, name), self.group)


class _ShardedRolloutPlan:
    """What one rank's streamed rollouts reuse from call to call: the two copy
    streams and their events, the rings of drives and soma history, the
    running dendrite / adaptation rows, one peer-exchange argument block per
    parity of the gathered buffers and a prepared launch per (ring slot, launch
    length, parity).  Only the exchange's epoch changes between launches; it is
    written into the argument block just before each launch.
    """

    def __init__(self, runtime: ShardedDendriticMatrixRuntime, key, capacity: int, v, vs) -> None:
        device = runtime.shard.device
        rows = runtime.shard.rows
        self.key, self.capacity, self.v, self.vs = key, capacity, v, vs
        self.device = device
        self.d = torch.empty_like(runtime.dendritic_state)
        self.a = torch.empty_like(runtime.adaptation_state)
        self.drive_ring = [torch.empty((capacity, 1, rows), device=device) for _ in range(2)]
        self.history = [torch.empty((capacity, 1, rows), device=device) for _ in range(2)]
        self.upload = torch.cuda.Stream(device=device)
        self.download = torch.cuda.Stream(device=device)
        self.uploaded = [torch.cuda.Event() for _ in range(2)]
        self.consumed = [torch.cuda.Event() for _ in range(2)]  # launch done with ring slot k
        self.saved = [torch.cuda.Event() for _ in range(2)]     # history[k] downloaded
        current = runtime.shard.current
        self.exchange = []
        for parity in range(2):
            runtime.shard.current = parity
            self.exchange.append(runtime._exchange())
        runtime.shard.current = current
        self.calls: dict[tuple[int, int, int], object] = {}

    def call(self, runtime: ShardedDendriticMatrixRuntime, k: int, length: int, parity: int):
        launch = self.calls.get((k, length, parity))
        if launch is None:
            rows = runtime.shard.rows
            s_rows = runtime.shard.own(parity)
            launch = runtime.extension.prepare_run_tiled_peers(
                s_rows, self.d, self.a, runtime.params, runtime.layout, self.drive_ring[k][0],
                0.0, self.v, self.vs, out=(s_rows, self.d, self.a), ticks=length,
                exchange=self.exchange[parity], status=runtime.status,
                rollout=(rows, self.history[k][:length]))
            self.calls[k, length, parity] = launch
        return launch

    def run(self, runtime: ShardedDendriticMatrixRuntime, drives, out, chunks):
        compute = torch.cuda.current_stream(self.device)
        upload, download = self.upload, self.download
        self.d.copy_(runtime.dendritic_state)
        self.a.copy_(runtime.adaptation_state)
        upload.wait_stream(compute)
        download.wait_stream(compute)
        lo = 0
        for c, length in enumerate(chunks):
            k, hi = c % 2, lo + length
            with torch.cuda.stream(upload):
                if c >= 2:
                    upload.wait_event(self.consumed[k])
                self.drive_ring[k][:length].copy_(drives[lo:hi], non_blocking=True)
                self.uploaded[k].record(upload)
            compute.wait_event(self.uploaded[k])
            if c >= 2:
                compute.wait_event(self.saved[k])
            parity = runtime.shard.current
            self.exchange[parity].epoch = runtime._peer_epoch
            self.call(runtime, k, length, parity)()
            runtime.shard.current = (parity + length) % 2
            runtime._peer_epoch += length
            runtime._tick += length
            self.consumed[k].record(compute)
            with torch.cuda.stream(download):
                download.wait_event(self.consumed[k])
                out[lo:hi].copy_(self.history[k][:length], non_blocking=True)
                self.saved[k].record(download)
            lo = hi
        compute.wait_stream(download)
        compute.wait_stream(upload)
        return self.d.clone(), self.a.clone()


def broadcast_graph(neurons: int, edges: int, *, seed: int, device: torch.device, group=None):
    """Rank 0 builds ``random_topology`` (the reference stream) and broadcasts its CSR.

    Returns ``(in_rowptr, in_col, in_weight)`` on ``device`` on every rank.
    """
    from .topology import random_topology

    rank = dist.get_rank(group)
    if rank == 0:
        graph = random_topology(neurons, edges, device="cpu", seed=seed, build_device=device)
        arrays = [graph.in_rowptr, graph.in_col, graph.in_weight]
        count = torch.tensor([graph.n_edges], device=device, dtype=torch.int64)
    else:
        count = torch.zeros(1, device=device, dtype=torch.int64)
    dist.broadcast(count, 0, group=group)
    m = int(count.item())
    if rank != 0:
        arrays = [torch.empty(neurons + 1, dtype=torch.int32, device=device),
                  torch.empty(m, dtype=torch.int32, device=device),
                  torch.empty(m, dtype=torch.float32, device=device)]
    for array in arrays:
        dist.broadcast(array, 0, group=group)
    return tuple(arrays)
