"""Drop-in native runtimes: ``NativeDendriticMatrixRuntime`` / ``NativeDendriticPELSRuntime``.

Same constructor arguments, ``step`` signature, attributes and error types as
the reference classes (src/neurosim_gpu/native_compartmental.py:46-177):

* states ``state``, ``dendritic_state``, ``adaptation_state`` (+ ``emitted_state``,
  ``persistent_current``, ``theta``, ``_tick`` for PELS) are plain tensors, so
  the checkpoint layout is unchanged;
* ``step`` returns the new state; returned tensors stay valid after later
  ticks (every tick writes a fresh allocation);
* ``last_backend`` is ``"unstepped"``, ``"native"``, ``"native-{fp16,fp8,nvfp4}-weight"``,
  ``"native-stats"`` (PELS statistics, counted in the kernel) or
  ``"reference-autograd"`` (a request that needs gradients);
* ``checkpoint_precision``, ``precision_execution``, ``weight_storage_bytes``
  and ``threads_per_row`` keep their meaning.

Every inference tick runs in ``libneurosim_b200.so``.  The only non-CUDA-kernel
path is the differentiable PyTorch tick used when autograd is requested, which
the kernels do not implement (as in the reference, native_compartmental.py:104-108).

``NativeDendriticMatrixRuntime.run(ticks, ...)`` advances many ticks by
replaying a captured CUDA graph of the native tick.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import native as _native
from . import tiled as _tiled
from .dynamics import DendriticDynamics
from .precision import encode_sparse_weights, validate_precision, weight_storage_bytes
from .topology import SparseTopology


@dataclass(frozen=True)
class RuntimeStats:
    """Per-tick emission statistics (runtime.py:40-43 of the reference)."""

    path: str
    active_neurons: int
    active_edges: int


def validate_emission_threshold(theta: torch.Tensor, topology: SparseTopology) -> torch.Tensor:
    """runtime.py:15-34: scalar or [N], non-negative; +inf only without out-edges."""
    if theta.ndim == 0:
        theta = theta.expand(topology.n_neurons)
    if theta.shape != (topology.n_neurons,):
        raise ValueError("theta must be scalar or have one value per neuron")
    if bool(torch.any(theta < 0)) or bool(torch.any(torch.isnan(theta))):
        raise ValueError("theta must be non-negative and finite, except +inf for "
                         "zero-outdegree neurons")
    invalid_infinity = torch.isposinf(theta) & (topology.out_degree > 0)
    if bool(torch.any(torch.isneginf(theta))) or bool(torch.any(invalid_infinity)):
        raise ValueError("infinite theta is allowed only for zero-outdegree neurons")
    return theta


class _NativeCompartments:
    """State ownership and argument handling shared by both runtimes."""

    topology: SparseTopology
    compartment_dynamics: DendriticDynamics
    state: torch.Tensor
    dendritic_state: torch.Tensor
    adaptation_state: torch.Tensor

    def _init_compartments(self, topology: SparseTopology, dynamics: DendriticDynamics,
                           initial_state: torch.Tensor, extension) -> None:
        if initial_state.device.type != "cuda" or initial_state.dtype != torch.float32:
            raise ValueError("native compartment runtime requires CUDA float32")
        if initial_state.ndim != 2 or initial_state.shape[1] != topology.n_neurons:
            raise ValueError("initial_state must have shape [batch, n_neurons]")
        if dynamics.soma.n_neurons != topology.n_neurons:
            raise ValueError("dynamics and topology neuron counts must match")
        for value in (dynamics.soma.alpha, topology.weight):
            if value.device != initial_state.device or value.dtype != initial_state.dtype:
                raise ValueError("state, topology and dynamics must match device and dtype")
        if not bool((torch.isfinite(initial_state) & (initial_state >= 0)
                     & (initial_state <= 1)).all()):
            raise ValueError("initial_state must be finite and in [0, 1]")
        self.topology = topology
        self.compartment_dynamics = dynamics
        self.dynamics = dynamics.soma
        self.state = initial_state
        self.dendritic_state = torch.zeros_like(initial_state)
        self.adaptation_state = torch.zeros_like(initial_state)
        self.extension = extension if extension is not None else _native.load_native_extension()
        self.last_backend = "unstepped"

    @property
    def device(self) -> torch.device:
        return self.state.device

    def _parameters(self) -> list[torch.Tensor]:
        return self.compartment_dynamics.parameters()

    def _needs_autograd(self, drive, dendritic_drive) -> bool:
        if not torch.is_grad_enabled():
            return False
        values = [self.state, self.dendritic_state, self.adaptation_state, self.topology.weight,
                  self.topology.in_weight, *self._parameters(), drive, dendritic_drive]
        if hasattr(self, "persistent_current"):
            values += [self.persistent_current, self.emitted_state]
        return any(isinstance(v, torch.Tensor) and v.requires_grad for v in values)

    def _drive(self, value, name: str = "drive") -> tuple[torch.Tensor | None, float]:
        if not isinstance(value, torch.Tensor):
            return None, float(value)
        if value.device != self.state.device or value.dtype != self.state.dtype:
            raise ValueError(f"{name} must match state device and dtype")
        try:
            return value.expand_as(self.state), 0.0
        except RuntimeError as error:
            raise ValueError(f"{name} must broadcast to [batch, n_neurons]") from error

    # Differentiable PyTorch tick, used only when autograd is requested.
    def _autograd_propagate(self, source: torch.Tensor) -> torch.Tensor:
        return torch.sparse.mm(self.topology.sparse_matrix(), source.T).T

    def _autograd_advance(self, current, drive, dendritic_drive) -> torch.Tensor:
        for name, value in (("drive", drive), ("dendritic_drive", dendritic_drive)):
            if isinstance(value, torch.Tensor):
                try:
                    shape = torch.broadcast_shapes(value.shape, self.state.shape)
                except RuntimeError as error:
                    raise ValueError(f"{name} must broadcast to [batch, n_neurons]") from error
                if shape != self.state.shape:
                    raise ValueError(f"{name} must broadcast to [batch, n_neurons]")
        state, dendrite, adaptation = self.compartment_dynamics.advance(
            self.state, self.dendritic_state, self.adaptation_state, current, drive,
            dendritic_drive=dendritic_drive)
        self.dendritic_state = dendrite
        self.adaptation_state = adaptation
        return state


class NativeDendriticMatrixRuntime(_NativeCompartments):
    """One CUDA launch per tick: CSR propagation fused with all three neuron states.

    States, parameters, drives and accumulation are CUDA float32.  Optional
    fp16 / fp8 / nvfp4 CSR weight storage is decoded in-register before the
    fp32 multiply; reduced storage is inference-only.  ``threads_per_row``
    picks 8/16/32 lanes per row (None: chosen from the mean degree).
    """

    def __init__(self, topology: SparseTopology, dynamics: DendriticDynamics,
                 initial_state: torch.Tensor, *, threads_per_row: int | None = None,
                 extension=None, weight_dtype: torch.dtype = torch.float32,
                 weight_format: str | None = None, precision: str | None = None,
                 kernel: str = "auto") -> None:
        if precision is not None:
            validate_precision(precision)
            if weight_format is not None or weight_dtype != torch.float32:
                raise ValueError("precision and weight_dtype/weight_format conflict")
            weight_dtype = torch.float16 if precision == "fp16" else torch.float32
            weight_format = precision if precision in ("fp8", "nvfp4") else None
        if threads_per_row not in (None, 8, 16, 32):
            raise ValueError("threads_per_row must be 8, 16, 32 or None")
        if initial_state.device.type != "cuda" or initial_state.dtype != torch.float32:
            raise ValueError("native compartment runtime requires CUDA float32")
        if weight_dtype not in (torch.float32, torch.float16):
            raise ValueError("weight_dtype must be torch.float32 or torch.float16")
        if weight_format not in (None, "fp8", "nvfp4"):
            raise ValueError("weight_format must be None, 'fp8' or 'nvfp4'")
        if weight_format is not None and weight_dtype != torch.float32:
            raise ValueError("weight_format and non-default weight_dtype conflict")
        if kernel not in ("auto", "csr", "tiled", "cluster"):
            raise ValueError("kernel must be 'auto', 'csr', 'tiled' or 'cluster'")
        self.kernel = kernel
        self._init_compartments(topology, dynamics, initial_state, extension)
        self._status = _tiled.status_word(initial_state.device)
        self._layout = None
        self._layout_key = None
        self._cluster = None
        self._cluster_key = None
        degree = topology.n_edges / max(topology.n_neurons, 1)
        # Lanes per row; each lane reads 4-edge chunks, so 32 lanes cover 128 edges.
        self.threads_per_row = threads_per_row or (8 if degree <= 16 else 16 if degree <= 48
                                                   else 32)
        # B >= 2: the batch kernel's lanes per row, the caller's or the
        # library's own choice from the mean degree.
        self._batch_width = threads_per_row or (8 if degree <= 24 else 16 if degree <= 64
                                                else 32)
        self.weight_dtype = weight_dtype
        self.weight_format = weight_format
        self.precision = "fp32"
        self._graphs: dict = {}
        self._rollout_plan = None
        self._invalidate_precision_cache()

    def _invalidate_precision_cache(self) -> None:
        self._rollout_plan = None
        self._packed_weight = None
        self._packed_weight_version = -1
        self._graphs = {}
        self._layout = None
        self._layout_key = None

    @property
    def kernel_path(self) -> str:
        """'cluster' (B = 1 small graph on one thread-block cluster), 'tiled'
        (B = 1, state gathered from shared memory) or 'csr' (any B)."""
        if self._cluster_slots() is not None:
            return "cluster"
        return "tiled" if self._tiled_layout() is not None else "csr"

    def _cluster_slots(self) -> int | None:
        """Edge slots per CTA of the cluster tick, or None if it is not used.

        ``kernel='auto'`` takes the cluster tick at B = 1 whenever the graph
        fits one cluster's shared memory (it keeps all state on chip between
        ticks, so it beats the grid-wide kernels on small graphs).
        """
        if self.kernel not in ("auto", "cluster") or self.state.shape[0] != 1:
            if self.kernel == "cluster":
                raise ValueError("the cluster tick takes B = 1")
            return None
        rowptr = self.topology.in_rowptr
        key = (rowptr.data_ptr(), self.topology.n_edges, self.state.device)
        if self._cluster_key != key:
            slots, smem = self.extension.cluster_plan(rowptr)
            fits = smem <= _tiled.smem_limit(self.state.device)
            if not fits and self.kernel == "cluster":
                raise ValueError(f"the graph needs {smem} bytes of shared memory per CTA; "
                                 "it does not fit the cluster tick")
            self._cluster = slots if fits else None
            self._cluster_key = key
        return self._cluster

    def check_status(self) -> None:
        """Raise if a tiled or cluster launch reported an error (reads the device):
        codes 1-6 are bounded-wait timeouts of the tiled kernel, 7 a cluster
        launch whose edge-slot count was too small (it wrote nothing)."""
        code = int(self._status.item())
        if code == 7:
            raise RuntimeError("cluster tick: edge slots exceed max_slots (code 7)")
        if code:
            raise RuntimeError(f"tiled tick pipeline timeout (code {code})")

    def _tiled_layout(self):
        """The column-blocked layout of the current weights, or None if not used."""
        if (self.kernel in ("csr", "cluster") or self.state.shape[0] != 1
                or self.topology.n_edges == 0):
            return None
        key = (self.topology.weight_version, self.checkpoint_precision, self.state.device)
        if self._layout_key != key:
            weight, scales, scale, _ = self._weights()
            device = self.state.device
            try:
                self._layout = _tiled.build_tiled_layout(
                    self.topology.in_rowptr, self.topology.in_col, weight.detach(),
                    neurons=self.topology.n_neurons, ctas=_tiled.sm_count(device),
                    smem_limit=_tiled.smem_limit(device), block_scales=scales,
                    global_scale=scale)
            except ValueError:
                if self.kernel == "tiled":
                    raise
                self._layout = None
            self._layout_key = key
        return self._layout

    def _prepare(self, s, d, a, u, us, v, vs, out, ticks: int = 1):
        """A launch callable for one tick from (s, d, a) into the three `out` tensors
        (``ticks`` > 1: that many ticks in one launch; cluster and tiled paths only)."""
        slots = self._cluster_slots()
        if slots is not None:
            weight, scales, scale, _ = self._weights()
            topology = self.topology
            return self.extension.prepare_run_cluster(
                s, d, a, self._parameters(), topology.in_rowptr, topology.in_col, weight, u, us,
                v, vs, scales, scale, out=out, ticks=ticks, max_slots=slots, status=self._status)
        layout = self._tiled_layout()
        if layout is not None:
            if s.stride(1) != 1 or s.data_ptr() % 16:
                s = s.contiguous().clone()
            return self.extension.prepare_step_tiled(s, d, a, self._parameters(), layout, u, us,
                                                     v, vs, out=out, status=self._status,
                                                     ticks=None if ticks == 1 else ticks)
        if ticks != 1:
            raise ValueError("the CSR path runs one tick per launch")
        weight, scales, scale, _ = self._weights()
        topology = self.topology
        width = self.threads_per_row if s.shape[0] == 1 else self._batch_width
        return self.extension.prepare_step(s, d, a, self._parameters(), topology.in_rowptr,
                                           topology.in_col, weight, u, us, v, vs,
                                           width, scales, scale, out=out)

    @property
    def checkpoint_precision(self) -> str:
        if self.weight_format is not None:
            return self.weight_format
        return "fp16" if self.weight_dtype == torch.float16 else "fp32"

    @property
    def precision_execution(self) -> str:
        return f"cuda-fused-{self.checkpoint_precision}-weights-fp32-fma"

    @property
    def weight_storage_bytes(self) -> int:
        """Logical inference payload in bytes, excluding the original topology."""
        return weight_storage_bytes(self.topology.n_edges, self.checkpoint_precision)

    def _weights(self):
        """(weight, block_scales, global_scale, backend) for the current weight_version."""
        weight = self.topology.in_weight
        if self.weight_format is None and self.weight_dtype == torch.float32:
            return weight, None, None, "native"
        if self._packed_weight_version != self.topology.weight_version:
            if self.weight_format is None:
                self._packed_weight = (weight.detach().to(torch.float16),)
            else:
                self._packed_weight = encode_sparse_weights(weight.detach(), self.weight_format)
            self._packed_weight_version = self.topology.weight_version
        packed = self._packed_weight
        scales = packed[1] if len(packed) > 1 else None
        scale = packed[2] if len(packed) > 2 else None
        return packed[0], scales, scale, f"native-{self.weight_format or 'fp16'}-weight"

    def _propagate(self, source: torch.Tensor) -> torch.Tensor:
        """W @ source (fp32 weights) in one native launch."""
        topology = self.topology
        return self.extension.csr_propagate(topology.in_rowptr, topology.in_col,
                                            topology.in_weight.detach(), source)

    def step(self, drive: torch.Tensor | float = 0.0, *,
             dendritic_drive: torch.Tensor | float = 0.0) -> torch.Tensor:
        if self._needs_autograd(drive, dendritic_drive):
            if self.weight_format is not None or self.weight_dtype == torch.float16:
                raise RuntimeError("native reduced-precision weight storage is inference-only")
            self.last_backend = "reference-autograd"
            self.state = self._autograd_advance(self._autograd_propagate(self.state), drive,
                                                dendritic_drive)
            return self.state
        u, us = self._drive(drive)
        v, vs = self._drive(dendritic_drive, "dendritic_drive")
        backend = self._weights()[3]
        _, views = _native._outputs(3, self.state)
        self._prepare(self.state, self.dendritic_state, self.adaptation_state, u, us, v, vs,
                      views)()
        self.state, self.dendritic_state, self.adaptation_state = views
        self.last_backend = backend
        return self.state

    # -- multi-tick rollout through a CUDA graph -----------------------------
    def run(self, ticks: int, drive: torch.Tensor | float = 0.0, *,
            dendritic_drive: torch.Tensor | float = 0.0, graph_ticks: int = 64) -> torch.Tensor:
        """Advance ``ticks`` ticks with fixed drives; returns the final state.

        On the tiled path (B = 1) one persistent cooperative launch runs all
        ``ticks`` ticks.  Otherwise the native tick is captured once into a CUDA
        graph of ``graph_ticks`` ticks over two resident state buffers and
        replayed, so the host issues one launch per ``graph_ticks`` ticks;
        tensor drives are read at replay time (their values may change between
        calls, their storage may not).  Results equal ``ticks`` calls of
        :meth:`step`.
        """
        if ticks < 0:
            raise ValueError("ticks must be non-negative")
        if self._needs_autograd(drive, dendritic_drive):
            raise RuntimeError("run() is inference-only; use step() for autograd")
        if ticks == 0:
            return self.state
        u, us = self._drive(drive)
        v, vs = self._drive(dendritic_drive, "dendritic_drive")
        weight, _, _, backend = self._weights()
        # Build the plan outside any capture.
        if self._cluster_slots() is not None or self._tiled_layout() is not None:
            # One launch runs every tick (a cluster or a persistent kernel).
            _, views = _native._outputs(3, self.state)
            self._prepare(self.state, self.dendritic_state, self.adaptation_state, u, us, v, vs,
                          views, ticks=ticks)()
            self.state, self.dendritic_state, self.adaptation_state = views
            self.last_backend = backend
            return self.state
        graph_ticks = max(1, min(graph_ticks, ticks))
        key = (graph_ticks, tuple(self.state.shape),
               None if u is None else (u.data_ptr(), u.stride()), us,
               None if v is None else (v.data_ptr(), v.stride()), vs,
               weight.data_ptr(), self.topology.weight_version,
               tuple(p.data_ptr() for p in self._parameters()))
        entry = self._graphs.get(key)
        if entry is None:
            self._graphs = {}
            entry = self._graphs[key] = _TickGraph(self, graph_ticks, u, us, v, vs)
        entry.load(self.state, self.dendritic_state, self.adaptation_state)
        for _ in range(ticks // graph_ticks):
            entry.replay()
        states = entry.result()
        rest = ticks % graph_ticks
        self.state, self.dendritic_state, self.adaptation_state = states
        for _ in range(rest):
            self.step(drive, dendritic_drive=dendritic_drive)
        self.last_backend = backend
        return self.state


    # -- streamed rollout: host drives in, host states out ----------------------
    def stream(self, drives: torch.Tensor, out: torch.Tensor | None = None, *,
               dendritic_drive: torch.Tensor | float = 0.0) -> torch.Tensor:
        """Advance ``len(drives)`` ticks; tick t is driven by ``drives[t]`` ([B, N]
        or broadcastable) and its new soma state is copied into ``out[t]``.

        ``drives`` and ``out`` ([T, B, N] float32) may live on the host: pinned
        host memory lets the copies overlap the ticks.  On the tiled and cluster
        paths (B = 1) the ticks run in rollout launches of up to 32 (tiled) or
        128 (cluster) ticks (``nsb_dendritic_rollout_tiled`` /
        ``nsb_dendritic_rollout_cluster``: one launch per chunk, each tick
        reading its own drive row and writing its own history row); chunk
        c + 1's drives are uploaded on one CUDA stream and chunk c - 1's states
        downloaded on another while chunk c runs.  The other paths launch one
        tick at a time with the same two-stream overlap.  Every tick's drive is
        copied in and its state copied out; ``out`` holds every tick's state
        when the call returns.  Equal to ``len(drives)`` calls of :meth:`step`
        with those drives, bit for bit.  Returns ``out`` (allocated pinned if
        not given).
        """
        if self._needs_autograd(0.0, dendritic_drive) or drives.requires_grad:
            raise RuntimeError("stream() is inference-only; use step() for autograd")
        ticks = drives.shape[0]
        state = self.state
        device = state.device
        batch, neurons = state.shape
        if out is None:
            out = torch.empty((ticks, batch, neurons), dtype=state.dtype,
                              pin_memory=drives.device.type == "cpu",
                              device=drives.device if drives.device.type == "cuda" else "cpu")
        if out.shape[:1] != (ticks,) or out.shape[1:] != state.shape or out.dtype != state.dtype:
            raise ValueError("out must be [T, B, N] float32")
        if ticks == 0:
            return out
        if drives.dim() == 2:
            drives = drives.unsqueeze(1)  # [T, N]: one drive row per tick
        v, vs = self._drive(dendritic_drive, "dendritic_drive")
        with torch.inference_mode():
            if self.kernel_path in ("tiled", "cluster"):
                final = self._stream_rollouts(drives, out, v, vs)
            else:
                final = self._stream_ticks(drives, out, v, vs)
        self.state, self.dendritic_state, self.adaptation_state = final
        self.last_backend = self._weights()[3]
        return out

    def _stream_rollouts(self, drives, out, v, vs):
        slots = self._cluster_slots()
        # A cluster tick takes ~2 us and moves a few KB of copies: uniform
        # launches of 128 ticks.  The tiled path starts and ends with short
        # launches (1, 2, 4, ... ticks) so that the upload before the first
        # launch and the download after the last one (0.66 MB per tick at
        # 166k, ~15 us each) are short; the next launch's drives (twice as
        # many ticks) upload within the running launch.  166k / 25M, 20 ticks,
        # graph replay: 1-2-4-6-4-2-1 38.9 us per step, 2-4-8-4-2 40.8-42.8.
        if slots is not None:
            chunks = _tiled.rollout_chunks(drives.shape[0], cap=128, first=128)
        else:
            chunks = _tiled.rollout_chunks(drives.shape[0], first=1)
        weight, scales, scale, _ = self._weights()
        key = (slots, self.kernel_path, self._layout_key, self._packed_weight_version,
               None if v is None else (v.data_ptr(), v.stride()), vs,
               tuple(p.data_ptr() for p in self._parameters()), weight.data_ptr())
        plan = self._rollout_plan
        if plan is None or plan.key != key or plan.capacity < max(chunks):
            # Rings as long as the longest launch any stream() call makes.
            capacity = 128 if slots is not None else _tiled.ROLLOUT_CAP
            plan = self._rollout_plan = _RolloutPlan(self, key, max(capacity, *chunks), v, vs)
        return plan.run(self, drives, out, chunks)

    def _stream_ticks(self, drives, out, v, vs):
        state = self.state
        device = state.device
        batch, neurons = state.shape
        ticks = drives.shape[0]
        drive_buf = [torch.empty_like(state) for _ in range(2)]
        buffers = [(torch.empty_like(state), torch.empty_like(state), torch.empty_like(state))
                   for _ in range(2)]
        for target, value in zip(buffers[0], (state, self.dendritic_state,
                                              self.adaptation_state)):
            target.copy_(value)
        # One launch callable per parity: tick t reads buffers[t % 2] and
        # drive_buf[t % 2] and writes buffers[(t + 1) % 2].
        calls = [self._prepare(*buffers[k], drive_buf[k], 0.0, v, vs, buffers[1 - k])
                 for k in range(2)]
        compute = torch.cuda.current_stream(device)
        upload = torch.cuda.Stream(device=device)
        download = torch.cuda.Stream(device=device)
        uploaded = [torch.cuda.Event() for _ in range(2)]
        consumed = [torch.cuda.Event() for _ in range(2)]   # tick t done with drive_buf / buffers[t % 2]
        saved = [torch.cuda.Event() for _ in range(2)]      # download of buffers[k] finished
        upload.wait_stream(compute)
        download.wait_stream(compute)
        for t in range(ticks):
            k = t % 2
            with torch.cuda.stream(upload):
                if t >= 2:
                    upload.wait_event(consumed[k])
                drive_buf[k].copy_(drives[t].expand(batch, neurons), non_blocking=True)
                uploaded[k].record(upload)
            compute.wait_event(uploaded[k])
            if t >= 1:
                compute.wait_event(saved[1 - k])  # buffers[1 - k] is downloaded, rewrite it
            calls[k]()
            consumed[k].record(compute)
            with torch.cuda.stream(download):
                download.wait_event(consumed[k])
                out[t].copy_(buffers[1 - k][0], non_blocking=True)
                saved[1 - k].record(download)
        compute.wait_stream(download)
        compute.wait_stream(upload)
        return tuple(x.clone() for x in buffers[ticks % 2])


class _RolloutPlan:
    """What a streamed rollout reuses from one ``stream()`` call to the next.

    The two copy streams, their events, the device rings of drives and soma
    history, the running state and a prepared launch callable per (ring slot,
    launch length) are built once per runtime (rebuilt only when the weights,
    parameters, dendritic drive or the widest launch change), so a call costs
    its copies and launches, not their set-up (~1.5 ms of host time per call
    otherwise).  Every launch runs in place on ``running``; the call copies
    the runtime's state in first and hands out a fresh copy at the end, so
    tensors returned earlier are never overwritten.

    A call that repeats the previous call's contiguous pinned (or device)
    ``drives`` and ``out`` buffers and launch lengths captures its copies and
    launches into one CUDA graph, and later calls with those buffers replay it:
    one graph launch instead of a few dozen stream operations issued from
    Python (the host latency before the first launch was ~70 us of a 20-tick
    call).  The graph reads the buffers' contents when it runs, so callers
    refill them in place between calls; the plan keeps references to them so
    their memory stays valid while the graph exists.  If the capture fails,
    the plan stays on the per-call path.
    """

    def __init__(self, runtime: "NativeDendriticMatrixRuntime", key, widest: int, v, vs) -> None:
        self.key = key
        state = runtime.state
        device = state.device
        neurons = state.shape[1]
        self.device = device
        self.capacity = widest
        self.block, self.running = _native._outputs(3, state)
        self.drive_ring = [torch.empty((widest, 1, neurons), device=device) for _ in range(2)]
        self.history = [torch.empty((widest, 1, neurons), device=device) for _ in range(2)]
        self.upload = torch.cuda.Stream(device=device)
        self.download = torch.cuda.Stream(device=device)
        self.uploaded = [torch.cuda.Event() for _ in range(2)]
        self.consumed = [torch.cuda.Event() for _ in range(2)]  # rollout done with ring slot k
        self.saved = [torch.cuda.Event() for _ in range(2)]     # history[k] downloaded
        self.v, self.vs = v, vs
        self.calls: dict[tuple[int, int], object] = {}
        self.seen = None       # graph key of the last call that ran without a graph
        self.graph = None      # captured rollout of graph_key's buffers and chunks
        self.graph_key = None
        self.graph_buffers = None
        self.capture_failed = False

    def call(self, runtime: "NativeDendriticMatrixRuntime", k: int, length: int):
        launch = self.calls.get((k, length))
        if launch is not None:
            return launch
        running, neurons = self.running, self.running[0].shape[1]
        rollout = (neurons, self.history[k][:length])
        slots = runtime._cluster_slots()
        if slots is not None:
            weight, scales, scale, _ = runtime._weights()
            topology = runtime.topology
            launch = runtime.extension.prepare_run_cluster(
                *running, runtime._parameters(), topology.in_rowptr, topology.in_col, weight,
                self.drive_ring[k][0], 0.0, self.v, self.vs, scales, scale, out=running,
                ticks=length, max_slots=slots, status=runtime._status, rollout=rollout)
        else:
            launch = runtime.extension.prepare_step_tiled(
                *running, runtime._parameters(), runtime._tiled_layout(), self.drive_ring[k][0],
                0.0, self.v, self.vs, out=running, status=runtime._status, ticks=length,
                rollout=rollout)
        self.calls[k, length] = launch
        return launch

    def run(self, runtime: "NativeDendriticMatrixRuntime", drives, out, chunks):
        key = self._graph_key(drives, out, chunks)
        if key is not None and key == self.graph_key:
            self._load_state(runtime)
            self.graph.replay()
        elif key is not None and key == self.seen and self._capture(runtime, drives, out,
                                                                     chunks, key):
            self._load_state(runtime)
            self.graph.replay()
        else:
            self._enqueue(runtime, drives, out, chunks, load_state=True)
            self.seen = key
        block = self.block.clone()
        return tuple(block[i] for i in range(3))

    def _graph_key(self, drives, out, chunks):
        """What a captured rollout depends on, or None when the call's buffers
        cannot be captured (pageable or non-contiguous host memory, or drives
        that need a dtype conversion)."""
        if self.capture_failed:
            return None
        for t in (drives, out):
            if not t.is_contiguous() or t.dtype != torch.float32:
                return None
            if t.device.type == "cpu":
                if not t.is_pinned():
                    return None
            elif t.device != self.device:
                return None
        return (drives.data_ptr(), tuple(drives.shape), drives.device.type,
                out.data_ptr(), tuple(out.shape), out.device.type, tuple(chunks))

    def _capture(self, runtime, drives, out, chunks, key) -> bool:
        """Capture the copies and launches of a call (every launch length was
        prepared by the previous call with this key)."""
        graph = torch.cuda.CUDAGraph()
        capture = torch.cuda.Stream(device=self.device)
        capture.wait_stream(torch.cuda.current_stream(self.device))
        try:
            with torch.cuda.graph(graph, stream=capture, capture_error_mode="thread_local"):
                self._enqueue(runtime, drives, out, chunks, load_state=False)
        except RuntimeError:
            torch.cuda.synchronize(self.device)
            self.capture_failed = True
            return False
        torch.cuda.current_stream(self.device).wait_stream(capture)
        self.graph, self.graph_key, self.graph_buffers = graph, key, (drives, out)
        return True

    def _enqueue(self, runtime, drives, out, chunks, *, load_state: bool) -> None:
        compute = torch.cuda.current_stream(self.device)
        upload, download = self.upload, self.download
        # The rings were last used by work on the compute stream.
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
            if c == 0 and load_state:  # the first upload is under way; now the state goes in
                self._load_state(runtime)
            compute.wait_event(self.uploaded[k])
            if c >= 2:
                compute.wait_event(self.saved[k])
            self.call(runtime, k, length)()
            self.consumed[k].record(compute)
            with torch.cuda.stream(download):
                download.wait_event(self.consumed[k])
                out[lo:hi].copy_(self.history[k][:length], non_blocking=True)
                self.saved[k].record(download)
            lo = hi
        compute.wait_stream(download)
        compute.wait_stream(upload)

    def _load_state(self, runtime: "NativeDendriticMatrixRuntime") -> None:
        """Copy the runtime's s, d, a into the running block: one copy when
        they are the three rows of one block (what stream() and run() hand
        out), else three."""
        s, d, a = runtime.state, runtime.dendritic_state, runtime.adaptation_state
        n = s.numel()
        if (all(t.is_contiguous() and t.numel() == n for t in (s, d, a))
                and d.data_ptr() == s.data_ptr() + 4 * n and a.data_ptr() == d.data_ptr() + 4 * n
                and s.untyped_storage().data_ptr() == a.untyped_storage().data_ptr()):
            self.block.copy_(s.as_strided(self.block.shape, self.block.stride(),
                                          s.storage_offset()))
            return
        for target, value in zip(self.running, (s, d, a)):
            target.copy_(value)


class _TickGraph:
    """A CUDA graph of ``ticks`` native ticks ping-ponging between two buffers."""

    def __init__(self, runtime: NativeDendriticMatrixRuntime, ticks: int, u, us, v, vs) -> None:
        state = runtime.state
        self.ticks = ticks
        self.buffers = [_native._outputs(3, state)[1] for _ in range(2)]
        self.graph = torch.cuda.CUDAGraph()
        stream = torch.cuda.Stream(device=state.device)
        stream.wait_stream(torch.cuda.current_stream(state.device))
        calls = []
        for k in range(ticks):
            src, dst = self.buffers[k % 2], self.buffers[(k + 1) % 2]
            calls.append(runtime._prepare(src[0], src[1], src[2], u, us, v, vs, dst))
        with torch.cuda.stream(stream):
            calls[0]()  # warm-up outside capture (kernel attributes, occupancy queries)
        torch.cuda.current_stream(state.device).wait_stream(stream)
        with torch.cuda.graph(self.graph, stream=stream):
            for call in calls:
                call()
        self.final = self.buffers[ticks % 2]

    def load(self, s, d, a) -> None:
        for buffer, value in zip(self.buffers[0], (s, d, a)):
            buffer.copy_(value)

    def replay(self) -> None:
        self.graph.replay()
        for target, source in zip(self.buffers[0], self.final):
            if target.data_ptr() != source.data_ptr():
                target.copy_(source)

    def result(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        return tuple(b.clone() for b in self.buffers[0])


class _EventGraph:
    """A CUDA graph of ``ticks`` PELS ticks from static state buffers."""

    def __init__(self, runtime, ticks: int, u, us, v, vs) -> None:
        state = runtime.state
        device = state.device
        ext, topology = runtime.extension, runtime.topology
        self.inputs = [torch.empty_like(state, memory_format=torch.contiguous_format)
                       for _ in range(4)]
        workspace = runtime._workspace_for(state)
        params = runtime._parameters()
        current = runtime.persistent_current
        hybrid = runtime._hybrid()  # built outside the capture

        # u / us: one drive per graph tick, or one for all of them.
        drive_at = (lambda k: (u[k % len(u)], us[k % len(us)]))

        def ticks_from(inputs):
            s, d, a, e = inputs
            for k in range(ticks):
                uk, usk = drive_at(k)
                s, d, a, e = ext.dendritic_event(
                    s, d, a, params, current, e, runtime.theta, topology.out_rowptr,
                    topology.dst, None, topology.weight.detach(), uk, usk, v, vs,
                    workspace=workspace, hybrid=hybrid)
            return s, d, a, e

        # Warm-up outside capture must not advance the simulation: run it on
        # copies and put the current back.
        saved = current.clone()
        stream = torch.cuda.Stream(device=device)
        stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(stream):
            for buffer, value in zip(self.inputs, (runtime.state, runtime.dendritic_state,
                                                   runtime.adaptation_state,
                                                   runtime.emitted_state)):
                buffer.copy_(value)
            ext.dendritic_event(*self.inputs[:3], params, current, self.inputs[3],
                                runtime.theta, topology.out_rowptr, topology.dst, None,
                                topology.weight.detach(), *drive_at(0), v, vs,
                                workspace=workspace, hybrid=hybrid)
            current.copy_(saved)
        torch.cuda.current_stream(device).wait_stream(stream)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            self.final = ticks_from(self.inputs)

    def load(self, s, d, a, e) -> None:
        for buffer, value in zip(self.inputs, (s, d, a, e)):
            buffer.copy_(value)

    def replay(self) -> None:
        self.graph.replay()
        for target, source in zip(self.inputs, self.final):
            target.copy_(source)

    def result(self):
        return tuple(b.clone() for b in self.inputs)


class NativeDendriticPELSRuntime(_NativeCompartments):
    """Two CUDA launches per tick: advance + emission, then the active-edge scatter.

    The advance kernel queues every emitting (b, n) with its delta on the
    device; the scatter visits only those sources' out-edges and adds
    delta * w into the persistent current with float atomics (non-deterministic
    summation order).  ``collect_stats=True`` returns counts the kernel
    accumulated; autograd requests use the differentiable PyTorch tick.
    """

    def __init__(self, topology: SparseTopology, dynamics: DendriticDynamics,
                 initial_state: torch.Tensor, *, theta: float | torch.Tensor,
                 extension=None, precision: str | None = None, propagation: str = "auto",
                 hybrid_gate: float = 0.15) -> None:
        if precision not in (None, "fp32"):
            raise ValueError("native PELS supports FP32 only")
        if propagation not in ("auto", "event", "hybrid"):
            raise ValueError("propagation must be 'auto', 'event' or 'hybrid'")
        if not 0.0 < hybrid_gate <= 1.0:
            raise ValueError("hybrid_gate must be in (0, 1]")
        if initial_state.device.type != "cuda" or initial_state.dtype != torch.float32:
            raise ValueError("native compartment runtime requires CUDA float32")
        self._init_compartments(topology, dynamics, initial_state, extension)
        theta = torch.as_tensor(theta, dtype=initial_state.dtype, device=initial_state.device)
        self.theta = validate_emission_threshold(theta, topology)
        self.precision = "fp32"
        self.propagation = "event"
        self.emitted_state = initial_state.clone()
        self.persistent_current = self._propagate(self.emitted_state)
        self._tick = 0
        self._weight_version = topology.weight_version
        self._workspace = None
        self.propagation_mode = propagation
        self.hybrid_gate = hybrid_gate
        self._hybrid_key = None
        self._hybrid_args = None
        self._status = _tiled.status_word(initial_state.device)

    def _invalidate_precision_cache(self) -> None:
        pass

    @property
    def checkpoint_precision(self) -> str:
        return "fp32"

    @property
    def precision_execution(self) -> str:
        return "cuda-fused-pels-fp32"

    def _propagate(self, source: torch.Tensor) -> torch.Tensor:
        topology = self.topology
        if torch.is_grad_enabled() and (source.requires_grad or topology.in_weight.requires_grad):
            return self._autograd_propagate(source)
        return self.extension.csr_propagate(topology.in_rowptr, topology.in_col,
                                            topology.in_weight.detach(), source)

    def _refresh_current(self) -> None:
        """Recompute W @ emitted after a versioned weight change (runtime.py:217-223)."""
        if self._weight_version != self.topology.weight_version:
            self.persistent_current = self._propagate(self.emitted_state).contiguous()
            self._weight_version = self.topology.weight_version

    @property
    def propagation_path(self) -> str:
        """'hybrid' (per tick on the device: active-edge scatter below the gate,
        tiled W @ delta at or above it) or 'event' (the scatter every tick)."""
        return "hybrid" if self._hybrid() is not None else "event"

    def check_status(self) -> None:
        """Raise if a hybrid tick's tiled launch reported a pipeline timeout."""
        code = int(self._status.item())
        if code:
            raise RuntimeError(f"tiled propagation pipeline timeout (code {code})")

    def _hybrid(self):
        """(layout, dense delta buffer, gate in edges, status) or None.

        ``propagation='auto'`` uses the hybrid tick at B = 1 for graphs of at
        least 2^20 edges: a tick whose emitting sources have at least
        ``hybrid_gate`` x M out-edges propagates its deltas with the tiled
        kernel (W @ delta, no atomics) instead of the scatter.
        """
        state = self.state
        topology = self.topology
        wanted = self.propagation_mode == "hybrid" or (
            self.propagation_mode == "auto" and topology.n_edges >= (1 << 20))
        if not wanted or state.shape[0] != 1 or topology.n_edges == 0:
            if self.propagation_mode == "hybrid" and state.shape[0] != 1:
                raise ValueError("the hybrid PELS tick takes B = 1")
            return None
        key = (topology.weight_version, state.device)
        if self._hybrid_key != key:
            device = state.device
            layout = _tiled.build_tiled_layout(
                topology.in_rowptr, topology.in_col, topology.in_weight.detach().float(),
                neurons=topology.n_neurons, ctas=_tiled.sm_count(device),
                smem_limit=_tiled.smem_limit(device))
            dense = torch.zeros(topology.n_neurons, device=device)
            gate = max(1, int(self.hybrid_gate * topology.n_edges))
            self._hybrid_args = (layout, dense, gate, self._status)
            self._hybrid_key = key
        return self._hybrid_args

    def _workspace_for(self, state: torch.Tensor) -> torch.Tensor:
        need = int(self.extension.lib.nsb_dendritic_event_workspace_size(*state.shape))
        if self._workspace is None or self._workspace.numel() < need \
                or self._workspace.device != state.device:
            self._workspace = torch.empty(need, dtype=torch.uint8, device=state.device)
        return self._workspace

    def step(self, drive: torch.Tensor | float = 0.0, *,
             dendritic_drive: torch.Tensor | float = 0.0, collect_stats: bool = False):
        if self._needs_autograd(drive, dendritic_drive):
            self.last_backend = "reference-autograd"
            return self._autograd_step(drive, dendritic_drive, collect_stats)
        u, us = self._drive(drive)
        v, vs = self._drive(dendritic_drive, "dendritic_drive")
        self._refresh_current()
        if not self.persistent_current.is_contiguous():
            self.persistent_current = self.persistent_current.contiguous()
        workspace = self._workspace_for(self.state)
        topology = self.topology
        # The advance reads the current before the scatter updates it (stream order).
        self.state, self.dendritic_state, self.adaptation_state, self.emitted_state = (
            self.extension.dendritic_event(
                self.state, self.dendritic_state, self.adaptation_state, self._parameters(),
                self.persistent_current, self.emitted_state, self.theta, topology.out_rowptr,
                topology.dst, None, topology.weight.detach(), u, us, v, vs,
                workspace=workspace, hybrid=self._hybrid()))
        self._tick += 1
        if not collect_stats:
            self.last_backend = "native"
            return self.state
        self.last_backend = "native-stats"
        counters = _native.EventCounters.from_buffer_copy(
            workspace[: ctypes.sizeof(_native.EventCounters)].cpu().numpy().tobytes())
        active, edges = int(counters.active_neurons), int(counters.active_edges)
        return self.state, RuntimeStats("event" if active else "idle", active, edges)

    def run(self, ticks: int, drive: torch.Tensor | float = 0.0, *,
            dendritic_drive: torch.Tensor | float = 0.0, graph_ticks: int = 64) -> torch.Tensor:
        """Advance ``ticks`` ticks; returns the final state.

        ``graph_ticks`` event ticks (advance + emit, scatter) are captured once
        into a CUDA graph over static state buffers and replayed; the
        persistent current is updated in place.  ``drive`` is a float, a
        tensor broadcastable to [B, N], or a list of ``graph_ticks`` such drives
        (tick t of every replay uses ``drive[t % graph_ticks]``: a periodic
        drive).  Equal to ``ticks`` calls of :meth:`step` with the same drives
        up to the summation order of the scatter's float atomics.
        """
        if ticks < 0:
            raise ValueError("ticks must be non-negative")
        cycle = list(drive) if isinstance(drive, (list, tuple)) else None
        if cycle is not None and len(cycle) != graph_ticks:
            raise ValueError("a drive cycle needs one drive per graph tick")
        if self._needs_autograd(drive if cycle is None else 0.0, dendritic_drive):
            raise RuntimeError("run() is inference-only; use step() for autograd")
        self._refresh_current()
        if cycle is None and ticks < graph_ticks or ticks == 0:
            for _ in range(ticks):
                self.step(drive, dendritic_drive=dendritic_drive)
            return self.state
        if cycle is not None and ticks % graph_ticks:
            raise ValueError("with a drive cycle, ticks must be a multiple of graph_ticks")
        graph_ticks = min(graph_ticks, ticks)
        if not self.persistent_current.is_contiguous():
            self.persistent_current = self.persistent_current.contiguous()
        drives = [self._drive(x) for x in (cycle if cycle is not None else [drive])]
        u = [d[0] for d in drives]
        us = [d[1] for d in drives]
        v, vs = self._drive(dendritic_drive, "dendritic_drive")
        key = (graph_ticks, tuple(self.state.shape),
               tuple(None if x is None else (x.data_ptr(), x.stride()) for x in u), tuple(us),
               None if v is None else (v.data_ptr(), v.stride()), vs,
               self.persistent_current.data_ptr(), self.topology.weight_version)
        graphs = getattr(self, "_graphs", None)
        if graphs is None:
            graphs = self._graphs = {}
        entry = graphs.get(key)
        if entry is None:
            graphs.clear()
            entry = graphs[key] = _EventGraph(self, graph_ticks, u, us, v, vs)
        entry.load(self.state, self.dendritic_state, self.adaptation_state, self.emitted_state)
        for _ in range(ticks // graph_ticks):
            entry.replay()
        (self.state, self.dendritic_state, self.adaptation_state,
         self.emitted_state) = entry.result()
        self._tick += ticks // graph_ticks * graph_ticks
        for _ in range(ticks % graph_ticks):
            self.step(drive, dendritic_drive=dendritic_drive)
        self.last_backend = "native"
        return self.state

    def _autograd_step(self, drive, dendritic_drive, collect_stats: bool):
        """Differentiable PELS tick (runtime.py:264-314 with the emit rule above)."""
        self._refresh_current()
        state = self._autograd_advance(self.persistent_current, drive, dendritic_drive)
        residual = state - self.emitted_state
        active = residual.detach().abs() >= self.theta
        delta = torch.where(active, residual, torch.zeros_like(residual))
        self.persistent_current = self.persistent_current + self._autograd_propagate(delta)
        self.emitted_state = self.emitted_state + delta
        self.state = state
        self._tick += 1
        if not collect_stats:
            return self.state
        pairs = torch.nonzero(active, as_tuple=False)
        edges = int(self.topology.out_degree[pairs[:, 1]].sum()) if pairs.numel() else 0
        count = int(active.sum())
        return self.state, RuntimeStats("event" if count else "idle", count, edges)
