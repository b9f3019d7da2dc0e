"""ctypes binding of ``libneurosim_b200.so`` and the drop-in extension object.

``load_native_extension()`` returns an object with the hot-path functions of
the reference's pybind11 module ``neurosim_gpu_native``
(csrc/bindings.cpp:137-143):

* ``dendritic_step(state, dendrite, adaptation, params, rowptr, source, weight,
  input, input_scalar, dendritic_input, dendritic_scalar, width,
  block_scales=None, global_scale=None) -> [s, d, a]``
* ``dendritic_event(state, dendrite, adaptation, params, current, emitted,
  theta, out_rowptr, dst, out_weight_index, weight, input, input_scalar,
  dendritic_input, dendritic_scalar) -> [s, d, a, emitted]`` (updates
  ``current`` in place)

with the same argument meaning, the same ownership (inputs borrowed; outputs
are fresh views of one allocation) and the same errors (``RuntimeError``
before any launch, csrc/compartmental.cu:29-70, 182-210, 244-256).  Calls go
to the C ABI on the caller's current CUDA stream, so they can be captured in
CUDA graphs.  ``dendritic_event`` also accepts ``out_weight_index=None`` with
the source-major ``topology.weight``, which the scatter reads coalesced.

There is no fallback: if the library is missing or the tensors are not CUDA
float32, the call fails.
"""

from __future__ import annotations

import ctypes
import functools
from pathlib import Path

import torch

LIBRARY_PATH = Path(__file__).resolve().parent / "libneurosim_b200.so"

F32, F16, E4M3, NVFP4 = 0, 1, 2, 3


class _View(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("batch_stride", ctypes.c_int64),
                ("neuron_stride", ctypes.c_int64), ("scalar", ctypes.c_float)]


class _Out(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("batch_stride", ctypes.c_int64),
                ("neuron_stride", ctypes.c_int64)]


class _Params(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p * 6), ("stride", ctypes.c_int64 * 6)]


class _Tick(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int64), ("neurons", ctypes.c_int64),
                ("state", _View), ("dendrite", _View), ("adaptation", _View),
                ("input", _View), ("dendritic_input", _View), ("params", _Params)]


class _TickOut(ctypes.Structure):
    _fields_ = [("state", _Out), ("dendrite", _Out), ("adaptation", _Out)]


class _Csr(ctypes.Structure):
    _fields_ = [("n_edges", ctypes.c_int64), ("rowptr", ctypes.c_void_p),
                ("col", ctypes.c_void_p), ("weight", ctypes.c_void_p),
                ("format", ctypes.c_int32), ("block_scales", ctypes.c_void_p),
                ("global_scale", ctypes.c_void_p)]


class _OutCsr(ctypes.Structure):
    _fields_ = [("n_edges", ctypes.c_int64), ("rowptr", ctypes.c_void_p),
                ("dst", ctypes.c_void_p), ("weight_index", ctypes.c_void_p),
                ("weight", ctypes.c_void_p)]


class _TiledLayout(ctypes.Structure):
    _fields_ = [("ctas", ctypes.c_int32), ("blocks", ctypes.c_int32),
                ("block_cols", ctypes.c_int32), ("buffers", ctypes.c_int32),
                ("format", ctypes.c_int32), ("splits", ctypes.c_int32),
                ("split_chunks", ctypes.c_int32), ("chunk", ctypes.c_int32),
                ("n_stages", ctypes.c_int64), ("n_tasks", ctypes.c_int64),
                ("n_slots", ctypes.c_int64), ("n_scale_pairs", ctypes.c_int64),
                ("rows", ctypes.c_int64), ("cols", ctypes.c_int64),
                ("stage_ptr", ctypes.c_void_p), ("stage_block", ctypes.c_void_p),
                ("task_ptr", ctypes.c_void_p), ("tasks", ctypes.c_void_p),
                ("task_rows", ctypes.c_void_p), ("col", ctypes.c_void_p),
                ("weight", ctypes.c_void_p), ("scale_pairs", ctypes.c_void_p),
                ("global_scale", ctypes.c_void_p)]


MAX_PEERS = 8


class _PeerExchange(ctypes.Structure):
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("row_offset", ctypes.c_int64),
                ("gathered", (ctypes.c_void_p * 2) * MAX_PEERS),
                ("counters", ctypes.c_void_p * MAX_PEERS),
                ("epoch", ctypes.c_uint64)]


class _EventRows(ctypes.Structure):
    _fields_ = [("row_offset", ctypes.c_int64), ("cols", ctypes.c_int64),
                ("current", ctypes.c_void_p), ("emitted", _View), ("theta", ctypes.c_void_p),
                ("theta_stride", ctypes.c_int64)]


class _DeltaExchange(ctypes.Structure):
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("delta", (ctypes.c_void_p * 2) * MAX_PEERS),
                ("counters", ctypes.c_void_p * MAX_PEERS)]


class _ScatterRows(ctypes.Structure):
    _fields_ = [("n_edges", ctypes.c_int64), ("rowptr", ctypes.c_void_p),
                ("dst", ctypes.c_void_p), ("weight", ctypes.c_void_p)]


EVENT_ROWS_WORKSPACE = 256


class EventCounters(ctypes.Structure):
    """Head of the nsb_dendritic_event workspace (nsb_event_counters)."""

    _fields_ = [("emitted_sources", ctypes.c_uint32), ("reserved", ctypes.c_uint32),
                ("active_neurons", ctypes.c_uint64), ("active_edges", ctypes.c_uint64),
                ("reserved2", ctypes.c_uint64)]


EXPORTED_SYMBOLS = ("nsb_dendritic_step", "nsb_csr_propagate",
                    "nsb_dendritic_event_workspace_size", "nsb_dendritic_event",
                    "nsb_tiled_smem_bytes", "nsb_tiled_workspace_size", "nsb_dendritic_step_tiled",
                    "nsb_dendritic_run_tiled", "nsb_dendritic_run_tiled_peers",
                    "nsb_ipc_export", "nsb_ipc_import", "nsb_ipc_release", "nsb_tiled_propagate",
                    "nsb_dendritic_event_noalloc", "nsb_dendritic_step_rows",
                    "nsb_cluster_slots", "nsb_cluster_smem_bytes", "nsb_dendritic_run_cluster",
                    "nsb_dendritic_event_rows", "nsb_event_scatter_rows", "nsb_encode_weights",
                    "nsb_dendritic_event_hybrid", "nsb_dendritic_rollout_tiled",
                    "nsb_dendritic_rollout_tiled_peers", "nsb_dendritic_rollout_cluster",
                    "nsb_dendritic_event_rows_gated", "nsb_event_scatter_rows_gated",
                    "nsb_tiled_propagate_rows_gated", "nsb_last_error", "nsb_abi_version")


@functools.lru_cache(maxsize=1)
def load_library() -> ctypes.CDLL:
    """Open the in-tree library (no JIT, no fallback)."""
    if not LIBRARY_PATH.exists():
        raise RuntimeError(
            f"{LIBRARY_PATH.name} is missing: build it with `python -m neurosim_gpu_b200.build` "
            "(nvcc, sm_100a).  The native runtimes have no CPU or PyTorch fallback.")
    lib = ctypes.CDLL(str(LIBRARY_PATH))
    p = ctypes.POINTER
    lib.nsb_dendritic_step.argtypes = [p(_Tick), p(_Csr), ctypes.c_int32, p(_TickOut),
                                       ctypes.c_void_p]
    lib.nsb_csr_propagate.argtypes = [ctypes.c_int64, ctypes.c_int64, p(_Csr), p(_View),
                                      p(_Out), ctypes.c_void_p]
    lib.nsb_dendritic_event_workspace_size.argtypes = [ctypes.c_int64, ctypes.c_int64]
    lib.nsb_dendritic_event_workspace_size.restype = ctypes.c_size_t
    lib.nsb_dendritic_event.argtypes = [p(_Tick), ctypes.c_void_p, p(_View), ctypes.c_void_p,
                                        ctypes.c_int64, p(_OutCsr), p(_TickOut), p(_Out),
                                        ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
    lib.nsb_tiled_smem_bytes.argtypes = [ctypes.c_int32, ctypes.c_int32]
    lib.nsb_tiled_smem_bytes.restype = ctypes.c_size_t
    lib.nsb_tiled_workspace_size.argtypes = [p(_TiledLayout)]
    lib.nsb_tiled_workspace_size.restype = ctypes.c_size_t
    lib.nsb_dendritic_step_tiled.argtypes = [p(_Tick), p(_TiledLayout), ctypes.c_void_p,
                                             p(_TickOut), ctypes.c_void_p, ctypes.c_size_t,
                                             ctypes.c_void_p, ctypes.c_void_p]
    lib.nsb_dendritic_run_tiled.argtypes = [p(_Tick), p(_TiledLayout), ctypes.c_int64,
                                            p(_TickOut), ctypes.c_void_p, ctypes.c_size_t,
                                            ctypes.c_void_p, ctypes.c_void_p]
    lib.nsb_dendritic_rollout_tiled.argtypes = [p(_Tick), p(_TiledLayout), ctypes.c_int64,
                                                ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                                                p(_TickOut), ctypes.c_void_p, ctypes.c_size_t,
                                                ctypes.c_void_p, ctypes.c_void_p]
    lib.nsb_dendritic_rollout_tiled_peers.argtypes = [
        p(_Tick), p(_TiledLayout), ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
        ctypes.c_int64, p(_PeerExchange), p(_TickOut), ctypes.c_void_p, ctypes.c_size_t,
        ctypes.c_void_p, ctypes.c_void_p]
    lib.nsb_dendritic_run_tiled_peers.argtypes = [p(_Tick), p(_TiledLayout), ctypes.c_int64,
                                                  p(_PeerExchange), p(_TickOut), ctypes.c_void_p,
                                                  ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p]
    lib.nsb_ipc_export.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64)]
    lib.nsb_ipc_import.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]
    lib.nsb_ipc_release.argtypes = [ctypes.c_void_p]
    lib.nsb_dendritic_step_rows.argtypes = [p(_Tick), p(_Csr), p(_View), ctypes.c_int64,
                                            ctypes.c_int32, p(_TickOut), ctypes.c_void_p]
    lib.nsb_tiled_propagate.argtypes = [ctypes.c_int64, p(_TiledLayout), ctypes.c_void_p,
                                        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                        ctypes.c_void_p, ctypes.c_void_p]
    lib.nsb_dendritic_event_noalloc.argtypes = [p(_Tick), ctypes.c_void_p, p(_View),
                                                ctypes.c_void_p, ctypes.c_int64, p(_OutCsr),
                                                p(_TickOut), p(_Out), ctypes.c_void_p]
    lib.nsb_cluster_slots.argtypes = [ctypes.c_int64, ctypes.c_void_p]
    lib.nsb_cluster_slots.restype = ctypes.c_int64
    lib.nsb_cluster_smem_bytes.argtypes = [ctypes.c_int64, ctypes.c_int64]
    lib.nsb_cluster_smem_bytes.restype = ctypes.c_size_t
    lib.nsb_dendritic_rollout_cluster.argtypes = [
        p(_Tick), p(_Csr), ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
        ctypes.c_int64, p(_TickOut), ctypes.c_void_p, ctypes.c_void_p]
    lib.nsb_dendritic_run_cluster.argtypes = [p(_Tick), p(_Csr), ctypes.c_int64, ctypes.c_int64,
                                              p(_TickOut), ctypes.c_void_p, ctypes.c_void_p]
    lib.nsb_dendritic_event_rows.argtypes = [p(_Tick), p(_EventRows), ctypes.c_void_p,
                                             p(_DeltaExchange), p(_TickOut), p(_Out),
                                             ctypes.c_void_p, ctypes.c_void_p]
    lib.nsb_event_scatter_rows.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                           ctypes.c_void_p, p(_ScatterRows), ctypes.c_void_p,
                                           p(_DeltaExchange), ctypes.c_void_p, ctypes.c_void_p,
                                           ctypes.c_void_p]
    lib.nsb_dendritic_event_rows_gated.argtypes = [p(_Tick), p(_EventRows), p(_DeltaExchange),
                                                   ctypes.c_void_p, p(_TickOut), p(_Out),
                                                   ctypes.c_void_p, ctypes.c_void_p]
    lib.nsb_event_scatter_rows_gated.argtypes = [ctypes.c_int64, ctypes.c_int64, p(_ScatterRows),
                                                 ctypes.c_void_p, p(_DeltaExchange),
                                                 ctypes.c_uint64, ctypes.c_void_p,
                                                 ctypes.c_void_p, ctypes.c_void_p]
    lib.nsb_tiled_propagate_rows_gated.argtypes = [p(_TiledLayout), ctypes.c_void_p,
                                                   ctypes.c_size_t, ctypes.c_void_p,
                                                   ctypes.c_uint64, ctypes.c_void_p,
                                                   ctypes.c_void_p, ctypes.c_void_p]
    lib.nsb_encode_weights.argtypes = [ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64,
                                       ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_void_p, ctypes.c_void_p]
    lib.nsb_dendritic_event_hybrid.argtypes = [
        p(_Tick), ctypes.c_void_p, p(_View), ctypes.c_void_p, ctypes.c_int64, p(_OutCsr),
        p(_TiledLayout), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_uint64,
        p(_TickOut), p(_Out), ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p]
    lib.nsb_last_error.restype = ctypes.c_char_p
    lib.nsb_abi_version.restype = ctypes.c_int
    for name in EXPORTED_SYMBOLS:
        getattr(lib, name).restype = getattr(lib, name).restype or ctypes.c_int
    if lib.nsb_abi_version() != 14:
        raise RuntimeError("libneurosim_b200.so ABI version mismatch")
    return lib


def ipc_export(tensor: torch.Tensor) -> tuple[bytes, int]:
    """(64-byte CUDA IPC handle of the tensor's allocation, byte offset of the tensor)."""
    lib = load_library()
    handle = ctypes.create_string_buffer(64)
    offset = ctypes.c_uint64()
    with torch.cuda.device(tensor.device):
        _raise_on_status(lib, lib.nsb_ipc_export(tensor.data_ptr(), handle, ctypes.byref(offset)))
    return handle.raw, int(offset.value)


def ipc_import(handle: bytes, device: torch.device) -> int:
    """Map another process's allocation into ``device`` (peer access on); its base address."""
    lib = load_library()
    base = ctypes.c_void_p()
    with torch.cuda.device(device):
        _raise_on_status(lib, lib.nsb_ipc_import(ctypes.create_string_buffer(handle, 64),
                                                 ctypes.byref(base)))
    return int(base.value)


def ipc_release(base: int, device: torch.device) -> None:
    lib = load_library()
    with torch.cuda.device(device):
        _raise_on_status(lib, lib.nsb_ipc_release(base))


def _check(ok: bool, message: str) -> None:
    if not ok:
        raise RuntimeError(message)


def _raise_on_status(lib: ctypes.CDLL, status: int) -> None:
    if status != 0:
        raise RuntimeError(lib.nsb_last_error().decode() or f"libneurosim_b200 status {status}")


def _float_on(value: torch.Tensor, state: torch.Tensor) -> None:
    _check(value.is_cuda and value.device == state.device,
           "all tensors must be on the state's CUDA device")
    _check(value.dtype == torch.float32, "all values must be float32")


def _view(value: torch.Tensor, state: torch.Tensor) -> _View:
    _float_on(value, state)
    _check(value.shape == state.shape, "state/current/drive shape mismatch")
    return _View(value.data_ptr(), value.stride(0), value.stride(1), 0.0)


def _drive(value: torch.Tensor | None, scalar: float, state: torch.Tensor) -> _View:
    if value is not None:
        return _view(value, state)
    return _View(None, 0, 0, float(scalar))


def _params(values, state: torch.Tensor) -> _Params:
    _check(len(values) == 6, "six neuron parameter vectors are required")
    result = _Params()
    for i, value in enumerate(values):
        _float_on(value, state)
        _check(value.dim() == 1 and value.numel() == state.size(1),
               "parameters must have one value per neuron")
        result.data[i] = value.data_ptr()
        result.stride[i] = value.stride(0)
    return result


def _index(value: torch.Tensor, state: torch.Tensor) -> None:
    _check(value.device == state.device and value.dtype == torch.int32
           and value.is_contiguous() and value.dim() == 1,
           "indices must be contiguous int32 vectors on the state device")


def _check_state(state: torch.Tensor) -> None:
    _check(state.is_cuda and state.dtype == torch.float32, "state must be CUDA float32")
    _check(state.dim() == 2 and state.size(1) > 0, "state must be [B,N], N > 0")


def _outputs(planes: int, state: torch.Tensor, neuron_major: bool = True
             ) -> tuple[torch.Tensor, list[torch.Tensor]]:
    """One fresh block holding `planes` [B,N] outputs.

    With B > 1 and ``neuron_major`` the block is [planes, N, B] and the
    returned [B,N] views have strides (1, B): the next matrix tick then
    gathers all batch rows of a source neuron from one 32-byte sector.
    """
    batch, neurons = state.shape
    if batch > 1 and neuron_major:
        block = torch.empty((planes, neurons, batch), device=state.device, dtype=torch.float32)
        return block, [block[i].t() for i in range(planes)]
    block = torch.empty((planes, batch, neurons), device=state.device, dtype=torch.float32)
    return block, [block[i] for i in range(planes)]


def _out(view: torch.Tensor) -> _Out:
    return _Out(view.data_ptr(), view.stride(0), view.stride(1))


def _tick(state, dendrite, adaptation, params, input, input_scalar, dendritic_input,
          dendritic_scalar) -> _Tick:
    return _Tick(state.size(0), state.size(1), _view(state, state), _view(dendrite, state),
                 _view(adaptation, state), _drive(input, input_scalar, state),
                 _drive(dendritic_input, dendritic_scalar, state), _params(params, state))


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def csr_arguments(rowptr: torch.Tensor, source: torch.Tensor, weight: torch.Tensor,
                  block_scales: torch.Tensor | None, global_scale: torch.Tensor | None,
                  state: torch.Tensor) -> _Csr:
    """Validate a destination-major CSR (compartmental.cu:187-209) into the C struct."""
    _index(rowptr, state)
    _index(source, state)
    edges = source.numel()
    quantized = weight.dtype == torch.uint8
    _check(weight.device == state.device and weight.is_contiguous() and weight.dim() == 1,
           "CSR weights must be a contiguous vector on the state device")
    _check(rowptr.numel() == state.size(1) + 1, "invalid CSR geometry")
    scale_ptr = scales_ptr = None
    if quantized:
        _check(global_scale is not None, "quantized CSR weights require a global scale")
        _float_on(global_scale, state)
        _check(global_scale.numel() == 1, "global scale must have one value")
        _check(weight.numel() == ((edges + 1) // 2 if block_scales is not None else edges),
               "invalid quantized CSR weight count")
        if block_scales is not None:
            _check(block_scales.device == state.device and block_scales.dtype == torch.uint8
                   and block_scales.is_contiguous() and block_scales.dim() == 1
                   and block_scales.numel() == (edges + 15) // 16,
                   "invalid NVFP4 block scales")
            scales_ptr = block_scales.data_ptr() if block_scales.numel() else None
            fmt = NVFP4
        else:
            fmt = E4M3
        scale_ptr = global_scale.data_ptr()
    else:
        _check(block_scales is None and global_scale is None and weight.numel() == edges
               and weight.dtype in (torch.float32, torch.float16),
               "invalid floating-point CSR weights")
        fmt = F32 if weight.dtype == torch.float32 else F16
    return _Csr(edges, rowptr.data_ptr(), source.data_ptr() if edges else None,
                weight.data_ptr() if edges else None, fmt, scales_ptr, scale_ptr)


class DendriticExtension:
    """The hot-path subset of the reference's ``neurosim_gpu_native`` module."""

    def __init__(self) -> None:
        self.lib = load_library()

    # -- matrix tick ---------------------------------------------------------
    def prepare_step(self, state, dendrite, adaptation, params, rowptr, source, weight,
                     input, input_scalar, dendritic_input, dendritic_scalar, width,
                     block_scales=None, global_scale=None, *, out):
        """Validate once and return a callable that enqueues the tick into ``out``.

        ``out`` is a triple of writable [B,N] float32 tensors (s', d', a').  The
        callable launches on the stream that is current when it is called, so
        it can be captured into a CUDA graph.
        """
        _check_state(state)
        tick = _tick(state, dendrite, adaptation, params, input, input_scalar,
                     dendritic_input, dendritic_scalar)
        csr = csr_arguments(rowptr, source, weight, block_scales, global_scale, state)
        _check(width in (4, 8, 16, 32), "width must be 4, 8, 16 or 32")
        _check(len(out) == 3, "three output tensors are required")
        for view in out:
            _float_on(view, state)
            _check(view.shape == state.shape, "output shape mismatch")
        result = _TickOut(_out(out[0]), _out(out[1]), _out(out[2]))
        lib, device, lanes = self.lib, state.device, int(width)
        keep = (state, dendrite, adaptation, params, rowptr, source, weight, input,
                dendritic_input, block_scales, global_scale, out)

        def launch() -> None:
            assert keep is not None
            with torch.cuda.device(device):
                status = lib.nsb_dendritic_step(ctypes.byref(tick), ctypes.byref(csr), lanes,
                                                ctypes.byref(result), _stream(device))
            _raise_on_status(lib, status)

        return launch

    def prepare_step_tiled(self, state, dendrite, adaptation, params, layout, input,
                           input_scalar, dendritic_input, dendritic_scalar, *, out, status=None,
                           source=None, ticks=None, rollout=None):
        """Like :meth:`prepare_step` for B = 1 over a :class:`~neurosim_gpu_b200.tiled.TiledLayout`.

        ``source`` (optional) is the full gathered state of ``layout.cols``
        floats when ``state`` holds only this layout's rows (row sharding).
        With ``ticks`` = T the launch runs T ticks in one cooperative kernel
        (``nsb_dendritic_run_tiled``): the first reads ``state`` / ``dendrite``
        / ``adaptation``, the later ones update ``out`` in place.  The launch
        uses the layout's own workspace (:meth:`TiledLayout.workspace`).
        ``rollout`` = ``(drive_tick_stride, history)`` gives each of the T ticks
        its own drive (tick k reads ``input`` moved on by k * drive_tick_stride
        floats) and, with ``history`` a contiguous [T, 1, N] tensor, keeps every
        tick's soma state there (``nsb_dendritic_rollout_tiled``).
        """
        _check_state(state)
        _check(state.size(0) == 1, "the tiled tick takes B = 1")
        gather = state if source is None else source
        _check(gather.is_cuda and gather.dtype == torch.float32 and gather.is_contiguous()
               and gather.data_ptr() % 16 == 0 and gather.numel() == layout.cols,
               "the tiled tick needs a contiguous, 16-byte aligned state")
        _check(layout.neurons == state.size(1), "layout and state neuron counts differ")
        _check(ticks is None or source is None, "multi-tick runs gather from their own state")
        drive_stride, history = (0, None) if rollout is None else rollout
        _check(rollout is None or ticks is not None, "a rollout needs ticks")
        if history is not None:
            _float_on(history, state)
            _check(history.is_contiguous() and history.numel() == ticks * layout.neurons,
                   "history must be a contiguous [T, 1, N] tensor")
        if drive_stride and input is not None:
            _check(input.numel() + (ticks - 1) * drive_stride <= input.untyped_storage().nbytes()
                   // 4 - input.storage_offset(), "the rollout's drives exceed their storage")
        tick = _tick(state, dendrite, adaptation, params, input, input_scalar,
                     dendritic_input, dendritic_scalar)
        for view in out:
            _float_on(view, state)
            _check(view.shape == state.shape, "output shape mismatch")
        result = _TickOut(_out(out[0]), _out(out[1]), _out(out[2]))
        c_layout = layout.c_struct()
        workspace = layout.workspace()
        status_ptr = status.data_ptr() if status is not None else None
        source_ptr = source.data_ptr() if source is not None else None
        lib, device = self.lib, state.device
        keep = (state, dendrite, adaptation, params, layout, input, dendritic_input, out, status,
                source, workspace, history)
        history_ptr = history.data_ptr() if history is not None else None

        def launch() -> None:
            assert keep is not None
            with torch.cuda.device(device):
                if rollout is not None:
                    code = lib.nsb_dendritic_rollout_tiled(
                        ctypes.byref(tick), ctypes.byref(c_layout), int(ticks), int(drive_stride),
                        history_ptr, layout.neurons, ctypes.byref(result), workspace.data_ptr(),
                        workspace.numel(), status_ptr, _stream(device))
                elif ticks is None:
                    code = lib.nsb_dendritic_step_tiled(
                        ctypes.byref(tick), ctypes.byref(c_layout), source_ptr,
                        ctypes.byref(result), workspace.data_ptr(), workspace.numel(), status_ptr,
                        _stream(device))
                else:
                    code = lib.nsb_dendritic_run_tiled(
                        ctypes.byref(tick), ctypes.byref(c_layout), int(ticks),
                        ctypes.byref(result), workspace.data_ptr(), workspace.numel(), status_ptr,
                        _stream(device))
            _raise_on_status(lib, code)

        return launch

    def cluster_plan(self, rowptr: torch.Tensor) -> tuple[int, int]:
        """``(max_slots, shared bytes per CTA)`` of the small-graph cluster tick."""
        host = rowptr.detach().to("cpu", torch.int32).contiguous()
        neurons = host.numel() - 1
        _check(neurons > 0, "invalid CSR geometry")
        slots = int(self.lib.nsb_cluster_slots(neurons, host.data_ptr()))
        _check(slots >= 0, "invalid CSR geometry")
        return slots, int(self.lib.nsb_cluster_smem_bytes(neurons, slots))

    def prepare_run_cluster(self, state, dendrite, adaptation, params, rowptr, source, weight,
                            input, input_scalar, dendritic_input, dendritic_scalar,
                            block_scales=None, global_scale=None, *, out, ticks, max_slots,
                            status=None, rollout=None):
        """A launch callable for ``ticks`` B = 1 ticks on one thread-block cluster.

        ``max_slots`` comes from :meth:`cluster_plan` of the same ``rowptr``.
        The first tick reads ``state`` / ``dendrite`` / ``adaptation``, the last
        writes ``out``; nothing else touches global memory in between, except
        for a ``rollout`` = ``(drive_tick_stride, history)``: tick k reads
        ``input`` moved on by k * drive_tick_stride floats and writes its soma
        state to ``history[k]`` (a contiguous [T, 1, N] tensor, or None)
        (``nsb_dendritic_rollout_cluster``).
        """
        _check_state(state)
        _check(state.size(0) == 1, "the cluster tick takes B = 1")
        _check(int(ticks) >= 1, "ticks must be positive")
        tick = _tick(state, dendrite, adaptation, params, input, input_scalar,
                     dendritic_input, dendritic_scalar)
        csr = csr_arguments(rowptr, source, weight, block_scales, global_scale, state)
        _check(len(out) == 3, "three output tensors are required")
        for view in out:
            _float_on(view, state)
            _check(view.shape == state.shape, "output shape mismatch")
        result = _TickOut(_out(out[0]), _out(out[1]), _out(out[2]))
        status_ptr = status.data_ptr() if status is not None else None
        lib, device, slots, count = self.lib, state.device, int(max_slots), int(ticks)
        drive_stride, history = (0, None) if rollout is None else rollout
        if history is not None:
            _float_on(history, state)
            _check(history.is_contiguous() and history.numel() == count * state.size(1),
                   "history must be a contiguous [T, 1, N] tensor")
        if drive_stride and input is not None:
            _check(input.numel() + (count - 1) * drive_stride <= input.untyped_storage().nbytes()
                   // 4 - input.storage_offset(), "the rollout's drives exceed their storage")
        history_ptr = history.data_ptr() if history is not None else None
        keep = (state, dendrite, adaptation, params, rowptr, source, weight, input,
                dendritic_input, block_scales, global_scale, out, status, history)

        def launch() -> None:
            assert keep is not None
            with torch.cuda.device(device):
                if rollout is None:
                    code = lib.nsb_dendritic_run_cluster(
                        ctypes.byref(tick), ctypes.byref(csr), slots, count,
                        ctypes.byref(result), status_ptr, _stream(device))
                else:
                    code = lib.nsb_dendritic_rollout_cluster(
                        ctypes.byref(tick), ctypes.byref(csr), slots, count, int(drive_stride),
                        history_ptr, state.size(1), ctypes.byref(result), status_ptr,
                        _stream(device))
            _raise_on_status(lib, code)

        return launch

    # -- weight encoder -----------------------------------------------------------
    def encode_weights(self, weight: torch.Tensor, precision: str):
        """``encode_sparse_weights`` on the device (``nsb_encode_weights``): returns
        (codes uint8, block scales uint8 or None, global scale float32 [1])."""
        _check(weight.is_cuda and weight.dtype == torch.float32 and weight.dim() == 1
               and weight.is_contiguous(), "the encoder takes a contiguous CUDA float32 vector")
        _check(precision in ("fp8", "nvfp4"), "compressed CSR encoding requires fp8 or nvfp4")
        n = weight.numel()
        device = weight.device
        nvfp4 = precision == "nvfp4"
        codes = torch.empty((n + 1) // 2 if nvfp4 else n, dtype=torch.uint8, device=device)
        scales = torch.empty((n + 15) // 16, dtype=torch.uint8, device=device) if nvfp4 else None
        scale = torch.empty(1, dtype=torch.float32, device=device)
        workspace = torch.empty(64, dtype=torch.int32, device=device)
        with torch.cuda.device(device):
            status = self.lib.nsb_encode_weights(
                NVFP4 if nvfp4 else E4M3, weight.data_ptr() if n else None, n,
                codes.data_ptr() if codes.numel() else None,
                scales.data_ptr() if scales is not None and scales.numel() else None,
                scale.data_ptr(), workspace.data_ptr(), _stream(device))
        _raise_on_status(self.lib, status)
        return codes, scales, scale

    # -- row-sharded PELS --------------------------------------------------------
    def prepare_event_rows(self, state, dendrite, adaptation, params, current, emitted, theta,
                           input, input_scalar, dendritic_input, dendritic_scalar, *,
                           row_offset, cols, delta, exchange, out, workspace, out_degree=None):
        """A launch callable for the advance + emit half of a row-sharded PELS tick.

        ``state`` ... ``theta`` are this rank's rows ([B, rows] / [rows]);
        ``delta`` is the gathered [cols, B] delta buffer (None with an
        ``exchange``, a :class:`_DeltaExchange`); ``out`` is (s, d, a, emitted).
        ``out_degree`` (int32 [rows], with an exchange, B = 1): also count the
        emitting rows' out-edges for a gated tick
        (``nsb_dendritic_event_rows_gated``).
        """
        _check_state(state)
        tick = _tick(state, dendrite, adaptation, params, input, input_scalar,
                     dendritic_input, dendritic_scalar)
        _view(current, state)
        _check(current.is_contiguous(), "persistent current must be contiguous")
        emitted_view = _view(emitted, state)
        _float_on(theta, state)
        _check(theta.dim() == 1 and theta.numel() == state.size(1), "theta must have a value per row")
        _check((delta is None) != (exchange is None), "give a delta buffer or an exchange")
        if delta is not None:
            _float_on(delta, state)
            _check(delta.is_contiguous() and delta.numel() == cols * state.size(0),
                   "delta must be a contiguous [cols, B] buffer")
        _check(len(out) == 4, "four output tensors are required")
        for view in out:
            _float_on(view, state)
            _check(view.shape == state.shape, "output shape mismatch")
        _check(workspace.device == state.device and workspace.numel() >= EVENT_ROWS_WORKSPACE,
               "row-event workspace too small")
        ev = _EventRows(int(row_offset), int(cols), current.data_ptr(), emitted_view,
                        theta.data_ptr(), theta.stride(0))
        result = _TickOut(_out(out[0]), _out(out[1]), _out(out[2]))
        out_emitted = _out(out[3])
        delta_ptr = delta.data_ptr() if delta is not None else None
        x = ctypes.byref(exchange) if exchange is not None else None
        lib, device = self.lib, state.device
        keep = (state, dendrite, adaptation, params, current, emitted, theta, input,
                dendritic_input, delta, exchange, out, workspace, out_degree)
        if out_degree is not None:
            _check(exchange is not None and state.size(0) == 1,
                   "a gated row tick needs B = 1 and an exchange")
            _check(out_degree.device == state.device and out_degree.dtype == torch.int32
                   and out_degree.is_contiguous() and out_degree.numel() == state.size(1),
                   "out_degree must be a contiguous int32 [rows]")

        def launch() -> None:
            assert keep is not None
            with torch.cuda.device(device):
                if out_degree is not None:
                    code = lib.nsb_dendritic_event_rows_gated(
                        ctypes.byref(tick), ctypes.byref(ev), x, out_degree.data_ptr(),
                        ctypes.byref(result), ctypes.byref(out_emitted), workspace.data_ptr(),
                        _stream(device))
                else:
                    code = lib.nsb_dendritic_event_rows(ctypes.byref(tick), ctypes.byref(ev),
                                                        delta_ptr, x, ctypes.byref(result),
                                                        ctypes.byref(out_emitted),
                                                        workspace.data_ptr(), _stream(device))
            _raise_on_status(lib, code)

        return launch

    def prepare_scatter_rows(self, batch, neurons, rows, delta, rowptr, dst, weight, current, *,
                             exchange, workspace, status=None, gate_edges=0):
        """A launch callable for the scatter half of a row-sharded PELS tick.

        ``gate_edges`` > 0 (B = 1, with an exchange): the gated scatter of a
        hybrid tick (``nsb_event_scatter_rows_gated``), which returns after its
        wait when the ranks' emitting sources have >= gate_edges out-edges.
        """
        _check(current.is_cuda and current.dtype == torch.float32 and current.is_contiguous()
               and tuple(current.shape) == (batch, rows), "current must be a contiguous [B, rows]")
        for array in (rowptr, dst):
            _check(array.device == current.device and array.dtype == torch.int32
                   and array.is_contiguous(), "index arrays must be contiguous int32")
        _check(weight.device == current.device and weight.dtype == torch.float32
               and weight.is_contiguous() and weight.numel() == dst.numel()
               and rowptr.numel() == neurons + 1, "invalid row-scatter topology geometry")
        _check((delta is None) != (exchange is None), "give a delta buffer or an exchange")
        edges = dst.numel()
        csr = _ScatterRows(edges, rowptr.data_ptr(), dst.data_ptr() if edges else None,
                           weight.data_ptr() if edges else None)
        delta_ptr = delta.data_ptr() if delta is not None else None
        x = ctypes.byref(exchange) if exchange is not None else None
        status_ptr = status.data_ptr() if status is not None else None
        lib, device = self.lib, current.device
        keep = (delta, rowptr, dst, weight, current, exchange, workspace, status)

        def launch() -> None:
            assert keep is not None
            with torch.cuda.device(device):
                if gate_edges:
                    code = lib.nsb_event_scatter_rows_gated(
                        int(neurons), int(rows), ctypes.byref(csr), current.data_ptr(), x,
                        int(gate_edges), workspace.data_ptr(), status_ptr, _stream(device))
                else:
                    code = lib.nsb_event_scatter_rows(int(batch), int(neurons), int(rows),
                                                      delta_ptr, ctypes.byref(csr),
                                                      current.data_ptr(), x,
                                                      workspace.data_ptr(), status_ptr,
                                                      _stream(device))
            _raise_on_status(lib, code)

        return launch

    def prepare_propagate_rows_gated(self, layout, current, gate_edges, *, workspace,
                                     status=None):
        """A launch callable for the gated tiled propagate of a hybrid row-sharded
        tick (``nsb_tiled_propagate_rows_gated``): at or above the gate,
        ``current`` ([1, rows]) += W[rows, :] @ the tick's gathered deltas."""
        _check(current.is_cuda and current.dtype == torch.float32 and current.is_contiguous()
               and current.numel() == layout.neurons, "current must be a contiguous [1, rows]")
        _check(layout.format == F32, "the gated propagate takes a float32 layout")
        _check(int(gate_edges) >= 1, "gate_edges must be at least 1")
        c_layout = layout.c_struct()
        tiled_workspace = layout.workspace()
        status_ptr = status.data_ptr() if status is not None else None
        lib, device = self.lib, current.device
        keep = (layout, current, workspace, status, tiled_workspace)

        def launch() -> None:
            assert keep is not None
            with torch.cuda.device(device):
                code = lib.nsb_tiled_propagate_rows_gated(
                    ctypes.byref(c_layout), tiled_workspace.data_ptr(), tiled_workspace.numel(),
                    current.data_ptr(), int(gate_edges), workspace.data_ptr(), status_ptr,
                    _stream(device))
            _raise_on_status(lib, code)

        return launch

    def prepare_run_tiled_peers(self, state, dendrite, adaptation, params, layout, input,
                                input_scalar, dendritic_input, dendritic_scalar, *, out, ticks,
                                exchange, status=None, rollout=None):
        """A launch callable for ``ticks`` row-sharded ticks with the exchange in the kernel.

        ``exchange`` is a :class:`_PeerExchange` (see ``nsb_dendritic_run_tiled_peers``);
        ``state`` is this rank's rows of the current gathered buffer, ``out`` the
        rows' dendrite / adaptation outputs (``out[0]`` is not written).
        ``rollout`` = ``(drive_tick_stride, history)``: tick k reads ``input``
        moved on by k * drive_tick_stride floats and writes the rows' new soma
        state into ``history[k]`` (a contiguous [T, 1, rows] tensor, or None)
        (``nsb_dendritic_rollout_tiled_peers``).
        """
        _check_state(state)
        _check(state.size(0) == 1, "the tiled tick takes B = 1")
        _check(layout.neurons == state.size(1), "layout and state neuron counts differ")
        tick = _tick(state, dendrite, adaptation, params, input, input_scalar,
                     dendritic_input, dendritic_scalar)
        for view in out:
            _float_on(view, state)
            _check(view.shape == state.shape, "output shape mismatch")
        result = _TickOut(_out(out[0]), _out(out[1]), _out(out[2]))
        c_layout = layout.c_struct()
        workspace = layout.workspace()
        status_ptr = status.data_ptr() if status is not None else None
        lib, device = self.lib, state.device
        drive_stride, history = (0, None) if rollout is None else rollout
        if history is not None:
            _float_on(history, state)
            _check(history.is_contiguous() and history.numel() == ticks * layout.neurons,
                   "history must be a contiguous [T, 1, rows] tensor")
        if drive_stride and input is not None:
            _check(input.numel() + (ticks - 1) * drive_stride <= input.untyped_storage().nbytes()
                   // 4 - input.storage_offset(), "the rollout's drives exceed their storage")
        history_ptr = history.data_ptr() if history is not None else None
        keep = (state, dendrite, adaptation, params, layout, input, dendritic_input, out, status,
                workspace, exchange, history)

        def launch() -> None:
            assert keep is not None
            with torch.cuda.device(device):
                if rollout is None:
                    code = lib.nsb_dendritic_run_tiled_peers(
                        ctypes.byref(tick), ctypes.byref(c_layout), int(ticks),
                        ctypes.byref(exchange), ctypes.byref(result), workspace.data_ptr(),
                        workspace.numel(), status_ptr, _stream(device))
                else:
                    code = lib.nsb_dendritic_rollout_tiled_peers(
                        ctypes.byref(tick), ctypes.byref(c_layout), int(ticks), int(drive_stride),
                        history_ptr, layout.neurons, ctypes.byref(exchange),
                        ctypes.byref(result), workspace.data_ptr(), workspace.numel(),
                        status_ptr, _stream(device))
            _raise_on_status(lib, code)

        return launch

    def prepare_step_rows(self, state, dendrite, adaptation, params, rowptr, source_col, weight,
                          input, input_scalar, dendritic_input, dendritic_scalar, width,
                          block_scales=None, global_scale=None, *, source, out):
        """A launch callable for a block of rows against the full gathered ``source``.

        ``state`` / ``dendrite`` / ``adaptation`` / drives / params are the rows'
        own ([B, rows]); the CSR holds those rows with columns indexing
        ``source`` ([B, n_cols]); ``out`` receives the rows' new states.
        """
        _check_state(state)
        tick = _tick(state, dendrite, adaptation, params, input, input_scalar,
                     dendritic_input, dendritic_scalar)
        _check(source.is_cuda and source.device == state.device and source.dtype == torch.float32
               and source.dim() == 2 and source.size(0) == state.size(0),
               "the gathered source must be a [B, n_cols] float32 tensor on the state device")
        csr = csr_arguments(rowptr, source_col, weight, block_scales, global_scale, state)
        _check(width in (4, 8, 16, 32), "width must be 4, 8, 16 or 32")
        for view in out:
            _float_on(view, state)
            _check(view.shape == state.shape, "output shape mismatch")
        result = _TickOut(_out(out[0]), _out(out[1]), _out(out[2]))
        src = _View(source.data_ptr(), source.stride(0), source.stride(1), 0.0)
        lib, device, lanes, cols = self.lib, state.device, int(width), source.size(1)
        keep = (state, dendrite, adaptation, params, rowptr, source_col, weight, input,
                dendritic_input, block_scales, global_scale, out, source)

        def launch() -> None:
            assert keep is not None
            with torch.cuda.device(device):
                code = lib.nsb_dendritic_step_rows(ctypes.byref(tick), ctypes.byref(csr),
                                                   ctypes.byref(src), cols, lanes,
                                                   ctypes.byref(result), _stream(device))
            _raise_on_status(lib, code)

        return launch

    def dendritic_step_tiled(self, state, dendrite, adaptation, params, layout, input,
                             input_scalar, dendritic_input, dendritic_scalar, status=None):
        _check_state(state)
        _, views = _outputs(3, state)
        self.prepare_step_tiled(state, dendrite, adaptation, params, layout, input, input_scalar,
                                dendritic_input, dendritic_scalar, out=views, status=status)()
        return views

    def tiled_propagate(self, layout, x, status=None):
        """j = W @ x for x [1,N] over a tiled layout; a fresh [1,N] tensor."""
        _check_state(x)
        _check(x.size(0) == 1 and x.stride(1) == 1 and x.data_ptr() % 16 == 0
               and layout.cols == layout.neurons == x.size(1),
               "the tiled product needs a contiguous, 16-byte aligned [1,N] source")
        result = torch.empty_like(x, memory_format=torch.contiguous_format)
        c_layout = layout.c_struct()
        workspace = layout.workspace()
        with torch.cuda.device(x.device):
            code = self.lib.nsb_tiled_propagate(x.size(1), ctypes.byref(c_layout), x.data_ptr(),
                                                result.data_ptr(), workspace.data_ptr(),
                                                workspace.numel(),
                                                status.data_ptr() if status is not None else None,
                                                _stream(x.device))
        _raise_on_status(self.lib, code)
        return result

    def dendritic_step(self, state, dendrite, adaptation, params, rowptr, source, weight,
                       input, input_scalar, dendritic_input, dendritic_scalar, width,
                       block_scales=None, global_scale=None):
        _check_state(state)
        _, views = _outputs(3, state)
        self.prepare_step(state, dendrite, adaptation, params, rowptr, source, weight, input,
                          input_scalar, dendritic_input, dendritic_scalar, width, block_scales,
                          global_scale, out=views)()
        return views

    # -- bare product --------------------------------------------------------
    def csr_propagate(self, rowptr, source, weight, x, block_scales=None, global_scale=None):
        """j = W @ x for x [B,N] in any weight format; a fresh contiguous [B,N] tensor."""
        _check_state(x)
        csr = csr_arguments(rowptr, source, weight, block_scales, global_scale, x)
        result = torch.empty(x.shape, device=x.device, dtype=torch.float32)
        src = _View(x.data_ptr(), x.stride(0), x.stride(1), 0.0)
        out = _Out(result.data_ptr(), result.stride(0), result.stride(1))
        with torch.cuda.device(x.device):
            status = self.lib.nsb_csr_propagate(x.size(0), x.size(1), ctypes.byref(csr),
                                                ctypes.byref(src), ctypes.byref(out),
                                                _stream(x.device))
        _raise_on_status(self.lib, status)
        return result

    # -- PELS tick -----------------------------------------------------------
    def event_workspace(self, state: torch.Tensor) -> torch.Tensor:
        size = int(self.lib.nsb_dendritic_event_workspace_size(state.size(0), state.size(1)))
        return torch.empty(size, dtype=torch.uint8, device=state.device)

    def dendritic_event(self, state, dendrite, adaptation, params, current, emitted, theta,
                        out_rowptr, dst, out_weight_index, weight, input, input_scalar,
                        dendritic_input, dendritic_scalar, *, workspace=None, hybrid=None):
        """The PELS tick (``dendritic_event``).  ``hybrid`` = (tiled layout of the
        float32 destination CSR, dense [N] delta buffer, gate in active edges,
        status word) selects ``nsb_dendritic_event_hybrid`` (B = 1)."""
        _check_state(state)
        tick = _tick(state, dendrite, adaptation, params, input, input_scalar,
                     dendritic_input, dendritic_scalar)
        emitted_view = _view(emitted, state)
        _view(current, state)
        _check(current.is_contiguous(), "persistent current must be contiguous")
        _index(out_rowptr, state)
        _index(dst, state)
        if out_weight_index is not None:
            _index(out_weight_index, state)
        _float_on(weight, state)
        _float_on(theta, state)
        _check(out_rowptr.numel() == state.size(1) + 1 and dst.numel() == weight.numel()
               and (out_weight_index is None or dst.numel() == out_weight_index.numel())
               and weight.is_contiguous() and weight.dim() == 1,
               "invalid event topology geometry")
        _check(theta.dim() == 1 and theta.numel() == state.size(1), "theta must have N values")
        edges = dst.numel()
        out_csr = _OutCsr(edges, out_rowptr.data_ptr(), dst.data_ptr() if edges else None,
                          out_weight_index.data_ptr() if (out_weight_index is not None and edges)
                          else None, weight.data_ptr() if edges else None)
        # The PELS tick gathers nothing, so its outputs stay batch-major like the current.
        block, views = _outputs(4, state, neuron_major=False)
        out = _TickOut(_out(views[0]), _out(views[1]), _out(views[2]))
        out_emitted = _out(views[3])
        if workspace is None:
            workspace = self.event_workspace(state)
        with torch.cuda.device(state.device):
            if hybrid is None:
                status = self.lib.nsb_dendritic_event(
                    ctypes.byref(tick), current.data_ptr(), ctypes.byref(emitted_view),
                    theta.data_ptr(), theta.stride(0), ctypes.byref(out_csr), ctypes.byref(out),
                    ctypes.byref(out_emitted), workspace.data_ptr(), workspace.numel(),
                    _stream(state.device))
            else:
                layout, dense, gate, word = hybrid
                _float_on(dense, state)
                _check(dense.is_contiguous() and dense.numel() == state.size(1),
                       "the hybrid delta buffer must be a contiguous [N]")
                c_layout = layout.c_struct()
                tiled_ws = layout.workspace()
                status = self.lib.nsb_dendritic_event_hybrid(
                    ctypes.byref(tick), current.data_ptr(), ctypes.byref(emitted_view),
                    theta.data_ptr(), theta.stride(0), ctypes.byref(out_csr),
                    ctypes.byref(c_layout), tiled_ws.data_ptr(), tiled_ws.numel(),
                    dense.data_ptr(), int(gate), ctypes.byref(out), ctypes.byref(out_emitted),
                    workspace.data_ptr(), workspace.numel(),
                    word.data_ptr() if word is not None else None, _stream(state.device))
        _raise_on_status(self.lib, status)
        return views


def _event_noalloc(ext: DendriticExtension, state, dendrite, adaptation, params, current,
                   emitted, theta, out_rowptr, dst, out_weight_index, weight, input,
                   input_scalar, dendritic_input, dendritic_scalar, *, out=None):
    """PELS tick through ``nsb_dendritic_event_noalloc``: no workspace from the caller.

    For hosts that cannot give the library scratch memory (device memory
    reserved up front by the application's own pool, or a foreign-language host
    without a CUDA allocator).  The library's fixed scratch array is shared by
    all such calls on a GPU, so calls must not overlap on the GPU.  Outputs are
    allocated here, as in :meth:`DendriticExtension.dendritic_event`, unless
    ``out`` gives the four [B, N] float32 tensors (s', d', a', emitted') to
    write, in which case nothing is allocated on the device.
    """
    _check_state(state)
    tick = _tick(state, dendrite, adaptation, params, input, input_scalar, dendritic_input,
                 dendritic_scalar)
    emitted_view = _view(emitted, state)
    _view(current, state)
    _check(current.is_contiguous(), "persistent current must be contiguous")
    _index(out_rowptr, state)
    _index(dst, state)
    if out_weight_index is not None:
        _index(out_weight_index, state)
    _float_on(weight, state)
    _float_on(theta, state)
    _check(theta.dim() == 1 and theta.numel() == state.size(1), "theta must have N values")
    edges = dst.numel()
    out_csr = _OutCsr(edges, out_rowptr.data_ptr(), dst.data_ptr() if edges else None,
                      out_weight_index.data_ptr() if (out_weight_index is not None and edges)
                      else None, weight.data_ptr() if edges else None)
    if out is None:
        _, views = _outputs(4, state, neuron_major=False)
    else:
        _check(len(out) == 4, "four output tensors are required")
        for view in out:
            _float_on(view, state)
            _check(view.shape == state.shape, "output shape mismatch")
        views = list(out)
    out = _TickOut(_out(views[0]), _out(views[1]), _out(views[2]))
    out_emitted = _out(views[3])
    with torch.cuda.device(state.device):
        status = ext.lib.nsb_dendritic_event_noalloc(
            ctypes.byref(tick), current.data_ptr(), ctypes.byref(emitted_view), theta.data_ptr(),
            theta.stride(0), ctypes.byref(out_csr), ctypes.byref(out), ctypes.byref(out_emitted),
            _stream(state.device))
    _raise_on_status(ext.lib, status)
    return views


DendriticExtension.dendritic_event_noalloc = _event_noalloc


@functools.lru_cache(maxsize=1)
def load_native_extension(verbose: bool = False) -> DendriticExtension:
    """The drop-in for the reference's loader (native.py:59-69); no JIT build."""
    return DendriticExtension()
