"""The C ABI library loads, exports what include/*.h declares, and rejects bad calls.

Runs without a GPU: every call below fails argument validation (or has B = 0)
before the library touches CUDA.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from neurosim_gpu_b200 import native

HEADERS = sorted((Path(__file__).resolve().parents[1] / "include").glob("*.h"))


def declared_symbols() -> list[str]:
    names = []
    for header in HEADERS:
        text = header.read_text()
        names += re.findall(r"NSB_API\s+[\w\s\*]+?\b(nsb_\w+)\s*\(", text)
    return names


@pytest.fixture(scope="module")
def lib():
    return native.load_library()


def test_every_declared_symbol_is_exported(lib):
    names = declared_symbols()
    assert "nsb_dendritic_step" in names and "nsb_dendritic_event" in names
    for name in names:
        assert hasattr(lib, name), name
    assert set(native.EXPORTED_SYMBOLS) <= set(names)


def test_abi_version_matches_header(lib):
    text = "".join(h.read_text() for h in HEADERS)
    version = int(re.search(r"#define NSB_ABI_VERSION (\d+)", text).group(1))
    assert lib.nsb_abi_version() == version


def test_event_workspace_size(lib):
    assert lib.nsb_dendritic_event_workspace_size(8, 50000) == 256 + 8 * 50000 * 8
    assert lib.nsb_dendritic_event_workspace_size(0, 10) == 256
    assert lib.nsb_dendritic_event_workspace_size(-1, 10) == 0


def _tick(batch=1, neurons=4, with_params=True):
    tick = native._Tick()
    tick.batch, tick.neurons = batch, neurons
    fake = ctypes.c_void_p(0x1000)  # never dereferenced: validation fails or B == 0 first
    for view in (tick.state, tick.dendrite, tick.adaptation):
        view.data, view.batch_stride, view.neuron_stride = fake.value, neurons, 1
    if with_params:
        for i in range(6):
            tick.params.data[i] = fake.value
            tick.params.stride[i] = 1
    return tick


def _csr(fmt=native.F32, edges=8, scale=None, scales=None):
    return native._Csr(edges, 0x2000, 0x3000, 0x4000, fmt, scales, scale)


def _out():
    o = native._TickOut()
    for view in (o.state, o.dendrite, o.adaptation):
        view.data, view.batch_stride, view.neuron_stride = 0x5000, 4, 1
    return o


def _step(lib, tick, csr, width=32, out=None):
    out = out if out is not None else _out()
    status = lib.nsb_dendritic_step(ctypes.byref(tick), ctypes.byref(csr), width,
                                    ctypes.byref(out), None)
    return status, lib.nsb_last_error().decode()


def test_step_rejects_bad_arguments_before_launch(lib):
    status, message = _step(lib, _tick(with_params=False), _csr())
    assert status == -1 and "parameter" in message
    status, message = _step(lib, _tick(), _csr(), width=7)
    assert status == -1 and "width" in message
    status, message = _step(lib, _tick(), _csr(fmt=9))
    assert status == -1 and "format" in message
    status, message = _step(lib, _tick(), _csr(fmt=native.E4M3))
    assert status == -1 and "global scale" in message
    status, message = _step(lib, _tick(), _csr(fmt=native.NVFP4, scale=0x6000))
    assert status == -1 and "NVFP4" in message
    status, message = _step(lib, _tick(), _csr(fmt=native.F16, scale=0x6000))
    assert status == -1 and "floating-point" in message
    status, message = _step(lib, _tick(neurons=0), _csr())
    assert status == -1 and "N > 0" in message
    bad_out = _out()
    bad_out.dendrite.data = None
    status, message = _step(lib, _tick(), _csr(), out=bad_out)
    assert status == -1 and "dendrite" in message
    status = lib.nsb_dendritic_step(None, None, 32, None, None)
    assert status == -1


def test_empty_batch_is_a_no_op(lib):
    status, message = _step(lib, _tick(batch=0), _csr())
    assert status == 0 and message == ""


def test_event_rejects_small_workspace(lib):
    tick = _tick()
    emitted = native._View(0x7000, 4, 1, 0.0)
    out_csr = native._OutCsr(8, 0x2000, 0x3000, None, 0x4000)
    out = _out()
    out_emitted = native._Out(0x8000, 4, 1)
    status = lib.nsb_dendritic_event(ctypes.byref(tick), 0x9000, ctypes.byref(emitted), 0xA000, 1,
                                     ctypes.byref(out_csr), ctypes.byref(out),
                                     ctypes.byref(out_emitted), 0xB000, 16, None)
    assert status == -3 and "workspace" in lib.nsb_last_error().decode()
    status = lib.nsb_dendritic_event(ctypes.byref(tick), 0x9000, ctypes.byref(emitted), None, 1,
                                     ctypes.byref(out_csr), ctypes.byref(out),
                                     ctypes.byref(out_emitted), 0xB000, 1 << 20, None)
    assert status == -1 and "theta" in lib.nsb_last_error().decode()


def test_empty_batch_needs_no_output_arrays(lib):
    out = native._TickOut()
    status, message = _step(lib, _tick(batch=0), _csr(), out=out)
    assert status == 0 and message == ""


def test_hybrid_event_rejects_bad_arguments(lib):
    """nsb_dendritic_event_hybrid validates like nsb_dendritic_event, then its own
    arguments (B = 1, an N x N float32 layout, a delta buffer, a gate >= 1)."""
    tick = _tick(batch=2, neurons=4)
    status = lib.nsb_dendritic_event_hybrid(ctypes.byref(tick), None, None, None, 0, None, None,
                                            None, 0, None, 1, None, None, None, 0, None, None)
    assert status != 0
    assert b"current" in lib.nsb_last_error() or b"required" in lib.nsb_last_error()


def test_rollout_rejects_bad_ticks_and_strides(lib):
    tick = _tick(batch=1)
    status = lib.nsb_dendritic_rollout_tiled(ctypes.byref(tick), None, 0, 0, None, 0, None,
                                             None, 0, None, None)
    assert status == -1 and b"ticks" in lib.nsb_last_error()
    status = lib.nsb_dendritic_rollout_tiled(ctypes.byref(tick), None, 4, -1, None, 0, None,
                                             None, 0, None, None)
    assert status == -1 and b"drive_tick_stride" in lib.nsb_last_error()
    status = lib.nsb_dendritic_rollout_tiled(ctypes.byref(tick), None, 4, 8, None, 0, None,
                                             None, 0, None, None)
    assert status != 0  # no layout


def test_peer_rollout_rejects_bad_ticks_strides_and_exchanges(lib):
    tick = _tick(batch=1)
    args = (None, None, None, 0, None, None)  # exchange, out, workspace, bytes, status, stream
    assert lib.nsb_dendritic_rollout_tiled_peers(ctypes.byref(tick), None, 0, 0, None, 0,
                                                 *args) == -1
    assert b"ticks" in lib.nsb_last_error()
    assert lib.nsb_dendritic_rollout_tiled_peers(ctypes.byref(tick), None, 3, -2, None, 0,
                                                 *args) == -1
    assert b"drive_tick_stride" in lib.nsb_last_error()
    assert lib.nsb_dendritic_rollout_tiled_peers(ctypes.byref(tick), None, 3, 4, None, 0,
                                                 *args) == -1
    assert b"peer exchange" in lib.nsb_last_error()


def test_cluster_rollout_rejects_bad_ticks_and_strides(lib):
    tick = _tick(batch=1)
    assert lib.nsb_dendritic_rollout_cluster(ctypes.byref(tick), None, 0, 0, 0, None, 0, None,
                                             None, None) == -1
    assert b"ticks" in lib.nsb_last_error()
    assert lib.nsb_dendritic_rollout_cluster(ctypes.byref(tick), None, 0, 5, -1, None, 0, None,
                                             None, None) == -1
    assert b"drive_tick_stride" in lib.nsb_last_error()
