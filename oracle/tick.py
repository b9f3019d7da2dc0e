"""CPU oracle for the dendritic tick -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module, and only as the checker or as the timed CPU
baseline.  The product package never imports it.

What it restates (paths relative to the reference project):

* ``oracle.c`` (loaded here through ctypes): the three-state tick of
  ``src/neurosim_gpu/compartmental.py:152-183`` / ``dynamics.py:41-61``, the
  CSR product of ``runtime.py:78-79`` and the PELS emit rule of
  ``runtime.py:225-253`` with the native ``emitted <- s_new`` assignment of
  ``csrc/compartmental.cu:156``.
* the numpy functions below: the weight quantizers of
  ``src/neurosim_gpu/precision.py:45-112`` (E4M3 per-tensor scale; NVFP4 =
  E2M1 codes in 16-element blocks with E4M3 block scales and an FP32 global
  scale, two codes per byte, low nibble first).

Parity is pinned by ``tests/golden/`` (fixtures generated from the reference
by ``tests/golden/make_golden.py``) and checked in ``tests/test_oracle_golden.py``.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "liboracle.so"
_SOURCE = _HERE / "oracle.c"

# precision.py:13-14 -- the E2M1 magnitudes and the midpoints between them.
E2M1_LEVELS = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)
E2M1_MIDPOINTS = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=np.float32)
_TINY = np.float32(np.finfo(np.float32).tiny)


def build_oracle(force: bool = False) -> Path:
    """Compile ``oracle.c`` into ``liboracle.so`` next to it (gcc, OpenMP)."""
    if force or not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < _SOURCE.stat().st_mtime:
        cmd = ["gcc", "-O2", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", "-fPIC",
               "-shared", str(_SOURCE), "-o", str(_LIB_PATH) + ".tmp", "-lm"]
        subprocess.run(cmd, check=True)
        os.replace(str(_LIB_PATH) + ".tmp", _LIB_PATH)
    return _LIB_PATH


_lib = None


def _load():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(str(build_oracle()))
        i64, i32p, f32p, u8p, c_int = (ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_void_p, ctypes.c_int)
        lib.orc_spmv.argtypes = [i64, i64, i32p, i32p, f32p, f32p, f32p, c_int]
        lib.orc_matrix_tick.argtypes = [i64, i64, i32p, i32p, f32p] + [f32p] * 6 + [f32p] * 3 + [c_int]
        lib.orc_advance.argtypes = [i64, i64] + [f32p] * 7 + [f32p] * 3 + [c_int]
        lib.orc_event_tick.argtypes = ([i64, i64, i32p, i32p, f32p] + [f32p] * 6
                                       + [f32p, f32p, f32p] + [f32p] * 4 + [u8p, c_int])
        lib.orc_max_threads.restype = c_int
        _lib = lib
    return _lib


def max_threads() -> int:
    return int(_load().orc_max_threads())


def _ptr(array: np.ndarray) -> int:
    return array.ctypes.data


def _f32(value, shape=None) -> np.ndarray:
    array = np.ascontiguousarray(np.asarray(value, dtype=np.float32))
    if shape is not None and array.shape != tuple(shape):
        array = np.ascontiguousarray(np.broadcast_to(array, shape))
    return array


@dataclass
class CSR:
    """Destination-major CSR W[dst, src] (the reference's in_rowptr / in_col / in_weight)."""

    n: int
    rowptr: np.ndarray
    col: np.ndarray
    weight: np.ndarray

    @classmethod
    def make(cls, n: int, rowptr, col, weight) -> "CSR":
        for name, value in (("rowptr", rowptr), ("col", col)):
            if not np.issubdtype(np.asarray(value).dtype, np.integer):
                raise TypeError(f"{name} must be an integer array (float32 cannot hold >2^24 offsets)")
        rowptr = np.ascontiguousarray(np.asarray(rowptr, dtype=np.int32))
        col = np.ascontiguousarray(np.asarray(col, dtype=np.int32))
        weight = _f32(weight)
        if rowptr.shape != (n + 1,) or col.shape != weight.shape:
            raise ValueError("invalid CSR geometry")
        return cls(n, rowptr, col, weight)

    def with_weight(self, weight) -> "CSR":
        return CSR.make(self.n, self.rowptr, self.col, weight)


def _params(params) -> np.ndarray:
    return _f32(np.stack([np.asarray(p, dtype=np.float32) for p in params]))


def spmv(csr: CSR, x, threads: int = 0) -> np.ndarray:
    x = _f32(x)
    batch = x.shape[0]
    y = np.empty((batch, csr.n), dtype=np.float32)
    if x.size:
        _load().orc_spmv(batch, csr.n, _ptr(csr.rowptr), _ptr(csr.col), _ptr(csr.weight),
                         _ptr(x), _ptr(y), threads)
    return y


def matrix_tick(csr: CSR, s, d, a, params, drive=0.0, dendritic_drive=0.0,
                threads: int = 0):
    """One DendriticMatrixRuntime.step: returns (s', d', a') as new arrays."""
    s = _f32(s)
    shape = s.shape
    d, a = _f32(d, shape), _f32(a, shape)
    u, v = _f32(drive, shape), _f32(dendritic_drive, shape)
    p = _params(params)
    out = np.empty((3,) + shape, dtype=np.float32)
    if s.size:
        _load().orc_matrix_tick(shape[0], csr.n, _ptr(csr.rowptr), _ptr(csr.col),
                                _ptr(csr.weight), _ptr(s), _ptr(d), _ptr(a), _ptr(u), _ptr(v),
                                _ptr(p), _ptr(out[0]), _ptr(out[1]), _ptr(out[2]), threads)
    return out[0], out[1], out[2]


def advance(j, s, d, a, params, drive=0.0, dendritic_drive=0.0, threads: int = 0):
    s = _f32(s)
    shape = s.shape
    j, d, a = _f32(j, shape), _f32(d, shape), _f32(a, shape)
    u, v = _f32(drive, shape), _f32(dendritic_drive, shape)
    p = _params(params)
    out = np.empty((3,) + shape, dtype=np.float32)
    if s.size:
        _load().orc_advance(shape[0], shape[1], _ptr(j), _ptr(s), _ptr(d), _ptr(a), _ptr(u),
                            _ptr(v), _ptr(p), _ptr(out[0]), _ptr(out[1]), _ptr(out[2]), threads)
    return out[0], out[1], out[2]


def event_tick(csr: CSR, s, d, a, params, current, emitted, theta, drive=0.0,
               dendritic_drive=0.0, threads: int = 0):
    """One native PELS tick.  Returns (s', d', a', emitted', current', active)."""
    s = _f32(s)
    shape = s.shape
    d, a = _f32(d, shape), _f32(a, shape)
    u, v = _f32(drive, shape), _f32(dendritic_drive, shape)
    current = _f32(current, shape).copy()
    emitted = _f32(emitted, shape)
    theta = _f32(theta, (csr.n,))
    p = _params(params)
    out = np.empty((4,) + shape, dtype=np.float32)
    active = np.zeros(shape, dtype=np.uint8)
    if s.size:
        _load().orc_event_tick(shape[0], csr.n, _ptr(csr.rowptr), _ptr(csr.col),
                               _ptr(csr.weight), _ptr(s), _ptr(d), _ptr(a), _ptr(u), _ptr(v),
                               _ptr(p), _ptr(current), _ptr(emitted), _ptr(theta),
                               _ptr(out[0]), _ptr(out[1]), _ptr(out[2]), _ptr(out[3]),
                               _ptr(active), threads)
    return out[0], out[1], out[2], out[3], current, active.astype(bool)


# ----------------------------------------------------------------------------
# Weight formats (precision.py:45-112), restated in numpy.
# ----------------------------------------------------------------------------

def e4m3_encode(value) -> np.ndarray:
    """Round float32 values (|x| <= 448, finite) to OCP E4M3FN bytes, ties to even."""
    x = np.asarray(value, dtype=np.float32)
    sign = (np.signbit(x).astype(np.uint16) << 7)
    ax = np.abs(x).astype(np.float64)
    mantissa, exponent = np.frexp(ax)              # ax = mantissa * 2**exponent, mantissa in [0.5, 1)
    e = exponent.astype(np.int64) - 1              # ax = (2*mantissa) * 2**e
    q = np.rint((2.0 * mantissa - 1.0) * 8.0)     # three mantissa bits, round half to even
    carry = q >= 8.0
    e = np.where(carry, e + 1, e)
    q = np.where(carry, 0.0, q)
    normal = ((e + 7) << 3) | q.astype(np.int64)
    subnormal = np.rint(ax * 512.0).astype(np.int64)  # units of 2**-9; 8 rolls into 2**-6
    code = np.where(ax < 2.0 ** -6, subnormal, normal)
    return (code.astype(np.uint16) | sign).astype(np.uint8)


def e4m3_decode(codes) -> np.ndarray:
    c = np.asarray(codes, dtype=np.uint8).astype(np.int64)
    sign = np.where(c & 0x80, -1.0, 1.0)
    e = (c >> 3) & 15
    m = c & 7
    value = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.exp2(e - 7.0))
    value = np.where((e == 15) & (m == 7), np.nan, value)
    return (sign * value).astype(np.float32)


def encode_fp8(weight):
    """precision.py:45-49: per-tensor scale = max(amax/448, tiny); codes = e4m3(w/scale)."""
    w = _f32(weight)
    amax = np.abs(w).max() if w.size else np.float32(0)
    scale = max(np.float32(amax) / np.float32(448.0), _TINY)
    scale = np.float32(scale)
    codes = e4m3_encode(np.clip(w / scale, np.float32(-448.0), np.float32(448.0)))
    return codes, None, np.array([scale], dtype=np.float32)


def encode_nvfp4(weight):
    """precision.py:52-90: E2M1 codes in 16-wide blocks, E4M3 block scales, FP32 global."""
    w = _f32(weight)
    width = w.size
    pad = (-width) % 16
    blocks = np.pad(w, (0, pad)).reshape(-1, 16)
    abs_blocks = np.abs(blocks)
    block_amax = abs_blocks.max(axis=1) if blocks.size else np.zeros(0, np.float32)
    amax = block_amax.max() if block_amax.size else np.float32(0)
    global_scale = np.float32(max(np.float32(amax) / np.float32(6.0 * 448.0), _TINY))
    six_global = np.float32(np.float32(6.0) * global_scale)
    block_scale = e4m3_encode(np.minimum(block_amax / six_global, np.float32(448.0)))
    denominator = (global_scale * e4m3_decode(block_scale)).astype(np.float32)
    safe = np.where(denominator > 0, denominator, np.float32(1.0)).astype(np.float32)
    normalized = (abs_blocks / safe[:, None]).astype(np.float32)
    nearest = np.searchsorted(E2M1_MIDPOINTS, normalized, side="left")
    tie = (nearest % 2 == 1) & (normalized == E2M1_MIDPOINTS[np.minimum(nearest, 6)])
    code = (nearest + tie).astype(np.uint8) | (np.signbit(blocks).astype(np.uint8) << 3)
    code = code.reshape(-1)
    packed = (code[0::2] | (code[1::2] << 4)).astype(np.uint8)
    return packed[: (width + 1) // 2].copy(), block_scale, np.array([global_scale], np.float32)


def decode_fp8(codes, scale) -> np.ndarray:
    return (e4m3_decode(codes) * np.float32(np.asarray(scale).reshape(-1)[0])).astype(np.float32)


def decode_nvfp4(packed, block_scales, global_scale, count: int) -> np.ndarray:
    packed = np.asarray(packed, dtype=np.uint8)
    codes = np.empty(packed.size * 2, dtype=np.uint8)
    codes[0::2] = packed & 15
    codes[1::2] = packed >> 4
    codes = codes[:count]
    block = (e4m3_decode(block_scales) * np.float32(np.asarray(global_scale).reshape(-1)[0]))
    block = block.astype(np.float32)
    magnitude = (E2M1_LEVELS[codes & 7] * block[np.arange(count) // 16]).astype(np.float32)
    return np.where(codes >= 8, -magnitude, magnitude).astype(np.float32)


def quantize_dequantize(weight, precision: str) -> np.ndarray:
    """precision.py:93-112 for a 1-D FP32 vector (no gradient)."""
    w = _f32(weight)
    if precision == "fp32" or w.size == 0:
        return w.copy()
    if precision == "fp16":
        return w.astype(np.float16).astype(np.float32)
    if precision == "fp8":
        codes, _, scale = encode_fp8(w)
        return decode_fp8(codes, scale)
    if precision == "nvfp4":
        packed, scales, scale = encode_nvfp4(w)
        return decode_nvfp4(packed, scales, scale, w.size)
    raise ValueError("precision must be 'fp32', 'fp16', 'fp8', or 'nvfp4'")


def encode_sparse_weights(weight, precision: str):
    if precision == "fp8":
        return encode_fp8(weight)
    if precision == "nvfp4":
        return encode_nvfp4(weight)
    raise ValueError("compressed CSR encoding requires fp8 or nvfp4")
