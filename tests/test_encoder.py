"""The CUDA weight encoder (nsb_encode_weights) against the reference's bytes.

Pinned to the fixtures written by the reference's own encode_sparse_weights
(tests/golden/precision.npz), then to the oracle encoder (oracle/tick.py, itself
pinned to those fixtures) on random, sign-of-zero, subnormal-range and exact
midpoint-tie inputs, and to the PyTorch-op encoder on the same device.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from _util import GOLDEN
from neurosim_gpu_b200 import load_native_extension, native
from neurosim_gpu_b200.precision import (E2M1_MIDPOINTS, encode_sparse_weights,
                                         encode_sparse_weights_torch)


def test_encoder_rejects_bad_arguments_cpu():
    lib = native.load_library()
    assert lib.nsb_encode_weights(native.F32, None, 0, None, None, None, None, None) != 0
    assert b"E4M3" in lib.nsb_last_error()
    assert lib.nsb_encode_weights(native.NVFP4, None, -1, None, None, None, None, None) != 0
    assert lib.nsb_encode_weights(native.NVFP4, 0x1000, 32, 0x2000, None, 0x3000, 0x4000,
                                  None) != 0  # no block-scale buffer
    assert b"block-scale" in lib.nsb_last_error()


def _check(value: np.ndarray, fmt: str, want=None):
    ext = load_native_extension()
    device_value = torch.from_numpy(value.astype(np.float32)).cuda()
    codes, scales, scale = ext.encode_weights(device_value, fmt)
    if want is None:
        want = oracle.encode_sparse_weights(value, fmt)
    w_codes, w_scales, w_scale = want
    assert np.array_equal(codes.cpu().numpy(), np.asarray(w_codes, np.uint8)), fmt
    assert np.array_equal(scale.cpu().numpy().view(np.uint32),
                          np.asarray(w_scale, np.float32).reshape(-1).view(np.uint32)), fmt
    if fmt == "nvfp4":
        assert np.array_equal(scales.cpu().numpy(), np.asarray(w_scales, np.uint8)), fmt
    else:
        assert scales is None
    # The PyTorch-op encoder on the same device gives the same bytes.
    t_codes, t_scales, t_scale = encode_sparse_weights_torch(device_value, fmt)
    assert torch.equal(t_codes.view(torch.uint8).cpu(), codes.cpu())
    assert torch.equal(t_scale.cpu(), scale.cpu())
    if fmt == "nvfp4":
        assert torch.equal(t_scales.view(torch.uint8).cpu(), scales.cpu())


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["fp8", "nvfp4"])
def test_encoder_matches_the_reference_fixtures(fmt):
    golden = np.load(GOLDEN / "precision.npz")
    names = sorted({k[: -len("_value")] for k in golden if k.endswith("_value")})
    assert "config0" in names
    for name in names:
        value = golden[f"{name}_value"]
        want = (golden[f"{name}_{fmt}_codes"],
                golden[f"{name}_{fmt}_scales"] if fmt == "nvfp4" else None,
                golden[f"{name}_{fmt}_scale"])
        _check(value, fmt, want)


@pytest.mark.gpu
def test_encoder_config0_pinned_values():
    """Config 0's graph: fp8 scale 4.06163e-4; nvfp4 9,902 code and 1,238 scale
    bytes, global 6.76938e-5 (values the reference prints for this graph)."""
    from neurosim_gpu_b200 import random_topology
    graph = random_topology(1000, 20000, device="cpu", seed=0)
    weight = graph.in_weight.cuda()
    _, _, scale = encode_sparse_weights(weight, "fp8")
    assert abs(float(scale) - 4.06163e-4) < 1e-9
    codes, scales, scale = encode_sparse_weights(weight, "nvfp4")
    assert codes.numel() == 9902 and scales.numel() == 1238
    assert abs(float(scale) - 6.76938e-5) < 1e-10


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["fp8", "nvfp4"])
@pytest.mark.parametrize("n", [0, 1, 2, 15, 16, 17, 31, 33, 1000, 100003, 1 << 20])
def test_encoder_random_sizes_match_the_oracle(fmt, n):
    rng = np.random.default_rng(n)
    value = (rng.standard_normal(n) * 0.05).astype(np.float32)
    if n > 8:
        value[::7] = 0.0
        value[3::11] = -0.0
        value[5::13] *= 1e-6      # far below the block scale: subnormal codes / zero codes
        value[1::17] *= 50.0      # a wide dynamic range inside blocks
    _check(value, fmt)


@pytest.mark.gpu
def test_encoder_exact_midpoint_ties_and_signs():
    """Global amax 2688 makes g = 1 exactly and a block amax of 6 * 2^j makes its
    scale 2^j, so |w| = midpoint * 2^j hits each E2M1 midpoint exactly."""
    blocks = [np.array([2688.0] + [0.0] * 15, np.float32)]
    for j in range(-6, 7):
        unit = np.float32(2.0 ** j)
        mids = np.array(E2M1_MIDPOINTS, np.float32) * unit
        block = np.concatenate([[6.0 * unit], mids, -mids, [-0.0]]).astype(np.float32)
        assert block.size == 16
        blocks.append(block)
    value = np.concatenate(blocks)
    _check(value, "nvfp4")
    _check(value / np.float32(7.0), "fp8")
    # The tie rule itself: midpoint i lands on code i + 1 for odd i, code i for even i.
    codes, _, _ = load_native_extension().encode_weights(torch.from_numpy(value).cuda(), "nvfp4")
    nib = np.empty(codes.numel() * 2, np.uint8)
    raw = codes.cpu().numpy()
    nib[0::2], nib[1::2] = raw & 15, raw >> 4
    block = nib[16:32]
    assert list(block[1:8]) == [0, 2, 2, 4, 4, 6, 6]
    assert list(block[8:15]) == [8 | c for c in (0, 2, 2, 4, 4, 6, 6)]
    assert block[15] == 8  # -0.0 keeps its sign bit


@pytest.mark.gpu
def test_runtime_uses_the_device_encoder_for_packed_weights():
    from _util import make
    from neurosim_gpu_b200 import NativeDendriticMatrixRuntime
    graph, model, state = make(500, 1, 9000)
    rt = NativeDendriticMatrixRuntime(graph, model, state, precision="nvfp4")
    codes, scales, scale, _ = rt._weights()
    want = oracle.encode_sparse_weights(graph.in_weight.cpu().numpy(), "nvfp4")
    assert np.array_equal(codes.cpu().numpy(), want[0])
    assert np.array_equal(scales.cpu().numpy(), want[1])
