"""Compressed CSR weight formats: E4M3 (fp8) and NVFP4 (E2M1 + block scales).

The encoders produce exactly the bytes of the reference quantizer
(src/neurosim_gpu/precision.py:45-90), which the CUDA tick decodes in-register:

* fp8:   scale = max(amax / 448, tiny);  code = e4m3(clamp(w / scale, +-448))
* nvfp4: g = max(amax / (6 * 448), tiny);
         block scale = e4m3(min(block_amax / (6 * g), 448)) per 16 consecutive
         weights; code = E2M1 magnitude nearest to |w| / (g * block scale),
         exact ties to the even code, sign in bit 3; two codes per byte with the
         even-indexed weight in the low nibble.
* decode: fp8 -> e4m3(code) * scale; nvfp4 -> level(code) * (e4m3(block) * g).

Device weights are encoded by the library's CUDA encoder, host weights by
PyTorch ops, once per ``weight_version`` (the runtime caches the packed
arrays); the per-tick decode is in the kernel.
"""

from __future__ import annotations

import functools
from typing import Literal, cast

import torch

Precision = Literal["fp32", "fp16", "fp8", "nvfp4"]
PRECISIONS = ("fp32", "fp16", "fp8", "nvfp4")
E2M1_LEVELS = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
E2M1_MIDPOINTS = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)
BLOCK = 16


@functools.lru_cache(maxsize=None)
def _levels(device: torch.device, dtype: torch.dtype) -> torch.Tensor:
    """Device-resident E2M1 magnitudes, created once per device (never inside a capture)."""
    with torch.inference_mode(False), torch.no_grad():
        return torch.tensor(E2M1_LEVELS, device=device, dtype=dtype)


def validate_precision(value: str) -> Precision:
    if value not in PRECISIONS:
        raise ValueError("precision must be 'fp32', 'fp16', 'fp8', or 'nvfp4'")
    return cast(Precision, value)


def _tiny() -> float:
    return torch.finfo(torch.float32).tiny


def _true_div(value: torch.Tensor, constant: float) -> torch.Tensor:
    """value / constant with IEEE division on every device.

    PyTorch divides a CUDA tensor by a Python scalar as value * (1 / scalar),
    which can differ from the CPU result by one ulp; a tensor divisor keeps
    the encoding identical on CPU and GPU.
    """
    return value / torch.full_like(value, constant)


def _fp8(value: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    amax = value.abs().amax() if value.numel() else value.new_zeros(())
    scale = _true_div(amax, 448.0).clamp_min(_tiny())
    codes = (value / scale).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return codes, scale


def _nvfp4(value: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """E2M1 codes [..., blocks, 16], E4M3 block scales [..., blocks], FP32 global scale."""
    width = value.shape[-1]
    pad = (-width) % BLOCK
    if pad:
        value = torch.nn.functional.pad(value, (0, pad))
    blocks = value.reshape(*value.shape[:-1], (width + pad) // BLOCK, BLOCK)
    magnitude = blocks.abs()
    block_amax = magnitude.amax(dim=-1, keepdim=True)
    amax = block_amax.amax() if value.numel() else value.new_zeros(())
    global_scale = _true_div(amax, 6.0 * 448.0).clamp_min(_tiny())
    block_scale = (block_amax / (6.0 * global_scale)).clamp_max(448.0).to(torch.float8_e4m3fn)
    denominator = global_scale * block_scale.float()
    normalized = magnitude / torch.where(denominator > 0, denominator, 1.0)
    # code = number of midpoints passed; an exact tie at midpoint i counts as
    # passed only for odd i, which lands it on the even code i + 1.
    code = torch.zeros_like(normalized, dtype=torch.uint8)
    for i, midpoint in enumerate(E2M1_MIDPOINTS):
        code += (normalized >= midpoint) if i % 2 else (normalized > midpoint)
    code |= blocks.signbit().to(torch.uint8) << 3
    return code, block_scale.squeeze(-1), global_scale


def encode_sparse_weights(value: torch.Tensor, precision: str
                          ) -> tuple[torch.Tensor, torch.Tensor | None, torch.Tensor]:
    """Packed CSR weight bytes, optional block-scale bytes and the FP32 global scale.

    Weights in device memory are encoded by the library's CUDA encoder
    (``nsb_encode_weights``, two launches); host weights by the same steps as
    PyTorch ops.  Both give the reference quantizer's bytes.
    """
    if value.ndim != 1 or value.dtype != torch.float32:
        raise ValueError("encoding requires a vector of FP32 CSR weights")
    if precision not in ("fp8", "nvfp4"):
        raise ValueError("compressed CSR encoding requires fp8 or nvfp4")
    if value.is_cuda:
        from .native import load_native_extension

        return load_native_extension().encode_weights(value.detach().contiguous(), precision)
    return encode_sparse_weights_torch(value, precision)


def encode_sparse_weights_torch(value: torch.Tensor, precision: str
                                ) -> tuple[torch.Tensor, torch.Tensor | None, torch.Tensor]:
    """The encoder as PyTorch ops on the weights' device (precision.py:76-90)."""
    if value.ndim != 1 or value.dtype != torch.float32:
        raise ValueError("encoding requires a vector of FP32 CSR weights")
    if precision == "fp8":
        codes, scale = _fp8(value.detach())
        return codes.view(torch.uint8), None, scale.reshape(1)
    if precision != "nvfp4":
        raise ValueError("compressed CSR encoding requires fp8 or nvfp4")
    codes, scales, scale = _nvfp4(value.detach())
    codes = codes.flatten()
    packed = codes[0::2] | (codes[1::2] << 4)
    return (packed[: (value.numel() + 1) // 2].contiguous(), scales.view(torch.uint8),
            scale.reshape(1))


def _straight_through(value: torch.Tensor, quantized: torch.Tensor) -> torch.Tensor:
    if torch.is_grad_enabled() and value.requires_grad:
        return quantized + (value - value.detach())
    return quantized


def quantize_dequantize(value: torch.Tensor, precision: str) -> torch.Tensor:
    """Round-trip through a format (straight-through gradient), as the kernel decodes it."""
    validate_precision(precision)
    if precision == "fp32" or value.numel() == 0:
        return value
    if value.dtype != torch.float32:
        raise ValueError("reduced-precision quantization requires an FP32 master tensor")
    if precision == "fp16":
        return _straight_through(value, value.detach().to(torch.float16).to(value.dtype))
    if precision == "fp8":
        codes, scale = _fp8(value.detach())
        decoded = codes.float() * scale
    else:
        vector = value.detach() if value.ndim else value.detach().reshape(1)
        codes, block_scales, scale = _nvfp4(vector)
        levels = _levels(value.device, value.dtype)
        magnitude = levels[(codes & 7).long()] * (block_scales.float() * scale).unsqueeze(-1)
        decoded = torch.where(codes >= 8, -magnitude, magnitude).flatten(-2)
        decoded = decoded[..., : vector.shape[-1]].reshape(value.shape)
    return _straight_through(value, decoded)


def e4m3_to_float(codes: torch.Tensor) -> torch.Tensor:
    """Exact float32 values of E4M3FN byte codes."""
    return codes.contiguous().view(torch.float8_e4m3fn).float()


def e2m1_to_float(codes: torch.Tensor) -> torch.Tensor:
    """Exact float32 values of 4-bit E2M1 codes (sign in bit 3)."""
    levels = _levels(codes.device, torch.float32)
    magnitude = levels[(codes & 7).long()]
    return torch.where(codes >= 8, -magnitude, magnitude)


def weight_storage_bytes(n_edges: int, precision: str) -> int:
    """Logical packed payload (native_compartmental.py:92-100)."""
    if precision == "nvfp4":
        return (n_edges + 1) // 2 + (n_edges + BLOCK - 1) // BLOCK + 4
    if precision == "fp8":
        return n_edges + 4
    return n_edges * (2 if precision == "fp16" else 4)
