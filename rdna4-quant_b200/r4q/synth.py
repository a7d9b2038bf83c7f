"""Seeded synthetic weights/activations in the reference's quantized format.

The quantizer here follows the reference's RTN quantizers (torch, runs on any
device so the large benchmark configurations are generated on the GPU):
  * INT4 asymmetric: quantize_to_int4_asymmetric (int4_quant_v2.py:17-47),
    nibble packing pack_int4_unsigned (:87-94), runtime interleave of
    (scale, zero) interleave_scale_zero (int4_engine_v5.py:95-102);
  * INT8 symmetric: quantize_to_int8_symmetric (int8_quant.py:14-33);
  * H32 block rotation: rotate_weight (hadamard_utils.py:38-54).
GPTQ needs calibration data that is not available, so RTN stands in for it.
This is data generation for tests and benchmarks, not part of the decode path.
"""
from __future__ import annotations

import math

import torch


def hadamard32(device, dtype=torch.float32) -> torch.Tensor:
    H = torch.ones(1, 1, dtype=torch.float64)
    while H.shape[0] < 32:
        H = torch.cat([torch.cat([H, H], 1), torch.cat([H, -H], 1)], 0)
    return (H / math.sqrt(32)).to(device=device, dtype=dtype)


def rotate_blocks(W: torch.Tensor) -> torch.Tensor:
    N, K = W.shape
    H = hadamard32(W.device, W.dtype)
    return (W.reshape(N, K // 32, 32) @ H).reshape(N, K)


def quantize_int4_asym(W: torch.Tensor):
    """W float32 [N, K] -> (packed u8 [N, K/2], sz fp16 [N, K/16])."""
    N, K = W.shape
    b = W.reshape(N, K // 32, 32).float()
    vmin = b.amin(-1, keepdim=True)
    vmax = b.amax(-1, keepdim=True)
    scale = (vmax - vmin) / 15.0
    scale = torch.where(scale > 0, scale, torch.ones_like(scale)).clamp(max=65504.0)
    zp = (-vmin / scale).round().clamp(0, 15)
    q = ((b / scale) + zp).round().clamp(0, 15).to(torch.uint8).reshape(N, K)
    packed = (q[:, 0::2] & 0x0F) | ((q[:, 1::2] & 0x0F) << 4)
    sz = torch.stack([scale.squeeze(-1).half(), zp.squeeze(-1).half()], -1).reshape(N, K // 16)
    return packed.contiguous(), sz.contiguous()


def quantize_int8_sym(W: torch.Tensor):
    """W float32 [N, K] -> (int8 [N, K], fp16 scales [N, K/32])."""
    N, K = W.shape
    b = W.reshape(N, K // 32, 32).float()
    scale = b.abs().amax(-1, keepdim=True) / 127.0
    scale = torch.where(scale > 0, scale, torch.ones_like(scale)).clamp(max=65504.0)
    q = (b / scale).round().clamp(-128, 127).to(torch.int8).reshape(N, K)
    return q.contiguous(), scale.squeeze(-1).half().contiguous()


def weight_fp32(N: int, K: int, gen: torch.Generator, device, std=0.02, outlier_frac=1e-3,
                outlier_mul=20.0, rotate=True) -> torch.Tensor:
    """N(0, std) with a seeded fraction of entries scaled by outlier_mul, then
    H32-rotated — the config-0 weight recipe."""
    W = torch.randn(N, K, generator=gen, device=device, dtype=torch.float32) * std
    if outlier_frac > 0:
        m = torch.rand(N, K, generator=gen, device=device) < outlier_frac
        W = torch.where(m, W * outlier_mul, W)
    return rotate_blocks(W) if rotate else W


def linear_int4(N, K, gen, device):
    return ('int4',) + quantize_int4_asym(weight_fp32(N, K, gen, device))


def linear_int8(N, K, gen, device):
    return ('int8',) + quantize_int8_sym(weight_fp32(N, K, gen, device))


def gemv_bytes(fmt: str, B: int, N: int, K: int) -> int:
    """Algorithmic HBM bytes of one GEMV: weights + disk-format block metadata
    (INT4: fp16 scale + u8 zero = 3 B per 32-block; INT8: fp16 scale) + the
    activation read and the output write."""
    act = 2 * B * K + 2 * B * N
    if fmt == 'int4':
        return N * K // 2 + 3 * N * K // 32 + act
    if fmt == 'int8':
        return N * K + 2 * N * K // 32 + act
    return 2 * N * K + act
