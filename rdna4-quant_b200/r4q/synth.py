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


def qwen3_14b_config(layers: int = 40) -> dict:
    return dict(num_layers=layers, hidden=5120, intermediate=17408, num_heads=40, num_kv_heads=8,
                head_dim=128, vocab=151936, rms_eps=1e-6, rope_theta=1e6)


def build_decode_model(cfg: dict, device, seed: int = 0, int8_frac: float = 0.2,
                       max_seq: int = 2304, batch: int = 1, lm_fp16: bool = True):
    """Random-init weights of a Qwen3-architecture decoder in the reference's
    runtime layout (benchmark config 3): per layer the fused qkv / o / gate_up /
    down projections, ``int8_frac`` of the (layer, projection) groups INT8 and
    the rest INT4 (chosen by ``seed``), fp16 embedding and lm_head, FP8 KV caches
    [batch, Hk, max_seq, head_dim].  Returns the keyword arguments of
    int4_hip.decode_step_logits (minus hidden_in/pos) plus 'embed'."""
    g = torch.Generator(device=device).manual_seed(seed)
    L, D, I = cfg['num_layers'], cfg['hidden'], cfg['intermediate']
    H, Hk, hd = cfg['num_heads'], cfg['num_kv_heads'], cfg['head_dim']
    groups = [(li, p) for li in range(L) for p in ('qkv', 'o', 'gate_up', 'down')]
    pick = torch.randperm(len(groups), generator=torch.Generator().manual_seed(seed))
    int8 = {groups[i] for i in pick[:int(round(int8_frac * len(groups)))].tolist()}
    shapes = {'qkv': ((H + 2 * Hk) * hd, D), 'o': (D, H * hd), 'gate_up': (2 * I, D), 'down': (D, I)}
    out = {k: [] for k in ('qkv_w', 'qkv_s', 'o_w', 'o_s', 'gu_w', 'gu_s', 'down_w', 'down_s',
                           'in_norm_w', 'post_norm_w', 'q_norm_w', 'k_norm_w', 'k_caches', 'v_caches')}
    names = {'qkv': 'qkv', 'o': 'o', 'gate_up': 'gu', 'down': 'down'}
    wbytes = 0
    for li in range(L):
        for p, (N, K) in shapes.items():
            if (li, p) in int8:
                _, w, s = linear_int8(N, K, g, device)
                wbytes += gemv_bytes('int8', 0, N, K)
            else:
                _, w, s = linear_int4(N, K, g, device)
                wbytes += gemv_bytes('int4', 0, N, K)
            out[names[p] + '_w'].append(w)
            out[names[p] + '_s'].append(s)
        for k, n in (('in_norm_w', D), ('post_norm_w', D), ('q_norm_w', hd), ('k_norm_w', hd)):
            out[k].append((1 + 0.01 * torch.randn(n, generator=g, device=device)).half())
        out['k_caches'].append(torch.zeros(batch, Hk, max_seq, hd, dtype=torch.uint8, device=device))
        out['v_caches'].append(torch.zeros(batch, Hk, max_seq, hd, dtype=torch.uint8, device=device))
    V = cfg['vocab']
    out['embed'] = (torch.randn(V, D, generator=g, device=device) * 0.02).half()
    out['final_norm_w'] = (1 + 0.01 * torch.randn(D, generator=g, device=device)).half()
    if lm_fp16:
        out['lm_w'] = (torch.randn(V, D, generator=g, device=device) * 0.02).half()
        out['lm_s'] = None
        wbytes += 2 * V * D
    else:
        _, out['lm_w'], out['lm_s'] = linear_int4(V, D, g, device)
        wbytes += gemv_bytes('int4', 0, V, D)
    inv = 1.0 / (cfg['rope_theta'] ** (torch.arange(0, hd, 2, device=device).float() / hd))
    f = torch.outer(torch.arange(max_seq + 128, device=device).float(), inv)
    out['rope_cos'], out['rope_sin'] = f.cos().half(), f.sin().half()
    out['weight_bytes'] = wbytes
    out['int8_groups'] = len(int8)
    return out


def fill_kv_synthetic(model: dict, ctx: int, seed: int = 0):
    """Stand-in for the prompt's prefill: FP8 K/V of ctx positions from seeded
    N(0,1) values through the reference encoder (fp16_to_fp8)."""
    from . import ops
    g = torch.Generator(device=model['k_caches'][0].device).manual_seed(seed)
    for kc, vc in zip(model['k_caches'], model['v_caches']):
        for c in (kc, vc):
            x = torch.randn(c.shape[0], c.shape[1], ctx, c.shape[3], generator=g, device=c.device).half()
            c[:, :, :ctx] = ops.fp16_to_fp8(x)
