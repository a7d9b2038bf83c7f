"""CPU oracle for the rdna4-quant decode hot path — TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it.
The product path (``rdna4-quant_b200/``) never imports it and fails loudly when
its CUDA library is missing.

It restates, in numpy, the arithmetic of the reference's decode path
(JohnTDI-cpu/rdna4-quant).  Every function cites the reference file:line whose
behaviour it follows.  Pinning:

* quantizer / pack / dequant / Hadamard / RMSNorm / RoPE tables are pinned
  bit-exactly (or to 1e-12 in fp64) against golden vectors produced by
  importing the reference's own Python modules (``tests/golden/make_golden.py``);
* the HIP-only numerics (FP8 E4M3 codec, the butterfly FWHT order, the fused
  residual/norm rounding points, head-norm+RoPE+KV write, split-K LSE merge)
  have no runnable reference here (HIP cannot be compiled); they are pinned by
  known-answer values read off the reference source and by cross-checks against
  the reference's Python equivalents (e.g. FWHT == x @ get_hadamard(32)).
"""
from __future__ import annotations

import math

import numpy as np

BLOCK = 32
INV_SQRT32 = np.float32(0.17677669529663689)  # int4_decode_step.hip:101


# --------------------------------------------------------------------------
# INT4 asymmetric quantizer / packing / dequant  (int4_quant_v2.py)
# --------------------------------------------------------------------------
def quantize_int4_asym(blocks: np.ndarray):
    """Restates ``quantize_to_int4_asymmetric`` (int4_quant_v2.py:17-47).

    blocks: float32 [..., 32].  Returns (q uint8 [...,32] in 0..15,
    scale float16 [...], zero uint8 [...]).  All arithmetic in float32 with
    round-half-to-even (torch.round semantics), as the reference does.
    """
    b = np.asarray(blocks, dtype=np.float32)
    vmin = b.min(axis=-1, keepdims=True)
    vmax = b.max(axis=-1, keepdims=True)
    scale = (vmax - vmin) / np.float32(15.0)
    scale = np.where(scale > 0, scale, np.float32(1.0)).astype(np.float32)
    scale = np.minimum(scale, np.float32(65504.0))
    zp = np.clip(np.round(-vmin / scale), 0, 15).astype(np.float32)
    q = np.clip(np.round(b / scale + zp), 0, 15).astype(np.uint8)
    return q, scale[..., 0].astype(np.float16), zp[..., 0].astype(np.uint8)


def pack_int4(q: np.ndarray) -> np.ndarray:
    """``pack_int4_unsigned`` (int4_quant_v2.py:87-94): byte = even | odd << 4."""
    q = np.asarray(q, dtype=np.uint8)
    return ((q[..., 0::2] & 0x0F) | ((q[..., 1::2] & 0x0F) << 4)).astype(np.uint8)


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    """``unpack_int4_unsigned`` (int4_quant_v2.py:97-102)."""
    p = np.asarray(packed, dtype=np.uint8)
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), dtype=np.uint8)
    out[..., 0::2] = p & 0x0F
    out[..., 1::2] = p >> 4
    return out


def dequant_int4(packed: np.ndarray, scale: np.ndarray, zero: np.ndarray) -> np.ndarray:
    """``dequantize_int4_asym`` (int4_quant_v2.py:105-127) and the device twin
    ``dequant_int4_kernel`` (int4_decode_step.hip:3568-3588):
    W = fp16((q - z) * s) with (q - z) * s evaluated in float32."""
    q = unpack_int4(packed).astype(np.float32)
    N, K = q.shape
    qb = q.reshape(N, K // BLOCK, BLOCK)
    s = np.asarray(scale, dtype=np.float16).astype(np.float32)[..., None]
    z = np.asarray(zero).astype(np.float32)[..., None]
    return ((qb - z) * s).reshape(N, K).astype(np.float16)


def interleave_scale_zero(scale: np.ndarray, zero: np.ndarray) -> np.ndarray:
    """``interleave_scale_zero`` (int4_engine_v5.py:95-102): fp16 [N, K/16]
    holding (scale, float(zero)) pairs per 32-block."""
    s = np.asarray(scale, dtype=np.float16)
    z = np.asarray(zero).astype(np.float32).astype(np.float16)
    return np.stack([s, z], axis=-1).reshape(s.shape[0], -1)


def split_scale_zero(sz: np.ndarray):
    """Inverse of :func:`interleave_scale_zero` (runtime layout -> disk layout)."""
    sz = np.asarray(sz, dtype=np.float16)
    N = sz.shape[0]
    pairs = sz.reshape(N, -1, 2)
    return pairs[..., 0].copy(), pairs[..., 1].astype(np.float32).astype(np.uint8)


def dequant_int4_runtime(packed: np.ndarray, sz: np.ndarray) -> np.ndarray:
    """``int4_hip.dequant_int4`` semantics on the runtime layout
    (int4_decode_step.hip:3568-3603): zero read back as fp16."""
    q = unpack_int4(packed).astype(np.float32)
    N, K = q.shape
    pairs = np.asarray(sz, dtype=np.float16).reshape(N, K // BLOCK, 2).astype(np.float32)
    qb = q.reshape(N, K // BLOCK, BLOCK)
    return ((qb - pairs[..., 1:2]) * pairs[..., 0:1]).reshape(N, K).astype(np.float16)


def dequant_int4_torch(packed, scale_fp16, zero_point, block_size: int = BLOCK):
    """``dequantize_int4_asym`` (int4_quant_v2.py:105-127) restated with the
    same torch operations in the same order — unpack (low nibble = even k,
    int4_quant_v2.py:97-102), float, (q - z) * s per block, cast to fp16 — so
    that the CPU baseline runs the reference's own PyTorch arithmetic.
    packed uint8 [N, K/2], scale fp16 [N, K/32], zero uint8 [N, K/32] (torch
    tensors); returns fp16 [N, K]."""
    import torch
    N = packed.shape[0]
    K = packed.shape[1] * 2
    lo = packed & 0x0F
    hi = (packed >> 4) & 0x0F
    q = torch.stack([lo, hi], dim=-1).reshape(N, K)
    qb = q.reshape(N, K // block_size, block_size).float()
    return ((qb - zero_point.float().unsqueeze(-1)) * scale_fp16.float().unsqueeze(-1)).reshape(N, K).half()


def quantize_int4_sym(blocks: np.ndarray):
    """``quantize_to_int4_symmetric`` (int4_quant_v2.py:131-139): int8 in -8..7."""
    b = np.asarray(blocks, dtype=np.float32)
    max_abs = np.abs(b).max(axis=-1, keepdims=True)
    scale = max_abs / np.float32(7.0)
    scale = np.where(scale > 0, scale, np.float32(1.0)).astype(np.float32)
    scale = np.minimum(scale, np.float32(65504.0))
    q = np.clip(np.round(b / scale), -8, 7).astype(np.int8)
    return q, scale[..., 0].astype(np.float16)


def pack_int4_signed(q: np.ndarray) -> np.ndarray:
    """``pack_int4`` (int4_quant_v2.py:157-161): two's-complement nibbles."""
    u = np.asarray(q, dtype=np.int8).view(np.uint8)
    return ((u[..., 0::2] & 0x0F) | ((u[..., 1::2] & 0x0F) << 4)).astype(np.uint8)


def convert_symmetric_to_asymmetric(packed: np.ndarray, scale: np.ndarray):
    """``convert_symmetric_to_asymmetric`` (int4_engine_v5.py:105-118):
    nibble n -> (n + 8) & 0xF, zero point 8; returns (packed, sz runtime)."""
    p = np.asarray(packed, dtype=np.uint8)
    lo = ((p & 0x0F) + 8) & 0x0F
    hi = ((p >> 4) + 8) & 0x0F
    newp = (lo | (hi << 4)).astype(np.uint8)
    zeros = np.full(np.asarray(scale).shape, 8, dtype=np.uint8)
    return newp, interleave_scale_zero(scale, zeros)


# --------------------------------------------------------------------------
# INT8 symmetric  (int8_quant.py)
# --------------------------------------------------------------------------
def quantize_int8_sym(blocks: np.ndarray):
    """``quantize_to_int8_symmetric`` (int8_quant.py:14-33)."""
    b = np.asarray(blocks, dtype=np.float32)
    max_abs = np.abs(b).max(axis=-1, keepdims=True)
    scale = max_abs / np.float32(127.0)
    scale = np.where(scale > 0, scale, np.float32(1.0)).astype(np.float32)
    scale = np.minimum(scale, np.float32(65504.0))
    q = np.clip(np.round(b / scale), -128, 127).astype(np.int8)
    return q, scale[..., 0].astype(np.float16)


def dequant_int8(w: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """``dequantize_int8`` (int8_quant.py:52-69): fp16(q * s) in float32."""
    q = np.asarray(w, dtype=np.int8).astype(np.float32)
    N, K = q.shape
    s = np.asarray(scale, dtype=np.float16).astype(np.float32)[..., None]
    return (q.reshape(N, K // BLOCK, BLOCK) * s).reshape(N, K).astype(np.float16)


# --------------------------------------------------------------------------
# Hadamard  (hadamard_utils.py, int4_decode_step.hip:87-102)
# --------------------------------------------------------------------------
def hadamard_matrix(n: int = 32) -> np.ndarray:
    """Normalised Sylvester matrix, ``get_hadamard`` (hadamard_utils.py:14-35)."""
    H = np.array([[1.0]])
    while H.shape[0] < n:
        H = np.block([[H, H], [H, -H]])
    return H / math.sqrt(n)


def fwht32(x: np.ndarray) -> np.ndarray:
    """Butterfly FWHT on every 32-element block of the last axis, float32,
    stage order 1,2,4,8,16 then * 1/sqrt(32) — ``fwht_inplace_32``
    (int4_decode_step.hip:87-102) and the shuffle form (e.g. :1044-1049)."""
    v = np.array(x, dtype=np.float32, copy=True)
    shp = v.shape
    v = v.reshape(-1, BLOCK)
    step = 1
    while step < BLOCK:
        idx = np.arange(BLOCK)
        lo = idx[(idx & step) == 0]
        a = v[:, lo].copy()
        b = v[:, lo + step].copy()
        v[:, lo] = a + b
        v[:, lo + step] = a - b
        step *= 2
    v *= INV_SQRT32
    return v.reshape(shp)


def rotate_blocks(x: np.ndarray) -> np.ndarray:
    """``rotate_weight`` / ``rotate_activation`` (hadamard_utils.py:38-88):
    x @ block_diag(H32, ...) in float64."""
    x = np.asarray(x, dtype=np.float64)
    H = hadamard_matrix(BLOCK)
    shp = x.shape
    return (x.reshape(-1, BLOCK) @ H).reshape(shp)


# --------------------------------------------------------------------------
# FP8 E4M3 codec of the reference (int4_decode_step.hip:47-81)
# --------------------------------------------------------------------------
def fp8_encode(x: np.ndarray) -> np.ndarray:
    """``f32_to_fp8e4m3`` (int4_decode_step.hip:47-68): clamp to +-448,
    flush |x| < 2^-6 to signed zero, round on the first dropped mantissa bit
    (ties away from zero), saturate the top binade to 0x7E."""
    v = np.asarray(x, dtype=np.float32)
    v = np.minimum(np.float32(448.0), v)          # fminf(448, v); NaN -> 448
    v = np.where(np.isnan(v), np.float32(448.0), v)
    v = np.maximum(np.float32(-448.0), v)
    f = v.view(np.uint32).astype(np.uint64)
    sign = ((f >> 24) & 0x80).astype(np.uint8)
    exp32 = ((f >> 23) & 0xFF).astype(np.int64)
    mant32 = (f & 0x7FFFFF).astype(np.int64)
    exp = exp32 - 127 + 7
    mant = mant32 >> 20
    rnd = (mant32 & 0x80000) != 0
    mant = mant + rnd
    carry = mant > 7
    mant = np.where(carry, 0, mant)
    exp = exp + carry
    out = (sign.astype(np.int64) | (exp << 3) | mant)
    out = np.where(exp >= 15, sign.astype(np.int64) | 0x7E, out)
    out = np.where(exp <= 0, sign, out)
    out = np.where(exp32 == 0, sign, out)
    return out.astype(np.uint8)


def fp8_decode(b: np.ndarray) -> np.ndarray:
    """``fp8e4m3_to_f32`` (int4_decode_step.hip:71-81): bit composition
    sign | (exp + 120) << 23 | mant << 20; bytes with zero magnitude -> +0.0."""
    u = np.asarray(b, dtype=np.uint8).astype(np.uint32)
    f = ((u & 0x80) << 24) | ((((u >> 3) & 0xF) + 120) << 23) | ((u & 0x7) << 20)
    out = f.astype(np.uint32).view(np.float32)
    return np.where((u & 0x7F) != 0, out, np.float32(0.0)).astype(np.float32)


def fp8_encodable_bytes() -> np.ndarray:
    """Bytes the reference encoder can emit: 0x00/0x80, every byte with an
    exponent field in 1..14, and 0x7E/0xFE (the whole top binade saturates)."""
    allb = np.arange(256, dtype=np.uint8)
    e = (allb >> 3) & 0xF
    ok = ((allb & 0x7F) == 0) | ((e >= 1) & (e <= 14)) | ((allb & 0x7F) == 0x7E)
    return allb[ok]


# --------------------------------------------------------------------------
# GEMV  (int4_decode_step.hip:116-170; int4_quant_v2.py:105-127)
# --------------------------------------------------------------------------
def gemv_int4(x: np.ndarray, packed: np.ndarray, sz: np.ndarray, acc: bool = False) -> np.ndarray:
    """Y[b, n] = fp16(sum_k fp16(W_deq)[n, k] * x[b, k]) with W_deq from the
    reference dequant (int4_quant_v2.py:105-127) — the reference test's
    ``x @ dequantize_int4_asym(...).T`` (tests/test_kernels.py:157-158) —
    accumulated in float64.  x fp16 [B, K] -> fp16 [B, N]."""
    W = dequant_int4_runtime(packed, sz).astype(np.float64)
    xb = np.atleast_2d(np.asarray(x, dtype=np.float16)).astype(np.float64)
    y = xb @ W.T
    return y if acc else y.astype(np.float16)


def gemv_int4_blockwise(x: np.ndarray, packed: np.ndarray, sz: np.ndarray, acc: bool = False) -> np.ndarray:
    """Kernel semantics of ``gemv_warp`` (int4_decode_step.hip:131-169):
    y = sum_b s_b * sum_{i in b} x_i (q_i - z_b), float64, no fp16 weight rounding."""
    q = unpack_int4(packed).astype(np.float64)
    N, K = q.shape
    pairs = np.asarray(sz, dtype=np.float16).reshape(N, K // BLOCK, 2).astype(np.float64)
    xb = np.atleast_2d(np.asarray(x, dtype=np.float16)).astype(np.float64)
    qb = q.reshape(N, K // BLOCK, BLOCK) - pairs[..., 1:2]
    xr = xb.reshape(xb.shape[0], K // BLOCK, BLOCK)
    part = np.einsum('nkj,bkj->bnk', qb, xr)
    y = np.einsum('bnk,nk->bn', part, pairs[..., 0])
    return y if acc else y.astype(np.float16)


def gemv_int8(x: np.ndarray, w: np.ndarray, scale: np.ndarray, acc: bool = False) -> np.ndarray:
    """INT8 GEMV oracle: x @ dequantize_int8(w, s).T (int8_quant.py:52-69), float64."""
    W = dequant_int8(w, scale).astype(np.float64)
    xb = np.atleast_2d(np.asarray(x, dtype=np.float16)).astype(np.float64)
    y = xb @ W.T
    return y if acc else y.astype(np.float16)


def gemv_fp16(x: np.ndarray, w: np.ndarray, acc: bool = False) -> np.ndarray:
    """fp16-weight GEMV (fp16 lm_head), float64 accumulate."""
    W = np.asarray(w, dtype=np.float16).astype(np.float64)
    xb = np.atleast_2d(np.asarray(x, dtype=np.float16)).astype(np.float64)
    y = xb @ W.T
    return y if acc else y.astype(np.float16)


# --------------------------------------------------------------------------
# Norms  (engine_utils.py:58-63, int4_decode_step.hip:1143-1237, :1031-1051)
# --------------------------------------------------------------------------
def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """``RMSNorm.forward`` CPU branch (engine_utils.py:58-63) and
    ``fused_rmsnorm`` (fused_ops.py:12-41): fp16(x * rsqrt(mean(x^2)+eps) * w)."""
    xf = np.asarray(x, dtype=np.float16).astype(np.float32)
    v = (xf.astype(np.float64) ** 2).mean(-1, keepdims=True)
    r = (1.0 / np.sqrt(v + eps)).astype(np.float32)
    return (xf * r * np.asarray(w, dtype=np.float16).astype(np.float32)).astype(np.float16)


def rmsnorm_fwht(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """``fused_rmsnorm_fwht`` (int4_decode_step.hip:1195-1237):
    y = fp16(FWHT32(x * rrms * w)), rrms over float32 x."""
    xf = np.asarray(x, dtype=np.float16).astype(np.float32)
    D = xf.shape[-1]
    ss = (xf.astype(np.float64) ** 2).sum(-1, keepdims=True)
    rrms = (1.0 / np.sqrt(ss / D + eps)).astype(np.float32)
    n = xf * rrms * np.asarray(w, dtype=np.float16).astype(np.float32)
    return fwht32(n).astype(np.float16)


def res_norm_fwht(a: np.ndarray, b: np.ndarray, w: np.ndarray, eps: float):
    """``fused_res_norm_fwht`` (int4_decode_step.hip:1143-1192):
    r = a + b (float32); res_out = fp16(r); rrms from the UNROUNDED r;
    y = fp16(FWHT32(fp16(r) * rrms * w)).  Returns (y, res_out)."""
    r = (np.asarray(a, dtype=np.float16).astype(np.float32)
         + np.asarray(b, dtype=np.float16).astype(np.float32))
    D = r.shape[-1]
    ss = (r.astype(np.float64) ** 2).sum(-1, keepdims=True)
    rrms = (1.0 / np.sqrt(ss / D + eps)).astype(np.float32)
    res = r.astype(np.float16)
    n = res.astype(np.float32) * rrms * np.asarray(w, dtype=np.float16).astype(np.float32)
    return fwht32(n).astype(np.float16), res


def silu_fwht(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    """``silu_hadamard_ds`` (int4_decode_step.hip:1031-1051):
    y = fp16(FWHT32(g / (1 + exp(-g)) * u))."""
    gf = np.asarray(g, dtype=np.float16).astype(np.float64)
    uf = np.asarray(u, dtype=np.float16).astype(np.float64)
    v = (gf / (1.0 + np.exp(-gf)) * uf).astype(np.float32)
    return fwht32(v).astype(np.float16)


# --------------------------------------------------------------------------
# RoPE / head norm / KV write  (engine_utils.py:70-107; hip:1620-1683)
# --------------------------------------------------------------------------
def rope_tables(dim: int, max_seq: int, theta: float = 1e6):
    """``precompute_rope_freqs`` (engine_utils.py:70-76) in float32 -> fp16."""
    inv = (np.float32(1.0) / (np.float32(theta) ** (np.arange(0, dim, 2, dtype=np.float32)
                                                   / np.float32(dim)))).astype(np.float32)
    t = np.arange(max_seq, dtype=np.float32)
    f = np.outer(t, inv).astype(np.float32)
    return np.cos(f).astype(np.float16), np.sin(f).astype(np.float16)


def head_norm_rope(x: np.ndarray, w: np.ndarray, cos_row: np.ndarray,
                   sin_row: np.ndarray, eps: float) -> np.ndarray:
    """Per-head RMSNorm then half-split RoPE, all in float32 with a single
    fp16 rounding at the end — ``head_rmsnorm_rope_kv`` (hip:1632-1648) and
    ``qknorm_rope_kernel`` (fused_ops.py:89-152).  x fp16 [..., H, D];
    returns float32 (caller rounds)."""
    xf = np.asarray(x, dtype=np.float16).astype(np.float32)
    D = xf.shape[-1]
    half = D // 2
    ss = (xf.astype(np.float64) ** 2).sum(-1, keepdims=True)
    rrms = (1.0 / np.sqrt(ss / D + eps)).astype(np.float32)
    wf = np.asarray(w, dtype=np.float16).astype(np.float32)
    ne = xf[..., :half] * rrms * wf[:half]
    no = xf[..., half:] * rrms * wf[half:]
    c = np.asarray(cos_row, dtype=np.float16).astype(np.float32)
    s = np.asarray(sin_row, dtype=np.float16).astype(np.float32)
    return np.concatenate([ne * c - no * s, no * c + ne * s], axis=-1)


def rope_only(x: np.ndarray, cos_row: np.ndarray, sin_row: np.ndarray) -> np.ndarray:
    """``rope_kernel`` (fused_ops.py:44-86): half-split RoPE, float32, fp16 out."""
    xf = np.asarray(x, dtype=np.float16).astype(np.float32)
    half = xf.shape[-1] // 2
    c = np.asarray(cos_row, dtype=np.float16).astype(np.float32)
    s = np.asarray(sin_row, dtype=np.float16).astype(np.float32)
    a, b = xf[..., :half], xf[..., half:]
    return np.concatenate([a * c - b * s, b * c + a * s], axis=-1).astype(np.float16)


def qknorm_rope_kv(q, k, v, qw, kw, cos_row, sin_row, eps, kv_scale=None):
    """``head_rmsnorm_rope_kv`` (int4_decode_step.hip:1620-1683) for one token.
    q [B,H,D], k/v [B,Hk,D] fp16.  Returns (q_out fp16, k_out fp16,
    k_bytes u8 [B,Hk,D], v_bytes u8 [B,Hk,D]).  With ``kv_scale`` (fp32
    [B?,Hk] or [Hk]) the stored byte is enc(x / s) — the per-head-scale option;
    scale 1.0 reproduces the reference bytes exactly."""
    qo = head_norm_rope(q, qw, cos_row, sin_row, eps)
    ko = head_norm_rope(k, kw, cos_row, sin_row, eps)
    vf = np.asarray(v, dtype=np.float16).astype(np.float32)
    if kv_scale is None:
        kb, vb = fp8_encode(ko), fp8_encode(vf)
    else:
        ks, vs = kv_scale
        ks = np.asarray(ks, dtype=np.float32)[..., None]
        vs = np.asarray(vs, dtype=np.float32)[..., None]
        kb, vb = fp8_encode(ko / ks), fp8_encode(vf / vs)
    return qo.astype(np.float16), ko.astype(np.float16), kb, vb


# --------------------------------------------------------------------------
# Attention  (int4_decode_step.hip:1326-1593)
# --------------------------------------------------------------------------
def attention_decode(q: np.ndarray, kc: np.ndarray, vc: np.ndarray, seq_len: int,
                     k_scale=None, v_scale=None, fwht_out: bool = False) -> np.ndarray:
    """fp32/64 softmax attention over the decoded FP8 cache for one query token
    per batch row (the split-K flash-decode computes exactly this up to
    summation order, hip:1326-1463).  GQA: query head h uses kv head
    h // (H / Hk).  q fp16 [B,H,D]; kc/vc u8 [B,Hk,max_seq,D]; scales fp32
    [B,Hk] or None.  Q stays in full precision (the reference's fp8 packing of Q,
    hip:1349-1358, is deliberately not reproduced).  Returns fp16 [B,H,D]
    (FWHT32 applied to the output when ``fwht_out``, hip:1448-1461)."""
    qf = np.asarray(q, dtype=np.float16).astype(np.float64)
    B, H, D = qf.shape
    Hk = kc.shape[1]
    g = H // Hk
    K = fp8_decode(kc[:, :, :seq_len]).astype(np.float64)
    V = fp8_decode(vc[:, :, :seq_len]).astype(np.float64)
    if k_scale is not None:
        K = K * np.asarray(k_scale, dtype=np.float64).reshape(B, Hk, 1, 1)
    if v_scale is not None:
        V = V * np.asarray(v_scale, dtype=np.float64).reshape(B, Hk, 1, 1)
    Kx = np.repeat(K, g, axis=1)
    Vx = np.repeat(V, g, axis=1)
    s = np.einsum('bhd,bhsd->bhs', qf, Kx) / math.sqrt(D)
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    o = np.einsum('bhs,bhsd->bhd', p, Vx).astype(np.float32)
    if fwht_out:
        o = fwht32(o)
    return o.astype(np.float16)


def flash_decode_splits(seq_len: int):
    """Split sizing of ``launch_flash_decode`` (int4_decode_step.hip:1565-1575):
    (block_s, n_splits); a single fused pass when seq_len <= 32."""
    if seq_len <= 32:
        return seq_len, 1
    bs = 32 if seq_len <= 256 else 64
    return bs, (seq_len + bs - 1) // bs


def lse_merge(pmax: np.ndarray, psum: np.ndarray, pout: np.ndarray) -> np.ndarray:
    """Log-sum-exp merge of split partials, ``flash_decode_reduce``
    (int4_decode_step.hip:1416-1463).  pmax/psum [S, ...], pout [S, ..., D]."""
    gm = pmax.max(0)
    corr = np.exp(pmax - gm)
    tot = (psum * corr).sum(0)
    o = (pout * corr[..., None]).sum(0)
    inv = np.where(tot > 0, 1.0 / np.where(tot > 0, tot, 1.0), 0.0)
    return o * inv[..., None]


# --------------------------------------------------------------------------
# Decode step composition  (int4_decode_step.hip:2343-2595)
# --------------------------------------------------------------------------
# INT4 GEMV arithmetic used by decode_layer/decode_step*: 'blockwise' is the
# reference decode kernel's (gemv_warp, int4_decode_step.hip:131-169: per-block
# fp32 dot times scale, weights never rounded); 'dequant' is the reference
# Python/prefill path's (dequantize_int4_asym to fp16, then matmul).
INT4_MODE = {'mode': 'blockwise'}


def linear(x, lin, acc=False):
    """Dispatch a linear layer by its precision: ('int4', packed, sz) |
    ('int8', w, s) | ('fp16', w).  ``acc=True`` returns the unrounded float64
    sums (a tensor-parallel partial) instead of fp16."""
    kind = lin[0]
    if kind == 'int4':
        if INT4_MODE['mode'] == 'blockwise':
            return gemv_int4_blockwise(x, lin[1], lin[2], acc)
        return gemv_int4(x, lin[1], lin[2], acc)
    if kind == 'int8':
        return gemv_int8(x, lin[1], lin[2], acc)
    return gemv_fp16(x, lin[1], acc)


def decode_layer(h, rot, layer, next_norm, cfg, kc, vc, pos, cos_row, sin_row, write_kv=True,
                 allreduce=None):
    """One transformer layer of ``int4_decode_step`` (hip:2474-2524) for a
    batch of rows sharing ``pos``.  h fp16 [B, D] is the residual stream and
    rot the already normalised+rotated layer input.  kc/vc u8
    [B,Hk,max_seq,hd] are updated in place.  The closing residual+norm uses
    ``next_norm`` (the next layer's input norm; layer 0's for the last layer,
    hip:2519-2523).  With ``write_kv=False`` the bytes already in the cache at
    ``pos`` are used instead of this layer's own encoding (to check a device
    step against the cache it wrote).  Tensor parallel (no reference
    counterpart): with ``allreduce`` given, ``layer``/``cfg`` describe this
    rank's shard (its heads, its intermediate slice; o/down column slices) and
    o_proj/down_proj produce unrounded partial sums that ``allreduce`` sums
    over ranks before the single fp16 rounding of the single-GPU step.
    Returns (h_new, rot_next)."""
    H, Hk, hd, I, eps = (cfg['num_heads'], cfg['num_kv_heads'], cfg['head_dim'],
                         cfg['intermediate_size'], cfg['rms_eps'])
    B = h.shape[0]
    qkv = linear(rot, layer['qkv'])
    qd, kd = H * hd, Hk * hd
    q = qkv[:, :qd].reshape(B, H, hd)
    k = qkv[:, qd:qd + kd].reshape(B, Hk, hd)
    v = qkv[:, qd + kd:qd + 2 * kd].reshape(B, Hk, hd)
    qo, _, kb, vb = qknorm_rope_kv(q, k, v, layer['q_norm'], layer['k_norm'],
                                   cos_row, sin_row, eps)
    if write_kv:
        kc[:, :, pos, :] = kb
        vc[:, :, pos, :] = vb
    att = attention_decode(qo, kc, vc, pos + 1, fwht_out=True).reshape(B, qd)
    if allreduce is None:
        o = linear(att, layer['o'])
    else:
        o = np.asarray(allreduce(linear(att, layer['o'], acc=True))).astype(np.float16)
    rot, r = res_norm_fwht(o, h, layer['post_norm'], eps)
    gu = linear(rot, layer['gate_up'])
    act = silu_fwht(gu[:, :I], gu[:, I:2 * I])
    if allreduce is None:
        d = linear(act, layer['down'])
    else:
        d = np.asarray(allreduce(linear(act, layer['down'], acc=True))).astype(np.float16)
    rot_next, h_new = res_norm_fwht(d, r, next_norm, eps)
    return h_new, rot_next


def decode_step(h, layers, cfg, kcs, vcs, pos, cos, sin, write_kv=True, allreduce=None):
    """``int4_decode_step`` (hip:2343-2528): returns the final hidden fp16 [B, D].
    ``allreduce``: tensor-parallel shards, see ``decode_layer``."""
    eps = cfg['rms_eps']
    h = np.atleast_2d(np.asarray(h, dtype=np.float16))
    rot = rmsnorm_fwht(h, layers[0]['in_norm'], eps)
    L = len(layers)
    for li, layer in enumerate(layers):
        nxt = layers[li + 1]['in_norm'] if li < L - 1 else layers[0]['in_norm']
        h, rot = decode_layer(h, rot, layer, nxt, cfg, kcs[li], vcs[li], pos,
                              cos[pos], sin[pos], write_kv, allreduce)
    return h


def decode_step_logits(h, layers, cfg, kcs, vcs, pos, cos, sin, final_norm, lm, write_kv=True):
    """``int4_decode_step_logits`` (hip:2534-2595): all layers, then
    RMSNorm+FWHT of the final hidden with ``final_norm`` and the lm_head GEMV.
    Returns (fp16 logits [B, vocab], final hidden fp16 [B, D])."""
    h = decode_step(h, layers, cfg, kcs, vcs, pos, cos, sin, write_kv)
    rot = rmsnorm_fwht(h, final_norm, cfg['rms_eps'])
    return linear(rot, lm), h


# --------------------------------------------------------------------------
# Batched prefill  (int4_prefill_logits, int4_decode_step.hip:2127-2320)
# --------------------------------------------------------------------------
def causal_attention(q, k, v):
    """softmax(q kᵀ / sqrt(D)) v over positions <= the query's, GQA; q fp16
    [M, H, D], k/v fp16 [M, Hk, D] -> fp16 [M, H, D] (float64 inside): the
    role SDPA(is_causal=True, enable_gqa=True) plays at :2268-2277."""
    qf = np.asarray(q, np.float16).astype(np.float64)
    kf = np.asarray(k, np.float16).astype(np.float64)
    vf = np.asarray(v, np.float16).astype(np.float64)
    M, H, D = qf.shape
    G = H // kf.shape[1]
    kf = np.repeat(kf, G, axis=1)
    vf = np.repeat(vf, G, axis=1)
    s = np.einsum('mhd,nhd->hmn', qf, kf) / np.sqrt(D)
    mask = np.triu(np.ones((M, M), bool), 1)
    s[:, mask] = -np.inf
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    return np.einsum('hmn,nhd->mhd', p, vf).astype(np.float16)


def prefill_logits(x, layers, cfg, cos, sin, final_norm, lm):
    """``int4_prefill_logits`` for hidden rows x fp16 [M, D] (the embedding of
    the prompt) at positions 0..M-1: per layer rmsnorm -> H32 -> qkv ->
    head norm + RoPE -> causal attention -> H32 -> o -> residual + norm ->
    H32 -> gate_up -> fp16(silu·up) -> H32 -> down -> residual + next norm;
    every stage rounds to fp16 where the reference's kernels do.  No KV cache
    is written (the reference prefill writes none).  Returns logits fp16
    [M, vocab]."""
    H, Hk, hd, I, eps = (cfg['num_heads'], cfg['num_kv_heads'], cfg['head_dim'],
                         cfg['intermediate_size'], cfg['rms_eps'])
    x = np.asarray(x, np.float16)
    M = x.shape[0]
    qd, kd = H * hd, Hk * hd
    normed = rmsnorm(x, layers[0]['in_norm'], eps)
    for li, ly in enumerate(layers):
        qkv = linear(fwht32(normed.astype(np.float32)).astype(np.float16), ly['qkv'])
        q = qkv[:, :qd].reshape(M, H, hd)
        k = qkv[:, qd:qd + kd].reshape(M, Hk, hd)
        v = qkv[:, qd + kd:qd + 2 * kd].reshape(M, Hk, hd)
        qn = np.stack([head_norm_rope(q[m], ly['q_norm'], cos[m], sin[m], eps) for m in range(M)]).astype(np.float16)
        kn = np.stack([head_norm_rope(k[m], ly['k_norm'], cos[m], sin[m], eps) for m in range(M)]).astype(np.float16)
        att = causal_attention(qn, kn, v).reshape(M, qd)
        o = linear(fwht32(att.astype(np.float32)).astype(np.float16), ly['o'])
        r = (o.astype(np.float32) + x.astype(np.float32))
        normed = rmsnorm_unrounded(r, ly['post_norm'], eps)
        r16 = r.astype(np.float16)
        gu = linear(fwht32(normed.astype(np.float32)).astype(np.float16), ly['gate_up'])
        g = gu[:, :I].astype(np.float64)
        act = (g / (1.0 + np.exp(-g)) * gu[:, I:2 * I].astype(np.float64)).astype(np.float32).astype(np.float16)
        d = linear(fwht32(act.astype(np.float32)).astype(np.float16), ly['down'])
        xr = d.astype(np.float32) + r16.astype(np.float32)
        nxt = layers[li + 1]['in_norm'] if li + 1 < len(layers) else layers[0]['in_norm']
        normed = rmsnorm_unrounded(xr, nxt, eps)
        x = xr.astype(np.float16)
    n = rmsnorm(x, final_norm, eps)
    return linear(fwht32(n.astype(np.float32)).astype(np.float16), lm)


def rmsnorm_unrounded(r, w, eps):
    """fused_res_norm_batched (:2017-2052): rrms from the fp32 sum r (not
    rounded first), y = fp16(r * rrms * w)."""
    rf = np.asarray(r, np.float32)
    D = rf.shape[-1]
    ss = (rf.astype(np.float64) ** 2).sum(-1, keepdims=True)
    rrms = (1.0 / np.sqrt(ss / D + eps)).astype(np.float32)
    return (rf * rrms * np.asarray(w, np.float16).astype(np.float32)).astype(np.float16)


# --------------------------------------------------------------------------
# Mixture-of-experts FFN (benchmark config 4; no reference counterpart — the
# composition the B200 MoE kernels implement, built from the dense path's
# pieces: routing softmax in fp32, top-k, renormalised weights; experts as
# the dense gate_up / silu·up+FWHT / down chain; weighted sum, residual).
# --------------------------------------------------------------------------
def moe_route(logits, topk):
    """logits fp16 [B, E] -> (ids [B, topk], wts [B, topk]): softmax over E in
    float64, top-k by value (ties to the lower index), renormalised."""
    lg = np.asarray(logits, np.float16).astype(np.float64)
    p = np.exp(lg - lg.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    order = np.argsort(-lg, axis=-1, kind='stable')[:, :topk]
    w = np.take_along_axis(p, order, -1)
    return order, w / w.sum(-1, keepdims=True)


def moe_expert(rot_row, gu, down, Ie):
    """One token through one INT4 expert: fp16(W_d · fp16(H32(silu(g) u)))."""
    g = linear(rot_row[None], gu)
    act = silu_fwht(g[:, :Ie], g[:, Ie:2 * Ie])
    return linear(act, down)[0]


def moe_combine(ys, wts, r16):
    """h = fp16(fp16(sum_k w_k y_k) + r) with y_k fp16 [topk, D]."""
    s = (np.asarray(wts, np.float64)[:, None] * np.asarray(ys, np.float16).astype(np.float64)).sum(0)
    return (s.astype(np.float16).astype(np.float32) + np.asarray(r16, np.float16).astype(np.float32)).astype(
        np.float16)
