"""Batched prefill: all layers over M prompt tokens, logits [M, vocab]
(int4_prefill_logits, int4_decode_step.hip:2127-2320).

The projections run on the tcgen05 tensor-core GEMM (INT4 weights
dequantised inside the kernel; INT8 layers dequantised to an fp16 scratch
first); norms, H32 rotations, head norm + RoPE and SiLU·up are this
library's row kernels with the reference's fp16 rounding points.  Causal GQA
attention over the prompt is torch's scaled_dot_product_attention, as in the
reference (:2264-2277).  No KV cache is written, as in the reference."""
from __future__ import annotations

import torch

from . import lib as L
from . import ops


class _Scratch:
    def __init__(self):
        self.buf = None

    def get(self, n, dev):
        if self.buf is None or self.buf.numel() < n or self.buf.device != dev:
            self.buf = torch.empty(n, dtype=torch.float16, device=dev)
        return self.buf[:n]


_scratch = _Scratch()


INT4_DEQUANT_MIN_M = 1024      # measured on B200: pp512 equal, pp2048 +8 % (18.2 k vs 16.9 k tok/s)


def linear(x: torch.Tensor, w: torch.Tensor, s, N: int) -> torch.Tensor:
    """x [M, K] @ W^T for INT4 (uint8 nibbles), INT8 or fp16 weights."""
    M, K = x.shape
    if w.dtype == torch.uint8:
        if M >= INT4_DEQUANT_MIN_M:
            # long prompts: the weight tile is reused by M / 128 CTAs, so one
            # dequant pass (bit-exact, the reference prefill's dequant_int4)
            # plus the fp16 GEMM beats dequantising inside every M tile
            wd = _scratch.get(N * K, x.device).view(N, K)
            ops.dequant_int4(w, s, N, K, out=wd)
            return ops.gemm(x, wd)
        return ops.gemm(x, w, s, N)
    if w.dtype == torch.int8:
        wd = _scratch.get(N * K, x.device).view(N, K)
        ops.dequant_int8(w, s, out=wd)
        return ops.gemm(x, wd)
    return ops.gemm(x, w)


def prefill_logits(hidden: torch.Tensor, qkv_w, qkv_s, o_w, o_s, gu_w, gu_s, down_w, down_s, in_norm_w,
                   post_norm_w, q_norm_w, k_norm_w, rope_cos, rope_sin, num_heads, num_kv_heads, head_dim,
                   hidden_size, intermediate_size, rms_eps, final_norm_w, lm_w, lm_s, lm_N, k_caches=None,
                   v_caches=None, batch_row: int = 0, k_scales=None, v_scales=None, last_only: bool = False):
    """hidden fp16 [M, D] (embedded prompt) -> logits fp16 [M, lm_N].

    With ``k_caches`` / ``v_caches`` (uint8 [B, Hk, max_seq, 128] per layer)
    the prompt's rotated K and V of every layer are written to positions
    0..M-1 of ``batch_row`` (an extension: the reference prefill writes no
    cache), so decoding can continue at position M.  ``last_only`` returns
    the logits of the last position only [1, lm_N]."""
    x = hidden.reshape(-1, int(hidden_size)).contiguous()
    M, D = x.shape
    dev = x.device
    H, Hk, hd, I = int(num_heads), int(num_kv_heads), int(head_dim), int(intermediate_size)
    qd, kvd = H * hd, Hk * hd
    qkv_n = qd + 2 * kvd
    pos = torch.arange(M, dtype=torch.int64, device=dev)
    normed = ops.rmsnorm(x, in_norm_w[0], rms_eps)
    nl = len(qkv_w)
    for li in range(nl):
        qkv = linear(ops.fwht_rows(normed), qkv_w[li], qkv_s[li], qkv_n)
        ops.head_norm_rope(qkv, qkv[:, qd:], q_w=q_norm_w[li], k_w=k_norm_w[li], cos=rope_cos, sin=rope_sin,
                           pos_dev=pos, q_out=qkv, k_out=qkv[:, qd:], B=M, H=H, Hk=Hk, D=hd, ld_in=qkv_n,
                           ld_out=qkv_n, eps=rms_eps, flags=L.HEAD_NORM | L.HEAD_ROPE)
        if k_caches is not None:
            L.call("r4q_kv_write_rows", qkv[:, qd:].data_ptr(), qkv[:, qd + kvd:].data_ptr(), qkv_n,
                   k_caches[li].data_ptr(), v_caches[li].data_ptr(), M, Hk, hd, int(k_caches[li].shape[2]), 0,
                   int(batch_row), ops._ptr(None if k_scales is None else k_scales[li]),
                   ops._ptr(None if v_scales is None else v_scales[li]), ops.stream_handle(dev))
        q = qkv[:, :qd].view(M, H, hd).transpose(0, 1).unsqueeze(0)
        k = qkv[:, qd:qd + kvd].view(M, Hk, hd).transpose(0, 1).unsqueeze(0)
        v = qkv[:, qd + kvd:].view(M, Hk, hd).transpose(0, 1).unsqueeze(0)
        att = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        att = att.squeeze(0).transpose(0, 1).reshape(M, qd)
        o = linear(ops.fwht_rows(att), o_w[li], o_s[li], D)
        normed, r = ops.rmsnorm(o, post_norm_w[li], rms_eps, res=x, want_res=True)
        gu = linear(ops.fwht_rows(normed), gu_w[li], gu_s[li], 2 * I)
        act = ops.fwht_rows(ops.silu_mul(gu))
        d = linear(act, down_w[li], down_s[li], D)
        nxt = in_norm_w[li + 1] if li + 1 < nl else in_norm_w[0]
        normed, x = ops.rmsnorm(d, nxt, rms_eps, res=r, want_res=True)
    if last_only:
        x = x[-1:].contiguous()
    n = ops.rmsnorm(x, final_norm_w, rms_eps)
    return linear(ops.fwht_rows(n), lm_w, lm_s, int(lm_N))
