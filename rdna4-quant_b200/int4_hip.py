"""Drop-in for the reference's native module ``int4_hip``
(hip_int4/int4_decode_step.hip:3620-3636), running on B200 through libr4q.so.

Same function names, argument order, tensor layouts and return shapes as the
reference pybind module; the reference engine (int4_engine_v5.py) imports it
with ``import int4_hip`` after putting this folder on ``sys.path``.  Unlike the
reference, failures raise ``r4q.lib.R4QError`` instead of returning silently.
"""
from __future__ import annotations

import torch

from r4q import decode as _dec
from r4q import lib as _lib
from r4q import ops as _ops

# CUDA-graph replay of the decode step (one capture per context; the position is
# a device scalar).  Set to False to enqueue the kernels eagerly.
USE_GRAPH = True


def dbg_gemv(X: torch.Tensor, W: torch.Tensor, S: torch.Tensor, N: int, K: int) -> torch.Tensor:
    """INT4 asym GEMV, X fp16 [K] -> Y fp16 [N] (int4_decode_step.hip:3541-3550)."""
    return _ops.gemv('int4', X.reshape(1, K), W, S, int(N), int(K)).reshape(int(N))


def dbg_gemm(X: torch.Tensor, W: torch.Tensor, S: torch.Tensor, M: int, N: int, K: int) -> torch.Tensor:
    """Batched INT4 GEMV, X fp16 [M, K] -> Y fp16 [M, N] (int4_decode_step.hip:3552-3563).
    Batches above 16 rows are processed 16 rows per launch."""
    M, N, K = int(M), int(N), int(K)
    X2 = X.reshape(M, K)
    Y = torch.empty(M, N, dtype=torch.float16, device=X.device)
    for r in range(0, M, 16):
        _ops.gemv('int4', X2[r:r + 16], W, S, N, K, out=Y[r:r + 16])
    return Y


def dequant_int4(packed: torch.Tensor, scales: torch.Tensor, N: int, K: int) -> torch.Tensor:
    """[N, K/2] u8 + [N, K/16] interleaved (scale, zero) fp16 -> [N, K] fp16,
    bit-exact (int4_decode_step.hip:3568-3603)."""
    return _ops.dequant_int4(packed, scales, int(N), int(K))


def fp16_to_fp8(src: torch.Tensor) -> torch.Tensor:
    """fp16 tensor -> uint8 tensor of the same shape, reference E4M3 encoder
    (int4_decode_step.hip:3606-3618)."""
    return _ops.fp16_to_fp8(src)


def dbg_rmsnorm(X: torch.Tensor, W: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm of the flat vector X (int4_decode_step.hip:3473-3484)."""
    return _ops.rmsnorm(X.reshape(1, -1), W, eps).reshape(X.shape)


def dbg_fused_res_norm(X: torch.Tensor, Res: torch.Tensor, W: torch.Tensor, eps: float):
    """[Y, ResOut]: r = X + Res in fp32, Y = RMSNorm(r) from the unrounded r,
    ResOut = fp16(r) (int4_decode_step.hip:818-846, 3524-3539)."""
    y, r = _ops.rmsnorm(X.reshape(1, -1), W, eps, res=Res.reshape(1, -1), want_res=True)
    return [y.reshape(X.shape), r.reshape(X.shape)]


def dbg_head_rmsnorm(Q, K, QW, KW, H, Hk, D, eps):
    """[Q_out, K_out]: per-head RMSNorm of flat Q [H*D], K [Hk*D] (hip:849-884, 3486-3504)."""
    H, Hk, D = int(H), int(Hk), int(D)
    qo, ko = torch.empty_like(Q), torch.empty_like(K)
    _ops.head_norm_rope(Q, K, q_w=QW, k_w=KW, q_out=qo, k_out=ko, H=H, Hk=Hk, D=D,
                        ld_in=0, ld_out=0, eps=eps, flags=_lib.HEAD_NORM)
    return [qo, ko]


def dbg_rope(Q, K, COS, SIN, H, Hk, D):
    """[Q_out, K_out]: half-split RoPE with the table rows COS/SIN [D/2]
    (hip:888-912, 3506-3522)."""
    H, Hk, D = int(H), int(Hk), int(D)
    qo, ko = torch.empty_like(Q), torch.empty_like(K)
    _ops.head_norm_rope(Q, K, cos=COS.reshape(1, -1), sin=SIN.reshape(1, -1), pos=0,
                        q_out=qo, k_out=ko, H=H, Hk=Hk, D=D, ld_in=0, ld_out=0,
                        flags=_lib.HEAD_ROPE)
    return [qo, ko]


def decode_step(hidden_in, qkv_w, qkv_s, qkv_N, o_w, o_s, o_N, gu_w, gu_s, gu_N, down_w, down_s,
                down_N, in_norm_w, post_norm_w, q_norm_w, k_norm_w, rope_cos, rope_sin, pos,
                num_heads, num_kv_heads, head_dim, hidden_size, intermediate_size, rms_eps,
                k_caches, v_caches, hadamard_mat=None):
    """All layers of one decode token; returns the final hidden state
    [B, 1, hidden] (int4_decode_step.hip:2343-2528).  Weights per layer are
    INT4 (uint8 packed + (scale, zero) pairs) or INT8 (int8 + fp16 scales);
    ``hadamard_mat`` is accepted and unused, as in the reference."""
    B = hidden_in.numel() // int(hidden_size)
    ctx = _dec.get_context(qkv_w, qkv_s, o_w, o_s, gu_w, gu_s, down_w, down_s, in_norm_w,
                           post_norm_w, q_norm_w, k_norm_w, rope_cos, rope_sin, num_heads,
                           num_kv_heads, head_dim, hidden_size, intermediate_size, rms_eps,
                           k_caches, v_caches, batch=B)
    h = hidden_in.reshape(B, int(hidden_size)).contiguous()
    out = torch.empty(B, 1, int(hidden_size), dtype=torch.float16, device=h.device)
    ctx.step(h, pos, hidden_out=out, use_graph=USE_GRAPH)
    return out


def decode_step_logits(hidden_in, qkv_w, qkv_s, qkv_N, o_w, o_s, o_N, gu_w, gu_s, gu_N, down_w,
                       down_s, down_N, in_norm_w, post_norm_w, q_norm_w, k_norm_w, rope_cos,
                       rope_sin, pos, num_heads, num_kv_heads, head_dim, hidden_size,
                       intermediate_size, rms_eps, k_caches, v_caches, final_norm_w, lm_w, lm_s,
                       lm_N, lm_K, hadamard_mat=None):
    """One decode token through every layer, the final RMSNorm+FWHT and the
    lm_head; returns logits [B, 1, lm_N] fp16 (int4_decode_step.hip:2534-2595).
    lm_head may be INT4 (the reference's converted symmetric INT4), INT8 or
    fp16 (lm_s None)."""
    B = hidden_in.numel() // int(hidden_size)
    ctx = _dec.get_context(qkv_w, qkv_s, o_w, o_s, gu_w, gu_s, down_w, down_s, in_norm_w,
                           post_norm_w, q_norm_w, k_norm_w, rope_cos, rope_sin, num_heads,
                           num_kv_heads, head_dim, hidden_size, intermediate_size, rms_eps,
                           k_caches, v_caches, final_norm_w, lm_w, lm_s, lm_N, batch=B)
    h = hidden_in.reshape(B, int(hidden_size)).contiguous()
    logits = torch.empty(B, 1, int(lm_N), dtype=torch.float16, device=h.device)
    ctx.step(h, pos, logits_out=logits, use_graph=USE_GRAPH)
    return logits


def _logits_ctx(hidden, qkv_w, qkv_s, o_w, o_s, gu_w, gu_s, down_w, down_s, in_norm_w, post_norm_w,
                q_norm_w, k_norm_w, rope_cos, rope_sin, num_heads, num_kv_heads, head_dim, hidden_size,
                intermediate_size, rms_eps, k_caches, v_caches, final_norm_w, lm_w, lm_s, lm_N):
    B = hidden.numel() // int(hidden_size)
    ctx = _dec.get_context(qkv_w, qkv_s, o_w, o_s, gu_w, gu_s, down_w, down_s, in_norm_w,
                           post_norm_w, q_norm_w, k_norm_w, rope_cos, rope_sin, num_heads,
                           num_kv_heads, head_dim, hidden_size, intermediate_size, rms_eps,
                           k_caches, v_caches, final_norm_w, lm_w, lm_s, lm_N, batch=B)
    return ctx, hidden.reshape(B, int(hidden_size)).contiguous()


def decode_loop(embed_weight, final_norm_w, lm_w, lm_s, lm_N, lm_K, first_token_hidden, num_tokens,
                qkv_w, qkv_s, qkv_N, o_w, o_s, o_N, gu_w, gu_s, gu_N, down_w, down_s, down_N,
                in_norm_w, post_norm_w, q_norm_w, k_norm_w, rope_cos, rope_sin, start_pos,
                num_heads, num_kv_heads, head_dim, hidden_size, intermediate_size, rms_eps,
                k_caches, v_caches, hadamard_mat=None):
    """Greedy decode of ``num_tokens`` tokens starting at ``start_pos`` from
    the first token's hidden state; token ids int64 on the CPU
    (int4_decode_step.hip:3284-3466): every token is one device-side step +
    argmax + embedding lookup, no host synchronisation until the end.
    Returns [num_tokens] for one row, [num_tokens, B] for a batch."""
    ctx, h = _logits_ctx(first_token_hidden, qkv_w, qkv_s, o_w, o_s, gu_w, gu_s, down_w, down_s,
                         in_norm_w, post_norm_w, q_norm_w, k_norm_w, rope_cos, rope_sin, num_heads,
                         num_kv_heads, head_dim, hidden_size, intermediate_size, rms_eps, k_caches,
                         v_caches, final_norm_w, lm_w, lm_s, lm_N)
    toks = ctx.loop(embed_weight, h, start_pos, num_tokens, use_graph=USE_GRAPH)
    toks = toks.cpu()
    return toks.reshape(-1) if toks.shape[1] == 1 else toks


def _bench(hidden_in, embed_weight, num_tokens, layer_args, use_graph):
    (qkv_w, qkv_s, qkv_N, o_w, o_s, o_N, gu_w, gu_s, gu_N, down_w, down_s, down_N, in_norm_w,
     post_norm_w, q_norm_w, k_norm_w, rope_cos, rope_sin, start_pos, num_heads, num_kv_heads,
     head_dim, hidden_size, intermediate_size, rms_eps, k_caches, v_caches, final_norm_w, lm_w,
     lm_s, lm_N, lm_K, hadamard_mat) = layer_args
    ctx, h = _logits_ctx(hidden_in, qkv_w, qkv_s, o_w, o_s, gu_w, gu_s, down_w, down_s, in_norm_w,
                         post_norm_w, q_norm_w, k_norm_w, rope_cos, rope_sin, num_heads, num_kv_heads,
                         head_dim, hidden_size, intermediate_size, rms_eps, k_caches, v_caches,
                         final_norm_w, lm_w, lm_s, lm_N)
    ctx.loop(embed_weight, h, start_pos, num_tokens, use_graph=use_graph)


def decode_bench(hidden_in, embed_weight, num_tokens, *layer_args):
    """Greedy decode of ``num_tokens`` tokens with per-kernel launches (no
    graph), as the reference's C++ benchmark loop (int4_decode_step.hip:
    2601-2795).  Returns None; the caller times it."""
    _bench(hidden_in, embed_weight, num_tokens, layer_args, False)


def decode_bench_graph(hidden_in, embed_weight, num_tokens, *layer_args):
    """The same with one CUDA-graph launch per token (int4_decode_step.hip:
    2801-3041); unlike the reference it keeps the argmax and the embedding
    lookup inside the graph.  Returns None; the caller times it."""
    _bench(hidden_in, embed_weight, num_tokens, layer_args, True)


def decode_profile(hidden_in, embed_weight, qkv_w, qkv_s, qkv_N, o_w, o_s, o_N, gu_w, gu_s, gu_N,
                   down_w, down_s, down_N, in_norm_w, post_norm_w, q_norm_w, k_norm_w, rope_cos,
                   rope_sin, start_pos, num_heads, num_kv_heads, head_dim, hidden_size,
                   intermediate_size, rms_eps, k_caches, v_caches, final_norm_w, lm_w, lm_s, lm_N,
                   lm_K, hadamard_mat=None):
    """[total_ms, gemv_ms, attn_ms, norm_ms, rest_ms] of one eager decode step
    at ``start_pos`` (int4_decode_step.hip:3047-3281)."""
    ctx, h = _logits_ctx(hidden_in, qkv_w, qkv_s, o_w, o_s, gu_w, gu_s, down_w, down_s, in_norm_w,
                         post_norm_w, q_norm_w, k_norm_w, rope_cos, rope_sin, num_heads, num_kv_heads,
                         head_dim, hidden_size, intermediate_size, rms_eps, k_caches, v_caches,
                         final_norm_w, lm_w, lm_s, lm_N)
    return ctx.profile(h, start_pos)


def prefill_logits(input_ids, embed_weight, final_norm_w, lm_w, lm_s, lm_N, lm_K, qkv_w, qkv_s, qkv_N,
                   o_w, o_s, o_N, gu_w, gu_s, gu_N, down_w, down_s, down_N, in_norm_w, post_norm_w,
                   q_norm_w, k_norm_w, rope_cos, rope_sin, num_heads, num_kv_heads, head_dim,
                   hidden_size, intermediate_size, rms_eps, hadamard_mat=None):
    """All layers over the prompt ``input_ids`` [M] -> logits [M, lm_N] fp16
    (int4_decode_step.hip:2127-2320), projections on the tcgen05 GEMM.
    Weights per layer may be INT4, INT8 or fp16; ``hadamard_mat`` is accepted
    and unused, as in the reference."""
    from r4q import prefill as _pf
    x = embed_weight[input_ids.reshape(-1).to(embed_weight.device)]
    return _pf.prefill_logits(x, qkv_w, qkv_s, o_w, o_s, gu_w, gu_s, down_w, down_s, in_norm_w,
                              post_norm_w, q_norm_w, k_norm_w, rope_cos, rope_sin, num_heads,
                              num_kv_heads, head_dim, hidden_size, intermediate_size, rms_eps,
                              final_norm_w, lm_w, lm_s, lm_N)
