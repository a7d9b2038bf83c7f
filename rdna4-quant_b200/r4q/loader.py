"""Checkpoint loader for the reference's quantised model directories.

Reads both on-disk variants into the runtime layout the kernels take:

* v5 pure INT4 (quantize_v5_pure_int4.py) and v4 mixed INT4/INT8
  (quantize_v4_gptq.py:352-416): per layer ``layer_NNN.pt`` with, per group
  g in (qkv, o, gate_up, down), either ``g_packed`` uint8 [N, K/2],
  ``g_scales`` fp16 [N, K/32], ``g_zeros`` uint8 [N, K/32] (INT4; precision
  tag ``int4a`` = asymmetric, ``int4`` = symmetric two's-complement nibbles
  with zeros 0) or ``g_weights`` int8 [N, K] + ``g_scales`` (precision
  ``int8``), plus ``g_N``, ``g_K`` and the four norm vectors;
* ``lm_head.pt`` symmetric (packed + scales, quantize_v4_gptq.py:437-444) or
  asymmetric (with zeros); ``embed.pt``; ``final_norm.pt``; ``meta.pt``.

Runtime layout (int4_engine_v5.py:95-118): INT4 weights keep their nibbles
and get the interleaved (scale, zero-as-fp16) pairs [N, K/16]; symmetric INT4
is converted to unsigned nibbles with zero point 8 (nibble + 8 mod 16), which
dequantises to the same values.  The reference engine reads only the v5
variant (int4_engine_v5.py:141-155); this loader also reads v4's INT8 groups
and symmetric INT4 groups.  The returned dict has the keyword names of
``synth.build_decode_model`` (qkv_w, qkv_s, ..., embed, final_norm_w, lm_w,
lm_s, rope_cos, rope_sin), so the decode, loop and prefill paths take it as
they take the synthetic model.
"""
from __future__ import annotations

from pathlib import Path

import torch

GROUPS = (('qkv', 'qkv'), ('o', 'o'), ('gate_up', 'gu'), ('down', 'down'))


def interleave_scale_zero(scales: torch.Tensor, zeros: torch.Tensor) -> torch.Tensor:
    """fp16 scales [N, K/32] + uint8 zeros [N, K/32] -> fp16 pairs [N, K/16]
    (scale, zero-as-fp16) per block (int4_engine_v5.py:95-102)."""
    pairs = torch.stack([scales.half(), zeros.to(torch.float32).half()], dim=-1).contiguous()
    return pairs.view(pairs.shape[0], -1)


def symmetric_to_unsigned(packed: torch.Tensor, scales: torch.Tensor):
    """Two's-complement nibbles (value = int4(n) * s) -> unsigned nibbles with
    zero point 8 (value = (n' - 8) * s), n' = (n + 8) mod 16 — the same values
    (int4_engine_v5.py:105-118).  Returns (packed', pairs)."""
    lo = (packed & 0x0F).to(torch.int32)
    hi = ((packed >> 4) & 0x0F).to(torch.int32)
    out = (((lo + 8) & 0x0F) | (((hi + 8) & 0x0F) << 4)).to(torch.uint8)
    zeros = torch.full(scales.shape, 8, dtype=torch.uint8)
    return out.contiguous(), interleave_scale_zero(scales, zeros)


def rope_tables(head_dim: int, rows: int, theta: float, device):
    """fp16 cos/sin [rows, head_dim/2] (engine_utils.precompute_rope_freqs,
    engine_utils.py:70-76)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device).float() / head_dim))
    f = torch.outer(torch.arange(rows, device=device).float(), inv)
    return f.cos().half().contiguous(), f.sin().half().contiguous()


def _group(ld: dict, g: str):
    """One projection group -> (kind, weight, scales-or-pairs)."""
    prec = ld.get(f'{g}_precision')
    if f'{g}_weights' in ld or prec == 'int8':
        return 'int8', ld[f'{g}_weights'].to(torch.int8).contiguous(), ld[f'{g}_scales'].half().contiguous()
    packed, scales = ld[f'{g}_packed'].to(torch.uint8), ld[f'{g}_scales']
    zeros = ld.get(f'{g}_zeros')
    if prec == 'int4' or zeros is None:     # symmetric two's-complement nibbles
        return ('int4',) + symmetric_to_unsigned(packed, scales)
    return 'int4', packed.contiguous(), interleave_scale_zero(scales, zeros)


def load_checkpoint(quant_dir, device='cuda', max_seq: int = 2048, batch: int = 1) -> tuple[dict, dict]:
    """Load a quantised model directory.  Returns (cfg, model): cfg with the
    synth keys (num_layers, hidden, intermediate, num_heads, num_kv_heads,
    head_dim, vocab, rms_eps, rope_theta, meta), model with per-projection
    lists on ``device`` plus empty FP8 KV caches [batch, Hk, max_seq, D]."""
    d = Path(quant_dir)
    meta = torch.load(d / 'meta.pt', weights_only=False)
    L = int(meta['num_layers'])
    hd = int(meta['head_dim'])
    m = {k: [] for k in ('qkv_w', 'qkv_s', 'o_w', 'o_s', 'gu_w', 'gu_s', 'down_w', 'down_s', 'in_norm_w',
                         'post_norm_w', 'q_norm_w', 'k_norm_w', 'k_caches', 'v_caches')}
    precisions = []
    for li in range(L):
        ld = torch.load(d / f'layer_{li:03d}.pt', weights_only=False)
        row = {}
        for g, key in GROUPS:
            kind, w, s = _group(ld, g)
            N, K = int(ld[f'{g}_N']), int(ld[f'{g}_K'])
            exp = (N, K // 2) if kind == 'int4' else (N, K)
            if tuple(w.shape) != exp:
                raise ValueError(f"layer {li} {g}: weight shape {tuple(w.shape)} != {exp}")
            m[key + '_w'].append(w.to(device))
            m[key + '_s'].append(s.to(device))
            row[g] = kind
        precisions.append(row)
        for k, name in (('in_norm', 'in_norm_w'), ('post_norm', 'post_norm_w'), ('q_norm', 'q_norm_w'),
                        ('k_norm', 'k_norm_w')):
            m[name].append(ld[k].half().contiguous().to(device))
        hk = int(meta['num_kv_heads'])
        m['k_caches'].append(torch.zeros(batch, hk, max_seq, hd, dtype=torch.uint8, device=device))
        m['v_caches'].append(torch.zeros(batch, hk, max_seq, hd, dtype=torch.uint8, device=device))
    lm = torch.load(d / 'lm_head.pt', weights_only=False)
    if 'zeros' in lm:
        m['lm_w'], m['lm_s'] = lm['packed'].to(torch.uint8).contiguous(), interleave_scale_zero(lm['scales'],
                                                                                               lm['zeros'])
    else:
        m['lm_w'], m['lm_s'] = symmetric_to_unsigned(lm['packed'].to(torch.uint8), lm['scales'])
    m['lm_w'], m['lm_s'] = m['lm_w'].to(device), m['lm_s'].to(device)
    m['embed'] = torch.load(d / 'embed.pt', weights_only=True).half().contiguous().to(device)
    m['final_norm_w'] = torch.load(d / 'final_norm.pt', weights_only=True).half().contiguous().to(device)
    m['rope_cos'], m['rope_sin'] = rope_tables(hd, max_seq + 128, float(meta['rope_theta']), device)
    cfg = dict(num_layers=L, hidden=int(meta['hidden_size']), intermediate=int(meta['intermediate_size']),
               num_heads=int(meta['num_heads']), num_kv_heads=int(meta['num_kv_heads']), head_dim=hd,
               vocab=int(lm['N']), rms_eps=float(meta['rms_eps']), rope_theta=float(meta['rope_theta']),
               lm_K=int(lm['K']), meta=meta, precisions=precisions)
    return cfg, m
