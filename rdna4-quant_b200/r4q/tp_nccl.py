"""Tensor-parallel decode with NCCL collectives between the GEMVs — the
comparison arm of the fused NVLink exchange (r4q.tp.TPDecoder).

Same shards, same kernels and the same rounding points as the fused path;
only the exchange differs: o_proj and down_proj write their unrounded fp32
partial sums to a local buffer (``out32``), ``torch.distributed.all_reduce``
(NCCL over NVLink/NVSwitch) sums them, and ``r4q_residual_f32`` forms
h = fp16(fp16(sum) + residual) with the per-16-row sums of squares the next
RMSNorm+FWHT prologue consumes.  The vocabulary slices of the lm_head are
gathered with ``all_gather_into_tensor``.  One decode token (step, device
argmax, embedding lookup) is captured in one CUDA graph, NCCL calls included.

NCCL's ring/tree sums are not in rank order, so unlike the fused exchange the
replicated hidden state is only equal across ranks to fp32 rounding; the
greedy tokens are compared with the fused arm by the tests at tolerance.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import lib as L
from . import ops
from .tp import fmt_of


class NcclTPDecoder:
    def __init__(self, shard: dict, cfg: dict, rank: int, world: int, batch: int = 1, group=None):
        self.s, self.cfg, self.B = shard, cfg, batch
        self.rank, self.world, self.group = rank, world, group
        dev = shard['embed'].device
        self.dev = dev
        D, I = cfg['hidden'], cfg['intermediate'] // world
        H, Hk, hd = cfg['num_heads'] // world, cfg['num_kv_heads'] // world, cfg['head_dim']
        self.H, self.Hk, self.hd, self.D, self.I = H, Hk, hd, D, I
        self.vl = int(shard['vocab']) // world
        f16 = dict(dtype=torch.float16, device=dev)
        B = batch
        self.h_in = torch.zeros(B, D, **f16)
        self.h = torch.zeros(B, D, **f16)
        self.r = torch.zeros(B, D, **f16)
        self.qkv = torch.zeros(B, (H + 2 * Hk) * hd, **f16)
        self.attn = torch.zeros(B, H, hd, **f16)
        self.gu = torch.zeros(B, 2 * I, **f16)
        self.part = torch.zeros(B, D, dtype=torch.float32, device=dev)
        self.ss_post = torch.zeros(D // 16, B, dtype=torch.float32, device=dev)
        self.ss_h = torch.zeros(D // 16, B, dtype=torch.float32, device=dev)
        self.lg_local = torch.zeros(B, self.vl, **f16)
        self.lg_all = torch.zeros(world, B, self.vl, **f16)
        self.seq = torch.ones(B, dtype=torch.int64, device=dev)
        self.tok = torch.zeros(B, dtype=torch.int64, device=dev)
        self.graph = None
        self.fmts = [{k: fmt_of(shard[k + '_w'][li]) for k in ('qkv', 'o', 'gu', 'down')}
                     for li in range(len(shard['qkv_w']))]

    def _gemv(self, li, key, x, N, K, **kw):
        s = self.s
        return ops.gemv(self.fmts[li][key], x, s[key + '_w'][li], s[key + '_s'][li], N, K, **kw)

    def _enqueue(self, greedy: bool):
        s, c = self.s, self.cfg
        D, I, H, Hk, hd, eps = self.D, self.I, self.H, self.Hk, self.hd, c['rms_eps']
        qkv_n = (H + 2 * Hk) * hd
        for li in range(len(s['qkv_w'])):
            hin = self.h_in if li == 0 else self.h
            self._gemv(li, 'qkv', hin, qkv_n, D, prologue=L.PRO_RMSNORM_FWHT, out=self.qkv,
                       norm_w=s['in_norm_w'][li], eps=eps, ss_in=None if li == 0 else self.ss_h)
            ops.attn_decode_fused(self.qkv, s['k_caches'][li], s['v_caches'][li], s['q_norm_w'][li],
                                  s['k_norm_w'][li], s['rope_cos'], s['rope_sin'], H, Hk, 0, fwht=True, eps=eps,
                                  out=self.attn, seq_dev=self.seq)
            self._gemv(li, 'o', self.attn.view(self.B, H * hd), D, H * hd, prologue=L.PRO_NONE, out32=self.part)
            dist.all_reduce(self.part, group=self.group)
            ops.residual_f32(self.part, hin, self.r, ss_out=self.ss_post)
            self._gemv(li, 'gu', self.r, 2 * I, D, prologue=L.PRO_RMSNORM_FWHT, out=self.gu,
                       norm_w=s['post_norm_w'][li], eps=eps, ss_in=self.ss_post)
            self._gemv(li, 'down', self.gu, D, I, prologue=L.PRO_SILU_FWHT, out32=self.part)
            dist.all_reduce(self.part, group=self.group)
            ops.residual_f32(self.part, self.r, self.h, ss_out=self.ss_h)
        lm_fmt = 'fp16' if s['lm_s'] is None else 'int4'
        ops.gemv(lm_fmt, self.h, s['lm_w'], s['lm_s'], self.vl, D, prologue=L.PRO_RMSNORM_FWHT,
                 out=self.lg_local, norm_w=s['final_norm_w'], eps=eps)
        dist.all_gather_into_tensor(self.lg_all, self.lg_local, group=self.group)
        if greedy:
            logits = self.lg_all.permute(1, 0, 2).reshape(self.B, -1)
            torch.argmax(logits, dim=-1, out=self.tok)
            self.h_in.copy_(s['embed'][self.tok])
            self.seq.add_(1)

    def loop(self, embed, h, start_pos: int, num_tokens: int) -> torch.Tensor:
        """Greedy tokens [num_tokens, batch] (device int64); one graph replay
        per token.  ``embed`` must be the shard's embedding table."""
        if embed is not self.s['embed']:
            raise ValueError("the captured graph reads the shard's embedding table")
        out = torch.empty(num_tokens, self.B, dtype=torch.int64, device=self.dev)
        self.h_in.copy_(h.reshape(self.B, self.D))
        self.seq.fill_(int(start_pos) + 1)
        if self.graph is None:
            st = torch.cuda.Stream(self.dev)
            st.wait_stream(torch.cuda.current_stream(self.dev))
            saved = (self.h_in.clone(), self.seq.clone())
            with torch.cuda.stream(st):
                self._enqueue(True)             # warm-up: workspaces, NCCL communicators
            torch.cuda.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=st):
                self._enqueue(True)
            torch.cuda.current_stream(self.dev).wait_stream(st)
            torch.cuda.synchronize()
            self.h_in.copy_(saved[0])
            self.seq.copy_(saved[1])
        for t in range(num_tokens):
            self.graph.replay()
            out[t].copy_(self.tok)
        return out
