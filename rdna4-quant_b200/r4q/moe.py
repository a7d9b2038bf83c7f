"""Mixture-of-experts decode (benchmark config 4: Qwen3-30B-A3B shape — 48
layers, hidden 2048, 32 query / 4 KV heads of 128, 128 experts with top-8
softmax routing, expert intermediate 768, INT4 block-32 asymmetric experts).

The reference engine is dense, so this model family has no reference
counterpart; it is built from the same pieces as the dense decode step
(dequant-GEMV with RMSNorm+FWHT prologues and residual epilogues, the fused
attention over the FP8 cache) plus the MoE kernels of ``csrc/moe.cu``:
fused router (RMSNorm+FWHT, fp16 H32-rotated router GEMV, top-k routing
and grouping by expert on the device, one launch) -> grouped expert gate_up (with the SiLU*up + FWHT epilogue) / down GEMVs -> weighted
combine with the residual.  One decode step is captured once in a CUDA graph
(positions live on the device) and replayed per token; no host
synchronisation inside the step.
"""
from __future__ import annotations


import torch

from . import lib as L
from . import ops, synth


def qwen3_30b_a3b_config(layers: int = 48) -> dict:
    return dict(num_layers=layers, hidden=2048, num_heads=32, num_kv_heads=4, head_dim=128, experts=128, topk=8,
                expert_inter=768, vocab=151936, rms_eps=1e-6, rope_theta=1e6)


def build_moe_model(cfg: dict, device, seed: int = 0, max_seq: int = 2304, batch: int = 1) -> dict:
    """Random-init weights of the config-4 architecture: INT4 qkv / o, fp16
    router [E, D] (H32-rotated like every projection), INT4 experts stacked
    per layer (gate_up [E*2Ie, D], down [E*D, Ie]), fp16 embedding and
    lm_head, FP8 KV caches [batch, Hk, max_seq, 128]."""
    g = torch.Generator(device=device).manual_seed(seed)
    Lr, D, H, Hk, hd = cfg['num_layers'], cfg['hidden'], cfg['num_heads'], cfg['num_kv_heads'], cfg['head_dim']
    E, Ie = cfg['experts'], cfg['expert_inter']
    m = {k: [] for k in ('qkv_w', 'qkv_s', 'o_w', 'o_s', 'router_w', 'egu_w', 'egu_s', 'edown_w', 'edown_s',
                         'in_norm_w', 'post_norm_w', 'q_norm_w', 'k_norm_w', 'k_caches', 'v_caches')}
    wbytes = 0
    for _ in range(Lr):
        for key, (N, K) in (('qkv', ((H + 2 * Hk) * hd, D)), ('o', (D, H * hd))):
            _, w, s = synth.linear_int4(N, K, g, device)
            m[key + '_w'].append(w)
            m[key + '_s'].append(s)
            wbytes += synth.gemv_bytes('int4', 0, N, K)
        rw = synth.rotate_blocks(torch.randn(E, D, generator=g, device=device) * 0.02)
        m['router_w'].append(rw.half().contiguous())
        for key, (N, K) in (('egu', (2 * Ie, D)), ('edown', (D, Ie))):
            w, s = synth.quantize_int4_asym(synth.weight_fp32(E * N, K, g, device))
            m[key + '_w'].append(w)
            m[key + '_s'].append(s)
        for k, n in (('in_norm_w', D), ('post_norm_w', D), ('q_norm_w', hd), ('k_norm_w', hd)):
            m[k].append((1 + 0.01 * torch.randn(n, generator=g, device=device)).half())
        m['k_caches'].append(torch.zeros(batch, Hk, max_seq, hd, dtype=torch.uint8, device=device))
        m['v_caches'].append(torch.zeros(batch, Hk, max_seq, hd, dtype=torch.uint8, device=device))
    V = cfg['vocab']
    m['embed'] = (torch.randn(V, D, generator=g, device=device) * 0.02).half()
    m['final_norm_w'] = (1 + 0.01 * torch.randn(D, generator=g, device=device)).half()
    m['lm_w'] = (torch.randn(V, D, generator=g, device=device) * 0.02).half()
    inv = 1.0 / (cfg['rope_theta'] ** (torch.arange(0, hd, 2, device=device).float() / hd))
    f = torch.outer(torch.arange(max_seq + 128, device=device).float(), inv)
    m['rope_cos'], m['rope_sin'] = f.cos().half(), f.sin().half()
    m['dense_weight_bytes'] = wbytes
    return m


def expert_bytes(cfg: dict, n_experts: int) -> int:
    """INT4 runtime bytes of n distinct experts (gate_up + down, nibbles + pairs)."""
    D, Ie = cfg['hidden'], cfg['expert_inter']
    return n_experts * (synth.gemv_bytes('int4', 0, 2 * Ie, D) + synth.gemv_bytes('int4', 0, D, Ie))


class MoEDecoder:
    """Batched decode steps of the config-4 model on one GPU, or expert-parallel
    over the ranks of ``comm`` (r4q.tp.Comm): every rank runs the attention,
    router and routing for all tokens (replicated, bit-identical), its own
    E / world experts, and the fp32 partial sums of the experts' weighted
    outputs are all-reduced over NVLink (r4q_comm_allreduce_f32, rank order)
    before the residual — so each token's expert outputs reach every rank in
    one exchange of B x hidden fp32 per layer."""

    def __init__(self, model: dict, cfg: dict, batch: int = 1, comm=None):
        self.m, self.cfg, self.B = model, cfg, batch
        self.comm = comm
        dev = model['embed'].device
        self.dev = dev
        D, H, Hk, hd = cfg['hidden'], cfg['num_heads'], cfg['num_kv_heads'], cfg['head_dim']
        E, k, Ie = cfg['experts'], cfg['topk'], cfg['expert_inter']
        f16 = dict(dtype=torch.float16, device=dev)
        B = batch
        self.h_in = torch.zeros(B, D, **f16)
        self.h = torch.zeros(B, D, **f16)
        self.r = torch.zeros(B, D, **f16)
        self.qkv = torch.zeros(B, (H + 2 * Hk) * hd, **f16)
        self.attn = torch.zeros(B, H, hd, **f16)
        self.rlog = torch.zeros(B, E, **f16)
        self.xn = torch.zeros(B, D, **f16)
        self.o16 = torch.zeros(B, D, **f16)
        self.act = torch.zeros(B * k, Ie, **f16)
        self.yk = torch.zeros(B * k, D, **f16)
        self.ss_post = torch.zeros(D // 16, B, dtype=torch.float32, device=dev)
        self.ss_h = torch.zeros(D // 16, B, dtype=torch.float32, device=dev)
        self.logits = torch.zeros(B, cfg['vocab'], **f16)
        self.seq = torch.ones(B, dtype=torch.int64, device=dev)
        W, rk = (comm.world, comm.rank) if comm is not None else (1, 0)
        if E % W:
            raise ValueError(f"{E} experts do not split over {W} ranks")
        self.e_lo, self.e_hi = rk * E // W, (rk + 1) * E // W
        self.rb = ops.MoeRouteBuffers(B, E, k, dev, self.e_lo, self.e_hi)
        # this rank's expert slices (views into the stacked per-layer tensors)
        gu_rows, d_rows = 2 * Ie, D
        self.egu = [(w[self.e_lo * gu_rows:self.e_hi * gu_rows], s[self.e_lo * gu_rows:self.e_hi * gu_rows])
                    for w, s in zip(model['egu_w'], model['egu_s'])]
        self.edown = [(w[self.e_lo * d_rows:self.e_hi * d_rows], s[self.e_lo * d_rows:self.e_hi * d_rows])
                      for w, s in zip(model['edown_w'], model['edown_s'])]
        if comm is not None:
            self.part = torch.zeros(B, D, dtype=torch.float32, device=dev)
            self.psum = torch.zeros(B, D, dtype=torch.float32, device=dev)
        self.graph = None

    def _enqueue(self):
        m, c = self.m, self.cfg
        D, H, Hk, hd = c['hidden'], c['num_heads'], c['num_kv_heads'], c['head_dim']
        Ie, eps = c['expert_inter'], c['rms_eps']
        qkv_n = (H + 2 * Hk) * hd
        big = self.B > 16          # the GEMV takes up to 16 rows: larger batches use the tensor-core GEMM
        for li in range(c['num_layers']):
            hin = self.h_in if li == 0 else self.h
            if big:
                ops.norm_fwht_rows(hin, m['in_norm_w'][li], eps, ss_in=None if li == 0 else self.ss_h, out=self.xn)
                ops.gemm(self.xn, m['qkv_w'][li], m['qkv_s'][li], qkv_n, out=self.qkv)
            else:
                ops.gemv('int4', hin, m['qkv_w'][li], m['qkv_s'][li], qkv_n, D, prologue=L.PRO_RMSNORM_FWHT,
                         out=self.qkv, norm_w=m['in_norm_w'][li], eps=eps, ss_in=None if li == 0 else self.ss_h)
            ops.attn_decode_fused(self.qkv, m['k_caches'][li], m['v_caches'][li], m['q_norm_w'][li],
                                  m['k_norm_w'][li], m['rope_cos'], m['rope_sin'], H, Hk, 0, fwht=True, eps=eps,
                                  out=self.attn, seq_dev=self.seq)
            if big:
                ops.gemm(self.attn.view(self.B, H * hd), m['o_w'][li], m['o_s'][li], D, out=self.o16)
                ops.residual_f16(self.o16, hin, self.r, ss_out=self.ss_post)
            else:
                ops.gemv('int4', self.attn.view(self.B, H * hd), m['o_w'][li], m['o_s'][li], D, H * hd,
                         out=self.r, residual=hin, ss_out=self.ss_post)
            # router: RMSNorm+FWHT of r as its own pass (measured on B200 at
            # B = 1: 4 + 8.6 us against 16.1 us with the norm inside the
            # router's CTAs), then logits + top-k + grouping in one launch
            ops.norm_fwht_rows(self.r, m['post_norm_w'][li], eps, ss_in=self.ss_post, out=self.xn)
            ops.moe_router(self.xn, m['router_w'][li], c['topk'], self.rb, logits=self.rlog)
            ops.moe_gemv(2, self.egu[li][0], self.egu[li][1], self.xn, self.rb, 2 * Ie, D, out=self.act)
            ops.moe_gemv(1, self.edown[li][0], self.edown[li][1], self.act, self.rb, D, Ie, out=self.yk)
            if self.comm is None:
                ops.moe_combine(self.yk, self.rb, self.r, out=self.h, ss_out=self.ss_h)
            else:
                ops.moe_combine(self.yk, self.rb, None, out32=self.part)
                self.comm.allreduce_f32(self.part, out=self.psum)
                ops.residual_f32(self.psum, self.r, self.h, ss_out=self.ss_h)
        if big:
            ops.norm_fwht_rows(self.h, m['final_norm_w'], eps, out=self.xn)
            ops.gemm(self.xn, m['lm_w'], None, c['vocab'], out=self.logits)
        else:
            ops.gemv('fp16', self.h, m['lm_w'], None, c['vocab'], D, prologue=L.PRO_RMSNORM_FWHT,
                     out=self.logits, norm_w=m['final_norm_w'], eps=eps)

    def step(self, hidden: torch.Tensor, pos: int, use_graph: bool = True) -> torch.Tensor:
        """hidden fp16 [B, D] at position pos -> logits [B, vocab] (the step's
        buffer; copy it before the next step).  K/V of pos go to the caches."""
        self.h_in.copy_(hidden.reshape(self.B, -1))
        self.seq.fill_(int(pos) + 1)
        if not use_graph:
            self._enqueue()
            return self.logits
        if self.graph is None:
            s = torch.cuda.Stream(self.dev)
            s.wait_stream(torch.cuda.current_stream(self.dev))
            with torch.cuda.stream(s):
                self._enqueue()                 # warm-up on the capture stream: workspaces, attributes
            torch.cuda.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=s):
                self._enqueue()
            torch.cuda.current_stream(self.dev).wait_stream(s)
        self.graph.replay()
        return self.logits
