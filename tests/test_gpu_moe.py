"""GPU: the mixture-of-experts decode step (benchmark config 4 architecture at
a small size) against the oracle composition of the same pieces.

Routing is a step function of the router logits: the device top-k must equal
the oracle top-k of the logits the device computed (bit-exact selection and
1e-6 weights), and the rest of the step is compared given that routing —
decode-step tolerance 2e-3 (see test_gpu_decode).  Plus the grouped expert
GEMV on its own at 1e-3 for batches 1, 5 and 40 (tokens per expert above one
8-token pass) in its three modes (plain rows of tokens, plain rows of
entries, gate_up with the SiLU*up + FWHT epilogue), and graph == eager."""
import numpy as np
import pytest
import torch

import r4q_oracle as O
from test_gpu_gemv import close

pytestmark = pytest.mark.gpu
CFG = dict(num_layers=2, hidden=256, num_heads=4, num_kv_heads=2, head_dim=128, experts=16, topk=4,
           expert_inter=128, vocab=512, rms_eps=1e-6, rope_theta=1e6)


def _np(t):
    return t.cpu().numpy()


def _lin4(w, s, e, N):
    return ('int4', _np(w[e * N:(e + 1) * N]), _np(s[e * N:(e + 1) * N]))


@pytest.mark.parametrize("B,D,Ie", [(1, 256, 128), (5, 256, 128), (40, 256, 128), (5, 4096, 128),
                                    (5, 256, 768), (6, 2048, 768)])
def test_grouped_expert_gemv(B, D, Ie):
    """D = 256: gate_up on the TMA-tile kernel, down (K = Ie = 128) on the
    register-staged one; D = 4096: gate_up (K = 4096, tile above 100 KB) on
    the register-staged kernel too; Ie = 768 (config 4): down on the TMA-tile
    kernel."""
    from r4q import ops, synth
    dev = torch.device('cuda')
    g = torch.Generator(device=dev).manual_seed(B + Ie)
    E, k = 16, 4
    wgu, sgu = synth.quantize_int4_asym(synth.weight_fp32(E * 2 * Ie, D, g, dev))
    wd, sd = synth.quantize_int4_asym(synth.weight_fp32(E * D, Ie, g, dev))
    logits = (torch.randn(B, E, generator=g, device=dev) * 2).half()
    x = torch.randn(B, D, generator=g, device=dev).half()
    rb = ops.moe_route(logits, k)
    gu = ops.moe_gemv(0, wgu, sgu, x, rb, 2 * Ie, D)
    act = ops.moe_gemv(2, wgu, sgu, x, rb, 2 * Ie, D)
    yk = ops.moe_gemv(1, wd, sd, act, rb, D, Ie)
    ids, w = O.moe_route(_np(logits), k)
    assert np.array_equal(_np(rb.ids), ids)
    assert np.allclose(_np(rb.wts), w, rtol=1e-5, atol=1e-6)
    O.INT4_MODE['mode'] = 'dequant'
    for b in range(B):
        for j in range(k):
            e = int(ids[b, j])
            ref_gu = O.linear(_np(x)[b:b + 1], _lin4(wgu, sgu, e, 2 * Ie))
            close(_np(gu)[b * k + j:b * k + j + 1], ref_gu)
            ref_act = O.silu_fwht(_np(gu)[b * k + j:b * k + j + 1, :Ie], _np(gu)[b * k + j:b * k + j + 1, Ie:])
            close(_np(act)[b * k + j:b * k + j + 1], ref_act)
            close(_np(yk)[b * k + j:b * k + j + 1], O.linear(_np(act)[b * k + j:b * k + j + 1], _lin4(wd, sd, e, D)))
    assert int(rb.status.item()) == 0
    # grouping: every entry once, experts ascending, token order inside
    cnt, off, lst = _np(rb.counts), _np(rb.offsets), _np(rb.list)
    for e in range(E):
        ent = lst[off[e]:off[e] + cnt[e]]
        assert np.all(ids.reshape(-1)[ent] == e) and np.all(np.diff(ent) > 0)
    assert sorted(lst.tolist()) == list(range(B * k))


@pytest.mark.parametrize("B", [1, 3, 40])
def test_fused_router(B):
    """r4q_moe_router: xn bit-identical to the row RMSNorm+FWHT pass, logits
    within fp16 rounding of xn · W_r, routing identical to r4q_moe_route on
    those logits; the precomputed-xn form gives the same logits; a second
    call (CTA counter reset by the kernel) repeats the first."""
    from r4q import ops
    dev = torch.device('cuda')
    g = torch.Generator(device=dev).manual_seed(40 + B)
    E, k, D = 16, 4, 256
    r = torch.randn(B, D, generator=g, device=dev).half()
    nw = (1 + 0.1 * torch.randn(D, generator=g, device=dev)).half()
    wr = (torch.randn(E, D, generator=g, device=dev) * 0.05).half()
    ss = (r.float() ** 2).view(B, D // 16, 16).sum(-1).t().contiguous()       # [D/16, B]
    ref_xn = ops.norm_fwht_rows(r, nw, 1e-6, ss_in=ss)
    rb = ops.MoeRouteBuffers(B, E, k, dev)
    xn = torch.empty(B, D, dtype=torch.float16, device=dev)
    lg = ops.moe_router(xn, wr, k, rb, x=r, ss_in=ss, norm_w=nw, eps=1e-6)
    torch.cuda.synchronize()
    assert torch.equal(xn, ref_xn)
    close(_np(lg), (ref_xn.float() @ wr.float().t()).cpu().numpy(), 1e-3)
    rb2 = ops.moe_route(lg, k, ops.MoeRouteBuffers(B, E, k, dev))
    for name in ('ids', 'wts', 'counts', 'offsets', 'list', 'n_active'):
        assert torch.equal(getattr(rb, name), getattr(rb2, name)), name
    na = int(rb.n_active.item())
    assert torch.equal(rb.active[:na], rb2.active[:na])
    rb3 = ops.MoeRouteBuffers(B, E, k, dev)
    lg3 = ops.moe_router(ref_xn.clone(), wr, k, rb3)
    lg4 = ops.moe_router(ref_xn.clone(), wr, k, rb3)
    torch.cuda.synchronize()
    assert torch.equal(lg3, lg) and torch.equal(lg4, lg) and torch.equal(rb3.ids, rb.ids)
    assert int(rb.done.item()) == 0 and int(rb3.done.item()) == 0


@pytest.mark.parametrize("B", [1, 4, 7, 20])
def test_moe_decode_step_vs_oracle(B):
    from r4q import moe
    dev = torch.device('cuda')
    c = CFG
    m = moe.build_moe_model(c, dev, seed=3, max_seq=64, batch=B)
    rng = np.random.default_rng(B)
    pos = 11
    for kc, vc in zip(m['k_caches'], m['v_caches']):
        kc[:, :, :pos] = torch.from_numpy(O.fp8_encode(rng.standard_normal((B, 2, pos, 128)).astype(np.float32))).cuda()
        vc[:, :, :pos] = torch.from_numpy(O.fp8_encode(rng.standard_normal((B, 2, pos, 128)).astype(np.float32))).cuda()
    h0 = m['embed'][torch.arange(B, device=dev) * 7 + 3]
    dec = moe.MoEDecoder(m, c, batch=B)
    eager = dec.step(h0, pos, use_graph=False).clone()
    torch.cuda.synchronize()
    graph = dec.step(h0, pos, use_graph=True).clone()
    torch.cuda.synchronize()
    assert torch.equal(eager, graph)
    # oracle, layer by layer, over the cache the GPU wrote and the GPU's routing
    D, H, Hk, hd, E, k, Ie = c['hidden'], c['num_heads'], c['num_kv_heads'], 128, c['experts'], c['topk'], c['expert_inter']
    eps = c['rms_eps']
    cos, sin = _np(m['rope_cos']), _np(m['rope_sin'])
    O.INT4_MODE['mode'] = 'blockwise' if B <= 2 else 'dequant'
    h = _np(h0)
    rot = O.rmsnorm_fwht(h, _np(m['in_norm_w'][0]), eps)
    dec2 = moe.MoEDecoder(m, c, batch=B)
    for li in range(c['num_layers']):
        qkv = O.linear(rot, ('int4', _np(m['qkv_w'][li]), _np(m['qkv_s'][li])))
        q = qkv[:, :H * hd].reshape(B, H, hd)
        kk = qkv[:, H * hd:(H + Hk) * hd].reshape(B, Hk, hd)
        v = qkv[:, (H + Hk) * hd:].reshape(B, Hk, hd)
        qo, _, _, _ = O.qknorm_rope_kv(q, kk, v, _np(m['q_norm_w'][li]), _np(m['k_norm_w'][li]), cos[pos], sin[pos], eps)
        att = O.attention_decode(qo, _np(m['k_caches'][li]), _np(m['v_caches'][li]), pos + 1, fwht_out=True)
        o = O.linear(att.reshape(B, H * hd), ('int4', _np(m['o_w'][li]), _np(m['o_s'][li])))
        rot2, r16 = O.res_norm_fwht(o, h, _np(m['post_norm_w'][li]), eps)
        logits = O.linear(rot2, ('fp16', _np(m['router_w'][li])))
        ids, wts = O.moe_route(logits, k)
        sums = []
        for b in range(B):
            ys = np.stack([O.moe_expert(rot2[b], _lin4(m['egu_w'][li], m['egu_s'][li], int(e), 2 * Ie),
                                        _lin4(m['edown_w'][li], m['edown_s'][li], int(e), D), Ie) for e in ids[b]])
            s = (wts[b][:, None] * ys.astype(np.float64)).sum(0).astype(np.float16)
            sums.append(s)
        nxt = _np(m['in_norm_w'][li + 1]) if li + 1 < c['num_layers'] else _np(m['final_norm_w'])
        if li + 1 < c['num_layers']:
            rot, h = O.res_norm_fwht(np.stack(sums), r16, nxt, eps)
        else:
            h = (np.stack(sums).astype(np.float32) + r16.astype(np.float32)).astype(np.float16)
    ref = O.linear(O.rmsnorm_fwht(h, _np(m['final_norm_w']), eps), ('fp16', _np(m['lm_w'])))
    close(_np(graph), ref, 2e-3)


def _ep_rank(rank, world, port, out_path, B):
    import os
    import torch.distributed as dist
    from r4q import moe, tp
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m = moe.build_moe_model(CFG, dev, seed=3, max_seq=64, batch=B)
        comm = tp.Comm(rank, world, max_batch=B, hidden=CFG['hidden'], sa_cap=1 << 16)
        dec = moe.MoEDecoder(m, CFG, batch=B, comm=comm)
        h0 = m['embed'][torch.arange(B, device=dev) * 7 + 3]
        a = dec.step(h0, 5).clone()
        b = dec.step(h0, 6).clone()
        torch.cuda.synchronize()
        comm.status()
        single = None
        if rank == 0:
            m1 = moe.build_moe_model(CFG, dev, seed=3, max_seq=64, batch=B)
            d1 = moe.MoEDecoder(m1, CFG, batch=B)
            d1.step(h0, 5)
            single = d1.step(h0, 6).cpu().numpy()
        dist.barrier()
        np.savez(f"{out_path}.{rank}.npz", a=a.cpu().numpy(), b=b.cpu().numpy(),
                 single=single if single is not None else np.zeros(0))
        comm.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_moe_expert_parallel_2gpu(tmp_path):
    """Expert parallelism over 2 GPUs (8 experts each, all-reduce of the fp32
    partials over NVLink): logits identical on both ranks and within 2e-3 of
    the 1-GPU decoder on the same model."""
    import torch.multiprocessing as mp
    from test_tp_cpu import free_port
    B = 3
    mp.spawn(_ep_rank, args=(2, free_port(), str(tmp_path / "m"), B), nprocs=2, join=True)
    r0, r1 = np.load(tmp_path / "m.0.npz"), np.load(tmp_path / "m.1.npz")
    assert np.array_equal(r0['a'], r1['a']) and np.array_equal(r0['b'], r1['b'])
    close(r0['b'], r0['single'], 2e-3)
