"""Tensor-parallel decode on 2 GPUs: one process per GPU, the NVLink exchange
(r4q_comm_*) inside the CUDA-graph decode step, against the oracle and against
the 1-GPU context.

Each rank shards the small mixed INT4/INT8 model with r4q.tp (the layout the
gloo test pins against the oracle), runs decode tokens with o_proj / down_proj
partials pushed into the peers' buffers and reduced there, and the lm_head
vocabulary gathered.  Checks: logits identical on both ranks, graph == eager,
logits within the decode-step tolerance of the oracle attending over the cache
the GPUs wrote, and of the 1-GPU context; the standalone all-reduce is exact
(fp32 sum in rank order); a wait that nobody answers times out into a status
instead of hanging.  Skipped with fewer than 2 GPUs."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import r4q_oracle as O
from test_gpu_gemv import close
from test_tp_cpu import CFG, D, EPS, HD, HK, H, I, L, MAXS, V, free_port, make_inputs, make_model

pytestmark = pytest.mark.gpu
STEP_TOL = 2e-3
POS = 21


def _ctx_args(layers, final, lm, kc, vc, dev, H_, HK_, I_, vocab_rows, batch, comm=None):
    from r4q import decode

    def t(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    g = {k: [] for k in ('qkv_w', 'qkv_s', 'o_w', 'o_s', 'gu_w', 'gu_s', 'down_w', 'down_s')}
    for ly in layers:
        for name, key in (('qkv', 'qkv'), ('o', 'o'), ('gate_up', 'gu'), ('down', 'down')):
            g[key + '_w'].append(t(ly[name][1]))
            g[key + '_s'].append(t(ly[name][2]))
    norms = [[t(ly[k]) for ly in layers] for k in ('in_norm', 'post_norm', 'q_norm', 'k_norm')]
    kcs = [t(kc[li]) for li in range(L)]
    vcs = [t(vc[li]) for li in range(L)]
    cos, sin = O.rope_tables(HD, MAXS + 8, 1e6)
    tc, ts = t(cos), t(sin)
    lm_w = t(lm[1])
    lm_s = t(lm[2]) if lm[0] != 'fp16' else None
    ctx = decode.get_context(g['qkv_w'], g['qkv_s'], g['o_w'], g['o_s'], g['gu_w'], g['gu_s'],
                             g['down_w'], g['down_s'], *norms, tc, ts, H_, HK_, HD, D, I_, EPS, kcs,
                             vcs, t(final), lm_w, lm_s, vocab_rows, batch=batch, comm=comm)
    keep = (g, norms, tc, ts, lm_w, lm_s)
    return ctx, kcs, vcs, keep


def _gpu_rank(rank, world, port, out_path, B):
    from r4q import decode, tp
    from r4q.lib import R4QError
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layers, final, lm = make_model(7)
        h, kc, vc = make_inputs(8, B, POS)
        comm = tp.Comm(rank, world, max_batch=B, hidden=D, vocab=V, sa_cap=1 << 16)
        shards = [tp.shard_layer(ly, CFG, rank, world) for ly in layers]
        kcl = np.stack([tp.shard_heads(kc[li], rank, world) for li in range(L)])
        vcl = np.stack([tp.shard_heads(vc[li], rank, world) for li in range(L)])
        out = {}
        for use_graph in (False, True):
            ctx, kcs, vcs, keep = _ctx_args(shards, final, tp.shard_lm(lm, rank, world), kcl, vcl, dev,
                                            H // world, HK // world, I // world, V // world, B, comm)
            hin = torch.from_numpy(h).to(dev)
            a = torch.empty(B, V, dtype=torch.float16, device=dev)
            b = torch.empty(B, V, dtype=torch.float16, device=dev)
            ctx.step(hin, POS, logits_out=a, use_graph=use_graph)
            ctx.step(hin, POS + 1, logits_out=b, use_graph=use_graph)
            torch.cuda.synchronize()
            comm.status()
            out[use_graph] = (a.cpu().numpy(), b.cpu().numpy(),
                              np.stack([k.cpu().numpy() for k in kcs]), np.stack([v.cpu().numpy() for v in vcs]))
            decode.clear_contexts()
            del ctx, kcs, vcs, keep
        # standalone all-reduce: exact fp32 sum in rank order
        xs = [np.random.default_rng(100 + r).standard_normal(4099).astype(np.float32) for r in range(world)]
        y = comm.allreduce_f32(torch.from_numpy(xs[rank]).to(dev))
        torch.cuda.synchronize()
        comm.status()
        ref = xs[0].copy()
        for r in range(1, world):
            ref = ref + xs[r]
        ar_exact = bool(np.array_equal(y.cpu().numpy(), ref))
        # 1-GPU context on rank 0 for comparison
        single = None
        if rank == 0:
            ctx1, _, _, keep1 = _ctx_args(layers, final, lm, kc, vc, dev, H, HK, I, V, B, None)
            s = torch.empty(B, V, dtype=torch.float16, device=dev)
            ctx1.step(torch.from_numpy(h).to(dev), POS, logits_out=s, use_graph=True)
            torch.cuda.synchronize()
            single = s.cpu().numpy()
            decode.clear_contexts()
            del ctx1, keep1
        dist.barrier()
        # timeout: rank 0 all-reduces alone; its wait gives up (~2 s) with a status
        timed_out = None
        if rank == 0:
            comm.allreduce_f32(torch.ones(64, device=dev))
            torch.cuda.synchronize()
            try:
                comm.status()
                timed_out = False
            except R4QError as e:
                timed_out = ("rank(s) 1" in str(e))
        dist.barrier()
        np.savez(f"{out_path}.{rank}.npz", eager_a=out[False][0], eager_b=out[False][1],
                 graph_a=out[True][0], graph_b=out[True][1], kc=out[True][2], vc=out[True][3],
                 ar_exact=ar_exact, single=single if single is not None else np.zeros(0),
                 timed_out=np.array(-1 if timed_out is None else int(timed_out)))
        comm.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("B", [1, 2])
def test_tp2_decode_vs_oracle_and_single_gpu(tmp_path, B):
    world = 2
    mp.spawn(_gpu_rank, args=(world, free_port(), str(tmp_path / "g"), B), nprocs=world, join=True)
    res = [np.load(tmp_path / f"g.{r}.npz") for r in range(world)]
    for r in range(world):
        for k in ('eager_a', 'eager_b', 'graph_a', 'graph_b'):
            assert np.array_equal(res[r][k], res[0][k]), k        # replicated logits
        assert np.array_equal(res[r]['graph_a'], res[r]['eager_a'])
        assert np.array_equal(res[r]['graph_b'], res[r]['eager_b'])
        assert bool(res[r]['ar_exact'])
    assert int(res[0]['timed_out']) == 1
    # oracle of the first token over the cache the GPUs wrote (heads of both ranks)
    layers, final, lm = make_model(7)
    h, kc, vc = make_inputs(8, B, POS)
    kg = np.concatenate([res[r]['kc'] for r in range(world)], axis=2)   # [L, B, HK, S, D]
    vg = np.concatenate([res[r]['vc'] for r in range(world)], axis=2)
    O.INT4_MODE['mode'] = 'blockwise'
    cos, sin = O.rope_tables(HD, MAXS + 8, 1e6)
    ref, _ = O.decode_step_logits(h, layers, CFG, [k.copy() for k in kg], [v.copy() for v in vg], POS,
                                  cos, sin, final, lm, write_kv=False)
    close(res[0]['graph_a'], ref, STEP_TOL)
    close(res[0]['graph_a'], res[0]['single'], STEP_TOL)


def _nccl_rank(rank, world, port, out_path):
    """The NCCL all-reduce arm (r4q.tp_nccl) against the fused exchange on the
    same shards: logits of one token at the decode-step tolerance, and the
    greedy tokens of a short loop."""
    from r4q import decode, synth, tp
    from r4q.tp_nccl import NcclTPDecoder
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        cfg = dict(num_layers=2, hidden=1024, intermediate=2048, num_heads=8, num_kv_heads=2, head_dim=128,
                   vocab=4096, rms_eps=1e-6, rope_theta=1e6)
        m = synth.build_decode_model(cfg, dev, seed=5, max_seq=96)
        synth.fill_kv_synthetic(m, 40, seed=2)
        sh = tp.shard_decode_model(m, cfg, rank, world)
        comm = tp.Comm(rank, world, max_batch=1, hidden=cfg['hidden'], vocab=cfg['vocab'])
        fused = tp.TPDecoder(sh, cfg, comm, batch=1)
        nccl = NcclTPDecoder(sh, cfg, rank, world, batch=1)
        h0 = m['embed'][7].reshape(1, -1).contiguous()
        lf = fused.step(h0, 40, use_graph=False).float().cpu().numpy()
        nccl.loop(sh['embed'], h0, 40, 1)
        ln = nccl.lg_all.permute(1, 0, 2).reshape(1, -1).float().cpu().numpy()
        tf = fused.loop(sh['embed'], h0, 41, 4).cpu().numpy()
        tn = nccl.loop(sh['embed'], h0, 41, 4).cpu().numpy()
        torch.cuda.synchronize()
        comm.status()
        np.savez(f"{out_path}.{rank}.npz", lf=lf, ln=ln, tf=tf, tn=tn)
        decode.clear_contexts()
        del fused, nccl
        comm.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_nccl_arm_matches_fused_exchange(tmp_path):
    world = 2
    mp.spawn(_nccl_rank, args=(world, free_port(), str(tmp_path / "n")), nprocs=world, join=True)
    res = [np.load(tmp_path / f"n.{r}.npz") for r in range(world)]
    for r in range(world):
        close(res[r]['ln'], res[r]['lf'], STEP_TOL)
        assert np.array_equal(res[r]['tn'], res[0]['tn'])          # replicated tokens
    assert (res[0]['tn'] == res[0]['tf']).mean() >= 0.75
