"""Tensor-parallel decode on CPU: the shard layout of r4q.tp composed with the
oracle, two gloo ranks, against the unsharded oracle step.

Each rank runs the oracle decode step on its own shard (its heads, its
intermediate slice, its KV heads, its vocabulary rows); o_proj / down_proj
partial sums are all-reduced over gloo (float64) before the fp16 rounding,
logits are all-gathered.  The result must equal the single-rank oracle up to
float64 summation order, and each rank's cache writes must be exactly its
heads' slice of the unsharded cache writes.  The same shard functions feed
the GPU contexts, so this pins the layout the device path relies on."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import r4q_oracle as O
from r4q import tp

D, I, H, HK, HD, V, MAXS, L = 512, 1024, 4, 2, 128, 1024, 64, 2
EPS = 1e-6
CFG = dict(num_heads=H, num_kv_heads=HK, head_dim=HD, hidden_size=D, intermediate_size=I, rms_eps=EPS)


def lin(rng, N, K, fmt):
    W = O.rotate_blocks(rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    if fmt == 'int8':
        q, s = O.quantize_int8_sym(W.reshape(N, K // 32, 32))
        return ('int8', q.reshape(N, K), s)
    if fmt == 'fp16':
        return ('fp16', W.astype(np.float16))
    q, s, z = O.quantize_int4_asym(W.reshape(N, K // 32, 32))
    return ('int4', O.pack_int4(q.reshape(N, K)), O.interleave_scale_zero(s, z))


def make_model(seed, fmts=('int4', 'int8'), lm_fmt='int4'):
    rng = np.random.default_rng(seed)
    layers = []
    for li in range(L):
        f = fmts[li % len(fmts)]
        layers.append({
            'qkv': lin(rng, (H + 2 * HK) * HD, D, f), 'o': lin(rng, D, H * HD, f),
            'gate_up': lin(rng, 2 * I, D, f), 'down': lin(rng, D, I, f),
            'in_norm': (1 + 0.1 * rng.standard_normal(D)).astype(np.float16),
            'post_norm': (1 + 0.1 * rng.standard_normal(D)).astype(np.float16),
            'q_norm': (1 + 0.1 * rng.standard_normal(HD)).astype(np.float16),
            'k_norm': (1 + 0.1 * rng.standard_normal(HD)).astype(np.float16)})
    final = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    lm = lin(rng, V, D, lm_fmt)
    return layers, final, lm


def make_inputs(seed, B, filled):
    rng = np.random.default_rng(seed)
    kc = np.zeros((L, B, HK, MAXS, HD), np.uint8)
    vc = np.zeros((L, B, HK, MAXS, HD), np.uint8)
    kc[..., :filled, :] = O.fp8_encode(rng.standard_normal((L, B, HK, filled, HD)).astype(np.float32))
    vc[..., :filled, :] = O.fp8_encode(rng.standard_normal((L, B, HK, filled, HD)).astype(np.float32))
    h = (rng.standard_normal((B, D)) * 0.5).astype(np.float16)
    return h, kc, vc


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _oracle_rank(rank, world, port, out_path, B, pos):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        O.INT4_MODE['mode'] = 'blockwise'
        layers, final, lm = make_model(7)
        h, kc, vc = make_inputs(8, B, pos)
        shards = [tp.shard_layer(ly, CFG, rank, world) for ly in layers]
        kcl = [tp.shard_heads(kc[li], rank, world) for li in range(L)]
        vcl = [tp.shard_heads(vc[li], rank, world) for li in range(L)]

        def allreduce(x):
            t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float64))
            dist.all_reduce(t)
            return t.numpy()

        cos, sin = O.rope_tables(HD, MAXS + 8, 1e6)
        hf = O.decode_step(h, shards, tp.local_cfg(CFG, world), kcl, vcl, pos, cos, sin,
                           allreduce=allreduce)
        rot = O.rmsnorm_fwht(hf, final, EPS)
        part = torch.from_numpy(np.ascontiguousarray(O.linear(rot, tp.shard_lm(lm, rank, world))))
        parts = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(parts, part)
        logits = torch.cat(parts, dim=1).numpy()
        np.savez(f"{out_path}.{rank}.npz", h=hf, logits=logits, kc=np.stack(kcl), vc=np.stack(vcl))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("B", [1, 2])
def test_tp2_oracle_matches_unsharded(tmp_path, B):
    world, pos = 2, 17
    mp.spawn(_oracle_rank, args=(world, free_port(), str(tmp_path / "r"), B, pos), nprocs=world, join=True)
    O.INT4_MODE['mode'] = 'blockwise'
    layers, final, lm = make_model(7)
    h, kc, vc = make_inputs(8, B, pos)
    cos, sin = O.rope_tables(HD, MAXS + 8, 1e6)
    kcs, vcs = [kc[li].copy() for li in range(L)], [vc[li].copy() for li in range(L)]
    ref, href = O.decode_step_logits(h, layers, CFG, kcs, vcs, pos, cos, sin, final, lm)
    res = [np.load(tmp_path / f"r.{r}.npz") for r in range(world)]
    for r in range(world):
        # replicated results: identical on every rank
        assert np.array_equal(res[r]['h'], res[0]['h'])
        assert np.array_equal(res[r]['logits'], res[0]['logits'])
        # each rank wrote exactly its heads' slice of the unsharded cache
        n = HK // world
        for li in range(L):
            assert np.array_equal(res[r]['kc'][li], kcs[li][:, r * n:(r + 1) * n])
            assert np.array_equal(res[r]['vc'][li], vcs[li][:, r * n:(r + 1) * n])
    d = np.abs(res[0]['h'].astype(np.float64) - href.astype(np.float64))
    assert d.max() <= 1e-3 * np.abs(href.astype(np.float64)).max()
    dl = np.abs(res[0]['logits'].astype(np.float64) - ref.astype(np.float64))
    assert dl.max() <= 1e-3 * np.abs(ref.astype(np.float64)).max()


def test_shard_layout_roundtrip():
    """Shards of every rank reassemble the full tensors (rows, columns, heads)."""
    layers, final, lm = make_model(3, fmts=('int4', 'int8', 'fp16'))
    for world in (1, 2):
        for ly in layers:
            sh = [tp.shard_layer(ly, CFG, r, world) for r in range(world)]
            # o / down: column shards concatenate back along K
            for name in ('o', 'down'):
                for j in range(1, len(ly[name])):
                    full = np.concatenate([s[name][j] for s in sh], axis=1)
                    assert np.array_equal(full, ly[name][j])
            # qkv rows: q heads of all ranks, then k, then v
            qd, kd = H * HD, HK * HD
            w = ly['qkv'][1]
            hl, kl = H // world * HD, HK // world * HD
            q = np.concatenate([s['qkv'][1][:hl] for s in sh])
            k = np.concatenate([s['qkv'][1][hl:hl + kl] for s in sh])
            v = np.concatenate([s['qkv'][1][hl + kl:] for s in sh])
            assert np.array_equal(np.concatenate([q, k, v]), w[:qd + 2 * kd])
            il = I // world
            g = np.concatenate([s['gate_up'][1][:il] for s in sh])
            u = np.concatenate([s['gate_up'][1][il:] for s in sh])
            assert np.array_equal(np.concatenate([g, u]), ly['gate_up'][1])
    with pytest.raises(ValueError):
        tp.shard_layer(layers[0], CFG, 0, 4)        # 2 KV heads do not split over 4
    with pytest.raises(ValueError):
        tp.shard_cols(layers[0]['o'], 16, 48)       # not whole 32-blocks


def test_tp_partial_gemv_sums_to_full():
    """Column-sharded partial sums (float64) add up to the unsharded GEMV."""
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((2, I)) * 0.5).astype(np.float16)
    for fmt in ('int4', 'int8', 'fp16'):
        full = lin(rng, D, I, fmt)
        O.INT4_MODE['mode'] = 'blockwise'
        ref = O.linear(x, full, acc=True)
        parts = sum(O.linear(x[:, r * I // 4:(r + 1) * I // 4], tp.shard_cols(full, r * I // 4, (r + 1) * I // 4),
                             acc=True) for r in range(4))
        assert np.allclose(parts, ref, rtol=1e-12, atol=1e-12)
