"""GPU parity of the split-K flash-decode attention over the FP8 cache
(benchmark config 2 shape: 40 query / 8 KV heads, head_dim 128; K/V ~ N(0,1)
stored as E4M3 with a per-head fp32 scale; Q ~ N(0,1) fp16).  Reference: fp32
softmax over the dequantised cache (oracle.attention_decode).  Tolerance 1e-3
relative (max-norm and L2, as for the GEMV)."""
import numpy as np
import pytest
import torch

import r4q_oracle as O
from test_gpu_gemv import close, cuda

pytestmark = pytest.mark.gpu
H, HK, D = 40, 8, 128


def make_cache(rng, B, ctx, max_seq, scaled):
    k = rng.standard_normal((B, HK, ctx, D)).astype(np.float16)
    v = rng.standard_normal((B, HK, ctx, D)).astype(np.float16)
    kc = np.zeros((B, HK, max_seq, D), np.uint8)
    vc = np.zeros((B, HK, max_seq, D), np.uint8)
    if scaled:
        ks = (np.abs(k.astype(np.float32)).max(axis=(2, 3)) / 448.0).astype(np.float32)
        vs = (np.abs(v.astype(np.float32)).max(axis=(2, 3)) / 448.0).astype(np.float32)
        kc[:, :, :ctx] = O.fp8_encode(k.astype(np.float32) / ks[:, :, None, None])
        vc[:, :, :ctx] = O.fp8_encode(v.astype(np.float32) / vs[:, :, None, None])
        return kc, vc, ks, vs
    kc[:, :, :ctx] = O.fp8_encode(k.astype(np.float32))
    vc[:, :, :ctx] = O.fp8_encode(v.astype(np.float32))
    return kc, vc, None, None


@pytest.mark.parametrize("B,ctx", [(1, 1), (1, 33), (1, 128), (4, 300), (1, 2048), (16, 128), (2, 4095)])
@pytest.mark.parametrize("scaled", [True, False])
def test_flash_decode_vs_fp32_softmax(B, ctx, scaled):
    from r4q import ops
    rng = np.random.default_rng(B * 10007 + ctx + scaled)
    max_seq = ctx + 17
    kc, vc, ks, vs = make_cache(rng, B, ctx, max_seq, scaled)
    q = rng.standard_normal((B, H, D)).astype(np.float16)
    o = ops.flash_decode(cuda(q), cuda(kc), cuda(vc), ctx,
                         k_scale=None if ks is None else cuda(ks),
                         v_scale=None if vs is None else cuda(vs)).cpu().numpy()
    ref = O.attention_decode(q, kc, vc, ctx, ks, vs)
    close(o, ref)


def test_flash_decode_fwht_epilogue_and_device_seq():
    from r4q import ops
    rng = np.random.default_rng(5)
    B, ctx, max_seq = 2, 777, 1024
    kc, vc, _, _ = make_cache(rng, B, ctx, max_seq, False)
    q = rng.standard_normal((B, H, D)).astype(np.float16)
    ref = O.attention_decode(q, kc, vc, ctx, fwht_out=True)
    o1 = ops.flash_decode(cuda(q), cuda(kc), cuda(vc), ctx, fwht=True).cpu().numpy()
    close(o1, ref)
    seq = torch.full((B,), ctx, dtype=torch.int64, device="cuda")
    o2 = ops.flash_decode(cuda(q), cuda(kc), cuda(vc), 0, fwht=True, seq_dev=seq).cpu().numpy()
    close(o2, ref)


def test_flash_decode_long_context():
    """ctx 32768 (config 2's longest), B = 1."""
    from r4q import ops
    rng = np.random.default_rng(6)
    ctx = 32768
    kc, vc, ks, vs = make_cache(rng, 1, ctx, ctx, True)
    q = rng.standard_normal((1, H, D)).astype(np.float16)
    o = ops.flash_decode(cuda(q), cuda(kc), cuda(vc), ctx, k_scale=cuda(ks), v_scale=cuda(vs))
    close(o.cpu().numpy(), O.attention_decode(q, kc, vc, ctx, ks, vs))


def test_flash_decode_repeatable_and_workspace_clean():
    from r4q import ops
    rng = np.random.default_rng(8)
    kc, vc, _, _ = make_cache(rng, 1, 500, 512, False)
    q = cuda(rng.standard_normal((1, H, D)).astype(np.float16))
    a = ops.flash_decode(q, cuda(kc), cuda(vc), 500)
    b = ops.flash_decode(q, cuda(kc), cuda(vc), 500)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("B,ctx,scaled", [(1, 1, False), (1, 64, False), (1, 65, True), (2, 300, False),
                                          (1, 2048, True), (4, 4097, False), (1, 9000, False)])
def test_fused_head_ops_attention_equals_two_kernels(B, ctx, scaled):
    """r4q_attn_decode_fused (q/k norm + RoPE + FP8 write of row ctx-1 +
    attention) leaves the same cache bytes and the same output, bit for bit,
    as r4q_head_norm_rope followed by r4q_flash_decode; and matches the oracle."""
    from r4q import lib as L, ops
    rng = np.random.default_rng(B * 31 + ctx)
    max_seq = ctx + 9
    kc, vc, ks, vs = make_cache(rng, B, ctx - 1, max_seq, scaled)
    qkv = (rng.standard_normal((B, (H + 2 * HK) * D)) * 2).astype(np.float16)
    qw = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    kw = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    cos, sin = O.rope_tables(D, max_seq + 4, 1e6)
    t = cuda
    tks, tvs = (None, None) if ks is None else (t(ks), t(vs))
    pos = ctx - 1
    # two kernels
    q1 = t(qkv)
    kc1, vc1 = t(kc), t(vc)
    ops.head_norm_rope(q1[:, :H * D], q1[:, H * D:], v=q1[:, (H + HK) * D:], q_w=t(qw), k_w=t(kw), cos=t(cos),
                       sin=t(sin), pos=pos, q_out=q1[:, :H * D], k_out=q1[:, H * D:], k_cache=kc1, v_cache=vc1,
                       k_scale=tks, v_scale=tvs, B=B, H=H, Hk=HK, D=D,
                       flags=L.HEAD_NORM | L.HEAD_ROPE | L.HEAD_KV)
    qn = q1[:, :H * D].reshape(B, H, D).contiguous()
    o1 = ops.flash_decode(qn, kc1, vc1, ctx, k_scale=tks, v_scale=tvs, fwht=True)
    # fused
    kc2, vc2 = t(kc), t(vc)
    o2 = ops.attn_decode_fused(t(qkv), kc2, vc2, t(qw), t(kw), t(cos), t(sin), H, HK, ctx, k_scale=tks,
                               v_scale=tvs, fwht=True)
    torch.cuda.synchronize()
    assert torch.equal(kc1, kc2) and torch.equal(vc1, vc2)
    assert torch.equal(o1, o2)
    ref = O.attention_decode(qn.cpu().numpy(), kc2.cpu().numpy(), vc2.cpu().numpy(), ctx, ks, vs, fwht_out=True)
    close(o2.cpu().numpy(), ref)
