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


def _torch_attention_ref(q, kc, vc, ctx, ks, vs):
    """fp64 softmax attention over the decoded cache, computed per (row, KV
    head) on the device to bound memory (the B = 16, ctx 32768 cache is 1 GB
    of bytes); FP8 bytes decoded with the reference codec's table
    (int4_decode_step.hip:71-81, restated in the oracle)."""
    lut = torch.from_numpy(O.fp8_decode(np.arange(256, dtype=np.uint8)).astype(np.float64)).to(q.device)
    B, Hq, Dd = q.shape
    Hk = kc.shape[1]
    g = Hq // Hk
    out = torch.empty(B, Hq, Dd, dtype=torch.float64, device=q.device)
    for b in range(B):
        for h in range(Hk):
            K = lut[kc[b, h, :ctx].long()] * ks[b, h].double()
            V = lut[vc[b, h, :ctx].long()] * vs[b, h].double()
            qq = q[b, h * g:(h + 1) * g].double()
            sc = (qq @ K.t()) / np.sqrt(Dd)
            out[b, h * g:(h + 1) * g] = torch.softmax(sc, dim=-1) @ V
    return out.float().cpu().numpy()


@pytest.mark.parametrize("B", [1, 4, 16])
@pytest.mark.parametrize("ctx", [128, 2048, 32768])
def test_flash_decode_config2_grid(B, ctx):
    """Benchmark config 2's whole grid (B 1/4/16 x ctx 128/2048/32768): K/V
    ~ N(0,1) stored as E4M3 with per-head fp32 scales, Q ~ N(0,1) fp16,
    against fp64 softmax attention over the dequantised cache (<= 1e-3)."""
    from r4q import ops
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(B * 1000 + ctx)
    k = torch.randn(B, HK, ctx, D, generator=g, device=dev)
    v = torch.randn(B, HK, ctx, D, generator=g, device=dev)
    ks = (k.abs().amax(dim=(2, 3)) / 448.0).float()
    vs = (v.abs().amax(dim=(2, 3)) / 448.0).float()
    kc = ops.fp16_to_fp8((k / ks[:, :, None, None]).half())
    vc = ops.fp16_to_fp8((v / vs[:, :, None, None]).half())
    del k, v
    q = torch.randn(B, H, D, generator=g, device=dev).half()
    o = ops.flash_decode(q, kc, vc, ctx, k_scale=ks, v_scale=vs).cpu().numpy()
    close(o, _torch_attention_ref(q, kc, vc, ctx, ks, vs))


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
