"""GPU: batched prefill (int4_hip.prefill_logits) on the tcgen05 GEMM against
the oracle's composition of the reference prefill (int4_prefill_logits,
int4_decode_step.hip:2127-2320) on a small Qwen3-shaped model with INT4 and
INT8 layers, INT4 or fp16 lm_head.  Every stage rounds to fp16 where the
reference does; the GPU accumulates in fp32 (tensor cores, SDPA) and the
oracle in fp64, so a rounding can land one ulp away and travel through the
later stages: 5e-3 relative (max-norm and L2) on the logits of 2 layers,
with each GEMM held to 1e-3 in its own test.  Plus the row kernels exactly."""
import numpy as np
import pytest
import torch

import r4q_oracle as O
from test_gpu_gemv import close, cuda
from test_tp_cpu import CFG, D, EPS, HD, HK, H, I, L, MAXS, V, make_model

pytestmark = pytest.mark.gpu


def _dev_lists(layers):
    g = {k: [] for k in ('qkv_w', 'qkv_s', 'o_w', 'o_s', 'gu_w', 'gu_s', 'down_w', 'down_s')}
    for ly in layers:
        for name, key in (('qkv', 'qkv'), ('o', 'o'), ('gate_up', 'gu'), ('down', 'down')):
            g[key + '_w'].append(cuda(ly[name][1]))
            g[key + '_s'].append(cuda(ly[name][2]) if len(ly[name]) > 2 else None)
    norms = [[cuda(ly[k]) for ly in layers] for k in ('in_norm', 'post_norm', 'q_norm', 'k_norm')]
    return g, norms


@pytest.mark.parametrize("M,lm_fmt", [(1, 'int4'), (37, 'fp16'), (200, 'int4')])
def test_prefill_logits_vs_oracle(M, lm_fmt):
    import int4_hip
    rng = np.random.default_rng(M)
    layers, final, lm = make_model(17, ('int4', 'int8'), lm_fmt)
    embed = (rng.standard_normal((V, D)) * 0.5).astype(np.float16)
    ids = rng.integers(0, V, M)
    cos, sin = O.rope_tables(HD, max(MAXS, M) + 8, 1e6)
    g, norms = _dev_lists(layers)
    lm_w = cuda(lm[1])
    lm_s = cuda(lm[2]) if lm[0] != 'fp16' else None
    out = int4_hip.prefill_logits(torch.from_numpy(ids).cuda(), cuda(embed), cuda(final), lm_w, lm_s, V, D,
                                  g['qkv_w'], g['qkv_s'], 0, g['o_w'], g['o_s'], 0, g['gu_w'], g['gu_s'], 0,
                                  g['down_w'], g['down_s'], 0, *norms, cuda(cos), cuda(sin), H, HK, HD, D, I,
                                  EPS, None)
    assert out.shape == (M, V) and out.dtype == torch.float16
    O.INT4_MODE['mode'] = 'dequant'
    ref = O.prefill_logits(embed[ids], layers, CFG, cos, sin, final, lm)
    close(out.cpu().numpy(), ref, 5e-3)


def test_row_kernels():
    from r4q import ops
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((5, 256)) * 3).astype(np.float16)
    y = ops.fwht_rows(cuda(x)).cpu().numpy()
    assert np.array_equal(y, O.fwht32(x.astype(np.float32)).astype(np.float16))
    gu = rng.standard_normal((3, 2 * 96)).astype(np.float16)
    a = ops.silu_mul(cuda(gu)).cpu().numpy().astype(np.float32)
    g = gu[:, :96].astype(np.float64)
    ra = (g / (1 + np.exp(-g)) * gu[:, 96:].astype(np.float64)).astype(np.float16).astype(np.float32)
    assert np.abs(a - ra).max() <= 1e-3 * np.abs(ra).max()
    q, s = O.quantize_int8_sym((rng.standard_normal((64, 128)) * 0.05).reshape(64, 4, 32))
    w = q.reshape(64, 128)
    d = ops.dequant_int8(cuda(w), cuda(s)).cpu().numpy()
    assert np.array_equal(d, O.dequant_int8(w, s))


def test_prefill_writes_kv_then_decode_continues():
    """prefill with caches writes the prompt's K/V (positions 0..M-1, within one
    FP8 code of the oracle's encoding on >= 95 % of bytes); a decode step at
    position M over that cache matches the oracle decode over the same bytes."""
    import int4_hip
    from r4q import decode, prefill
    rng = np.random.default_rng(4)
    M, B = 23, 1
    layers, final, lm = make_model(29, ('int4', 'int8'), 'int4')
    embed = (rng.standard_normal((V, D)) * 0.5).astype(np.float16)
    ids = rng.integers(0, V, M)
    cos, sin = O.rope_tables(HD, MAXS + 8, 1e6)
    g, norms = _dev_lists(layers)
    kcs = [torch.zeros(B, HK, MAXS, HD, dtype=torch.uint8, device='cuda') for _ in range(L)]
    vcs = [torch.zeros(B, HK, MAXS, HD, dtype=torch.uint8, device='cuda') for _ in range(L)]
    lm_w, lm_s = cuda(lm[1]), cuda(lm[2])
    x = cuda(embed)[torch.from_numpy(ids).cuda()]
    last = prefill.prefill_logits(x, g['qkv_w'], g['qkv_s'], g['o_w'], g['o_s'], g['gu_w'], g['gu_s'], g['down_w'],
                                  g['down_s'], *norms, cuda(cos), cuda(sin), H, HK, HD, D, I, EPS, cuda(final),
                                  lm_w, lm_s, V, k_caches=kcs, v_caches=vcs, last_only=True)
    assert last.shape == (1, V)
    tok = int(last.reshape(-1).argmax())
    h = cuda(embed[tok]).reshape(1, 1, D)
    lg = int4_hip.decode_step_logits(h, g['qkv_w'], g['qkv_s'], 0, g['o_w'], g['o_s'], 0, g['gu_w'], g['gu_s'], 0,
                                     g['down_w'], g['down_s'], 0, *norms, cuda(cos), cuda(sin), M, H, HK, HD, D, I,
                                     EPS, kcs, vcs, cuda(final), lm_w, lm_s, V, D, None)
    torch.cuda.synchronize()
    O.INT4_MODE['mode'] = 'blockwise'
    ref, _ = O.decode_step_logits(embed[tok].reshape(1, D), layers, CFG, [k.cpu().numpy() for k in kcs],
                                  [v.cpu().numpy() for v in vcs], M, cos, sin, final, lm, write_kv=False)
    close(lg.cpu().numpy().reshape(1, V), ref, 2e-3)
    # the prompt rows against the oracle's own K (layer 0 is exact up to GEMM rounding)
    O.INT4_MODE['mode'] = 'dequant'
    qd, kd = H * HD, HK * HD
    normed = O.rmsnorm(embed[ids], layers[0]['in_norm'], EPS)
    qkv = O.linear(O.fwht32(normed.astype(np.float32)).astype(np.float16), layers[0]['qkv'])
    kn = np.stack([O.head_norm_rope(qkv[m, qd:qd + kd].reshape(HK, HD), layers[0]['k_norm'], cos[m], sin[m], EPS)
                   for m in range(M)]).astype(np.float16)
    want = O.fp8_encode(kn.astype(np.float32)).transpose(1, 0, 2)        # [HK, M, HD]
    got = kcs[0].cpu().numpy()[0, :, :M]
    dlt = got.astype(np.int32) - want.astype(np.int32)
    assert (dlt != 0).mean() <= 0.05 and np.abs(dlt).max() <= 1
    decode.clear_contexts()
