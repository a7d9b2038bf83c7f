"""Parity of one decode layer at the full Qwen3-14B shape (hidden 5120, 40 query
/ 8 KV heads of 128, intermediate 17408) plus the final norm and the fp16
lm_head (vocabulary 151936), kernel by kernel against the CPU oracle.

Every kernel of the decode step is called through the same entry points the
decode context uses, in the same order, and each output is compared with the
oracle evaluated on the GPU's own inputs for that kernel, so each comparison
isolates one kernel:

  qkv GEMV (RMSNorm+FWHT prologue)      <= 1e-3 relative
  head norm + RoPE + FP8 K/V write       bytes equal (<= 1 code on 0.1 %)
  attention over the cache (+ FWHT)      <= 1e-3
  o GEMV + residual (r, sums of squares) <= 1e-3
  gate_up GEMV (RMSNorm+FWHT from them)  <= 1e-3
  down GEMV (SiLU*up+FWHT) + residual    <= 1e-3
  lm_head (final RMSNorm+FWHT, fp16 W)   <= 1e-3

Relative error is max |y - ref| / max |ref| and ||y - ref|| / ||ref||.  The
INT4 GEMVs at B <= 2 compute the reference decode kernel's blockwise
arithmetic (per-block fp32 dot times scale), so the oracle runs in that mode;
at B > 2 they use the exact fp16 dequantised weights (the reference's Python
path), the oracle's 'dequant' mode.  Weights are generated on the GPU (seeded
synthetic data in the reference's quantized layout) and copied to the host
for the oracle."""
import numpy as np
import pytest
import torch

import r4q_oracle as O
from test_gpu_gemv import close

pytestmark = pytest.mark.gpu
D, I, H, HK, HD, V = 5120, 17408, 40, 8, 128, 151936
EPS = 1e-6
TOL = 1e-3
CTX = 96


def _np(t):
    return t.cpu().numpy()


def _layer(fmt, dev, seed):
    from r4q import synth
    g = torch.Generator(device=dev).manual_seed(seed)
    mk = synth.linear_int4 if fmt == 'int4' else synth.linear_int8
    shapes = {'qkv': ((H + 2 * HK) * HD, D), 'o': (D, H * HD), 'gate_up': (2 * I, D), 'down': (D, I)}
    ly = {k: mk(N, K, g, dev) for k, (N, K) in shapes.items()}
    for k, n in (('in_norm', D), ('post_norm', D), ('q_norm', HD), ('k_norm', HD)):
        ly[k] = (1 + 0.05 * torch.randn(n, generator=g, device=dev)).half()
    return ly


def _host(lin):
    return tuple([lin[0]] + [_np(a) for a in lin[1:]])


def _oracle_lin(x, lin):
    return O.linear(x, lin)


def _fp16_gemv_chunked(x, w_dev, chunk=16384):
    """fp16-weight GEMV oracle (float64 accumulate) over row chunks of a
    device weight (the full lm_head in float64 would need 6 GB)."""
    out = []
    for r0 in range(0, w_dev.shape[0], chunk):
        out.append(O.gemv_fp16(x, _np(w_dev[r0:r0 + chunk]), acc=True))
    return np.concatenate(out, axis=1).astype(np.float16)


@pytest.mark.parametrize("fmt,B,with_lm", [('int4', 1, True), ('int4', 4, False), ('int8', 1, False)])
def test_full_shape_layer_kernel_by_kernel(fmt, B, with_lm):
    from r4q import lib as L, ops
    dev = torch.device("cuda", 0)
    O.INT4_MODE['mode'] = 'blockwise' if B <= 2 else 'dequant'
    ly = _layer(fmt, dev, seed=101 + B)
    hl = {k: _host(ly[k]) for k in ('qkv', 'o', 'gate_up', 'down')}
    g = torch.Generator(device=dev).manual_seed(7)
    h = (0.5 * torch.randn(B, D, generator=g, device=dev)).half()
    kc = ops.fp16_to_fp8(torch.randn(B, HK, CTX + 8, HD, generator=g, device=dev).half())
    vc = ops.fp16_to_fp8(torch.randn(B, HK, CTX + 8, HD, generator=g, device=dev).half())
    cos_np, sin_np = O.rope_tables(HD, CTX + 8, 1e6)
    cos, sin = torch.from_numpy(cos_np).to(dev), torch.from_numpy(sin_np).to(dev)
    pos = CTX
    kc0, vc0 = _np(kc), _np(vc)

    # qkv: RMSNorm + FWHT prologue (sums of squares computed from x)
    qkv = ops.gemv(fmt, h, ly['qkv'][1], ly['qkv'][2], (H + 2 * HK) * HD, D, prologue=L.PRO_RMSNORM_FWHT,
                   norm_w=ly['in_norm'], eps=EPS)
    rot = O.rmsnorm_fwht(_np(h), _np(ly['in_norm']), EPS)
    close(_np(qkv), _oracle_lin(rot, hl['qkv']), TOL)

    # head norm + RoPE + K/V write + attention over [0, pos] with the FWHT epilogue
    seq = torch.full((B,), pos + 1, dtype=torch.int64, device=dev)
    att = ops.attn_decode_fused(qkv, kc, vc, ly['q_norm'], ly['k_norm'], cos, sin, H, HK, 0, fwht=True, eps=EPS,
                                seq_dev=seq)
    q_np = _np(qkv)
    qd, kd = H * HD, HK * HD
    qo, _, kb, vb = O.qknorm_rope_kv(q_np[:, :qd].reshape(B, H, HD), q_np[:, qd:qd + kd].reshape(B, HK, HD),
                                     q_np[:, qd + kd:].reshape(B, HK, HD), _np(ly['q_norm']), _np(ly['k_norm']),
                                     cos_np[pos], sin_np[pos], EPS)
    kg, vg = _np(kc), _np(vc)
    assert np.array_equal(kg[:, :, :pos], kc0[:, :, :pos]) and np.array_equal(vg[:, :, pos + 1:], vc0[:, :, pos + 1:])
    for got, want in ((kg[:, :, pos], kb), (vg[:, :, pos], vb)):
        d = got.astype(np.int32) - want.astype(np.int32)
        assert np.abs(d).max() <= 1 and (d != 0).mean() <= 1e-3
    att_ref = O.attention_decode(qo, kg, vg, pos + 1, fwht_out=True)
    close(_np(att).reshape(B, -1), att_ref.reshape(B, -1), TOL)

    # o_proj + residual epilogue: r = fp16(fp16(o) + h), sums of squares of the unrounded sum
    r = torch.empty(B, D, dtype=torch.float16, device=dev)
    ss_post = torch.zeros(D // 16, B, device=dev)
    ops.gemv(fmt, att.reshape(B, -1), ly['o'][1], ly['o'][2], D, qd, out=r, residual=h, ss_out=ss_post)
    o_ref = _oracle_lin(_np(att).reshape(B, -1), hl['o'])
    _, r_ref = O.res_norm_fwht(o_ref, _np(h), _np(ly['post_norm']), EPS)
    close(_np(r), r_ref, TOL)
    ss_ref = (_np(r).astype(np.float64) ** 2).sum(-1)
    np.testing.assert_allclose(_np(ss_post).sum(0), ss_ref, rtol=1e-3)

    # gate_up: RMSNorm + FWHT prologue from the epilogue's sums of squares
    gu = ops.gemv(fmt, r, ly['gate_up'][1], ly['gate_up'][2], 2 * I, D, prologue=L.PRO_RMSNORM_FWHT,
                  norm_w=ly['post_norm'], eps=EPS, ss_in=ss_post)
    rot_g = O.rmsnorm_fwht(_np(r), _np(ly['post_norm']), EPS)
    close(_np(gu), _oracle_lin(rot_g, hl['gate_up']), TOL)

    # down: SiLU(gate) * up + FWHT prologue, residual epilogue -> h_new
    h_new = torch.empty(B, D, dtype=torch.float16, device=dev)
    ss_h = torch.zeros(D // 16, B, device=dev)
    ops.gemv(fmt, gu, ly['down'][1], ly['down'][2], D, I, prologue=L.PRO_SILU_FWHT, out=h_new, residual=r,
             ss_out=ss_h)
    gu_np = _np(gu)
    act = O.silu_fwht(gu_np[:, :I], gu_np[:, I:])
    d_ref = _oracle_lin(act, hl['down'])
    _, h_ref = O.res_norm_fwht(d_ref, _np(r), _np(ly['in_norm']), EPS)
    close(_np(h_new), h_ref, TOL)

    if with_lm:
        # final RMSNorm + FWHT and the fp16 lm_head over the whole vocabulary
        lm_w = (0.02 * torch.randn(V, D, generator=g, device=dev)).half()
        final = (1 + 0.05 * torch.randn(D, generator=g, device=dev)).half()
        logits = ops.gemv('fp16', h_new, lm_w, None, V, D, prologue=L.PRO_RMSNORM_FWHT, norm_w=final, eps=EPS,
                          ss_in=ss_h)
        rot_f = O.rmsnorm_fwht(_np(h_new), _np(final), EPS)
        close(_np(logits), _fp16_gemv_chunked(rot_f, lm_w), TOL)
    ops.check_status(dev)
