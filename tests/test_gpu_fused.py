"""GPU parity of the GEMV fusions that replace fused_res_norm_fwht /
fused_rmsnorm_fwht (int4_decode_step.hip:1143-1237): the residual epilogue
with per-tile sums of squares feeding the RMSNorm+FWHT prologue of the next
GEMV.  Tolerance 1e-3 relative (see test_gpu_gemv.close)."""
import numpy as np
import pytest
import torch

import r4q_oracle as O
from test_gpu_gemv import close, cuda, make_int4

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B", [1, 4, 16])
def test_rmsnorm_prologue_from_x(B):
    from r4q import lib as L, ops
    rng = np.random.default_rng(21 + B)
    N, K = 2048, 5120
    packed, sz = make_int4(rng, N, K)
    x = (rng.standard_normal((B, K)) * 3).astype(np.float16)
    nw = (1 + 0.01 * rng.standard_normal(K)).astype(np.float16)
    y = ops.gemv('int4', cuda(x), cuda(packed), cuda(sz), N, K, prologue=L.PRO_RMSNORM_FWHT,
                 norm_w=cuda(nw), eps=1e-6).cpu().numpy()
    close(y, O.gemv_int4(O.rmsnorm_fwht(x, nw, 1e-6), packed, sz))


@pytest.mark.parametrize("B", [1, 16])
@pytest.mark.parametrize("Kin", [5120, 17408])
def test_residual_epilogue_then_norm_prologue(B, Kin):
    """o = W_o x ; r = o + h (epilogue, + ss partials) ; gu = W_gu FWHT(norm(r))."""
    from r4q import lib as L, ops
    rng = np.random.default_rng(B + Kin)
    D, N2 = 5120, 4096
    po, so = make_int4(rng, D, Kin)
    pg, sg = make_int4(rng, N2, D)
    x = rng.standard_normal((B, Kin)).astype(np.float16)
    h = (rng.standard_normal((B, D)) * 4).astype(np.float16)
    nw = (1 + 0.01 * rng.standard_normal(D)).astype(np.float16)
    r = torch.empty(B, D, dtype=torch.float16, device='cuda')
    ss = torch.zeros(D // 16, B, dtype=torch.float32, device='cuda')
    ops.gemv('int4', cuda(x), cuda(po), cuda(so), D, Kin, out=r, residual=cuda(h), ss_out=ss)
    gu = ops.gemv('int4', r, cuda(pg), cuda(sg), N2, D, prologue=L.PRO_RMSNORM_FWHT,
                  norm_w=cuda(nw), eps=1e-6, ss_in=ss)
    o_ref = O.gemv_int4(x, po, so)
    rot_ref, r_ref = O.res_norm_fwht(o_ref, h, nw, 1e-6)
    close(r.cpu().numpy(), r_ref)
    ssr = ((o_ref.astype(np.float32) + h.astype(np.float32)).astype(np.float64) ** 2).sum(1)
    got = ss.cpu().numpy().astype(np.float64).sum(0)
    assert np.allclose(got, ssr, rtol=2e-3)
    close(gu.cpu().numpy(), O.gemv_int4(rot_ref, pg, sg))


def test_residual_epilogue_aliasing_in_place():
    """y may alias the residual (h <- down(x) + h)."""
    from r4q import ops
    rng = np.random.default_rng(77)
    D, K = 5120, 17408
    p, s = make_int4(rng, D, K)
    x = rng.standard_normal((1, K)).astype(np.float16)
    h = rng.standard_normal((1, D)).astype(np.float16)
    ht = cuda(h)
    ops.gemv('int4', cuda(x), cuda(p), cuda(s), D, K, out=ht, residual=ht)
    ref = (O.gemv_int4(x, p, s).astype(np.float32) + h.astype(np.float32)).astype(np.float16)
    close(ht.cpu().numpy(), ref)


@pytest.mark.parametrize("fmt", ['int4', 'int8'])
@pytest.mark.parametrize("B,N,K", [(1, 5120, 640), (1, 5120, 2176), (2, 5120, 17408), (4, 1024, 5120),
                                   (16, 5120, 2048)])
def test_fp32_partial_output(fmt, B, N, K):
    """fp32 output (tensor-parallel partial): fp16(y32) equals the fp16 output
    bit for bit on every path (direct and split-K merge), including the
    o_proj / down_proj column-shard widths of TP=8 (640, 2176)."""
    from r4q import ops
    rng = np.random.default_rng(B * 7 + K)
    x = rng.standard_normal((B, K)).astype(np.float16)
    if fmt == 'int4':
        w, s = make_int4(rng, N, K)
    else:
        q, s = O.quantize_int8_sym((rng.standard_normal((N, K)) * 0.05).reshape(N, K // 32, 32))
        w = q.reshape(N, K)
    y16 = ops.gemv(fmt, cuda(x), cuda(w), cuda(s), N, K)
    y32 = ops.gemv(fmt, cuda(x), cuda(w), cuda(s), N, K, out32=torch.empty(B, N, device='cuda'))
    assert y32.dtype == torch.float32
    assert torch.equal(y32.half(), y16)
    ref = O.linear(x, (fmt, w, s), acc=True)
    close(y32.cpu().numpy(), ref)
