"""GPU parity of the norm / RoPE / FP8-KV-write ops and of the fused_ops and
int4_hip.dbg_* drop-ins against the CPU oracle.  fp16 outputs: within 2 fp16
ulps of the oracle (both compute in fp32 with a single rounding; only the
sum-of-squares order differs).  V cache bytes: bit-exact.  K cache bytes: the
encoder input is a computed fp32, so a value within an ulp of a rounding edge
may land one code away: at most 0.1 % of bytes, each off by one code."""
import numpy as np
import pytest
import torch

import r4q_oracle as O
from test_gpu_gemv import cuda

pytestmark = pytest.mark.gpu


def ulp_close(got, ref, ulps=2):
    got = np.asarray(got, np.float16).astype(np.float64)
    ref = np.asarray(ref, np.float16).astype(np.float64)
    tol = ulps * np.maximum(np.abs(ref), 2.0 ** -14) * 2.0 ** -10
    bad = np.abs(got - ref) > tol
    assert not bad.any(), (np.argwhere(bad)[:5], got[bad][:5], ref[bad][:5])


def kv_bytes_close(got, ref):
    got = np.asarray(got, np.int32)
    ref = np.asarray(ref, np.int32)
    diff = got != ref
    assert diff.mean() <= 1e-3, diff.mean()
    if diff.any():
        assert np.abs(got[diff] - ref[diff]).max() == 1


@pytest.mark.parametrize("rows,D", [(1, 5120), (4, 5120), (3, 17408), (2, 128)])
def test_rmsnorm_rows(rows, D):
    from r4q import ops
    rng = np.random.default_rng(rows + D)
    x = (rng.standard_normal((rows, D)) * 3).astype(np.float16)
    w = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    ulp_close(ops.rmsnorm(cuda(x), cuda(w), 1e-6).cpu().numpy(), O.rmsnorm(x, w, 1e-6))


def test_dbg_rmsnorm_and_fused_res_norm():
    import int4_hip
    rng = np.random.default_rng(1)
    D = 5120
    x = rng.standard_normal(D).astype(np.float16)
    r = rng.standard_normal(D).astype(np.float16)
    w = (1 + 0.01 * rng.standard_normal(D)).astype(np.float16)
    ulp_close(int4_hip.dbg_rmsnorm(cuda(x), cuda(w), 1e-6).cpu().numpy(), O.rmsnorm(x[None], w, 1e-6)[0])
    y, ro = int4_hip.dbg_fused_res_norm(cuda(x), cuda(r), cuda(w), 1e-6)
    s = x.astype(np.float32) + r.astype(np.float32)          # unrounded residual (hip:818-846)
    rrms = 1.0 / np.sqrt((s.astype(np.float64) ** 2).mean() + 1e-6)
    ulp_close(y.cpu().numpy(), (s * np.float32(rrms) * w.astype(np.float32)).astype(np.float16))
    assert np.array_equal(ro.cpu().numpy().view(np.uint16), s.astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("B", [1, 3])
@pytest.mark.parametrize("scaled", [False, True])
def test_qknorm_rope_kv_write(B, scaled):
    from r4q import lib as L, ops
    rng = np.random.default_rng(7 + B + scaled)
    H, Hk, D, max_seq, pos = 40, 8, 128, 16, 5
    qkv = (rng.standard_normal((B, (H + 2 * Hk) * D)) * 2).astype(np.float16)
    qw = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    kw = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    cos, sin = O.rope_tables(D, 64, 1e6)
    kc = np.full((B, Hk, max_seq, D), 0x55, np.uint8)
    vc = np.full((B, Hk, max_seq, D), 0x66, np.uint8)
    ks = (rng.random((B, Hk)) * 0.5 + 0.05).astype(np.float32) if scaled else None
    vs = (rng.random((B, Hk)) * 0.5 + 0.05).astype(np.float32) if scaled else None
    t_qkv, t_kc, t_vc = cuda(qkv), cuda(kc), cuda(vc)
    base = t_qkv
    q, k, v = base, base[:, H * D:], base[:, (H + Hk) * D:]
    ops.head_norm_rope(q, k, v=v, q_w=cuda(qw), k_w=cuda(kw), cos=cuda(cos), sin=cuda(sin),
                       pos=pos, q_out=q, k_out=k, k_cache=t_kc, v_cache=t_vc,
                       k_scale=None if ks is None else cuda(ks),
                       v_scale=None if vs is None else cuda(vs), B=B, H=H, Hk=Hk, D=D,
                       eps=1e-6, flags=L.HEAD_NORM | L.HEAD_ROPE | L.HEAD_KV)
    out = t_qkv.cpu().numpy()
    qo, ko, kb, vb = O.qknorm_rope_kv(qkv[:, :H * D].reshape(B, H, D),
                                      qkv[:, H * D:(H + Hk) * D].reshape(B, Hk, D),
                                      qkv[:, (H + Hk) * D:].reshape(B, Hk, D), qw, kw, cos[pos],
                                      sin[pos], 1e-6, None if ks is None else (ks, vs))
    ulp_close(out[:, :H * D].reshape(B, H, D), qo)
    ulp_close(out[:, H * D:(H + Hk) * D].reshape(B, Hk, D), ko)
    assert np.array_equal(out[:, (H + Hk) * D:], qkv[:, (H + Hk) * D:])   # V untouched
    got_k, got_v = t_kc.cpu().numpy(), t_vc.cpu().numpy()
    kv_bytes_close(got_k[:, :, pos], kb)
    assert np.array_equal(got_v[:, :, pos], vb)
    other = [i for i in range(max_seq) if i != pos]
    assert (got_k[:, :, other] == 0x55).all() and (got_v[:, :, other] == 0x66).all()


def test_fused_ops_dropins():
    import fused_ops
    rng = np.random.default_rng(3)
    H, Hk, D = 40, 8, 128
    cos, sin = O.rope_tables(D, 300, 1e6)
    q = rng.standard_normal((1, H, 1, D)).astype(np.float16)
    k = rng.standard_normal((1, Hk, 1, D)).astype(np.float16)
    qw = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    kw = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    x = rng.standard_normal((3, 5120)).astype(np.float16)
    w = (1 + 0.1 * rng.standard_normal(5120)).astype(np.float16)
    ulp_close(fused_ops.fused_rmsnorm(cuda(x), cuda(w)).cpu().numpy(), O.rmsnorm(x, w, 1e-6))
    for position in (123, torch.tensor([123], device="cuda")):
        qo, ko = fused_ops.fused_qknorm_rope_decode(cuda(q), cuda(k), cuda(qw), cuda(kw), cuda(cos),
                                                    cuda(sin), position)
        ulp_close(qo.cpu().numpy()[0, :, 0], O.head_norm_rope(q[0, :, 0], qw, cos[123], sin[123], 1e-6))
        ulp_close(ko.cpu().numpy()[0, :, 0], O.head_norm_rope(k[0, :, 0], kw, cos[123], sin[123], 1e-6))
        qo, ko = fused_ops.fused_rope_decode(cuda(q), cuda(k), cuda(cos), cuda(sin), position)
        ulp_close(qo.cpu().numpy()[0, :, 0], O.rope_only(q[0, :, 0], cos[123], sin[123]))
        ulp_close(ko.cpu().numpy()[0, :, 0], O.rope_only(k[0, :, 0], cos[123], sin[123]))


def test_dbg_head_ops():
    import int4_hip
    rng = np.random.default_rng(4)
    H, Hk, D = 40, 8, 128
    q = rng.standard_normal(H * D).astype(np.float16)
    k = rng.standard_normal(Hk * D).astype(np.float16)
    qw = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    kw = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    qo, ko = int4_hip.dbg_head_rmsnorm(cuda(q), cuda(k), cuda(qw), cuda(kw), H, Hk, D, 1e-6)
    ulp_close(qo.cpu().numpy(), O.rmsnorm(q.reshape(H, D), qw, 1e-6).reshape(-1))
    ulp_close(ko.cpu().numpy(), O.rmsnorm(k.reshape(Hk, D), kw, 1e-6).reshape(-1))
    cos, sin = O.rope_tables(D, 20, 1e6)
    qo, ko = int4_hip.dbg_rope(cuda(q), cuda(k), cuda(cos[17]), cuda(sin[17]), H, Hk, D)
    ulp_close(qo.cpu().numpy(), O.rope_only(q.reshape(H, D), cos[17], sin[17]).reshape(-1))
    ulp_close(ko.cpu().numpy(), O.rope_only(k.reshape(Hk, D), cos[17], sin[17]).reshape(-1))
