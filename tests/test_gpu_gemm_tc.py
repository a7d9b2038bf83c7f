"""GPU: the tcgen05 prefill GEMM (r4q_gemm_fp16 / r4q_gemm_int4) against an
fp64 reference of the same fp16 operands — the reference prefill's dequantise
(bit-exact dequant_int4) then matmul.  Tolerance 1e-3 relative (max-norm and
L2) as for the GEMV; every tile edge (M, N not multiples of 128 / 256, K
multiple of 64 or, for fp16, of 8)."""
import numpy as np
import pytest
import torch

import r4q_oracle as O
from test_gpu_gemv import close, cuda, make_int4

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (1, 256, 128), (200, 300, 520), (512, 1024, 2048),
                                   (37, 5120, 5120)])
def test_gemm_fp16(M, N, K):
    from r4q import ops
    rng = np.random.default_rng(M + N + K)
    x = rng.standard_normal((M, K)).astype(np.float16)
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float16)
    y = ops.gemm(cuda(x), cuda(w)).cpu().numpy()
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    close(y, ref)


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (5, 512, 1024), (300, 1000, 5120), (512, 7168, 5120)])
def test_gemm_int4_vs_dequant_matmul(M, N, K):
    from r4q import ops
    rng = np.random.default_rng(7 * M + N + K)
    packed, sz = make_int4(rng, N, K)
    x = rng.standard_normal((M, K)).astype(np.float16)
    y = ops.gemm(cuda(x), cuda(packed), cuda(sz), N).cpu().numpy()
    W = O.dequant_int4_runtime(packed, sz).astype(np.float64)
    close(y, x.astype(np.float64) @ W.T)
    # same as the fp16 GEMM over the kernel-dequantised weights
    Wd = ops.dequant_int4(cuda(packed), cuda(sz), N, K)
    y16 = ops.gemm(cuda(x), Wd).cpu().numpy()
    assert np.array_equal(y, y16)


def test_gemm_repeat_and_status_clean():
    from r4q import ops
    rng = np.random.default_rng(3)
    x = cuda(rng.standard_normal((256, 512)).astype(np.float16))
    w = cuda((rng.standard_normal((512, 512)) * 0.05).astype(np.float16))
    a = ops.gemm(x, w)
    b = ops.gemm(x, w)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert int(ops._status_ws(x.device)[:4].view(torch.int32)[0]) == 0


@pytest.mark.parametrize("M,N,K,int4", [(64, 5120, 2048, True), (16, 2048, 4096, True), (1, 2048, 4096, False)])
def test_gemm_split_k_decode_sizes(M, N, K, int4):
    """Decode-sized M: K split over gridDim.z, fp32 partials merged by the
    tile's last CTA in split order — within tolerance of the reference,
    identical on repeat, counters left zero."""
    from r4q import ops
    from r4q import lib as Lb
    assert Lb.LIB.r4q_gemm_workspace_bytes(M, N, K) > 256          # the split path is taken
    rng = np.random.default_rng(M + K)
    x = rng.standard_normal((M, K)).astype(np.float16)
    if int4:
        packed, sz = make_int4(rng, N, K)
        W = O.dequant_int4_runtime(packed, sz).astype(np.float64)
        args = (cuda(packed), cuda(sz), N)
    else:
        w = (rng.standard_normal((N, K)) * 0.05).astype(np.float16)
        W = w.astype(np.float64)
        args = (cuda(w),)
    a = ops.gemm(cuda(x), *args)
    b = ops.gemm(cuda(x), *args)
    torch.cuda.synchronize()
    close(a.cpu().numpy(), x.astype(np.float64) @ W.T)
    assert torch.equal(a, b)
    ws = ops._status_ws(a.device)
    assert int(ws[:4].view(torch.int32)[0]) == 0
    assert int(ws[256:256 + 4096].count_nonzero()) == 0
