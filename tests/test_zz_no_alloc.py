"""The allocation-free INT4 GEMV entry point (r4q_gemv_int4_noalloc).

It exists for callers that cannot allocate device memory — code inside a stream
capture that must not allocate, or a plugin whose host process owns the device
allocator.  It must give the same results as r4q_gemv_int4 with a workspace, on
repeated calls (its static scratch keeps the previous call's contents), and refuse
sizes beyond its fixed scratch.  This file is collected last on purpose."""
import ctypes

import numpy as np
import pytest
import torch

import r4q_oracle as O
from test_gpu_gemv import TOL, close, cuda, make_int4

pytestmark = pytest.mark.gpu


def _noalloc(x, w, s, N, K, prologue=0):
    from r4q import lib as L
    B = x.shape[0]
    y = torch.empty(B, N, dtype=torch.float16, device=x.device)
    st = L.LIB.r4q_gemv_int4_noalloc(x.data_ptr(), x.stride(0) if B > 1 else K, w.data_ptr(),
                                     s.data_ptr(), y.data_ptr(), N if B == 1 else y.stride(0),
                                     B, N, K, prologue,
                                     torch.cuda.current_stream().cuda_stream)
    assert st == 0, L.last_error()
    return y


# The scratch holds 4 MiB of fp32 partials + the counters: the same byte count
# given to r4q_gemv_int4 as its workspace makes both entry points plan the
# same K split, so their outputs must then be equal bit for bit.
NOALLOC_WS_BYTES = 256 + 64 * 1024 + 4 * 1024 * 1024


def _with_workspace(x, w, s, N, K, prologue, ws_bytes):
    from r4q import lib as L
    B = x.shape[0]
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=x.device)
    y = torch.empty(B, N, dtype=torch.float16, device=x.device)
    L.call("r4q_gemv_int4", x.data_ptr(), x.stride(0) if B > 1 else K, w.data_ptr(), s.data_ptr(),
           y.data_ptr(), N if B == 1 else y.stride(0), B, N, K, prologue, ws.data_ptr(), ws_bytes,
           torch.cuda.current_stream().cuda_stream)
    return y


# (N, K, B): small and split-K shapes, a batch above 8, B * N close to the
# limit (16 x 32768 = the limit: the partials of a two-way split fill the scratch) and
# B * N exactly at the limit (2 x 262144, the largest N a GEMV takes).
@pytest.mark.parametrize("N,K,B", [(1024, 5120, 1), (1024, 5120, 4), (5120, 17408, 1), (7168, 5120, 16),
                                   (32768, 2048, 16), (262144, 128, 2)])
def test_noalloc_matches_workspace_entry_point(N, K, B):
    from r4q import lib as L, ops
    rng = np.random.default_rng(N + K + B)
    packed, sz = make_int4(rng, N, K, outliers=N * K <= 1 << 27)
    x = cuda(rng.standard_normal((B, K)).astype(np.float16))
    w, s = cuda(packed), cuda(sz)
    ref = ops.gemv('int4', x, w, s, N, K, prologue=L.PRO_FWHT).cpu().numpy()
    same_plan = _with_workspace(x, w, s, N, K, L.PRO_FWHT, NOALLOC_WS_BYTES)
    for _ in range(2):                       # two calls in a row share the scratch
        y = _noalloc(x, w, s, N, K, prologue=L.PRO_FWHT)
        torch.cuda.synchronize()
        assert torch.equal(y, same_plan)
        close(y.cpu().numpy(), ref, TOL)
    ops.check_status(x.device)               # includes the static scratch's status word
    if N * K <= 1 << 26:
        close(y.cpu().numpy(), O.gemv_int4(O.fwht32(x.cpu().numpy().astype(np.float32)).astype(np.float16),
                                           packed, sz), TOL)


def test_noalloc_rejects_sizes_beyond_scratch():
    from r4q import lib as L
    fake = ctypes.c_void_p(256)
    st = L.LIB.r4q_gemv_int4_noalloc(fake, 5120, fake, fake, fake, 65536, 16, 65536, 5120, 0, None)
    assert st == -3
    assert "static scratch" in L.last_error()
