"""Torch-tensor front end over the C ABI: shape checks, output allocation,
per-(device, stream) GEMV workspaces.  Device memory and streams come from
PyTorch; all arithmetic runs in libr4q.so."""
from __future__ import annotations

import ctypes as C
import threading

import torch

from . import lib as L

_ws_lock = threading.Lock()
_ws: dict = {}


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_handle(dev: torch.device) -> int:
    """cudaStream_t of torch's current stream on dev (the raw-handle query
    costs a fraction of building a torch.cuda.Stream object per call)."""
    if _raw_stream is not None:
        return _raw_stream(dev.index if dev.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(dev).cuda_stream


def _require_cuda(*ts: torch.Tensor) -> torch.device:
    idx = ts[0].get_device()
    for t in ts:
        if not t.is_cuda:
            raise ValueError("r4q ops take CUDA tensors only (no CPU fallback)")
        if t.get_device() != idx:
            raise ValueError("all tensors must be on the same device")
    return ts[0].device


# Workspaces replaced by larger ones stay referenced: a CUDA graph captured
# earlier may still use them.
_retired: list = []


def _grown(cache: dict, key, need: int, minimum: int, dev) -> torch.Tensor:
    """The cached zero-filled uint8 workspace for key, replaced by a larger one
    when it holds fewer than `need` bytes (call with _ws_lock held)."""
    cur = cache.get(key)
    if cur is None or cur.numel() < need:
        if cur is not None:
            _retired.append(cur)
        cur = torch.zeros(max(need, minimum), dtype=torch.uint8, device=dev)
        cache[key] = cur
    return cur


def gemv_workspace(dev: torch.device, B: int, N: int, K: int, stream: int | None = None) -> torch.Tensor:
    """Zero-filled workspace for GEMV split-K partials, cached per
    (device, stream).  The kernels leave it zeroed after every call."""
    need = int(L.LIB.r4q_gemv_workspace_bytes(B, N, K))
    key = (dev.index, stream_handle(dev) if stream is None else stream)
    cur = _ws.get(key)          # lock-free hit; replacement happens under the lock
    if cur is not None and cur.numel() >= need:
        return cur
    with _ws_lock:
        return _grown(_ws, key, need, 1 << 20, dev)


def check_status(dev: torch.device | int | None = None, clear: bool = True) -> None:
    """Raise ``R4QError`` (code R4Q_ERR_TIMEOUT) if a bounded device-side wait
    of a GEMV, GEMM or attention kernel gave up since the last check on this
    device: the outputs of those kernels are then not valid.  Reads the status
    word of every workspace these wrappers hold for the device, and of the
    allocation-free GEMV's static scratch (synchronises each stream)."""
    if dev is None:
        dev = torch.cuda.current_device()
    idx = dev if isinstance(dev, int) else (dev.index if dev.index is not None else torch.cuda.current_device())
    with _ws_lock:
        items = [(k, t) for cache in (_ws, _gws, _aws) for k, t in cache.items() if k[0] == idx]
    err = None
    with torch.cuda.device(idx):
        for (_, stream), t in items:
            st = L.LIB.r4q_ws_status(t.data_ptr(), 1 if clear else 0, stream)
            if st != 0 and err is None:
                err = L.R4QError(st, "r4q_ws_status", L.last_error())
        st = L.LIB.r4q_ws_status(None, 1 if clear else 0, None)
        if st != 0 and err is None:
            err = L.R4QError(st, "r4q_ws_status(noalloc scratch)", L.last_error())
    if err is not None:
        raise err


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_FMT = {'int4': L.W_INT4, 'int8': L.W_INT8, 'fp16': L.W_FP16}


def gemv(fmt: str, x: torch.Tensor, w: torch.Tensor, s: torch.Tensor | None, N: int, K: int,
         prologue: int = L.PRO_NONE, out: torch.Tensor | None = None, *,
         norm_w: torch.Tensor | None = None, eps: float = 1e-6,
         ss_in: torch.Tensor | None = None, residual: torch.Tensor | None = None,
         ss_out: torch.Tensor | None = None, out32: torch.Tensor | None = None) -> torch.Tensor:
    """y[B, N] = prologue(x)[B, K] @ dequant(W)^T for fmt in {'int4','int8','fp16'}.

    Optional fusions: RMSNorm prologue (``prologue=PRO_RMSNORM_FWHT`` with
    ``norm_w`` and, optionally, ``ss_in`` partial sums of squares [P, B]);
    residual epilogue y = fp16(fp16(acc) + residual) with ``ss_out`` [N/16, B]
    receiving the sums of squares of the unrounded sums.  ``out32`` (fp32 [B, N]):
    write the unrounded fp32 sums there instead (no fp16 output, no residual)."""
    dev = _require_cuda(x, w)
    if x.dtype != torch.float16:
        raise TypeError("x must be float16")
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    B = x2.shape[0]
    kin = 2 * K if prologue == L.PRO_SILU_FWHT else K
    if x2.shape[1] < kin:
        raise ValueError(f"x has {x2.shape[1]} columns, need {kin}")
    if out is None and out32 is None:
        out = torch.empty(B, N, dtype=torch.float16, device=dev)
    st = stream_handle(dev)
    ws = gemv_workspace(dev, B, N, K, st)
    ldx = x2.stride(0) if B > 1 else kin
    yt = out if out32 is None else out32
    ldy = yt.stride(0) if B > 1 else N
    fused = None
    if (norm_w is not None or residual is not None or ss_out is not None or ss_in is not None
            or out32 is not None):
        if residual is not None:
            residual = residual.reshape(B, -1)
        fused = L.GemvFused(
            norm_w=_ptr(norm_w), eps=float(eps), ss_in=_ptr(ss_in),
            ss_in_parts=0 if ss_in is None else int(ss_in.shape[0]),
            residual=_ptr(residual), ldres=N if residual is None else residual.stride(0),
            ss_out=_ptr(ss_out), y32=_ptr(out32))
    L.call("r4q_gemv", _FMT[fmt], x2.data_ptr(), ldx, w.data_ptr(), _ptr(s), _ptr(out), ldy,
           B, N, K, prologue, None if fused is None else C.byref(fused), ws.data_ptr(), ws.numel(),
           st)
    return out if out32 is None else out32


def dequant_int4(packed: torch.Tensor, sz: torch.Tensor, N: int, K: int,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    dev = _require_cuda(packed, sz)
    out = out if out is not None else torch.empty(N, K, dtype=torch.float16, device=dev)
    L.call("r4q_dequant_int4", packed.data_ptr(), sz.data_ptr(), out.data_ptr(), N, K,
           stream_handle(dev))
    return out


def fp16_to_fp8(src: torch.Tensor) -> torch.Tensor:
    dev = _require_cuda(src)
    s = src.contiguous()
    out = torch.empty(s.shape, dtype=torch.uint8, device=dev)
    L.call("r4q_fp16_to_fp8", s.data_ptr(), out.data_ptr(), s.numel(), stream_handle(dev))
    return out


def fp8_to_fp32(src: torch.Tensor) -> torch.Tensor:
    dev = _require_cuda(src)
    s = src.contiguous()
    out = torch.empty(s.shape, dtype=torch.float32, device=dev)
    L.call("r4q_fp8_to_fp32", s.data_ptr(), out.data_ptr(), s.numel(), stream_handle(dev))
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6, res: torch.Tensor | None = None,
            want_res: bool = False):
    """y = fp16(v * rsqrt(mean(v^2) + eps) * w), v = x (+ res) over the last axis."""
    dev = _require_cuda(x, w)
    D = x.shape[-1]
    x2 = x.reshape(-1, D).contiguous()
    r2 = None if res is None else res.reshape(-1, D).contiguous()
    y = torch.empty_like(x2)
    ro = torch.empty_like(x2) if want_res else None
    L.call("r4q_rmsnorm", x2.data_ptr(), _ptr(r2), w.data_ptr(), y.data_ptr(), _ptr(ro),
           x2.shape[0], D, D, float(eps), stream_handle(dev))
    y = y.reshape(x.shape)
    return (y, ro.reshape(x.shape)) if want_res else y


def head_norm_rope(q, k, *, v=None, q_w=None, k_w=None, cos=None, sin=None, pos=0,
                   pos_dev=None, q_out=None, k_out=None, k_cache=None, v_cache=None,
                   k_scale=None, v_scale=None, B=1, H=0, Hk=0, D=128, ld_in=None, ld_out=None,
                   eps=1e-6, flags=0):
    """Per-head norm / RoPE / FP8 KV write (r4q_head_norm_rope); tensors as described
    in include/r4q.h.  Outputs are written in place into q_out / k_out."""
    dev = _require_cuda(q if q is not None else k)
    max_seq = 0 if k_cache is None else int(k_cache.shape[-2])
    L.call("r4q_head_norm_rope", _ptr(q), _ptr(k), _ptr(v), _ptr(q_w), _ptr(k_w), _ptr(cos),
           _ptr(sin), 0 if cos is None else cos.stride(0), int(pos), _ptr(pos_dev), _ptr(q_out),
           _ptr(k_out), _ptr(k_cache), _ptr(v_cache), _ptr(k_scale), _ptr(v_scale), B, H, Hk, D,
           ld_in if ld_in is not None else (H + 2 * Hk) * D,
           ld_out if ld_out is not None else (H + 2 * Hk) * D,
           max_seq, float(eps), flags, stream_handle(dev))


_aws: dict = {}


def attn_workspace(dev: torch.device, B: int, H: int, Hk: int, max_seq: int) -> torch.Tensor:
    need = int(L.LIB.r4q_flash_decode_workspace_bytes(B, H, Hk, max_seq))
    key = (dev.index, stream_handle(dev))
    with _ws_lock:
        return _grown(_aws, key, need, 1 << 16, dev)


def flash_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, seq_len: int,
                 *, k_scale=None, v_scale=None, fwht: bool = False, out=None, seq_dev=None):
    """q fp16 [B, H, 128]; caches uint8 [B, Hk, max_seq, 128] -> o fp16 [B, H, 128]."""
    dev = _require_cuda(q, k_cache, v_cache)
    B, H, D = q.shape
    Hk, max_seq = k_cache.shape[1], k_cache.shape[2]
    q2 = q.reshape(B, H * D).contiguous()
    o = out if out is not None else torch.empty(B, H, D, dtype=torch.float16, device=dev)
    ws = attn_workspace(dev, B, H, Hk, max_seq)
    L.call("r4q_flash_decode", q2.data_ptr(), H * D, k_cache.data_ptr(), v_cache.data_ptr(),
           _ptr(k_scale), _ptr(v_scale), o.data_ptr(), H * D, B, H, Hk, D, max_seq, int(seq_len),
           _ptr(seq_dev), L.ATTN_FWHT if fwht else 0, ws.data_ptr(), ws.numel(),
           stream_handle(dev))
    return o


def attn_decode_fused(qkv, k_cache, v_cache, q_w, k_w, cos, sin, H, Hk, seq_len, *, k_scale=None,
                      v_scale=None, fwht=False, eps=1e-6, out=None, seq_dev=None):
    """Head norm + RoPE + FP8 KV write of the new token and attention in one
    launch (r4q_attn_decode_fused).  qkv fp16 [B, (H + 2 Hk) * 128]; caches
    uint8 [B, Hk, max_seq, 128] (row seq_len - 1 is written) -> o [B, H, 128]."""
    dev = _require_cuda(qkv, k_cache, v_cache)
    B = qkv.shape[0]
    D = 128
    max_seq = int(k_cache.shape[2])
    o = out if out is not None else torch.empty(B, H, D, dtype=torch.float16, device=dev)
    ws = attn_workspace(dev, B, H, Hk, max_seq)
    L.call("r4q_attn_decode_fused", qkv.data_ptr(), qkv.stride(0), q_w.data_ptr(), k_w.data_ptr(),
           cos.data_ptr(), sin.data_ptr(), cos.stride(0), float(eps), k_cache.data_ptr(), v_cache.data_ptr(),
           _ptr(k_scale), _ptr(v_scale), o.data_ptr(), H * D, B, H, Hk, D, max_seq, int(seq_len),
           _ptr(seq_dev), L.ATTN_FWHT if fwht else 0, ws.data_ptr(), ws.numel(), stream_handle(dev))
    return o


_gws: dict = {}


def _status_ws(dev, nbytes: int = 256):
    """Per (device, stream) GEMM workspace (status word, split counters, fp32
    partials), zeroed once and grown on demand; the kernels leave it zero.
    Grow it outside graph capture (a warm-up call at the same shape)."""
    key = (dev.index, stream_handle(dev))
    with _ws_lock:
        return _grown(_gws, key, nbytes, 256, dev)


def gemm(x: torch.Tensor, w: torch.Tensor, s: torch.Tensor | None = None, N: int | None = None,
         out: torch.Tensor | None = None) -> torch.Tensor:
    """y[M, N] = x[M, K] @ W[N, K]^T on the tcgen05 tensor cores.  W is fp16
    [N, K], or INT4 nibbles [N, K/2] with (scale, zero) pairs ``s`` [N, K/16]
    (dequantised in the kernel, bit-exact to dequant_int4)."""
    dev = _require_cuda(x, w)
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    M, K = x2.shape
    N = int(w.shape[0]) if N is None else N
    y = out if out is not None else torch.empty(M, N, dtype=torch.float16, device=dev)
    ws = _status_ws(dev, int(L.LIB.r4q_gemm_workspace_bytes(M, N, K)))
    st = stream_handle(dev)
    if s is None:
        L.call("r4q_gemm_fp16", x2.data_ptr(), x2.stride(0), w.data_ptr(), y.data_ptr(), y.stride(0), M, N, K,
               ws.data_ptr(), ws.numel(), st)
    else:
        L.call("r4q_gemm_int4", x2.data_ptr(), x2.stride(0), w.data_ptr(), s.data_ptr(), y.data_ptr(),
               y.stride(0), M, N, K, ws.data_ptr(), ws.numel(), st)
    return y


def fwht_rows(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """fp16(H32 x) on every 32-element block of each row (hadamard_rotate_batched)."""
    dev = _require_cuda(x)
    x2 = x.reshape(-1, x.shape[-1])
    y = out if out is not None else torch.empty_like(x2)
    L.call("r4q_fwht_rows", x2.data_ptr(), x2.stride(0), y.data_ptr(), y.stride(0), x2.shape[0], x2.shape[1],
           stream_handle(dev))
    return y


def silu_mul(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """fp16(silu(x[:, :I]) * x[:, I:]) (silu_mul_batched)."""
    dev = _require_cuda(x)
    I = x.shape[-1] // 2
    y = out if out is not None else torch.empty(x.shape[0], I, dtype=torch.float16, device=dev)
    L.call("r4q_silu_mul", x.data_ptr(), x.stride(0), y.data_ptr(), y.stride(0), x.shape[0], I,
           stream_handle(dev))
    return y


def dequant_int8(w: torch.Tensor, s: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    dev = _require_cuda(w, s)
    N, K = w.shape
    y = out if out is not None else torch.empty(N, K, dtype=torch.float16, device=dev)
    L.call("r4q_dequant_int8", w.data_ptr(), s.data_ptr(), y.data_ptr(), N, K, stream_handle(dev))
    return y


class MoeRouteBuffers:
    """Device buffers of one routing: ids, wts and the grouping by expert."""

    def __init__(self, B: int, E: int, topk: int, dev, e_lo: int = 0, e_hi: int | None = None):
        i32 = dict(dtype=torch.int32, device=dev)
        self.B, self.E, self.topk = B, E, topk
        self.e_lo, self.e_hi = e_lo, (E if e_hi is None else e_hi)
        self.ids = torch.empty(B, topk, **i32)
        self.wts = torch.empty(B, topk, dtype=torch.float32, device=dev)
        self.counts = torch.empty(E, **i32)
        self.offsets = torch.empty(E + 1, **i32)
        self.list = torch.empty(B * topk, **i32)
        self.active = torch.empty(E, **i32)
        self.n_active = torch.empty(1, **i32)
        self.done = torch.zeros(1, **i32)          # CTA counter of the fused router (kept zero between calls)
        self.status = torch.zeros(1, **i32)        # set by a kernel whose bounded wait gave up


def moe_route(logits: torch.Tensor, topk: int, rb: MoeRouteBuffers | None = None) -> MoeRouteBuffers:
    dev = _require_cuda(logits)
    B, E = logits.shape
    rb = rb if rb is not None else MoeRouteBuffers(B, E, topk, dev)
    L.call("r4q_moe_route", logits.data_ptr(), B, E, topk, rb.e_lo, rb.e_hi, rb.ids.data_ptr(), rb.wts.data_ptr(),
           rb.counts.data_ptr(), rb.offsets.data_ptr(), rb.list.data_ptr(), rb.active.data_ptr(),
           rb.n_active.data_ptr(), stream_handle(dev))
    return rb


def moe_router(xn: torch.Tensor, router_w: torch.Tensor, topk: int, rb: MoeRouteBuffers,
               logits: torch.Tensor | None = None, x: torch.Tensor | None = None, ss_in: torch.Tensor | None = None,
               norm_w: torch.Tensor | None = None, eps: float = 1e-6) -> torch.Tensor:
    """Fused router (r4q_moe_router): with x / ss_in / norm_w, xn is written
    as fp16(H32(RMSNorm(x))); otherwise xn is the given normalised input.
    Router logits fp16 [B, E] go to ``logits`` (returned) and the routing to rb."""
    dev = _require_cuda(xn, router_w)
    B, D = xn.shape
    E = router_w.shape[0]
    lg = logits if logits is not None else torch.empty(B, E, dtype=torch.float16, device=dev)
    if norm_w is not None and (x is None or ss_in is None):
        raise ValueError("moe_router: the fused norm needs x and ss_in")
    L.call("r4q_moe_router", _ptr(x), _ptr(ss_in), 0 if ss_in is None else int(ss_in.shape[0]), _ptr(norm_w),
           float(eps), xn.data_ptr(), router_w.data_ptr(), lg.data_ptr(), B, D, E, topk, rb.e_lo, rb.e_hi,
           rb.ids.data_ptr(), rb.wts.data_ptr(), rb.counts.data_ptr(), rb.offsets.data_ptr(), rb.list.data_ptr(),
           rb.active.data_ptr(), rb.n_active.data_ptr(), rb.done.data_ptr(), stream_handle(dev))
    return lg


def norm_fwht_rows(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6, ss_in: torch.Tensor | None = None,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    dev = _require_cuda(x, w)
    rows, D = x.shape
    y = out if out is not None else torch.empty_like(x)
    L.call("r4q_norm_fwht_rows", x.data_ptr(), _ptr(ss_in), 0 if ss_in is None else int(ss_in.shape[0]),
           w.data_ptr(), float(eps), y.data_ptr(), rows, D, stream_handle(dev))
    return y


def moe_gemv(mode: int, w: torch.Tensor, sz: torch.Tensor, x: torch.Tensor, rb: MoeRouteBuffers, N: int, K: int,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """Grouped INT4 expert GEMV (r4q_moe_gemv) over experts [rb.e_lo, rb.e_hi);
    w [(e_hi-e_lo)*N, K/2], sz [(e_hi-e_lo)*N, K/16].  mode 0: x rows are
    tokens (entry j reads x[j // topk]); mode 1: x rows are entries; mode 2:
    gate_up (N = 2 Ie) with the SiLU(gate)*up + H32 FWHT epilogue, x rows
    tokens.  Returns y [B*topk, N] (mode 2: [B*topk, N/2]), one row per routed
    entry; rows of other GPUs' experts untouched."""
    dev = _require_cuda(w, sz, x)
    y = out if out is not None else torch.empty(rb.B * rb.topk, N // 2 if mode == 2 else N, dtype=torch.float16,
                                                device=dev)
    L.call("r4q_moe_gemv", mode, w.data_ptr(), sz.data_ptr(), x.data_ptr(), x.stride(0), y.data_ptr(), y.stride(0),
           N, K, rb.E, rb.e_lo, rb.e_hi, rb.B, rb.topk, rb.counts.data_ptr(), rb.offsets.data_ptr(), rb.list.data_ptr(),
           rb.active.data_ptr(), rb.n_active.data_ptr(), rb.status.data_ptr(), stream_handle(dev))
    return y


def moe_combine(y: torch.Tensor, rb: MoeRouteBuffers, res: torch.Tensor | None, out: torch.Tensor | None = None,
                ss_out: torch.Tensor | None = None, out32: torch.Tensor | None = None) -> torch.Tensor:
    """h = fp16(fp16(sum of this GPU's routed outputs) + res), or with out32 the fp32 partial."""
    dev = _require_cuda(y)
    D = y.shape[1]
    h = out if (out is not None or out32 is not None) else torch.empty(rb.B, D, dtype=torch.float16, device=dev)
    L.call("r4q_moe_combine", y.data_ptr(), rb.wts.data_ptr(), rb.ids.data_ptr(), rb.e_lo, rb.e_hi, _ptr(res),
           _ptr(h), _ptr(out32), _ptr(ss_out), rb.B, D, rb.topk, stream_handle(dev))
    return h if out32 is None else out32


def residual_f32(s: torch.Tensor, res: torch.Tensor | None, out: torch.Tensor, ss_out=None) -> torch.Tensor:
    dev = _require_cuda(s)
    B, D = s.shape
    L.call("r4q_residual_f32", s.data_ptr(), _ptr(res), out.data_ptr(), _ptr(ss_out), B, D, stream_handle(dev))
    return out


def residual_f16(a: torch.Tensor, res: torch.Tensor | None, out: torch.Tensor, ss_out=None) -> torch.Tensor:
    dev = _require_cuda(a)
    B, D = a.shape
    L.call("r4q_residual_f16", a.data_ptr(), _ptr(res), out.data_ptr(), _ptr(ss_out), B, D, stream_handle(dev))
    return out
