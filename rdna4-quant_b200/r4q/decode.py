"""Decode-step contexts: turn the reference's per-layer tensor lists into the C
runtime's model description (include/r4q.h r4q_model_desc / r4q_layer_desc)
and keep one context per distinct set of weights and caches."""
from __future__ import annotations

import ctypes as C
import threading

import torch

from . import lib as L
from . import ops

_lock = threading.Lock()
_ctx: dict = {}


def weight_format(w: torch.Tensor) -> int:
    """uint8 [N, K/2] -> INT4, int8 [N, K] -> INT8, fp16 [N, K] -> FP16."""
    if w.dtype == torch.uint8:
        return L.W_INT4
    if w.dtype == torch.int8:
        return L.W_INT8
    if w.dtype == torch.float16:
        return L.W_FP16
    raise TypeError(f"unsupported weight dtype {w.dtype}")


class DecodeContext:
    def __init__(self, model: L.ModelDesc, layers, keepalive):
        self.model = model
        self.layers = (L.LayerDesc * max(1, len(layers)))(*layers)
        self.keepalive = keepalive
        h = C.c_void_p()
        L.call("r4q_decode_ctx_create", C.byref(model), self.layers, C.byref(h))
        self.handle = h

    def step(self, hidden_in, pos, hidden_out=None, logits_out=None, use_graph=True):
        dev = hidden_in.device
        L.call("r4q_decode_step", self.handle, hidden_in.data_ptr(), int(pos),
               None if hidden_out is None else hidden_out.data_ptr(),
               None if logits_out is None else logits_out.data_ptr(), 1 if use_graph else 0,
               ops.stream_handle(dev))

    def step_rows(self, hidden_in, positions, hidden_out=None, logits_out=None, use_graph=True):
        """One step with a position per row (r4q_decode_step_rows)."""
        B = self.model.batch
        if len(positions) != B:
            raise ValueError(f"{len(positions)} positions for a batch of {B}")
        pos = (C.c_int * B)(*[int(p) for p in positions])
        L.call("r4q_decode_step_rows", self.handle, hidden_in.data_ptr(), pos,
               None if hidden_out is None else hidden_out.data_ptr(),
               None if logits_out is None else logits_out.data_ptr(), 1 if use_graph else 0,
               ops.stream_handle(hidden_in.device))

    def loop(self, embed, hidden_first, start_pos, num_tokens, use_graph=True):
        """Greedy tokens [num_tokens, batch] int64 on the device (r4q_decode_loop)."""
        dev = hidden_first.device
        out = torch.empty(int(num_tokens), self.model.batch, dtype=torch.int64, device=dev)
        if num_tokens:
            L.call("r4q_decode_loop", self.handle, embed.data_ptr(), hidden_first.data_ptr(), int(start_pos),
                   int(num_tokens), out.data_ptr(), 1 if use_graph else 0, ops.stream_handle(dev))
        return out

    def profile(self, hidden_in, pos):
        """[total, gemv, attention, norm, rest] ms of one eager step (r4q_decode_profile)."""
        out = (C.c_float * 5)()
        L.call("r4q_decode_profile", self.handle, hidden_in.data_ptr(), int(pos), out,
               ops.stream_handle(hidden_in.device))
        return [float(v) for v in out]

    def status(self, clear: bool = True) -> None:
        """Raise ``R4QError`` (R4Q_ERR_TIMEOUT) if a bounded wait of one of this
        context's kernels gave up since the last check (synchronises)."""
        L.call("r4q_decode_status", self.handle, 1 if clear else 0)

    def __del__(self):
        try:
            if getattr(self, "handle", None):
                L.LIB.r4q_decode_ctx_destroy(self.handle)
        except Exception:
            pass


def _p(t):
    return None if t is None else t.data_ptr()


def get_context(qkv_w, qkv_s, o_w, o_s, gu_w, gu_s, down_w, down_s, in_norm_w, post_norm_w,
                q_norm_w, k_norm_w, rope_cos, rope_sin, num_heads, num_kv_heads, head_dim,
                hidden_size, intermediate_size, rms_eps, k_caches, v_caches, final_norm_w=None,
                lm_w=None, lm_s=None, lm_N=0, batch=1, k_scales=None, v_scales=None, comm=None):
    """Context for these weights/caches.  With ``comm`` (r4q.tp.Comm of
    world > 1) the tensors are this rank's shards and the head / intermediate
    / vocabulary counts are the local ones (r4q.tp.local_cfg)."""
    n = len(qkv_w)
    max_seq = int(k_caches[0].shape[-2]) if n else 1
    key = (tuple(t.data_ptr() for t in (*qkv_w, *o_w, *gu_w, *down_w, *k_caches, *v_caches)),
           _p(final_norm_w), _p(lm_w), int(lm_N), int(batch), int(hidden_size),
           int(intermediate_size), int(num_heads), int(num_kv_heads), int(head_dim), max_seq,
           float(rms_eps), _p(rope_cos), torch.cuda.current_device(),
           None if comm is None else comm.handle.value)
    with _lock:
        ctx = _ctx.get(key)
        if ctx is not None:
            return ctx
        layers = []
        for li in range(n):
            d = L.LayerDesc()
            d.qkv_fmt, d.o_fmt = weight_format(qkv_w[li]), weight_format(o_w[li])
            d.gate_up_fmt, d.down_fmt = weight_format(gu_w[li]), weight_format(down_w[li])
            d.qkv_w, d.qkv_s = qkv_w[li].data_ptr(), qkv_s[li].data_ptr()
            d.o_w, d.o_s = o_w[li].data_ptr(), o_s[li].data_ptr()
            d.gate_up_w, d.gate_up_s = gu_w[li].data_ptr(), gu_s[li].data_ptr()
            d.down_w, d.down_s = down_w[li].data_ptr(), down_s[li].data_ptr()
            d.in_norm, d.post_norm = in_norm_w[li].data_ptr(), post_norm_w[li].data_ptr()
            d.q_norm, d.k_norm = q_norm_w[li].data_ptr(), k_norm_w[li].data_ptr()
            d.k_cache, d.v_cache = k_caches[li].data_ptr(), v_caches[li].data_ptr()
            d.k_scale = None if k_scales is None else k_scales[li].data_ptr()
            d.v_scale = None if v_scales is None else v_scales[li].data_ptr()
            layers.append(d)
        m = L.ModelDesc()
        m.num_layers, m.batch, m.hidden, m.intermediate = n, int(batch), int(hidden_size), int(intermediate_size)
        m.num_heads, m.num_kv_heads, m.head_dim, m.max_seq = (int(num_heads), int(num_kv_heads),
                                                              int(head_dim), max_seq)
        m.rms_eps = float(rms_eps)
        m.rope_cos, m.rope_sin, m.rope_stride = rope_cos.data_ptr(), rope_sin.data_ptr(), rope_cos.stride(0)
        m.final_norm = _p(final_norm_w)
        if lm_w is not None:
            m.lm_fmt = weight_format(lm_w)
            m.lm_w, m.lm_s = lm_w.data_ptr(), _p(lm_s) if m.lm_fmt != L.W_FP16 else None
            m.lm_n = int(lm_N)
        if comm is not None and comm.world > 1:
            m.tp_rank, m.tp_size, m.comm = comm.rank, comm.world, comm.handle.value
        else:
            m.tp_rank, m.tp_size, m.comm = 0, 1, None
        keep = (comm, qkv_w, qkv_s, o_w, o_s, gu_w, gu_s, down_w, down_s, in_norm_w, post_norm_w,
                q_norm_w, k_norm_w, rope_cos, rope_sin, k_caches, v_caches, final_norm_w, lm_w,
                lm_s, k_scales, v_scales)
        ctx = DecodeContext(m, layers, keep)
        _ctx[key] = ctx
        return ctx


def clear_contexts():
    """Drop every cached decode context (frees their scratch)."""
    with _lock:
        _ctx.clear()
