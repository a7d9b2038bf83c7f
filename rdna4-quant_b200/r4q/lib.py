"""ctypes binding of libr4q.so (the C ABI in include/r4q.h).

Every wrapper raises ``R4QError`` on a non-zero status, with the library's
message.  There is deliberately no fallback path: a missing library is an
import error.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent.parent
_SO = Path(os.environ.get("R4Q_LIB", _PKG / "libr4q.so"))


class R4QError(RuntimeError):
    def __init__(self, code: int, what: str, msg: str):
        super().__init__(f"{what} failed with r4q status {code}: {msg}")
        self.code = code


def _load():
    if not _SO.exists():
        raise ImportError(
            f"libr4q.so not found at {_SO}: build it with `python -m r4q.build` "
            "(or __graft_entry__.build()); r4q has no CPU fallback")
    try:  # make sure torch's CUDA runtime is loaded first so both share it
        import torch  # noqa: F401
    except Exception:
        pass
    return C.CDLL(str(_SO))


LIB = _load()


class GemvFused(C.Structure):
    """r4q_gemv_fused (include/r4q.h)."""
    _fields_ = [("norm_w", C.c_void_p), ("eps", C.c_float), ("ss_in", C.c_void_p),
                ("ss_in_parts", C.c_int), ("residual", C.c_void_p), ("ldres", C.c_long),
                ("ss_out", C.c_void_p), ("y32", C.c_void_p)]

vp, i32, i64, sz_t, f32 = C.c_void_p, C.c_int, C.c_long, C.c_size_t, C.c_float


class LayerDesc(C.Structure):
    """r4q_layer_desc (include/r4q.h)."""
    _fields_ = [("qkv_fmt", C.c_int), ("o_fmt", C.c_int), ("gate_up_fmt", C.c_int),
                ("down_fmt", C.c_int)] + [(n, C.c_void_p) for n in (
                    "qkv_w", "qkv_s", "o_w", "o_s", "gate_up_w", "gate_up_s", "down_w", "down_s",
                    "in_norm", "post_norm", "q_norm", "k_norm", "k_cache", "v_cache", "k_scale",
                    "v_scale")]


class ModelDesc(C.Structure):
    """r4q_model_desc (include/r4q.h)."""
    _fields_ = [(n, C.c_int) for n in ("num_layers", "batch", "hidden", "intermediate", "num_heads",
                                        "num_kv_heads", "head_dim", "max_seq")] + [
        ("rms_eps", C.c_float), ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p),
        ("rope_stride", C.c_long), ("final_norm", C.c_void_p), ("lm_fmt", C.c_int),
        ("lm_w", C.c_void_p), ("lm_s", C.c_void_p), ("lm_n", C.c_int), ("tp_rank", C.c_int),
        ("tp_size", C.c_int), ("comm", C.c_void_p)]

_SIGS = {
    "r4q_last_error": (C.c_char_p, []),
    "r4q_version": (i32, []),
    "r4q_ws_status": (i32, [vp, i32, vp]),
    "r4q_debug_spin_limit": (i64, [i64]),
    "r4q_decode_status": (i32, [vp, i32]),
    "r4q_gemv_workspace_bytes": (sz_t, [i32, i32, i32]),
    "r4q_gemv_int4": (i32, [vp, i64, vp, vp, vp, i64, i32, i32, i32, i32, vp, sz_t, vp]),
    "r4q_gemv_int8": (i32, [vp, i64, vp, vp, vp, i64, i32, i32, i32, i32, vp, sz_t, vp]),
    "r4q_gemv_fp16": (i32, [vp, i64, vp, vp, i64, i32, i32, i32, i32, vp, sz_t, vp]),
    "r4q_gemv": (i32, [i32, vp, i64, vp, vp, vp, i64, i32, i32, i32, i32, C.POINTER(GemvFused),
                       vp, sz_t, vp]),
    "r4q_gemv_int4_noalloc": (i32, [vp, i64, vp, vp, vp, i64, i32, i32, i32, i32, vp]),
    "r4q_rmsnorm": (i32, [vp, vp, vp, vp, vp, i32, i32, i64, f32, vp]),
    "r4q_head_norm_rope": (i32, [vp, vp, vp, vp, vp, vp, vp, i64, i32, vp, vp, vp, vp, vp, vp, vp,
                                 i32, i32, i32, i32, i64, i64, i32, f32, i32, vp]),
    "r4q_flash_decode_workspace_bytes": (sz_t, [i32, i32, i32, i32]),
    "r4q_flash_decode": (i32, [vp, i64, vp, vp, vp, vp, vp, i64, i32, i32, i32, i32, i32, i32, vp,
                               i32, vp, sz_t, vp]),
    "r4q_attn_decode_fused": (i32, [vp, i64, vp, vp, vp, vp, i64, f32, vp, vp, vp, vp, vp, i64, i32, i32,
                                    i32, i32, i32, i32, vp, i32, vp, sz_t, vp]),
    "r4q_gemm_fp16": (i32, [vp, i64, vp, vp, i64, i32, i32, i32, vp, sz_t, vp]),
    "r4q_gemm_int4": (i32, [vp, i64, vp, vp, vp, i64, i32, i32, i32, vp, sz_t, vp]),
    "r4q_gemm_workspace_bytes": (sz_t, [i32, i32, i32]),
    "r4q_fwht_rows": (i32, [vp, i64, vp, i64, i32, i32, vp]),
    "r4q_silu_mul": (i32, [vp, i64, vp, i64, i32, i32, vp]),
    "r4q_dequant_int8": (i32, [vp, vp, vp, i32, i32, vp]),
    "r4q_kv_write_rows": (i32, [vp, vp, i64, vp, vp, i32, i32, i32, i32, i32, i32, vp, vp, vp]),
    "r4q_moe_route": (i32, [vp, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp]),
    "r4q_norm_fwht_rows": (i32, [vp, vp, i32, vp, f32, vp, i32, i32, vp]),
    "r4q_moe_router": (i32, [vp, vp, i32, vp, f32, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp,
                             vp, vp, vp]),
    "r4q_moe_gemv": (i32, [i32, vp, vp, vp, i64, vp, i64, i32, i32, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp,
                           vp, vp]),
    "r4q_moe_combine": (i32, [vp, vp, vp, i32, i32, vp, vp, vp, vp, i32, i32, i32, vp]),
    "r4q_residual_f32": (i32, [vp, vp, vp, vp, i32, i32, vp]),
    "r4q_residual_f16": (i32, [vp, vp, vp, vp, i32, i32, vp]),
    "r4q_decode_ctx_create": (i32, [C.POINTER(ModelDesc), C.POINTER(LayerDesc), C.POINTER(C.c_void_p)]),
    "r4q_decode_ctx_destroy": (None, [vp]),
    "r4q_decode_step": (i32, [vp, vp, i32, vp, vp, i32, vp]),
    "r4q_decode_step_rows": (i32, [vp, vp, vp, vp, vp, i32, vp]),
    "r4q_decode_tp_trace": (i32, [vp, vp]),
    "r4q_decode_loop": (i32, [vp, vp, vp, i32, i32, vp, i32, vp]),
    "r4q_decode_profile": (i32, [vp, vp, i32, vp, vp]),
    "r4q_comm_create": (i32, [i32, i32, i32, i32, i32, i64, C.POINTER(C.c_void_p), vp]),
    "r4q_comm_open": (i32, [vp, vp]),
    "r4q_comm_status": (i32, [vp]),
    "r4q_comm_clear_status": (i32, [vp]),
    "r4q_comm_allreduce_f32": (i32, [vp, vp, vp, i64, vp]),
    "r4q_comm_destroy": (None, [vp]),
    "r4q_dequant_int4": (i32, [vp, vp, vp, i32, i32, vp]),
    "r4q_fp16_to_fp8": (i32, [vp, vp, i64, vp]),
    "r4q_fp8_to_fp32": (i32, [vp, vp, i64, vp]),
}

COMM_HANDLE_BYTES = 64

EXPORTS = []
for _name, (_res, _args) in _SIGS.items():
    if hasattr(LIB, _name):
        _f = getattr(LIB, _name)
        _f.restype = _res
        _f.argtypes = _args
        EXPORTS.append(_name)


def last_error() -> str:
    return LIB.r4q_last_error().decode(errors="replace")


def call(name: str, *args) -> None:
    st = getattr(LIB, name)(*args)
    if st != 0:
        raise R4QError(st, name, last_error())


# activation prologues (enum in include/r4q.h)
PRO_NONE, PRO_FWHT, PRO_SILU_FWHT, PRO_RMSNORM_FWHT = 0, 1, 2, 3
W_INT4, W_INT8, W_FP16 = 0, 1, 2
HEAD_NORM, HEAD_ROPE, HEAD_KV = 1, 2, 4
ATTN_FWHT = 1
