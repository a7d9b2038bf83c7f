"""Drop-in for the reference's ``fused_ops`` module (fused_ops.py), on B200.

Same entry points and argument meaning as the Triton originals; the work runs
in libr4q.so (no Triton).  ``position`` may be an int or a device int64 tensor
(read on the device, so a captured graph can advance it without recapture).
"""
from __future__ import annotations

import torch

from r4q import lib as _lib
from r4q import ops as _ops


def fused_rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """x [*, D] fp16, weight [D] fp16 -> fp16 [*, D] (fused_ops.py:28-41)."""
    return _ops.rmsnorm(x, weight, eps)


def _qk(q, k, qw, kw, cos, sin, position, eps, flags):
    B, H, S, D = q.shape
    _, Hk, _, _ = k.shape
    qf = q.reshape(H, D).contiguous()
    kf = k.reshape(Hk, D).contiguous()
    qo, ko = torch.empty_like(qf), torch.empty_like(kf)
    pos_dev = None
    pos = 0
    if isinstance(position, int):
        pos = position
    else:
        pos_dev = position.reshape(-1)[:1].to(torch.int64).contiguous()
    # q and k live in separate buffers: one call per side keeps ld_in simple
    _ops.head_norm_rope(qf, None, q_w=qw, cos=cos, sin=sin, pos=pos, pos_dev=pos_dev, q_out=qo,
                        H=H, Hk=0, D=D, ld_in=0, ld_out=0, eps=eps, flags=flags)
    _ops.head_norm_rope(None, kf, k_w=kw, cos=cos, sin=sin, pos=pos, pos_dev=pos_dev, k_out=ko,
                        H=0, Hk=Hk, D=D, ld_in=0, ld_out=0, eps=eps, flags=flags)
    return qo.reshape(B, H, S, D), ko.reshape(B, Hk, S, D)


def fused_qknorm_rope_decode(q, k, q_norm_weight, k_norm_weight, cos, sin, position, eps=1e-6):
    """Per-head RMSNorm then RoPE at ``position`` for one decode token
    (fused_ops.py:155-181).  q [1, H, 1, D], k [1, Hk, 1, D]."""
    return _qk(q, k, q_norm_weight, k_norm_weight, cos, sin, position, eps,
               _lib.HEAD_NORM | _lib.HEAD_ROPE)


def fused_rope_decode(q, k, cos, sin, position):
    """RoPE at ``position`` for one decode token (fused_ops.py:184-215)."""
    return _qk(q, k, None, None, cos, sin, position, 0.0, _lib.HEAD_ROPE)
