"""Generate the golden fixtures in this folder by running the reference's own
Python math (JohnTDI-cpu/rdna4-quant) on seeded inputs.

Run once in a container where the reference checkout exists:

    python tests/golden/make_golden.py /path/to/rdna4-quant

It imports the reference modules ``int4_quant_v2``, ``int8_quant``,
``hadamard_utils`` and ``engine_utils`` (CPU torch) and writes
``golden_ref.npz``.  Nothing at test time reads the reference checkout: the
tests only load the committed ``.npz``.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    import int4_quant_v2 as q4
    import int8_quant as q8
    import hadamard_utils as hu
    import engine_utils as eu

    out = {}
    g = torch.Generator().manual_seed(1234)

    # --- config-0 style weight: N(0, 0.02), 0.1 % outliers x20, H32-rotated ---
    N, K = 64, 256
    W = torch.randn(N, K, generator=g) * 0.02
    mask = torch.rand(N, K, generator=g) < 0.001
    W = torch.where(mask, W * 20.0, W)
    Wr = hu.rotate_weight(W.float(), 32)
    qv, sc, zp, rec = q4.quantize_to_int4_asymmetric(Wr.reshape(N, K // 32, 32))
    packed = q4.pack_int4_unsigned(qv.reshape(N, K))
    out['w_fp32'] = W.numpy()
    out['w_rot'] = Wr.numpy()
    out['q4_q'] = qv.reshape(N, K).numpy()
    out['q4_scale'] = sc.numpy()
    out['q4_zero'] = zp.numpy()
    out['q4_packed'] = packed.numpy()
    out['q4_unpacked'] = q4.unpack_int4_unsigned(packed).numpy()
    out['q4_deq'] = q4.dequantize_int4_asym(packed, sc, zp, block_size=32).numpy()

    # edge blocks: constant (scale 0 -> 1), all-negative, huge range, tiny
    E = torch.zeros(8, 32)
    E[1] = 3.0
    E[2] = -torch.linspace(1, 2, 32)
    E[3] = torch.linspace(-1e5, 1e5, 32)
    E[4] = torch.linspace(-1e-6, 1e-6, 32)
    E[5] = torch.linspace(0, 1, 32)
    E[6, ::2] = 1.0
    E[7] = torch.linspace(-7.5, 7.5, 32)
    eq, es, ez, _ = q4.quantize_to_int4_asymmetric(E)
    out['edge_in'] = E.numpy()
    out['edge_q'] = eq.numpy()
    out['edge_scale'] = es.numpy()
    out['edge_zero'] = ez.numpy()

    # activation x ~ N(0,1) fp16, rotated the same way
    x = torch.randn(2, K, generator=g).half()
    xr = hu.rotate_activation(x.float(), 32).half()
    out['x_fp16'] = x.numpy()
    out['x_rot'] = xr.numpy()
    Wd = q4.dequantize_int4_asym(packed, sc, zp, block_size=32)
    out['gemv_ref'] = (xr.float() @ Wd.float().T).half().numpy()

    # symmetric INT4 (lm_head format) and its signed unpack
    qs, ss, _ = q4.quantize_to_int4_symmetric(Wr.reshape(N, K // 32, 32))
    ps = q4.pack_int4(qs.reshape(N, K))
    out['q4s_q'] = qs.reshape(N, K).numpy()
    out['q4s_scale'] = ss.numpy()
    out['q4s_packed'] = ps.numpy()
    out['q4s_deq'] = (q4.unpack_int4(ps).float().reshape(N, K // 32, 32)
                      * ss.float().unsqueeze(-1)).reshape(N, K).half().numpy()

    # INT8 symmetric
    q8v, s8, _ = q8.quantize_to_int8_symmetric(Wr.reshape(N, K // 32, 32))
    out['q8_w'] = q8v.reshape(N, K).numpy()
    out['q8_scale'] = s8.numpy()
    out['q8_deq'] = q8.dequantize_int8(q8v.reshape(N, K), s8, block_size=32).numpy()

    # Hadamard
    out['h32'] = hu.get_hadamard(32, dtype=torch.float64).numpy()
    a = torch.randn(3, 128, generator=g, dtype=torch.float64)
    out['rot_in'] = a.numpy()
    out['rot_out'] = hu.rotate_activation(a, 32).numpy()

    # RMSNorm CPU branch
    xn = (torch.randn(4, 512, generator=g) * 2).half()
    wn = (1 + 0.01 * torch.randn(512, generator=g)).half()
    out['rms_x'] = xn.numpy()
    out['rms_w'] = wn.numpy()
    out['rms_y'] = eu.RMSNorm(wn, 1e-6).forward(xn).numpy()

    # RoPE tables and apply_rope
    cos, sin = eu.precompute_rope_freqs(128, 96, theta=1000000.0, device='cpu')
    out['rope_cos'] = cos.numpy()
    out['rope_sin'] = sin.numpy()
    xq = torch.randn(1, 4, 3, 128, generator=g).half()
    pid = torch.tensor([[5, 17, 95]])
    out['rope_x'] = xq.numpy()
    out['rope_pos'] = pid.numpy()
    out['rope_y'] = eu.apply_rope(xq, cos, sin, pid).numpy()

    dst = Path(__file__).with_name('golden_ref.npz')
    np.savez_compressed(dst, **out)
    print('wrote', dst, {k: v.shape for k, v in out.items()})


if __name__ == '__main__':
    if len(sys.argv) != 2:
        sys.exit("usage: python make_golden.py <reference checkout>")
    main(sys.argv[1])
