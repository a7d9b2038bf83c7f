"""Write small quantised-model directories in the reference's on-disk formats
with the reference's own quantiser and packer functions, plus the weights the
reference's dequantisers reconstruct from them, to pin the checkpoint loader.

    python tests/golden/make_ckpt.py /path/to/rdna4-quant

Writes ``ckpt_v4/`` (v4 mixed: asymmetric INT4, symmetric INT4 and INT8
groups, symmetric INT4 lm_head — quantize_v4_gptq.py:352-468) and
``ckpt_v5/`` (v5 pure asymmetric INT4 with an asymmetric lm_head), each with
``expected.npz`` holding the fp16 weights the reference dequantisers
(dequantize_int4_asym, unpack_int4 * scale, dequantize_int8) give.  Tests
read only these files.  Shapes follow a tiny Qwen3 layout (hidden 128,
2 query / 1 KV heads of 128, intermediate 256, vocabulary 256) so the
decode kernels can run the loaded model too.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

D, I, H, HK, HD, V = 128, 256, 2, 1, 128, 256


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    import int4_quant_v2 as q4
    import int8_quant as q8

    here = Path(__file__).resolve().parent
    g = torch.Generator().manual_seed(99)
    shapes = {'qkv': ((H + 2 * HK) * HD, D), 'o': (D, H * HD), 'gate_up': (2 * I, D), 'down': (D, I)}

    def weight(N, K):
        return torch.randn(N, K, generator=g) * 0.05

    def int4a(W):
        N, K = W.shape
        q, s, z, _ = q4.quantize_to_int4_asymmetric(W.reshape(N, K // 32, 32))
        packed = q4.pack_int4_unsigned(q.reshape(N, K))
        deq = q4.dequantize_int4_asym(packed, s, z)
        return {'packed': packed, 'scales': s, 'zeros': z}, deq

    def int4s(W):
        N, K = W.shape
        q, s, _ = q4.quantize_to_int4_symmetric(W.reshape(N, K // 32, 32))
        packed = q4.pack_int4(q.reshape(N, K))
        deq = (q4.unpack_int4(packed).reshape(N, K // 32, 32).float() * s.float().unsqueeze(-1)).reshape(N, K).half()
        return {'packed': packed, 'scales': s, 'zeros': torch.zeros_like(s, dtype=torch.uint8)}, deq

    def int8(W):
        N, K = W.shape
        q, s, _ = q8.quantize_to_int8_symmetric(W.reshape(N, K // 32, 32))
        q = q.reshape(N, K)
        return {'weights': q, 'scales': s}, q8.dequantize_int8(q, s)

    variants = {
        'ckpt_v4': [{'qkv': 'int4a', 'o': 'int8', 'gate_up': 'int4', 'down': 'int4a'},
                    {'qkv': 'int8', 'o': 'int4a', 'gate_up': 'int4a', 'down': 'int8'}],
        'ckpt_v5': [{'qkv': 'int4a', 'o': 'int4a', 'gate_up': 'int4a', 'down': 'int4a'}],
    }
    for name, layers in variants.items():
        d = here / name
        d.mkdir(exist_ok=True)
        expected = {}
        for li, prec in enumerate(layers):
            ld = {}
            for grp, (N, K) in shapes.items():
                W = weight(N, K)
                kind = prec[grp]
                if kind == 'int8':
                    data, deq = int8(W)
                    ld[f'{grp}_weights'], ld[f'{grp}_scales'] = data['weights'], data['scales']
                else:
                    data, deq = (int4a if kind == 'int4a' else int4s)(W)
                    ld[f'{grp}_packed'], ld[f'{grp}_scales'] = data['packed'], data['scales']
                    ld[f'{grp}_zeros'] = data['zeros']
                ld[f'{grp}_precision'] = kind
                ld[f'{grp}_N'], ld[f'{grp}_K'] = N, K
                expected[f'l{li}_{grp}'] = deq.numpy()
            for k, n in (('in_norm', D), ('post_norm', D), ('q_norm', HD), ('k_norm', HD)):
                ld[k] = (1 + 0.05 * torch.randn(n, generator=g)).to(torch.bfloat16)
                expected[f'l{li}_{k}'] = ld[k].half().numpy()
            torch.save(ld, d / f'layer_{li:03d}.pt')
        Wlm = weight(V, D)
        if name == 'ckpt_v5':
            data, deq = int4a(Wlm)
            lm = {'packed': data['packed'], 'scales': data['scales'], 'zeros': data['zeros'], 'N': V, 'K': D}
        else:
            data, deq = int4s(Wlm)
            lm = {'packed': data['packed'], 'scales': data['scales'], 'N': V, 'K': D,
                  'rotation': 'hadamard', 'quant_format': 'int4_symmetric'}
        torch.save(lm, d / 'lm_head.pt')
        expected['lm'] = deq.numpy()
        embed = (torch.randn(V, D, generator=g) * 0.5).to(torch.bfloat16)
        fnorm = (1 + 0.05 * torch.randn(D, generator=g)).to(torch.bfloat16)
        torch.save(embed, d / 'embed.pt')
        torch.save(fnorm, d / 'final_norm.pt')
        expected['embed'], expected['final_norm'] = embed.half().numpy(), fnorm.half().numpy()
        meta = {'model_name': 'tiny-qwen3', 'num_layers': len(layers), 'hidden_size': D, 'intermediate_size': I,
                'num_heads': H, 'num_kv_heads': HK, 'head_dim': HD, 'rms_eps': 1e-6, 'rope_theta': 1e6,
                'block_size': 32, 'method': name}
        torch.save(meta, d / 'meta.pt')
        np.savez_compressed(d / 'expected.npz', **expected)
        print('wrote', d)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python make_ckpt.py <reference checkout>")
    main(sys.argv[1])
