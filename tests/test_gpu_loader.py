"""GPU: a model loaded by r4q.loader from the reference-format v4 checkpoint
(mixed INT4 / INT8, symmetric lm_head) decodes through int4_hip exactly as the
oracle composition of the same loaded tensors (decode-step tolerance 2e-3,
see test_gpu_decode), and prefill runs on it."""
from pathlib import Path

import numpy as np
import pytest
import torch

import r4q_oracle as O
from test_gpu_gemv import close

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"


def _tuple(w, s):
    w = w.cpu().numpy()
    return ('int4', w, s.cpu().numpy()) if w.dtype == np.uint8 else ('int8', w, s.cpu().numpy())


def test_loaded_checkpoint_decodes():
    import int4_hip
    from r4q import decode, loader
    cfg, m = loader.load_checkpoint(GOLD / "ckpt_v4", device='cuda', max_seq=64)
    D, H, HK, HD, I, V = cfg['hidden'], cfg['num_heads'], cfg['num_kv_heads'], cfg['head_dim'], cfg['intermediate'], cfg['vocab']
    rng = np.random.default_rng(0)
    pos = 9
    for kc, vc in zip(m['k_caches'], m['v_caches']):
        kc[:, :, :pos] = torch.from_numpy(O.fp8_encode(rng.standard_normal((1, HK, pos, HD)).astype(np.float32))).cuda()
        vc[:, :, :pos] = torch.from_numpy(O.fp8_encode(rng.standard_normal((1, HK, pos, HD)).astype(np.float32))).cuda()
    h = m['embed'][17].reshape(1, 1, D)
    lg = int4_hip.decode_step_logits(h, m['qkv_w'], m['qkv_s'], 0, m['o_w'], m['o_s'], 0, m['gu_w'], m['gu_s'], 0,
                                     m['down_w'], m['down_s'], 0, m['in_norm_w'], m['post_norm_w'], m['q_norm_w'],
                                     m['k_norm_w'], m['rope_cos'], m['rope_sin'], pos, H, HK, HD, D, I,
                                     cfg['rms_eps'], m['k_caches'], m['v_caches'], m['final_norm_w'], m['lm_w'],
                                     m['lm_s'], V, D, None)
    torch.cuda.synchronize()
    layers = [{'qkv': _tuple(m['qkv_w'][li], m['qkv_s'][li]), 'o': _tuple(m['o_w'][li], m['o_s'][li]),
               'gate_up': _tuple(m['gu_w'][li], m['gu_s'][li]), 'down': _tuple(m['down_w'][li], m['down_s'][li]),
               'in_norm': m['in_norm_w'][li].cpu().numpy(), 'post_norm': m['post_norm_w'][li].cpu().numpy(),
               'q_norm': m['q_norm_w'][li].cpu().numpy(), 'k_norm': m['k_norm_w'][li].cpu().numpy()}
              for li in range(cfg['num_layers'])]
    ocfg = dict(num_heads=H, num_kv_heads=HK, head_dim=HD, hidden_size=D, intermediate_size=I,
                rms_eps=cfg['rms_eps'])
    O.INT4_MODE['mode'] = 'blockwise'
    ref, _ = O.decode_step_logits(h.cpu().numpy().reshape(1, D), layers, ocfg,
                                  [k.cpu().numpy() for k in m['k_caches']], [v.cpu().numpy() for v in m['v_caches']],
                                  pos, m['rope_cos'].cpu().numpy(), m['rope_sin'].cpu().numpy(),
                                  m['final_norm_w'].cpu().numpy(), _tuple(m['lm_w'], m['lm_s']), write_kv=False)
    close(lg.cpu().numpy().reshape(1, V), ref, 2e-3)
    decode.clear_contexts()
    ids = torch.tensor([3, 17, 200, 5], device='cuda')
    out = int4_hip.prefill_logits(ids, m['embed'], m['final_norm_w'], m['lm_w'], m['lm_s'], V, D, m['qkv_w'],
                                  m['qkv_s'], 0, m['o_w'], m['o_s'], 0, m['gu_w'], m['gu_s'], 0, m['down_w'],
                                  m['down_s'], 0, m['in_norm_w'], m['post_norm_w'], m['q_norm_w'], m['k_norm_w'],
                                  m['rope_cos'], m['rope_sin'], H, HK, HD, D, I, cfg['rms_eps'], None)
    O.INT4_MODE['mode'] = 'dequant'
    pref = O.prefill_logits(m['embed'][ids].cpu().numpy(), layers, ocfg, m['rope_cos'].cpu().numpy(),
                            m['rope_sin'].cpu().numpy(), m['final_norm_w'].cpu().numpy(), _tuple(m['lm_w'], m['lm_s']))
    close(out.cpu().numpy(), pref, 5e-3)
