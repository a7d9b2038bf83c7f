"""Checkpoint loader (r4q.loader) on directories written by the reference's
own quantisers in its v4 (mixed INT4 asym / INT4 sym / INT8, symmetric lm_head)
and v5 (pure INT4, asymmetric lm_head) formats (tests/golden/make_ckpt.py).
The runtime-layout tensors the loader returns must dequantise, with this
library's dequantisers, to exactly the fp16 weights the reference's
dequantisers give."""
from pathlib import Path

import numpy as np
import pytest
import torch

import r4q_oracle as O
from r4q import loader

GOLD = Path(__file__).resolve().parent / "golden"


def _deq(w, s):
    w = w.cpu().numpy()
    s = s.cpu().numpy()
    if w.dtype == np.uint8:
        return O.dequant_int4_runtime(w, s)
    return O.dequant_int8(w, s)


@pytest.mark.parametrize("name", ["ckpt_v4", "ckpt_v5"])
def test_loader_matches_reference_dequant(name):
    cfg, m = loader.load_checkpoint(GOLD / name, device='cpu', max_seq=64)
    exp = np.load(GOLD / name / "expected.npz")
    assert cfg['hidden'] == 128 and cfg['num_heads'] == 2 and cfg['num_kv_heads'] == 1 and cfg['vocab'] == 256
    for li in range(cfg['num_layers']):
        for g, key in loader.GROUPS:
            got = _deq(m[key + '_w'][li], m[key + '_s'][li])
            assert np.array_equal(got, exp[f'l{li}_{g}']), (li, g)
        for k, name2 in (('in_norm', 'in_norm_w'), ('post_norm', 'post_norm_w'), ('q_norm', 'q_norm_w'),
                         ('k_norm', 'k_norm_w')):
            assert np.array_equal(m[name2][li].numpy(), exp[f'l{li}_{k}'])
    assert np.array_equal(_deq(m['lm_w'], m['lm_s']), exp['lm'])
    assert np.array_equal(m['embed'].numpy(), exp['embed'])
    assert np.array_equal(m['final_norm_w'].numpy(), exp['final_norm'])
    assert m['rope_cos'].shape == (64 + 128, 64) and m['k_caches'][0].shape == (1, 1, 64, 128)


def test_symmetric_conversion_all_nibbles():
    """Every two's-complement nibble n maps to n' with (n' - 8) == int4(n)."""
    packed = torch.arange(256, dtype=torch.int32).to(torch.uint8).reshape(1, 256)
    scales = torch.ones(1, 16, dtype=torch.float16)
    out, pairs = loader.symmetric_to_unsigned(packed, scales)
    lo, hi = (packed & 15).to(torch.int32), (packed >> 4).to(torch.int32)
    slo, shi = torch.where(lo > 7, lo - 16, lo), torch.where(hi > 7, hi - 16, hi)
    assert torch.equal((out & 15).to(torch.int32) - 8, slo) and torch.equal((out >> 4).to(torch.int32) - 8, shi)
    assert torch.equal(pairs.view(1, 16, 2)[..., 1], torch.full((1, 16), 8.0, dtype=torch.float16))
