"""Pins the CPU oracle against the reference's own outputs (golden vectors made
by tests/golden/make_golden.py) and against known answers read off the HIP
source for the numerics that have no runnable reference."""
from pathlib import Path

import numpy as np
import pytest

import r4q_oracle as O

G = np.load(Path(__file__).parent / "golden" / "golden_ref.npz")


def test_quantizer_bit_exact():
    N, K = G['w_rot'].shape
    q, s, z = O.quantize_int4_asym(G['w_rot'].reshape(N, K // 32, 32))
    assert np.array_equal(q.reshape(N, K), G['q4_q'])
    assert np.array_equal(s.view(np.uint16), G['q4_scale'].view(np.uint16))
    assert np.array_equal(z, G['q4_zero'])


def test_quantizer_edge_blocks():
    q, s, z = O.quantize_int4_asym(G['edge_in'])
    assert np.array_equal(q, G['edge_q'])
    assert np.array_equal(s.view(np.uint16), G['edge_scale'].view(np.uint16))
    assert np.array_equal(z, G['edge_zero'])


def test_pack_unpack_dequant_bit_exact():
    packed = O.pack_int4(G['q4_q'])
    assert np.array_equal(packed, G['q4_packed'])
    assert np.array_equal(O.unpack_int4(packed), G['q4_unpacked'])
    deq = O.dequant_int4(packed, G['q4_scale'], G['q4_zero'])
    assert np.array_equal(deq.view(np.uint16), G['q4_deq'].view(np.uint16))
    # runtime (interleaved) layout gives the same bits
    sz = O.interleave_scale_zero(G['q4_scale'], G['q4_zero'])
    assert sz.shape == (packed.shape[0], packed.shape[1] * 2 // 16)
    deq2 = O.dequant_int4_runtime(packed, sz)
    assert np.array_equal(deq2.view(np.uint16), G['q4_deq'].view(np.uint16))
    s2, z2 = O.split_scale_zero(sz)
    assert np.array_equal(z2, G['q4_zero'])


def test_torch_dequant_restatement_bit_exact():
    """The torch restatement the CPU baseline times equals the reference's
    dequantize_int4_asym output (golden vectors it wrote) bit for bit, and the
    reference function itself where the reference tree is importable."""
    import torch
    packed = torch.from_numpy(G['q4_packed'])
    s = torch.from_numpy(G['q4_scale'])
    z = torch.from_numpy(G['q4_zero'])
    deq = O.dequant_int4_torch(packed, s, z).numpy()
    assert np.array_equal(deq.view(np.uint16), G['q4_deq'].view(np.uint16))
    ref_dir = Path("/root/reference")
    if (ref_dir / "int4_quant_v2.py").exists():
        import importlib.util
        spec = importlib.util.spec_from_file_location("ref_int4_quant_v2", ref_dir / "int4_quant_v2.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        ref = mod.dequantize_int4_asym(packed, s, z).numpy()
        assert np.array_equal(deq.view(np.uint16), ref.view(np.uint16))


def test_symmetric_lm_head_conversion():
    N, K = G['w_rot'].shape
    q, s = O.quantize_int4_sym(G['w_rot'].reshape(N, K // 32, 32))
    assert np.array_equal(q.reshape(N, K), G['q4s_q'])
    assert np.array_equal(s.view(np.uint16), G['q4s_scale'].view(np.uint16))
    p = O.pack_int4_signed(q.reshape(N, K))
    assert np.array_equal(p, G['q4s_packed'])
    p2, sz = O.convert_symmetric_to_asymmetric(p, s)
    deq = O.dequant_int4_runtime(p2, sz)
    assert np.array_equal(deq.view(np.uint16), G['q4s_deq'].view(np.uint16))


def test_int8_bit_exact():
    N, K = G['w_rot'].shape
    q, s = O.quantize_int8_sym(G['w_rot'].reshape(N, K // 32, 32))
    assert np.array_equal(q.reshape(N, K), G['q8_w'])
    assert np.array_equal(s.view(np.uint16), G['q8_scale'].view(np.uint16))
    deq = O.dequant_int8(G['q8_w'], G['q8_scale'])
    assert np.array_equal(deq.view(np.uint16), G['q8_deq'].view(np.uint16))


def test_hadamard_and_fwht():
    # the reference builds H in float32 before widening, hence 1e-8
    assert np.abs(O.hadamard_matrix(32) - G['h32']).max() < 1e-8
    assert np.abs(O.rotate_blocks(G['rot_in']) - G['rot_out']).max() < 1e-7
    # butterfly order equals the matrix product (float32 rounding only)
    y = O.fwht32(G['rot_in'].astype(np.float32))
    assert np.abs(y - G['rot_out']).max() < 1e-5
    # H32 is an involution
    assert np.abs(O.fwht32(y) - G['rot_in']).max() < 1e-5


def test_rmsnorm_matches_reference():
    y = O.rmsnorm(G['rms_x'], G['rms_w'], 1e-6)
    diff = np.abs(y.astype(np.float32) - G['rms_y'].astype(np.float32))
    # reference reduces in float32; allow one fp16 ulp
    assert diff.max() <= np.abs(G['rms_y'].astype(np.float32)).max() * 2 ** -10


def test_rope_tables_and_rotation():
    c, s = O.rope_tables(128, 96, 1e6)
    dc = np.abs(c.astype(np.float32) - G['rope_cos'].astype(np.float32)).max()
    ds = np.abs(s.astype(np.float32) - G['rope_sin'].astype(np.float32)).max()
    assert dc <= 2 ** -11 and ds <= 2 ** -11
    x = G['rope_x'][0]                              # [H, S, D]
    for j, p in enumerate(G['rope_pos'][0]):
        y = O.rope_only(x[:, j], G['rope_cos'][p], G['rope_sin'][p])
        ref = G['rope_y'][0][:, j].astype(np.float32)
        # reference applies RoPE in fp16 arithmetic; ours is float32
        assert np.abs(y.astype(np.float32) - ref).max() <= 4e-3 * max(1.0, np.abs(ref).max())


def test_gemv_oracle_matches_reference_test_math():
    y = O.gemv_int4(G['x_rot'], G['q4_packed'],
                    O.interleave_scale_zero(G['q4_scale'], G['q4_zero']))
    ref = G['gemv_ref'].astype(np.float32)
    assert np.abs(y.astype(np.float32) - ref).max() <= 1e-3 * np.abs(ref).max()
    yb = O.gemv_int4_blockwise(G['x_rot'], G['q4_packed'],
                               O.interleave_scale_zero(G['q4_scale'], G['q4_zero']))
    assert np.abs(yb.astype(np.float32) - ref).max() <= 2e-3 * np.abs(ref).max()


@pytest.mark.parametrize("val,byte", [
    (250.0, 0x7E), (300.0, 0x7E), (-300.0, 0xFE), (448.0, 0x7E), (1e30, 0x7E),
    (0.01, 0x00), (-0.01, 0x80), (2.0 ** -6, 0x08), (2.0 ** -7, 0x00),
    (1.0, 0x38), (1.0625, 0x39), (1.1875, 0x3A), (-1.0625, 0xB9),
    (240.0, 0x77), (248.0, 0x7E), (0.0, 0x00), (-0.0, 0x80), (float('nan'), 0x7E),
])
def test_fp8_encoder_known_answers(val, byte):
    """Values derived by hand from f32_to_fp8e4m3 (int4_decode_step.hip:47-68)."""
    assert int(O.fp8_encode(np.array([val], np.float32))[0]) == byte


def test_fp8_decoder_known_answers():
    b = np.array([0x00, 0x80, 0x38, 0x7E, 0xFE, 0x08, 0x01, 0x7F], np.uint8)
    d = O.fp8_decode(b)
    assert d[0] == 0 and d[1] == 0 and not np.signbit(d[1])
    assert d[2] == 1.0 and d[3] == 448.0 and d[4] == -448.0 and d[5] == 2.0 ** -6
    # exponent-field-0 bytes decode as 2^-7 * (1 + m/8) in the reference (no subnormals)
    assert d[6] == 2.0 ** -7 * (1 + 1 / 8)
    assert d[7] == 480.0


def test_fp8_roundtrip_all_encodable():
    b = O.fp8_encodable_bytes()
    assert len(b) == 2 + 2 * 14 * 8 + 2   # zeros, exponents 1..14, 0x7E/0xFE
    assert np.array_equal(O.fp8_encode(O.fp8_decode(b)), np.where(b == 0x80, 0x00, b))


def test_flash_split_sizing():
    assert O.flash_decode_splits(32) == (32, 1)
    assert O.flash_decode_splits(33) == (32, 2)
    assert O.flash_decode_splits(256) == (32, 8)
    assert O.flash_decode_splits(257) == (64, 5)


def test_lse_merge_equals_full_softmax():
    rng = np.random.default_rng(0)
    s = rng.standard_normal(200)
    v = rng.standard_normal((200, 8))
    full = (np.exp(s - s.max()) / np.exp(s - s.max()).sum()) @ v
    parts = np.array_split(np.arange(200), 7)
    pm = np.array([s[p].max() for p in parts])
    ps = np.array([np.exp(s[p] - s[p].max()).sum() for p in parts])
    po = np.array([np.exp(s[p] - s[p].max()) @ v[p] for p in parts])
    assert np.abs(O.lse_merge(pm, ps, po) - full).max() < 1e-12
