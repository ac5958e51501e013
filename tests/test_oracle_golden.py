"""Pins the CPU oracle (oracle/fp4x_oracle.py) to golden vectors produced by the reference's own functions
(tests/golden/make_golden.py).  Quantizers must match bit for bit; dequantize-then-matmul outputs to fp32
rounding of the reference's float32 matmul."""
import os

import numpy as np
import pytest

from oracle import fp4x_oracle as O

FIX = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_fixtures.npz"))


def x_of(name):
    return O.bf16_bits_to_f32(FIX[name])


def close(a, b, rtol=2e-6):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return np.abs(a - b).max() <= rtol * max(np.abs(b).max(), 1e-30)


def test_w8_quantizer_bit_exact():
    q, s = O.quantize_w8(FIX["w8_w"])
    assert np.array_equal(q, FIX["w8_q"])
    assert np.array_equal(s.view(np.uint32), FIX["w8_s"].view(np.uint32))
    q, s = O.quantize_w8(FIX["w8k320_w"])
    assert np.array_equal(q, FIX["w8k320_q"]) and np.array_equal(s, FIX["w8k320_s"])


def test_w8_gemv_semantics():
    for m in (3, 16):
        y = O.w8_linear(x_of(f"x{m}_k512"), FIX["w8_q"], FIX["w8_s"])
        assert close(y, FIX[f"w8_y{m}"])


def test_w6_quantizer_bit_exact():
    L, H, S = O.quantize_w6(FIX["w6_w"])
    assert np.array_equal(L, FIX["w6_L"]) and np.array_equal(H, FIX["w6_H"])
    assert np.array_equal(S.view(np.uint16), FIX["w6_S"].view(np.uint16))
    L, H, S = O.quantize_w6(FIX["w6z_w"])
    assert np.array_equal(L, FIX["w6z_L"]) and np.array_equal(H, FIX["w6z_H"])
    assert np.array_equal(S.view(np.uint16), FIX["w6z_S"].view(np.uint16))


def test_w6_gemv_semantics():
    for m in (3, 16):
        y = O.w6_linear(x_of(f"x{m}_k512"), FIX["w6_L"], FIX["w6_H"], FIX["w6_S"])
        assert close(y, FIX[f"w6_y{m}"])


def test_nv4_quantizer_bit_exact():
    P, S, gs = O.quantize_nv4(FIX["nv4_w"])
    assert np.array_equal(P, FIX["nv4_P"]) and np.array_equal(S, FIX["nv4_S"])
    assert gs == float(FIX["nv4_gs"])


def test_nv4_dequant_and_gemv():
    d = O.dequant_nv4(FIX["nv4_P"], FIX["nv4_S"], float(FIX["nv4_gs"]))
    assert np.array_equal(d, FIX["nv4_deq"])
    y = O.nv4_linear(x_of("x3_k512"), FIX["nv4_P"], FIX["nv4_S"], float(FIX["nv4_gs"]))
    assert close(y, FIX["nv4_y3"])


@pytest.mark.parametrize("grp", [16, 32])
def test_int2_quantizer_dequant_gemv(grp):
    P, S = O.quantize_int2(FIX[f"i2g{grp}_w"], group=grp)
    assert np.array_equal(P, FIX[f"i2g{grp}_P"])
    assert np.array_equal(S.view(np.uint16), FIX[f"i2g{grp}_S"].view(np.uint16))
    assert np.array_equal(O.dequant_int2(P, S), FIX[f"i2g{grp}_deq"])
    y = O.int2_logits(x_of("x3_k512"), P, S)
    assert close(y, FIX[f"i2g{grp}_y3"])


def test_mx8_dequant_and_gemv():
    d = O.mx8_dequant(FIX["mx8_codes"], FIX["mx8_scales"])
    assert np.array_equal(d, FIX["mx8_deq"])
    for m in (3, 16):
        assert close(O.mx8_linear(x_of(f"x{m}_k512"), FIX["mx8_codes"], FIX["mx8_scales"]), FIX[f"mx8_y{m}"])


def test_interleave_up_permutation():
    q = np.arange(128, dtype=np.int64).reshape(-1, 1)
    qo, _ = O.interleave_up(q, q, 4, 8)
    assert np.array_equal(qo[:, 0], FIX["ileave_perm"])


def test_mx8_packer_roundtrip():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((32, 256)) * 0.02).astype(np.float32)
    w[0, :32] = 0.0
    codes, sc = O.quantize_mx8(w)
    d = O.mx8_dequant(codes, sc)
    # every 32-group's largest code is within one e4m3 step of 448, and the dequant error is within e4m3 rounding
    amax = np.abs(w.reshape(32, 8, 32)).max(-1)
    assert np.all(sc[amax == 0] == 0)
    rel = np.abs(d - w).reshape(32, 8, 32).max(-1) / np.maximum(amax, 1e-30)
    assert rel.max() <= 2.0 ** -4 + 1e-7
    assert np.all(np.abs(O.e4m3_decode(codes)) <= 448)


def test_bf16_rounding_nearest_even():
    vals = np.array([1.0, 1.00390625, 1.0078125, 1.01171875, -3.0e38, 1e-40], dtype=np.float32)
    got = O.bf16(vals)
    assert got[0] == 1.0 and got[1] == 1.0 and got[2] == 1.0078125 and got[3] == 1.015625
    assert np.isfinite(got[4]) and got[5] == O.bf16(np.float32(1e-40))


def test_e4m3_encode_matches_table_roundtrip():
    codes = np.arange(0, 256, dtype=np.uint8)
    vals = O.e4m3_decode(codes)
    fin = np.isfinite(vals)
    enc = O.e4m3_encode(vals[fin])
    # +0/-0 both encode; everything else round-trips to the same code
    assert np.array_equal(O.e4m3_decode(enc), vals[fin])
