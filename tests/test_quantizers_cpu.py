"""The plugin's weight-preparation functions (torch, run here on CPU) must produce the reference's packed bytes
bit for bit: checked against the golden fixtures generated from the reference's own quantizers."""
import os

import numpy as np
import pytest
import torch

import fp4x_kernels as F
from oracle import fp4x_oracle as O

FIX = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_fixtures.npz"))


def T(a):
    return torch.from_numpy(np.ascontiguousarray(a))


def test_quantize_w8_matches_reference():
    q, s = F.quantize_w8(T(FIX["w8_w"]))
    assert np.array_equal(q.numpy(), FIX["w8_q"]) and np.array_equal(s.numpy(), FIX["w8_s"])
    q, s = F.quantize_w8(T(FIX["w8k320_w"]))
    assert np.array_equal(q.numpy(), FIX["w8k320_q"]) and np.array_equal(s.numpy(), FIX["w8k320_s"])


@pytest.mark.parametrize("case", ["w6", "w6z"])
def test_quantize_w6_matches_reference(case):
    L, H, S = F.quantize_w6(T(FIX[f"{case}_w"]))
    assert np.array_equal(L.numpy(), FIX[f"{case}_L"]) and np.array_equal(H.numpy(), FIX[f"{case}_H"])
    assert np.array_equal(S.numpy().view(np.uint16), FIX[f"{case}_S"].view(np.uint16))


def test_quantize_w6_awq_matches_reference():
    torch.manual_seed(1234)
    L, H, S, it = F.quantize_w6_awq(T(FIX["awq_w"]), T(FIX["awq_h"]), 31, 0, -1.0)
    assert F._AWQ_LOG[-1] == float(FIX["awq_alpha"])
    assert np.array_equal(L.numpy(), FIX["awq_L"]) and np.array_equal(H.numpy(), FIX["awq_H"])
    assert np.array_equal(S.numpy().view(np.uint16), FIX["awq_S"].view(np.uint16))
    assert np.array_equal(it.view(torch.int16).numpy().view(np.uint16), FIX["awq_invt"])


def test_quantize_nv4_and_dequant_match_reference():
    P, S, gs = F.quantize_nv4(T(FIX["nv4_w"]))
    assert np.array_equal(P.numpy(), FIX["nv4_P"])
    assert np.array_equal(S.view(torch.uint8).numpy(), FIX["nv4_S"])
    assert gs == float(FIX["nv4_gs"])
    d = F.dequant_nv4(P, S, gs)
    assert np.array_equal(d.numpy(), FIX["nv4_deq"])


@pytest.mark.parametrize("grp", [16, 32])
def test_quantize_int2_and_dequant_match_reference(grp):
    P, S = F.quantize_int2(T(FIX[f"i2g{grp}_w"]), group=grp)
    assert np.array_equal(P.numpy(), FIX[f"i2g{grp}_P"])
    assert np.array_equal(S.numpy().view(np.uint16), FIX[f"i2g{grp}_S"].view(np.uint16))
    assert np.array_equal(F.dequant_int2(P, S).numpy(), FIX[f"i2g{grp}_deq"])


def test_mx8_dequant_matches_reference():
    w = T(FIX["mx8_codes"]).view(torch.float8_e4m3fn)
    d = F.mx8_dequant(w, T(FIX["mx8_scales"]))
    assert np.array_equal(d.numpy(), FIX["mx8_deq"])
    d2 = F.mx8_dequant(T(FIX["mx8_codes"]), T(FIX["mx8_scales"]))  # uint8 view accepted too
    assert np.array_equal(d2.numpy(), FIX["mx8_deq"])


def test_quantize_mx8_matches_oracle():
    g = torch.Generator().manual_seed(3)
    w = torch.randn(64, 256, generator=g) * 0.02
    w[1, :32] = 0
    w[2, :32] *= 1e-30
    codes, sc = F.quantize_mx8(w)
    oc, osc = O.quantize_mx8(w.numpy())
    assert np.array_equal(codes.view(torch.uint8).numpy(), oc)
    assert np.array_equal(sc.numpy(), osc)


def test_interleave_up_matches_reference():
    q = torch.arange(128).view(-1, 1).repeat(1, 64).to(torch.int8)
    s = torch.arange(128).view(-1, 1).float()
    _, so = F.HCFused.interleave_up(q, s, 4, 8)
    assert np.array_equal(so[:, 0].long().numpy(), FIX["ileave_perm"])


def test_packed_cache_roundtrip_cpu(tmp_path):
    """PackedCache writes the packed tuple once (safetensors) and loads it back bit for bit, python floats included."""
    w = torch.randn(64, 512, generator=torch.Generator().manual_seed(2)) * 0.02
    cache = F.PackedCache(str(tmp_path), "cpu")
    built = cache.get("blk.0/nv4", lambda: F.quantize_nv4(w))
    assert (tmp_path / "blk.0_nv4.safetensors").exists()
    loaded = cache.get("blk.0/nv4", lambda: pytest.fail("must load from disk"))
    assert isinstance(loaded[2], float) and loaded[2] == built[2]
    assert torch.equal(loaded[0], built[0]) and torch.equal(loaded[1].view(torch.uint8), built[1].view(torch.uint8))


def test_unswizzle_scales_cpu_matches_index_formula():
    n, kb = 256, 32
    sc = torch.arange(n * kb, dtype=torch.int64).remainder(251).to(torch.uint8).view(n, kb)
    out = F.nv4_unswizzle_scales(sc)
    flat = sc.reshape(-1)
    for row in (0, 1, 31, 32, 127, 128, 200, 255):
        for col in (0, 3, 4, 17, 31):
            a, d, c, b, e = row // 128, (row // 32) % 4, row % 32, col // 4, col % 4
            assert out[row, col] == flat[(((a * (kb // 4) + b) * 32 + c) * 4 + d) * 4 + e]


def test_eager_baseline_restatement_matches_oracle():
    """The CPU baseline's torch eager dequantizers (oracle/fp4x_eager.py) equal the numpy oracle's weights."""
    import sys, os
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
    import fp4x_eager as E
    w = torch.randn(64, 512, generator=torch.Generator().manual_seed(4)) * 0.02
    c, s = F.quantize_mx8(w)
    assert np.array_equal(E.mx8_dequant(c, s).numpy(), O.mx8_dequant(c.view(torch.uint8).numpy(), s.numpy()))
    q, s = F.quantize_w8(w)
    assert np.array_equal(E.w8_dequant(q, s).numpy(), O.w8_weights(q.numpy(), s.numpy()))
    L, H, S = F.quantize_w6(w)
    assert np.array_equal(E.w6_dequant(L, H, S).numpy(), O.w6_weights(L.numpy(), H.numpy(), S.numpy()))
    P, S, gs = F.quantize_nv4(w)
    assert np.array_equal(E.nv4_dequant(P, S).numpy(), O.nv4_weights(P.numpy(), S.view(torch.uint8).numpy()))
    P, S = F.quantize_int2(w)
    assert np.array_equal(E.int2_dequant(P, S).numpy(), O.int2_weights(P.numpy(), S.numpy()))
