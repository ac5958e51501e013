"""Weight preparation on the GPU (fp4x_prep.cu) against the reference's quantizers and dequantizers.

* Bit-exact against the golden fixtures, which the reference's own functions produced on the CPU
  (tests/golden/make_golden.py), with the division mode that reproduces the CPU (FP4X_DIV_IEEE).
* Bit-exact against the same torch op sequence run on the GPU (the reference's quantizers applied to CUDA tensors,
  restated in fp4x_kernels._torch_*), with the default mode, at the model's shapes.
* Dequantizers exact; the NVFP4 scale un-swizzle and the HC interleave equal their torch index expressions.
"""
import numpy as np
import pytest
import torch

import fp4x_kernels as F
import fp4x_native as N

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLD = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "ref_fixtures.npz"))


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def same(a, b):
    a = a.detach().cpu()
    b = torch.as_tensor(b)
    if a.dtype != b.dtype and a.element_size() == b.element_size():
        b = b.view(a.dtype)
    return torch.equal(a, b.cpu())


def test_w8_matches_fixtures_ieee():
    for key in ("w8", "w8k320"):
        q, s = F.quantize_w8(cuda(GOLD[f"{key}_w"]), div_mode=N.DIV_IEEE)
        assert same(q, GOLD[f"{key}_q"]) and same(s, GOLD[f"{key}_s"])


def test_w6_matches_fixtures_ieee():
    for key in ("w6", "w6z"):
        L, H, S = F.quantize_w6(cuda(GOLD[f"{key}_w"]), div_mode=N.DIV_IEEE)
        assert same(L, GOLD[f"{key}_L"]) and same(H, GOLD[f"{key}_H"]) and same(S, GOLD[f"{key}_S"])


def test_nv4_matches_fixtures_ieee():
    P, S, gs = F.quantize_nv4(cuda(GOLD["nv4_w"]), div_mode=N.DIV_IEEE)
    assert gs == float(GOLD["nv4_gs"])
    assert same(P, GOLD["nv4_P"]) and same(S.view(torch.uint8), GOLD["nv4_S"])
    assert same(F.dequant_nv4(P, S, gs), GOLD["nv4_deq"])


@pytest.mark.parametrize("grp", [16, 32])
def test_int2_matches_fixtures_ieee(grp):
    P, S = F.quantize_int2(cuda(GOLD[f"i2g{grp}_w"]), group=grp, div_mode=N.DIV_IEEE)
    assert same(P, GOLD[f"i2g{grp}_P"]) and same(S, GOLD[f"i2g{grp}_S"])
    assert same(F.dequant_int2(P, S), GOLD[f"i2g{grp}_deq"])


def test_mx8_dequant_matches_fixture():
    out = F.mx8_dequant(cuda(GOLD["mx8_codes"]), cuda(GOLD["mx8_scales"]))
    assert same(out, GOLD["mx8_deq"])


@pytest.fixture(scope="module")
def model_weights():
    g = torch.Generator(device=DEV).manual_seed(5)
    return {"qkvz": torch.randn(16384, 2560, device=DEV, generator=g) * 0.02,
            "out": torch.randn(2560, 4096, device=DEV, generator=g) * 0.02,
            "gate": torch.randn(512, 2560, device=DEV, generator=g).to(torch.bfloat16) * 0.02,
            "head": torch.randn(8192, 2560, device=DEV, generator=g) * 0.02}


def test_native_matches_torch_on_cuda(model_weights):
    """The default division mode gives the bytes of the reference's torch quantizers run on this GPU."""
    w = model_weights
    for key in ("out", "gate"):
        for a, b in zip(F.quantize_w8(w[key]), F._torch_quantize_w8(w[key])):
            assert torch.equal(a, b), key
        for a, b in zip(F.quantize_w6(w[key]), F._torch_quantize_w6(w[key])):
            assert torch.equal(a, b), key
    P, S, gs = F.quantize_nv4(w["qkvz"])
    P2, S2, gs2 = F._torch_quantize_nv4(w["qkvz"])
    assert gs == gs2 and torch.equal(P, P2) and torch.equal(S.view(torch.uint8), S2.view(torch.uint8))
    for grp in (16, 32):
        for a, b in zip(F.quantize_int2(w["head"], group=grp), F._torch_quantize_int2(w["head"], group=grp)):
            assert torch.equal(a, b)


def test_dequantizers_match_torch(model_weights):
    codes, sc = F.quantize_mx8(model_weights["head"])
    assert torch.equal(F.mx8_dequant(codes, sc), F._torch_mx8_dequant(codes, sc))
    P, S, gs = F.quantize_nv4(model_weights["out"])
    assert torch.equal(F.dequant_nv4(P, S, gs), F._torch_dequant_nv4(P, S, gs))
    P, S = F.quantize_int2(model_weights["head"])
    assert torch.equal(F.dequant_int2(P, S), F._torch_dequant_int2(P, S))


def test_unswizzle_and_interleave_match_torch():
    g = torch.Generator(device=DEV).manual_seed(9)
    sc = torch.randint(0, 255, (512, 160), device=DEV, generator=g, dtype=torch.uint8)
    want = sc.reshape(512 // 128, 160 // 4, 32, 4, 4).transpose(1, 3).reshape(512, 160)
    assert torch.equal(F.nv4_unswizzle_scales(sc), want)
    q = torch.randint(-127, 127, (10240, 512), device=DEV, generator=g, dtype=torch.int8)
    s = torch.rand(10240, 8, device=DEV, generator=g)
    qi, si = F.HCFused.interleave_up(q, s, 4, 8)
    perm = torch.arange(10240, device=DEV).view(4, 10240 // 32, 8).transpose(0, 1).reshape(-1)
    assert torch.equal(qi, q.index_select(0, perm)) and torch.equal(si, s.index_select(0, perm))


def test_packed_cache_roundtrip(tmp_path):
    w = torch.randn(256, 512, device=DEV, generator=torch.Generator(device=DEV).manual_seed(3)) * 0.02
    cache = F.PackedCache(str(tmp_path), DEV)
    built = cache.get("layer0.qkvz", lambda: F.quantize_nv4(w))
    loaded = cache.get("layer0.qkvz", lambda: pytest.fail("must load from disk"))
    assert loaded[2] == built[2]
    assert torch.equal(loaded[0], built[0]) and torch.equal(loaded[1].view(torch.uint8), built[1].view(torch.uint8))
