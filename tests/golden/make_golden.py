"""Generate the golden fixtures in this directory by running the reference plugin's own functions on CPU.

The reference kernel library (`x/fp4x_kernels.py` of the reference checkout) imports torch and triton only, so
its quantizers, dequantizers and the `HCFused.interleave_up` row permutation run here without a GPU.  Its Triton
kernels cannot run without a GPU, so the "reference output" of each GEMV is the reference's dequantize-then-matmul
semantics evaluated with torch on CPU: the kernel's bf16 weights (the reference's dequantizer, or the
per-group product the Triton kernel forms at the cited lines) times `x.float()`, as the reference's own tuners do
(`x/probes/tune.py:27,33`).

Run from the repository root:  python tests/golden/make_golden.py path/to/reference/x/fp4x_kernels.py
(or set FP4X_REFERENCE_KERNELS to that path).  The fixtures are committed; this script is only needed to
regenerate them.
"""
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load_ref(path):
    spec = importlib.util.spec_from_file_location("ref_fp4x_kernels", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def bf16_bits(t):
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def main():
    ref_path = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FP4X_REFERENCE_KERNELS")
    if not ref_path:
        raise SystemExit("usage: make_golden.py path/to/reference/x/fp4x_kernels.py (or set FP4X_REFERENCE_KERNELS)")
    R = load_ref(ref_path)
    g = torch.Generator().manual_seed(0)
    out = {}

    def randn(*shape, std=1.0):
        return torch.randn(*shape, generator=g) * std

    # activations, bf16 ~ N(0,1)
    for m in (1, 3, 16):
        out[f"x{m}_k512"] = bf16_bits(randn(m, 512))
    out["x3_k320"] = bf16_bits(randn(3, 320))
    x3 = torch.from_numpy(out["x3_k512"].view(np.int16)).view(torch.bfloat16).float()
    x16 = torch.from_numpy(out["x16_k512"].view(np.int16)).view(torch.bfloat16).float()

    # ---- W8 g64 (K:138-144), weights ~ N(0, 0.02)
    w = randn(96, 512, std=0.02)
    q, s = R.quantize_w8(w)
    out["w8_w"], out["w8_q"], out["w8_s"] = w.numpy(), q.numpy(), s.numpy()
    wk = (q.float().view(96, 8, 64) * s[..., None]).view(96, 512).to(torch.bfloat16).float()  # K:126-129
    out["w8_y3"], out["w8_y16"] = (x3 @ wk.T).numpy(), (x16 @ wk.T).numpy()
    w320 = randn(64, 320, std=0.02)
    q320, s320 = R.quantize_w8(w320)
    out["w8k320_w"], out["w8k320_q"], out["w8k320_s"] = w320.numpy(), q320.numpy(), s320.numpy()

    # ---- W6 g32 (K:179-202)
    w = randn(96, 512, std=0.02)
    L, H, S = R.quantize_w6(w)
    out["w6_w"], out["w6_L"], out["w6_H"], out["w6_S"] = w.numpy(), L.numpy(), H.numpy(), S.numpy()
    lo = torch.stack([L & 15, L >> 4], -1).view(96, 512).int()
    hi = torch.stack([(H >> (2 * R.ORDER[t])) & 3 for t in range(4)], -1).view(96, 512).int()
    qq = (lo | (hi << 4)) - 32  # K:163-167
    wk = (qq.float().view(96, 16, 32) * S.float()[..., None]).view(96, 512).to(torch.bfloat16).float()  # K:170
    out["w6_y3"], out["w6_y16"] = (x3 @ wk.T).numpy(), (x16 @ wk.T).numpy()
    # a small-scale corner: one all-zero row and one tiny row exercise the 6.2e-5 clamp
    wz = randn(8, 64, std=0.02)
    wz[0] = 0
    wz[1] *= 1e-5
    out["w6z_w"] = wz.numpy()
    out["w6z_L"], out["w6z_H"], out["w6z_S"] = [t.numpy() for t in R.quantize_w6(wz)]

    # ---- W6 AWQ quality probe quantizer (K:218-255), seeded randperm
    wa = randn(64, 256, std=0.02)
    ha = randn(256).abs() + 0.1
    torch.manual_seed(1234)
    La, Ha, Sa, it = R.quantize_w6_awq(wa, ha, 31, 0, -1.0)
    out["awq_w"], out["awq_h"] = wa.numpy(), ha.numpy()
    out["awq_L"], out["awq_H"], out["awq_S"] = La.numpy(), Ha.numpy(), Sa.numpy()
    out["awq_invt"] = bf16_bits(it)
    out["awq_alpha"] = np.array(R._AWQ_LOG[-1], dtype=np.float64)

    # ---- NVFP4 (K:277-300, K:420-426)
    w = randn(96, 512, std=0.02)
    P, Sn, gs = R.quantize_nv4(w)
    out["nv4_w"], out["nv4_P"], out["nv4_S"] = w.numpy(), P.numpy(), Sn.view(torch.uint8).numpy()
    out["nv4_gs"] = np.array(gs, dtype=np.float64)
    deq = R.dequant_nv4(P, Sn, gs)
    out["nv4_deq"] = deq.numpy()
    lut = torch.tensor([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6])
    v = torch.stack([lut[(P & 15).long()], lut[(P >> 4).long()]], -1).view(96, 512)
    wk = (v.view(96, 32, 16) * Sn.float()[..., None]).view(96, 512).to(torch.bfloat16).float()  # K:92
    out["nv4_y3"] = ((x3 @ wk.T) * torch.tensor(gs, dtype=torch.float32)).numpy()  # K:94

    # ---- INT2 g16 / g32 (K:330-357)
    for grp in (16, 32):
        w = randn(96, 512, std=0.02)
        P2, S2 = R.quantize_int2(w, group=grp)
        out[f"i2g{grp}_w"], out[f"i2g{grp}_P"], out[f"i2g{grp}_S"] = w.numpy(), P2.numpy(), S2.numpy()
        d = R.dequant_int2(P2, S2)
        out[f"i2g{grp}_deq"] = d.numpy()
        out[f"i2g{grp}_y3"] = (x3 @ d.to(torch.bfloat16).float().T).numpy()  # K:321-322

    # ---- MXFP8: random e4m3 codes and e8m0 exponents 118..125 as in x/probes/tune.py:25-26
    wc = (randn(96, 512) * 0.5).to(torch.float8_e4m3fn)
    se = torch.randint(118, 126, (96, 16), generator=g, dtype=torch.uint8)
    out["mx8_codes"], out["mx8_scales"] = wc.view(torch.uint8).numpy(), se.numpy()
    d = R.mx8_dequant(wc, se)
    out["mx8_deq"] = d.numpy()
    out["mx8_y3"], out["mx8_y16"] = (x3 @ d.T).numpy(), (x16 @ d.T).numpy()

    # ---- HCFused.interleave_up row permutation (K:513-517)
    qi = torch.arange(4 * 32).view(-1, 1).to(torch.int8).repeat(1, 64)
    si = torch.arange(4 * 32).view(-1, 1).float()
    qo, so = R.HCFused.interleave_up(qi, si, 4, 8)
    out["ileave_perm"] = so[:, 0].long().numpy()

    np.savez_compressed(os.path.join(HERE, "ref_fixtures.npz"), **out)
    total = sum(a.nbytes for a in out.values())
    print(f"wrote {len(out)} arrays ({total / 1e3:.0f} kB raw) to {HERE}/ref_fixtures.npz")


if __name__ == "__main__":
    main()
