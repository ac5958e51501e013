"""GPU parity of the decode GEMVs and the hyper-connection mixer against the CPU oracle.

Tolerances (max |out - ref| / max |ref|, the metric of the reference's tuners, x/probes/tune.py:42):
* fp32 outputs of formats whose weights the kernels form exactly like the reference (MXFP8, NVFP4, BF16, INT2):
  5e-5 (fp32 summation order only);
* W8 / W6 (group scale applied to the fp32 group sum instead of to each bf16 weight): 1e-2, the north-star bound;
* bf16 outputs: 1e-2.
"""
import numpy as np
import pytest
import torch

import fp4x_kernels as F
import fp4x_native as N
from oracle import fp4x_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel_err(out, ref):
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return np.abs(out - ref).max() / max(np.abs(ref).max(), 1e-30)


def gen(seed, *shape, std=1.0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g) * std


def xbf(seed, m, k):
    return gen(seed, m, k).to(torch.bfloat16)


def xnp(x):
    return x.float().numpy()


def check_counters_zero():
    for buf in N._counters.values():
        assert int(buf.abs().sum().item()) == 0, "arrival counters must return to zero"


SHAPES = [(100, 512), (2560, 2560), (512, 2560), (2560, 4096)]
MS = [1, 3, 8, 9, 16]


@pytest.mark.parametrize("n,k", SHAPES)
@pytest.mark.parametrize("m", MS)
def test_mx8(n, k, m):
    w = gen(0, n, k, std=0.02)
    codes, sc = F.quantize_mx8(w)
    x = xbf(1, m, k)
    ref = O.mx8_linear(xnp(x), codes.view(torch.uint8).numpy(), sc.numpy())
    out = F.mx8_linear(x.to(DEV), codes.to(DEV), sc.to(DEV), None, out_dtype=torch.float32)
    assert rel_err(out.cpu(), ref) < 5e-5
    outb = F.mx8_linear(x.to(DEV), codes.to(DEV), sc.to(DEV), None)
    assert outb.dtype == torch.bfloat16 and rel_err(outb.float().cpu(), ref) < 1e-2
    check_counters_zero()


@pytest.mark.parametrize("n,k", SHAPES + [(64, 320)])
@pytest.mark.parametrize("m", MS)
def test_w8(n, k, m):
    w = gen(2, n, k, std=0.02)
    q, s = F.quantize_w8(w)
    x = xbf(3, m, k)
    ref = O.w8_linear(xnp(x), q.numpy(), s.numpy())
    out = F.w8_linear(x.to(DEV), q.to(DEV), s.to(DEV), None, out_dtype=torch.float32)
    assert rel_err(out.cpu(), ref) < 1e-2
    # against the exact-scale product (what the kernel computes) the error is fp32 summation only
    exact = np.asarray(xnp(x), np.float64) @ (q.numpy().astype(np.float64).reshape(n, k // 64, 64) *
                                              s.numpy()[..., None].astype(np.float64)).reshape(n, k).T
    assert rel_err(out.cpu(), exact) < 5e-5
    check_counters_zero()


@pytest.mark.parametrize("n,k", SHAPES)
@pytest.mark.parametrize("m", MS)
def test_w6(n, k, m):
    w = gen(4, n, k, std=0.02)
    L, H, S = F.quantize_w6(w)
    x = xbf(5, m, k)
    ref = O.w6_linear(xnp(x), L.numpy(), H.numpy(), S.numpy())
    out = F.w6_linear(x.to(DEV), L.to(DEV), H.to(DEV), S.to(DEV), None, out_dtype=torch.float32)
    assert rel_err(out.cpu(), ref) < 1e-2
    qv = O.w6_codes(L.numpy(), H.numpy()).astype(np.float64).reshape(n, k // 32, 32)
    exact = np.asarray(xnp(x), np.float64) @ (qv * S.numpy().astype(np.float64)[..., None]).reshape(n, k).T
    assert rel_err(out.cpu(), exact) < 5e-5
    check_counters_zero()


@pytest.mark.parametrize("n,k", SHAPES)
@pytest.mark.parametrize("m", MS)
def test_nv4(n, k, m):
    w = gen(6, n, k, std=0.02)
    P, S, gs = F.quantize_nv4(w)
    x = xbf(7, m, k)
    ref = O.nv4_linear(xnp(x), P.numpy(), S.view(torch.uint8).numpy(), gs)
    out = F.nv4_linear(x.to(DEV), P.to(DEV), S.to(DEV), gs, out_dtype=torch.float32)
    assert rel_err(out.cpu(), ref) < 5e-5
    check_counters_zero()


@pytest.mark.parametrize("n,k", [(100, 512), (2560, 2560), (512, 4096)])
@pytest.mark.parametrize("m", [1, 3, 16])
def test_bf16(n, k, m):
    w = gen(8, n, k, std=0.02).to(torch.bfloat16)
    x = xbf(9, m, k)
    ref = O.bf16_linear(xnp(x), w.float().numpy())
    out = F.bf16_linear(x.to(DEV), w.to(DEV), None, out_dtype=torch.float32)
    assert rel_err(out.cpu(), ref) < 5e-5


@pytest.mark.parametrize("n,k,grp", [(1000, 2560, 16), (4096, 2560, 32), (256, 512, 16)])
@pytest.mark.parametrize("m", [1, 3, 16])
def test_int2_logits(n, k, grp, m):
    w = gen(10, n, k, std=0.02)
    P, S = F.quantize_int2(w, group=grp)
    x = xbf(11, m, k)
    ref = O.int2_logits(xnp(x), P.numpy(), S.numpy())
    out = F.int2_logits(x.to(DEV), P.to(DEV), S.to(DEV), n)
    assert out.dtype == torch.float32
    assert rel_err(out.cpu(), ref) < 5e-5
    ob = torch.empty((m, n), dtype=torch.bfloat16, device=DEV)
    out2 = F.int2_logits(x.to(DEV), P.to(DEV), S.to(DEV), n, out_bf16=ob)
    assert torch.equal(ob, out2.to(torch.bfloat16))


def test_edge_cases_m0_large_m_strided_and_dtypes():
    n, k = 300, 1024
    w = gen(12, n, k, std=0.02)
    codes, sc = F.quantize_mx8(w)
    cw, cs = codes.to(DEV), sc.to(DEV)
    # M = 0
    assert F.mx8_linear(torch.empty(0, k, dtype=torch.bfloat16, device=DEV), cw, cs, None).shape == (0, n)
    # M = 40 (> 16) runs in chunks of 16
    x = xbf(13, 40, k)
    ref = O.mx8_linear(xnp(x), codes.view(torch.uint8).numpy(), sc.numpy())
    assert rel_err(F.mx8_linear(x.to(DEV), cw, cs, None, out_dtype=torch.float32).cpu(), ref) < 5e-5
    # strided activations (a column slice of a wider buffer)
    wide = xbf(14, 5, 2 * k).to(DEV)
    xs = wide[:, :k]
    ref = O.mx8_linear(xnp(xs.cpu()), codes.view(torch.uint8).numpy(), sc.numpy())
    assert rel_err(F.mx8_linear(xs, cw, cs, None, out_dtype=torch.float32).cpu(), ref) < 5e-5
    # f16 output
    o16 = F.mx8_linear(xs, cw, cs, None, out_dtype=torch.float16)
    assert o16.dtype == torch.float16 and rel_err(o16.float().cpu(), ref) < 1e-2


def test_large_and_tiny_activations_are_exact():
    """Activations spanning many binades: the per-token power-of-two f16 scaling keeps products exact."""
    n, k = 256, 2560
    w = gen(15, n, k, std=0.02)
    codes, sc = F.quantize_mx8(w)
    x = xbf(16, 4, k)
    x[0] *= 3.0e4
    x[1] *= 1.0e-6
    x[2, :64] = 1.0e5
    ref = O.mx8_linear(xnp(x), codes.view(torch.uint8).numpy(), sc.numpy())
    out = F.mx8_linear(x.to(DEV), codes.to(DEV), sc.to(DEV), None, out_dtype=torch.float32).cpu()
    for r in range(4):
        assert rel_err(out[r:r + 1], ref[r:r + 1]) < 5e-5, r


def test_c_abi_rejects_bad_arguments():
    x = torch.zeros(3, 512, dtype=torch.bfloat16, device=DEV)
    q = torch.zeros(64, 512, dtype=torch.int8, device=DEV)
    s = torch.ones(64, 8, dtype=torch.float32, device=DEV)
    with pytest.raises(N.Fp4xError):  # M > 16 through the raw ABI
        out = torch.empty(17, 64, dtype=torch.bfloat16, device=DEV)
        N.call("fp4x_w8_linear", N.ptr(x), 512, N.ptr(q), N.ptr(s), N.ptr(out), 64, 0, 17, 64, 512, None, 0, None,
               0, N.stream_of(x))
    with pytest.raises(N.Fp4xError):  # K not a multiple of 64
        out = torch.empty(3, 64, dtype=torch.bfloat16, device=DEV)
        N.call("fp4x_w8_linear", N.ptr(x), 512, N.ptr(q), N.ptr(s), N.ptr(out), 64, 0, 3, 64, 500, None, 0, None,
               0, N.stream_of(x))
    with pytest.raises(N.Fp4xError):  # bad dtype code
        N.call("fp4x_w8_linear", N.ptr(x), 512, N.ptr(q), N.ptr(s), N.ptr(out), 64, 7, 3, 64, 512, None, 0, None,
               0, N.stream_of(x))
    assert N.device_error() == 0


def test_router_gate_batch():
    m, n, k, cnt = 3, 512, 2560, 48
    qs, ss, xs, refs = [], [], [], []
    for i in range(cnt):
        q, s = F.quantize_w8(gen(100 + i, n, k, std=0.02))
        x = xbf(200 + i, m, k)
        refs.append(O.w8_linear(xnp(x), q.numpy(), s.numpy()))
        qs.append(q.to(DEV)); ss.append(s.to(DEV)); xs.append(x.to(DEV))
    batch = F.W8Batch(xs, qs, ss, out_dtype=torch.float32)
    outs = batch.run()
    for o, r in zip(outs, refs):
        assert rel_err(o.cpu(), r) < 1e-2
    outs2 = batch.run()
    assert all(torch.equal(a, b) for a, b in zip(outs, outs2))
    check_counters_zero()


# ----------------------------------------------------------------------------------------------------------
# hyper-connection mixer
# ----------------------------------------------------------------------------------------------------------

def mixer_case(m, synthetic=True, seed=20):
    hc, H = 4, 2560
    if synthetic:
        nd, lr = 512, 512
    else:
        nd, lr = 336, 320
    kd = hc * H
    wd = gen(seed, nd, kd, std=0.02)
    wu = gen(seed + 1, hc * H, lr, std=0.02)
    x = xbf(seed + 2, m, kd)
    qd, sd = F.quantize_w8(wd)
    qu, su = F.quantize_w8(wu)
    return dict(hc=hc, H=H, nd=nd, lr=lr, x=x, qd=qd, sd=sd, qu=qu, su=su)


@pytest.mark.parametrize("m", [1, 3, 16])
@pytest.mark.parametrize("synthetic", [True, False])
def test_hc_fused_equals_unfused_and_oracle(m, synthetic):
    c = mixer_case(m, synthetic)
    hc, lr = c["hc"], c["lr"]
    x = c["x"].to(DEV)
    qd, sd, qu, su = (c[k].to(DEV) for k in ("qd", "sd", "qu", "su"))
    fx = F.HCFused(DEV, n_down=c["nd"])
    qi, si = F.HCFused.interleave_up(qu, su, hc, 8)
    di, bot = fx.down(x, qd, sd, lr, hc)
    out = F.HCFused.up(bot, qi, si, x, hc, (8, 64, 8))
    di_u, bot_u, out_u = F.hc_mixer_unfused(x, qd, sd, qu, su, lr, hc)
    assert torch.equal(di, di_u) and torch.equal(bot, bot_u) and torch.equal(out, out_u)
    # oracle: reference rounding points; the W8 GEMVs differ by the bf16 rounding of the weights
    odi, obot, oout = O.hc_mixer(xnp(c["x"]), c["qd"].numpy(), c["sd"].numpy(), c["qu"].numpy(), c["su"].numpy(),
                                 lr, hc)
    assert rel_err(di.float().cpu(), odi) < 1e-2
    assert rel_err(bot.float().cpu(), obot) < 1e-2
    assert rel_err(out.float().cpu(), oout) < 1e-2
    # the same epilogues applied to the kernel's own down output are exact up to one bf16 step
    _, ebot = O.hc_down_epilogue(di.float().cpu().numpy(), lr, hc)
    assert np.abs(ebot - bot.float().cpu().numpy()).max() <= np.abs(ebot).max() * 2.0 ** -7
    # repeat: deterministic, counters clean
    di2, bot2 = fx.down(x, qd, sd, lr, hc)
    assert torch.equal(di, di2) and torch.equal(bot, bot2)
    check_counters_zero()
    if not synthetic:
        inj = di[:, lr:lr + hc]
        assert inj.shape == (m, hc)
