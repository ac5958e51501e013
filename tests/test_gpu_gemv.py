"""GPU parity of the decode GEMVs and the hyper-connection mixer against the CPU oracle.

Tolerances (max |out - ref| / max |ref|, the metric of the reference's tuners, x/probes/tune.py:42):
* fp32 outputs: 5e-5.  Every format's weights are formed exactly as the reference forms them (MXFP8, NVFP4, BF16,
  INT2 exactly; W8 / W6 as bf16(f32(q) * s) per weight, K:126-130 and K:168-170), so the only difference from the
  oracle's float64 sums is fp32 accumulation;
* bf16 outputs: 1e-2.

The shapes cover every configuration the benchmark quotes (BASELINE C2: K = 2560, N in {2560, 16384}, M in
{1, 2, 4, 8, 16}; C5: W6 2560x4096 and 4096x2560, the 48 router gates 512x2560), each plan kind the planner picks
for them (cluster split-K for small row counts, single-matrix stream-K with workspace partials at 16,384 rows, the
16-token plans that read the raw activation panel from global memory) and small ragged shapes.
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
    for buf in N.counter_buffers():
        assert int(buf.abs().sum().item()) == 0, "arrival counters must return to zero"


SHAPES = [(100, 512), (2560, 2560), (512, 2560), (2560, 4096), (4096, 2560)]
MS = [1, 3, 8, 9, 16]
BIG_MS = [1, 2, 4, 8, 12, 16]


@pytest.fixture(scope="module")
def big_w8():
    w = gen(42, 16384, 2560, std=0.02)
    q, s = F.quantize_w8(w)
    return q, s, O.w8_weights(q.numpy(), s.numpy()).astype(np.float64)


@pytest.fixture(scope="module")
def big_w6():
    w = gen(43, 16384, 2560, std=0.02)
    L, H, S = F.quantize_w6(w)
    return L, H, S, O.w6_weights(L.numpy(), H.numpy(), S.numpy()).astype(np.float64)


@pytest.fixture(scope="module")
def big_mx8():
    # 8,128 rows: below the tensor-core kernel's 8,192-row floor, so 9..16 tokens run the register-decode kernel
    w = gen(44, 8128, 2560, std=0.02)
    codes, sc = F.quantize_mx8(w)
    return codes, sc, O.mx8_dequant(codes.view(torch.uint8).numpy(), sc.numpy()).astype(np.float64)


@pytest.fixture(scope="module")
def big_nv4():
    # 8,128 rows (127 row tiles of 128): below the tensor-core kernel's 8,192-row floor, so 9..16 tokens run the
    # register-decode kernel (16,384 rows at 9..16 tokens are covered in test_gpu_tc.py)
    w = gen(45, 8128, 2560, std=0.02)
    P, S, gs = F.quantize_nv4(w)
    return P, S, gs, O.nv4_weights(P.numpy(), S.view(torch.uint8).numpy()).astype(np.float64)


@pytest.mark.parametrize("m", BIG_MS)
def test_w8_16384x2560(big_w8, m):
    """C2(a) at N = 16384: the single-matrix stream-K plan (partial slots in the workspace, last-arriver sum)."""
    q, s, wdeq = big_w8
    x = xbf(60 + m, m, 2560)
    ref = xnp(x).astype(np.float64) @ wdeq.T
    qd, sd, xd = q.to(DEV), s.to(DEV), x.to(DEV)
    out = F.w8_linear(xd, qd, sd, None, out_dtype=torch.float32)
    assert rel_err(out.cpu(), ref) < 5e-5
    outb = F.w8_linear(xd, qd, sd, None)
    assert rel_err(outb.float().cpu(), ref) < 1e-2
    assert torch.equal(F.w8_linear(xd, qd, sd, None, out_dtype=torch.float32), out)  # deterministic
    check_counters_zero()


@pytest.mark.parametrize("m", BIG_MS)
def test_w6_16384x2560(big_w6, m):
    """C2(b) at N = 16384 (16-token plans keep the raw activation panel in global memory)."""
    L, H, S, wdeq = big_w6
    x = xbf(70 + m, m, 2560)
    ref = xnp(x).astype(np.float64) @ wdeq.T
    Ld, Hd, Sd, xd = L.to(DEV), H.to(DEV), S.to(DEV), x.to(DEV)
    out = F.w6_linear(xd, Ld, Hd, Sd, None, out_dtype=torch.float32)
    assert rel_err(out.cpu(), ref) < 5e-5
    outb = F.w6_linear(xd, Ld, Hd, Sd, None)
    assert rel_err(outb.float().cpu(), ref) < 1e-2
    assert torch.equal(F.w6_linear(xd, Ld, Hd, Sd, None, out_dtype=torch.float32), out)
    check_counters_zero()


@pytest.mark.parametrize("m", [9, 12, 16])
def test_mx8_8128x2560_register_path(big_mx8, m):
    """MXFP8 at 9..16 tokens: the register-decode kernel (16-token plans read the activation panel from L2)."""
    codes, sc, wdeq = big_mx8
    x = xbf(80 + m, m, 2560)
    ref = xnp(x).astype(np.float64) @ wdeq.T
    out = F.mx8_linear(x.to(DEV), codes.to(DEV), sc.to(DEV), None, out_dtype=torch.float32)
    assert rel_err(out.cpu(), ref) < 5e-5
    check_counters_zero()


@pytest.mark.parametrize("m", [9, 12, 16])
def test_nv4_8128x2560_register_path(big_nv4, m):
    """NVFP4 at 9..16 tokens on the register-decode kernel (the 16-token plans)."""
    P, S, gs, wdeq = big_nv4
    x = xbf(90 + m, m, 2560)
    ref = (xnp(x).astype(np.float64) @ wdeq.T) * np.float64(np.float32(gs))
    out = F.nv4_linear(x.to(DEV), P.to(DEV), S.to(DEV), gs, out_dtype=torch.float32)
    assert rel_err(out.cpu(), ref) < 5e-5
    outb = F.nv4_linear(x.to(DEV), P.to(DEV), S.to(DEV), gs)
    assert rel_err(outb.float().cpu(), ref) < 1e-2
    check_counters_zero()


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


@pytest.mark.parametrize("n,k", SHAPES + [(64, 320), (13312, 2560)])
@pytest.mark.parametrize("m", MS + [2, 4])
def test_w8(n, k, m):
    w = gen(2, n, k, std=0.02)
    q, s = F.quantize_w8(w)
    x = xbf(3, m, k)
    ref = O.w8_linear(xnp(x), q.numpy(), s.numpy())
    out = F.w8_linear(x.to(DEV), q.to(DEV), s.to(DEV), None, out_dtype=torch.float32)
    assert rel_err(out.cpu(), ref) < 5e-5
    outb = F.w8_linear(x.to(DEV), q.to(DEV), s.to(DEV), None)
    assert rel_err(outb.float().cpu(), ref) < 1e-2
    check_counters_zero()


def test_w8_weight_rounding_point():
    """One row whose weights differ between bf16(q * s) (the reference, K:126-130) and q * s applied to the group
    sum: a one-hot activation reads a single weight, which must be the reference's bf16 value exactly."""
    n, k = 64, 512
    q = torch.zeros(n, k, dtype=torch.int8)
    q[:, 5] = torch.arange(-32, 32, dtype=torch.int8)
    s = torch.full((n, k // 64), 1.0 / 3.0, dtype=torch.float32)
    x = torch.zeros(1, k, dtype=torch.bfloat16)
    x[0, 5] = 1.0
    out = F.w8_linear(x.to(DEV), q.to(DEV), s.to(DEV), None, out_dtype=torch.float32).cpu().numpy()[0]
    want = O.w8_weights(q.numpy(), s.numpy())[:, 5]
    assert np.array_equal(out, want)
    assert not np.array_equal(out, q.numpy()[:, 5].astype(np.float32) * np.float32(1.0 / 3.0))


def test_w6_weight_rounding_point():
    """W6 codes -32..31 under an fp16 scale with 11 significant bits: each weight is bf16((q - 32) * s) (K:168-170)."""
    n, k = 64, 512
    codes = torch.arange(64, dtype=torch.int32)  # q + 32 for q = -32..31, one per row
    full = torch.full((n, k), 32, dtype=torch.int32)
    full[:, 7] = codes
    lo, hi = full & 15, full >> 4
    L = (lo[:, 0::2] | (lo[:, 1::2] << 4)).to(torch.uint8)
    H = (hi[:, 0::4] | (hi[:, 2::4] << 2) | (hi[:, 1::4] << 4) | (hi[:, 3::4] << 6)).to(torch.uint8)
    S = torch.full((n, k // 32), 0.0123, dtype=torch.float16)
    x = torch.zeros(1, k, dtype=torch.bfloat16)
    x[0, 7] = 1.0
    out = F.w6_linear(x.to(DEV), L.to(DEV), H.to(DEV), S.to(DEV), None, out_dtype=torch.float32).cpu().numpy()[0]
    want = O.w6_weights(L.numpy(), H.numpy(), S.numpy())[:, 7]
    assert np.array_equal(out, want)


@pytest.mark.parametrize("n,k", SHAPES)
@pytest.mark.parametrize("m", MS + [2, 4])
def test_w6(n, k, m):
    w = gen(4, n, k, std=0.02)
    L, H, S = F.quantize_w6(w)
    x = xbf(5, m, k)
    ref = O.w6_linear(xnp(x), L.numpy(), H.numpy(), S.numpy())
    out = F.w6_linear(x.to(DEV), L.to(DEV), H.to(DEV), S.to(DEV), None, out_dtype=torch.float32)
    assert rel_err(out.cpu(), ref) < 5e-5
    outb = F.w6_linear(x.to(DEV), L.to(DEV), H.to(DEV), S.to(DEV), None)
    assert rel_err(outb.float().cpu(), ref) < 1e-2
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


@pytest.mark.parametrize("m", [1, 3, 16])
def test_router_gate_batch(m):
    n, k, cnt = 512, 2560, 48
    qs, ss, xs, refs = [], [], [], []
    for i in range(cnt):
        q, s = F.quantize_w8(gen(100 + i, n, k, std=0.02))
        x = xbf(200 + i, m, k)
        refs.append(O.w8_linear(xnp(x), q.numpy(), s.numpy()))
        qs.append(q.to(DEV)); ss.append(s.to(DEV)); xs.append(x.to(DEV))
    batch = F.W8Batch(xs, qs, ss, out_dtype=torch.float32)
    outs = batch.run()
    for o, r in zip(outs, refs):
        assert rel_err(o.cpu(), r) < 5e-5
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


def bf16_ulp(v):
    """Spacing of bf16 values at |v| (normal range)."""
    v = np.maximum(np.abs(np.asarray(v, dtype=np.float64)), 2.0 ** -126)
    return 2.0 ** (np.floor(np.log2(v)) - 7)


def within_ulps(a, b, n=1):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return bool(np.all(np.abs(a - b) <= n * bf16_ulp(np.maximum(np.abs(a), np.abs(b))) + 1e-30))


@pytest.mark.parametrize("m", [1, 3, 16])
@pytest.mark.parametrize("synthetic", [True, False])
def test_hc_fused_equals_unfused_and_oracle(m, synthetic):
    """The fused mixer against the reference's unfused W8 semantics (P:231-247 with the rounding points of
    K:451-493): every W8 weight is bf16(q * s), so the fp32 sums differ from the oracle's exact ones by fp32
    accumulation alone.  di is within one bf16 step of the oracle; bot and the block input are within one bf16
    step of the oracle's epilogues applied to the kernel's own di / bot (a one-step difference in di moves the
    values computed from it)."""
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
    xn, qdn, sdn, qun, sun = xnp(c["x"]), c["qd"].numpy(), c["sd"].numpy(), c["qu"].numpy(), c["su"].numpy()
    odi, obot, oout = O.hc_mixer(xn, qdn, sdn, qun, sun, lr, hc)
    dik, botk, outk = di.float().cpu().numpy(), bot.float().cpu().numpy(), out.float().cpu().numpy()
    # down projection: fp32 sum of the reference's bf16 weights, rounded once to bf16
    assert within_ulps(dik, odi, 1)
    assert rel_err(dik, odi) < 1e-2 and rel_err(botk, obot) < 1e-2 and rel_err(outk, oout) < 1e-2
    # SiLU epilogue on the kernel's di, and the gate-mean epilogue on the up sums of the kernel's bot
    _, ebot = O.hc_down_epilogue(dik, lr, hc)
    assert within_ulps(botk, ebot, 1)
    g = O.w8_linear(botk, qun, sun)
    eout = O.hc_up_epilogue(g, xn, hc)
    assert within_ulps(outk, eout, 1)
    # repeat: deterministic, counters clean
    di2, bot2 = fx.down(x, qd, sd, lr, hc)
    assert torch.equal(di, di2) and torch.equal(bot, bot2)
    check_counters_zero()
    if not synthetic:
        inj = di[:, lr:lr + hc]
        assert inj.shape == (m, hc)
