"""GPU parity of the tcgen05 NVFP4 and MXFP8 GEMVs (shapes with at least 8,192 rows and M <= 16 tokens take the
block-scaled tensor-core kernel; the others take the register-decode kernel, covered in test_gpu_gemv.py).

The tensor-core kernel multiplies the stored e2m1 weights and e4m3 scales exactly and writes each activation as six
e2m1 terms with e4m3 block scales; what the terms leave out is below 9e-5 of the token's largest element.
Tolerances (max |out - ref| / max |ref|, the reference tuners' metric, x/probes/tune.py:42): fp32 outputs 2e-4,
bf16 outputs 1e-2 (the dense-GEMV bound).
"""
import numpy as np
import pytest
import torch

import fp4x_kernels as F
from oracle import fp4x_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
K = 2560


def rel_err(out, ref):
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return np.abs(out - ref).max() / max(np.abs(ref).max(), 1e-30)


@pytest.fixture(scope="module")
def nv4_weights():
    g = torch.Generator().manual_seed(31)
    n = 16384 + 64  # a partial last row block
    w = torch.randn(n, K, generator=g) * 0.02
    P, S, gs = F.quantize_nv4(w)
    return P, S, gs, O.nv4_weights(P.numpy(), S.view(torch.uint8).numpy()).astype(np.float64)


@pytest.fixture(scope="module")
def nv4_weights_16384():
    g = torch.Generator().manual_seed(32)
    w = torch.randn(16384, K, generator=g) * 0.02  # 128 row tiles: the activation terms are shared by clusters
    P, S, gs = F.quantize_nv4(w)
    return P, S, gs, O.nv4_weights(P.numpy(), S.view(torch.uint8).numpy()).astype(np.float64)


@pytest.mark.parametrize("m", range(1, 9))
def test_nv4_tc_clustered_terms_match_oracle(nv4_weights_16384, m):
    """16384 rows (the C2 / C5 shape): 128 CTAs in clusters that prepare the activation terms once per cluster."""
    P, S, gs, wdeq = nv4_weights_16384
    g = torch.Generator().manual_seed(400 + m)
    x = torch.randn(m, K, generator=g).to(torch.bfloat16)
    ref = (x.double().numpy() @ wdeq.T) * np.float64(np.float32(gs))
    Pd, Sd, xd = P.to(DEV), S.to(DEV), x.to(DEV)
    y32 = F.nv4_linear(xd, Pd, Sd, gs, out_dtype=torch.float32).cpu()
    assert rel_err(y32, ref) < 2e-4
    assert torch.equal(F.nv4_linear(xd, Pd, Sd, gs, out_dtype=torch.float32).cpu(), y32)


@pytest.mark.parametrize("m", [9, 11, 12, 13, 16])
def test_nv4_tc_16_tokens_matches_oracle(nv4_weights, nv4_weights_16384, m):
    """9..16 tokens (C2(c) at M = 16) on the 12- and 16-token kernels: activations read through L2, the tokens
    beyond M are zero blocks, the epilogue folds the term columns chunk by chunk."""
    for P, S, gs, wdeq in (nv4_weights, nv4_weights_16384):
        g = torch.Generator().manual_seed(500 + m)
        x = torch.randn(m, K, generator=g).to(torch.bfloat16)
        x[m // 2] *= 300.0  # one token far larger than the others: each token keeps its own pre-scale
        ref = (x.double().numpy() @ wdeq.T) * np.float64(np.float32(gs))
        Pd, Sd, xd = P.to(DEV), S.to(DEV), x.to(DEV)
        y32 = F.nv4_linear(xd, Pd, Sd, gs, out_dtype=torch.float32).cpu()
        for i in range(m):  # per token: the bound is relative to the token's own largest output
            assert rel_err(y32[i], ref[i]) < 2e-4, i
        yb = F.nv4_linear(xd, Pd, Sd, gs).cpu()
        assert rel_err(yb.float(), ref) < 1e-2
        # a strided activation view (rows of a wider buffer) gives the same bits
        xw = torch.zeros(m, K + 64, dtype=torch.bfloat16, device=DEV)
        xw[:, :K] = xd
        assert torch.equal(F.nv4_linear(xw[:, :K], Pd, Sd, gs, out_dtype=torch.float32).cpu(), y32)


@pytest.mark.parametrize("m", range(1, 9))
def test_nv4_tc_matches_oracle(nv4_weights, m):
    P, S, gs, wdeq = nv4_weights
    g = torch.Generator().manual_seed(100 + m)
    x = torch.randn(m, K, generator=g).to(torch.bfloat16)
    ref = (x.double().numpy() @ wdeq.T) * np.float64(np.float32(gs))
    Pd, Sd, xd = P.to(DEV), S.to(DEV), x.to(DEV)
    y32 = F.nv4_linear(xd, Pd, Sd, gs, out_dtype=torch.float32).cpu()
    assert rel_err(y32, ref) < 2e-4
    y16 = F.nv4_linear(xd, Pd, Sd, gs).float().cpu()
    assert rel_err(y16, ref) < 1e-2
    # deterministic
    assert torch.equal(F.nv4_linear(xd, Pd, Sd, gs, out_dtype=torch.float32).cpu(), y32)


def test_nv4_tc_dynamic_range_and_zero_token(nv4_weights):
    P, S, gs, wdeq = nv4_weights
    g = torch.Generator().manual_seed(7)
    x = torch.randn(4, K, generator=g) * 1e-2
    x[0, ::97] = 300.0          # a few large elements
    x[1] *= 1e-6                # a tiny token
    x[2] = 0.0                  # an all-zero token
    x[3, :16] = 0.0             # an all-zero 16-block
    x = x.to(torch.bfloat16)
    ref = (x.double().numpy() @ wdeq.T) * np.float64(np.float32(gs))
    y = F.nv4_linear(x.to(DEV), P.to(DEV), S.to(DEV), gs, out_dtype=torch.float32).cpu().numpy()
    for r in (0, 1, 3):
        assert rel_err(y[r], ref[r]) < 2e-4, r
    assert np.all(y[2] == 0.0)


# ----------------------------------------------------------------------------------------------------------
# MXFP8 (kind::mxf8f6f4): e4m3 weights with e8m0 scales consumed as stored; activations as four e4m3 terms with
# power-of-two scales per 32 elements (what they leave out is below 2^-15 of each block's largest element)
# ----------------------------------------------------------------------------------------------------------

@pytest.fixture(scope="module")
def mx8_weights():
    g = torch.Generator().manual_seed(41)
    n = 16384 + 64
    w = torch.randn(n, K, generator=g) * 0.02
    codes, sc = F.quantize_mx8(w)
    return codes, sc, O.mx8_dequant(codes.view(torch.uint8).numpy(), sc.numpy()).astype(np.float64)


@pytest.mark.parametrize("m", range(1, 9))
def test_mx8_tc_matches_oracle(mx8_weights, m):
    codes, sc, wdeq = mx8_weights
    g = torch.Generator().manual_seed(200 + m)
    x = torch.randn(m, K, generator=g).to(torch.bfloat16)
    ref = x.double().numpy() @ wdeq.T
    cd, sd, xd = codes.to(DEV), sc.to(DEV), x.to(DEV)
    y32 = F.mx8_linear(xd, cd, sd, None, out_dtype=torch.float32).cpu()
    assert rel_err(y32, ref) < 2e-4
    y16 = F.mx8_linear(xd, cd, sd, None).float().cpu()
    assert rel_err(y16, ref) < 1e-2
    assert torch.equal(F.mx8_linear(xd, cd, sd, None, out_dtype=torch.float32).cpu(), y32)


@pytest.mark.parametrize("m", [9, 12, 13, 16])
def test_mx8_tc_16_tokens_matches_oracle(mx8_weights, m):
    """9..16 tokens on the 12- / 16-token kernels (activations read through L2, chunked epilogue), with a zero token
    and a tiny one among them."""
    codes, sc, wdeq = mx8_weights
    g = torch.Generator().manual_seed(600 + m)
    x = torch.randn(m, K, generator=g)
    x[1] = 0.0
    x[m - 1] *= 1e-6
    x = x.to(torch.bfloat16)
    ref = x.double().numpy() @ wdeq.T
    cd, sd, xd = codes.to(DEV), sc.to(DEV), x.to(DEV)
    y32 = F.mx8_linear(xd, cd, sd, None, out_dtype=torch.float32).cpu()
    for i in range(m):
        if i == 1:
            assert torch.all(y32[1] == 0.0)
        else:
            assert rel_err(y32[i], ref[i]) < 2e-4, i
    y16 = F.mx8_linear(xd, cd, sd, None).float().cpu()
    assert rel_err(y16, ref) < 1e-2
    assert torch.equal(F.mx8_linear(xd, cd, sd, None, out_dtype=torch.float32).cpu(), y32)


def test_mx8_tc_dynamic_range_and_zero_token(mx8_weights):
    codes, sc, wdeq = mx8_weights
    g = torch.Generator().manual_seed(9)
    x = torch.randn(4, K, generator=g) * 1e-2
    x[0, ::97] = 3000.0
    x[1] *= 1e-8
    x[2] = 0.0
    x[3, :32] = 0.0
    x = x.to(torch.bfloat16)
    ref = x.double().numpy() @ wdeq.T
    y = F.mx8_linear(x.to(DEV), codes.to(DEV), sc.to(DEV), None, out_dtype=torch.float32).cpu().numpy()
    for r in (0, 1, 3):
        assert rel_err(y[r], ref[r]) < 2e-4, r
    assert np.all(y[2] == 0.0)


# ----------------------------------------------------------------------------------------------------------
# INT2 head logits (kind::f16, A operand decoded into tensor memory): the decoded weights are the reference's
# bf16((code - 1.5) * s) exactly, so the only difference from the oracle's exact sums is fp32 accumulation
# (the bound of the register-decode kernel's test, 5e-5 of max |ref|, applies unchanged).
# ----------------------------------------------------------------------------------------------------------

@pytest.fixture(scope="module")
def int2_weights():
    g = torch.Generator().manual_seed(51)
    n = 16384 + 64  # a partial last tile
    w = torch.randn(n, K, generator=g) * 0.02
    P, S = F.quantize_int2(w, group=16)
    return P, S


@pytest.mark.parametrize("m", [1, 3, 8, 16])
def test_int2_tc_matches_oracle(int2_weights, m):
    P, S = int2_weights
    n = P.shape[0]
    g = torch.Generator().manual_seed(300 + m)
    x = torch.randn(m, K, generator=g).to(torch.bfloat16)
    ref = O.int2_logits(x.float().numpy(), P.numpy(), S.numpy())
    Pd, Sd, xd = P.to(DEV), S.to(DEV), x.to(DEV)
    ob = torch.empty((m, n), dtype=torch.bfloat16, device=DEV)
    out = F.int2_logits(xd, Pd, Sd, n, out_bf16=ob)
    assert rel_err(out.cpu(), ref) < 5e-5
    assert torch.equal(ob, out.to(torch.bfloat16))
    assert torch.equal(F.int2_logits(xd, Pd, Sd, n), out)  # deterministic


def test_int2_tc_rows_independent_of_tile_position(int2_weights):
    """A row's logit does not depend on where its 128-row tile starts: a vocabulary shard that starts mid-tile gives
    the same bits as the whole head (what the sharded head's merge relies on)."""
    P, S = int2_weights
    x = torch.randn(3, K, generator=torch.Generator().manual_seed(77)).to(torch.bfloat16).to(DEV)
    Pd, Sd = P.to(DEV), S.to(DEV)
    n = P.shape[0]
    full = F.int2_logits(x, Pd, Sd, n)
    part = F.int2_logits(x, Pd[64:], Sd[64:], n - 64)
    assert torch.equal(part, full[:, 64:])


@pytest.mark.parametrize("grp,k", [(32, 2560), (16, 4096), (32, 4096)])
def test_int2_tc_groups_and_depths(grp, k):
    g = torch.Generator().manual_seed(61 + k + grp)
    n = 8192
    w = torch.randn(n, k, generator=g) * 0.02
    P, S = F.quantize_int2(w, group=grp)
    x = torch.randn(3, k, generator=g).to(torch.bfloat16)
    ref = O.int2_logits(x.float().numpy(), P.numpy(), S.numpy())
    out = F.int2_logits(x.to(DEV), P.to(DEV), S.to(DEV), n)
    assert rel_err(out.cpu(), ref) < 5e-5
