"""GPU parity of the tcgen05 NVFP4 GEMV (shapes with M <= 8 tokens and at least 8,192 rows take the block-scaled
tensor-core kernel; the others take the register-decode kernel, covered in test_gpu_gemv.py).

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


@pytest.mark.parametrize("m", [1, 3, 5, 8])
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
