"""fp4x_mx8_linear_noalloc (static library scratch, no caller workspace) against fp4x_mx8_linear (caller scratch
from torch), called through the C ABI.  Kept in its own file that is collected last.

Tolerance: max |a - b| / max |b| < 1e-2 (the dense GEMV bound); both calls in a row are checked.
"""
import ctypes

import pytest
import torch

import fp4x_kernels as F
import fp4x_native as N

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def reference_call(x, w8, s):
    m, k = x.shape
    n = w8.shape[0]
    out = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
    ws, cnt = N.scratch(N.FMT_MX8, m, n, k, DEV)
    N.call("fp4x_mx8_linear", N.ptr(x), x.stride(0), N.ptr(w8), N.ptr(s), N.ptr(out), out.stride(0), 0, m, n, k,
           *N.scratch_args(ws, cnt), N.stream_of(x))
    return out


def noalloc_call(x, w8, s, n=None):
    m, k = x.shape
    n = w8.shape[0] if n is None else n
    out = torch.empty(m, w8.shape[0], dtype=torch.bfloat16, device=DEV)
    rc = N.lib().fp4x_mx8_linear_noalloc(N.ptr(x), x.stride(0), N.ptr(w8), N.ptr(s), N.ptr(out), out.stride(0), 0,
                                         m, n, k, N.stream_of(x))
    return rc, out


@pytest.mark.parametrize("m", [1, 3, 16])
@pytest.mark.parametrize("n,k", [(16384, 2560), (2560, 2560), (100, 512)])
def test_noalloc_matches_scratch_entry(m, n, k):
    g = torch.Generator().manual_seed(n + k + m)
    w = (torch.randn(n, k, generator=g) * 0.02).to(DEV)
    codes, sc = F.quantize_mx8(w)
    w8 = codes.view(torch.uint8).contiguous()
    s = sc.contiguous()
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(DEV)
    ref = reference_call(x, w8, s)
    for _ in range(2):
        rc, out = noalloc_call(x, w8, s)
        torch.cuda.synchronize()
        assert rc == 0, N.lib().fp4x_last_error_message().decode()
        assert rel(out, ref) < 1e-2
    assert N.device_error() == 0


def test_noalloc_rejects_shapes_beyond_static_scratch():
    # 2^21 rows at M=16 need 131,072 arrival counters; the static scratch holds 32,768.  The call is rejected on the
    # host before anything is launched, so the small buffers below are never read.
    x = torch.zeros(16, 512, dtype=torch.bfloat16, device=DEV)
    w8 = torch.zeros(64, 512, dtype=torch.uint8, device=DEV)
    s = torch.zeros(64, 16, dtype=torch.uint8, device=DEV)
    n0 = N.launch_count()
    rc, _ = noalloc_call(x, w8, s, n=1 << 21)
    assert rc == N.ERR_WORKSPACE
    assert b"static scratch" in N.lib().fp4x_last_error_message()
    assert N.launch_count() == n0
