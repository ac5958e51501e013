"""fp4x_mx8_linear_noalloc (static library scratch, no caller workspace), called through the C ABI, against the CPU
oracle and against fp4x_mx8_linear (caller scratch from torch).  Kept in its own file that is collected last.

Tolerances (max |a - b| / max |b|): fp32 output against the oracle's exact sums 5e-5 (fp32 summation only, as for
every dense GEMV); bf16 output against the scratch-taking entry 1e-2.  Two calls in a row are checked, since the
static scratch keeps what the previous call left in it.
"""
import numpy as np
import pytest
import torch

import fp4x_kernels as F
import fp4x_native as N
from oracle import fp4x_oracle as O

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


def noalloc_call(x, w8, s, n=None, dtype=torch.bfloat16):
    m, k = x.shape
    n = w8.shape[0] if n is None else n
    out = torch.empty(m, w8.shape[0], dtype=dtype, device=DEV)
    rc = N.lib().fp4x_mx8_linear_noalloc(N.ptr(x), x.stride(0), N.ptr(w8), N.ptr(s), N.ptr(out), out.stride(0),
                                         N.dtype_code(dtype), m, n, k, N.stream_of(x))
    return rc, out


def case(m, n, k):
    g = torch.Generator().manual_seed(n + k + m)
    w = torch.randn(n, k, generator=g) * 0.02
    codes, sc = F.quantize_mx8(w)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    oracle = O.mx8_linear(x.float().numpy(), codes.view(torch.uint8).numpy(), sc.numpy())
    return x.to(DEV), codes.view(torch.uint8).contiguous().to(DEV), sc.contiguous().to(DEV), oracle


@pytest.mark.parametrize("m", [1, 3, 16])
@pytest.mark.parametrize("n,k", [(16384, 2560), (2560, 2560), (100, 512)])
def test_noalloc_matches_oracle_and_scratch_entry(m, n, k):
    x, w8, s, oracle = case(m, n, k)
    ref = reference_call(x, w8, s)
    for _ in range(2):
        rc, out = noalloc_call(x, w8, s, dtype=torch.float32)
        torch.cuda.synchronize()
        assert rc == 0, N.lib().fp4x_last_error_message().decode()
        got = out.cpu().double().numpy()
        assert np.abs(got - oracle).max() / np.abs(oracle).max() < 5e-5
        rc, outb = noalloc_call(x, w8, s)
        torch.cuda.synchronize()
        assert rc == 0, N.lib().fp4x_last_error_message().decode()
        assert rel(outb, ref) < 1e-2
    assert N.device_error() == 0


def test_noalloc_counters_are_reset_after_a_device_error():
    """A wait that gives up can leave static counters mid-count; clearing the device error word zeroes them.  The
    leftover count is planted on the host (a counter write), the error word is set by a bounded wait that expires on
    purpose (nothing faults), and after the clear the entry point gives the oracle's answer again."""
    x, w8, s, oracle = case(3, 16384, 2560)  # a stream-K plan: its row blocks use the static counters
    st = N.stream_of(x)
    for i in range(4):
        assert N.lib().fp4x_test_set_static_counter(i, 5, st) == 0
    assert N.lib().fp4x_test_expire_wait(1000000, st) == 0
    code = N.device_error(clear=True)
    assert code == 1
    assert N.device_error() == 0
    for _ in range(2):
        rc, out = noalloc_call(x, w8, s, dtype=torch.float32)
        torch.cuda.synchronize()
        assert rc == 0
        got = out.cpu().double().numpy()
        assert np.abs(got - oracle).max() / np.abs(oracle).max() < 5e-5


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
