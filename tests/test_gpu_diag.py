"""GPU checks of the two additions with no reference counterpart: the L2 prefetch of later weights
(fp4x_prefetch_l2) and the launch timeline diagnostic (fp4x_timeline_begin / fp4x_timeline_end)."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for _p in (_ROOT, os.path.join(_ROOT, "qwen3.8-flash-next-fp4-local-spark_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import fp4x_kernels as F  # noqa: E402
import fp4x_native as N  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_prefetch_leaves_results_and_error_word_alone():
    g = torch.Generator(device=DEV)
    g.manual_seed(5)
    w = torch.randn(4096, 2560, device=DEV, generator=g) * 0.02
    q, s = F.quantize_w8(w)
    x = torch.randn(3, 2560, device=DEV, generator=g).to(torch.bfloat16)
    ref = F.w8_linear(x, q, s)
    raw = torch.empty(1000003, dtype=torch.uint8, device=DEV)
    # whole tensors, an unaligned slice, a strided view, a range shorter than 16 bytes and an empty tensor
    F.prefetch_l2(q, s, raw[3:], raw[7:12], w[:, ::2], torch.empty(0, device=DEV))
    F.prefetch_l2()
    out = F.w8_linear(x, q, s)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert N.device_error(clear=False) == 0


def test_prefetch_rejects_more_than_16_ranges_and_host_tensors():
    t = torch.empty(64, device=DEV)
    with pytest.raises(N.Fp4xError):
        F.prefetch_l2(*([t] * 17))
    with pytest.raises(ValueError):
        F.prefetch_l2(torch.empty(64))


def _timeline_child():
    N.use_timeline_library()
    g = torch.Generator(device=DEV)
    g.manual_seed(6)
    q, s = F.quantize_w8(torch.randn(4096, 2560, device=DEV, generator=g) * 0.02)
    P, S, gs = F.quantize_nv4(torch.randn(16384, 2560, device=DEV, generator=g) * 0.02)
    x = torch.randn(3, 2560, device=DEV, generator=g).to(torch.bfloat16)
    F.w8_linear(x, q, s)
    F.nv4_linear(x, P, S, gs)
    torch.cuda.synchronize()
    tl = N.Timeline(8, DEV)
    tl.begin()
    a = F.w8_linear(x, q, s)
    b = F.nv4_linear(x, P, S, gs)
    c = F.w8_linear(x, q, s)
    n = tl.end()
    torch.cuda.synchronize()
    assert n == 3
    t = tl.read().astype(np.int64)
    for r in t:
        assert r[N.TL_START_FIRST] <= r[N.TL_START_LAST] and r[N.TL_WAIT_FIRST] <= r[N.TL_WAIT_LAST]
        # start, wait, rows landed, converted, accumulated, stored
        assert (r[N.TL_START_FIRST] <= r[N.TL_WAIT_FIRST] <= r[N.TL_X_LANDED] <= r[N.TL_STAGED] <= r[N.TL_LOOP_DONE]
                <= r[N.TL_STORED])
        assert r[N.TL_FIRST_STAGE] > 0 and r[N.TL_STORED] - r[N.TL_START_FIRST] < 10_000_000_000
    for r in (t[0], t[2]):  # register-decode kernel: k-group handover and the cross-CTA sums come before the store
        assert r[N.TL_LOOP_DONE] <= r[N.TL_HANDOVER] <= r[N.TL_REDUCED] <= r[N.TL_STORED]
    assert t[1, N.TL_HANDOVER] == 0 and t[1, N.TL_REDUCED] == 0  # not stamped by the tensor-core kernel
    # each waits for the one before
    assert t[0, N.TL_STORED] <= t[1, N.TL_WAIT_FIRST] and t[1, N.TL_STORED] <= t[2, N.TL_WAIT_FIRST]
    # the timeline only observes: the results equal an unrecorded run
    assert torch.equal(a, c) and torch.equal(b, F.nv4_linear(x, P, S, gs))
    # uninstalled: later launches take no record
    F.w8_linear(x, q, s)
    assert N.lib().fp4x_timeline_end() == 3


def test_timeline_records_one_launch_per_gemv_in_order():
    """Runs in a child process: the timeline lives in the diagnostic twin library, and this process has loaded
    the product library already."""
    env = dict(os.environ)
    env.pop("FP4X_LIB", None)
    r = subprocess.run([sys.executable, os.path.abspath(__file__)], capture_output=True, text=True, timeout=600,
                       env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "timeline ok" in r.stdout


def test_product_library_has_no_timeline():
    with pytest.raises(N.Fp4xError, match="FP4X_TIMELINE"):
        N.Timeline(4, DEV).begin()


if __name__ == "__main__":
    _timeline_child()
    print("timeline ok")
