"""Failure paths on the GPU without a GPU fault: bounded device waits that give up, and concurrent streams.

* A wait that runs out (an mbarrier that no thread arrives on, through the library's production bounded wait with
  a 1 ms limit) records its code in the device error word and returns; the host reads FP4X_ERR_DEVICE, the context
  stays usable and the next calls are correct.
* Calls on different streams get different arrival-counter arrays: three GEMVs that use split-K counters run
  concurrently on three streams for 100 iterations and every result equals the single-stream result bit for bit
  (vLLM overlaps decode linears on two streams, README.md:208 of the reference).
"""
import ctypes

import numpy as np
import pytest
import torch

import fp4x_kernels as F
import fp4x_native as N
from oracle import fp4x_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def gen(seed, *shape, std=1.0):
    return torch.randn(*shape, generator=torch.Generator().manual_seed(seed)) * std


def test_expired_wait_reports_device_error_and_context_survives():
    x = gen(1, 3, 2560).to(torch.bfloat16)
    q, s = F.quantize_w8(gen(2, 512, 2560, std=0.02))
    ref = O.w8_linear(x.float().numpy(), q.numpy(), s.numpy())
    st = N.stream_of(x.to(DEV))
    assert N.device_error() == 0
    assert N.lib().fp4x_test_expire_wait(1000000, st) == 0
    c = ctypes.c_int(0)
    rc = N.lib().fp4x_device_error(st, 0, ctypes.byref(c))  # read without clearing
    assert rc == N.ERR_DEVICE and c.value == 1
    code = N.device_error(clear=True)
    assert code == 1 and N.device_error() == 0
    for b in N.counter_buffers():
        assert int(b.abs().sum().item()) == 0
    out = F.w8_linear(x.to(DEV), q.to(DEV), s.to(DEV), None, out_dtype=torch.float32).cpu().numpy()
    assert np.abs(out - ref).max() / np.abs(ref).max() < 5e-5
    with pytest.raises(N.Fp4xError):
        N.call("fp4x_test_expire_wait", 10, st)  # limit below 1 us is rejected on the host


def test_three_streams_do_not_share_counters():
    m = 3
    x = gen(3, m, 2560).to(torch.bfloat16).to(DEV)
    xw = gen(4, m, 4096).to(torch.bfloat16).to(DEV)
    P, S, gs = F.quantize_nv4(gen(5, 16384, 2560, std=0.02).to(DEV))
    L, H, S6 = F.quantize_w6(gen(6, 2560, 4096, std=0.02).to(DEV))
    q8, s8 = F.quantize_w8(gen(7, 16384, 2560, std=0.02).to(DEV))
    ops = [lambda: F.nv4_linear(x, P, S, gs, out_dtype=torch.float32),
           lambda: F.w6_linear(xw, L, H, S6, None, out_dtype=torch.float32),
           lambda: F.w8_linear(x, q8, s8, None, out_dtype=torch.float32)]
    want = [op() for op in ops]
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream() for _ in ops]
    for st in streams:
        st.wait_stream(torch.cuda.current_stream())
    outs = [[] for _ in ops]
    for _ in range(100):
        for i, (op, st) in enumerate(zip(ops, streams)):
            with torch.cuda.stream(st):
                outs[i].append(op())
    torch.cuda.synchronize()
    for i in range(len(ops)):
        for o in outs[i]:
            assert torch.equal(o, want[i]), f"stream {i} differs from the single-stream result"
    assert N.device_error() == 0
    for b in N.counter_buffers():
        assert int(b.abs().sum().item()) == 0


def test_many_graph_captures_on_fresh_streams():
    """Each capture on a new stream gets counters of its own (spares first, then a buffer allocated inside the
    capture); 40 graphs, more than the stream pool holds, all replay to the eager result."""
    x = gen(8, 3, 2560).to(torch.bfloat16).to(DEV)
    q8, s8 = F.quantize_w8(gen(9, 16384, 2560, std=0.02).to(DEV))
    want = F.w8_linear(x, q8, s8, None, out_dtype=torch.float32)
    graphs, outs = [], []
    for _ in range(40):
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(st):
            with torch.cuda.graph(g, stream=st):
                outs.append(F.w8_linear(x, q8, s8, None, out_dtype=torch.float32))
        torch.cuda.current_stream().wait_stream(st)
        graphs.append(g)
    for g in graphs:
        g.replay()
    torch.cuda.synchronize()
    assert all(torch.equal(o, want) for o in outs)
    assert N.device_error() == 0
