"""ctypes binding of libfp4x.so (include/fp4x.h) for the torch host code.

torch provides device memory and the current stream; every call passes raw pointers, integer sizes and the
stream handle to the C ABI.  There is no fallback: if the library is missing or a call fails, a Python exception
is raised.  Scratch memory for split reductions is allocated here through torch's caching allocator (so it is
safe under CUDA-graph capture).  The arrival counters live in persistent zeroed int32 buffers that the kernels
leave zeroed after every call, one per (device, stream): calls issued on different streams may run at the same time
(vLLM overlaps decode linears on two streams) and never share a counter.
"""
from __future__ import annotations

import ctypes
import os
import threading

import numpy as np
import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("FP4X_LIB", os.path.join(_HERE, "libfp4x.so"))
# the diagnostic twin with the launch-timeline stamps compiled in (build_native.py --timeline)
TIMELINE_LIB_PATH = os.path.join(_HERE, "libfp4x_timeline.so")

OK = 0
ERR_INVALID_ARG, ERR_UNSUPPORTED, ERR_WORKSPACE, ERR_CUDA, ERR_DEVICE = -1, -2, -3, -4, -5
FMT_MX8, FMT_W8, FMT_W6, FMT_NV4, FMT_BF16, FMT_INT2 = range(6)
IN_F32, IN_BF16, IN_F16 = range(3)
DIV_IEEE, DIV_RECIP = 0, 1
_DTYPES = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_sz = ctypes.c_size_t
_f32 = ctypes.c_float
_ip = ctypes.POINTER(ctypes.c_int32)


class W8Item(ctypes.Structure):
    """fp4x_w8_item of include/fp4x.h."""
    _fields_ = [("x", ctypes.c_void_p), ("q", ctypes.c_void_p), ("s", ctypes.c_void_p), ("out", ctypes.c_void_p)]

class StepOpC(ctypes.Structure):
    """fp4x_step_op of include/fp4x.h."""
    _fields_ = [("kind", ctypes.c_int), ("x", ctypes.c_void_p), ("x_stride", ctypes.c_int64),
                ("p0", ctypes.c_void_p), ("p1", ctypes.c_void_p), ("s", ctypes.c_void_p), ("gs", ctypes.c_float),
                ("out", ctypes.c_void_p), ("out2", ctypes.c_void_p), ("out_stride", ctypes.c_int64),
                ("out_dtype", ctypes.c_int), ("n", ctypes.c_int64), ("k", ctypes.c_int64), ("lr", ctypes.c_int64),
                ("hc", ctypes.c_int64), ("bj", ctypes.c_int64), ("nrm", ctypes.c_void_p),
                ("nrm_stride", ctypes.c_int64)]


STEP_NV4, STEP_W6, STEP_W8, STEP_HC_DOWN, STEP_HC_UP, STEP_MX8 = range(6)

# argument signatures of every exported entry point (must match include/fp4x.h)
_SIGS = {
    "fp4x_version": ([], _i32),
    "fp4x_last_error_message": ([], ctypes.c_char_p),
    "fp4x_launch_count": ([], _i64),
    "fp4x_device_error": ([_p, _i32, ctypes.POINTER(ctypes.c_int)], _i32),
    "fp4x_test_expire_wait": ([_i64, _p], _i32),
    "fp4x_test_set_static_counter": ([_i64, ctypes.c_int32, _p], _i32),
    "fp4x_gemv_query": ([_i32, _i64, _i64, _i64, _i64, _i32, ctypes.POINTER(_sz), ctypes.POINTER(_i64)], _i32),
    "fp4x_plan_describe": ([_i32, _i64, _i64, _i64, _i64, _i32, _i32, ctypes.c_char_p, _sz], _i32),
    "fp4x_mx8_linear": ([_p, _i64, _p, _p, _p, _i64, _i32, _i64, _i64, _i64, _p, _sz, _p, _i64, _p], _i32),
    "fp4x_mx8_linear_noalloc": ([_p, _i64, _p, _p, _p, _i64, _i32, _i64, _i64, _i64, _p], _i32),
    "fp4x_bf16_linear": ([_p, _i64, _p, _p, _i64, _i32, _i64, _i64, _i64, _p, _sz, _p, _i64, _p], _i32),
    "fp4x_nv4_linear": ([_p, _i64, _p, _p, _f32, _p, _i64, _i32, _i64, _i64, _i64, _p, _sz, _p, _i64, _p], _i32),
    "fp4x_w8_linear": ([_p, _i64, _p, _p, _p, _i64, _i32, _i64, _i64, _i64, _p, _sz, _p, _i64, _p], _i32),
    "fp4x_w6_linear": ([_p, _i64, _p, _p, _p, _p, _i64, _i32, _i64, _i64, _i64, _p, _sz, _p, _i64, _p], _i32),
    "fp4x_int2_logits": ([_p, _i64, _p, _p, _i32, _p, _i64, _i32, _p, _i64, _i64, _i64, _p, _sz, _p, _i64, _p],
                         _i32),
    "fp4x_w8_batch_table_bytes": ([_i64], _sz),
    "fp4x_w8_batch_prepare": ([_p, _i64, _i64, _i64, _p, _sz], _i32),
    "fp4x_w8_linear_batched": ([_p, _i64, _i64, _i64, _i32, _i64, _i64, _i64, _p, _sz, _p, _i64, _p], _i32),
    "fp4x_hc_down": ([_p, _i64, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _sz, _p, _i64, _p], _i32),
    "fp4x_hc_up": ([_p, _i64, _p, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _i64, _p], _i32),
    "fp4x_hc_mixer_unfused": ([_p, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _p,
                               _sz, _p, _i64, _p], _i32),
    "fp4x_topk_query": ([_i64, _i64, _i64, ctypes.POINTER(_sz), ctypes.POINTER(_i64)], _i32),
    "fp4x_topk": ([_p, _i64, _i64, _i64, _i64, _p, _i64, _p, _i64, _p, _sz, _p, _i64, _p], _i32),
    "fp4x_refine_mx8": ([_p, _i64, _i32, _p, _i64, _p, _i32, _i64, _p, _p, _i64, _i64, _i64, _p, _i64, _p], _i32),
    "fp4x_refine_nv4": ([_p, _i64, _p, _i64, _p, _i32, _i64, _p, _p, _f32, _i64, _i64, _i64, _p], _i32),
    "fp4x_argmax_candidates": ([_p, _i64, _p, _i64, _i64, _i64, _p, _p], _i32),
    "fp4x_fast_head_query": ([_i64, _i64, _i64, _i64, _i32, ctypes.POINTER(_sz), ctypes.POINTER(_i64)], _i32),
    "fp4x_fast_head": ([_p, _i64, _p, _p, _i32, _p, _p, _i64, _i64, _i64, _i64, _p, _i64, _p, _p, _p, _p, _p, _sz,
                        _p, _i64, _p], _i32),
    "fp4x_draft_head": ([_p, _i64, _p, _p, _i32, _p, _p, _f32, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _i64, _i64,
                         _p, _sz, _p, _i64, _p], _i32),
    "fp4x_head_merge": ([_p, _p, _p, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p], _i32),
    "fp4x_step_query": ([_p, _i64, _i64, _i32, ctypes.POINTER(_sz), ctypes.POINTER(_sz), ctypes.POINTER(_i64)], _i32),
    "fp4x_step_prepare": ([_p, _i64, _i64, _i32, _p, _sz, _p, _sz, _p, _i64], _i32),
    "fp4x_step_run": ([_p, _p], _i32),
    "fp4x_step_release": ([_p], _i32),
    "fp4x_step_trace": ([_p, _p, _i64], _i32),
    "fp4x_quantize_w8": ([_p, _i32, _i64, _i64, _p, _p, _i32, _p], _i32),
    "fp4x_quantize_w6": ([_p, _i32, _i64, _i64, _i32, _p, _p, _p, _i32, _p], _i32),
    "fp4x_amax": ([_p, _i32, _i64, _p, _p], _i32),
    "fp4x_quantize_nv4": ([_p, _i32, _i64, _i64, ctypes.c_double, _p, _p, _i32, _p], _i32),
    "fp4x_quantize_int2": ([_p, _i32, _i64, _i64, _i32, _p, _p, _i32, _p], _i32),
    "fp4x_mx8_dequant": ([_p, _p, _i64, _i64, _p, _p], _i32),
    "fp4x_dequant_nv4": ([_p, _p, ctypes.c_double, _i64, _i64, _p, _p], _i32),
    "fp4x_dequant_int2": ([_p, _p, _i32, _i64, _i64, _p, _p], _i32),
    "fp4x_nv4_unswizzle_scales": ([_p, _i64, _i64, _p, _p], _i32),
    "fp4x_interleave_rows": ([_p, _i64, _i64, _i64, _i64, _p, _p], _i32),
    "fp4x_prefetch_l2": ([_p, _p, _i32, _p], _i32),
    "fp4x_timeline_begin": ([_p, _i64], _i32),
    "fp4x_timeline_end": ([], _i64),
}

_lib = None
_lock = threading.Lock()


class Fp4xError(RuntimeError):
    def __init__(self, fn, code, msg):
        super().__init__(f"{fn} failed ({code}): {msg}")
        self.code = code


def lib():
    """Load libfp4x.so (raises if it is missing: the CUDA path is the only path)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(f"libfp4x.so not found at {LIB_PATH}; build it with build_native.py")
                L = ctypes.CDLL(LIB_PATH)
                for name, (args, ret) in _SIGS.items():
                    f = getattr(L, name)
                    f.argtypes = args
                    f.restype = ret
                _lib = L
    return _lib


def exported_symbols():
    return list(_SIGS)


def _check(name, rc):
    if rc != OK:
        msg = lib().fp4x_last_error_message()
        raise Fp4xError(name, rc, msg.decode() if msg else "")


def call(name, *args):
    _check(name, getattr(lib(), name)(*args))


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def stream_of(t=None):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device if t is not None else None).cuda_stream)


def dtype_code(dt):
    try:
        return _DTYPES[dt]
    except KeyError:
        raise ValueError(f"unsupported output dtype {dt}") from None


# ---------------------------------------------------------------------------------------------------------
# scratch
# ---------------------------------------------------------------------------------------------------------
_counters = {}   # (device index, stream handle) -> zeroed int32 counter buffer
_spares = {}     # device index -> zeroed buffers kept for streams first seen under CUDA-graph capture
_retired = []    # buffers replaced by larger ones (captured graphs may still point at them)
COUNTER_WORDS = 1 << 16
SPARES_PER_DEVICE = 4


def _device_index(device):
    d = torch.device(device) if device is not None else torch.device("cuda")
    return d.index if d.index is not None else torch.cuda.current_device()


def counters(device, n):
    """Persistent zeroed int32 arrival counters for the current stream of `device`.

    Each (device, stream) pair has its own buffer, so kernels launched on different streams never share a counter.
    A stream that is first seen while it is being captured takes one of the zeroed spare buffers allocated with the
    device's first buffer; when none is left, the buffer is allocated inside the capture (from the graph's memory
    pool, zeroed by a memset node that every replay runs).  Buffers are never freed (a captured graph may hold their
    address)."""
    dev = _device_index(device)
    key = (dev, torch.cuda.current_stream(dev).cuda_stream)
    buf = _counters.get(key)
    if buf is not None and buf.numel() >= n:
        return buf
    if torch.cuda.is_current_stream_capturing():
        spares = _spares.get(dev, [])
        for i, sp in enumerate(spares):
            if sp.numel() >= n:
                _counters[key] = spares.pop(i)
                return _counters[key]
        if buf is not None:
            _retired.append(buf)
        buf = torch.zeros(max(n, COUNTER_WORDS), dtype=torch.int32, device=torch.device("cuda", dev))
        _counters[key] = buf
        return buf
    size = max(n, COUNTER_WORDS, 0 if buf is None else 2 * buf.numel())
    if buf is not None:
        _retired.append(buf)
    buf = torch.zeros(size, dtype=torch.int32, device=torch.device("cuda", dev))
    _counters[key] = buf
    spares = _spares.setdefault(dev, [])
    while len(spares) < SPARES_PER_DEVICE:
        spares.append(torch.zeros(max(size, COUNTER_WORDS), dtype=torch.int32, device=torch.device("cuda", dev)))
    return buf


def counter_buffers(device=None):
    """Every counter buffer of `device` (all devices when None), in use, spare or retired."""
    out = list(_counters.items())
    bufs = [b for (d, _), b in out if device is None or d == _device_index(device)]
    for d, sp in _spares.items():
        if device is None or d == _device_index(device):
            bufs.extend(sp)
    bufs.extend(b for b in _retired if device is None or b.device.index == _device_index(device))
    return bufs


def reset_counters(device=None):
    """Zero every counter buffer of `device` (after a bounded device wait gave up, some may be left non-zero)."""
    for b in counter_buffers(device):
        b.zero_()


_queries = {}


def query(fmt, m, n, k, batch=1, group=16):
    """(workspace bytes, counters) of a GEMV-family call; the plan depends on the shape and the device only, so
    the answer is remembered per (device, shape) and eager calls pay one ctypes round trip per new shape."""
    key = (torch.cuda.current_device() if torch.cuda.is_available() else -1, fmt, m, n, k, batch, group)
    hit = _queries.get(key)
    if hit is not None:
        return hit
    ws = _sz(0)
    nc = _i64(0)
    call("fp4x_gemv_query", fmt, m, n, k, batch, group, ctypes.byref(ws), ctypes.byref(nc))
    _queries[key] = (ws.value, nc.value)
    return ws.value, nc.value


def scratch(fmt, m, n, k, device, batch=1, group=16):
    """(workspace tensor or None, counters tensor or None) for one GEMV-family call."""
    wsb, nc = query(fmt, m, n, k, batch, group)
    ws = torch.empty(wsb, dtype=torch.uint8, device=device) if wsb else None
    cnt = counters(device, nc) if nc else None
    return ws, cnt


def scratch_args(ws, cnt):
    return (ptr(ws), ws.numel() if ws is not None else 0, ptr(cnt), cnt.numel() if cnt is not None else 0)


def head_scratch(m, v, k, c, group, device):
    ws = _sz(0)
    nc = _i64(0)
    call("fp4x_fast_head_query", m, v, k, c, group, ctypes.byref(ws), ctypes.byref(nc))
    return (torch.empty(ws.value, dtype=torch.uint8, device=device), counters(device, nc.value))


def topk_scratch(m, v, c, device):
    ws = _sz(0)
    nc = _i64(0)
    call("fp4x_topk_query", m, v, c, ctypes.byref(ws), ctypes.byref(nc))
    return (torch.empty(ws.value, dtype=torch.uint8, device=device), counters(device, nc.value))


def plan(fmt, m, n, k, batch=1, group=16, whole=False):
    """The launch plan the library picks for a GEMV of this shape (diagnostic text)."""
    buf = ctypes.create_string_buffer(512)
    call("fp4x_plan_describe", fmt, m, n, k, batch, group, 1 if whole else 0, buf, 512)
    return buf.value.decode()


# launch timeline words (TlWord in csrc/fp4x_common.cuh)
(TL_START_FIRST, TL_START_LAST, TL_WAIT_LAST, TL_X_LANDED, TL_STAGED, TL_FIRST_STAGE, TL_LOOP_DONE, TL_HANDOVER,
 TL_REDUCED, TL_STORED, TL_WAIT_FIRST) = range(11)


def use_timeline_library():
    """Load the diagnostic twin (libfp4x_timeline.so) instead of libfp4x.so; must run before the first library call
    of the process."""
    global LIB_PATH
    if _lib is not None and LIB_PATH != TIMELINE_LIB_PATH:
        raise RuntimeError("libfp4x.so is already loaded in this process")
    LIB_PATH = TIMELINE_LIB_PATH


class Timeline:
    """Diagnostic launch timeline (fp4x_timeline_begin / fp4x_timeline_end; needs the timeline library, see
    use_timeline_library): `begin()`, launch or capture the GEMVs,
    `end()`; then `arm()` before a run (or graph replay) and `read()` after it: a uint64 array [launches, 16] of
    globaltimer stamps, the words named by the TL_* constants (latest over the launch's CTAs, earliest for the
    *_FIRST words; TL_HANDOVER and TL_REDUCED stay 0 in the tensor-core kernels)."""

    WORDS = 16

    def __init__(self, count, device):
        self.buf = torch.zeros(count, self.WORDS, dtype=torch.int64, device=device)
        self.n = 0

    def begin(self):
        self.arm()
        call("fp4x_timeline_begin", ptr(self.buf), self.buf.shape[0])

    def end(self):
        self.n = int(lib().fp4x_timeline_end())
        return self.n

    def arm(self):
        self.buf.zero_()
        self.buf[:, TL_START_FIRST] = -1  # all ones: the minimum words
        self.buf[:, TL_WAIT_FIRST] = -1

    def read(self):
        return self.buf[: self.n].cpu().numpy().view(np.uint64)


def launch_count():
    """Kernels the library has launched (or recorded into a graph under capture) since it was loaded."""
    return int(lib().fp4x_launch_count())


def device_error(clear=True, device=None):
    """The device error word of `device` (0: no bounded wait gave up since the last clear).  With `clear`, a non-zero
    word is reset together with every arrival counter of the device (the library's static counters included), since
    a kernel that gave up may have left its counters mid-count."""
    code = ctypes.c_int(0)
    st = stream_of(None if device is None else torch.empty(0, device=device))
    rc = lib().fp4x_device_error(st, 1 if clear else 0, ctypes.byref(code))
    if rc not in (OK, ERR_DEVICE):
        return rc
    if clear and code.value:
        torch.cuda.synchronize(device)
        reset_counters(device)
        torch.cuda.synchronize(device)
    return code.value
