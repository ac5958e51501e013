"""ctypes binding of libfp4x.so (include/fp4x.h) for the torch host code.

torch provides device memory and the current stream; every call passes raw pointers, integer sizes and the
stream handle to the C ABI.  There is no fallback: if the library is missing or a call fails, a Python exception
is raised.  Scratch memory for split reductions is allocated here through torch's caching allocator (so it is
safe under CUDA-graph capture); the arrival counters live in one persistent zeroed int32 buffer per device that
the kernels leave zeroed after every call.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("FP4X_LIB", os.path.join(_HERE, "libfp4x.so"))

OK = 0
ERR_INVALID_ARG, ERR_UNSUPPORTED, ERR_WORKSPACE, ERR_CUDA, ERR_DEVICE = -1, -2, -3, -4, -5
FMT_MX8, FMT_W8, FMT_W6, FMT_NV4, FMT_BF16, FMT_INT2 = range(6)
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

# argument signatures of every exported entry point (must match include/fp4x.h)
_SIGS = {
    "fp4x_version": ([], _i32),
    "fp4x_last_error_message": ([], ctypes.c_char_p),
    "fp4x_launch_count": ([], _i64),
    "fp4x_device_error": ([_p, _i32, ctypes.POINTER(ctypes.c_int)], _i32),
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
_counters = {}


def counters(device, n):
    """Persistent zeroed int32 arrival counters on `device` (grown on demand, never during capture)."""
    key = torch.device(device).index if torch.device(device).index is not None else torch.cuda.current_device()
    buf = _counters.get(key)
    if buf is None or buf.numel() < n:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("fp4x counter buffer must be sized before CUDA-graph capture "
                               "(run the call once eagerly first)")
        size = max(n, 1 << 16, 0 if buf is None else 2 * buf.numel())
        buf = torch.zeros(size, dtype=torch.int32, device=torch.device("cuda", key))
        _counters[key] = buf
    return buf


def query(fmt, m, n, k, batch=1, group=16):
    ws = _sz(0)
    nc = _i64(0)
    call("fp4x_gemv_query", fmt, m, n, k, batch, group, ctypes.byref(ws), ctypes.byref(nc))
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


def launch_count():
    """Kernels the library has launched (or recorded into a graph under capture) since it was loaded."""
    return int(lib().fp4x_launch_count())


def device_error(clear=True, device=None):
    code = ctypes.c_int(0)
    rc = lib().fp4x_device_error(stream_of(None if device is None else torch.empty(0, device=device)),
                                 1 if clear else 0, ctypes.byref(code))
    return code.value if rc in (OK, ERR_DEVICE) else rc
