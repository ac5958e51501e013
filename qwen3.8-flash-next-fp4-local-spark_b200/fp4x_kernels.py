"""fp4x decode kernel library for B200 (sm_100a): drop-in replacement for the reference plugin's `fp4x_kernels`.

Same public names, call signatures and packed weight layouts as the reference module (`x/fp4x_kernels.py`,
cited K:<line>); the Triton bodies are replaced by hand-written sm_100a CUDA kernels in libfp4x.so, reached
through the C ABI in include/fp4x.h (see fp4x_native.py).  The Triton tile configurations (`cfg`, `BN`, `BK`,
`nw`, ...) are still accepted so that callers are unchanged; the native kernels plan their own launch from the
shape and the device.

Numerics
* Products are exact and sums are fp32, as in the reference.  MXFP8, NVFP4, INT2 and BF16 weights are
  multiplied exactly as the reference forms them (bf16-rounded dequantized weights).  W8 and W6 apply the group
  scale to each group's fp32 partial sum (exact q * s instead of bf16(q * s)); the difference is the bf16
  rounding of the weight (<= 2^-9 relative per weight).
* Activations are converted to f16 with a power-of-two scale per token and K-panel for the fp8/int weight
  formats (exact for every element within 2^31 of the panel maximum) and stay bf16 for BF16/INT2 weights.

Weight preparation (the quantizers and dequantizers) runs in torch on the weights' device and reproduces the
reference's packing bit for bit.
"""
from __future__ import annotations

import ctypes

import torch

import fp4x_native as N

# K:327-328: element j of each 4-group lives in bit pair ORDER[j]
ORDER = (0, 2, 1, 3)
_AWQ_LOG = []  # alpha chosen by each quantize_w6_awq call (K:253-254)
_E2M1 = None
_E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


# ----------------------------------------------------------------------------------------------------------
# argument plumbing
# ----------------------------------------------------------------------------------------------------------

def _act(x2):
    """bf16 activations with 16-byte aligned rows and unit column stride."""
    if x2.dtype != torch.bfloat16:
        x2 = x2.to(torch.bfloat16)
    if x2.stride(-1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
        if x2.data_ptr() % 16:
            x2 = x2.clone()
    return x2


def _rows(t):
    return t if t.is_contiguous() else t.contiguous()


def _u8(t):
    return t.view(torch.uint8) if t.dtype != torch.uint8 and t.element_size() == 1 else t


def _chunks(m):
    for a in range(0, m, 16):
        yield a, min(m, a + 16)


def _linear(fmt, fn, x2, planes, n, k, out_dtype, extra=(), group=16, post_args=()):
    """Shared driver of the single-matrix GEMVs: M <= 16 per launch (larger M is split)."""
    x2 = _act(x2)
    m = x2.shape[0]
    out = torch.empty((m, n), dtype=out_dtype, device=x2.device)
    if m == 0:
        return out
    st = N.stream_of(x2)
    for a, b in _chunks(m):
        xs = x2[a:b]
        mm = b - a
        ws, cnt = N.scratch(fmt, mm, n, k, x2.device, 1, group)
        o = out[a:b]
        N.call(fn, N.ptr(xs), xs.stride(0), *[N.ptr(p) for p in planes], *post_args, N.ptr(o), o.stride(0),
               N.dtype_code(out_dtype), *extra, mm, n, k, *N.scratch_args(ws, cnt), st)
    return out


# ----------------------------------------------------------------------------------------------------------
# dense decode GEMVs
# ----------------------------------------------------------------------------------------------------------

def mx8_linear(x2, w8, s, cfg=None, out_dtype=torch.bfloat16):
    """out = x2 . deq(w8)^T with MXFP8 weights: e4m3 codes [N, K] + e8m0 scales [N, K/32] (K:9-29, K:65)."""
    n, k = w8.shape
    return _linear(N.FMT_MX8, "fp4x_mx8_linear", x2, (_rows(_u8(w8)), _rows(_u8(s))), n, k, out_dtype)


def bf16_linear(x2, w, cfg=None, out_dtype=torch.bfloat16):
    """BF16-weight GEMV (K:32-47, K:69)."""
    n, k = w.shape
    if w.dtype != torch.bfloat16:
        raise TypeError("bf16_linear expects bf16 weights")
    return _linear(N.FMT_BF16, "fp4x_bf16_linear", x2, (_rows(w),), n, k, out_dtype)


def nv4_linear(x2, wp, s, gs, cfg=(32, 256, 4), out_dtype=torch.bfloat16):
    """NVFP4: e2m1 pairs [N, K/2] (low nibble = even k), e4m3 scales [N, K/16], fp32 global scale gs
    (K:73-113)."""
    n = wp.shape[0]
    k = wp.shape[1] * 2
    x2 = _act(x2)
    m = x2.shape[0]
    out = torch.empty((m, n), dtype=out_dtype, device=x2.device)
    if m == 0:
        return out
    g = float(gs)
    st = N.stream_of(x2)
    wp, s = _rows(wp), _rows(_u8(s))
    for a, b in _chunks(m):
        xs, o = x2[a:b], out[a:b]
        ws, cnt = N.scratch(N.FMT_NV4, b - a, n, k, x2.device)
        N.call("fp4x_nv4_linear", N.ptr(xs), xs.stride(0), N.ptr(wp), N.ptr(s), g, N.ptr(o), o.stride(0),
               N.dtype_code(out_dtype), b - a, n, k, *N.scratch_args(ws, cnt), st)
    return out


def w8_linear(x2, q, s, cfg=None, out_dtype=torch.bfloat16):
    """int8 codes [N, K] with fp32 scales per 64-group [N, K/64] (K:116-148)."""
    n, k = q.shape
    return _linear(N.FMT_W8, "fp4x_w8_linear", x2, (_rows(q), _rows(s.float())), n, k, out_dtype)


def w6_linear(x2, L, H, S, cfg=None, out_dtype=torch.bfloat16):
    """6-bit g32: low-nibble plane [N, K/2], high-bit-pair plane [N, K/4], fp16 scales [N, K/32]
    (K:151-176, K:270)."""
    n = L.shape[0]
    k = L.shape[1] * 2
    return _linear(N.FMT_W6, "fp4x_w6_linear", x2, (_rows(L), _rows(H), _rows(S)), n, k, out_dtype)


def int2_logits(x, P, S, N_rows=None, BN=64, BK=512, nw=4, RS=None, out_dtype=torch.float32, out_bf16=None, **kw):
    """Coarse logits from 2-bit codes [V, K/4] with fp16 group scales [V, K/G] (K:304-325, K:359-364).
    Values are x . bf16((code - 1.5) * s).  `out_bf16`, if given ([M, V] bf16), also receives a bf16 copy."""
    if "N" in kw:
        N_rows = kw.pop("N")
    if kw:
        raise TypeError(f"unexpected arguments {sorted(kw)}")
    if RS is not None:
        raise NotImplementedError("ROW_SCALE (e4m3 group scales with per-row fp32 scales) is not supported")
    x = _act(x)
    m, k = x.shape
    n = int(P.shape[0] if N_rows is None else N_rows)
    group = k // S.shape[1]
    out = torch.empty((m, n), dtype=out_dtype, device=x.device)
    if m == 0:
        return out
    P, S = _rows(P), _rows(S)
    st = N.stream_of(x)
    for a, b in _chunks(m):
        xs, o = x[a:b], out[a:b]
        ob = out_bf16[a:b] if out_bf16 is not None else None
        ws, cnt = N.scratch(N.FMT_INT2, b - a, n, k, x.device, 1, group)
        N.call("fp4x_int2_logits", N.ptr(xs), xs.stride(0), N.ptr(P), N.ptr(S), group, N.ptr(o), o.stride(0),
               N.dtype_code(out_dtype), N.ptr(ob), b - a, n, k, *N.scratch_args(ws, cnt), st)
    return out


class W8Batch:
    """Batched W8 GEMVs of one shape in one launch (the router gates, P:258-272 with FP4X_GATE=w8).

    The device table (TMA descriptors of the weights plus the activation/output pointers) is built once from the
    given buffers, so the launch itself needs no host work; callers write new activations into the same `xs`."""

    def __init__(self, xs, qs, ss, outs=None, out_dtype=torch.bfloat16):
        assert len(xs) == len(qs) == len(ss) and len(qs) > 0
        self.n, self.k = qs[0].shape
        self.m = xs[0].shape[0]
        dev = qs[0].device
        self.xs = [_act(x) for x in xs]
        for x in self.xs:
            assert x.shape == self.xs[0].shape and x.stride(0) == self.xs[0].stride(0)
        self.qs = [_rows(q) for q in qs]
        self.ss = [_rows(s.float()) for s in ss]
        self.out_dtype = out_dtype
        self.outs = outs if outs is not None else [torch.empty((self.m, self.n), dtype=out_dtype, device=dev)
                                                   for _ in qs]
        items = (N.W8Item * len(qs))()
        for i, (x, q, s, o) in enumerate(zip(self.xs, self.qs, self.ss, self.outs)):
            items[i] = N.W8Item(x.data_ptr(), q.data_ptr(), s.data_ptr(), o.data_ptr())
        nbytes = N.lib().fp4x_w8_batch_table_bytes(len(qs))
        self.table = torch.empty(nbytes + 64, dtype=torch.uint8, device=dev)
        off = (-self.table.data_ptr()) % 64
        self.table_view = self.table[off:off + nbytes]
        N.call("fp4x_w8_batch_prepare", items, len(qs), self.n, self.k, N.ptr(self.table_view), nbytes)
        self.ws, self.cnt = N.scratch(N.FMT_W8, self.m, self.n, self.k, dev, len(qs))

    def run(self):
        N.call("fp4x_w8_linear_batched", N.ptr(self.table_view), len(self.qs), self.xs[0].stride(0),
               self.outs[0].stride(0), N.dtype_code(self.out_dtype), self.m, self.n, self.k,
               *N.scratch_args(self.ws, self.cnt), N.stream_of(self.table))
        return self.outs


def w8_linear_batched(xs, qs, ss, out_dtype=torch.bfloat16):
    """Eager convenience wrapper of W8Batch (builds the pointer table on every call)."""
    return W8Batch(xs, qs, ss, out_dtype=out_dtype).run()


# ----------------------------------------------------------------------------------------------------------
# LM heads: top-C selection and exact rescoring (K:367-417, P:309-378)
# ----------------------------------------------------------------------------------------------------------

def topk_indices(vals, C):
    """Exact top-C per row of fp32 values [M, V]: (indices int32 [M, C] in ascending index order, values [M, C]).
    Order of the selection: value descending, then index ascending."""
    vals = vals if vals.dtype == torch.float32 else vals.float()
    vals = _rows(vals)
    m, v = vals.shape
    idx = torch.empty((m, C), dtype=torch.int32, device=vals.device)
    sel = torch.empty((m, C), dtype=torch.float32, device=vals.device)
    ws, cnt = N.topk_scratch(m, v, C, vals.device)
    N.call("fp4x_topk", N.ptr(vals), vals.stride(0), m, v, C, N.ptr(idx), C, N.ptr(sel), C, N.ptr(ws), ws.numel(),
           N.ptr(cnt), cnt.numel(), N.stream_of(vals))
    return idx, sel


def _idx_args(idx):
    if idx.dtype not in (torch.int32, torch.int64):
        raise TypeError("candidate indices must be int32 or int64")
    idx = _rows(idx)
    return N.ptr(idx), 1 if idx.dtype == torch.int64 else 0, idx.stride(0)


def refine_mx8_(out, x, idx, w8, s_u8, BC=16, BK=256, nw=4):
    """In place: out[m, idx[m, c]] = exact MXFP8 row idx[m, c] . x[m] (fp32 accumulate), K:384-388."""
    x = _act(x)
    m, C = idx.shape
    k = x.shape[1]
    if m == 0 or C == 0:
        return out
    if out.stride(-1) != 1:
        raise ValueError("out must have unit column stride")
    pi, i64, ild = _idx_args(idx)
    N.call("fp4x_refine_mx8", N.ptr(out), out.stride(0), N.dtype_code(out.dtype), N.ptr(x), x.stride(0), pi, i64,
           ild, N.ptr(_rows(_u8(w8))), N.ptr(_rows(_u8(s_u8))), m, C, k, None, 0, N.stream_of(x))
    return out


def refine_nv4(x, idx, wp, s, gs, BC=16, BK=256, nw=4):
    """[M, C] exact NVFP4 logits of candidate rows idx[m, c] (fp32 accumulate), K:412-417."""
    x = _act(x)
    m, C = idx.shape
    k = x.shape[1]
    out = torch.empty((m, C), dtype=torch.float32, device=x.device)
    if m == 0 or C == 0:
        return out
    pi, i64, ild = _idx_args(idx)
    N.call("fp4x_refine_nv4", N.ptr(out), C, N.ptr(x), x.stride(0), pi, i64, ild, N.ptr(_rows(wp)),
           N.ptr(_rows(_u8(s))), float(gs), m, C, k, N.stream_of(x))
    return out


def fast_head(h, P, S, w8, s_u8, C=512, out=None):
    """Fused fast target head (P:370-378): INT2 coarse logits, exact top-C (fp32 coarse values, ties to the lower
    vocab id), exact MXFP8 rescore scattered into the coarse bf16 logits.
    Returns (full bf16 [M, V], idx int32 [M, C] ascending, exact fp32 [M, C], argmax int32 [M])."""
    h = _act(h)
    m, k = h.shape
    v = P.shape[0]
    group = k // S.shape[1]
    full = out if out is not None else torch.empty((m, v), dtype=torch.bfloat16, device=h.device)
    idx = torch.empty((m, C), dtype=torch.int32, device=h.device)
    exact = torch.empty((m, C), dtype=torch.float32, device=h.device)
    amax = torch.empty((m,), dtype=torch.int32, device=h.device)
    ws, cnt = N.head_scratch(m, v, k, C, group, h.device)
    N.call("fp4x_fast_head", N.ptr(h), h.stride(0), N.ptr(_rows(P)), N.ptr(_rows(S)), group, N.ptr(_rows(_u8(w8))),
           N.ptr(_rows(_u8(s_u8))), m, v, k, C, N.ptr(full), full.stride(0), N.ptr(idx), N.ptr(exact), None,
           N.ptr(amax), N.ptr(ws), ws.numel(), N.ptr(cnt), cnt.numel(), N.stream_of(h))
    return full, idx, exact, amax


def draft_head(h, P, S, wp, sn, gs, C=64, ids=None, full_vocab=None):
    """Fused draft head (P:315-327): INT2 coarse logits over the draft rows, top-C, exact NVFP4 rescore.
    Returns (idx int32 [M, C] ascending draft-row indices, vals fp32 [M, C], full) where full is the
    [M, full_vocab] bf16 tensor of -inf with vals scattered at ids[idx] when ids/full_vocab are given."""
    h = _act(h)
    m, k = h.shape
    v = P.shape[0]
    group = k // S.shape[1]
    idx = torch.empty((m, C), dtype=torch.int32, device=h.device)
    vals = torch.empty((m, C), dtype=torch.float32, device=h.device)
    full = None
    if ids is not None and full_vocab is not None:
        full = torch.empty((m, full_vocab), dtype=torch.bfloat16, device=h.device)
        ids = _rows(ids.long())
    ws, cnt = N.head_scratch(m, v, k, C, group, h.device)
    N.call("fp4x_draft_head", N.ptr(h), h.stride(0), N.ptr(_rows(P)), N.ptr(_rows(S)), group, N.ptr(_rows(wp)),
           N.ptr(_rows(_u8(sn))), float(gs), m, v, k, C, N.ptr(idx), N.ptr(vals), N.ptr(ids), N.ptr(full),
           full_vocab or 0, full_vocab or 0, N.ptr(ws), ws.numel(), N.ptr(cnt), cnt.numel(), N.stream_of(h))
    return idx, vals, full


def head_merge(coarse, exact, gidx, V):
    """Merge the candidates of a vocab-sharded head: inputs [P, M, C] (coarse fp32, exact fp32, global ids int32)
    -> (idx int32 [M, C] ascending, exact fp32 [M, C], argmax int32 [M]) of the global top-C by coarse value."""
    p, m, C = coarse.shape
    idx = torch.empty((m, C), dtype=torch.int32, device=coarse.device)
    co = torch.empty((m, C), dtype=torch.float32, device=coarse.device)
    ex = torch.empty((m, C), dtype=torch.float32, device=coarse.device)
    amax = torch.empty((m,), dtype=torch.int32, device=coarse.device)
    N.call("fp4x_head_merge", N.ptr(_rows(coarse)), N.ptr(_rows(exact)), N.ptr(_rows(gidx)), p, m, C, V, N.ptr(idx),
           N.ptr(co), N.ptr(ex), N.ptr(amax), N.stream_of(coarse))
    return idx, co, ex, amax


# ----------------------------------------------------------------------------------------------------------
# hyper-connection mixer (K:429-526)
# ----------------------------------------------------------------------------------------------------------

class HCFused:
    """Fused W8 hyper-connection mixer (two kernels per mixer): K:496-526.

    The split-K reduction of the down projection is deterministic (fixed-order sum of per-warp partial slots)
    and self-cleaning; the arrival counters are shared by every mixer, so calls must be stream-ordered, as in
    the reference."""

    def __init__(self, device, n_down=336, max_m=16, bn=32):
        self.device = torch.device(device)
        self.n_down, self.max_m = n_down, max_m
        # counters are allocated eagerly so that later calls can be captured
        self.cnt = N.counters(self.device, 1 << 12)

    def down(self, x, q, s, lr, hc, cfg=(32, 512, 4, 4)):
        x = _act(x)
        m, k = x.shape
        n = q.shape[0]
        di = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
        bot = torch.empty((m, lr), dtype=torch.bfloat16, device=x.device)
        ws, cnt = N.scratch(N.FMT_W8, m, n, k, x.device)
        N.call("fp4x_hc_down", N.ptr(x), x.stride(0), N.ptr(_rows(q)), N.ptr(_rows(s.float())), N.ptr(di),
               N.ptr(bot), m, n, k, lr, hc, *N.scratch_args(ws, cnt), N.stream_of(x))
        return di, bot

    @staticmethod
    def interleave_up(q, s, hc, bj):
        """Reorder up rows [HC*H, K] so that each BJ-column tile holds its HC stream rows contiguously
        (K:513-517): new row (j*HC + s)*BJ + t = old row s*H + j*BJ + t.  CUDA tensors: one gather kernel per
        plane (fp4x_interleave_rows)."""
        n = q.shape[0]
        if q.is_cuda and s.is_cuda:
            return _interleave_native(q, hc, bj), _interleave_native(s, hc, bj)
        h = n // hc
        perm = torch.arange(n, device=q.device).view(hc, h // bj, bj).transpose(0, 1).reshape(-1)
        return q.index_select(0, perm).contiguous(), s.index_select(0, perm).contiguous()

    @staticmethod
    def up(bot, qi, si, normalized, hc, cfg=(8, 64, 8)):
        bj = cfg[0]
        bot = _act(bot)
        m, k = bot.shape
        n = qi.shape[0]
        h = n // hc
        out = torch.empty((m, h), dtype=torch.bfloat16, device=bot.device)
        nrm = _act(normalized)
        N.call("fp4x_hc_up", N.ptr(bot), bot.stride(0), N.ptr(_rows(qi)), N.ptr(_rows(si.float())), N.ptr(nrm),
               nrm.stride(0), N.ptr(out), m, n, k, hc, bj, N.stream_of(bot))
        return out


def hc_mixer_unfused(x, qd, sd, qu, su, lr, hc):
    """The unfused W8 mixer route (P:231-247): down GEMV + cast, scaled SiLU, up GEMV on the original row
    order, gate-mean.  Bit-identical to HCFused.down + HCFused.up.  Returns (di, bot, block_input)."""
    x = _act(x)
    m, k = x.shape
    nd, nu = qd.shape[0], qu.shape[0]
    di = torch.empty((m, nd), dtype=torch.bfloat16, device=x.device)
    bot = torch.empty((m, lr), dtype=torch.bfloat16, device=x.device)
    g = torch.empty((m, nu), dtype=torch.bfloat16, device=x.device)
    out = torch.empty((m, nu // hc), dtype=torch.bfloat16, device=x.device)
    ws, cnt = N.scratch(N.FMT_W8, m, nd, k, x.device)
    N.call("fp4x_hc_mixer_unfused", N.ptr(x), x.stride(0), N.ptr(_rows(qd)), N.ptr(_rows(sd.float())),
           N.ptr(_rows(qu)), N.ptr(_rows(su.float())), N.ptr(di), N.ptr(bot), N.ptr(g), N.ptr(out), m, nd, k, lr,
           hc, nu, *N.scratch_args(ws, cnt), N.stream_of(x))
    return di, bot, out


# ----------------------------------------------------------------------------------------------------------
# weight preparation (torch; restates the reference quantizers so the packed bytes are identical)
# ----------------------------------------------------------------------------------------------------------

def _row_blocks(n, rows):
    for a in range(0, n, rows):
        yield a, min(n, a + rows)


@torch.no_grad()
def _torch_quantize_w8(w):
    """Symmetric int8 per 64-group: s = max(amax, 1e-12) / 127, q = clamp(round(w / s), +-127) (K:138-144)."""
    n, k = w.shape
    q = torch.empty((n, k), dtype=torch.int8, device=w.device)
    s = torch.empty((n, k // 64), dtype=torch.float32, device=w.device)
    for a, b in _row_blocks(n, 4096):
        grp = w[a:b].float().reshape(b - a, k // 64, 64)
        sc = grp.abs().amax(dim=-1).clamp_min(1e-12) / 127.0
        q[a:b] = torch.round(grp / sc.unsqueeze(-1)).clamp(-127, 127).to(torch.int8).reshape(b - a, k)
        s[a:b] = sc
    return q, s


def _w6_pack(codes):
    """codes int32 [R, K] in 0..63 -> (low-nibble plane [R, K/2], high-bit-pair plane [R, K/4])."""
    lo = codes & 15
    hi = codes >> 4
    L = (lo[:, 0::2] | (lo[:, 1::2] << 4)).to(torch.uint8)
    H = hi[:, 0::4] | (hi[:, 1::4] << (2 * ORDER[1])) | (hi[:, 2::4] << (2 * ORDER[2])) | (hi[:, 3::4] << (2 * ORDER[3]))
    return L, H.to(torch.uint8)


def _w6_scale_search(f, qmax, clip, weight=None):
    """fp16-rounded g32 scales for f [R, G, 32]; with clip > 0, the scale minimising the (weighted) squared error
    over a grid of clip ratios 0.70..0.98 (K:205-215)."""
    s = (f.abs().amax(-1, keepdim=True) / qmax).to(torch.float16).float().clamp_min(6.2e-5)
    if not clip:
        return s

    def err(sc):
        d = (torch.round(f / sc).clamp(-qmax - 1, qmax) * sc - f) ** 2
        return (d if weight is None else d * weight).sum(-1, keepdim=True)

    best, best_s = err(s), s
    for c in torch.linspace(0.70, 0.98, clip).tolist():
        cand = (s * c).to(torch.float16).float().clamp_min(6.2e-5)
        e = err(cand)
        take = e < best
        best = torch.where(take, e, best)
        best_s = torch.where(take, cand, best_s)
    return best_s


@torch.no_grad()
def _torch_quantize_w6(w, qmax=31, clip_search=0):
    """6-bit g32 (K:179-202): s = max(fp16(amax/qmax), 6.2e-5), codes = clamp(round(w/s), -qmax-1, qmax) + 32.
    Returns (L [N,K/2] u8, H [N,K/4] u8, S [N,K/32] f16)."""
    n, k = w.shape
    L = torch.empty((n, k // 2), dtype=torch.uint8, device=w.device)
    H = torch.empty((n, k // 4), dtype=torch.uint8, device=w.device)
    S = torch.empty((n, k // 32), dtype=torch.float16, device=w.device)
    for a, b in _row_blocks(n, 2048):
        f = w[a:b].float().view(-1, k // 32, 32)
        s = _w6_scale_search(f, qmax, clip_search)
        codes = (torch.round(f / s).clamp(-qmax - 1, qmax).to(torch.int32) + 32).view(-1, k)
        L[a:b], H[a:b] = _w6_pack(codes)
        S[a:b] = s.squeeze(-1).to(torch.float16)
    return L, H, S


@torch.no_grad()
def quantize_w6_awq(w, h, qmax=31, clip=0, alpha=-1.0):
    """Activation-aware W6 g32 quality probe (K:218-255).  h [K] = mean x^2 per input channel.  The weight is
    quantized as W * t with t a power of two per input channel (t = a^alpha normalised, a = sqrt(h)); alpha is
    grid-searched on up to 1024 random rows when negative.  Returns (L, H, S, inv_t bf16 [K])."""
    n, k = w.shape
    a = h.float().clamp_min(1e-12).sqrt()
    a = a / a.mean()
    hw = (a * a).view(1, k // 32, 32)
    rows = torch.randperm(n, device=w.device)[:min(n, 1024)]

    def t_for(al):
        return torch.exp2(torch.round(torch.log2(a ** al / (a ** al).mean())))

    def weighted_err(t, rr):
        tv = t.view(1, k // 32, 32)
        f = (w[rr].float() * t).view(-1, k // 32, 32)
        sc = _w6_scale_search(f, qmax, clip, hw / tv ** 2)
        d = torch.round(f / sc).clamp(-qmax - 1, qmax) * sc / tv - w[rr].float().view(-1, k // 32, 32)
        return ((d * d) * hw).sum().item()

    best_a = alpha
    if alpha < 0:
        best_a, best_e = 0.0, None
        for al in [i / 10 for i in range(11)]:
            e = weighted_err(t_for(al), rows)
            if best_e is None or e < best_e:
                best_e, best_a = e, al
    t = t_for(best_a)
    tv = t.view(1, k // 32, 32)
    L = torch.empty((n, k // 2), dtype=torch.uint8, device=w.device)
    H = torch.empty((n, k // 4), dtype=torch.uint8, device=w.device)
    S = torch.empty((n, k // 32), dtype=torch.float16, device=w.device)
    for r0, r1 in _row_blocks(n, 2048):
        f = (w[r0:r1].float() * t).view(-1, k // 32, 32)
        s = _w6_scale_search(f, qmax, clip, hw / tv ** 2)
        codes = (torch.round(f / s).clamp(-qmax - 1, qmax).to(torch.int32) + 32).view(-1, k)
        L[r0:r1], H[r0:r1] = _w6_pack(codes)
        S[r0:r1] = s.squeeze(-1).to(torch.float16)
    _AWQ_LOG.append(best_a)
    return L, H, S, (1.0 / t).to(torch.bfloat16)


@torch.no_grad()
def _torch_mx8_dequant(w8, s_u8, rows=2048):
    """MXFP8 -> fp32 [N, K]: e4m3 * 2^(s - 127) (K:261-267)."""
    n, k = w8.shape
    codes = w8.view(torch.float8_e4m3fn) if w8.dtype == torch.uint8 else w8
    out = torch.empty((n, k), dtype=torch.float32, device=w8.device)
    for a, b in _row_blocks(n, rows):
        scale = torch.exp2(s_u8[a:b].float() - 127).unsqueeze(-1)
        out[a:b] = (codes[a:b].float().view(b - a, k // 32, 32) * scale).view(b - a, k)
    return out


@torch.no_grad()
def quantize_mx8(w):
    """MXFP8 packing of a float matrix (the synthetic-weight recipe; served weights come packed from b12x):
    e8m0 byte = 127 + ceil(log2(amax32 / 448)), codes = e4m3(w / 2^(byte - 127)).  Not in the reference module.
    Returns (codes float8_e4m3fn [N, K], scales uint8 [N, K/32])."""
    n, k = w.shape
    f = w.float().view(n, k // 32, 32)
    amax = f.abs().amax(-1)
    mant, expo = torch.frexp(amax / 448.0)
    ce = torch.where(mant > 0.5, expo, expo - 1)
    ce = torch.where(amax == 0, torch.full_like(ce, -127), ce)
    sbyte = (ce + 127).clamp(0, 254).to(torch.uint8)
    codes = (f.double() / torch.exp2(ce.double()).unsqueeze(-1)).float().to(torch.float8_e4m3fn).view(n, k)
    return codes, sbyte


@torch.no_grad()
def _torch_quantize_nv4(w, rows=2048):
    """NVFP4 (K:277-300): gs = max(amax/6/448, 1e-30) (python float), block scale = e4m3(clamp(amax16/6/gs,
    2^-9, 448)), magnitudes by nearest e2m1 level with ties to the lower level.  Returns (P, S e4m3, gs)."""
    global _E2M1
    n, k = w.shape
    if _E2M1 is None or _E2M1.device != w.device:
        _E2M1 = torch.tensor(_E2M1_VALUES, device=w.device)
    amax_all = 0.0
    for a, b in _row_blocks(n, rows):
        amax_all = max(amax_all, w[a:b].float().abs().max().item())
    gs = max(amax_all / 6.0 / 448.0, 1e-30)
    P = torch.empty((n, k // 2), dtype=torch.uint8, device=w.device)
    S = torch.empty((n, k // 16), dtype=torch.float8_e4m3fn, device=w.device)
    mids = (_E2M1[1:] + _E2M1[:-1]) / 2
    for a, b in _row_blocks(n, rows):
        f = w[a:b].float().view(-1, k // 16, 16)
        blk = (f.abs().amax(-1, keepdim=True) / 6.0 / gs).clamp(min=2 ** -9, max=448.0).to(torch.float8_e4m3fn)
        v = (f / (blk.float() * gs)).clamp(-6, 6)
        code = torch.bucketize(v.abs(), mids) | ((v < 0).to(torch.int64) << 3)
        code = code.view(-1, k)
        P[a:b] = (code[:, 0::2] | (code[:, 1::2] << 4)).to(torch.uint8)
        S[a:b] = blk.view(-1, k // 16)
    return P, S, gs


@torch.no_grad()
def _torch_dequant_nv4(P, S, gs):
    """[N, K/2] e2m1 pairs + [N, K/16] e4m3 scales -> fp32 [N, K] = v * s * gs (K:420-426)."""
    lut = torch.tensor(_E2M1_VALUES + tuple(-v for v in _E2M1_VALUES), device=P.device)
    n = P.shape[0]
    v = torch.stack([lut[(P & 15).long()], lut[(P >> 4).long()]], -1).view(n, -1)
    return (v.view(n, -1, 16) * S.float().unsqueeze(-1) * gs).view(n, -1)


@torch.no_grad()
def _torch_quantize_int2(weight, scale_fmt="fp16", group=16):
    """INT2 per group (K:330-351): s = max(amax, 1e-8)/1.5 (fp16, or e4m3 relative to an fp32 row scale),
    code = clamp(floor(w/s) + 2, 0, 3), value (code - 1.5) * s; 4 codes per byte at bit pairs ORDER.
    Returns (packed, s) for fp16 scales, (packed, s_e4m3, row_scale) for e4m3."""
    n, k = weight.shape
    packed = torch.empty((n, k // 4), dtype=torch.uint8, device=weight.device)
    sdt = torch.float16 if scale_fmt == "fp16" else torch.float8_e4m3fn
    scales = torch.empty((n, k // group), dtype=sdt, device=weight.device)
    rowsc = torch.empty((n,), dtype=torch.float32, device=weight.device)
    for a, b in _row_blocks(n, 8192):
        f = weight[a:b].float().view(-1, k // group, group)
        s = f.abs().amax(-1, keepdim=True).clamp_min(1e-8) / 1.5
        if scale_fmt == "fp16":
            s = s.half()
            sf = s.float()
        else:
            rs = s.amax(1, keepdim=True) / 448.0
            s = (s / rs).to(torch.float8_e4m3fn)
            sf = s.float() * rs
            rowsc[a:b] = rs.view(-1)
        code = (torch.floor(f / sf) + 2).clamp(0, 3).to(torch.uint8).view(-1, k // 4, 4)
        byte = code[..., 0] << (2 * ORDER[0])
        for j in range(1, 4):
            byte = byte | (code[..., j] << (2 * ORDER[j]))
        packed[a:b] = byte
        scales[a:b] = s.squeeze(-1)
    return (packed, scales) if scale_fmt == "fp16" else (packed, scales, rowsc)


def _torch_dequant_int2(packed, scales):
    """fp32 (code - 1.5) * s (K:353-357)."""
    n = packed.shape[0]
    k = packed.shape[1] * 4
    codes = torch.stack([(packed >> (2 * ORDER[j])) & 3 for j in range(4)], -1).view(n, k).float() - 1.5
    g = k // scales.shape[1]
    return (codes.view(n, k // g, g) * scales.float().unsqueeze(-1)).view(n, k)


# ----------------------------------------------------------------------------------------------------------
# weight preparation entry points: CUDA tensors run the native kernels (libfp4x.so, fp4x_prep.cu); CPU tensors
# run the torch restatements above (there is no GPU to run on).  The packed bytes are the reference's: its
# quantizers evaluate `tensor / scalar` as a multiplication by the fp32 reciprocal on CUDA devices and as a
# division on the CPU, and the native kernels follow the device's rule by default (FP4X_PREP_DIV=ieee|recip
# overrides it).
# ----------------------------------------------------------------------------------------------------------

def _prep_mode():
    import os
    v = os.environ.get("FP4X_PREP_DIV", "recip").lower()
    if v not in ("ieee", "recip"):
        raise ValueError("FP4X_PREP_DIV must be 'ieee' or 'recip'")
    return N.DIV_IEEE if v == "ieee" else N.DIV_RECIP


def _prep_input(w):
    """(contiguous weights, input dtype code) for the native quantizers."""
    codes = {torch.float32: N.IN_F32, torch.bfloat16: N.IN_BF16, torch.float16: N.IN_F16}
    if w.dtype not in codes:
        w = w.float()
    w = w.contiguous()
    return w, codes[w.dtype]


def prefetch_l2(*tensors):
    """Pull the tensors' bytes (a later op's packed weights and scales) from HBM into L2 on the current stream
    (fp4x_prefetch_l2).  Not part of the reference API: a decode step issues it one op ahead so the dependent GEMV
    chain reads its weights from L2 while HBM keeps streaming.  At most 16 tensors per call."""
    ts = [t for t in tensors if t is not None and t.numel() > 0]
    if not ts:
        return
    for t in ts:
        if not t.is_cuda:
            raise ValueError("prefetch_l2 takes CUDA tensors")
    ptrs = (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])
    # the span from the first to the last element (the whole tensor when it is contiguous)
    spans = [(sum((n - 1) * st for n, st in zip(t.shape, t.stride())) + 1) * t.element_size() for t in ts]
    sizes = (ctypes.c_int64 * len(ts))(*spans)
    N.call("fp4x_prefetch_l2", ctypes.cast(ptrs, ctypes.c_void_p), ctypes.cast(sizes, ctypes.c_void_p), len(ts),
           N.stream_of(ts[0]))


def _interleave_native(t, hc, bj):
    t = t.contiguous()
    n = t.shape[0]
    out = torch.empty_like(t)
    row_bytes = t.numel() * t.element_size() // n
    N.call("fp4x_interleave_rows", N.ptr(t), row_bytes, n, hc, bj, N.ptr(out), N.stream_of(t))
    return out


@torch.no_grad()
def quantize_w8(w, div_mode=None):
    """Symmetric int8 per 64-group: s = max(amax, 1e-12) / 127, q = clamp(round(w / s), +-127) (K:138-144).
    Returns (q int8 [N, K], s fp32 [N, K/64])."""
    if not w.is_cuda:
        return _torch_quantize_w8(w)
    n, k = w.shape
    wc, code = _prep_input(w)
    q = torch.empty((n, k), dtype=torch.int8, device=w.device)
    s = torch.empty((n, k // 64), dtype=torch.float32, device=w.device)
    N.call("fp4x_quantize_w8", N.ptr(wc), code, n, k, N.ptr(q), N.ptr(s),
           _prep_mode() if div_mode is None else div_mode, N.stream_of(wc))
    return q, s


@torch.no_grad()
def quantize_w6(w, qmax=31, clip_search=0, div_mode=None):
    """6-bit g32 (K:179-202): s = max(fp16(amax/qmax), 6.2e-5), codes = clamp(round(w/s), -qmax-1, qmax) + 32.
    Returns (L [N,K/2] u8, H [N,K/4] u8, S [N,K/32] f16).  The clip search (clip_search > 0, a quality probe of the
    reference whose choice depends on the summation order of torch's reductions) stays in torch."""
    if not w.is_cuda or clip_search:
        return _torch_quantize_w6(w, qmax, clip_search)
    n, k = w.shape
    wc, code = _prep_input(w)
    L = torch.empty((n, k // 2), dtype=torch.uint8, device=w.device)
    H = torch.empty((n, k // 4), dtype=torch.uint8, device=w.device)
    S = torch.empty((n, k // 32), dtype=torch.float16, device=w.device)
    N.call("fp4x_quantize_w6", N.ptr(wc), code, n, k, int(qmax), N.ptr(L), N.ptr(H), N.ptr(S),
           _prep_mode() if div_mode is None else div_mode, N.stream_of(wc))
    return L, H, S


@torch.no_grad()
def quantize_nv4(w, rows=2048, div_mode=None):
    """NVFP4 (K:277-300): gs = max(amax/6/448, 1e-30) (python float), block scale = e4m3(clamp(amax16/6/gs,
    2^-9, 448)), magnitudes by nearest e2m1 level with ties to the lower level.  Returns (P, S e4m3, gs)."""
    if not w.is_cuda:
        return _torch_quantize_nv4(w, rows)
    n, k = w.shape
    wc, code = _prep_input(w)
    amax = torch.empty((1,), dtype=torch.float32, device=w.device)
    N.call("fp4x_amax", N.ptr(wc), code, wc.numel(), N.ptr(amax), N.stream_of(wc))
    gs = max(float(amax.item()) / 6.0 / 448.0, 1e-30)  # a host sync, as the reference's .item()
    P = torch.empty((n, k // 2), dtype=torch.uint8, device=w.device)
    S = torch.empty((n, k // 16), dtype=torch.float8_e4m3fn, device=w.device)
    N.call("fp4x_quantize_nv4", N.ptr(wc), code, n, k, gs, N.ptr(P), N.ptr(S),
           _prep_mode() if div_mode is None else div_mode, N.stream_of(wc))
    return P, S, gs


@torch.no_grad()
def quantize_int2(weight, scale_fmt="fp16", group=16, div_mode=None):
    """INT2 per group (K:330-351): s = max(amax, 1e-8)/1.5 (fp16, or e4m3 relative to an fp32 row scale),
    code = clamp(floor(w/s) + 2, 0, 3), value (code - 1.5) * s; 4 codes per byte at bit pairs ORDER.
    Returns (packed, s) for fp16 scales, (packed, s_e4m3, row_scale) for e4m3 (torch only: the reference does
    not ship that variant)."""
    if not weight.is_cuda or scale_fmt != "fp16":
        return _torch_quantize_int2(weight, scale_fmt, group)
    n, k = weight.shape
    wc, code = _prep_input(weight)
    P = torch.empty((n, k // 4), dtype=torch.uint8, device=weight.device)
    S = torch.empty((n, k // group), dtype=torch.float16, device=weight.device)
    N.call("fp4x_quantize_int2", N.ptr(wc), code, n, k, group, N.ptr(P), N.ptr(S),
           _prep_mode() if div_mode is None else div_mode, N.stream_of(wc))
    return P, S


@torch.no_grad()
def mx8_dequant(w8, s_u8, rows=2048):
    """MXFP8 -> fp32 [N, K]: e4m3 * 2^(s - 127) (K:261-267)."""
    if not w8.is_cuda:
        return _torch_mx8_dequant(w8, s_u8, rows)
    n, k = w8.shape
    w, s = _rows(_u8(w8)), _rows(_u8(s_u8))
    out = torch.empty((n, k), dtype=torch.float32, device=w8.device)
    N.call("fp4x_mx8_dequant", N.ptr(w), N.ptr(s), n, k, N.ptr(out), N.stream_of(w))
    return out


@torch.no_grad()
def dequant_nv4(P, S, gs):
    """[N, K/2] e2m1 pairs + [N, K/16] e4m3 scales -> fp32 [N, K] = v * s * gs (K:420-426)."""
    if not P.is_cuda:
        return _torch_dequant_nv4(P, S, gs)
    n, k = P.shape[0], P.shape[1] * 2
    out = torch.empty((n, k), dtype=torch.float32, device=P.device)
    N.call("fp4x_dequant_nv4", N.ptr(_rows(P)), N.ptr(_rows(_u8(S))), float(gs), n, k, N.ptr(out), N.stream_of(P))
    return out


@torch.no_grad()
def dequant_int2(packed, scales):
    """fp32 (code - 1.5) * s (K:353-357)."""
    if not packed.is_cuda or scales.dtype != torch.float16:
        return _torch_dequant_int2(packed, scales)
    n, k = packed.shape[0], packed.shape[1] * 4
    group = k // scales.shape[1]
    out = torch.empty((n, k), dtype=torch.float32, device=packed.device)
    N.call("fp4x_dequant_int2", N.ptr(_rows(packed)), N.ptr(_rows(scales)), group, n, k, N.ptr(out),
           N.stream_of(packed))
    return out


@torch.no_grad()
def nv4_unswizzle_scales(sc):
    """NVFP4 scales stored as swizzled 128-row x 4-column tiles -> row-major [N, K/16] (the preparation of the
    draft head's source scales, x/fp4patch.py:296: reshape(n//128, kb//4, 32, 4, 4).transpose(1, 3))."""
    n, kb = sc.shape
    u = _u8(sc)
    if not sc.is_cuda:
        return u.reshape(n // 128, kb // 4, 32, 4, 4).transpose(1, 3).reshape(n, kb).view(sc.dtype)
    u = _rows(u)
    out = torch.empty((n, kb), dtype=torch.uint8, device=sc.device)
    N.call("fp4x_nv4_unswizzle_scales", N.ptr(u), n, kb, N.ptr(out), N.stream_of(u))
    return out.view(sc.dtype)


class PackedCache:
    """Packed weights kept on disk between runs (safetensors files, one per weight), so a restarted server skips
    the quantization pass that the reference repeats lazily on every start (x/fp4patch.py:61-83, :206-214).

    get(name, build) returns the tuple `build()` produces (tensors, plus python floats such as the NVFP4 global
    scale), loading it from `<dir>/<name>.safetensors` when present and writing it there otherwise."""

    def __init__(self, directory, device="cuda"):
        import os
        self.dir = directory
        self.device = torch.device(device)
        os.makedirs(directory, exist_ok=True)

    def path(self, name):
        import os
        safe = "".join(c if c.isalnum() or c in "._-" else "_" for c in name)
        return os.path.join(self.dir, safe + ".safetensors")

    def get(self, name, build):
        import os
        from safetensors.torch import load_file, save_file
        p = self.path(name)
        if os.path.exists(p):
            d = load_file(p, device=str(self.device))
            items = []
            for i in range(len(d)):
                t = d[f"{i}"]
                items.append(float(t.item()) if t.dtype == torch.float64 and t.dim() == 0 else t)
            return tuple(items)
        out = build()
        tensors = {}
        for i, v in enumerate(out):
            tensors[f"{i}"] = (v.detach().contiguous().cpu() if torch.is_tensor(v)
                               else torch.tensor(float(v), dtype=torch.float64))
        tmp = p + ".tmp"
        save_file(tensors, tmp)
        os.replace(tmp, p)
        return out


# ----------------------------------------------------------------------------------------------------------
# a decode step in one persistent launch (fp4x_step_*)
# ----------------------------------------------------------------------------------------------------------

class StepProgram:
    """The GEMV-family ops of a decode step, run as one persistent launch (one CTA per SM).

    Record the ops with the methods below (inputs and outputs are caller-owned tensors that must stay alive), then
    prepare() once outside graph capture and run() every step.  Each op computes what its standalone entry point
    computes (the same weights and rounding points; partial sums in a fixed order).  With serial=True every op also
    waits for the op recorded before it, the order of a single stream; otherwise an op waits only for the earlier
    ops whose buffers it reads or overwrites.  1..8 tokens."""

    def __init__(self, device, m, serial=True):
        if not 1 <= m <= 8:
            raise ValueError("StepProgram runs 1..8 tokens")
        self.device = torch.device(device)
        self.m = m
        self.serial = serial
        self.ops = []
        self.keep = []
        self.table = None

    def _add(self, kind, x, p0, p1, s, out, n, k, gs=1.0, out2=None, out_dtype=torch.bfloat16, lr=0, hc=0, bj=0,
             nrm=None):
        if self.table is not None:
            raise RuntimeError("the step is already prepared")
        if x.shape[0] != self.m or x.dtype != torch.bfloat16 or x.stride(-1) != 1:
            raise ValueError(f"activations must be bf16 [{self.m}, k] with unit column stride")
        self.keep.extend(t for t in (x, p0, p1, s, out, out2, nrm) if t is not None)
        op = N.StepOpC(kind, x.data_ptr(), x.stride(0), p0.data_ptr(), 0 if p1 is None else p1.data_ptr(),
                       s.data_ptr(), float(gs), out.data_ptr(), 0 if out2 is None else out2.data_ptr(),
                       out.stride(0), N.dtype_code(out_dtype), n, k, lr, hc, bj,
                       0 if nrm is None else nrm.data_ptr(), 0 if nrm is None else nrm.stride(0))
        self.ops.append(op)
        return out

    def nv4(self, x, wp, s, gs, out):
        return self._add(N.STEP_NV4, x, _rows(wp), None, _rows(_u8(s)), out, wp.shape[0], wp.shape[1] * 2, gs=gs,
                         out_dtype=out.dtype)

    def w6(self, x, L, H, S, out):
        return self._add(N.STEP_W6, x, _rows(L), _rows(H), _rows(S), out, L.shape[0], L.shape[1] * 2,
                         out_dtype=out.dtype)

    def w8(self, x, q, s, out):
        return self._add(N.STEP_W8, x, _rows(q), None, _rows(s.float()), out, q.shape[0], q.shape[1],
                         out_dtype=out.dtype)

    def mx8(self, x, w8, s, out):
        return self._add(N.STEP_MX8, x, _rows(_u8(w8)), None, _rows(_u8(s)), out, w8.shape[0], w8.shape[1],
                         out_dtype=out.dtype)

    def hc_down(self, x, q, s, di, bot, lr, hc):
        return self._add(N.STEP_HC_DOWN, x, _rows(q), None, _rows(s.float()), di, q.shape[0], q.shape[1], out2=bot,
                         lr=lr, hc=hc)

    def hc_up(self, bot, qi, si, nrm, out, hc, bj=8):
        return self._add(N.STEP_HC_UP, bot, _rows(qi), None, _rows(si.float()), out, qi.shape[0], qi.shape[1],
                         hc=hc, bj=bj, nrm=nrm)

    def prepare(self):
        arr = (N.StepOpC * len(self.ops))(*self.ops)
        tb, wb, nc = N._sz(0), N._sz(0), N._i64(0)
        N.call("fp4x_step_query", arr, len(self.ops), self.m, 1 if self.serial else 0, ctypes.byref(tb),
               ctypes.byref(wb), ctypes.byref(nc))
        self.table = torch.empty(tb.value + 64, dtype=torch.uint8, device=self.device)
        off = (-self.table.data_ptr()) % 64
        self.table_view = self.table[off:off + tb.value]
        self.ws = torch.empty(max(wb.value, 16), dtype=torch.uint8, device=self.device)
        self.cnt = torch.zeros(nc.value, dtype=torch.int32, device=self.device)
        N.call("fp4x_step_prepare", arr, len(self.ops), self.m, 1 if self.serial else 0, N.ptr(self.table_view),
               tb.value, N.ptr(self.ws), self.ws.numel(), N.ptr(self.cnt), nc.value)
        return self

    def run(self):
        if self.table is None:
            self.prepare()
        N.call("fp4x_step_run", N.ptr(self.table_view), N.stream_of(self.table))

    def trace(self, on=True):
        """Diagnostic: record a [CTAs, ops, 8] timeline on later runs (ns: op start, inputs ready, staged, done,
        first weight stage ready, stage loop done, last flush done); returns the int64 buffer (read it after the
        run), or None when turned off."""
        if self.table is None:
            self.prepare()
        if not on:
            N.call("fp4x_step_trace", N.ptr(self.table_view), None, 0)
            return None
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        buf = torch.zeros(sms, len(self.ops), 8, dtype=torch.int64, device=self.device)
        N.call("fp4x_step_trace", N.ptr(self.table_view), N.ptr(buf), buf.numel())
        self._trace = buf
        return buf

    def __del__(self):
        if getattr(self, "table", None) is not None:
            try:
                N.lib().fp4x_step_release(N.ptr(self.table_view))
            except Exception:  # noqa: BLE001 - interpreter shutdown
                pass
