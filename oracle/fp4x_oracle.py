"""CPU oracle for the fp4x decode-GEMV path.  TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the arithmetic of the reference plugin's kernel library
(`x/fp4x_kernels.py`, cited below as K:<line>) and of its dispatch layer (`x/fp4patch.py`, cited as
P:<line>).  It is the checker for the CUDA path: only `tests/`, `__graft_entry__.smoke()` and the
`cpu_baseline` / `--impl reference` legs of `bench.py` may import it.  The product path
(`fp4x_kernels.py`, `libfp4x.so`) never imports or calls anything here.

Pinning: the quantizers, dequantizers and dequantize-then-matmul outputs below are checked bit-exactly
(quantizers) or to fp32 rounding (matmuls) against golden vectors produced by running the reference's own
functions on CPU (`tests/golden/make_golden.py`, fixtures in `tests/golden/*.npz`).  The epilogues of the
fused hyper-connection kernels and the fast-head selection are restated from the Triton source lines cited
in each function (the Triton kernels themselves cannot run without a GPU).

Conventions
-----------
* bf16 / f16 / e4m3 values are carried as float32 (or float64) numpy arrays holding exactly representable
  values; `bf16()` rounds to nearest-even like `torch.Tensor.to(torch.bfloat16)`.
* Matrix products are accumulated in float64 so that the oracle gives the exact sum of the (exactly
  representable) products; the CUDA kernels accumulate in fp32 and are compared within stated tolerances.
"""
from __future__ import annotations

import numpy as np

# K:327-328: element j of each 4-group lives in bit pair ORDER[j]
ORDER = (0, 2, 1, 3)

# ----------------------------------------------------------------------------------------------------------
# scalar formats
# ----------------------------------------------------------------------------------------------------------


def bf16(a) -> np.ndarray:
    """Round float32 values to bfloat16 (nearest-even), returned as float32."""
    a = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).copy()
    nan = np.isnan(a)
    out[nan] = np.nan
    return out


def bf16_bits_to_f32(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(a) -> np.ndarray:
    return (bf16(a).view(np.uint32) >> 16).astype(np.uint16)


def _e4m3_table() -> np.ndarray:
    t = np.zeros(256, dtype=np.float32)
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        m = b & 7
        if e == 15 and m == 7:
            t[b] = np.nan
        elif e == 0:
            t[b] = s * (m / 8.0) * 2.0 ** -6
        else:
            t[b] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return t


E4M3 = _e4m3_table()
_E4M3_POS = E4M3[:127].astype(np.float64)  # codes 0x00..0x7e, increasing, all finite


def e4m3_decode(b) -> np.ndarray:
    return E4M3[np.asarray(b, dtype=np.uint8)]


def e4m3_encode(a) -> np.ndarray:
    """float -> e4m3fn byte, round-to-nearest-even (ties to the even code).  |a| must be <= 448."""
    a = np.asarray(a, dtype=np.float32).astype(np.float64)
    mag = np.abs(a)
    hi = np.searchsorted(_E4M3_POS, mag, side="left").clip(0, 126)
    lo = (hi - 1).clip(0, 126)
    dlo = mag - _E4M3_POS[lo]
    dhi = _E4M3_POS[hi] - mag
    pick_hi = (dhi < dlo) | ((dhi == dlo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo).astype(np.uint8)
    code = np.where(mag == 0, 0, code).astype(np.uint8)
    sign = (np.signbit(a)).astype(np.uint8) << 7
    return (code | sign).astype(np.uint8)


E2M1 = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], dtype=np.float32)  # K:423


def _f32(v) -> np.float32:
    return np.float32(v)


# ----------------------------------------------------------------------------------------------------------
# quantizers (restatements of the reference's torch quantizers)
# ----------------------------------------------------------------------------------------------------------


def quantize_w8(w):
    """K:138-144.  Returns (q int8 [N,K], s float32 [N,K/64])."""
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    f = w.reshape(n, k // 64, 64)
    s = np.maximum(np.abs(f).max(-1), _f32(1e-12)) / _f32(127.0)
    q = np.clip(np.rint(f / s[..., None]), -127, 127).astype(np.int8).reshape(n, k)
    return q, s.astype(np.float32)


def quantize_w6(w, qmax: int = 31):
    """K:179-202 (clip_search=0).  Returns (L u8 [N,K/2], H u8 [N,K/4], S f16 [N,K/32])."""
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    f = w.reshape(n, k // 32, 32)
    s = (np.abs(f).max(-1, keepdims=True) / _f32(qmax)).astype(np.float16).astype(np.float32)
    s = np.maximum(s, _f32(6.2e-5))
    q = (np.clip(np.rint(f / s), -qmax - 1, qmax).astype(np.int32) + 32).reshape(n, k)
    lo = q & 15
    hi = q >> 4
    L = (lo[:, 0::2] | (lo[:, 1::2] << 4)).astype(np.uint8)
    H = (hi[:, 0::4] | (hi[:, 2::4] << 2) | (hi[:, 1::4] << 4) | (hi[:, 3::4] << 6)).astype(np.uint8)
    S = s.reshape(n, k // 32).astype(np.float16)
    return L, H, S


def quantize_nv4(w):
    """K:277-300.  Returns (P u8 [N,K/2] low nibble = even k, S e4m3 bytes [N,K/16], gs python float)."""
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    amax_all = float(np.abs(w).max())
    gs = max(amax_all / 6.0 / 448.0, 1e-30)
    gs32 = _f32(gs)
    f = w.reshape(n, k // 16, 16)
    sc = np.abs(f).max(-1, keepdims=True) / _f32(6.0) / gs32
    sc = np.clip(sc, _f32(2.0 ** -9), _f32(448.0))
    sb = e4m3_encode(sc)
    sf = e4m3_decode(sb) * gs32
    v = np.clip(f / sf, _f32(-6), _f32(6))
    mids = (E2M1[1:8] + E2M1[0:7]) / _f32(2)
    mag = np.searchsorted(mids, np.abs(v), side="left").astype(np.int64)
    q = (mag | ((v < 0).astype(np.int64) << 3)).reshape(n, k)
    P = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)
    return P, sb.reshape(n, k // 16), gs


def quantize_int2(w, group: int = 16):
    """K:330-351 (scale_fmt="fp16").  Returns (P u8 [N,K/4], S f16 [N,K/group])."""
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    f = w.reshape(n, k // group, group)
    s = (np.maximum(np.abs(f).max(-1, keepdims=True), _f32(1e-8)) / _f32(1.5)).astype(np.float16)
    sf = s.astype(np.float32)
    idx = np.clip(np.floor(f / sf) + 2, 0, 3).astype(np.uint8).reshape(n, k // 4, 4)
    b = np.zeros((n, k // 4), dtype=np.uint8)
    for j in range(4):
        b |= (idx[..., j] << (2 * ORDER[j])).astype(np.uint8)
    return b, s.reshape(n, k // group)


def quantize_mx8(w):
    """MXFP8 packing used for the synthetic weights (BASELINE C1 recipe; in the served model the packing comes
    from b12x): e8m0 byte = 127 + ceil(log2(amax32 / 448)) (amax = 0 -> byte 0), codes = e4m3(w / 2^e).
    Returns (codes u8 [N,K], scales u8 [N,K/32])."""
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    f = w.reshape(n, k // 32, 32)
    amax = np.abs(f).max(-1)
    ratio = amax / _f32(448.0)
    m, e = np.frexp(ratio)
    ce = np.where(m > 0.5, e, e - 1)
    ce = np.where(amax == 0, -127, ce).astype(np.int64)
    sbyte = (127 + ce).clip(0, 254).astype(np.uint8)
    scale = np.ldexp(np.float64(1.0), ce).astype(np.float64)
    vals = (f.astype(np.float64) / scale[..., None]).astype(np.float32)
    codes = e4m3_encode(vals).reshape(n, k)
    return codes, sbyte


# ----------------------------------------------------------------------------------------------------------
# dequantizers: exact fp32 values (reference dequantizers) and the kernels' bf16 weights
# ----------------------------------------------------------------------------------------------------------


def mx8_dequant(w8, s):
    """K:261-267: e4m3 * 2^(s-127) in fp32 (exact)."""
    n, k = w8.shape
    v = e4m3_decode(w8).reshape(n, k // 32, 32).astype(np.float64)
    sc = np.ldexp(1.0, np.asarray(s, dtype=np.int64) - 127)
    return (v * sc[..., None]).reshape(n, k).astype(np.float32)


def w8_weights(q, s):
    """K:126-129: bf16(f32(q) * s) per 64-group."""
    n, k = q.shape
    f = q.astype(np.float32).reshape(n, k // 64, 64) * s.astype(np.float32)[..., None]
    return bf16(f.reshape(n, k))


def w6_codes(L, H):
    """K:160-167: q = (lo | hi << 4) - 32, with hi bit pairs in ORDER."""
    n = L.shape[0]
    k = L.shape[1] * 2
    L = L.astype(np.int32)
    H = H.astype(np.int32)
    lo = np.empty((n, k), dtype=np.int32)
    lo[:, 0::2] = L & 15
    lo[:, 1::2] = L >> 4
    hi = np.empty((n, k), dtype=np.int32)
    for t in range(4):
        hi[:, t::4] = (H >> (2 * ORDER[t])) & 3
    return (lo | (hi << 4)) - 32


def w6_weights(L, H, S):
    """K:168-170: bf16(f32(q) * f32(s)) per 32-group."""
    q = w6_codes(L, H).astype(np.float32)
    n, k = q.shape
    f = q.reshape(n, k // 32, 32) * S.astype(np.float32)[..., None]
    return bf16(f.reshape(n, k))


def nv4_values(P):
    n = P.shape[0]
    v = np.empty((n, P.shape[1] * 2), dtype=np.float32)
    v[:, 0::2] = E2M1[P & 15]
    v[:, 1::2] = E2M1[P >> 4]
    return v


def nv4_weights(P, S):
    """K:85-92: bf16(e2m1 * f32(e4m3 scale)) per 16-group (the global scale is applied after the sum, K:94)."""
    v = nv4_values(P)
    n, k = v.shape
    f = v.reshape(n, k // 16, 16) * e4m3_decode(S).reshape(n, k // 16, 1)
    return bf16(f.reshape(n, k))


def dequant_nv4(P, S, gs):
    """K:420-426: fp32 v * s * gs."""
    v = nv4_values(P)
    n, k = v.shape
    return (v.reshape(n, k // 16, 16) * e4m3_decode(S).reshape(n, k // 16, 1) * _f32(gs)).reshape(n, k)


def int2_codes(P):
    n = P.shape[0]
    k = P.shape[1] * 4
    c = np.empty((n, k), dtype=np.int32)
    for t in range(4):
        c[:, t::4] = (P.astype(np.int32) >> (2 * ORDER[t])) & 3
    return c


def dequant_int2(P, S):
    """K:353-357: fp32 (code - 1.5) * s."""
    c = int2_codes(P).astype(np.float32) - _f32(1.5)
    n, k = c.shape
    g = k // S.shape[1]
    return (c.reshape(n, k // g, g) * S.astype(np.float32)[..., None]).reshape(n, k)


def int2_weights(P, S):
    """K:318-322: bf16((code - 1.5) * f32(s))."""
    return bf16(dequant_int2(P, S))


# ----------------------------------------------------------------------------------------------------------
# GEMV semantics: out = x . W^T with the kernels' weights, exact (float64) sums
# ----------------------------------------------------------------------------------------------------------


def _mm(x, wt):
    return np.asarray(x, dtype=np.float64) @ np.asarray(wt, dtype=np.float64).T


def mx8_linear(x, w8, s):
    """K:9-29 / K:65: x . bf16(mx8_dequant)^T (the dequant is exact in bf16)."""
    return _mm(x, mx8_dequant(w8, s))


def w8_linear(x, q, s):
    """K:116-135 / K:147."""
    return _mm(x, w8_weights(q, s))


def w6_linear(x, L, H, S):
    """K:151-176 / K:270."""
    return _mm(x, w6_weights(L, H, S))


def nv4_linear(x, P, S, gs):
    """K:73-113: (x . bf16(v*s)^T) * gs."""
    return _mm(x, nv4_weights(P, S)) * np.float64(_f32(gs))


def bf16_linear(x, w):
    """K:32-47 / K:69."""
    return _mm(x, w)


def int2_logits(x, P, S):
    """K:304-325 / K:359-364 (ROW_SCALE off)."""
    return _mm(bf16(x), int2_weights(P, S))


def refine_mx8_rows(x, idx, w8, s):
    """K:367-381: exact fp32 dots of MXFP8 rows idx[m, c] with x[m] (returned as float64 exact sums)."""
    m, C = idx.shape
    out = np.empty((m, C), dtype=np.float64)
    for i in range(m):
        rows = mx8_dequant(w8[idx[i]], s[idx[i]])
        out[i] = rows.astype(np.float64) @ np.asarray(x[i], dtype=np.float64)
    return out


def refine_nv4_rows(x, idx, P, S, gs):
    """K:391-409: sum of bf16(v*s) * x, times gs."""
    m, C = idx.shape
    out = np.empty((m, C), dtype=np.float64)
    for i in range(m):
        rows = nv4_weights(P[idx[i]], S[idx[i]])
        out[i] = (rows.astype(np.float64) @ np.asarray(x[i], dtype=np.float64)) * np.float64(_f32(gs))
    return out


# ----------------------------------------------------------------------------------------------------------
# hyper-connection mixer (K:438-526, P:201-247)
# ----------------------------------------------------------------------------------------------------------


def sigmoid32(t):
    t = np.asarray(t, dtype=np.float32)
    return (_f32(1.0) / (_f32(1.0) + np.exp(-t))).astype(np.float32)


def hc_down_epilogue(total, lr: int, hc: int):
    """K:460-464: di = bf16(sum); bot = bf16(t * sigmoid(t)), t = bf16(f32(di) / HC), for cols < LR."""
    di = bf16(np.asarray(total, dtype=np.float32))
    t = bf16(di / _f32(hc))
    bot = bf16(t[:, :lr] * sigmoid32(t[:, :lr]))
    return di, bot


def hc_up_epilogue(g_total, nrm, hc: int):
    """K:486-493 on un-interleaved gate logits g_total [M, HC*H] (row s*H + j): returns [M, H] bf16 values.
    Stream sum order ((s0 + s1) + (s2 + s3)) (pairwise), which the CUDA kernels also use."""
    m, n = g_total.shape
    h = n // hc
    g = bf16(np.asarray(g_total, dtype=np.float32))
    gate = bf16(sigmoid32(g))
    nrm = np.asarray(nrm, dtype=np.float32)[:, : hc * h]
    prods = [bf16(nrm[:, s * h:(s + 1) * h] * gate[:, s * h:(s + 1) * h]) for s in range(hc)]
    tot = _pairwise_sum(prods)
    return bf16(tot / _f32(hc))


def _pairwise_sum(terms):
    terms = [np.asarray(t, dtype=np.float32) for t in terms]
    while len(terms) > 1:
        nxt = []
        for i in range(0, len(terms), 2):
            nxt.append((terms[i] + terms[i + 1]).astype(np.float32) if i + 1 < len(terms) else terms[i])
        terms = nxt
    return terms[0]


def interleave_up(q, s, hc: int, bj: int):
    """K:513-517: reorder [HC*H, K] rows so each BJ-column tile holds its HC stream rows contiguously."""
    n = q.shape[0]
    h = n // hc
    idx = np.arange(n).reshape(hc, h // bj, bj).transpose(1, 0, 2).reshape(-1)
    return q[idx], s[idx]


def hc_mixer(x, qd, sd, qu, su, lr: int, hc: int):
    """P:231-247 (unfused W8 route) == P:201-220 (fused route): returns (di, bot, block_input) as float32
    arrays of bf16 values.  qu/su are in the ORIGINAL (non-interleaved) row order."""
    total = w8_linear(x, qd, sd)
    di, bot = hc_down_epilogue(total, lr, hc)
    g = w8_linear(bot, qu, su)
    return di, bot, hc_up_epilogue(g, x, hc)


# ----------------------------------------------------------------------------------------------------------
# fast LM head (P:370-378) and draft head (P:315-327)
# ----------------------------------------------------------------------------------------------------------


def topk_order(vals, c: int):
    """Indices of the c largest values per row, ordered by (value desc, index asc)."""
    vals = np.asarray(vals, dtype=np.float64)
    m, v = vals.shape
    out = np.empty((m, c), dtype=np.int64)
    for i in range(m):
        order = np.lexsort((np.arange(v), -vals[i]))
        out[i] = order[:c]
    return out


def fast_head(h, P, S, w8, s, C: int = 512):
    """Coarse INT2 logits -> top-C -> exact MXFP8 rescore scattered into the coarse bf16 vector.
    Returns (full bf16-valued logits float32 [M,V], idx [M,C], exact [M,C] float64, coarse float64 [M,V])."""
    coarse = int2_logits(h, P, S)
    idx = topk_order(coarse, C)
    exact = refine_mx8_rows(h, idx, w8, s)
    full = bf16(coarse.astype(np.float32))
    for i in range(full.shape[0]):
        full[i, idx[i]] = bf16(exact[i].astype(np.float32))
    return full, idx, exact, coarse


def draft_head(h, P, S, wp, sn, gs, C: int = 64):
    """INT2 coarse over the draft rows -> top-C -> exact NVFP4 rescore.  Returns (idx [M,C], vals [M,C])."""
    coarse = int2_logits(h, P, S)
    idx = topk_order(coarse, C)
    return idx, refine_nv4_rows(h, idx, wp, sn, gs), coarse


def ambiguous_topk(vals, c: int, bound):
    """For set comparisons under fp32 summation-order noise: returns (sure_in, sure_out) boolean masks.
    sure_in: value > v_c + bound (must be selected); sure_out: value < v_c - bound (must not be)."""
    vals = np.asarray(vals, dtype=np.float64)
    srt = -np.sort(-vals, axis=1)
    vc = srt[:, c - 1:c]
    bound = np.asarray(bound, dtype=np.float64)
    return vals > vc + bound, vals < vc - bound
