"""The reference's CPU path for the decode GEMVs, restated in torch eager: dequantize, then `x.float() @ W.T`.
TEST AND BASELINE INFRASTRUCTURE ONLY (bench.py's cpu_baseline / --impl reference legs).

The reference has no CPU kernels of its own: on a machine without its Triton kernels, the same arithmetic is its
torch dequantizers (`x/fp4x_kernels.py`, cited K:<line>) followed by an fp32 matmul, which is also how its tuners
build their reference outputs (`x/probes/tune.py:27,33`).  The reference cannot be installed here (it has no
package metadata), so these functions restate those dequantizers in torch on the same packed layouts:

* mx8_dequant      K:261-267   e4m3 * 2^(e - 127), fp32
* w8_dequant       K:126-129   bf16(f32(q) * s) per 64-group (the kernel's weights), as fp32
* w6_dequant       K:160-170   bf16((q - 32) * f32(s)) per 32-group, as fp32
* nv4_dequant      K:85-92     bf16(e2m1 * f32(e4m3 scale)) per 16-group, as fp32 (times gs after the sum, K:94)
* int2_dequant     K:316-322   bf16((code - 1.5) * f32(s)), as fp32

Two variants are timed (the baseline plan of the survey): (i) dequantize on every call, what an eager forward does,
and (ii) the matmul alone against weights dequantized once beforehand.
"""
from __future__ import annotations

import torch

ORDER = (0, 2, 1, 3)  # K:327-328
_E2M1 = torch.tensor([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], dtype=torch.float32)


def mx8_dequant(w8, s):
    n, k = w8.shape
    v = w8.view(torch.float8_e4m3fn).float().view(n, k // 32, 32)
    return (v * torch.exp2(s.float() - 127.0)[..., None]).view(n, k)


def w8_dequant(q, s):
    n, k = q.shape
    return (q.float().view(n, k // 64, 64) * s.float()[..., None]).to(torch.bfloat16).float().view(n, k)


def w6_dequant(L, H, S):
    n = L.shape[0]
    k = L.shape[1] * 2
    Li, Hi = L.to(torch.int32), H.to(torch.int32)
    lo = torch.stack((Li & 15, Li >> 4), -1).view(n, k)
    hi = torch.stack([(Hi >> (2 * ORDER[t])) & 3 for t in range(4)], -1).view(n, k)
    q = ((lo | (hi << 4)) - 32).float().view(n, k // 32, 32)
    return (q * S.float()[..., None]).to(torch.bfloat16).float().view(n, k)


def nv4_dequant(P, S):
    n = P.shape[0]
    k = P.shape[1] * 2
    Pi = P.to(torch.int64)
    v = _E2M1[torch.stack((Pi & 15, Pi >> 4), -1).view(n, k)].view(n, k // 16, 16)
    sc = S.view(torch.float8_e4m3fn).float()
    return (v * sc[..., None]).to(torch.bfloat16).float().view(n, k)


def int2_dequant(P, S):
    n = P.shape[0]
    k = P.shape[1] * 4
    Pi = P.to(torch.int32)
    c = torch.stack([(Pi >> (2 * ORDER[t])) & 3 for t in range(4)], -1).view(n, k).float() - 1.5
    g = k // S.shape[1]
    return (c.view(n, k // g, g) * S.float()[..., None]).to(torch.bfloat16).float().view(n, k)


def matmul(x, w):
    """fp32 product of bf16 activations [M, K] with fp32 weights [N, K]."""
    return x.float() @ w.T
