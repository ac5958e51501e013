"""GPU parity of the LM-head path: exact top-C selection, exact MXFP8 / NVFP4 rescoring, the fused fast and
draft heads, and the merge of a vocab-sharded head.

Set semantics: the top-C set is defined on fp32 coarse values with the total order (value desc, index asc).
Against the oracle's float64 coarse values, indices whose value lies within the fp32 accumulation bound of the
C-th value are ambiguous (not checked); all others must agree.  Against the kernel's own fp32 coarse values the
selection must be exact.
"""
import numpy as np
import pytest
import torch

import fp4x_kernels as F
from oracle import fp4x_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def gen(seed, *shape, std=1.0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g) * std


def exact_topc(vals, C):
    """(value desc, index asc) top-C of float values per row, returned as sorted index arrays."""
    vals = np.asarray(vals)
    out = []
    for r in vals:
        order = np.lexsort((np.arange(r.size), -r.astype(np.float64)))
        out.append(np.sort(order[:C]))
    return np.stack(out)


@pytest.mark.parametrize("m,v,c", [(1, 1000, 10), (3, 248320, 512), (16, 65536, 64), (4, 5000, 4096)])
def test_topk_exact_on_fp32(m, v, c):
    vals = gen(1, m, v) * 3
    vals[0, 7] = vals[0].max() + 1  # a clear maximum
    idx, sel = F.topk_indices(vals.to(DEV), c)
    ref = exact_topc(vals.numpy(), c)
    assert np.array_equal(idx.cpu().numpy(), ref)
    assert np.array_equal(sel.cpu().numpy(), np.take_along_axis(vals.numpy(), ref, 1))


def test_topk_ties_and_overflow_path():
    m, v, c = 3, 200000, 512
    vals = gen(2, m, v).to(torch.bfloat16).float()  # heavy ties
    vals[1] = 1.0                                   # all equal: candidate list overflows, index order decides
    vals[2, ::3] = 5.0                              # 66667 equal maxima
    idx, _ = F.topk_indices(vals.to(DEV), c)
    ref = exact_topc(vals.numpy(), c)
    assert np.array_equal(idx.cpu().numpy(), ref)
    assert np.array_equal(idx[1].cpu().numpy(), np.arange(c))
    # scratch is left clean: a second call gives the same answer
    idx2, _ = F.topk_indices(vals.to(DEV), c)
    assert torch.equal(idx, idx2)


def mx8_head(v, k, seed):
    w = gen(seed, v, k, std=0.02)
    codes, sc = F.quantize_mx8(w.to(DEV))
    return codes, sc


@pytest.mark.parametrize("m", [1, 3, 16])
def test_refine_mx8_exact_and_in_place(m):
    v, k, c = 4096, 2560, 512
    codes, sc = mx8_head(v, k, 3)
    x = gen(4, m, k).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(v, generator=torch.Generator().manual_seed(10 + i))[:c] for i in range(m)])
    out = torch.zeros(m, v, dtype=torch.bfloat16, device=DEV)
    F.refine_mx8_(out, x.to(DEV), idx.to(DEV), codes, sc)
    ref = O.refine_mx8_rows(x.float().numpy(), idx.numpy(), codes.view(torch.uint8).cpu().numpy(), sc.cpu().numpy())
    got = np.take_along_axis(out.float().cpu().numpy(), idx.numpy(), 1)
    assert np.abs(got - O.bf16(ref.astype(np.float32))).max() <= np.abs(ref).max() * 2.0 ** -8
    untouched = torch.ones(m, v, dtype=torch.bool)
    untouched.scatter_(1, idx, False)
    assert out.cpu()[untouched].abs().max().item() == 0.0
    out32 = torch.zeros(m, v, dtype=torch.float32, device=DEV)
    F.refine_mx8_(out32, x.to(DEV), idx.to(torch.int32).to(DEV), codes, sc)
    got32 = np.take_along_axis(out32.cpu().numpy(), idx.numpy(), 1)
    assert np.abs(got32 - ref).max() <= 2e-6 * np.abs(ref).max()


@pytest.mark.parametrize("m", [1, 3])
def test_refine_nv4(m):
    v, k, c = 2048, 2560, 64
    P, S, gs = F.quantize_nv4(gen(5, v, k, std=0.02).to(DEV))
    x = gen(6, m, k).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(v, generator=torch.Generator().manual_seed(20 + i))[:c] for i in range(m)])
    out = F.refine_nv4(x.to(DEV), idx.to(DEV), P, S, gs)
    ref = O.refine_nv4_rows(x.float().numpy(), idx.numpy(), P.cpu().numpy(), S.view(torch.uint8).cpu().numpy(), gs)
    assert np.abs(out.cpu().numpy() - ref).max() <= 2e-6 * np.abs(ref).max()


def coarse_bound(x, P, S, rows):
    """fp32 accumulation bound for the coarse logits of `rows`: K * 2^-23 * sum |x_k w_k| (generous)."""
    w = O.int2_weights(P[rows], S[rows]).astype(np.float64)
    k = w.shape[1]
    return (np.abs(x.astype(np.float64)) @ np.abs(w).T) * (k * 2.0 ** -23)


@pytest.mark.parametrize("m", [1, 3, 16])
def test_fast_head_full_vocab(m):
    """248320-row INT2 head + top-512 + exact MXFP8 rescore, checked by size-independent properties plus the
    oracle on the selected rows and a sample of the others."""
    V, K, C = 248320, 2560, 512
    w = gen(7, V, K, std=0.02).to(DEV)
    codes, sc = F.quantize_mx8(w)
    P, S = F.quantize_int2(F.mx8_dequant(codes, sc), group=16)
    del w
    h = gen(8, m, K).to(torch.bfloat16)
    full, idx, exact, amax = F.fast_head(h.to(DEV), P, S, codes, sc, C)
    coarse = F.int2_logits(h.to(DEV), P, S, V)  # the same fp32 coarse values the head ranks
    idx_np = idx.cpu().numpy()
    # (1) the selection is the exact top-C of the fp32 coarse values
    assert np.array_equal(idx_np, exact_topc(coarse.cpu().numpy(), C))
    # (2) coarse values agree with the oracle on the selected rows and on a sample
    Pn, Sn = P.cpu().numpy(), S.cpu().numpy()
    xs = h.float().numpy()
    rng = np.random.default_rng(0)
    sample = rng.choice(V, 2048, replace=False)
    for i in range(m):
        rows = np.concatenate([idx_np[i], sample])
        ref = O.int2_logits(xs[i:i + 1], Pn[rows], Sn[rows])[0]
        bound = coarse_bound(xs[i:i + 1], Pn, Sn, rows)[0]
        assert np.all(np.abs(coarse.cpu().numpy()[i, rows] - ref) <= bound + 1e-30)
    # (3) exact values = oracle MXFP8 dots of the selected rows; full logits carry them, coarse elsewhere
    ex_ref = O.refine_mx8_rows(xs, idx_np.astype(np.int64), codes.view(torch.uint8).cpu().numpy(), sc.cpu().numpy())
    assert np.abs(exact.cpu().numpy() - ex_ref).max() <= 2e-6 * np.abs(ex_ref).max()
    fullc = full.cpu()
    assert torch.equal(torch.gather(fullc, 1, idx.long().cpu()), exact.cpu().to(torch.bfloat16))
    mask = torch.ones(m, V, dtype=torch.bool)
    mask.scatter_(1, idx.long().cpu(), False)
    assert torch.equal(fullc[mask], coarse.cpu().to(torch.bfloat16)[mask])
    # (4) argmax = exact argmax over the candidates (first maximum = lower vocab id)
    for i in range(m):
        e = exact.cpu().numpy()[i]
        j = np.lexsort((idx_np[i], -e.astype(np.float64)))[0]
        assert amax[i].item() == idx_np[i, j]


def test_fast_head_against_oracle_small_vocab():
    V, K, C, m = 20000, 2560, 512, 3
    w = gen(9, V, K, std=0.02)
    codes, sc = F.quantize_mx8(w)
    P, S = F.quantize_int2(F.mx8_dequant(codes, sc), group=16)
    h = gen(10, m, K).to(torch.bfloat16)
    full, idx, exact, amax = F.fast_head(h.to(DEV), P.to(DEV), S.to(DEV), codes.to(DEV), sc.to(DEV), C)
    ofull, oidx, oexact, ocoarse = O.fast_head(h.float().numpy(), P.numpy(), S.numpy(),
                                               codes.view(torch.uint8).numpy(), sc.numpy(), C)
    bound = coarse_bound(h.float().numpy(), P.numpy(), S.numpy(), np.arange(V))
    sure_in, sure_out = O.ambiguous_topk(ocoarse, C, bound)
    got = np.zeros((m, V), dtype=bool)
    np.put_along_axis(got, idx.cpu().numpy().astype(np.int64), True, 1)
    assert np.all(got[sure_in]) and not np.any(got[sure_out])
    # argmax agrees with the oracle's exact argmax (unless the top two exact values are within fp32 noise)
    for i in range(m):
        oe = oexact[i]
        top2 = np.sort(oe)[-2:]
        if top2[1] - top2[0] > 1e-5 * abs(top2[1]):
            assert amax[i].item() == oidx[i][np.argmax(oe)]


def test_draft_head_with_scatter():
    Vd, K, C, m, Vfull = 65536, 2560, 64, 3, 248320
    wd = gen(11, Vd, K, std=0.02).to(DEV)
    wp, sn, gs = F.quantize_nv4(wd)
    P, S = F.quantize_int2(F.dequant_nv4(wp, sn, gs), group=16)
    ids = torch.sort(torch.randperm(Vfull, generator=torch.Generator().manual_seed(12))[:Vd]).values.to(DEV)
    h = gen(13, m, K).to(torch.bfloat16).to(DEV)
    idx, vals, full = F.draft_head(h, P, S, wp, sn, gs, C, ids=ids, full_vocab=Vfull)
    coarse = F.int2_logits(h, P, S, Vd)
    assert np.array_equal(idx.cpu().numpy(), exact_topc(coarse.cpu().numpy(), C))
    ref = O.refine_nv4_rows(h.float().cpu().numpy(), idx.cpu().numpy().astype(np.int64), wp.cpu().numpy(),
                            sn.view(torch.uint8).cpu().numpy(), gs)
    assert np.abs(vals.cpu().numpy() - ref).max() <= 2e-6 * np.abs(ref).max()
    fc = full.cpu()
    gid = ids.cpu()[idx.long().cpu()]
    assert torch.equal(torch.gather(fc, 1, gid), vals.cpu().to(torch.bfloat16))
    mask = torch.ones_like(fc, dtype=torch.bool)
    mask.scatter_(1, gid, False)
    assert torch.isinf(fc[mask]).all() and (fc[mask] < 0).all()


@pytest.mark.parametrize("parts", [2, 4, 8])
def test_sharded_head_merge_equals_unsharded(parts):
    """Vocab-sharded head on one GPU: per-shard coarse + local top-C + exact rescore, then the merge kernel.
    The merged set and argmax must equal the unsharded head's."""
    V, K, C, m = 248320, 2560, 512, 3
    w = gen(14, V, K, std=0.02).to(DEV)
    codes, sc = F.quantize_mx8(w)
    P, S = F.quantize_int2(F.mx8_dequant(codes, sc), group=16)
    del w
    h = gen(15, m, K).to(torch.bfloat16).to(DEV)
    _, idx_full, exact_full, amax_full = F.fast_head(h, P, S, codes, sc, C)
    per = V // parts
    co, ex, gi = [], [], []
    for p in range(parts):
        sl = slice(p * per, (p + 1) * per)
        coarse = F.int2_logits(h, P[sl], S[sl], per)
        li, lv = F.topk_indices(coarse, C)
        exact = torch.empty(m, C, dtype=torch.float32, device=DEV)
        out = torch.zeros(m, per, dtype=torch.float32, device=DEV)
        F.refine_mx8_(out, h, li, codes[sl], sc[sl])
        exact = torch.gather(out, 1, li.long())
        co.append(lv); ex.append(exact); gi.append(li + p * per)
    idx, _, exm, amax = F.head_merge(torch.stack(co), torch.stack(ex), torch.stack(gi), V)
    assert torch.equal(idx, idx_full)
    assert torch.equal(amax, amax_full)
    assert torch.equal(exm, exact_full)


def test_sharded_head_single_rank_full_equals_fast_head():
    """world = 1: ShardedFastHead.full is F.fast_head (no collective)."""
    from fp4x_shard import ShardedFastHead
    V, K, C, m = 20000, 2560, 512, 3
    w = gen(16, V, K, std=0.02).to(DEV)
    codes, sc = F.quantize_mx8(w)
    P, S = F.quantize_int2(F.mx8_dequant(codes, sc), group=16)
    h = gen(17, m, K).to(torch.bfloat16).to(DEV)
    ref = F.fast_head(h, P, S, codes, sc, C)
    got = ShardedFastHead(P, S, codes, sc, V, 0, 1, C=C).full(h)
    for a, b in zip(got, ref):
        assert torch.equal(a, b)
