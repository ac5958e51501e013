"""The reference plugin's own call sequences (x/fp4patch.py) replayed against this library on the GPU.

The plugin imports the kernel library as `F` and chains its calls; these tests run those chains verbatim (the
Triton tile arguments included, which this library accepts and ignores) and check each against the CPU oracle or
against this library's fused equivalents:

* fast head (P:370-378): int2_logits(..., out_dtype=bf16) -> torch.topk on the bf16 logits -> refine_mx8_ in place;
  the plugin's self-check (P:360-368: argmax agrees with the exact head, top-20 within 1e-2) must pass, and the
  sequence is compared with F.fast_head, which ranks the fp32 coarse values;
* draft head (P:315-327): int2_logits -> topk -> refine_nv4 -> scatter into -inf, against F.draft_head;
* fused hyper-connection mixer at the served geometry (P:201-220, n_down 336 = 320 + 4 injection + padding);
* the W8 decode hook for MTP linears and router gates (P:258-272) and the dense W6 / NVFP4 routes (P:123-133).
"""
import numpy as np
import pytest
import torch

import fp4x_kernels as F
from oracle import fp4x_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
K = 2560


def gen(seed, *shape, std=1.0):
    return torch.randn(*shape, generator=torch.Generator().manual_seed(seed)) * std


def rel_err(out, ref):
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return np.abs(out - ref).max() / max(np.abs(ref).max(), 1e-30)


@pytest.fixture(scope="module")
def head():
    v = 65536
    w = gen(1, v, K, std=0.02)
    codes, sc = F.quantize_mx8(w)
    P, S = F.quantize_int2(F.mx8_dequant(codes, sc), group=16)
    exact = O.mx8_dequant(codes.view(torch.uint8).numpy(), sc.numpy()).astype(np.float64)
    return v, codes.to(DEV), sc.to(DEV), P.to(DEV), S.to(DEV), exact


@pytest.mark.parametrize("m", [1, 3])
def test_fast_head_plugin_sequence(head, m):
    v, w, s, P, S, exact = head
    C = 512
    h = gen(10 + m, m, K).to(torch.bfloat16).to(DEV)
    # P:370-378, verbatim call sequence
    coarse = F.int2_logits(h, P, S, w.shape[0], out_dtype=torch.bfloat16)
    idx = torch.topk(coarse, C, dim=-1).indices
    out = F.refine_mx8_(coarse, h, idx, w, s)
    assert out is coarse and out.dtype == torch.bfloat16
    # the plugin's self-check against the exact head (P:363-367), whose logits are bf16 as well: argmax agrees and
    # the exact top-20 logits are the exact head's bf16 values (to one bf16 step: fp32 summation order)
    ref = h.float().cpu().numpy().astype(np.float64) @ exact.T
    got = out.float().cpu().numpy()
    # both heads return bf16 logits, whose argmax takes the first of equal bf16 values
    assert np.array_equal(got.argmax(-1), O.bf16(ref.astype(np.float32)).argmax(-1))
    top = np.argsort(-ref, axis=1)[:, :20]
    want = O.bf16(np.take_along_axis(ref, top, 1).astype(np.float32)).astype(np.float64)
    diff = np.abs(np.take_along_axis(got, top, 1) - want)
    assert np.all(diff <= 2.0 ** (np.floor(np.log2(np.abs(want))) - 7))
    # the selected rows hold the exact values (bf16)
    sel = idx.cpu().numpy()
    assert np.abs(np.take_along_axis(got, sel, 1) - O.bf16(np.take_along_axis(ref, sel, 1).astype(np.float32))).max() \
        <= np.abs(ref).max() * 2.0 ** -8
    # against the fused head, which ranks the fp32 coarse values: same argmax; the candidate sets differ only where
    # bf16 rounding reorders near-equal coarse values at the selection boundary
    full, fidx, fexact, famax = F.fast_head(h, P, S, w, s, C)
    assert np.array_equal(famax.cpu().numpy(), ref.argmax(-1))  # the fused head's argmax is over fp32 exact values
    for r in range(m):
        a, b = set(sel[r].tolist()), set(fidx[r].cpu().numpy().tolist())
        assert len(a ^ b) <= 0.05 * C, f"row {r}: {len(a ^ b)} candidates differ"


def test_draft_head_plugin_sequence():
    vd, vocab, dc = 8192, 248320, 64
    w = gen(2, vd, K, std=0.02)
    wp, sn, gs = F.quantize_nv4(w)
    c = F.quantize_int2(F.dequant_nv4(wp, sn, gs), group=16)
    ids = torch.sort(torch.randperm(vocab, generator=torch.Generator().manual_seed(3))[:vd]).values
    wp, sn, Pc, Sc, ids = wp.to(DEV), sn.to(DEV), c[0].to(DEV), c[1].to(DEV), ids.to(DEV)
    h = gen(4, 3, K).to(torch.bfloat16).to(DEV)
    # P:316-327, verbatim
    co = F.int2_logits(h, Pc, Sc, ids.numel())
    cand = torch.topk(co, dc, dim=-1).indices
    vals = F.refine_nv4(h, cand, wp, sn, gs)
    full = torch.full((h.shape[0], vocab), float("-inf"), dtype=torch.bfloat16, device=DEV)
    full = full.scatter_(1, ids[cand], vals.to(torch.bfloat16))
    # the fused draft head: the same candidates (fp32 ranking in both) and the same vector
    fidx, fvals, ffull = F.draft_head(h, Pc, Sc, wp, sn, gs, dc, ids=ids, full_vocab=vocab)
    for r in range(3):
        assert set(cand[r].cpu().tolist()) == set(fidx[r].cpu().tolist())
    assert torch.equal(full, ffull)
    ref = O.refine_nv4_rows(h.float().cpu().numpy(), cand.cpu().numpy(), wp.cpu().numpy(),
                            sn.view(torch.uint8).cpu().numpy(), gs)
    assert rel_err(vals.cpu().numpy(), ref) < 5e-5


def test_hc_mixer_plugin_route_served_geometry():
    hc, H, lr = 4, 2560, 320
    wd = gen(5, 336, hc * H, std=0.02)       # input_mix_weight_down_block_inject (use_combine)
    wu = gen(6, hc * H, lr, std=0.02)         # input_mix_weight_up
    x = gen(7, 3, hc * H).to(torch.bfloat16).to(DEV)
    q8 = F.quantize_w8(wd.to(DEV))
    qu = F.HCFused.interleave_up(*F.quantize_w8(wu.to(DEV)), hc, 8)
    fx = F.HCFused(x.device)                   # P:212, default n_down = 336
    di, bot = fx.down(x, *q8, lr, hc, (32, 256, 8, 4))
    block_input = F.HCFused.up(bot, *qu, x, hc, (8, 64, 4))
    injection = di[:, lr:lr + hc]
    assert block_input.shape == (3, H) and injection.shape == (3, hc)
    qd, sd = q8
    qun, sun = F.quantize_w8(wu.to(DEV))
    di_u, bot_u, out_u = F.hc_mixer_unfused(x, qd, sd, qun, sun, lr, hc)
    assert torch.equal(di, di_u) and torch.equal(bot, bot_u) and torch.equal(block_input, out_u)
    odi, obot, oout = O.hc_mixer(x.float().cpu().numpy(), qd.cpu().numpy(), sd.cpu().numpy(), qun.cpu().numpy(),
                                 sun.cpu().numpy(), lr, hc)
    assert rel_err(di.float().cpu(), odi) < 1e-2 and rel_err(block_input.float().cpu(), oout) < 1e-2


@pytest.mark.parametrize("n,k", [(13312, 2560), (2560, 5120), (512, 2560)])
def test_w8_hook_mtp_and_gate_shapes(n, k):
    """FP4X_MTP_W8 / FP4X_GATE=w8 route: op(x2, weight, True) -> w8_linear(x, *quantize_w8(w), cfg) (P:185,261)."""
    w = gen(n + k, n, k, std=0.02).to(DEV)
    x = gen(8, 3, k).to(torch.bfloat16).to(DEV)
    q, s = F.quantize_w8(w)
    y = F.w8_linear(x.contiguous(), q, s, (32, 256 if k % 256 == 0 else 64, 1, 4))
    ref = O.w8_linear(x.float().cpu().numpy(), q.cpu().numpy(), s.cpu().numpy())
    assert y.dtype == torch.bfloat16 and rel_err(y.float().cpu(), ref) < 1e-2
    g = F.bf16_linear(x, w.to(torch.bfloat16), (16, 256, 1, 4))    # FP4X_GATE=bf16 (P:270)
    assert rel_err(g.float().cpu(), O.bf16_linear(x.float().cpu().numpy(),
                                                  w.to(torch.bfloat16).float().cpu().numpy())) < 1e-2


def test_dense_routes():
    """FP4X_DENSE=w6 and the NVFP4 shapes (P:123-133): the lazily quantized weight, then the GEMV with the plugin's
    cfg tuple."""
    n, k = 4096, 2560
    wf = gen(9, n, k, std=0.02).to(DEV)
    x = gen(10, 3, k).to(torch.bfloat16).to(DEV)
    q6 = F.quantize_w6(wf, 31, 0)
    y6 = F.w6_linear(x, *q6, (32, 256, 1, 4))
    ref6 = O.w6_linear(x.float().cpu().numpy(), *(t.cpu().numpy() for t in q6))
    assert rel_err(y6.float().cpu(), ref6) < 1e-2
    q4 = F.quantize_nv4(wf)
    y4 = F.nv4_linear(x, *q4, (32, 256, 4))
    ref4 = O.nv4_linear(x.float().cpu().numpy(), q4[0].cpu().numpy(), q4[1].view(torch.uint8).cpu().numpy(), q4[2])
    assert rel_err(y4.float().cpu(), ref4) < 1e-2
