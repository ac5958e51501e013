"""Vocab-sharded fast LM head over several GPUs of one box (one process per GPU, torch.distributed over NCCL).

The reference runs its head on one GPU (`x/fp4patch.py:370-378`: INT2 coarse logits, top-512, exact MXFP8
rescore).  Here the vocabulary rows are split into contiguous shards, one per rank.  Each rank runs the fused
head on its shard (coarse pass, local top-C, local exact rescore), the ranks exchange their C candidates with one
all-gather of a packed [3, M, C] tensor (coarse fp32, exact fp32, global vocab id as int32 bits), and every rank
merges the P*C candidates with the merge kernel: the global top-C by coarse value (value descending, id
ascending) and the argmax of the exact values among them.

This is exact: the global top-C is a subset of the union of the per-shard top-Cs, and the coarse value of a row
does not depend on how the vocabulary is split (the INT2 kernel sums each row in an order fixed by K alone).

`ShardedFastHead.full` also returns the whole [M, V] bf16 logit vector the single-GPU head returns (coarse values,
with the exact values of the selected rows scattered in, `x/fp4patch.py:378`): one more all-gather of the shards'
bf16 logits, after which the rows a shard rescored but the merge did not select get their coarse value back.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

import fp4x_kernels as F
import fp4x_native as N


def shard_range(V, rank, world):
    """Contiguous row range [start, stop) of `rank`: equal shards, the last one takes the remainder."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    per = V // world
    if per < 1:
        raise ValueError(f"vocabulary of {V} rows cannot be split {world} ways")
    start = rank * per
    stop = V if rank == world - 1 else start + per
    return start, stop


def pack_candidates(coarse, exact, gidx):
    """[M, C] coarse fp32, exact fp32, int32 global ids -> one contiguous fp32 [3, M, C] (ids as raw bits)."""
    if coarse.shape != exact.shape or coarse.shape != gidx.shape:
        raise ValueError("candidate tensors must share one [M, C] shape")
    if gidx.dtype != torch.int32:
        raise TypeError("global ids must be int32")
    return torch.stack((coarse.float(), exact.float(), gidx.view(torch.float32)))


def unpack_candidates(gathered, world, m, c):
    """fp32 [world * 3 * M * C] from the all-gather -> (coarse [P, M, C], exact [P, M, C], gidx int32 [P, M, C])."""
    g = gathered.view(world, 3, m, c)
    return g[:, 0].contiguous(), g[:, 1].contiguous(), g[:, 2].contiguous().view(torch.int32)


def gather_candidates(coarse, exact, gidx, group=None):
    """All-gather every rank's [M, C] candidates (one collective) -> three [P, M, C] tensors, rank order."""
    world = dist.get_world_size(group)
    m, c = coarse.shape
    packed = pack_candidates(coarse, exact, gidx).reshape(-1)
    out = torch.empty(world * packed.numel(), dtype=torch.float32, device=packed.device)
    dist.all_gather_into_tensor(out, packed, group=group)
    return unpack_candidates(out, world, m, c)


def gather_full(full_local, V, rank, world, group=None):
    """All-gather every rank's bf16 logits [M, rows_r] into [M, V] (shards in rank order; the last shard, which may
    be longer, sets the padded width of the collective)."""
    m, rows = full_local.shape
    start, stop = shard_range(V, rank, world)
    if rows != stop - start:
        raise ValueError(f"rank {rank} holds {rows} logits, expected {stop - start}")
    width = V - shard_range(V, world - 1, world)[0]
    buf = full_local
    if rows != width:
        buf = torch.zeros((m, width), dtype=full_local.dtype, device=full_local.device)
        buf[:, :rows] = full_local
    out = torch.empty((world * m, width), dtype=full_local.dtype, device=full_local.device)
    dist.all_gather_into_tensor(out, buf.contiguous(), group=group)
    out = out.view(world, m, width)
    full = torch.empty((m, V), dtype=full_local.dtype, device=full_local.device)
    for r in range(world):
        a, b = shard_range(V, r, world)
        full[:, a:b] = out[r, :, :b - a]
    return full


def fix_full(full, co, gi, idx, exact):
    """In place: the rows every shard rescored get their coarse value back (bf16 of the fp32 coarse logit), then the
    merged selection gets its exact values.  co, gi: [P, M, C] gathered candidates; idx, exact: [M, C] merged."""
    p, m, c = co.shape
    full.scatter_(1, gi.permute(1, 0, 2).reshape(m, p * c).long(), co.permute(1, 0, 2).reshape(m, p * c).to(full.dtype))
    full.scatter_(1, idx.long(), exact.to(full.dtype))
    return full


class ShardedFastHead:
    """This rank's shard of the fast target head.

    P, S: INT2 codes / fp16 scales of rows [start, stop) (`quantize_int2` layout); w8, s8: the MXFP8 rows of the
    same range (`quantize_mx8` layout); V: the full vocabulary.  Calling it with h [M, K] bf16 returns, on every
    rank, (idx int32 [M, C] ascending global ids, coarse fp32 [M, C], exact fp32 [M, C], argmax int32 [M])."""

    def __init__(self, P, S, w8, s8, V, rank, world, C=512, group=None):
        self.start, self.stop = shard_range(V, rank, world)
        rows = self.stop - self.start
        if P.shape[0] != rows or w8.shape[0] != rows:
            raise ValueError(f"shard holds {P.shape[0]} rows, expected {rows}")
        if rows < C:
            raise ValueError(f"shard of {rows} rows is smaller than C={C}")
        self.P, self.S, self.w8, self.s8 = F._rows(P), F._rows(S), F._rows(F._u8(w8)), F._rows(F._u8(s8))
        self.V, self.C, self.rank, self.world, self.group = V, C, rank, world, group

    def local(self, h, argmax=False):
        """The shard's own candidates: (coarse, exact, global ids) [M, C] each, and the coarse bf16 logits; with
        `argmax`, also the global id of the largest exact value among the shard's candidates ([M] int32), which on a
        single shard is the head's answer (no merge needed)."""
        h = F._act(h)
        m, k = h.shape
        rows = self.stop - self.start
        group = k // self.S.shape[1]
        full = torch.empty((m, rows), dtype=torch.bfloat16, device=h.device)
        idx = torch.empty((m, self.C), dtype=torch.int32, device=h.device)
        exact = torch.empty((m, self.C), dtype=torch.float32, device=h.device)
        coarse = torch.empty((m, self.C), dtype=torch.float32, device=h.device)
        amax = torch.empty((m,), dtype=torch.int32, device=h.device) if argmax else None
        ws, cnt = N.head_scratch(m, rows, k, self.C, group, h.device)
        N.call("fp4x_fast_head", N.ptr(h), h.stride(0), N.ptr(self.P), N.ptr(self.S), group, N.ptr(self.w8),
               N.ptr(self.s8), m, rows, k, self.C, N.ptr(full), full.stride(0), N.ptr(idx), N.ptr(exact),
               N.ptr(coarse), N.ptr(amax), N.ptr(ws), ws.numel(), N.ptr(cnt), cnt.numel(), N.stream_of(h))
        gidx = idx + self.start if self.start else idx
        if argmax:
            return coarse, exact, gidx, full, (amax + self.start if self.start else amax)
        return coarse, exact, gidx, full

    def __call__(self, h):
        coarse, exact, gidx, _ = self.local(h)
        if self.world == 1:
            co, ex, gi = coarse[None], exact[None], gidx[None]
        else:
            co, ex, gi = gather_candidates(coarse, exact, gidx, self.group)
        return F.head_merge(co, ex, gi, self.V)

    def full(self, h):
        """The single-GPU head's outputs on every rank: (full bf16 [M, V], idx int32 [M, C], exact fp32 [M, C],
        argmax int32 [M]) -- `F.fast_head`'s return, bit for bit."""
        coarse, exact, gidx, full_local = self.local(h)
        if self.world == 1:
            co, ex, gi = coarse[None], exact[None], gidx[None]
        else:
            co, ex, gi = gather_candidates(coarse, exact, gidx, self.group)
        idx, _, exm, amax = F.head_merge(co, ex, gi, self.V)
        if self.world == 1:
            return full_local, idx, exm, amax
        full = gather_full(full_local, self.V, self.rank, self.world, self.group)
        return fix_full(full, co, gi, idx, exm), idx, exm, amax
