"""Vocab-sharded fast LM head over several GPUs of one box (one process per GPU, torch.distributed over NCCL).

The reference runs its head on one GPU (`x/fp4patch.py:370-378`: INT2 coarse logits, top-512, exact MXFP8
rescore).  Here the vocabulary rows are split into contiguous shards, one per rank.  Each rank runs the fused
head on its shard (coarse pass, local top-C, local exact rescore), the ranks exchange their C candidates with one
all-gather of a packed [3, M, C] tensor (coarse fp32, exact fp32, global vocab id as int32 bits), and every rank
merges the P*C candidates with the merge kernel: the global top-C by coarse value (value descending, id
ascending) and the argmax of the exact values among them.

This is exact: the global top-C is a subset of the union of the per-shard top-Cs, and the coarse value of a row
does not depend on how the vocabulary is split (the INT2 kernel sums each row in an order fixed by K alone).
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
        self.V, self.C, self.world, self.group = V, C, world, group

    def local(self, h):
        """The shard's own candidates: (coarse, exact, global ids) [M, C] each, and the coarse bf16 logits."""
        h = F._act(h)
        m, k = h.shape
        rows = self.stop - self.start
        group = k // self.S.shape[1]
        full = torch.empty((m, rows), dtype=torch.bfloat16, device=h.device)
        idx = torch.empty((m, self.C), dtype=torch.int32, device=h.device)
        exact = torch.empty((m, self.C), dtype=torch.float32, device=h.device)
        coarse = torch.empty((m, self.C), dtype=torch.float32, device=h.device)
        ws, cnt = N.head_scratch(m, rows, k, self.C, group, h.device)
        N.call("fp4x_fast_head", N.ptr(h), h.stride(0), N.ptr(self.P), N.ptr(self.S), group, N.ptr(self.w8),
               N.ptr(self.s8), m, rows, k, self.C, N.ptr(full), full.stride(0), N.ptr(idx), N.ptr(exact),
               N.ptr(coarse), None, N.ptr(ws), ws.numel(), N.ptr(cnt), cnt.numel(), N.stream_of(h))
        return coarse, exact, idx + self.start, full

    def __call__(self, h):
        coarse, exact, gidx, _ = self.local(h)
        if self.world == 1:
            co, ex, gi = coarse[None], exact[None], gidx[None]
        else:
            co, ex, gi = gather_candidates(coarse, exact, gidx, self.group)
        return F.head_merge(co, ex, gi, self.V)
