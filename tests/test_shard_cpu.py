"""Host logic of the vocab-sharded head (fp4x_shard.py) on CPU: shard ranges, candidate packing, and the
candidate exchange over a world-size-2 gloo process group; plus the exactness argument of the merge, checked with
the oracle (the global top-C equals the top-C of the union of the shard top-Cs)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fp4x_shard import fix_full, gather_candidates, gather_full, pack_candidates, shard_range, unpack_candidates
from oracle import fp4x_oracle as O


def test_shard_range_covers_vocab():
    for V, world in ((248320, 1), (248320, 2), (248320, 8), (65536, 4), (1000, 3)):
        spans = [shard_range(V, r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == V
        assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
    with pytest.raises(ValueError):
        shard_range(100, 2, 2)
    with pytest.raises(ValueError):
        shard_range(1, 0, 2)


def test_pack_unpack_roundtrip():
    g = torch.Generator().manual_seed(3)
    m, c = 3, 512
    co = torch.randn(m, c, generator=g)
    ex = torch.randn(m, c, generator=g)
    gi = torch.randint(0, 248320, (m, c), generator=g, dtype=torch.int32)
    packed = pack_candidates(co, ex, gi)
    assert packed.shape == (3, m, c) and packed.dtype == torch.float32
    # two ranks' packs laid end to end, as the all-gather produces them
    both = torch.cat([packed.reshape(-1), packed.reshape(-1) * 0 + packed.reshape(-1)])
    a, b, ids = unpack_candidates(both, 2, m, c)
    assert torch.equal(a[0], co) and torch.equal(b[1], ex) and torch.equal(ids[0], gi) and torch.equal(ids[1], gi)
    with pytest.raises(TypeError):
        pack_candidates(co, ex, gi.long())


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m, c = 3, 64
        g = torch.Generator().manual_seed(100 + rank)
        co = torch.randn(m, c, generator=g)
        ex = torch.randn(m, c, generator=g)
        gi = torch.randint(rank * 1000, rank * 1000 + 1000, (m, c), generator=g, dtype=torch.int32)
        a, b, ids = gather_candidates(co, ex, gi)
        ok = True
        for r in range(world):
            g2 = torch.Generator().manual_seed(100 + r)
            ok &= torch.equal(a[r], torch.randn(m, c, generator=g2))
            ok &= torch.equal(b[r], torch.randn(m, c, generator=g2))
            ok &= torch.equal(ids[r], torch.randint(r * 1000, r * 1000 + 1000, (m, c), generator=g2,
                                                    dtype=torch.int32))
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def test_gather_candidates_two_ranks_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results == {0: True, 1: True}


def test_sharded_topc_union_contains_global_topc():
    """The merge step's exactness: the global top-C (value desc, id asc) is the top-C of the union of per-shard
    top-Cs, for any split, ties included."""
    rng = np.random.default_rng(5)
    V, m, C = 4096, 3, 64
    vals = rng.standard_normal((m, V)).astype(np.float32)
    vals[:, 100:140] = vals[:, 50:51]  # a block of exact ties
    ref = O.topk_order(vals, C)
    for parts in (2, 4, 8):
        per = V // parts
        cand_v, cand_i = [], []
        for p in range(parts):
            local = O.topk_order(vals[:, p * per:(p + 1) * per], C) + p * per
            cand_i.append(local)
            cand_v.append(np.take_along_axis(vals, local, axis=1))
        ci = np.concatenate(cand_i, axis=1)
        cv = np.concatenate(cand_v, axis=1)
        for r in range(m):
            order = np.lexsort((ci[r], -cv[r].astype(np.float64)))[:C]
            assert np.array_equal(np.sort(ci[r][order]), np.sort(ref[r]))


def _full_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        V, m = 1001, 3  # 3 ranks: shards of 333, 333, 335 (the last one is longer)
        ref = (torch.arange(m * V, dtype=torch.float32).reshape(m, V) * 0.25).to(torch.bfloat16)
        a, b = shard_range(V, rank, world)
        full = gather_full(ref[:, a:b].clone(), V, rank, world)
        q.put((rank, bool(torch.equal(full, ref))))
    finally:
        dist.destroy_process_group()


def test_gather_full_unequal_shards_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_full_worker, args=(r, 3, port, q)) for r in range(3)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results == {0: True, 1: True, 2: True}


def test_fix_full_restores_unselected_candidates():
    """After the all-gather every shard's rescored rows carry exact values; only the merged selection may keep them."""
    g = torch.Generator().manual_seed(9)
    P_, m, V, C = 2, 3, 400, 8
    coarse = torch.randn(m, V, generator=g)
    exact = coarse + 0.01 * torch.randn(m, V, generator=g)
    per = V // P_
    gi = torch.stack([torch.stack([torch.randperm(per, generator=g)[:C] + p * per for _ in range(m)])
                      for p in range(P_)]).to(torch.int32)                      # [P, M, C] shard candidates
    co = torch.gather(coarse[None].expand(P_, m, V), 2, gi.long())
    full = coarse.to(torch.bfloat16)
    for p in range(P_):                                                         # what each shard's head wrote
        full.scatter_(1, gi[p].long(), torch.gather(exact, 1, gi[p].long()).to(torch.bfloat16))
    idx = torch.sort(gi.permute(1, 0, 2).reshape(m, P_ * C)[:, ::2], dim=1).values[:, :C]  # a merged selection
    exm = torch.gather(exact, 1, idx.long())
    fix_full(full, co, gi, idx, exm)
    want = coarse.to(torch.bfloat16)
    want.scatter_(1, idx.long(), exm.to(torch.bfloat16))
    assert torch.equal(full, want)


def _lost_rank_worker(rank, world, port, q):
    """Rank 1 joins the group and leaves before the candidate exchange; rank 0 must get an error from its all-gather
    within the group's short timeout instead of waiting for ever."""
    import datetime
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()
        os._exit(0)  # between steps, with nothing in flight
    m, c = 3, 16
    co, ex = torch.zeros(m, c), torch.zeros(m, c)
    gi = torch.zeros(m, c, dtype=torch.int32)
    t0 = time.time()
    try:
        gather_candidates(co, ex, gi)
        q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001 - any failure of the collective is the expected outcome
        q.put((rank, f"raised after {time.time() - t0:.1f} s: {type(e).__name__}"))
    q.close()
    q.join_thread()
    os._exit(0)


def test_gather_candidates_raises_when_a_rank_is_gone():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_lost_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert results[1] == "left"
    assert results[0].startswith("raised after"), results[0]
    assert float(results[0].split()[2]) < 60.0
