"""Vocab-sharded fast head over two GPUs (one process per GPU, NCCL all-gather): the merged candidates and argmax
equal the unsharded head's, and so does the full [M, V] bf16 logit vector.  Skipped unless two GPUs are visible."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

V, K, C, M = 248320, 2560, 512, 3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _head(dev):
    import fp4x_kernels as F
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    w = torch.randn(V, K, device=dev, generator=g) * 0.02
    codes, sc = F.quantize_mx8(w)
    del w
    P, S = F.quantize_int2(F.mx8_dequant(codes, sc), group=16)
    g.manual_seed(78)
    h = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    return codes, sc, P, S, h


def _worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        import fp4x_kernels as F
        from fp4x_shard import ShardedFastHead, shard_range
        codes, sc, P, S, h = _head(dev)
        a, b = shard_range(V, rank, world)
        head = ShardedFastHead(P[a:b], S[a:b], codes[a:b], sc[a:b], V, rank, world, C=C)
        idx, _, exact, amax = head(h)
        full_ref, idx_full, exact_full, amax_full = F.fast_head(h, P, S, codes, sc, C)
        full, idx2, exact2, amax2 = head.full(h)
        torch.cuda.synchronize()
        ok = torch.equal(idx, idx_full) and torch.equal(amax, amax_full) and torch.equal(exact, exact_full)
        ok = ok and torch.equal(full, full_ref) and torch.equal(idx2, idx_full) and torch.equal(amax2, amax_full)
        ok = ok and torch.equal(exact2, exact_full)
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_head_two_gpus_equals_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert results == {0: True, 1: True}
