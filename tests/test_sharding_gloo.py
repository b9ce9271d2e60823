"""Batch/row sharding on CPU gloo ranks (world 2 and 3): every rank computes
its shard with the CPU oracle, shards are gathered, and the result equals
the unsharded computation."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from practice_cuda_b200.sharding import gather_shards, shard_range, shard_sizes


def test_shard_range_partitions():
    for total in [0, 1, 7, 32, 33]:
        for world in [1, 2, 3, 4, 8]:
            ranges = [shard_range(total, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == total
            for (s0, e0), (s1, _) in zip(ranges, ranges[1:]):
                assert e0 == s1
            sizes = shard_sizes(total, world)
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, total, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle

        g = torch.Generator().manual_seed(0)
        a = torch.randn((total, 8, 256), generator=g).bfloat16()
        b = (torch.randn((total, 256, 16), generator=g) * 0.02).bfloat16()
        b0, b1 = shard_range(total, rank, world)
        ya, sa = oracle.per_block_quant(a[b0:b1], block_m=1, block_n=128)
        yb, sb = oracle.per_block_quant(b[b0:b1], block_m=128, block_n=128)
        c = oracle.scaled_bmm_promoted_reference(ya, sa, yb, sb, qbm=1, qbk=128, qbn=128, out_dtype=torch.float32)
        full = gather_shards(c, total)
        if rank == 0:
            ya, sa = oracle.per_block_quant(a, block_m=1, block_n=128)
            yb, sb = oracle.per_block_quant(b, block_m=128, block_n=128)
            ref = oracle.scaled_bmm_promoted_reference(ya, sa, yb, sb, qbm=1, qbk=128, qbn=128,
                                                       out_dtype=torch.float32)
            q.put(bool(torch.equal(full, ref)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,total", [(2, 5), (3, 7)])
def test_sharded_bmm_gloo(world, total):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, total, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert q.get() is True
