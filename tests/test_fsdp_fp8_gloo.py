"""Host-side logic of the FSDP2 per-block FP8 all-gather on CPU gloo ranks
(world 1 and 2).  The quantizer is swapped for the CPU oracle (the product
runs the CUDA kernel); every rank checks that the unsharded weight FSDP2
hands the linear is exactly the 128x128 quantization of the full weight."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def distribute_like(param, full):
    """``full`` laid out like the (possibly sharded) parameter."""
    from torch.distributed.tensor import DTensor, distribute_tensor

    if isinstance(param, DTensor):
        return distribute_tensor(full, param.device_mesh, param.placements)
    return full


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch.distributed as dist
    from torch.distributed.fsdp import fully_shard

    import oracle
    import practice_cuda_b200.fsdp_fp8 as ff
    from practice_cuda_b200.fp8_linear import BlockFP8Weight, FP8BlockLinear

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        calls = []

        def counting_quant(w):
            calls.append(1)
            return oracle.per_block_quant(w, block_m=128, block_n=128)

        ff.quantize_weight = counting_quant
        torch.manual_seed(0)
        full = torch.randn(512, 384) * 0.02
        m = torch.nn.Sequential(FP8BlockLinear(384, 512, bias=False))
        with torch.no_grad():
            m[0].weight.copy_(full)
        ff.enable_fp8_all_gather(m)
        fully_shard(m)
        seen = {}

        def fwd(self, x):
            w = self.weight
            seen["type"] = type(w)
            seen["data"] = w._data.view(torch.uint8).clone()
            seen["scale"] = w._scale.clone()
            return x @ torch.zeros(384, 512)

        FP8BlockLinear.forward = fwd
        for _ in range(2):  # first unshard and the re-gather into `out`
            m(torch.randn(2, 384))
        def matches(w_full):
            ref_q, ref_s = oracle.per_block_quant(w_full, block_m=128, block_n=128)
            return (seen["type"] is BlockFP8Weight and torch.equal(seen["data"], ref_q.view(torch.uint8))
                    and torch.equal(seen["scale"], ref_s))

        ok = matches(full)
        ok = ok and len(calls) == 1  # the re-gather reused the cached quantization
        # An in-place update (what the optimizer does) invalidates the cache.
        delta = torch.randn(512, 384, generator=torch.Generator().manual_seed(1)) * 0.01
        m.reshard()  # the optimizer steps on sharded parameters
        with torch.no_grad():
            m[0].weight.add_(distribute_like(m[0].weight, delta))
        w1 = m[0].weight.full_tensor()
        m(torch.randn(2, 384))
        ok = ok and matches(w1) and len(calls) == 2
        # precompute after another update: the next unshard quantizes nothing.
        m.reshard()
        with torch.no_grad():
            m[0].weight.add_(distribute_like(m[0].weight, delta))
        w2 = m[0].weight.full_tensor()
        ok = ok and ff.precompute_fp8_block_weights(m) == 1 and len(calls) == 3
        m(torch.randn(2, 384))
        ok = ok and matches(w2) and len(calls) == 3
        # Writes through aliases of the parameter (what EMA updates and
        # checkpoint loaders do via .data / .detach()) also invalidate it.
        for alias in (lambda w: w.data, lambda w: w.detach()):
            m.reshard()
            with torch.no_grad():
                local = m[0].weight
                local = getattr(local, "_local_tensor", local)
                alias(local).add_(alias(local) * 0 + 0.001)
            w3 = m[0].weight.full_tensor()
            before = len(calls)
            m(torch.randn(2, 384))
            ok = ok and matches(w3) and len(calls) == before + 1
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [1, 2])
def test_fp8_all_gather_hooks_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    results = sorted(q.get() for _ in range(world))
    assert all(ok for _, ok in results), results


def test_shard_not_tile_aligned_rejected():
    import practice_cuda_b200.fsdp_fp8 as ff

    w = ff.FP8AllGatherWeight(torch.zeros(100, 128))

    class _Mesh:
        def size(self):
            return 2

    with pytest.raises(ValueError, match="whole 128-row tiles"):
        w.fsdp_pre_all_gather(_Mesh(), torch.Size([200, 128]), (128, 1), None, None)
