"""Column-sharded matmul across 2 GPUs over NCCL (skipped with fewer than 2 GPUs). The gathered
output equals, bit for bit, the single-GPU results of the same column shards (same kernel, same
shape, same K order); against the unsharded product it agrees within the GEMM tolerance (a shard
can get a different automatic K split than the full matrix)."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, ret):
    import datetime

    import torch.distributed as dist

    import gtx16_fp16 as g
    from gtx16_fp16.dist import ShardedMatmul, batch_slice, gather_rows, shard_bounds

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        gen = torch.Generator(device="cuda").manual_seed(0)
        M, K, N = 1024, 2048, 4096
        a = torch.randn(M, K, device="cuda", generator=gen).half()
        w = (torch.randn(K, N, device="cuda", generator=gen) * K ** -0.5).half()
        n0, n1 = shard_bounds(N, world, rank)
        y = ShardedMatmul(w[:, n0:n1].contiguous(), N)(a)
        shards = [g.mm_t(a, w[:, b0:b1].contiguous(), None, torch.float16)
                  for b0, b1 in (shard_bounds(N, world, r) for r in range(world))]
        ok = torch.equal(y, torch.cat(shards, dim=1))
        ref = a.double() @ w.double()
        ok = ok and ((y.double() - ref).norm() / ref.norm()).item() < 1e-3
        full = g.mm_t(a, w, None, torch.float16)
        rows = gather_rows(full[batch_slice(M, world, rank)], M)
        ok = ok and torch.equal(rows, full)
        torch.cuda.synchronize()
        ret[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


def test_sharded_matmul_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ret = mp.Manager().dict()
    mp.spawn(_worker, args=(2, _free_port(), ret), nprocs=2, join=True)
    assert dict(ret) == {0: True, 1: True}
