"""Host-side logic of the multi-GPU path on CPU: shard arithmetic, and the exchange of
ShardedMatmul / gather_rows on world_size-2 gloo ranks (the local GEMM is a CPU stand-in; on the GPU
it is gtx16_fp16.mm_t)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gtx16_fp16.dist import ShardedMatmul, batch_slice, gather_rows, shard_bounds


@pytest.mark.parametrize("n,world", [(16384, 1), (16384, 2), (16384, 8), (1032, 3), (8, 2), (4104, 8), (776, 5)])
def test_shard_bounds_cover_exactly(n, world):
    spans = [shard_bounds(n, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0
    for a, b in spans:
        assert a % 8 == 0 and b % 8 == 0 and b >= a
    widths = [b - a for a, b in spans]
    assert max(widths) - min(widths) <= 8


def test_shard_bounds_rejects_bad_input():
    with pytest.raises(ValueError):
        shard_bounds(12, 2, 0)
    with pytest.raises(ValueError):
        shard_bounds(16, 2, 2)


@pytest.mark.parametrize("batch,world", [(256, 1), (256, 8), (10, 3), (2, 4)])
def test_batch_slice_partitions(batch, world):
    got = []
    for r in range(world):
        s = batch_slice(batch, world, r)
        got.extend(range(batch)[s])
    assert got == list(range(batch))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_total, ret):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        M, K = 24, 40
        a = torch.randn(M, K, generator=g)
        w = torch.randn(K, n_total, generator=g)
        n0, n1 = shard_bounds(n_total, world, rank)
        sm = ShardedMatmul(w[:, n0:n1].contiguous(), n_total, out_dtype=torch.float32,
                           local_mm=lambda x, ws: x @ ws)
        y = sm(a)
        ok = torch.allclose(y, a @ w, rtol=1e-5, atol=1e-5)
        rows = gather_rows(a[batch_slice(M, world, rank)] * 2, M)
        ok = ok and torch.equal(rows, a * 2)
        ret[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_total", [64, 72])  # equal shards / unequal shards
def test_sharded_matmul_gloo_world2(n_total):
    world = 2
    ret = mp.Manager().dict()
    mp.spawn(_worker, args=(world, _free_port(), n_total, ret), nprocs=world, join=True)
    assert dict(ret) == {0: True, 1: True}


class _FakeMulticast:
    """Stands in for dist.MulticastBuffer on gloo ranks: construction fails on the ranks listed in
    `fail`, otherwise it yields a buffer with a multicast address; close() is collective."""
    fail = ()
    closed = 0

    def __init__(self, shape, dtype, device, group=None):
        if dist.get_rank() in self.fail:
            raise RuntimeError("multicast object could not be created")
        self.mc_ptr = 1
        self.group = group

    @staticmethod
    def supported(device):
        return True

    def close(self):
        type(self).closed += 1
        dist.barrier(group=self.group)


class _FakePeer:
    def __init__(self, shape, dtype, device, group=None):
        self.shape = shape


def _exchange_worker(rank, world, port, fail, multicast, ret):
    import gtx16_fp16.dist as gdist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _FakeMulticast.fail = fail
        gdist.MulticastBuffer, gdist.PeerBuffer = _FakeMulticast, _FakePeer
        sm = ShardedMatmul(torch.zeros(8, 16), 16 * world, out_dtype=torch.float32,
                           local_mm=lambda x, ws: x @ ws, multicast=multicast)
        try:
            buf = sm._exchange_buffer(24, torch.device("cpu"))
            kind = type(buf).__name__
        except RuntimeError:
            kind = "raised"
        dist.barrier()  # every rank left the agreement with the same collectives
        ret[rank] = (kind, _FakeMulticast.closed)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fail,multicast,want", [
    ((), None, {0: ("_FakeMulticast", 0), 1: ("_FakeMulticast", 0)}),
    ((0,), None, {0: ("_FakePeer", 0), 1: ("_FakePeer", 1)}),
    ((1,), False, {0: ("_FakePeer", 0), 1: ("_FakePeer", 0)}),
    ((0,), True, {0: ("raised", 0), 1: ("raised", 1)}),
])
def test_exchange_buffer_ranks_agree_gloo_world2(fail, multicast, want):
    """The fused path's buffer choice: one rank's failed multicast set-up sends every rank to peer
    stores (the rank that built one releases it), multicast=False never tries, multicast=True
    raises on every rank."""
    world = 2
    ret = mp.Manager().dict()
    mp.spawn(_exchange_worker, args=(world, _free_port(), fail, multicast, ret), nprocs=world, join=True)
    assert dict(ret) == want
