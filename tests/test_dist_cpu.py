"""Host-side logic of the multi-GPU path on CPU: shard arithmetic, and the exchange of
ShardedMatmul / gather_rows on world_size-2 gloo ranks (the local GEMM is a CPU stand-in; on the GPU
it is gtx16_fp16.mm_t)."""
import os
import socket
import time

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
    ret = mp.get_context("spawn").Manager().dict()
    mp.spawn(_worker, args=(world, _free_port(), n_total, ret), nprocs=world, join=True)
    assert dict(ret) == {0: True, 1: True}


class _FakeMulticast:
    """Stands in for dist.MulticastBuffer on gloo ranks. Ranks in `unsupported` report no multicast
    support; allocation (local) fails on the ranks in `fail`; the rendezvous (collective, like the
    real one) yields no multicast address on the ranks in `no_mc`. close() is collective, release()
    local; both are counted."""
    unsupported = ()
    fail = ()
    no_mc = ()
    closed = 0
    released = 0

    def __init__(self, shape, dtype, device, group=None):
        if dist.get_rank() in self.fail:
            raise RuntimeError("symmetric memory could not be allocated")
        self.mc_ptr = 0
        self.group = group

    def rendezvous(self):
        dist.barrier(group=self.group)
        self.mc_ptr = 0 if dist.get_rank() in self.no_mc else 1

    @staticmethod
    def supported(device):
        return dist.get_rank() not in _FakeMulticast.unsupported

    def release(self):
        type(self).released += 1

    def close(self):
        type(self).closed += 1
        dist.barrier(group=self.group)


class _FakePeer:
    def __init__(self, shape, dtype, device, group=None):
        self.shape = shape


def _exchange_worker(rank, world, port, case, multicast, ret):
    import gtx16_fp16.dist as gdist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        for k, v in case.items():
            setattr(_FakeMulticast, k, v)
        gdist.MulticastBuffer, gdist.PeerBuffer = _FakeMulticast, _FakePeer
        sm = ShardedMatmul(torch.zeros(8, 16), 16 * world, out_dtype=torch.float32,
                           local_mm=lambda x, ws: x @ ws, multicast=multicast)
        try:
            buf = sm._exchange_buffer(24, torch.device("cpu"))
            kind = type(buf).__name__
        except RuntimeError:
            kind = "raised"
        dist.barrier()  # every rank left the agreement with the same collectives
        ret[rank] = (kind, _FakeMulticast.closed, _FakeMulticast.released)
    finally:
        dist.destroy_process_group()


MC, PEER = "_FakeMulticast", "_FakePeer"


# Each rank builds two multicast buffers (output slots and completion counter), so a failed set-up
# closes or releases two per rank.
@pytest.mark.parametrize("case,multicast,want", [
    ({}, None, {0: (MC, 0, 0), 1: (MC, 0, 0)}),
    # one rank without multicast support: nobody allocates, nobody enters the rendezvous
    ({"unsupported": (1,)}, None, {0: (PEER, 0, 0), 1: (PEER, 0, 0)}),
    # one rank's first allocation fails: the other releases both its buffers locally, no rendezvous
    ({"fail": (0,)}, None, {0: (PEER, 0, 0), 1: (PEER, 0, 2)}),
    # the rendezvous gives one rank no multicast address: both close both buffers (collectively)
    ({"no_mc": (1,)}, None, {0: (PEER, 2, 0), 1: (PEER, 2, 0)}),
    ({"fail": (1,)}, False, {0: (PEER, 0, 0), 1: (PEER, 0, 0)}),
    ({"fail": (0,)}, True, {0: ("raised", 0, 0), 1: ("raised", 0, 2)}),
    ({"unsupported": (0,)}, True, {0: ("raised", 0, 0), 1: ("raised", 0, 0)}),
])
def test_exchange_buffer_ranks_agree_gloo_world2(case, multicast, want):
    """The fused path's buffer choice: whatever one rank finds (no multicast support, a failed
    allocation, no multicast address) sends every rank to peer stores with the same collectives;
    multicast=False never tries, multicast=True raises on every rank."""
    world = 2
    ret = mp.get_context("spawn").Manager().dict()
    mp.spawn(_exchange_worker, args=(world, _free_port(), case, multicast, ret), nprocs=world, join=True)
    assert dict(ret) == want


def _leaving_worker(rank, world, port, ret):
    """Rank 1 takes part in one step of ShardedMatmul and leaves between steps (its process ends,
    no collective in flight); rank 0 starts the next step and must get an error on the host within
    the process group's timeout instead of waiting for good."""
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    g = torch.Generator().manual_seed(0)
    a = torch.randn(16, 24, generator=g)
    w = torch.randn(24, 32, generator=g)
    n0, n1 = shard_bounds(32, world, rank)
    sm = ShardedMatmul(w[:, n0:n1].contiguous(), 32, out_dtype=torch.float32, local_mm=lambda x, ws: x @ ws)
    ok = torch.allclose(sm(a), a @ w, rtol=1e-5, atol=1e-5)  # step 1: both ranks
    dist.barrier()
    if rank == 1:
        ret[rank] = ("left", bool(ok), 0.0)
        os._exit(0)  # leaves between steps, without any goodbye to its peer
    time.sleep(0.5)
    t0 = time.perf_counter()
    try:
        sm(a)  # step 2: the peer is gone
        ret[rank] = ("no error", bool(ok), time.perf_counter() - t0)
    except RuntimeError:
        ret[rank] = ("error", bool(ok), time.perf_counter() - t0)
    os._exit(0)  # the process group cannot be torn down cleanly without the peer


def test_rank_leaving_between_steps_is_detected_gloo_world2():
    world = 2
    ret = mp.get_context("spawn").Manager().dict()
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, world, port, ret)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert ret[1][:2] == ("left", True)
    kind, step1_ok, dt = ret[0]
    assert step1_ok and kind == "error"
    assert dt < 30.0  # within the 5 s process-group timeout plus slack, not an endless wait
