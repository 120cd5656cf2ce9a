"""Column-sharded matmul across 2 GPUs (skipped with fewer than 2 GPUs).

Fused path (fp16 activations, M > 8, NCCL): every rank's GEMM epilogue writes its output tiles into
both ranks' full output buffers, once through an NVLink multicast address (torch symmetric memory)
where the GPUs support it, and with stores into each peer's CUDA IPC mapping otherwise (both paths
are run). On the multicast path the kernel's CTAs signal completion through a multicast counter
and two output slots alternate (no host collective per call): ten calls in a row are exact and no
completion wait times out. The result equals, bit for bit, the same column shards computed on one GPU with g16_gemm
and ksplit = 1 (same kernel, same K order), and the fp64 product within the GEMM tolerance; two
calls in a row check the ordering of buffer reuse.
Gather path (fused=False): mm_t per shard and one NCCL all-gather; equals the single-GPU shards.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard_gemm_ksplit1(a, w_shard, out_dtype):
    from gtx16_fp16 import _native
    L = _native.lib()
    M, K = a.shape
    n = w_shard.shape[1]
    out = torch.empty(M, n, dtype=out_dtype, device=a.device)
    st = L.g16_gemm(a.data_ptr(), w_shard.data_ptr(), out.data_ptr(), _native.dtype_code(out_dtype), None, None,
                    M, K, n, 1, None, 0, _native.stream_handle(a.device.index or 0))
    _native.check(st, "g16_gemm")
    return out


def _worker(rank, world, port, ret):
    import datetime

    import torch.distributed as dist

    import gtx16_fp16 as g
    from gtx16_fp16 import _native
    from gtx16_fp16.dist import MulticastBuffer, ShardedMatmul, batch_slice, gather_rows, shard_bounds

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    results = {}
    ShardedMatmul.SIGNAL_WAIT_US = 2_000_000  # a wrong counter target fails fast here
    try:
        for mc in (None, False):  # None: NVLink multicast where supported; False: peer stores
            for M, K, N, out_dtype in ((1024, 2048, 4096, torch.float16), (1000, 1024, 4104, torch.float32)):
                gen = torch.Generator(device="cuda").manual_seed(M + N)
                w = (torch.randn(K, N, device="cuda", generator=gen) * K ** -0.5).half()
                n0, n1 = shard_bounds(N, world, rank)
                fused = ShardedMatmul(w[:, n0:n1].contiguous(), N, out_dtype=out_dtype, multicast=mc)
                tag = f"{'peer' if mc is False else 'auto'} {M}x{K}x{N} {out_dtype}"
                for call in range(2):
                    a = torch.randn(M, K, device="cuda", generator=gen).half()
                    assert fused.fused_applies(a)
                    y = fused(a).clone()
                    shards = [_shard_gemm_ksplit1(a, w[:, b0:b1].contiguous(), out_dtype)
                              for b0, b1 in (shard_bounds(N, world, r) for r in range(world))]
                    ref = a.double() @ w.double()
                    results[f"fused {tag} call {call} bitwise"] = torch.equal(y, torch.cat(shards, dim=1))
                    results[f"fused {tag} call {call} fp64"] = ((y.double() - ref).norm() / ref.norm()).item() < 1e-3
                if mc is False:
                    results[f"fused {tag} took the peer path"] = not isinstance(fused._bufs[M], MulticastBuffer)
                else:
                    is_mc = isinstance(fused._bufs[M], MulticastBuffer)
                    ret[f"multicast {rank}"] = is_mc
                    if is_mc:
                        # ten calls in a row through the counter-based completion wait, each result
                        # compared (on the calling stream) before the next call, as documented
                        ok = True
                        for _ in range(10):
                            a_next = torch.randn(M, K, device="cuda", generator=gen).half()
                            y_next = fused(a_next)
                            want = torch.cat([_shard_gemm_ksplit1(a_next, w[:, b0:b1].contiguous(), out_dtype)
                                              for b0, b1 in (shard_bounds(N, world, r) for r in range(world))], 1)
                            ok = ok and torch.equal(y_next, want)
                        results[f"fused {tag} multicast signals"] = ok
                        results[f"fused {tag} no wait timed out"] = _native.device_status(clear=True) == _native.OK
                fused.close()
        # gather path (mm_t per shard + NCCL all-gather)
        gen = torch.Generator(device="cuda").manual_seed(0)
        M, K, N = 1024, 2048, 4096
        a = torch.randn(M, K, device="cuda", generator=gen).half()
        w = (torch.randn(K, N, device="cuda", generator=gen) * K ** -0.5).half()
        n0, n1 = shard_bounds(N, world, rank)
        y = ShardedMatmul(w[:, n0:n1].contiguous(), N, fused=False)(a)
        shards = [g.mm_t(a, w[:, b0:b1].contiguous(), None, torch.float16)
                  for b0, b1 in (shard_bounds(N, world, r) for r in range(world))]
        results["gather bitwise"] = torch.equal(y, torch.cat(shards, dim=1))
        full = g.mm_t(a, w, None, torch.float16)
        rows = gather_rows(full[batch_slice(M, world, rank)], M)
        results["gather_rows"] = torch.equal(rows, full)
        torch.cuda.synchronize()
        ret[rank] = results
    finally:
        dist.destroy_process_group()


def test_sharded_matmul_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ret = mp.get_context("spawn").Manager().dict()
    mp.spawn(_worker, args=(2, _free_port(), ret), nprocs=2, join=True)
    got = {k: v for k, v in dict(ret).items() if isinstance(k, int)}
    print("multicast path used:", {k: v for k, v in dict(ret).items() if not isinstance(k, int)})
    assert sorted(got) == [0, 1]
    for rank, res in got.items():
        bad = [k for k, v in res.items() if not v]
        assert not bad, f"rank {rank}: {bad}"
