"""Multi-GPU use of the hot path (one process per GPU, torch.distributed over NCCL / NVLink).

The reference is single-GPU. Two ways of using several GPUs of one box are provided, both for
shapes that shard naturally:

* ``ShardedMatmul``: out[M, N] = a[M, K] @ w_t[K, N] with w_t split by columns. Rank r keeps its
  column shard w_t[:, n_r0:n_r1] resident, computes out[:, n_r0:n_r1] with ``mm_t`` and the shards
  are exchanged with one NCCL all-gather (the only collective on the path). Every rank ends with
  the full output. Shard boundaries are multiples of 8 columns (the kernels' N % 8 rule).
* ``batch_slice``: data parallelism over a batch of independent inputs (model inference): rank r
  takes a contiguous slice; there is no collective on the data path, only an optional gather of
  the (small) results.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


def shard_bounds(n: int, world: int, rank: int, align: int = 8) -> tuple[int, int]:
    """[n0, n1) of rank `rank` when n columns are split over `world` ranks in blocks of `align`.

    Units of `align` columns are dealt as evenly as possible, the first ranks taking one more."""
    if n % align != 0:
        raise ValueError(f"n={n} is not a multiple of {align}")
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    units = n // align
    base, extra = divmod(units, world)
    u0 = rank * base + min(rank, extra)
    u1 = u0 + base + (1 if rank < extra else 0)
    return u0 * align, u1 * align


def batch_slice(batch: int, world: int, rank: int) -> slice:
    """Contiguous slice of a batch of `batch` items taken by `rank` (first ranks take one more)."""
    base, extra = divmod(batch, world)
    b0 = rank * base + min(rank, extra)
    return slice(b0, b0 + base + (1 if rank < extra else 0))


@dataclass
class ShardedMatmul:
    """Column-sharded matmul with an all-gather of the output shards.

    w_shard: this rank's [K, n1 - n0] fp16 columns of w_t (resident), from ``shard_bounds``.
    n_total: N of the full w_t. group: process group (None = default). The output of ``__call__``
    is the full [M, N] tensor on every rank; ``local`` returns only this rank's shard.
    ``local_mm`` computes one shard (default ``gtx16_fp16.mm_t``); tests pass a CPU stand-in to
    exercise the exchange logic on gloo ranks.
    """

    w_shard: torch.Tensor
    n_total: int
    group: object = None
    out_dtype: torch.dtype = torch.float16
    local_mm: object = None

    def __post_init__(self):
        self.world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(self.group) if dist.is_initialized() else 0
        n0, n1 = shard_bounds(self.n_total, self.world, self.rank)
        if self.w_shard.shape[1] != n1 - n0:
            raise ValueError(f"rank {self.rank}: w_shard has {self.w_shard.shape[1]} columns, expected {n1 - n0}")
        self.n0, self.n1 = n0, n1
        self.widths = [b - a for a, b in (shard_bounds(self.n_total, self.world, r) for r in range(self.world))]
        if self.local_mm is None:
            from .ops import mm_t
            self.local_mm = lambda a, w: mm_t(a, w, None, self.out_dtype)

    def local(self, a: torch.Tensor) -> torch.Tensor:
        return self.local_mm(a, self.w_shard)

    def __call__(self, a: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        c_local = self.local(a).contiguous()
        M = a.shape[0]
        if self.world == 1:
            if out is not None:
                out.copy_(c_local)
                return out
            return c_local
        if out is None:
            out = torch.empty(M, self.n_total, dtype=c_local.dtype, device=c_local.device)
        if len(set(self.widths)) == 1:
            # equal shards: one all_gather_into_tensor into [P, M, N/P], then interleave the columns
            buf = torch.empty(self.world * M * self.widths[0], dtype=c_local.dtype, device=c_local.device)
            dist.all_gather_into_tensor(buf, c_local.reshape(-1), group=self.group)
            out.copy_(buf.view(self.world, M, self.widths[0]).permute(1, 0, 2).reshape(M, self.n_total))
        else:
            # unequal shards (N not a multiple of 8 * world): pad every shard to the widest one
            wmax = max(self.widths)
            padded = torch.zeros(M, wmax, dtype=c_local.dtype, device=c_local.device)
            padded[:, : c_local.shape[1]] = c_local
            buf = torch.empty(self.world * M * wmax, dtype=c_local.dtype, device=c_local.device)
            dist.all_gather_into_tensor(buf, padded.reshape(-1), group=self.group)
            buf = buf.view(self.world, M, wmax)
            torch.cat([buf[r, :, : self.widths[r]] for r in range(self.world)], dim=1, out=out)
        return out


def gather_rows(local: torch.Tensor, batch: int, group=None) -> torch.Tensor:
    """All-gather per-rank row blocks produced from ``batch_slice`` back into [batch, ...] (every rank)."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return local
    sizes = [batch_slice(batch, world, r).stop - batch_slice(batch, world, r).start for r in range(world)]
    smax = max(sizes)
    padded = torch.zeros((smax,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    padded[: local.shape[0]] = local
    buf = torch.empty((world * smax,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(buf, padded.contiguous(), group=group)
    return torch.cat([buf[r * smax: r * smax + sizes[r]] for r in range(world)], dim=0)
