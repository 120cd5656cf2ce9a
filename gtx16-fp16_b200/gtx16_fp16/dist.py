"""Multi-GPU use of the hot path (one process per GPU, torch.distributed over NCCL / NVLink).

The reference is single-GPU. Two ways of using several GPUs of one box are provided, both for
shapes that shard naturally:

* ``ShardedMatmul``: out[M, N] = a[M, K] @ w_t[K, N] with w_t split by columns. Rank r keeps its
  column shard w_t[:, n_r0:n_r1] resident and computes out[:, n_r0:n_r1]. On CUDA with NCCL and
  fp16 activations the exchange is fused into the GEMM: where the GPUs support NVLink multicast
  (NVLS) the epilogue writes every output tile once through a multicast address bound to all
  ranks' output buffers (``MulticastBuffer``: torch symmetric memory) and the switch delivers it
  everywhere; the kernel's CTAs then signal a multicast counter and a bounded wait on this GPU's
  copy of it ends the call (g16_gemm_allgather_mc), so a call makes no host collective at all. Two
  output slots alternate: a peer writes the slot of call i + 1 only after this rank's kernel of
  call i has finished, i.e. after this rank's stream has passed everything it enqueued before
  call i, including its reads of the result of call i - 1 (the same slot).
  Without multicast the epilogue stores every tile into each rank's full output buffer
  (``PeerBuffer``: CUDA IPC mappings over NVLink) and two one-element all-reduces per call order
  the buffer's reuse. Either way the all-gather overlaps the math and no separate copy pass is
  needed. Otherwise (fp32 activations, M <= 8, gloo) the shards are computed with ``mm_t`` and
  exchanged with one NCCL all-gather. Every rank ends with the full output. Shard boundaries are
  multiples of 8 columns (the kernels' N % 8 rule).
* ``batch_slice``: data parallelism over a batch of independent inputs (model inference): rank r
  takes a contiguous slice; there is no collective on the data path, only an optional gather of
  the (small) results.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

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


class _CudaArray:
    """A raw device allocation described by __cuda_array_interface__ (wrapped by torch.as_tensor)."""

    def __init__(self, ptr: int, shape: tuple, dtype: torch.dtype):
        typestr = {torch.float16: "<f2", torch.float32: "<f4"}[dtype]
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerBuffer:
    """A [rows, cols] buffer on every rank of `group`, mapped into every other rank with CUDA IPC.

    ``tensor`` is this rank's buffer; ``ptrs[r]`` is rank r's buffer as this process addresses it
    (its own for r == rank). Collective: every rank constructs it with the same shape and dtype,
    and every rank calls ``close()`` (peers unmap before owners free). The tensor must not be
    used after ``close()``."""

    def __init__(self, shape: tuple, dtype: torch.dtype, device: torch.device, group=None):
        from . import _native
        L = _native.lib()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.shape, self.dtype = tuple(shape), dtype
        nbytes = torch.tensor([], dtype=dtype).element_size()
        for d in self.shape:
            nbytes *= d
        with torch.cuda.device(device):
            own = ctypes.c_void_p()
            _native.check(L.g16_ipc_alloc(max(nbytes, 256), ctypes.byref(own)), "g16_ipc_alloc")
            self._own = own.value
            handle = ctypes.create_string_buffer(_native.IPC_HANDLE_BYTES)
            _native.check(L.g16_ipc_get_handle(own, handle), "g16_ipc_get_handle")
            handles = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=group)
            self.ptrs, self._opened = [], []
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.ptrs.append(self._own)
                    continue
                p = ctypes.c_void_p()
                _native.check(L.g16_ipc_open(ctypes.create_string_buffer(h, len(h)), ctypes.byref(p)),
                              "g16_ipc_open")
                self.ptrs.append(p.value)
                self._opened.append(p.value)
            self.tensor = torch.as_tensor(_CudaArray(self._own, self.shape, dtype), device=device)

    def close(self):
        from . import _native
        if self._own is None:
            return
        L = _native.lib()
        torch.cuda.synchronize()
        for p in self._opened:
            _native.check(L.g16_ipc_close(ctypes.c_void_p(p)), "g16_ipc_close")
        self._opened = []
        dist.barrier(group=self.group)  # every peer has unmapped this rank's buffer
        _native.check(L.g16_ipc_free(ctypes.c_void_p(self._own)), "g16_ipc_free")
        self._own = None
        self.tensor = None


class MulticastBuffer:
    """A [rows, cols] buffer on every rank of `group` in torch symmetric memory, with the NVLink
    multicast address (``mc_ptr``) that writes all ranks' copies at once.

    Set-up has two steps so that callers can agree between them: construction allocates this
    rank's copy and is local (no collective); ``rendezvous()`` is collective and sets ``mc_ptr``
    (0 when the group has no multicast object). After a rendezvous ``close()`` is collective; a
    buffer that never took part in one is dropped with the local ``release()``."""

    def __init__(self, shape: tuple, dtype: torch.dtype, device: torch.device, group=None):
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group if group is not None else dist.group.WORLD
        self.shape, self.dtype = tuple(shape), dtype
        self.tensor = symm_mem.empty(*self.shape, dtype=dtype, device=device)
        self._handle = None
        self.mc_ptr = 0

    def rendezvous(self):
        import torch.distributed._symmetric_memory as symm_mem
        self._handle = symm_mem.rendezvous(self.tensor, self.group)
        self.mc_ptr = int(self._handle.multicast_ptr) if self._handle.multicast_ptr else 0

    @staticmethod
    def supported(device: torch.device) -> bool:
        """Whether this GPU can use NVLink multicast through torch symmetric memory."""
        if device.type != "cuda":
            return False
        try:
            import torch.distributed._symmetric_memory as symm_mem
            return bool(symm_mem._SymmetricMemory.has_multicast_support(symm_mem.DeviceType.CUDA,
                                                                        device.index or 0))
        except (ImportError, AttributeError, RuntimeError):
            return False

    def release(self):
        self._handle = None
        self.tensor = None

    def close(self):
        if self.tensor is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)  # no peer writes into this buffer any more
        self.release()


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
    fused: bool | None = None  # None: the fused exchange whenever it applies (see the module doc)
    scatter_flags: int = 0     # G16_SCATTER_* store method of the fused path (0: the library's default)
    multicast: bool | None = None  # NVLink multicast exchange: None = where supported, False = never
    _bufs: dict = field(default_factory=dict, repr=False)

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

    def fused_applies(self, a: torch.Tensor) -> bool:
        """The fused GEMM + exchange runs for fp16 CUDA activations with M > 8 over NCCL."""
        if self.fused is False or self.world == 1 or not a.is_cuda:
            return False
        ok = (a.dtype == torch.float16 and a.dim() == 2 and a.shape[0] > 8 and self.w_shard.is_cuda
              and self.w_shard.dtype == torch.float16 and self.out_dtype in (torch.float16, torch.float32)
              and self.world <= 8 and dist.get_backend(self.group) == "nccl")
        if self.fused and not ok:
            raise ValueError("ShardedMatmul(fused=True) needs fp16 CUDA activations with M > 8 over NCCL "
                             "(at most 8 ranks)")
        return ok

    def _fused_call(self, a: torch.Tensor, out: torch.Tensor | None) -> torch.Tensor:
        from . import _native
        a = a.contiguous()
        M, K = a.shape
        buf = self._bufs.get(M)
        if buf is None:
            buf = self._exchange_buffer(M, a.device)
            self._bufs[M] = buf
            if isinstance(buf, MulticastBuffer):
                self._init_signals(buf, M, K, a.device)
            else:
                self._flag = torch.zeros(1, dtype=torch.int32, device=a.device)
        if isinstance(buf, MulticastBuffer):
            return self._multicast_call(buf, a, out)
        # Peers are done with their outputs of the previous call before any tile lands there.
        dist.all_reduce(self._flag, group=self.group)
        ptrs = (ctypes.c_void_p * self.world)(*buf.ptrs)
        st = _native.lib().g16_gemm_scatter(
            a.data_ptr(), self.w_shard.data_ptr(), ptrs, self.world, _native.dtype_code(self.out_dtype), None,
            None, M, K, self.n1 - self.n0, self.n_total, self.n0, self.scatter_flags,
            _native.stream_handle(a.device.index or 0))
        _native.check(st, "g16_gemm_scatter")
        # Every peer's kernel (and so every tile it stored here) has completed.
        dist.all_reduce(self._flag, group=self.group)
        if out is not None:
            out.copy_(buf.tensor)
            return out
        return buf.tensor

    # Longest a rank's stream waits for its peers' tiles before the library records a timeout.
    SIGNAL_WAIT_US = 30_000_000

    def _init_signals(self, buf: MulticastBuffer, M: int, K: int, device: torch.device):
        """Set-up of the multicast path (collective): zero every GPU's counter before any rank can
        signal, and agree on the counter increments per call (the CTAs of all ranks)."""
        from . import _native
        n = _native.lib().g16_gemm_allgather_signals(M, K, self.n1 - self.n0)
        if n < 0:
            raise _native.G16Error(-n, "g16_gemm_allgather_signals")
        total = torch.tensor([n], dtype=torch.int64, device=device)
        dist.all_reduce(total, group=self.group)
        buf.flag.tensor.zero_()
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)  # every counter is zero before the first signal
        buf.signals = int(total.item())
        buf.target = 0
        buf.calls = 0

    def _multicast_call(self, buf: MulticastBuffer, a: torch.Tensor, out: torch.Tensor | None) -> torch.Tensor:
        from . import _native
        M, K = a.shape
        slot = buf.calls % 2
        buf.calls += 1
        buf.target = (buf.target + buf.signals) & 0xFFFFFFFF
        esz = torch.tensor([], dtype=self.out_dtype).element_size()
        st = _native.lib().g16_gemm_allgather_mc(
            a.data_ptr(), self.w_shard.data_ptr(), buf.mc_ptr + slot * M * self.n_total * esz,
            _native.dtype_code(self.out_dtype), None, None, M, K, self.n1 - self.n0, self.n_total, self.n0,
            buf.flag.mc_ptr, buf.flag.tensor.data_ptr(), buf.target, self.SIGNAL_WAIT_US,
            _native.stream_handle(a.device.index or 0))
        _native.check(st, "g16_gemm_allgather_mc")
        res = buf.tensor[slot * M:(slot + 1) * M]
        if out is not None:
            out.copy_(res)
            return out
        return res

    def _exchange_buffer(self, M: int, device: torch.device):
        """The output buffer of the fused path for M rows (collective). A MulticastBuffer where every
        rank can build one with a multicast address, else a PeerBuffer.

        Every step whose outcome can differ between ranks ends in a MIN all-reduce of a success flag,
        so all ranks take the same collectives and the same buffer: (1) multicast support, a local
        query; (2) this rank's allocation, local; (3) the rendezvous, a collective, and its multicast
        address. A rank whose support or allocation failed therefore never leaves its peers waiting
        inside the rendezvous. (The rendezvous itself cannot be guarded this way: a rank that raises
        inside it raises on its own.)"""
        def agree(ok: bool) -> bool:
            t = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MIN, group=self.group)
            return bool(t.item())

        if self.multicast is not False and agree(MulticastBuffer.supported(device)):
            # two output slots, used alternately, and the completion counter (multicast too)
            bufs = []
            try:
                bufs.append(MulticastBuffer((2 * M, self.n_total), self.out_dtype, device, self.group))
                bufs.append(MulticastBuffer((1, 64), torch.int32, device, self.group))
            except RuntimeError:
                pass
            if agree(len(bufs) == 2):
                for b in bufs:
                    b.rendezvous()
                if agree(all(b.mc_ptr != 0 for b in bufs)):
                    bufs[0].flag = bufs[1]
                    return bufs[0]
                for b in bufs:
                    b.close()
            else:
                for b in bufs:
                    b.release()
        if self.multicast:
            raise RuntimeError("ShardedMatmul(multicast=True): no NVLink multicast on this group")
        return PeerBuffer((M, self.n_total), self.out_dtype, device, self.group)

    def close(self):
        """Release the fused path's buffers (collective: every rank calls it)."""
        for buf in self._bufs.values():
            flag = getattr(buf, "flag", None)
            buf.close()
            if flag is not None:
                flag.close()
        self._bufs.clear()

    def __call__(self, a: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """The full [M, N] output on every rank. On the fused path the returned tensor is one of
        this instance's output buffers for M rows: it stays valid until this rank's next call with
        the same M (or ``close()``), and must be read on the calling stream (make every call of an
        instance on one stream); pass ``out`` to keep a copy."""
        if self.fused_applies(a):
            return self._fused_call(a, out)
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
