"""KV-head sharding of the retrieval path across the GPUs of one node.

The reference is single-GPU.  KV heads are independent through scoring,
selection and attention (GQA groups never cross KV heads), so rank r of N owns
KV heads [r*KVH/N, (r+1)*KVH/N) -- their K/V cache and bit-plane metadata --
and the query heads that read them, [r*QH/N, (r+1)*QH/N).  Each rank runs the
whole decode step on its heads; one all-gather of the per-head attention
outputs per layer gives every rank the full [B, QH, D] input of the replicated
output projection.  The all-gather is the only collective on the path.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    kv_start: int
    kv_end: int
    q_start: int
    q_end: int

    @property
    def kv_slice(self) -> slice:
        return slice(self.kv_start, self.kv_end)

    @property
    def q_slice(self) -> slice:
        return slice(self.q_start, self.q_end)

    @property
    def kv_heads(self) -> int:
        return self.kv_end - self.kv_start

    @property
    def q_heads(self) -> int:
        return self.q_end - self.q_start

    def local_head_to_kv(self, device=None) -> torch.Tensor:
        group = self.q_heads // self.kv_heads
        return torch.arange(self.q_heads, device=device, dtype=torch.int64) // group


def head_shard(q_heads: int, kv_heads: int, world: int, rank: int) -> HeadShard:
    """The heads rank ``rank`` of ``world`` owns."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if kv_heads % world:
        raise ValueError(f"{kv_heads} KV heads cannot be split evenly over {world} ranks")
    if q_heads % kv_heads:
        raise ValueError("query heads must be a multiple of KV heads")
    kv_local = kv_heads // world
    q_local = q_heads // world
    return HeadShard(rank, world, rank * kv_local, (rank + 1) * kv_local,
                     rank * q_local, (rank + 1) * q_local)


def gather_heads(local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather per-rank head outputs [B, QH/N, D] into [B, QH, D] (rank order).

    One ``all_gather_into_tensor`` (NCCL over NVLink on GPUs, gloo on CPU).
    """
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if world == 1:
        return local
    batch, q_local, dim = (int(x) for x in local.shape)
    flat = torch.empty((world * batch * q_local * dim,), device=local.device, dtype=local.dtype)
    dist.all_gather_into_tensor(flat, local.contiguous().view(-1), group=group)
    return flat.view(world, batch, q_local, dim).permute(1, 0, 2, 3).reshape(batch, world * q_local, dim)


class _PeerArea:
    """This rank's receive area in device memory, mapped by every peer of ``group``.

    Collective: each rank allocates ``nbytes`` (popkv_peer_alloc, zeroed), the
    64-byte CUDA IPC handles are exchanged with ``all_gather_object`` (any
    backend), and each rank maps its peers' areas.  ``ptrs`` holds every rank's
    area base in rank order (a device int64 array), ``own`` this rank's.
    """

    def __init__(self, nbytes: int, device, group=None) -> None:
        import ctypes

        import torch.distributed as dist

        from . import _lib
        self._lib = _lib
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        lib = _lib.lib()
        self.nbytes = int(nbytes)
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        with torch.cuda.device(self.device):
            _lib.check(lib.popkv_peer_alloc(int(nbytes), ctypes.byref(ptr), handle))
        self.own = ptr
        self._opened: list = []
        handles: list = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        bases = []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    bases.append(ptr.value)
                    continue
                p = ctypes.c_void_p()
                _lib.check(lib.popkv_peer_open(h, ctypes.byref(p)))
                self._opened.append(p)
                bases.append(p.value)
        self.ptrs = torch.tensor(bases, dtype=torch.int64, device=self.device)
        # Launch epoch, CTAs done in the launch, wait-gave-up flag, poll limit
        # override (0: the kernels' default of about a second).
        self.state = torch.zeros(4, dtype=torch.int32, device=self.device)

    def error(self) -> bool:
        return bool(int(self.state[2].item()))

    def reset(self) -> None:
        """Zero this rank's area and launch state, in step with every peer (collective).

        After a wait gave up (``error()``), the ranks' launch epochs may differ
        and every later exchange would time out; all ranks call ``reset`` with
        no launch in flight to start again from epoch 0.
        """
        import torch.distributed as dist
        import ctypes
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # no peer still writes into this area
        with torch.cuda.device(self.device):
            self._lib.check(self._lib.lib().popkv_peer_clear(
                ctypes.c_void_p(self.own.value), self.nbytes, self._lib.stream_of(self.device)))
            self.state[:3].zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # every area is clean before any rank launches again

    def close(self) -> None:
        """Unmap the peers and free this rank's area (collective: all ranks call it)."""
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        lib = self._lib.lib()
        with torch.cuda.device(self.device):
            for p in self._opened:
                self._lib.check(lib.popkv_peer_close(p))
            self._opened = []
            if self.own is not None:
                self._lib.check(lib.popkv_peer_free(self.own))
                self.own = None


class PeerGather:
    """Merge fused with the all-gather over NVLink peer memory (popkv_attn_merge_gather).

    Every rank of ``group`` constructs one, collectively (a ``_PeerArea`` of
    2 x world x rows x 128 (value, epoch) words).  ``launch`` then merges this
    rank's ``rows`` split states and leaves all ranks' merged rows in
    ``output`` [world * rows, 128], rank-major.  Every rank must launch the
    same sequence of steps; ``error()`` reports a wait for a peer that gave up.
    """

    HEAD_DIM = 128

    def __init__(self, rows: int, dtype: torch.dtype, device, group=None) -> None:
        from . import _lib
        self._lib = _lib
        self.rows = int(rows)
        self.dtype = dtype
        self.device = torch.device(device)
        import torch.distributed as dist
        world = dist.get_world_size(group)
        self.area = _PeerArea(2 * world * self.rows * self.HEAD_DIM * 8, self.device, group)
        self.world, self.rank = self.area.world, self.area.rank
        self.state = self.area.state
        self.output = torch.empty((self.world * self.rows, self.HEAD_DIM), dtype=dtype, device=self.device)

    def launch(self, partials: torch.Tensor, splits: int, stream) -> None:
        """Merge ``partials`` [rows, splits, 130] and gather into ``output`` on ``stream``."""
        import ctypes
        lib, _lib = self._lib.lib(), self._lib
        self._lib.check(lib.popkv_attn_merge_gather(
            _lib.ptr(partials), self.rows, int(splits), self.HEAD_DIM, _lib.dtype_code(self.output),
            self.rank, self.world, _lib.ptr(self.area.ptrs), ctypes.c_void_p(self.area.own.value),
            _lib.ptr(self.state), _lib.ptr(self.output), stream))

    def error(self) -> bool:
        return self.area.error()

    def reset(self) -> None:
        """Clear the area and launch state on every rank together (collective), after ``error()``."""
        self.area.reset()

    def close(self) -> None:
        """Unmap the peers and free this rank's area (collective: all ranks call it)."""
        self.area.close()


class PeerSum:
    """In-place all-reduce (sum) of short vectors over NVLink peer memory (popkv_peer_sum).

    For the tensor-parallel decode's partial products: one launch, no NCCL
    kernel, and the next kernel of the step may start filling its weight ring
    while the words cross NVLink.  Constructed collectively for vectors of
    exactly ``count`` values of ``dtype``; every rank must launch the same
    sequence of sums.  The sum is taken in fp32 in rank order and rounded
    once, so all ranks hold identical bits.
    """

    def __init__(self, count: int, dtype: torch.dtype, device, group=None) -> None:
        import torch.distributed as dist

        from . import _lib
        self._lib = _lib
        self.count = int(count)
        self.dtype = dtype
        elem = torch.empty((), dtype=dtype).element_size()
        if self.count <= 0 or (self.count * elem) % 4:
            raise ValueError("count * element size must be a positive multiple of 4 bytes")
        self.words = self.count * elem // 4
        world = dist.get_world_size(group)
        self.area = _PeerArea(2 * world * self.words * 8, device, group)
        self.world, self.rank = self.area.world, self.area.rank
        self.state = self.area.state

    def launch(self, data: torch.Tensor, stream) -> None:
        """Replace ``data`` (``count`` contiguous values) by the sum over ranks, on ``stream``."""
        import ctypes
        if data.dtype != self.dtype or data.numel() != self.count or not data.is_contiguous():
            raise ValueError(f"PeerSum expects {self.count} contiguous {self.dtype} values")
        lib, _lib = self._lib.lib(), self._lib
        _lib.check(lib.popkv_peer_sum(
            _lib.ptr(data), _lib.dtype_code(data), self.count, self.rank, self.world, _lib.ptr(self.area.ptrs),
            ctypes.c_void_p(self.area.own.value), _lib.ptr(self.state), stream))

    def error(self) -> bool:
        return self.area.error()

    def reset(self) -> None:
        """Clear the area and launch state on every rank together (collective), after ``error()``."""
        self.area.reset()

    def close(self) -> None:
        """Unmap the peers and free this rank's area (collective: all ranks call it)."""
        self.area.close()
