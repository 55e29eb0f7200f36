"""KV-head sharding of the paged hot path over several GPUs (one process each).

Partition.  With ``W`` ranks, rank ``r`` owns KV heads
``[r*KVH/W, (r+1)*KVH/W)`` and the query heads that read them,
``[r*H/W, (r+1)*H/W)`` - contiguous because query head ``h`` reads KV head
``h // group`` (src/llmopt/attention/paged_attention.py:189-210).  Each rank
holds its heads' slice of the block pool as its own ``PagedKVCache`` with
``KVH/W`` heads; block tables and context lengths are replicated (the host
``BlockPool`` stays one instance), so the same physical block ids are used on
every GPU.

Exchange.  Attention is independent per (sequence, KV head); the only
cross-GPU step is an all-gather of the outputs, gathered head-major as
``[H, seq, q_len, head_dim]`` so that a permuted view gives ``[seq, H, q_len,
head_dim]`` with no extra copy.  Two transports:

* ``"peer"`` (default): the combine kernel itself stores every merged row into
  every rank's gathered buffer over NVLink (peer-mapped ``cudaMalloc`` memory
  shared through CUDA IPC, see :class:`PeerGroup`) and ends with a bounded
  cross-rank barrier on flags in peer memory - compute and exchange in one
  kernel, no separate collective.
* ``"nccl"``: the combine writes this rank's heads into the all-gather input
  and ``all_gather_into_tensor`` over NCCL follows.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _lib
from .attention import PagedAttention, PagedAttentionConfig
from .cache import PagedKVCache


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    kv_lo: int
    kv_hi: int
    q_lo: int
    q_hi: int

    @property
    def kv_heads(self) -> int:
        return self.kv_hi - self.kv_lo

    @property
    def q_heads(self) -> int:
        return self.q_hi - self.q_lo


def shard_heads(num_heads: int, num_kv_heads: int, world: int, rank: int) -> HeadShard:
    """The KV and query head ranges rank ``rank`` of ``world`` owns."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if num_heads % num_kv_heads:
        raise ValueError("num_heads must be divisible by num_kv_heads")
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} KV heads cannot be split over {world} ranks")
    kv = num_kv_heads // world
    q = num_heads // world
    return HeadShard(rank, world, rank * kv, (rank + 1) * kv, rank * q, (rank + 1) * q)


def gather_heads(local_head_major: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather ``[H/W, seq, q_len, D]`` shards into a ``[seq, H, q_len, D]`` view."""
    world = dist.get_world_size(group)
    h_local = local_head_major.shape[0]
    full = torch.empty((world * h_local, *local_head_major.shape[1:]),
                       dtype=local_head_major.dtype, device=local_head_major.device)
    dist.all_gather_into_tensor(full, local_head_major.contiguous(), group=group)
    return full.permute(1, 0, 2, 3)


class CudaPeerMemory:
    """Device buffers shared between the ranks' processes through CUDA IPC.

    Thin wrapper over ``llmopt_peer_alloc`` / ``_open`` / ``_close`` / ``_free``;
    :class:`PeerGroup` takes any object with these four methods, so its
    exchange and sizing logic can run against a fake on CPU.
    """

    def __init__(self, device: torch.device) -> None:
        self.device = device.index

    def alloc(self, nbytes: int) -> tuple[int, bytes]:
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(_lib.PEER_HANDLE_BYTES)
        _lib.check(_lib.lib().llmopt_peer_alloc(self.device, nbytes, ctypes.byref(ptr), handle),
                   "peer_alloc")
        return int(ptr.value), bytes(handle.raw)

    def open(self, handle: bytes) -> int:
        ptr = ctypes.c_void_p()
        _lib.check(_lib.lib().llmopt_peer_open(self.device, handle, ctypes.byref(ptr)),
                   "peer_open")
        return int(ptr.value)

    def close(self, ptr: int) -> None:
        _lib.check(_lib.lib().llmopt_peer_close(self.device, ptr), "peer_close")

    def free(self, ptr: int) -> None:
        _lib.check(_lib.lib().llmopt_peer_free(self.device, ptr), "peer_free")


class _RawDevice:
    """``__cuda_array_interface__`` over memory this module owns (no copy, no free)."""

    def __init__(self, ptr: int, nbytes: int) -> None:
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 2, "strides": None}


def _next_epoch(epoch: int) -> int:
    """The epoch after ``epoch``, modulo 2^32.

    The first call gets 1 (the flags start at 0).  After 0xFFFFFFFF comes 0:
    the kernel compares flags by serial-number arithmetic, and the parity keeps
    alternating the two gathered buffers across the wrap.
    """
    return (epoch + 1) & 0xFFFFFFFF


@dataclass
class _Mapped:
    nbytes: int
    local: int             # this rank's allocation
    ptrs: list             # every rank's allocation as mapped here (local at [rank])


class PeerGroup:
    """Peer-mapped flags and two gathered buffers for the fused all-gather.

    Every rank of ``group`` must create it, size it and call it in the same
    order with the same sizes (the head-sharded forward does).  Buffers grow
    collectively (synchronise, barrier, unmap, free, allocate, exchange the
    IPC handles with ``all_gather_object``, map); the steady state allocates
    nothing.  Calls alternate between the two buffers, so the result of one
    call stays intact until the call after next.  Growth replaces the
    buffers, so before capturing calls in a CUDA graph ``reserve`` the largest
    size the graph will need.
    """

    def __init__(self, group=None, device: torch.device | None = None, memory=None) -> None:
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _lib.MAX_PEERS:
            raise ValueError(f"a peer group holds at most {_lib.MAX_PEERS} ranks")
        self.device = device if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.memory = memory if memory is not None else CudaPeerMemory(self.device)
        self.epoch = 0
        self._flags = self._map(_lib.PEER_FLAGS_BYTES)
        self._bufs: list[_Mapped | None] = [None, None]
        self._arrays: dict = {}

    def _map(self, nbytes: int) -> _Mapped:
        local, handle = self.memory.alloc(nbytes)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=self.group)
        ptrs = [local if r == self.rank else self.memory.open(h) for r, h in enumerate(handles)]
        return _Mapped(nbytes, local, ptrs)

    def _unmap(self, m: _Mapped) -> None:
        for r, p in enumerate(m.ptrs):
            if r != self.rank:
                self.memory.close(p)
        dist.barrier(group=self.group)     # every peer has unmapped before the free
        self.memory.free(m.local)

    def _quiesce(self) -> None:
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    def reserve(self, nbytes: int) -> None:
        """Make both gathered buffers at least ``nbytes`` (collective when they grow)."""
        if all(b is not None and b.nbytes >= nbytes for b in self._bufs):
            return
        size = 1 << max(20, (nbytes - 1).bit_length())
        self._quiesce()
        for i, b in enumerate(self._bufs):
            if b is not None:
                self._unmap(b)
            self._bufs[i] = None
        self._bufs = [self._map(size), self._map(size)]
        self._arrays.clear()

    def next_call(self, nbytes: int):
        """Epoch, buffer index and ctypes pointer arrays for the next gathered call."""
        self.reserve(nbytes)
        self.epoch = _next_epoch(self.epoch)
        which = self.epoch & 1
        arrays = self._arrays.get(which)
        if arrays is None:
            arr = ctypes.c_void_p * self.world
            arrays = (arr(*self._bufs[which].ptrs), arr(*self._flags.ptrs))
            self._arrays[which] = arrays
        return self.epoch, which, arrays[0], arrays[1]

    def local_buffer(self, which: int) -> torch.Tensor:
        """This rank's gathered buffer ``which`` as a uint8 CUDA tensor (no copy)."""
        key = ("tensor", which)
        t = self._arrays.get(key)
        if t is None:
            b = self._bufs[which]
            t = torch.as_tensor(_RawDevice(b.local, b.nbytes), device=self.device)
            self._arrays[key] = t
        return t

    def close(self) -> None:
        """Release every mapping and allocation (collective)."""
        self._quiesce()
        for b in self._bufs:
            if b is not None:
                self._unmap(b)
        self._bufs = [None, None]
        if self._flags is not None:
            self._unmap(self._flags)
            self._flags = None
        self._arrays.clear()


class ShardedPagedAttention:
    """``PagedAttention`` over this rank's head shard plus the output all-gather.

    ``transport="peer"`` fuses the all-gather into the combine kernel (NVLink
    peer stores + on-device barrier); its result is a view of a buffer owned by
    the group that the call after next overwrites - ``clone()`` it to keep it.
    ``transport="nccl"`` runs ``all_gather_into_tensor`` after the combine.
    """

    def __init__(self, num_heads: int, num_kv_heads: int, head_dim: int,
                 scale: float | None = None, config: PagedAttentionConfig | None = None,
                 group=None, split_mode: str = "auto", transport: str = "peer") -> None:
        if transport not in ("peer", "nccl"):
            raise ValueError("transport must be 'peer' or 'nccl'")
        self.group = group
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        self.shard = shard_heads(num_heads, num_kv_heads, world, rank)
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.transport = transport
        self.local = PagedAttention(self.shard.q_heads, self.shard.kv_heads, head_dim,
                                    scale=scale if scale is not None else head_dim ** -0.5,
                                    config=config, split_mode=split_mode)
        self.peers: PeerGroup | None = None

    def local_query(self, query: torch.Tensor) -> torch.Tensor:
        """This rank's heads of a full ``[seq, H, q_len, D]`` query."""
        return query[:, self.shard.q_lo:self.shard.q_hi]

    def _buffer(self, seq: int, q_len: int, dtype, device) -> torch.Tensor:
        # A fresh all-gather input per call (the caching allocator makes it cheap):
        # a cached one replaced when the shape changes would leave a captured CUDA
        # graph writing into freed memory.
        return torch.empty((self.shard.q_heads, seq, q_len, self.head_dim), dtype=dtype,
                           device=device)

    def forward(self, query_local: torch.Tensor, cache: PagedKVCache, layer_idx: int,
                block_ids: torch.Tensor, context_lens: torch.Tensor,
                query_lens: int | None = None, phases: int = _lib.PHASE_ALL) -> torch.Tensor:
        """``[seq, H, q_len, D]`` output from this rank's ``[seq, H/W, q_len, D]`` query.

        With ``transport="peer"``, ``phases`` may split the call into the
        split-K kernel and the fused combine + all-gather (both with the same
        arguments); the gathered view is returned by the call that combines.
        """
        seq, _, q_len, _ = query_local.shape
        device = cache.key_cache.device
        if self.transport == "nccl":
            head_major = self._buffer(seq, q_len, query_local.dtype, device)
            self.local.forward_with_lse(query_local, cache, layer_idx, block_ids, context_lens,
                                        query_lens, want_lse=False,
                                        out=head_major.permute(1, 0, 2, 3))
            return gather_heads(head_major, self.group)
        if self.peers is None:
            self.peers = PeerGroup(self.group, device)
        dtype = query_local.dtype if query_local.dtype in (
            torch.float32, torch.float16, torch.bfloat16) else torch.float32
        elem = torch.finfo(dtype).bits // 8
        nbytes = self.num_heads * seq * q_len * self.head_dim * elem
        if phases & _lib.PHASE_COMBINE:
            epoch, which, bufs, flags = self.peers.next_call(nbytes)
        else:
            # The split phase touches no peer memory; it only needs the shapes
            # and this rank's slice of the buffer the next combine will use.
            self.peers.reserve(nbytes)
            epoch = _next_epoch(self.peers.epoch)
            which = epoch & 1
            bufs = flags = None
        full = self.peers.local_buffer(which)[:nbytes].view(dtype).view(
            self.num_heads, seq, q_len, self.head_dim)
        own = full[self.shard.q_lo:self.shard.q_hi].permute(1, 0, 2, 3)
        if bufs is None:
            self.local.forward_with_lse(query_local, cache, layer_idx, block_ids, context_lens,
                                        query_lens, want_lse=False, out=own, phases=phases)
        else:
            self.local.forward_with_lse(query_local, cache, layer_idx, block_ids, context_lens,
                                        query_lens, want_lse=False, out=own, phases=phases,
                                        gather=(bufs, flags, self.peers.world, self.peers.rank,
                                                epoch))
        return full.permute(1, 0, 2, 3)

    def close(self) -> None:
        """Release the peer buffers (collective; call on every rank before shutdown)."""
        if self.peers is not None:
            self.peers.close()
            self.peers = None


def local_cache(num_layers: int, num_blocks: int, block_size: int, num_kv_heads: int,
                head_dim: int, dtype: torch.dtype, device, group=None) -> PagedKVCache:
    """This rank's slice of the block pool: the same block ids, ``KVH/W`` heads."""
    world = dist.get_world_size(group)
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} KV heads cannot be split over {world} ranks")
    return PagedKVCache(num_layers, num_blocks, block_size, num_kv_heads // world, head_dim,
                        dtype=dtype, device=device)
