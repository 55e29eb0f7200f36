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
cross-GPU step is an all-gather of the outputs.  Each rank's combine kernel
writes its heads head-major, ``[H/W, seq, q_len, head_dim]``, straight into
the all-gather input, so ``all_gather_into_tensor`` over NCCL yields
``[H, seq, q_len, head_dim]`` and a permuted view gives ``[seq, H, q_len,
head_dim]`` with no extra copy.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

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


class ShardedPagedAttention:
    """``PagedAttention`` over this rank's head shard plus the output all-gather."""

    def __init__(self, num_heads: int, num_kv_heads: int, head_dim: int,
                 scale: float | None = None, config: PagedAttentionConfig | None = None,
                 group=None, split_mode: str = "auto") -> None:
        self.group = group
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        self.shard = shard_heads(num_heads, num_kv_heads, world, rank)
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.local = PagedAttention(self.shard.q_heads, self.shard.kv_heads, head_dim,
                                    scale=scale if scale is not None else head_dim ** -0.5,
                                    config=config, split_mode=split_mode)
        self._bufs: dict = {}

    def local_query(self, query: torch.Tensor) -> torch.Tensor:
        """This rank's heads of a full ``[seq, H, q_len, D]`` query."""
        return query[:, self.shard.q_lo:self.shard.q_hi]

    def _buffer(self, seq: int, q_len: int, dtype, device) -> torch.Tensor:
        key = (seq, q_len, dtype, device)
        buf = self._bufs.get(key)
        if buf is None:
            buf = torch.empty((self.shard.q_heads, seq, q_len, self.head_dim), dtype=dtype,
                              device=device)
            self._bufs = {key: buf}
        return buf

    def forward(self, query_local: torch.Tensor, cache: PagedKVCache, layer_idx: int,
                block_ids: torch.Tensor, context_lens: torch.Tensor,
                query_lens: int | None = None) -> torch.Tensor:
        """``[seq, H, q_len, D]`` output from this rank's ``[seq, H/W, q_len, D]`` query."""
        seq, _, q_len, _ = query_local.shape
        head_major = self._buffer(seq, q_len, query_local.dtype, cache.key_cache.device)
        self.local.forward_with_lse(query_local, cache, layer_idx, block_ids, context_lens,
                                    query_lens, want_lse=False,
                                    out=head_major.permute(1, 0, 2, 3))
        return gather_heads(head_major, self.group)


def local_cache(num_layers: int, num_blocks: int, block_size: int, num_kv_heads: int,
                head_dim: int, dtype: torch.dtype, device, group=None) -> PagedKVCache:
    """This rank's slice of the block pool: the same block ids, ``KVH/W`` heads."""
    world = dist.get_world_size(group)
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} KV heads cannot be split over {world} ranks")
    return PagedKVCache(num_layers, num_blocks, block_size, num_kv_heads // world, head_dim,
                        dtype=dtype, device=device)
