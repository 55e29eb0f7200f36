"""Head-sharding plumbing on CPU: shard ranges and the output all-gather (gloo, 2 ranks).

The kernels themselves need a GPU; what is tested here is the host logic that
surrounds them on several ranks: which heads each rank owns, and that the
head-major all-gather reassembles ``[seq, H, q_len, D]`` exactly.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import load_package


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_heads_partition():
    from importlib import import_module

    d = import_module("quantized-llm-inference-engine-_b200.dist")
    for world in (1, 2, 4, 8):
        shards = [d.shard_heads(64, 8, world, r) for r in range(world)]
        assert [s.kv_lo for s in shards] == [r * 8 // world for r in range(world)]
        assert shards[-1].kv_hi == 8 and shards[-1].q_hi == 64
        for s in shards:
            # query head h reads KV head h // group: the query range maps into the KV range
            group = 64 // 8
            assert s.q_lo // group == s.kv_lo and (s.q_hi - 1) // group == s.kv_hi - 1
    with pytest.raises(ValueError):
        d.shard_heads(32, 8, 3, 0)
    with pytest.raises(ValueError):
        d.shard_heads(32, 8, 2, 2)


def _worker(rank: int, world: int, port: int, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    from importlib import import_module

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        d = import_module("quantized-llm-inference-engine-_b200.dist")
        seq, H, q_len, D = 3, 8, 2, 4
        g = torch.Generator().manual_seed(0)
        full = torch.randn(seq, H, q_len, D, generator=g)      # what every rank should end with
        shard = d.shard_heads(H, 4, world, rank)
        local = full[:, shard.q_lo:shard.q_hi].permute(1, 0, 2, 3).contiguous()  # head-major
        got = d.gather_heads(local)
        result_q.put((rank, bool(torch.equal(got, full)), tuple(got.shape)))
    finally:
        dist.destroy_process_group()


def test_head_major_all_gather_world2():
    load_package()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok, _ in results)
    assert all(shape == (3, 8, 2, 4) for _, _, shape in results)


class _FakePeerMemory:
    """Host stand-in for CUDA IPC: handles encode (rank, pointer), mappings are logged."""

    def __init__(self, rank: int):
        self.rank = rank
        self.next = 1
        self.live: dict[int, int] = {}
        self.opened: list[int] = []
        self.closed: list[int] = []
        self.freed: list[int] = []

    def alloc(self, nbytes):
        ptr = (self.rank + 1) << 32 | self.next << 8
        self.next += 1
        self.live[ptr] = nbytes
        return ptr, f"{self.rank}:{ptr}".encode()

    def open(self, handle):
        owner, ptr = handle.decode().split(":")
        assert int(owner) != self.rank, "a rank must not map its own handle"
        mapped = int(ptr) | 1   # a distinct address for the mapping
        self.opened.append(mapped)
        return mapped

    def close(self, ptr):
        assert ptr in self.opened and ptr not in self.closed
        self.closed.append(ptr)

    def free(self, ptr):
        assert ptr in self.live
        del self.live[ptr]
        self.freed.append(ptr)


def _peer_group_worker(rank: int, world: int, port: int, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    from importlib import import_module

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        d = import_module("quantized-llm-inference-engine-_b200.dist")
        mem = _FakePeerMemory(rank)
        pg = d.PeerGroup(device=torch.device("cpu"), memory=mem)
        checks = []
        # Flags: own allocation at [rank], every other slot is that peer's mapping.
        f = pg._flags
        checks.append(f.ptrs[rank] == f.local)
        checks.append(all(((p >> 32) - 1) == r and p & 1 for r, p in enumerate(f.ptrs)
                          if r != rank))
        e1, w1, bufs1, flags1 = pg.next_call(1000)
        e2, w2, bufs2, _ = pg.next_call(1000)
        checks.append((e1, w1, e2, w2) == (1, 1, 2, 0))
        checks.append(len(mem.live) == 3)                      # flags + two buffers, no regrowth
        checks.append(all(b.nbytes == 1 << 20 for b in pg._bufs))
        checks.append(list(bufs1) == pg._bufs[1].ptrs and list(bufs2) == pg._bufs[0].ptrs)
        checks.append(list(flags1) == f.ptrs)
        old = [b.local for b in pg._bufs]
        e3, w3, _, _ = pg.next_call((2 << 20) + 1)            # grows collectively
        checks.append((e3, w3) == (3, 1))
        checks.append(all(b.nbytes == 4 << 20 for b in pg._bufs))
        checks.append(sorted(mem.freed) == sorted(old))
        # the epoch wraps modulo 2^32 and keeps alternating the two buffers
        pg.epoch = 0xFFFFFFFE
        wrap = [pg.next_call(1000)[:2] for _ in range(3)]
        checks.append(wrap == [(0xFFFFFFFF, 1), (0, 0), (1, 1)])
        pg.close()
        checks.append(not mem.live and sorted(mem.closed) == sorted(mem.opened))
        checks.append(len(mem.opened) == 5 * (world - 1))   # flags + 2 + 2 buffers per peer
        result_q.put((rank, checks))
    finally:
        dist.destroy_process_group()


def test_peer_group_exchange_and_growth_world2():
    load_package()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_group_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, checks in results:
        assert all(checks), (rank, checks)
