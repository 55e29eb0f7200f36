"""One rank of the multi-GPU head-sharding check (launched by test_gpu_dist.py via torchrun).

Every rank builds the same seeded decode and prefill cases, keeps its KV heads'
slice of the pool, runs ShardedPagedAttention with both transports (NCCL
all-gather, and the combine kernel's own NVLink peer stores + barrier), several
calls each, and compares the gathered [seq, H, q_len, D] output with the CPU
oracle.
Rank 0 prints one "OK <world>" line when every rank passed.
"""

from __future__ import annotations

import datetime
import importlib
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.dirname(HERE), HERE, os.path.join(HERE, "golden")]

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from _gpu import to_dev  # noqa: E402
from cases import build_paged_case  # noqa: E402
from oracle import paged_oracle as po  # noqa: E402


def check_case(case, dev, pkg, pdist, transport="nccl", repeats=1) -> float:
    world, rank = dist.get_world_size(), dist.get_rank()
    H, KVH = case["heads"], case["kv_heads"]
    shard = pdist.shard_heads(H, KVH, world, rank)
    L, nb, bs, _, d = case["key_cache"].shape
    cache = pdist.local_cache(L, nb, bs, KVH, d, torch.bfloat16, dev)
    kc = to_dev(case["key_cache"], "bf16", dev)
    vc = to_dev(case["value_cache"], "bf16", dev)
    cache.key_cache.copy_(kc[:, :, :, shard.kv_lo:shard.kv_hi])
    cache.value_cache.copy_(vc[:, :, :, shard.kv_lo:shard.kv_hi])
    attn = pdist.ShardedPagedAttention(H, KVH, d, transport=transport)
    q = to_dev(case["query"], "bf16", dev)
    table = torch.from_numpy(case["block_ids"]).to(dev)
    ctx = torch.from_numpy(case["context_lens"]).to(dev)
    want, _ = po.paged_attention(case["query"], "bf16", case["key_cache"], case["value_cache"],
                                 "bf16", 0, case["block_ids"], case["context_lens"], H, KVH,
                                 q_len=case["q_len"], acc=np.float32)
    worst = 0.0
    outs = []
    for i in range(repeats):
        # Alternate the whole call with the split / combine halves.
        if i % 2 == 0:
            out = attn.forward(attn.local_query(q), cache, 0, table, ctx, case["q_len"])
        else:
            attn.forward(attn.local_query(q), cache, 0, table, ctx, case["q_len"],
                         phases=pkg._lib.PHASE_SPLIT)
            out = attn.forward(attn.local_query(q), cache, 0, table, ctx, case["q_len"],
                               phases=pkg._lib.PHASE_COMBINE)
        outs.append(out)
        torch.cuda.synchronize(dev)
        worst = max(worst, float(np.abs(out.float().cpu().numpy() - want).max()))
    if repeats > 1:
        # The previous call's gathered view is still intact (two alternating buffers).
        worst = max(worst, float(np.abs(outs[-2].float().cpu().numpy() - want).max()))
    if pkg._runtime.read_and_clear_errors(dev):
        worst = float("inf")
    attn.close()
    return worst


def main() -> None:
    rank = int(os.environ["RANK"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    pkg = importlib.import_module("quantized-llm-inference-engine-_b200")
    pdist = importlib.import_module("quantized-llm-inference-engine-_b200.dist")
    errs = []
    decode = build_paged_case(70, batch=6, heads=32, kv_heads=8, head_dim=128, block_size=16,
                              ctx=[1, 17, 300, 1000, 64, 2048], kv_kind="bf16", q_kind="bf16",
                              value_scale=0.5)
    prefill = build_paged_case(71, batch=3, heads=32, kv_heads=8, head_dim=128, block_size=16,
                               ctx=[100, 300, 64], kv_kind="bf16", q_kind="bf16", q_len=48)
    for transport in ("nccl", "peer"):
        errs.append(check_case(decode, dev, pkg, pdist, transport, repeats=3))
        errs.append(check_case(prefill, dev, pkg, pdist, transport, repeats=2))
    worst = torch.tensor([max(errs)], device=dev)
    dist.all_reduce(worst, op=dist.ReduceOp.MAX)
    if rank == 0:
        status = "OK" if worst.item() <= 2e-2 else "FAIL"
        print(f"{status} {dist.get_world_size()} max_abs_err={worst.item():.3e}", flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
