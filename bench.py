#!/usr/bin/env python
"""Paged-decode benchmark on B200 (Llama-3-8B attention shape).

One step = one layer's decode hot path for a batch: the KV append of one new
token per sequence (``PagedKVCache.write_decode``), the split-K paged decode
attention kernel, the LSE combine, and - with N > 1 GPUs - the NCCL all-gather
of the head-sharded outputs.  Workload per GPU (weak scaling): 64 sequences,
32 query / 8 KV heads, head_dim 128, block_size 16, context U[1024, 8192],
bf16 K/V/q ~ 0.5*N(0,1), random block tables over a pool of sum(blocks)+10%.
With N GPUs the batch is 64*N sequences and each GPU owns 8/N KV heads of all
of them (its slice of the pool; tables replicated).

Printed (rank 0, one JSON line):
  value     whole-job algorithmic HBM GB/s of the step (decode + append bytes of
            all ranks / device time, max over ranks), inputs resident in HBM;
  e2e       the same metric through the public Python API with host buffers:
            pinned H2D of q, new K/V, block table, lengths; D2H of the output;
  roofline  the split-K decode kernel alone: algorithmic bytes per launch over
            its CUDA-event time, against the measured HBM copy bandwidth;
  cpu_baseline / --impl reference: the CPU oracle port of the reference path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""

from __future__ import annotations

import argparse
import datetime
import importlib
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
PACKAGE = "quantized-llm-inference-engine-_b200"

METRIC = "paged-decode attn HBM GB/s (% of ~8 TB/s) and decode tok/s at 1/2/4/8 B200"
HEADS, KV_HEADS, HEAD_DIM, BLOCK = 32, 8, 128, 16
FALLBACK_HBM_GBS = 6650.0
PROFILE_TRAFFIC = os.path.join(REPO, "profiles", "decode_tma_config2.txt")


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--batch", type=int, default=64, help="sequences per GPU")
    p.add_argument("--ctx-lo", type=int, default=1024)
    p.add_argument("--ctx-hi", type=int, default=8192)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--transport", choices=("peer", "nccl"), default="peer",
                   help="N>1 output all-gather: fused into the combine kernel over NVLink "
                        "peer memory, or NCCL all_gather_into_tensor after it")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--config", choices=("c2", "c3", "c4", "c5", "rope", "step", "fp8", "quant"),
                   default="c2",
                   help="c2 (default, the headline line): Llama-3-8B decode; c3: chunked "
                        "prefill; c4: 128k-context decode sharded by KV head (strong "
                        "scaling); c5: shared-prefix decode (strong scaling); rope: the "
                        "fused rotary + KV append of a 16 x 256-token prefill chunk and of "
                        "a 64-sequence decode step (weak scaling by KV head); step: a whole "
                        "decode step (device-side metadata advance, rotary append, "
                        "attention) replayed from a CUDA graph vs launched eagerly, beside "
                        "the reference runner's host-side metadata build; fp8: the config-2 "
                        "decode step over an e4m3 KV cache beside the bf16 one (1 GPU); "
                        "quant: QuantLinear's fused int4 dequantize-GEMM on the Llama-3-8B "
                        "MLP shapes beside the dense bf16 GEMM (1 GPU)")
    return p.parse_args(argv)


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------

def make_workload(args, world: int):
    """Context lengths, block tables and pool size (identical on every rank)."""
    batch = args.batch * world
    rng = np.random.default_rng(args.seed)
    ctx = rng.integers(args.ctx_lo, args.ctx_hi + 1, size=batch).astype(np.int64)
    nblk = (ctx + BLOCK - 1) // BLOCK
    num_blocks = int(nblk.sum() * 1.10) + 1
    perm = rng.permutation(num_blocks)
    table = np.full((batch, int(nblk.max())), -1, dtype=np.int32)
    o = 0
    for s, n in enumerate(nblk):
        table[s, :n] = perm[o:o + n]
        o += int(n)
    offsets = ctx - 1                      # the new token's position (slot (ctx-1) % 16)
    return dict(batch=batch, ctx=ctx, table=table, num_blocks=num_blocks, offsets=offsets)


def step_bytes(ctx, kv_heads: int, q_heads: int, batch: int) -> tuple[int, int]:
    """Algorithmic bytes of one step on one GPU: (decode, append)."""
    from oracle.paged_oracle import decode_bytes

    dec = decode_bytes(ctx, kv_heads, HEAD_DIM, 2, batch, q_heads, 2, 2, BLOCK)
    app = batch * kv_heads * HEAD_DIM * 2 * (2 + 2)   # K and V rows: read bf16 + write bf16
    return dec, app


def measured_hbm_peak():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic():
    """DRAM bytes per decode launch from the committed ncu summary, if present."""
    try:
        with open(PROFILE_TRAFFIC) as f:
            for line in f:
                if line.startswith("dram_bytes_per_launch:"):
                    return int(float(line.split(":", 1)[1].split()[0]))
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------------
# clocks (NVML) during the timed region
# ---------------------------------------------------------------------------

_REASONS = {
    0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
    0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
    0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
}


class ClockSampler:
    def __init__(self, device_index: int):
        self.samples: list[int] = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._handle = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(device_index)
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            self._nvml = pynvml
            self._handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
            # the first queries of a handle are slow: make them before any timed region
            pynvml.nvmlDeviceGetClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
            pynvml.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
        except Exception:
            self._handle = None

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
            except Exception:
                pass
            time.sleep(0.0002)

    def start(self):
        if self._handle is not None:
            # The launching thread holds the GIL while it issues kernels; a short
            # switch interval lets the sampler run inside a timed region of a
            # few milliseconds.
            self._switch = sys.getswitchinterval()
            sys.setswitchinterval(1e-4)
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self) -> dict:
        if self._thread is not None:
            self._stop.set()
            self._thread.join()
            sys.setswitchinterval(self._switch)
        names = sorted(n for bit, n in _REASONS.items() if self.reasons & bit)
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}


KERNEL_ITERS = 200


def kernel_loop_ms(fn, dev, barrier, iters: int = KERNEL_ITERS) -> float:
    """Average device time of ``fn`` over ``iters`` back-to-back calls.

    Two events on the current stream bracket the loop (the stream every kernel
    of the step is launched on); three untimed calls come first.
    """
    import torch

    for _ in range(3):
        fn()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    barrier()
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize(dev)
    return a.elapsed_time(b) / iters


# ---------------------------------------------------------------------------
# CPU oracle timing (cpu_baseline leg and the --impl reference arm)
# ---------------------------------------------------------------------------

def _cpu_threads() -> int:
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    return torch.get_num_threads()


def cpu_oracle_sample(wl: dict, seqs: list[int], seed: int):
    """Host-side inputs for the CPU port on a subset of the workload's sequences."""
    import torch

    g = torch.Generator().manual_seed(seed + 17)
    table = wl["table"][seqs].astype(np.int64)
    used = np.unique(table[table >= 0])
    remap = np.full(wl["num_blocks"], -1, dtype=np.int64)
    remap[used] = np.arange(used.size)
    sub_table = np.where(table >= 0, remap[np.maximum(table, 0)], -1)
    shape = (1, int(used.size), BLOCK, KV_HEADS, HEAD_DIM)
    n = len(seqs)

    def rnd(*shape, scale=0.5):
        return (torch.randn(shape, generator=g) * scale).to(torch.bfloat16)

    return dict(kc=rnd(*shape), vc=rnd(*shape), q=rnd(n, HEADS, 1, HEAD_DIM),
                kn=rnd(n, KV_HEADS, HEAD_DIM), table=torch.from_numpy(sub_table),
                ctx=torch.from_numpy(wl["ctx"][seqs].copy()),
                offsets=torch.from_numpy(wl["offsets"][seqs].copy()), np_ctx=wl["ctx"][seqs])


def cpu_oracle_step(s: dict) -> None:
    """The reference path restated with torch CPU ops (all host threads, bf16 math as the
    reference): write_decode, then forward with the default split_size 512."""
    from oracle import paged_oracle_torch as pt

    pt.write_decode(s["kc"], s["vc"], 0, s["table"], s["offsets"], s["kn"], s["kn"])
    pt.forward(s["q"], s["kc"], s["vc"], 0, s["table"], s["ctx"], HEADS, KV_HEADS,
               split_kv=True, split_size=512)


def cpu_sample_bytes(s: dict) -> int:
    dec, app = step_bytes(s["np_ctx"], KV_HEADS, HEADS, len(s["np_ctx"]))
    return dec + app


def time_cpu(wl: dict, seed: int, budget_s: float):
    """A bounded sample (first n sequences) whose oracle step takes about ``budget_s``."""
    _cpu_threads()
    s = cpu_oracle_sample(wl, [0], seed)
    cpu_oracle_step(s)                      # first call pays one-time costs
    t0 = time.perf_counter()
    cpu_oracle_step(s)
    one = max(time.perf_counter() - t0, 1e-3)
    n = int(max(1, min(wl["batch"], budget_s / one)))
    seqs = list(range(n))
    return cpu_oracle_sample(wl, seqs, seed), seqs


def cpu_baseline(wl: dict, seed: int, total_budget_s: float = 20.0) -> dict:
    s, seqs = time_cpu(wl, seed, budget_s=total_budget_s / 4)
    cpu_oracle_step(s)                                   # warm-up
    times = []
    for _ in range(3):
        t0 = time.perf_counter()
        cpu_oracle_step(s)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": round(cpu_sample_bytes(s) / t / 1e9, 4), "unit": "GB/s",
            "cores": _cpu_threads(), "kind": "port",
            "sample": (f"first {len(seqs)} of {wl['batch']} sequences of the workload "
                       f"(append + split_size-512 decode, torch CPU bf16 restatement of the "
                       f"reference path), median of 3 after 1 warm-up, {t:.2f} s/step"),
            "seconds_per_sample": round(t, 4)}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    if rank != 0:
        return
    wl = make_workload(args, max(world, 1))
    # Size one step so that warm-up + timed steps finish within ~3 minutes.
    per_step = max(0.2, min(5.0, 180.0 / max(1, args.steps + args.warmup)))
    s, seqs = time_cpu(wl, args.seed, budget_s=per_step)
    for _ in range(args.warmup):
        cpu_oracle_step(s)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        cpu_oracle_step(s)
        times.append(time.perf_counter() - t0)
    t = sum(times) / len(times)
    value = cpu_sample_bytes(s) / t / 1e9
    cores = _cpu_threads()
    sample = (f"first {len(seqs)} of {wl['batch']} sequences per step (append + split_size-512 "
              f"decode, torch CPU bf16 restatement of the reference path)")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s",
        "n_gpus": max(world, 1), "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(t * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config2 paged decode (append + attention), CPU oracle port of "
                               "the reference path", "global_batch": wl["batch"],
                   "seq_len": f"U[{args.ctx_lo},{args.ctx_hi}]", "heads": HEADS,
                   "kv_heads": KV_HEADS, "head_dim": HEAD_DIM, "block_size": BLOCK},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": cores,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    pkg = importlib.import_module(PACKAGE)
    pdist = importlib.import_module(f"{PACKAGE}.dist")
    _lib = importlib.import_module(f"{PACKAGE}._lib")

    wl = make_workload(args, world)
    B = wl["batch"]
    shard = pdist.shard_heads(HEADS, KV_HEADS, world, rank)
    kvh, qh = shard.kv_heads, shard.q_heads
    cache = pkg.PagedKVCache(1, wl["num_blocks"], BLOCK, kvh, HEAD_DIM, dtype=torch.bfloat16,
                             device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    for t in (cache.key_cache, cache.value_cache):
        for i in range(0, t.shape[1], 4096):     # fill in slices: bounded temporaries
            sl = t[:, i:i + 4096]
            sl.copy_(torch.randn(sl.shape, generator=g, device=dev) * 0.5)
    table = torch.from_numpy(wl["table"]).to(dev)
    ctx = torch.from_numpy(wl["ctx"]).to(dev)
    offs = torch.from_numpy(wl["offsets"]).to(dev)
    q = (torch.randn((B, qh, 1, HEAD_DIM), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    knew = (torch.randn((B, kvh, HEAD_DIM), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    vnew = (torch.randn((B, kvh, HEAD_DIM), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    attn = pkg.PagedAttention(qh, kvh, HEAD_DIM)
    head_major = torch.empty((qh, B, 1, HEAD_DIM), dtype=torch.bfloat16, device=dev)
    out_view = head_major.permute(1, 0, 2, 3)
    peer = world > 1 and args.transport == "peer"
    gathered = (torch.empty((HEADS, B, 1, HEAD_DIM), dtype=torch.bfloat16, device=dev)
                if world > 1 and not peer else None)
    # With the peer transport the combine kernel also delivers every rank's
    # heads to every rank (NVLink stores + on-device barrier).
    sharded_step = (pdist.ShardedPagedAttention(HEADS, KV_HEADS, HEAD_DIM, transport="peer")
                    if peer else None)

    def append():
        cache.write_decode(0, table, offs, knew, vnew)

    def decode():
        if peer:
            sharded_step.forward(q, cache, 0, table, ctx, 1, phases=_lib.PHASE_SPLIT)
        else:
            attn.forward_with_lse(q, cache, 0, table, ctx, 1, want_lse=False, out=out_view,
                                  phases=_lib.PHASE_SPLIT)

    def combine():
        if peer:
            sharded_step.forward(q, cache, 0, table, ctx, 1, phases=_lib.PHASE_COMBINE)
        else:
            attn.forward_with_lse(q, cache, 0, table, ctx, 1, want_lse=False, out=out_view,
                                  phases=_lib.PHASE_COMBINE)

    def gather():
        if gathered is not None:
            dist.all_gather_into_tensor(gathered, head_major)

    def step():
        append()
        decode()
        combine()
        gather()

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(max(args.warmup, 3)):
        step()
    # The timed region holds the steps and nothing else: an event between two
    # kernels would break the programmatic-launch overlap of the step.
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    barrier()
    sampler.start()
    start.record()
    for _ in range(args.steps):
        step()
    end.record()
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    ms_total = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms_total], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    # Per-kernel durations (the roofline's denominator): each kernel of the
    # step alone, KERNEL_ITERS launches back to back on the launching stream,
    # after the timed region.
    append_ms = kernel_loop_ms(append, dev, barrier)
    decode_ms = kernel_loop_ms(decode, dev, barrier)
    combine_ms = kernel_loop_ms(combine, dev, barrier)
    gather_ms = kernel_loop_ms(gather, dev, barrier) if gathered is not None else 0.0
    ms_step = ms_total / args.steps
    dec_bytes, app_bytes = step_bytes(wl["ctx"], kvh, qh, B)
    value = world * (dec_bytes + app_bytes) / (ms_step * 1e-3) / 1e9

    # ---- end to end through the public API, host buffers ----------------------------
    e2e = None
    if not args.no_e2e:
        # The step's inputs live in one pinned host buffer (q, new K, new V,
        # block table, context lengths, offsets; 256-byte aligned slices) and
        # cross PCIe in one copy per step; the result comes back in one copy.
        srcs = (q, knew, vnew, table, ctx, offs)
        offsets, total = [], 0
        for t in srcs:
            offsets.append(total)
            total += (t.numel() * t.element_size() + 255) // 256 * 256
        host = torch.empty(total, dtype=torch.uint8, pin_memory=True)
        dev_buf = torch.empty(total, dtype=torch.uint8, device=dev)

        def views(buf):
            out = []
            for t, o in zip(srcs, offsets):
                n = t.numel() * t.element_size()
                out.append(buf[o:o + n].view(t.dtype).view(t.shape))
            return out

        for hv, t in zip(views(host), srcs):
            hv.copy_(t.cpu())
        # Two device input slots and two pinned output slots: step i's inputs
        # cross PCIe on one copy stream while step i-1 computes, and its result
        # comes back on another copy stream while step i+1 computes.  Every
        # copy of every step is inside the timed region.
        dev_bufs = [dev_buf, torch.empty(total, dtype=torch.uint8, device=dev)]
        slots_in = [views(b) for b in dev_bufs]
        # Each rank reads back its own heads of the result (head-major, contiguous),
        # so the job as a whole copies the output to the host exactly once.
        out_shape = (qh, B, 1, HEAD_DIM) if world > 1 else (B, qh, 1, HEAD_DIM)
        out_h = [torch.empty(out_shape, dtype=torch.bfloat16, pin_memory=True) for _ in range(2)]
        out_d = [torch.empty((B, qh, 1, HEAD_DIM), dtype=torch.bfloat16, device=dev)
                 for _ in range(2)]
        sharded = (pdist.ShardedPagedAttention(HEADS, KV_HEADS, HEAD_DIM,
                                               transport=args.transport)
                   if world > 1 else None)
        comp = torch.cuda.current_stream(dev)
        h2d_stream = torch.cuda.Stream(dev)
        d2h_stream = torch.cuda.Stream(dev)
        in_ready = [torch.cuda.Event() for _ in range(2)]
        comp_done = [torch.cuda.Event() for _ in range(2)]
        out_done = [torch.cuda.Event() for _ in range(2)]
        for ev_list in (comp_done, out_done):
            for ev in ev_list:
                ev.record(comp)

        counter = [0]   # one count across warm-up and timed steps: slots keep alternating

        def e2e_step():
            slot = counter[0] & 1
            counter[0] += 1
            with torch.cuda.stream(h2d_stream):
                h2d_stream.wait_event(comp_done[slot])      # step i-2 no longer reads the slot
                dev_bufs[slot].copy_(host, non_blocking=True)
                in_ready[slot].record(h2d_stream)
            comp.wait_event(in_ready[slot])
            comp.wait_event(out_done[slot])                 # step i-2's result has left
            q_d, k_d, v_d, table_d, ctx_d, offs_d = slots_in[slot]
            cache.write_decode(0, table_d, offs_d, k_d, v_d)
            if world > 1:
                full = sharded.forward(q_d, cache, 0, table_d, ctx_d, 1)
                res = full.permute(1, 0, 2, 3)[shard.q_lo:shard.q_hi]
            else:
                res = attn.forward_with_lse(q_d, cache, 0, table_d, ctx_d, 1, want_lse=False,
                                            out=out_d[slot])[0]
            comp_done[slot].record(comp)
            with torch.cuda.stream(d2h_stream):
                d2h_stream.wait_event(comp_done[slot])
                out_h[slot].copy_(res, non_blocking=True)
                out_done[slot].record(d2h_stream)

        for _ in range(max(args.warmup, 3)):
            e2e_step()
        e_start = torch.cuda.Event(enable_timing=True)
        e_end = torch.cuda.Event(enable_timing=True)
        barrier()
        e_start.record(comp)
        h2d_stream.wait_stream(comp)
        d2h_stream.wait_stream(comp)
        for _ in range(args.steps):
            e2e_step()
        comp.wait_stream(h2d_stream)
        comp.wait_stream(d2h_stream)
        e_end.record(comp)
        torch.cuda.synchronize(dev)
        e_ms = e_start.elapsed_time(e_end)
        if world > 1:
            t = torch.tensor([e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_ms = float(t.item())
        h2d = int(host.numel())
        e2e = {"value": round(world * (dec_bytes + app_bytes) / (e_ms / args.steps * 1e-3) / 1e9,
                              2),
               "unit": "GB/s", "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(out_h[0].numel() * out_h[0].element_size()),
               "copies": "pipelined: H2D and D2H on two copy streams, two slots each",
               "ms_per_step": round(e_ms / args.steps, 4),
               "decode_tok_s": round(B / (e_ms / args.steps * 1e-3), 1)}

        if sharded is not None:
            sharded.close()
    if sharded_step is not None:
        sharded_step.close()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(wl, args.seed)

    if world > 1:
        dist.barrier()
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    peak, peak_kind = measured_hbm_peak()
    achieved = dec_bytes / (decode_ms * 1e-3) / 1e9
    gather_desc = (" combine fused with the all-gather over NVLink peer stores" if peer
                   else " + NCCL all-gather")
    kernel_ms = {"append": round(append_ms, 5), "decode_split": round(decode_ms, 5),
                 ("combine_gather" if peer else "combine"): round(combine_ms, 5)}
    if gathered is not None:
        kernel_ms["nccl_all_gather"] = round(gather_ms, 5)
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": max(args.warmup, 3),
        "ms_per_step": round(ms_step, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded ctx U[1024,8192], random block tables, K/V/q 0.5*N(0,1) bf16",
        "config": {
            "workload": "config2: Llama-3-8B-shaped paged decode step (KV append + split-K "
                        "decode + LSE combine" + (gather_desc if world > 1 else "") + ")",
            "global_batch": B, "seq_len": f"U[{args.ctx_lo},{args.ctx_hi}]",
            "heads": HEADS, "kv_heads": KV_HEADS, "head_dim": HEAD_DIM, "block_size": BLOCK,
            "parallelism": (f"kv-head shard x{world} (tables replicated,{gather_desc})"
                            if world > 1 else "single GPU"),
            "per_gpu": f"{args.batch * world} seqs x {kvh} KV heads",
            "l2": f"inputs larger than L2 (KV pool {2 * cache.key_cache.nbytes / 1e9:.2f} GB "
                  f"per GPU vs 126 MB L2)",
            "split": "auto (balanced split-K over SMs)",
        },
        "decode_tok_s": round(B / (ms_step * 1e-3), 1),
        "kernel_ms": kernel_ms,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": profiled_traffic(),
                     "kernel": "decode_tma_kernel (split-K paged decode)",
                     "bytes_per_launch": int(dec_bytes), "peak_kind": f"{peak_kind} hbm_gbs",
                     "timing": f"CUDA events around {KERNEL_ITERS} back-to-back decode launches "
                               f"on the launching stream, after the timed region",
                     "kernel_share_of_step": round(decode_ms / ms_step, 4)},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": 3 * args.steps,
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# secondary configs (c3 prefill, c4 long context, c5 shared prefix)
# ---------------------------------------------------------------------------

def _tables_from_counts(rng, nblk, num_blocks, shared=None):
    """Tables over a permuted pool; ``shared`` = ids every row starts with."""
    perm = rng.permutation(num_blocks)
    o = 0
    lead = [] if shared is None else list(shared)
    if shared is not None:
        perm = np.setdiff1d(perm, np.asarray(shared), assume_unique=True)
        perm = rng.permutation(perm)
    width = int(max(nblk)) + len(lead)
    table = np.full((len(nblk), width), -1, dtype=np.int32)
    for s, n in enumerate(nblk):
        table[s, :len(lead)] = lead
        table[s, len(lead):len(lead) + n] = perm[o:o + n]
        o += int(n)
    return table


def extra_workload(args, world: int) -> dict:
    rng = np.random.default_rng(args.seed + {"c3": 3, "c4": 4, "c5": 5}[args.config])
    if args.config == "c3":
        B, q_len, H, KVH = 16, 256, 32, 8
        prefix = (rng.integers(0, 4097, size=B) // BLOCK) * BLOCK
        ctx = prefix + q_len
        nblk = (ctx + BLOCK - 1) // BLOCK
        nb = int(nblk.sum() * 1.10) + 1
        return dict(kind="prefill", batch=B, q_len=q_len, heads=H, kv_heads=KVH, ctx=ctx,
                    offsets=prefix, table=_tables_from_counts(rng, nblk, nb), num_blocks=nb,
                    scaling="weak", note="B16 x 256-token chunks, prefix U[0,4096] block-aligned")
    if args.config == "c4":
        B, H, KVH = 4, 64, 8
        ctx = np.full(B, 131072, dtype=np.int64)
        nblk = ctx // BLOCK
        nb = int(nblk.sum() * 1.10) + 1
        return dict(kind="decode", batch=B, q_len=1, heads=H, kv_heads=KVH, ctx=ctx,
                    offsets=ctx - 1, table=_tables_from_counts(rng, nblk, nb), num_blocks=nb,
                    scaling="strong", note="B4 x 131072 context, 64 q / 8 KV heads")
    B, H, KVH, shared_blocks = 256, 32, 8, 128
    suffix = rng.integers(64, 1025, size=B)
    ctx = shared_blocks * BLOCK + suffix
    nsuf = (suffix + BLOCK - 1) // BLOCK
    nb = int((shared_blocks + nsuf.sum()) * 1.10) + 1
    shared = rng.choice(nb, size=shared_blocks, replace=False)
    table = _tables_from_counts(rng, nsuf, nb, shared=shared)
    return dict(kind="decode", batch=B, q_len=1, heads=H, kv_heads=KVH, ctx=ctx,
                offsets=ctx - 1, table=table, num_blocks=nb, scaling="strong",
                unique_tokens=int(shared_blocks * BLOCK + suffix.sum()),
                note="B256, 2048-token prefix on 128 shared blocks + private U[64,1024]")


def run_extra(args) -> None:
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    pkg = importlib.import_module(PACKAGE)
    pdist = importlib.import_module(f"{PACKAGE}.dist")
    from oracle.paged_oracle import decode_bytes, prefill_flops

    wl = extra_workload(args, world)
    B, H, KVH, q_len = wl["batch"], wl["heads"], wl["kv_heads"], wl["q_len"]
    shard = pdist.shard_heads(H, KVH, world, rank)
    kvh, qh = shard.kv_heads, shard.q_heads
    cache = pkg.PagedKVCache(1, wl["num_blocks"], BLOCK, kvh, HEAD_DIM, dtype=torch.bfloat16,
                             device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(2000 + rank)
    for t in (cache.key_cache, cache.value_cache):
        for i in range(0, t.shape[1], 4096):
            sl = t[:, i:i + 4096]
            sl.copy_(torch.randn(sl.shape, generator=g, device=dev))
    table = torch.from_numpy(wl["table"]).to(dev)
    ctx = torch.from_numpy(wl["ctx"]).to(dev)
    offs = torch.from_numpy(np.asarray(wl["offsets"], dtype=np.int64)).to(dev)
    q = torch.randn((B, qh, q_len, HEAD_DIM), generator=g, device=dev).to(torch.bfloat16)
    shape_new = (B, q_len, kvh, HEAD_DIM) if wl["kind"] == "prefill" else (B, kvh, HEAD_DIM)
    knew = torch.randn(shape_new, generator=g, device=dev).to(torch.bfloat16)
    vnew = torch.randn(shape_new, generator=g, device=dev).to(torch.bfloat16)
    attn = pkg.PagedAttention(qh, kvh, HEAD_DIM)
    head_major = torch.empty((qh, B, q_len, HEAD_DIM), dtype=torch.bfloat16, device=dev)
    out_view = head_major.permute(1, 0, 2, 3)
    peer = world > 1 and args.transport == "peer"
    gathered = (torch.empty((H, B, q_len, HEAD_DIM), dtype=torch.bfloat16, device=dev)
                if world > 1 and not peer else None)
    sharded = (pdist.ShardedPagedAttention(H, KVH, HEAD_DIM, transport="peer")
               if peer else None)

    def append():
        if wl["kind"] == "prefill":
            cache.write(0, table, offs, knew, vnew)
        else:
            cache.write_decode(0, table, offs, knew, vnew)

    def attention():
        if peer:
            sharded.forward(q, cache, 0, table, ctx, q_len)
        else:
            attn.forward_with_lse(q, cache, 0, table, ctx, q_len, want_lse=False, out=out_view)

    def step():
        append()
        attention()
        if gathered is not None:
            dist.all_gather_into_tensor(gathered, head_major)

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(max(args.warmup, 3)):
        step()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    sampler = ClockSampler(local)
    sampler.start()
    start.record()
    for _ in range(args.steps):
        step()
    end.record()
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    iters = max(20, min(KERNEL_ITERS, int(2000 / max(ms_step, 1e-3))))
    append_ms = kernel_loop_ms(append, dev, barrier, iters)
    attn_ms = kernel_loop_ms(attention, dev, barrier, iters)
    if rank == 0:
        line = {"config": args.config, "workload": wl["note"], "n_gpus": world,
                "exchange": (("combine fused with the all-gather (NVLink peer stores)" if peer
                              else "NCCL all-gather") if world > 1 else None),
                "scaling": wl["scaling"], "steps": args.steps, "ms_per_step": round(ms_step, 5),
                "append_ms": round(append_ms, 5), "attention_ms": round(attn_ms, 5),
                "clocks": clocks}
        if wl["kind"] == "prefill":
            flops = prefill_flops(wl["ctx"] - q_len, q_len, H, HEAD_DIM)
            app = B * q_len * KVH * HEAD_DIM * 2 * 4
            peak, peak_kind = 1590.0, "fallback"
            try:
                with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
                    peak, peak_kind = float(json.load(f)["bf16_tflops"]), "measured"
            except Exception:
                pass
            # The kernel the library picks for head_dim 128 (LLMOPT_B200_PREFILL).
            choice = os.environ.get("LLMOPT_B200_PREFILL", "") or "pair"
            kernel = {"tc": "prefill_tc_kernel (one SM, one query tile)",
                      "fa": "prefill_fa_kernel (one SM, two query tiles)"}.get(
                          choice, "prefill_pair_kernel (2-SM pairs, cta_group::2)")
            tf = flops / (attn_ms * 1e-3) / 1e12
            line.update({"metric": "chunked-prefill causal attention TFLOP/s", "unit": "TFLOP/s",
                         "value": round(tf, 1), "algorithmic_flops": int(flops),
                         "append_GBps": round(app / (append_ms * 1e-3) / 1e9, 1),
                         "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peak,
                                      "unit": "TFLOP/s", "frac": round(tf / peak, 4),
                                      "kernel": kernel,
                                      "peak_kind": f"{peak_kind} bf16_tflops (burst)"}})
        else:
            dec = decode_bytes(wl["ctx"], KVH, HEAD_DIM, 2, B, H, 2, 2, BLOCK)
            value = dec / (ms_step * 1e-3) / 1e9
            line.update({"metric": "paged-decode attn HBM GB/s (whole job)", "unit": "GB/s",
                         "value": round(value, 1), "decode_tok_s": round(B / (ms_step * 1e-3), 1),
                         "per_gpu_attention_GBps": round(
                             decode_bytes(wl["ctx"], kvh, HEAD_DIM, 2, B, qh, 2, 2, BLOCK)
                             / (attn_ms * 1e-3) / 1e9, 1)})
            if "unique_tokens" in wl:
                uniq = wl["unique_tokens"] * KVH * HEAD_DIM * 2 * 2
                line["unique_GBps"] = round(uniq / (ms_step * 1e-3) / 1e9, 1)
                line["l2_reuse_logical_over_unique"] = round(
                    int(wl["ctx"].sum()) / wl["unique_tokens"], 2)
        print(json.dumps(line), flush=True)
    if sharded is not None:
        sharded.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_rope(args) -> None:
    """Fused rotary + KV append (one kernel) against the same steps as the
    reference layer writes them (layers.py:106-134) in torch ops on the GPU
    followed by the KV write kernel.  Llama-3-8B heads, bf16, 500k rope base."""
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    pkg = importlib.import_module(PACKAGE)
    pdist = importlib.import_module(f"{PACKAGE}.dist")
    shard = pdist.shard_heads(HEADS, KV_HEADS, world, rank)
    qh, kvh, D = shard.q_heads, shard.kv_heads, HEAD_DIM
    rot = pkg.RotaryEmbedding(D, 16384, 500000.0, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(3000 + rank)
    peak, peak_kind = measured_hbm_peak()
    results = {}
    for name, B, q_len in (("prefill_chunk", 16, 256), ("decode", 64, 1)):
        rng = np.random.default_rng(args.seed + q_len)
        ctx0 = rng.integers(1024, 8192, size=B)
        width = (int(ctx0.max()) + q_len + BLOCK - 1) // BLOCK + 1
        nblk = B * width
        table = torch.from_numpy(rng.permutation(nblk).reshape(B, width).astype(np.int32)).to(dev)
        offs = torch.from_numpy(ctx0.astype(np.int64)).to(dev)
        pos = (offs[:, None] + torch.arange(q_len, device=dev)[None]).reshape(-1)
        T = B * q_len
        qp = torch.randn((T, qh * D), generator=g, device=dev).to(torch.bfloat16)
        kp = torch.randn((T, kvh * D), generator=g, device=dev).to(torch.bfloat16)
        vp = torch.randn((T, kvh * D), generator=g, device=dev).to(torch.bfloat16)
        cache = pkg.PagedKVCache(1, nblk, BLOCK, kvh, D, dtype=torch.bfloat16, device=dev)

        def fused():
            return pkg.rope_kv_append(qp, kp, vp, pos, rot, cache, 0, table, token_offsets=offs,
                                      q_len=q_len, num_heads=qh)

        def unfused():
            cos = rot.cos_cached[pos].to(torch.bfloat16).view(B, q_len, D).unsqueeze(1)
            sin = rot.sin_cached[pos].to(torch.bfloat16).view(B, q_len, D).unsqueeze(1)
            q = qp.view(B, q_len, qh, D).permute(0, 2, 1, 3)
            k = kp.view(B, q_len, kvh, D).permute(0, 2, 1, 3)
            v = vp.view(B, q_len, kvh, D).permute(0, 2, 1, 3)

            def rotate_half(x):
                return torch.cat((-x[..., D // 2:], x[..., :D // 2]), dim=-1)
            q = q * cos + rotate_half(q) * sin
            k = k * cos + rotate_half(k) * sin
            bk = k.permute(0, 2, 1, 3).contiguous()
            bv = v.permute(0, 2, 1, 3).contiguous()
            if q_len == 1:
                cache.write_decode(0, table, offs, bk[:, 0], bv[:, 0])
            else:
                cache.write(0, table, offs, bk, bv)
            return q

        def timed(fn, n):
            # Device time: the call is captured once in a CUDA graph and replayed,
            # so host launch overhead (which dominates the small decode shape)
            # is not measured for either path.
            for _ in range(max(args.warmup, 3)):
                fn()
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                fn()
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                fn()
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize(dev)
            if world > 1:
                dist.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(n):
                graph.replay()
            b.record()
            torch.cuda.synchronize(dev)
            del graph
            ms = a.elapsed_time(b) / n
            if world > 1:
                t = torch.tensor([ms], device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms = float(t.item())
            return ms

        sampler = ClockSampler(local)
        sampler.start()
        f_ms = timed(fused, args.steps)
        clocks = sampler.stop()
        u_ms = timed(unfused, max(args.steps // 4, 10))
        # Algorithmic bytes: q/k/v rows read, rotated q and the K/V cache rows written,
        # the two fp32 table rows read per token.
        nbytes = T * ((qh + 2 * kvh) * D * 2 * 2 + 2 * D * 4)
        results[name] = {"tokens_per_gpu": T, "fused_us": round(f_ms * 1e3, 2),
                         "unfused_torch_us": round(u_ms * 1e3, 2),
                         "speedup": round(u_ms / f_ms, 2),
                         "GBps_per_gpu": round(nbytes / (f_ms * 1e-3) / 1e9, 1),
                         "bytes_per_launch": int(nbytes), "clocks": clocks}
        del cache
        torch.cuda.empty_cache()
    if rank == 0:
        pre = results["prefill_chunk"]
        achieved = pre["GBps_per_gpu"]
        line = {"config": "rope", "metric": "fused rotary + KV append GB/s (whole job)",
                "unit": "GB/s", "value": round(achieved * world, 1), "n_gpus": world,
                "scaling": "weak", "steps": args.steps, "dtype": "bf16",
                "data": "synthetic: projections N(0,1) bf16, positions = offsets U[1024,8192) + "
                        "token index, random block tables",
                "workload": "Llama-3-8B heads (32 q / 8 KV, head_dim 128), rope base 500000; "
                            "value = 16 x 256-token prefill chunk",
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": round(achieved / peak, 4),
                             "kernel": "rope_append_kernel", "peak_kind": f"{peak_kind} hbm_gbs"},
                "shapes": results}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_step(args) -> None:
    """One Llama-3-8B decode step for 64 sequences on one GPU: DecodeStepState
    advance + fused rotary append + split-K attention + combine, captured once
    in a CUDA graph and replayed, against the same calls launched eagerly, and
    the host work the reference runner does per step to build the same
    metadata (model_runner.py:169-230: a Python loop over requests, torch.full
    of the table on the device, one copy per table row)."""
    import time

    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    pkg = importlib.import_module(PACKAGE)
    B, H, KVH, D = 64, HEADS, KV_HEADS, HEAD_DIM
    rng = np.random.default_rng(args.seed)
    ctx0 = rng.integers(1024, 8192, size=B)
    width = int((ctx0.max() + 4 * (args.steps + args.warmup) + 64) // BLOCK) + 2
    nblk = B * width
    perm = rng.permutation(nblk)
    blocks = {f"r{i}": [int(x) for x in perm[i * width:i * width + int(ctx0[i]) // BLOCK + 1]]
              for i in range(B)}
    used = {rid: len(b) for rid, b in blocks.items()}
    committed = {f"r{i}": int(ctx0[i]) for i in range(B)}
    cache = pkg.PagedKVCache(1, nblk, BLOCK, KVH, D, dtype=torch.bfloat16, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(4000)
    for t in (cache.key_cache, cache.value_cache):
        for i in range(0, t.shape[1], 4096):
            sl = t[:, i:i + 4096]
            sl.copy_(torch.randn(sl.shape, generator=g, device=dev) * 0.5)
    rot = pkg.RotaryEmbedding(D, 16384, 500000.0, device=dev)
    attn = pkg.PagedAttention(H, KVH, D)
    qp = torch.randn((B, H * D), generator=g, device=dev).to(torch.bfloat16)
    kp = torch.randn((B, KVH * D), generator=g, device=dev).to(torch.bfloat16)
    vp = torch.randn((B, KVH * D), generator=g, device=dev).to(torch.bfloat16)
    # capacity: the first step admits every sequence with all of its blocks
    state = pkg.DecodeStepState(B, width, device=dev, capacity=B * (width + 1))
    for rid in committed:
        state.admit(rid, blocks[rid], committed[rid])
    table, ctx, offs, pos = state.step()
    for rid in committed:
        committed[rid] += 1
    out = torch.empty((B, H, 1, D), dtype=torch.bfloat16, device=dev)

    def schedule():
        # host decisions of one step: a block for every sequence crossing into a new one
        for rid in committed:
            if committed[rid] // BLOCK >= used[rid]:
                state.append_block(rid, blocks_spare.pop())
                used[rid] += 1
            committed[rid] += 1
    taken = {x for b in blocks.values() for x in b}
    blocks_spare = [int(x) for x in perm if int(x) not in taken]

    def device_step():
        state.launch(batch=B)
        q = pkg.rope_kv_append(qp, kp, vp, pos, rot, cache, 0, table, token_offsets=offs,
                               q_len=1, num_heads=H)
        attn.forward_with_lse(q, cache, 0, table, ctx, 1, want_lse=False, out=out)

    stage_updates = state.stage

    steps = args.steps
    for _ in range(max(args.warmup, 3)):
        schedule()
        stage_updates()
        device_step()
    torch.cuda.synchronize(dev)
    # eager: host launches every kernel of every step
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    a.record()
    for _ in range(steps):
        schedule()
        stage_updates()
        device_step()
    b.record()
    torch.cuda.synchronize(dev)
    eager_wall = (time.perf_counter() - t0) / steps * 1e3
    eager_dev = a.elapsed_time(b) / steps
    # graph: one replay per step (the update count is read on the device)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        state._dev[0] = 0
        device_step()
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    for rid in committed:
        committed[rid] += 1
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        device_step()
    sampler = ClockSampler(0)
    sampler.start()
    t0 = time.perf_counter()
    a.record()
    for _ in range(steps):
        schedule()
        stage_updates()
        graph.replay()
    b.record()
    torch.cuda.synchronize(dev)
    graph_wall = (time.perf_counter() - t0) / steps * 1e3
    graph_dev = a.elapsed_time(b) / steps
    clocks = sampler.stop()
    del graph
    # the reference runner's per-step host metadata build, for the same batch
    reqs = list(committed)
    t0 = time.perf_counter()
    for _ in range(steps):
        w = max(len(v) for v in blocks.values())
        tab = torch.full((B, w), -1, dtype=torch.int32, device=dev)
        for row, rid in enumerate(reqs):
            tab[row, :len(blocks[rid])] = torch.tensor(blocks[rid], dtype=torch.int32)
        torch.tensor([committed[r] + 1 for r in reqs], dtype=torch.long, device=dev)
        torch.tensor([committed[r] for r in reqs], dtype=torch.long, device=dev)
        torch.cat([torch.tensor([committed[r]], dtype=torch.long) for r in reqs]).to(dev)
    torch.cuda.synchronize(dev)
    ref_meta = (time.perf_counter() - t0) / steps * 1e3
    ok = pkg._runtime.read_and_clear_errors(dev) == 0
    line = {"config": "step", "metric": "decode step latency (one layer), ms", "unit": "ms",
            "higher_is_better": False, "n_gpus": 1, "steps": steps, "dtype": "bf16",
            "workload": "Llama-3-8B heads, 64 sequences, context U[1024,8192): metadata advance + "
                        "fused rotary append + split-K attention + combine",
            "graph_replay_ms": round(graph_wall, 4), "graph_device_ms": round(graph_dev, 4),
            "eager_ms": round(eager_wall, 4), "eager_device_ms": round(eager_dev, 4),
            "reference_host_metadata_ms": round(ref_meta, 4), "device_errors_clear": ok,
            "clocks": clocks}
    print(json.dumps(line), flush=True)


def run_fp8(args) -> None:
    """Config-2 decode step over an FP8 (e4m3 + per-row scale) KV cache, one GPU,
    beside the same step over the bf16 cache: append (quantizing) + split-K
    decode + combine.  Bytes are the fp8 step's algorithmic bytes (codes, row
    scales, q, out, block table)."""
    import torch

    if int(os.environ.get("WORLD_SIZE", "1")) != 1:
        print(json.dumps({"config": "fp8", "skipped": "single-GPU line"}), flush=True)
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    pkg = importlib.import_module(PACKAGE)
    _lib = importlib.import_module(f"{PACKAGE}._lib")
    from oracle.paged_oracle import decode_bytes

    wl = make_workload(args, 1)
    B = wl["batch"]
    g = torch.Generator(device=dev)
    g.manual_seed(3000)
    table = torch.from_numpy(wl["table"]).to(dev)
    ctx = torch.from_numpy(wl["ctx"]).to(dev)
    offs = torch.from_numpy(wl["offsets"]).to(dev)
    q = (torch.randn((B, HEADS, 1, HEAD_DIM), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    knew = (torch.randn((B, KV_HEADS, HEAD_DIM), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    vnew = (torch.randn((B, KV_HEADS, HEAD_DIM), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    out = torch.empty((B, HEADS, 1, HEAD_DIM), dtype=torch.bfloat16, device=dev)
    attn = pkg.PagedAttention(HEADS, KV_HEADS, HEAD_DIM)
    ctx_np = wl["ctx"]
    lines = {}
    for name, dt in (("bf16", torch.bfloat16), ("fp8", torch.float8_e4m3fn)):
        cache = pkg.PagedKVCache(1, wl["num_blocks"], BLOCK, KV_HEADS, HEAD_DIM, dtype=dt,
                                 device=dev)
        for t in (cache.key_cache, cache.value_cache):
            for i in range(0, t.shape[1], 4096):
                sl = t[:, i:i + 4096]
                if dt == torch.bfloat16:
                    sl.copy_(torch.randn(sl.shape, generator=g, device=dev) * 0.5)
                else:   # finite codes (no NaN pattern), either sign
                    codes = torch.randint(0, 0x7E, sl.shape, generator=g, device=dev,
                                          dtype=torch.int32)
                    sign = torch.randint(0, 2, sl.shape, generator=g, device=dev,
                                         dtype=torch.int32) << 7
                    sl.view(torch.uint8).copy_((codes | sign).to(torch.uint8))
        if cache.is_fp8:
            for s in (cache.key_scale, cache.value_scale):
                s.copy_(torch.rand(s.shape, generator=g, device=dev) * (1.0 / 448) + 1e-4)

        def append():
            cache.write_decode(0, table, offs, knew, vnew)

        def decode():
            attn.forward_with_lse(q, cache, 0, table, ctx, 1, want_lse=False, out=out,
                                  phases=_lib.PHASE_SPLIT)

        def combine():
            attn.forward_with_lse(q, cache, 0, table, ctx, 1, want_lse=False, out=out,
                                  phases=_lib.PHASE_COMBINE)

        def step():
            append()
            decode()
            combine()

        def barrier():
            torch.cuda.synchronize(dev)

        for _ in range(max(args.warmup, 3)):
            step()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        sampler = ClockSampler(0)
        sampler.start()
        start.record()
        for _ in range(args.steps):
            step()
        end.record()
        torch.cuda.synchronize(dev)
        clocks = sampler.stop()
        append_ms = kernel_loop_ms(append, dev, barrier)
        decode_ms = kernel_loop_ms(decode, dev, barrier)
        combine_ms = kernel_loop_ms(combine, dev, barrier)
        ms_step = start.elapsed_time(end) / args.steps
        kv_bytes = 1 if cache.is_fp8 else 2
        dec = decode_bytes(ctx_np, KV_HEADS, HEAD_DIM, kv_bytes, B, HEADS, 2, 2, BLOCK)
        if cache.is_fp8:
            dec += int(ctx_np.sum()) * KV_HEADS * 2 * 4        # K and V row scales
        lines[name] = dict(
            ms_per_step=round(ms_step, 5), decode_tok_s=round(B / (ms_step * 1e-3), 1),
            bytes_per_step=int(dec), step_GBps=round(dec / (ms_step * 1e-3) / 1e9, 1),
            kernel_ms={"append": round(append_ms, 5), "decode_split": round(decode_ms, 5),
                       "combine": round(combine_ms, 5)},
            decode_kernel_GBps=round(dec / (decode_ms * 1e-3) / 1e9, 1), clocks=clocks)
        del cache
        torch.cuda.empty_cache()
    peak, peak_kind = measured_hbm_peak()
    f8 = lines["fp8"]
    print(json.dumps({
        "config": "fp8",
        "metric": "paged-decode step, e4m3 KV cache (codes + fp32 row scales), HBM GB/s",
        "unit": "GB/s", "value": f8["step_GBps"], "n_gpus": 1, "steps": args.steps,
        "workload": "config2 shape (B64, H32/KVH8, D128, ctx U[1024,8192]) decode step: "
                    "quantizing append + split-K decode + combine",
        "fp8": f8, "bf16": lines["bf16"],
        "speedup_vs_bf16_step": round(lines["bf16"]["ms_per_step"] / f8["ms_per_step"], 3),
        "roofline": {"bound": "hbm", "achieved": f8["decode_kernel_GBps"], "peak": peak,
                     "unit": "GB/s", "frac": round(f8["decode_kernel_GBps"] / peak, 4),
                     "kernel": "decode_fp8_kernel", "peak_kind": f"{peak_kind} hbm_gbs"},
    }), flush=True)


def run_quant(args) -> None:
    """QuantLinear.forward (fused dequantize-GEMM over packed 4-bit codes) on the
    Llama-3-8B MLP projections, beside what the reference's forward runs in the
    steady state: F.linear over its cached dense bf16 copy (a cuBLAS GEMM)."""
    import torch

    if int(os.environ.get("WORLD_SIZE", "1")) != 1:
        print(json.dumps({"config": "quant", "skipped": "single-GPU line"}), flush=True)
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    pkg = importlib.import_module(PACKAGE)
    from types import SimpleNamespace

    group, bits = 128, 4
    g = torch.Generator(device=dev)
    g.manual_seed(4000)
    peak, peak_kind = measured_hbm_peak()
    rows = []
    for (k, n) in ((4096, 14336), (14336, 4096)):
        # random codes / scales of the reference's layout (values do not matter
        # for timing; parity is the tests' job)
        qweight = torch.randint(0, 256, (n, k // 2), generator=g, device=dev,
                                dtype=torch.int32).to(torch.uint8)
        scales = (torch.rand((n, k // group), generator=g, device=dev) * 0.01 + 1e-3)
        zeros = torch.zeros_like(scales)
        qt = SimpleNamespace(qweight=qweight, scales=scales, zeros=zeros, bits=bits,
                             group_size=group, symmetric=True)
        lin = torch.nn.Linear(k, n, bias=False, device=dev, dtype=torch.bfloat16)
        layer = pkg.QuantLinear.from_float(lin, qt, compute_dtype=torch.bfloat16)
        dense = layer.dequantized_weight(dev)            # the reference's cached copy
        for m in (1, 16, 64):
            x = (torch.randn((m, k), generator=g, device=dev)).to(torch.bfloat16)
            # the packed weight (29 MB) fits in L2: flush it before every timed call
            flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

            def timed(fn, iters):
                # Replayed from a CUDA graph, so the events time the GPU work and
                # not the host's launch path; L2 flushed before every replay.
                for _ in range(max(args.warmup, 3)):
                    fn()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    fn()
                for _ in range(3):
                    graph.replay()
                evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                       for _ in range(iters)]
                for a, b in evs:
                    flush.zero_()
                    a.record()
                    graph.replay()
                    b.record()
                torch.cuda.synchronize(dev)
                del graph
                return statistics.median(a.elapsed_time(b) for a, b in evs)

            iters = max(10, min(args.steps, 50))
            ms_q = timed(lambda: layer(x), iters)
            ms_d = timed(lambda: torch.nn.functional.linear(x, dense), iters)
            # algorithmic bytes: packed codes + fp32 scales (symmetric: no zeros
            # are read) + the bf16 input and output rows
            wb = n * k * bits // 8 + 4 * n * (k // group) + 2 * m * (k + n)
            db = n * k * 2 + 2 * m * (k + n)
            rows.append({"k": k, "n": n, "tokens": m,
                         "quant_ms": round(ms_q, 5), "dense_bf16_ms": round(ms_d, 5),
                         "speedup_vs_dense": round(ms_d / ms_q, 3),
                         "quant_GBps": round(wb / (ms_q * 1e-3) / 1e9, 1),
                         "quant_frac_of_hbm": round(wb / (ms_q * 1e-3) / 1e9 / peak, 4),
                         "dense_GBps": round(db / (ms_d * 1e-3) / 1e9, 1),
                         "quant_TFLOPs": round(2 * m * n * k / (ms_q * 1e-3) / 1e12, 2)})
            del flush
    top = max(rows, key=lambda r: r["quant_frac_of_hbm"])
    print(json.dumps({
        "config": "quant",
        "metric": "QuantLinear.forward (int4, group 128, bf16) weight-stream GB/s",
        "unit": "GB/s", "value": top["quant_GBps"], "n_gpus": 1,
        "workload": "Llama-3-8B MLP projections (4096->14336, 14336->4096), 1/16/64 tokens; "
                    "each call replayed from a CUDA graph, L2 flushed before every replay; "
                    "median of CUDA-event times",
        "rows": rows,
        "roofline": {"bound": "hbm", "achieved": top["quant_GBps"], "peak": peak,
                     "unit": "GB/s", "frac": top["quant_frac_of_hbm"],
                     "kernel": "wq_gemm_acc_kernel", "peak_kind": f"{peak_kind} hbm_gbs"},
    }), flush=True)


def main(argv=None):
    args = parse_args(argv)
    if args.impl == "reference":
        run_reference(args)
    elif args.config == "step":
        run_step(args)
    elif args.config == "rope":
        run_rope(args)
    elif args.config == "fp8":
        run_fp8(args)
    elif args.config == "quant":
        run_quant(args)
    elif args.config != "c2":
        run_extra(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
