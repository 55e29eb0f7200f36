"""Seeded input builders for the golden parity cases.

Shared by ``make_golden.py`` (which feeds these inputs to the reference
implementation and records its outputs) and by the tests (which rebuild the same
inputs, check their checksum against the one recorded with the outputs, and run
the oracle or the CUDA library on them).  Everything is numpy: the GPU box has
no copy of the reference, only these builders and the committed outputs.

Storage kinds follow ``oracle.paged_oracle``: ``"f32"``, ``"f16"``, and
``"bf16"`` as uint16 bit patterns.
"""

from __future__ import annotations

import hashlib
import math

import numpy as np

from oracle.paged_oracle import from_f32


def checksum(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def _normal(rng: np.random.Generator, shape, scale: float = 1.0) -> np.ndarray:
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(scale)).astype(np.float32)


def _tables(rng, ctx, block_size, num_blocks, width=None, pad_extra=0):
    """Random block tables drawn without replacement from one permutation."""
    nblk = [-(-int(c) // block_size) for c in ctx]
    width = width if width is not None else max(max(nblk), 1) + pad_extra
    perm = rng.permutation(num_blocks)
    table = np.full((len(ctx), width), -1, dtype=np.int64)
    o = 0
    for s, n in enumerate(nblk):
        table[s, :n] = perm[o:o + n]
        o += n
    return table


def build_paged_case(seed: int, *, batch, heads, kv_heads, head_dim, block_size, ctx,
                     kv_kind, q_kind, q_len=1, value_scale=1.0, pool_extra=0.10,
                     num_blocks=None, width=None, holes=(), layers=1, layer=0):
    """A paged-attention input set: caches, tables, context lengths, query.

    ``holes`` is a list of ``(seq, column)`` table entries to overwrite with -1.
    Caches are filled everywhere (unused blocks too) so stray reads would show.
    """
    rng = np.random.default_rng(seed)
    ctx = np.asarray(ctx, dtype=np.int64)
    nblk_total = int(sum(-(-int(c) // block_size) for c in ctx))
    if num_blocks is None:
        num_blocks = max(int(nblk_total * (1 + pool_extra)) + 1, 1)
    table = _tables(rng, ctx, block_size, num_blocks, width=width)
    for s, c in holes:
        table[s, c] = -1
    shape = (layers, num_blocks, block_size, kv_heads, head_dim)
    k = from_f32(_normal(rng, shape, value_scale), kv_kind)
    v = from_f32(_normal(rng, shape, value_scale), kv_kind)
    q = from_f32(_normal(rng, (batch, heads, q_len, head_dim), value_scale), q_kind)
    return dict(
        key_cache=k, value_cache=v, block_ids=table, context_lens=ctx, query=q,
        kv_kind=kv_kind, q_kind=q_kind, heads=heads, kv_heads=kv_heads, head_dim=head_dim,
        block_size=block_size, q_len=q_len, layer=layer,
    )


def paged_checksum(case: dict) -> str:
    return checksum(case["key_cache"], case["value_cache"], case["block_ids"],
                    case["context_lens"], case["query"])


# ---------------------------------------------------------------------------
# named cases (regenerated from seeds; outputs recorded by make_golden.py)
# ---------------------------------------------------------------------------

def case_c1(seed: int = 0) -> dict:
    """B8, H8/KVH2, D64, bs16, fp32, ctx U{16..512}, pool 512."""
    rng = np.random.default_rng(seed + 1000)
    ctx = rng.integers(16, 513, size=8)
    return build_paged_case(seed, batch=8, heads=8, kv_heads=2, head_dim=64, block_size=16,
                            ctx=ctx, kv_kind="f32", q_kind="f32", num_blocks=512)


def case_c1_splits(case: dict) -> int:
    """``split_size`` giving 4 chunks of the longest context (config 1's split run)."""
    return int(math.ceil(int(np.max(case["context_lens"])) / 4))


def case_bf16_decode(seed: int = 1) -> dict:
    """Llama-3-8B head shape, ragged edge lengths (1, 15, 16, 17, 300, 1000)."""
    return build_paged_case(seed, batch=6, heads=32, kv_heads=8, head_dim=128, block_size=16,
                            ctx=[1, 15, 16, 17, 300, 1000], kv_kind="bf16", q_kind="bf16",
                            value_scale=0.5, width=70)


def case_bf16_prefill(seed: int = 2) -> dict:
    """Chunked prefill: q_len 40 over prefixes 0, 160 and an unaligned 37."""
    prefix = np.array([0, 160, 37])
    q_len = 40
    return build_paged_case(seed, batch=3, heads=8, kv_heads=2, head_dim=128, block_size=16,
                            ctx=prefix + q_len, kv_kind="bf16", q_kind="bf16", q_len=q_len)


def case_edge_f32(seed: int = 3, q_len: int = 1) -> dict:
    """fp32, group 4, D16, bs4: an empty sequence, ctx 1 < q_len, and a -1 hole."""
    return build_paged_case(seed, batch=4, heads=4, kv_heads=1, head_dim=16, block_size=4,
                            ctx=[0, 1, 7, 13], kv_kind="f32", q_kind="f32", q_len=q_len,
                            holes=[(3, 1)], width=6)


def case_mixed_q(seed: int = 4) -> dict:
    """fp32 query over a bf16 cache (the tiny engine's combination), D16, group 2."""
    return build_paged_case(seed, batch=3, heads=4, kv_heads=2, head_dim=16, block_size=16,
                            ctx=[5, 33, 64], kv_kind="bf16", q_kind="f32", layers=2, layer=1)


def case_f16_decode(seed: int = 5) -> dict:
    """fp16 cache and query, D64, group 8, block_size 8."""
    return build_paged_case(seed, batch=3, heads=16, kv_heads=2, head_dim=64, block_size=8,
                            ctx=[9, 64, 129], kv_kind="f16", q_kind="f16")


def case_bf16_decode_d256(seed: int = 6) -> dict:
    """head_dim 256 (the largest the tensor-core decode takes), group 4."""
    return build_paged_case(seed, batch=4, heads=8, kv_heads=2, head_dim=256, block_size=16,
                            ctx=[3, 64, 250, 511], kv_kind="bf16", q_kind="bf16",
                            value_scale=0.5)


def case_f16_prefill(seed: int = 7) -> dict:
    """fp16 chunked prefill on the tensor-core path: q_len 24 x group 4 = 96 rows,
    prefixes 40 (unaligned) and 100."""
    prefix = np.array([40, 100])
    q_len = 24
    return build_paged_case(seed, batch=2, heads=8, kv_heads=2, head_dim=128, block_size=16,
                            ctx=prefix + q_len, kv_kind="f16", q_kind="f16", q_len=q_len,
                            value_scale=0.5)


ATTENTION_CASES = {
    "c1": case_c1,
    "bf16_decode": case_bf16_decode,
    "bf16_prefill": case_bf16_prefill,
    "edge_f32_q1": lambda: case_edge_f32(q_len=1),
    "edge_f32_q3": lambda: case_edge_f32(q_len=3),
    "mixed_q": case_mixed_q,
    "f16_decode": case_f16_decode,
    "bf16_decode_d256": case_bf16_decode_d256,
    "f16_prefill": case_f16_prefill,
}

#: (name, softcap, split_kv, split_size or None for the case default) runs recorded per case.
ATTENTION_RUNS = {
    "c1": [("dense", 0.0, False, 512), ("split4", 0.0, True, "c1_split")],
    "bf16_decode": [("dense", 0.0, False, 512), ("split", 0.0, True, 64)],
    "bf16_prefill": [("dense", 0.0, False, 512), ("split", 0.0, True, 40)],
    "edge_f32_q1": [("dense", 0.0, False, 512), ("split", 0.0, True, 3), ("softcap", 5.0, True, 5)],
    "edge_f32_q3": [("dense", 0.0, False, 512), ("split", 0.0, True, 3), ("softcap", 5.0, False, 512)],
    "mixed_q": [("dense", 0.0, False, 512), ("split", 0.0, True, 16)],
    "f16_decode": [("dense", 0.0, False, 512), ("split", 2.5, True, 24)],
    "bf16_decode_d256": [("dense", 0.0, False, 512), ("split", 0.0, True, 64)],
    "f16_prefill": [("dense", 0.0, False, 512), ("split", 0.0, True, 32)],
}


# ---------------------------------------------------------------------------
# KV append cases (bit-exact)
# ---------------------------------------------------------------------------

def _special_values(rng, shape) -> np.ndarray:
    """Normal values salted with RNE ties, subnormals, infinities and extremes."""
    x = _normal(rng, shape, 3.0).reshape(-1)
    specials = np.array([
        1.00390625, -1.00390625, 1.01171875, 3.0e-39, -1.0e-40, 1.0e-45, np.inf, -np.inf,
        3.3961776e38, -3.3961776e38, 65504.0, 65520.0, 6.0e-8, 0.0, -0.0, 2.0 ** -14,
    ], dtype=np.float32)
    idx = rng.choice(x.size, size=min(x.size, 4 * specials.size), replace=False)
    x[idx] = np.resize(specials, idx.size)
    return x.reshape(shape)


def case_write(seed: int = 10, in_kind: str = "f32", kv_kind: str = "bf16") -> dict:
    """``PagedKVCache.write``: q_len 11 over blocks of 4, odd offsets, a -1 stop."""
    rng = np.random.default_rng(seed)
    B, q_len, kvh, d, bs, nb = 4, 11, 2, 8, 4, 40
    table = np.full((B, 7), -1, dtype=np.int64)
    perm = rng.permutation(nb)
    table[0, :4] = perm[0:4]          # offset 3: crosses 3 block boundaries
    table[1, :6] = perm[4:10]         # offset 13: starts in column 3
    table[2, :2] = perm[10:12]        # -1 at column 2 stops the walk after 8 - 5 = 3 rows
    table[3, :7] = perm[12:19]        # offset 0
    offsets = np.array([3, 13, 5, 0], dtype=np.int64)
    keys = from_f32(_special_values(rng, (B, q_len, kvh, d)), in_kind)
    values = from_f32(_special_values(rng, (B, q_len, kvh, d)), in_kind)
    shape = (2, nb, bs, kvh, d)
    kc = from_f32(_normal(rng, shape), kv_kind)
    vc = from_f32(_normal(rng, shape), kv_kind)
    return dict(key_cache=kc, value_cache=vc, block_ids=table, token_offsets=offsets,
                keys=keys, values=values, in_kind=in_kind, kv_kind=kv_kind, layer=1)


def case_write_decode(seed: int = 11, in_kind: str = "f32", kv_kind: str = "bf16") -> dict:
    """``PagedKVCache.write_decode``: includes a -1 and an out-of-range id (both go to
    block 0, the reference's behaviour) and a negative offset (wraps to the last column)."""
    rng = np.random.default_rng(seed)
    B, kvh, d, bs, nb = 6, 2, 16, 8, 30
    table = np.full((B, 5), -1, dtype=np.int64)
    perm = rng.permutation(nb)
    for s in range(B):
        table[s] = perm[(5 * s) % 25:(5 * s) % 25 + 5]
    table[2, 1] = -1
    table[3, 0] = nb + 7
    offsets = np.array([0, 7, 9, 3, 39, -1], dtype=np.int64)
    keys = from_f32(_special_values(rng, (B, kvh, d)), in_kind)
    values = from_f32(_special_values(rng, (B, kvh, d)), in_kind)
    shape = (1, nb, bs, kvh, d)
    kc = from_f32(_normal(rng, shape), kv_kind)
    vc = from_f32(_normal(rng, shape), kv_kind)
    return dict(key_cache=kc, value_cache=vc, block_ids=table, token_offsets=offsets,
                keys=keys, values=values, in_kind=in_kind, kv_kind=kv_kind, layer=0)


WRITE_CASES = {
    "write_f32_to_bf16": lambda: case_write(in_kind="f32", kv_kind="bf16"),
    "write_bf16_to_bf16": lambda: case_write(seed=12, in_kind="bf16", kv_kind="bf16"),
    "write_f32_to_f16": lambda: case_write(seed=13, in_kind="f32", kv_kind="f16"),
    "write_f32_to_f32": lambda: case_write(seed=14, in_kind="f32", kv_kind="f32"),
    "write_decode_f32_to_bf16": lambda: case_write_decode(in_kind="f32", kv_kind="bf16"),
    "write_decode_f16_to_bf16": lambda: case_write_decode(seed=15, in_kind="f16", kv_kind="bf16"),
    "write_decode_bf16_to_f32": lambda: case_write_decode(seed=16, in_kind="bf16", kv_kind="f32"),
}


# ---------------------------------------------------------------------------
# Rotary embedding + KV append cases (bit-exact)
# ---------------------------------------------------------------------------

def case_rope(seed: int = 30, model_kind: str = "bf16", kv_kind: str = "bf16", q_len: int = 1,
              heads: int = 8, kv_heads: int = 2, head_dim: int = 64, max_pos: int = 96,
              base: float = 10000.0) -> dict:
    """The rotary + append step of the attention layer.  Decode (q_len 1) uses
    write_decode with a -1 entry (redirected to block 0) and a negative offset;
    chunks use write with odd offsets and a -1 that stops a sequence's walk.
    Positions include 0 and the last table row."""
    rng = np.random.default_rng(seed)
    bs = 8
    if q_len == 1:
        seq, width, nb = 6, 5, 32
        table = np.full((seq, width), -1, dtype=np.int64)
        perm = rng.permutation(nb)
        for s in range(seq):
            table[s] = perm[(5 * s) % 27:(5 * s) % 27 + 5]
        table[2, 1] = -1
        offsets = np.array([0, 7, 9, 3, 33, -1], dtype=np.int64)
        positions = np.array([0, 7, max_pos - 1, 3, 33, 50], dtype=np.int64)
    else:
        seq, width, nb = 3, 6, 30
        table = np.full((seq, width), -1, dtype=np.int64)
        perm = rng.permutation(nb)
        table[0, :4] = perm[0:4]
        table[1, :6] = perm[4:10]
        table[2, :2] = perm[10:12]               # -1 at column 2 stops the walk
        offsets = np.array([3, 13, 5], dtype=np.int64)
        positions = np.concatenate([off + np.arange(q_len) for off in offsets]).astype(np.int64)
        positions[-1] = max_pos - 1
    T = seq * q_len
    q_proj = from_f32(_normal(rng, (T, heads * head_dim), 2.0), model_kind)
    k_proj = from_f32(_normal(rng, (T, kv_heads * head_dim), 2.0), model_kind)
    v_proj = from_f32(_normal(rng, (T, kv_heads * head_dim), 2.0), model_kind)
    shape = (2, nb, bs, kv_heads, head_dim)
    kc = from_f32(_normal(rng, shape), kv_kind)
    vc = from_f32(_normal(rng, shape), kv_kind)
    return dict(q_proj=q_proj, k_proj=k_proj, v_proj=v_proj, positions=positions,
                key_cache=kc, value_cache=vc, block_ids=table, token_offsets=offsets,
                model_kind=model_kind, kv_kind=kv_kind, layer=1, seq=seq, q_len=q_len,
                heads=heads, kv_heads=kv_heads, head_dim=head_dim, max_pos=max_pos, base=base)


ROPE_CASES = {
    "rope_decode_bf16": lambda: case_rope(),
    "rope_chunk_bf16": lambda: case_rope(seed=31, q_len=11, heads=4, kv_heads=2, head_dim=32),
    "rope_chunk_f32_to_bf16": lambda: case_rope(seed=32, model_kind="f32", q_len=7, heads=6,
                                                kv_heads=3, head_dim=16),
    "rope_decode_f16_to_f32": lambda: case_rope(seed=33, model_kind="f16", kv_kind="f32",
                                                head_dim=128, heads=4, kv_heads=1),
}


def rope_checksum(case: dict) -> str:
    return checksum(case["q_proj"], case["k_proj"], case["v_proj"], case["positions"],
                    case["key_cache"], case["value_cache"], case["block_ids"],
                    case["token_offsets"])


# ---------------------------------------------------------------------------
# Decode-step metadata scenario (requests joining, growing, leaving)
# ---------------------------------------------------------------------------

STEP_BLOCK_SIZE = 16
STEP_SCRIPT = {
    0: [("admit", "a", 30), ("admit", "b", 16), ("admit", "c", 5)],
    3: [("release", "b"), ("admit", "d", 47)],
    5: [("release", "a")],
    6: [("admit", "e", 1), ("admit", "f", 63), ("admit", "g", 15)],
    9: [("release", "c"), ("release", "f")],
    11: [("admit", "h", 200)],
}
STEP_COUNT = 14


def step_scenario():
    """Yields, per decode step, (events, committed, block_map): the scheduling
    events of the step (('admit', id, blocks, committed), ('append', id, block),
    ('release', id)) and the state the reference's runner reads for it: the
    committed tokens and block ids of every running request, in admission
    order.  A request's blocks always cover the position its next token
    takes; block ids come from a counter."""
    bs = STEP_BLOCK_SIZE
    next_block = [0]
    committed: dict = {}
    blocks: dict = {}

    def take(n):
        out = list(range(next_block[0], next_block[0] + n))
        next_block[0] += n
        return out

    for step in range(STEP_COUNT):
        events = []
        for ev in STEP_SCRIPT.get(step, []):
            if ev[0] == "release":
                committed.pop(ev[1])
                blocks.pop(ev[1])
                events.append(("release", ev[1]))
        for ev in STEP_SCRIPT.get(step, []):
            if ev[0] == "admit":
                rid, n = ev[1], ev[2]
                committed[rid] = n
                blocks[rid] = take(n // bs + 1)
                events.append(("admit", rid, list(blocks[rid]), n))
        for rid in committed:
            if committed[rid] // bs >= len(blocks[rid]):
                b = take(1)[0]
                blocks[rid].append(b)
                events.append(("append", rid, b))
        yield events, dict(committed), {k: list(v) for k, v in blocks.items()}
        for rid in committed:
            committed[rid] += 1


def write_checksum(case: dict) -> str:
    return checksum(case["key_cache"], case["value_cache"], case["block_ids"],
                    case["token_offsets"], case["keys"], case["values"])


def case_merge(seed: int = 20) -> dict:
    """``merge_states`` inputs: [2, 3, 5, 16] partials with some -inf LSEs."""
    rng = np.random.default_rng(seed)
    o1 = _normal(rng, (2, 3, 5, 16))
    o2 = _normal(rng, (2, 3, 5, 16))
    l1 = _normal(rng, (2, 3, 5), 4.0)
    l2 = _normal(rng, (2, 3, 5), 4.0)
    l1[0, 0, :2] = -np.inf
    l2[0, 0, 1:3] = -np.inf
    l1[1, 2, 4] = -np.inf
    l2[1, 2, 4] = -np.inf
    return dict(o1=o1, o2=o2, l1=l1, l2=l2)


# ---------------------------------------------------------------------------
# Weight-only quantized linear (QuantLinear over RTN / GPTQ packed weights)
# ---------------------------------------------------------------------------

def case_quant(seed: int, *, out_features: int, in_features: int, bits: int, group: int,
               symmetric: bool, m: int, bias: bool = True, kind: str = "f32",
               strategy: str = "rtn", calib: int = 0) -> dict:
    """A linear layer's float weight, bias and input, plus (for GPTQ) the
    calibration activations whose second moment drives the quantizer."""
    rng = np.random.default_rng(seed)
    w = _normal(rng, (out_features, in_features), 0.05)
    w[0, :group] *= 8.0                         # one outlier group
    b = _normal(rng, (out_features,), 0.1) if bias else None
    x = _normal(rng, (m, in_features))
    xc = _normal(rng, (calib, in_features)) if calib else None
    return dict(weight=w, bias=b, x=from_f32(x, kind), x_kind=kind, bits=bits, group=group,
                symmetric=symmetric, strategy=strategy, calib=xc,
                shape=(out_features, in_features))


QUANT_CASES = {
    "quant_rtn4_sym_g64": lambda: case_quant(40, out_features=48, in_features=256, bits=4,
                                             group=64, symmetric=True, m=5),
    "quant_rtn4_asym_g128": lambda: case_quant(41, out_features=40, in_features=256, bits=4,
                                               group=128, symmetric=False, m=3),
    "quant_rtn8_sym_g64": lambda: case_quant(42, out_features=32, in_features=128, bits=8,
                                             group=64, symmetric=True, m=4, bias=False),
    "quant_rtn8_asym_g32": lambda: case_quant(43, out_features=24, in_features=128, bits=8,
                                              group=32, symmetric=False, m=2),
    "quant_rtn2_sym_g32": lambda: case_quant(44, out_features=16, in_features=128, bits=2,
                                             group=32, symmetric=True, m=3),
    "quant_gptq4_sym_g64": lambda: case_quant(45, out_features=32, in_features=128, bits=4,
                                              group=64, symmetric=True, m=4, strategy="gptq",
                                              calib=64),
    "quant_rtn4_sym_g64_bf16": lambda: case_quant(46, out_features=64, in_features=256, bits=4,
                                                  group=64, symmetric=True, m=6, kind="bf16"),
    "quant_rtn4_asym_g64_f16": lambda: case_quant(47, out_features=64, in_features=192, bits=4,
                                                  group=64, symmetric=False, m=3, kind="f16"),
    # one group per row (the quantizers take group_size = in_features)
    "quant_rtn4_asym_row_bf16": lambda: case_quant(48, out_features=64, in_features=256, bits=4,
                                                   group=256, symmetric=False, m=9, kind="bf16"),
    "quant_gptq4_asym_g128_bf16": lambda: case_quant(49, out_features=64, in_features=256,
                                                     bits=4, group=128, symmetric=False, m=5,
                                                     kind="bf16", strategy="gptq", calib=96),
    "quant_rtn2_asym_g64_f16": lambda: case_quant(50, out_features=64, in_features=256, bits=2,
                                                  group=64, symmetric=False, m=7, kind="f16"),
    "quant_rtn8_sym_g128_bf16": lambda: case_quant(51, out_features=64, in_features=256, bits=8,
                                                   group=128, symmetric=True, m=33, kind="bf16"),
}
