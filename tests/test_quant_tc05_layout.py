"""CPU restatement of ``wq_gemm_tc05_kernel`` (csrc/quant_linear.cu).

The tcgen05 quantized-linear kernel is checked on the CPU in three parts, with
its constants read from the kernel source:

* the dequantization arithmetic: the 2^23 magic with the nibble left in place
  (2^23 + q * 16^j), one fused multiply-add by (16^-j, -(2^(23-4j) + c)), the
  zero-point subtraction and the scale multiply in float32, then the rounding
  to the compute dtype - bit for bit against the oracle's ``(q - z) * s``
  (the reference's dequantization) over random code words, scales of every
  magnitude and fractional zero points;
* the data path of whole CTAs: the codes box as the TMA writes it with the
  128-byte swizzle, each thread's chunk reads, the per-slice group constants
  the codes warp stages, the A operand (its swizzled shared-memory tile, or
  its tensor-memory columns), the token
  boxes as the MMA reads them through the K-major 128-byte-swizzle rule, the
  split of the k range, the accumulation and the output / split partials
  (summed in split order with the bias) - against the oracle's
  ``x @ W^T + b``, and the host's split count;
* the mbarrier protocol as a randomized interleaving of the codes loader,
  the token loader, the MMA issuer (with asynchronous MMA completion) and the
  dequantize warps: every wait must end, every consumer must find the slice
  it expects in its slot, no slot may be rewritten while an MMA still reads
  it, and no waiter may fall two phases behind a barrier.

The model takes a warp's shared-memory reads as done when it reads; the
kernel therefore releases a codes stage only after its math has consumed
them (an arrival right after the loads let the codes warp refill the stage
under loads still in flight).  ``test_release_follows_the_math`` checks that
order in the source.

This does not run the kernel.
"""

from __future__ import annotations

import os
import random
import re

import numpy as np
import pytest

from conftest import REPO
from oracle import paged_oracle as po
from oracle import quant_oracle as qo

SRC = os.path.join(REPO, "quantized-llm-inference-engine-_b200", "csrc", "quant_linear.cu")


def _constants():
    text = open(SRC).read()
    body = text[text.index("namespace tc05 {"):text.index("}  // namespace tc05")]
    env = {}
    for name, expr in re.findall(r"constexpr (?:int|uint32_t|bool) (\w+) = ([^;]+);", body):
        expr = re.sub(r"\(int\)", "", expr).replace("/", "//")
        expr = expr.replace("false", "False").replace("true", "True")
        # C conditionals: (a ? b : c) and a ? b : c
        expr = re.sub(r"\(([^()?]+)\?([^():]+):([^()]+)\)", r"((\2) if (\1) else (\3))", expr)
        m = re.fullmatch(r"([^?]+)\?([^:]+):(.+)", expr)
        if m:
            expr = "((%s) if (%s) else (%s))" % (m.group(2), m.group(1), m.group(3))
        env[name] = eval(expr, {}, dict(env))
    return env


C = _constants()
BM, SLICE, STAGE = C["kBM"], C["kSliceK"], C["kStageK"]
SLICE_COLS, XBOXES, WORDS, QUARTERS = C["kSliceCols"], C["kXBoxes"], C["kWords"], C["kQuarters"]
SPS, CODE_STAGES, ASLOTS, MAX_XSLOTS = C["kSlicesPerStage"], C["kCodeStages"], C["kASlots"], C["kMaxXSlots"]
DQ_WARPS, SETS, MAX_BN, XBYTES = C["kDqWarps"], C["kSets"], C["kMaxBN"], C["kXBytes"]
ACC_COL, TMEM_COLS, SLOTS_PER_SET = C["kAccCol"], C["kTmemCols"], C["kSlotsPerSet"]
A_IN_SMEM = C["kAInSmem"]


def a_slot(s):
    """A slot of slice s (the kernel's a_slot): each set owns its slots."""
    return (s % SETS) * SLOTS_PER_SET + (s // SETS) % SLOTS_PER_SET


def a_use(s):
    """How many times slice s's slot was used before it (a_use)."""
    return s // SETS // SLOTS_PER_SET


def bn_of(m):
    return MAX_BN if m >= MAX_BN else (m + 15) & ~15


def x_slots(bn):
    return min(MAX_XSLOTS, XBYTES // (bn * 128 * XBOXES))


def test_constants_fit():
    assert STAGE % SLICE == 0 and SLICE % 64 == 0
    assert ACC_COL + MAX_BN <= TMEM_COLS and TMEM_COLS in (32, 64, 128, 256, 512)
    assert ASLOTS == SETS * SLOTS_PER_SET
    assert A_IN_SMEM or ASLOTS * SLICE_COLS <= ACC_COL
    # every set has a slice in each full stage (one codes_empty arrival per
    # warp per stage: at the set's last slice there)
    assert DQ_WARPS % 4 == 0 and SETS <= SPS and SLOTS_PER_SET >= 1
    for bn in range(16, MAX_BN + 1, 16):
        assert 2 <= x_slots(bn) <= MAX_XSLOTS
        assert x_slots(bn) * bn * 128 * XBOXES <= XBYTES
        assert (bn * 128) % 1024 == 0        # every token box starts on a swizzle atom
    smem = C["kSmem"]
    assert smem <= 227 * 1024
    for off in ("kOffCodes", "kOffA", "kOffX", "kOffS", "kOffZ", "kOffBar"):
        assert C[off] % 1024 == 0
    assert C["kOffBar"] + C["kBarBytes"] + 1024 == smem


def test_host_boxes_match_the_kernel():
    """The launch's tensor maps: codes boxes of 128 bytes x kBM rows, token
    boxes of 64 columns (the 128-byte swizzle span) x bn rows."""
    text = open(SRC).read()
    call = text[text.index("if (!tensor_map_2d(&tm_codes"):]
    call = call[:call.index("return cudaErrorInvalidValue")]
    codes_args = re.search(r"tensor_map_2d\(&tm_codes,([^;]*?)\) \|\|", call, re.S).group(1)
    x_args = re.search(r"tensor_map_2d\(&tm_x,([^;]*?)\)\) \{", call, re.S).group(1)
    codes_box = [t.strip() for t in codes_args.split(",")][-2:]
    x_box = [t.strip() for t in x_args.split(",")][-2:]
    assert codes_box == ["128", "tc05::kBM"], codes_box
    assert x_box[0] == "64" and "tokens" in x_box[1], x_box


def test_release_follows_the_math():
    """The dequantize warps arrive on codes_empty inside the store loop, after
    the dequant8 calls that consume the stage's words and constants."""
    text = open(SRC).read()
    body = text[text.index("// ---- dequantize (warps 0 .. kDqWarps - 1) ----"):]
    body = body[:body.index("// ---- epilogue")]
    first_math = body.index("dequant8<DT, SYM>(")
    release = body.index("mbar_arrive(&bars->codes_empty[cs])")
    assert body.count("mbar_arrive(&bars->codes_empty[cs])") == 1
    assert first_math < release


# ---- dequantization arithmetic --------------------------------------------------

def kernel_dequant(words, scale, zero, bits, sym, kind):
    """dequant8 for arrays of code words (uint32) and per-word scale / zero:
    returns [n, 8] 16-bit patterns in code order."""
    w = np.asarray(words, np.uint32)
    u = w >> np.uint32(16)
    zc = float(1 << (bits - 1)) if sym else 0.0
    outs = []
    for j in range(8):
        src = w if j < 4 else u
        jj = j % 4
        bits_v = np.uint32(0x4B000000) | (src & np.uint32(0xF << (4 * jj)))
        v = bits_v.view(np.float32).astype(np.float64)
        mult = 16.0 ** -jj
        add = -(2.0 ** (23 - 4 * jj) + zc)
        exact = v * mult + add                    # one fused multiply-add, exact
        d = exact.astype(np.float32)
        assert (d.astype(np.float64) == exact).all()
        if not sym:
            d = (d + (-np.asarray(zero, np.float32))).astype(np.float32)
        d = (d * np.asarray(scale, np.float32)).astype(np.float32)
        outs.append(po.from_f32(d, kind))
    return np.stack(outs, axis=1)


def oracle_dequant(words, scale, zero, bits, sym, kind):
    w = np.asarray(words, np.uint32)
    q = np.stack([(w >> np.uint32(4 * j)) & np.uint32(0xF) for j in range(8)], axis=1)
    n = q.shape[0]
    return qo.dequantize_codes(q.reshape(n, 8), np.asarray(scale, np.float32).reshape(n, 1),
                               np.asarray(zero, np.float32).reshape(n, 1), bits, 8, kind, sym)


@pytest.mark.parametrize("kind", ["bf16", "f16"])
@pytest.mark.parametrize("bits,sym", [(4, True), (4, False), (2, True), (2, False)])
def test_dequant_bit_exact(kind, bits, sym):
    rng = np.random.default_rng(bits * 10 + sym + (kind == "f16"))
    n = 20000
    nib = rng.integers(0, 1 << bits, size=(n, 8), dtype=np.uint32)
    words = np.zeros(n, np.uint32)
    for j in range(8):
        words |= nib[:, j] << np.uint32(4 * j)
    mags = [1e-3, 0.02, 0.7, 3.0, 1e-30, 1e30, 2.0 ** -120, 6e-5, 60000.0]
    scale = (rng.choice(mags, n) * rng.uniform(0.5, 2.0, n) *
             rng.choice([1.0, -1.0], n)).astype(np.float32)
    if sym:
        zero = np.zeros(n, np.float32)
    else:
        zero = np.where(rng.random(n) < 0.5, rng.integers(0, 1 << bits, n).astype(np.float32),
                        rng.uniform(-2.0, (1 << bits) + 2.0, n)).astype(np.float32)
    with np.errstate(over="ignore", under="ignore", invalid="ignore"):
        got = kernel_dequant(words, scale, zero, bits, sym, kind)
        want = oracle_dequant(words, scale, zero, bits, sym, kind)
    assert got.dtype == want.dtype
    assert np.array_equal(got.view(np.uint16), want.view(np.uint16))


# ---- data path of whole CTAs ----------------------------------------------------

def sw128_read(tile, rows, kk):
    """The MMA's view of a K-major 128-byte-swizzled tile for the K = 16 step kk
    (start address + 32 kk): [rows, 16] 16-bit patterns."""
    out = np.zeros((rows, 16), np.int64)
    for i in range(rows):
        for e in range(16):
            logical = kk * 32 + 2 * e
            chunk = logical // 16
            phys = (i // 8) * 1024 + (i % 8) * 128 + 16 * (chunk ^ (i % 8)) + logical % 16
            out[i, e] = int(tile[phys]) | int(tile[phys + 1]) << 8
    return out


def tma_box_sw128(src_rows, x0, y0, inner_bytes, rows):
    """A TMA box of `rows` x 128 bytes at byte column x0, row y0 of a 2-D byte
    tensor [outer, inner_bytes], 128-byte swizzle, zero outside the tensor."""
    tile = np.zeros(rows * 128, np.int64)
    outer = src_rows.shape[0]
    for i in range(rows):
        for c in range(8):
            for b in range(16):
                col = x0 + 16 * c + b
                v = 0
                if y0 + i < outer and col < inner_bytes:
                    v = int(src_rows[y0 + i, col])
                tile[(i // 8) * 1024 + (i % 8) * 128 + 16 * (c ^ (i % 8)) + b] = v
    return tile


def bf16_value(bits16):
    return po.to_f32(np.asarray(bits16, np.uint16), "bf16").astype(np.float64)


def run_segment(qw, scales, zeros, x_bytes, a, rbase, m0, kb, length):
    """One segment's accumulator [BM, bn], as the CTA's roles build it."""
    n, k, m, group, sym, bits = a["n"], a["k"], a["m"], a["group"], a["sym"], a["bits"]
    bn = bn_of(m)
    groups = k // group
    acc = np.zeros((BM, bn))
    for st in range((length + SPS - 1) // SPS):
        c0 = kb + st * STAGE
        in_stage = min(SPS, length - st * SPS)
        codes = tma_box_sw128(qw, c0 // 2, rbase, k // 2, BM)
        # group constants the codes warp stages: [slice][32 columns][row]
        sst = np.full(SPS * QUARTERS * BM, np.nan, np.float32)
        zst = np.full(SPS * QUARTERS * BM, np.nan, np.float32)
        for sub in range(in_stage):
            for hf in range(QUARTERS):
                g = (c0 + sub * SLICE + hf * 32) // group
                assert g < groups
                for r in range(BM):
                    sst[(sub * QUARTERS + hf) * BM + r] = scales[rbase + r, g]
                    if not sym:
                        zst[(sub * QUARTERS + hf) * BM + r] = zeros[rbase + r, g]
        for sub in range(in_stage):
            j = st * SPS + sub                      # slice of the segment
            # dequantize warps: thread r builds its row's A slot (tensor-memory
            # columns, or a K-major 128-byte-swizzled shared-memory tile)
            a_cols = np.full((BM, SLICE_COLS, 2), -1, np.int64)
            a_tile = np.full(BM * 128, -1, np.int64)
            for r in range(BM):
                raw = []
                for i in range(WORDS // 4):
                    pos = 16 * ((QUARTERS * sub + i) ^ (r & 7))
                    raw += list(codes[r * 128 + pos:r * 128 + pos + 16])
                words = np.array([raw[4 * w] | raw[4 * w + 1] << 8 | raw[4 * w + 2] << 16
                                  | raw[4 * w + 3] << 24 for w in range(WORDS)], np.uint32)
                o = sub * QUARTERS * BM + r
                sc = np.array([sst[o + i * BM] for i in range(QUARTERS)], np.float32)
                zp = np.array([0.0 if sym else zst[o + i * BM] for i in range(QUARTERS)],
                              np.float32)
                assert not np.isnan(sc).any()
                pairs = kernel_dequant(words, sc[np.arange(WORDS) // 4], zp[np.arange(WORDS) // 4],
                                       bits, sym, "bf16")            # [words, 8]
                for hh in range(WORDS // 8):
                    for c in range(8):
                        for t in range(4):
                            col = 32 * hh + 4 * c + t
                            a_cols[r, col] = pairs[8 * hh + c, 2 * t:2 * t + 2]
                        pos = r * 128 + 16 * ((4 * hh + c) ^ (r & 7))
                        for e in range(8):
                            a_tile[pos + 2 * e] = int(pairs[8 * hh + c, e]) & 0xFF
                            a_tile[pos + 2 * e + 1] = int(pairs[8 * hh + c, e]) >> 8
            assert (a_cols >= 0).all()
            if A_IN_SMEM:
                assert (a_tile >= 0).all()
            # MMA: per token box, 4 K = 16 steps; the segment's first resets
            for b in range(XBOXES):
                tile = tma_box_sw128(x_bytes, 2 * (kb + j * SLICE + 64 * b), m0, 2 * k, bn)
                for kk in range(4):
                    if A_IN_SMEM:                       # descriptor start + 32 (4b + kk)
                        a_bits = sw128_read(a_tile, BM, 4 * b + kk)
                    else:
                        first = (4 * b + kk) * 8        # A columns of this K step
                        a_bits = a_cols[:, first:first + 8, :].reshape(BM, 16)
                    b_bits = sw128_read(tile, bn, kk)
                    acc += bf16_value(a_bits) @ bf16_value(b_bits).T
    return acc


def tc05_splits(ctas, tiles, sms=148):
    """The host's split count (tc05_splits): fewest waves x 128-column tiles per
    CTA, plus one tile per split."""
    best, best_used = None, 1
    for want in range(1, min(16, tiles) + 1):
        per = -(-tiles // want)
        used = -(-tiles // per)
        waves = -(-(ctas * used) // sms)
        cost = waves * per + (used if used > 1 else 0)
        if best is None or cost < best:
            best, best_used = cost, used
    return best_used


def emulate(n, k, m, bits, group, sym, splits, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
    s, z = qo.choose_qparams(w, bits, group, sym)
    codes = qo.quantize_to_codes(w, s, z, bits, group, sym)
    qw = qo.pack_int4(codes)
    x = po.from_f32(rng.standard_normal((m, k)).astype(np.float32), "bf16")   # uint16 bits
    bias = po.from_f32(rng.standard_normal(n).astype(np.float32), "bf16")
    x_bytes = x.view(np.uint8).reshape(m, 2 * k)
    a = dict(n=n, k=k, m=m, group=group, sym=sym, bits=bits)
    bn = bn_of(m)
    tiles = k // 128
    per = -(-tiles // splits)
    nsplit = -(-tiles // per)
    kps = per * 128
    bias_v = bf16_value(bias)
    partial = np.zeros((nsplit, m, n))
    mark = np.zeros((m, n), np.int64)
    for bx in range(n // BM):
        for by in range(nsplit):
            for bz in range(-(-m // bn)):
                rbase, m0, kb = bx * BM, bz * bn, by * kps
                length = (min(kb + kps, k) - kb) // SLICE
                acc = run_segment(qw, s, z, x_bytes, a, rbase, m0, kb, length)
                for r in range(BM):
                    for j in range(bn):
                        tok = m0 + j
                        if tok >= min(m, m0 + bn):
                            break
                        partial[by, tok, rbase + r] += acc[r, j]
                        mark[tok, rbase + r] += 1
    assert (mark == nsplit).all()
    # one split: the kernel adds the bias; more: the reduce kernel, in split order
    y = partial[0] if nsplit == 1 else sum(partial[i] for i in range(nsplit))
    y = y + bias_v
    want = qo.quant_linear(x, "bf16", qw, s, z, bits, group, sym, (n, k), bias)
    err = np.abs(y - want).max()
    assert err < 1e-9 * max(1.0, np.abs(want).max()), err


def test_split_plan():
    # Llama-3-8B MLP shapes: 112 row blocks x 32 tiles -> one split; 32 row
    # blocks x 112 tiles -> 4 splits of 28 tiles (one wave of 128 CTAs)
    assert tc05_splits(112, 32) == 1
    assert tc05_splits(32, 112) == 4
    for ctas in (1, 8, 37, 112, 300):
        for tiles in (1, 2, 7, 32, 112):
            sp = tc05_splits(ctas, tiles)
            assert 1 <= sp <= min(16, tiles)


CASES = [
    (128, 256, 1, 4, 128, True, 1),
    (128, 512, 20, 4, 32, False, 2),
    (128, 384, 33, 2, 64, True, 3),       # 2-bit codes, odd slice counts per split
    (256, 768, 17, 4, 192, False, 2),     # a group that straddles slices
    (256, 256, 5, 4, 256, True, 1),
    (128, 256, 300, 4, 128, True, 2),     # two token blocks
]


@pytest.mark.parametrize("case", CASES)
def test_cta_data_path(case):
    emulate(*case, seed=sum(case) % 89)


# ---- mbarrier protocol ------------------------------------------------------------

class Barrier:
    def __init__(self, name, count):
        self.name, self.count, self.pending, self.done = name, count, count, 0

    def arrive(self, n=1):
        self.pending -= n
        assert self.pending >= 0, self.name
        if self.pending == 0:
            self.done += 1
            self.pending = self.count

    def ready(self, phase):
        """The hardware compares parities only: a waiter for phase p is valid
        while p or p - 1 is the last completed phase (done in {p, p + 1});
        one that is two phases behind, or ahead of the current phase, would
        pass or block on the wrong phase."""
        assert self.done <= phase + 1, f"{self.name}: waiter lapped (phase {phase}, done {self.done})"
        assert self.done >= phase, f"{self.name}: waiter ahead (phase {phase}, done {self.done})"
        return self.done > phase


def simulate(nslices, bn, seed):
    """One CTA over `nslices` 64-column slices."""
    rnd = random.Random(seed)
    xs = x_slots(bn)
    nstages = (nslices + SPS - 1) // SPS
    codes_full = [Barrier(f"codes_full{i}", 1 + 32) for i in range(CODE_STAGES)]
    codes_empty = [Barrier(f"codes_empty{i}", DQ_WARPS) for i in range(CODE_STAGES)]
    x_full = [Barrier(f"x_full{i}", 1) for i in range(MAX_XSLOTS)]
    x_empty = [Barrier(f"x_empty{i}", 1) for i in range(MAX_XSLOTS)]
    a_full = [Barrier(f"a_full{i}", 4) for i in range(ASLOTS)]
    a_empty = [Barrier(f"a_empty{i}", 1) for i in range(ASLOTS)]
    acc_full = Barrier("acc_full", 1)
    codes_ring = [None] * CODE_STAGES          # stage whose codes landed
    codes_readers = [set() for _ in range(CODE_STAGES)]
    x_ring = [None] * MAX_XSLOTS
    a_ring = [dict() for _ in range(ASLOTS)]   # warp quarter -> slice written
    mma_reading = {}                           # ("a", slot) / ("x", slot) -> slice, until complete
    inflight = []                              # asynchronous completions

    def wait(b, phase):
        while not b.ready(phase):
            yield

    def codes_loader():
        for st in range(nstages):
            cs = st % CODE_STAGES
            if st >= CODE_STAGES:
                yield from wait(codes_empty[cs], st // CODE_STAGES - 1)
                assert codes_readers[cs] == set(range(DQ_WARPS)), \
                    "codes stage refilled before every dequantize warp read it"
            codes_readers[cs] = set()
            codes_ring[cs] = None

            def land(cs=cs, st=st):
                codes_ring[cs] = st
                codes_full[cs].arrive(1)
            inflight.append(land)                 # TMA bytes (+ the expect_tx arrival)
            for _ in range(32):                   # the lanes' cp.async arrivals
                inflight.append(lambda cs=cs: codes_full[cs].arrive(1))
            yield

    def tokens_loader():
        slot, rnd_ = 0, 0
        for s in range(nslices):
            if s >= xs:
                yield from wait(x_empty[slot], rnd_ - 1)
            assert ("x", slot) not in mma_reading, "token slot refilled under an MMA"
            x_ring[slot] = None

            def land(slot=slot, s=s):
                x_ring[slot] = s
                x_full[slot].arrive()
            inflight.append(land)
            slot += 1
            if slot == xs:
                slot, rnd_ = 0, rnd_ + 1
            yield

    def mma():
        slot, rnd_ = 0, 0
        for s in range(nslices):
            asl = a_slot(s)
            yield from wait(a_full[asl], a_use(s))
            yield from wait(x_full[slot], rnd_)
            assert all(a_ring[asl].get(q) == s for q in range(4)), ("A slot", s, a_ring[asl])
            assert x_ring[slot] == s
            mma_reading[("a", asl)] = s
            mma_reading[("x", slot)] = s

            def done(asl=asl, slot=slot):
                del mma_reading[("a", asl)]
                del mma_reading[("x", slot)]
                a_empty[asl].arrive()
                x_empty[slot].arrive()
            inflight.append(done)
            slot += 1
            if slot == xs:
                slot, rnd_ = 0, rnd_ + 1
            yield

        def drained():                            # the final commit: after every MMA
            if mma_reading:
                inflight.append(drained)
            else:
                acc_full.arrive()
        inflight.append(drained)

    def dequant(warp):
        q, h = warp % 4, warp // 4
        for s in range(h, nslices, SETS):
            st, sub = s // SPS, s % SPS
            cs = st % CODE_STAGES
            in_stage = min(SPS, nslices - st * SPS)
            if sub < SETS:                        # the set's first slice of the stage
                yield from wait(codes_full[cs], st // CODE_STAGES)
            assert codes_ring[cs] == st, ("codes stage", s, codes_ring[cs])
            yield
            if sub + SETS >= in_stage:            # its last: the stage is released
                codes_readers[cs].add(warp)
                codes_empty[cs].arrive()
            asl = a_slot(s)
            if a_use(s) > 0:
                yield from wait(a_empty[asl], a_use(s) - 1)
            assert ("a", asl) not in mma_reading, "A slot rewritten under an MMA"
            a_ring[asl][q] = s
            yield
            a_full[asl].arrive()
        yield from wait(acc_full, 0)

    agents = [codes_loader(), tokens_loader(), mma()] + [dequant(w) for w in range(DQ_WARPS)]
    live = list(agents)
    steps = 0
    while live or inflight:
        steps += 1
        assert steps < 600000, "no progress (a wait that is never satisfied)"
        if inflight and (not live or rnd.random() < 0.3):
            inflight.pop(rnd.randrange(len(inflight)))()
            continue
        agent = rnd.choice(live)
        try:
            next(agent)
        except StopIteration:
            live.remove(agent)
    assert acc_full.done == 1


@pytest.mark.parametrize("nslices", [1, 2, 3, 5, 8, 13, 32, 57])
@pytest.mark.parametrize("bn", [16, 64, 256])
def test_protocol_interleavings(nslices, bn):
    for seed in range(12):
        simulate(nslices, bn, seed)
