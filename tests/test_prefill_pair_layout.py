"""CPU checks of the 2-SM pair prefill kernel's layout and synchronisation.

``prefill_pair_kernel`` (csrc/prefill_pair.cu) is restated on the CPU:

* the shared-memory map (query tiles, K and V rings, barrier block) and every
  TMA destination and MMA operand window inside it, with the 1024-byte
  alignment the 128-byte swizzle needs, and the tensor-memory columns of S, P
  and O;
* the barrier protocol of one pair as a randomized interleaving of its
  agents - both CTAs' K loader, V loader, relay and two softmax groups, and
  the even CTA's MMA issuer - using the kernel's stage indices, phase
  parities and arrival counts.  Every run must finish (no wait is left
  unsatisfied), every consumer must find the tile it expects in the ring slot
  it reads, and no waiter may fall two phases behind a barrier (the
  hardware's parity test would then block or pass on the wrong phase).

The constants are read from the kernel source, so the checks follow it.  This
does not run the kernel.
"""

from __future__ import annotations

import os
import random
import re

import pytest

from conftest import REPO

SRC = os.path.join(REPO, "quantized-llm-inference-engine-_b200", "csrc", "prefill_pair.cu")


def _constants():
    text = open(SRC).read()
    out = {}
    for name in ("kBS", "kM", "kN", "kD", "kKStages", "kVStages", "kBitsRing", "kReadyRing"):
        m = re.search(r"constexpr int %s = (\d+);" % name, text)
        assert m, name
        out[name] = int(m.group(1))
    out["kTmemCols"] = int(re.search(r"constexpr uint32_t kTmemCols = (\d+);", text).group(1))
    return out


C = _constants()


def test_shared_memory_map():
    bs, m, n, d = C["kBS"], C["kM"], C["kN"], C["kD"]
    subs = d // 64
    q_sub = m * 128                       # 128 rows x 64 dims
    k_sub = (n // 2) * 128                # 64 keys x 64 dims (this CTA's half)
    k_stage = subs * k_sub
    v_stage = n * 128                     # 128 keys x this CTA's 64 dims
    off_q = 0
    off_k = off_q + 2 * subs * q_sub
    off_v = off_k + C["kKStages"] * k_stage
    off_bar = off_v + C["kVStages"] * v_stage
    total = off_bar + 512
    assert total <= 227 * 1024
    for off in (off_q, off_k, off_v):
        assert off % 1024 == 0
    box = bs * 128                        # one 16-row box (2 KB)
    for crank in (0, 1):
        # K: blocks [4 crank, 4 crank + 4) of a tile, box (i - 4 crank) of each sub
        for st in range(C["kKStages"]):
            for i in range(4 * crank, 4 * crank + 4):
                for sub in range(subs):
                    dst = off_k + st * k_stage + sub * k_sub + (i - 4 * crank) * box
                    assert dst % 1024 == 0
                    assert off_k <= dst and dst + box <= off_v
        # V: all 8 blocks of the tile, this CTA's 64 dims
        for st in range(C["kVStages"]):
            for i in range(n // bs):
                dst = off_v + st * v_stage + i * box
                assert dst % 1024 == 0 and dst + box <= off_bar
    # MMA operand windows (byte ranges read per K = 16 step)
    for q in range(2):
        for kk in range(d // 16):
            a = off_q + q * subs * q_sub + (kk >> 2) * q_sub + (kk & 3) * 32
            assert off_q <= a and a + (m - 1) * 128 + 32 <= off_k      # 128 rows, 32 bytes
    for st in range(C["kKStages"]):
        for kk in range(d // 16):
            b = off_k + st * k_stage + (kk >> 2) * k_sub + (kk & 3) * 32
            assert b + (n // 2 - 1) * 128 + 32 <= off_k + (st + 1) * k_stage
    for st in range(C["kVStages"]):
        for kk in range(n // 16):
            b = off_v + st * v_stage + kk * 16 * 128
            assert b + 16 * 128 <= off_v + (st + 1) * v_stage        # 16 keys x 128 bytes


def test_tensor_memory_columns():
    cols = C["kTmemCols"]
    spans = []
    for q in range(2):
        s = (q * 128, q * 128 + C["kN"])                  # S of tile q (fp32 per key)
        p = (q * 128, q * 128 + C["kN"] // 2)             # P over its first 64 columns
        o = (256 + q * 128, 256 + q * 128 + C["kD"])      # O (fp32 per dim)
        assert p[0] >= s[0] and p[1] <= s[1]
        spans += [s, o]
    spans.sort()
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 <= b0
    assert spans[-1][1] <= cols and cols in (32, 64, 128, 256, 512)


class Barrier:
    """An mbarrier: arrivals per phase, completed phases, tx bytes pending."""

    def __init__(self, name, count):
        self.name, self.count = name, count
        self.pending = count
        self.done = 0            # completed phases

    def arrive(self, n=1):
        self.pending -= n
        assert self.pending >= 0, self.name
        if self.pending == 0:
            self.done += 1
            self.pending = self.count

    def ready(self, phase):
        """The waiter wants phase `phase` (0-based) complete; the hardware only
        sees its parity, so falling two phases behind is an error."""
        assert self.done <= phase + 1, f"{self.name}: waiter lapped (phase {phase}, done {self.done})"
        return self.done > phase


def simulate(n_q, seed):
    ks, vs, br, rr = C["kKStages"], C["kVStages"], C["kBitsRing"], C["kReadyRing"]
    n_tiles = max(n_q)
    rnd = random.Random(seed)
    cta = []
    for c in range(2):
        cta.append(dict(
            q_full=Barrier(f"q_full{c}", 1),
            k_full=[Barrier(f"k_full{c}.{i}", 1) for i in range(ks)],
            k_empty=[Barrier(f"k_empty{c}.{i}", 1) for i in range(ks)],
            v_full=[Barrier(f"v_full{c}.{i}", 1) for i in range(vs)],
            v_empty=[Barrier(f"v_empty{c}.{i}", 1) for i in range(vs)],
            bits_full=[Barrier(f"bits_full{c}.{i}", 1) for i in range(br)],
            s_full=[Barrier(f"s_full{c}.{q}", 1) for q in range(2)],
            o_final=[Barrier(f"o_final{c}.{q}", 1) for q in range(2)],
            k_ring=[None] * ks, v_ring=[None] * vs, tile_bits=[None] * br, s_bits=[None] * br,
            S=[None, None], P=[None, None]))
    lead = dict(q_ready=Barrier("q_ready", 2),
                ready=[Barrier(f"ready.{i}", 2) for i in range(rr)],
                p_full=[Barrier(f"p_full.{q}", 8) for q in range(2)])
    inflight = []                              # (barrier, action) copies not yet landed

    def commit(name, idx=None):
        for c in range(2):
            b = cta[c][name] if idx is None else cta[c][name][idx]
            b.arrive()

    def wait(b, phase):
        while not b.ready(phase):
            yield

    def loader(c, is_k):
        x = cta[c]
        stages = ks if is_k else vs
        ring = x["k_ring"] if is_k else x["v_ring"]
        full = x["k_full"] if is_k else x["v_full"]
        empty = x["k_empty"] if is_k else x["v_empty"]
        if is_k:
            inflight.append((x["q_full"], None))
        for j in range(n_tiles):
            st = j % stages
            if j >= stages:
                yield from wait(empty[st], j // stages - 1)
            if is_k:
                x["tile_bits"][j % br] = j
            inflight.append((full[st], (ring, st, j)))
            yield

    def relay(c):
        x = cta[c]

        def k_staged(j):
            yield from wait(x["k_full"][j % ks], j // ks)
            assert x["k_ring"][j % ks] == j and x["tile_bits"][j % br] == j
            x["s_bits"][j % br] = j
            x["bits_full"][j % br].arrive()

        yield from wait(x["q_full"], 0)
        yield from k_staged(0)
        lead["q_ready"].arrive()
        for j in range(n_tiles):
            yield from wait(x["v_full"][j % vs], j // vs)
            assert x["v_ring"][j % vs] == j
            if j + 1 < n_tiles:
                yield from k_staged(j + 1)
            lead["ready"][j % rr].arrive()
            yield

    def mma():
        def qk(q, j):
            for c in range(2):
                assert cta[c]["k_ring"][j % ks] == j
                cta[c]["S"][q] = j
            commit("s_full", q)

        def pv(q, j):
            for c in range(2):
                assert cta[c]["v_ring"][j % vs] == j and cta[c]["P"][q] == j
            if j == n_q[q] - 1:
                commit("o_final", q)

        yield from wait(lead["q_ready"], 0)
        if n_q[0] > 0:
            qk(0, 0)
        if n_q[1] > 0:
            qk(1, 0)
        commit("k_empty", 0)
        for j in range(n_tiles):
            yield from wait(lead["ready"][j % rr], j // rr)
            nxt = False
            last_q = 1 if j < n_q[1] else 0
            for q in range(2):
                if j < n_q[q]:
                    yield from wait(lead["p_full"][q], j)
                    pv(q, j)
                    if q == last_q:
                        commit("v_empty", j % vs)
                    if j + 1 < n_q[q]:
                        nxt = True
                        qk(q, j + 1)
            if nxt:
                commit("k_empty", (j + 1) % ks)
            yield

    def softmax(c, q):
        x = cta[c]
        for j in range(n_q[q]):
            yield from wait(x["bits_full"][j % br], j // br)
            assert x["s_bits"][j % br] == j
            yield from wait(x["s_full"][q], j)
            assert x["S"][q] == j
            x["P"][q] = j
            lead["p_full"][q].arrive(4)          # the tile's 4 warps in this CTA
            yield
        if n_q[q] > 0:
            yield from wait(x["o_final"][q], 0)

    agents = [loader(c, k) for c in range(2) for k in (True, False)]
    agents += [relay(c) for c in range(2)] + [mma()]
    agents += [softmax(c, q) for c in range(2) for q in range(2)]
    live = list(agents)
    steps = 0
    while live or inflight:
        steps += 1
        assert steps < 200000, "no progress (a wait that is never satisfied)"
        # land a random in-flight copy now and then
        if inflight and (not live or rnd.random() < 0.3):
            b, act = inflight.pop(rnd.randrange(len(inflight)))
            if act is not None:
                ring, st, j = act
                ring[st] = j
            b.arrive()
            continue
        agent = rnd.choice(live)
        try:
            next(agent)
        except StopIteration:
            live.remove(agent)


@pytest.mark.parametrize("n_q", [(1, 1), (3, 4), (9, 9), (20, 21), (0, 2), (2, 0), (17, 16)])
def test_pair_protocol_interleavings(n_q):
    for seed in range(25):
        simulate(n_q, seed)
