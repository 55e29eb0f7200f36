"""CPU emulation of the mma.sync quantized-linear kernel's index arithmetic.

``wq_gemm_acc_kernel`` (2/4-bit codes, group scale on the fp32 accumulators)
is restated thread by thread: the cp.async copy slots and their source bounds,
the shared-memory swizzles, the ldmatrix / MMA fragment maps (m16n8k16), the
group cursors of split k ranges and the epilogue's output map.  (The tcgen05
kernel has its own restatement, ``test_quant_tc05_layout.py``.)  Values are carried exactly in
float64, so each result must equal the oracle's ``x @ W^T`` to rounding.

This checks the layouts on the CPU before and beside the GPU runs; it does not
run the kernels.
"""

from __future__ import annotations

import itertools

import numpy as np
import pytest

from oracle import paged_oracle as po
from oracle import quant_oracle as qo


# wq_gemm_acc_kernel
KKT, KROWS, KTHREADS, KCHUNKS, KSTAGES = 128, 64, 128, 16, 4


def w_piece_pos(r, p):
    return p ^ ((r >> 1) & 3)


def x_chunk_pos(i, c):
    return c ^ ((i & 1) << 2)


def acc_run_cta(qw_bytes, scales, zeros, x, a, bx, by, bz, MT, GPT, partial, out):
    n, k, m, group, sym, bits = a["n"], a["k"], a["m"], a["group"], a["sym"], a["bits"]
    NT = MT // 8
    WPG = 4 // GPT
    rbase = bx * KROWS
    m0 = bz * MT
    kb = by * a["k_per_split"]
    ke = min(kb + a["k_per_split"], k)
    ntiles = (ke - kb) // KKT
    mrem = m - m0
    n_tiles = NT if mrem >= MT else (mrem + 7) // 8
    groups = k // group
    row_bytes = k // 2
    tile0 = kb // KKT
    tpg = 1 if GPT > 1 else group // KKT
    # shared memory stages: w as bytes [64][64], x as [MT][16] chunks of 8 elements, s/z
    stages = [dict(w=np.full((KROWS, 64), -1, np.int64), x=np.full((MT, KCHUNKS, 8), np.nan),
                   s=np.full((KROWS, GPT), np.nan), z=np.full((KROWS, GPT), np.nan))
              for _ in range(KSTAGES)]
    state = dict(g_cur=tile0 * GPT if GPT > 1 else tile0 // tpg, g_in=0 if GPT > 1 else tile0 % tpg)
    kXPer = MT * KCHUNKS // KTHREADS
    kGPer = (KROWS * GPT + KTHREADS - 1) // KTHREADS
    flat_q = qw_bytes.reshape(-1)

    def issue(t):
        stg = stages[t % KSTAGES]
        for tid in range(KTHREADS):
            # codes
            for q in range(2):
                row = (tid >> 2) + 32 * q
                src = (rbase + (tid >> 2)) * row_bytes + kb // 2 + 16 * (tid & 3) + q * 32 * row_bytes + t * 64
                dst = (tid >> 2) * 64 + 16 * w_piece_pos(tid >> 2, tid & 3) + q * 32 * 64
                assert dst // 64 == row
                assert 0 <= src and src + 16 <= flat_q.size
                stg["w"].reshape(-1)[dst:dst + 16] = flat_q[src:src + 16]
            # x
            xr0, xc = tid >> 4, tid & 15
            x_valid = (mrem - xr0 + 7) // 8 if mrem > xr0 else 0
            for q in range(kXPer):
                tok_local = xr0 + 8 * q
                pos = x_chunk_pos(xr0, xc)
                assert pos == x_chunk_pos(tok_local, xc)
                if q < x_valid:
                    tok = m0 + tok_local
                    col = kb + 8 * xc + t * KKT
                    assert tok < m and col + 8 <= k
                    stg["x"][tok_local, pos] = x[tok, col:col + 8]
                else:
                    stg["x"][tok_local, pos] = 0.0
            # group constants
            for q in range(kGPer):
                i = tid + q * KTHREADS
                if i < KROWS * GPT:
                    r, g = i // GPT, i % GPT
                    gi = (rbase + r) * groups + state["g_cur"] + g
                    assert state["g_cur"] + g < groups
                    stg["s"][r, g] = scales.reshape(-1)[gi]
                    if not sym:
                        stg["z"][r, g] = zeros.reshape(-1)[gi]
        if GPT > 1:
            state["g_cur"] += GPT
        else:
            state["g_in"] += 1
            if state["g_in"] == tpg:
                state["g_in"] = 0
                state["g_cur"] += 1

    acc = np.zeros((4, 32, NT, 4))
    zsym = float(1 << (bits - 1))
    for t in range(min(KSTAGES - 1, ntiles)):
        issue(t)
    for t in range(ntiles):
        if t + KSTAGES - 1 < ntiles:
            # the kernel issues after the barrier; the stage it overwrites is (t-1)'s
            issue(t + KSTAGES - 1)
        stg = stages[t % KSTAGES]
        # column range this tile must cover, to check the staged data belongs to tile t
        for warp in range(4):
            # ldmatrix: lanes give row addresses; lane L -> matrix L>>3, row L&7
            addr = {}
            for h in range(2):
                for L in range(32):
                    lr = warp * 16 + (L & 7)
                    off = lr * 64 + 16 * w_piece_pos(lr, L >> 3) + h * 8 * 64
                    addr[(h, L >> 3, L & 7)] = off
            cw = np.zeros((32, 2, 4), np.uint64)
            wflat = stg["w"].reshape(-1)
            for lane in range(32):
                gid, tid4 = lane >> 2, lane & 3
                for h in range(2):
                    for j in range(4):  # matrix j: thread gets row gid, word tid4
                        off = addr[(h, j, gid)] + 4 * tid4
                        b = wflat[off:off + 4]
                        assert (b >= 0).all()
                        cw[lane, h, j] = int(b[0]) | int(b[1]) << 8 | int(b[2]) << 16 | int(b[3]) << 24
            part = np.zeros((32, NT, 4))
            for w in range(4):
                g = w // WPG
                if w % WPG == 0:
                    part[:] = 0
                # per lane pair values (code j, code j+4) minus zero
                pa = np.zeros((32, 2, 4, 2))
                for lane in range(32):
                    gid = lane >> 2
                    wrow = warp * 16 + gid
                    for h in range(2):
                        zf = zsym if sym else stg["z"][wrow + 8 * h, g]
                        word = int(cw[lane, h, w])
                        for j in range(4):
                            v = (word >> (4 * j)) & 0x000F000F
                            lo, hi = v & 0xF, (v >> 16) & 0xF
                            pa[lane, h, j] = (lo - zf, hi - zf)
                for nt in range(NT):
                    if nt >= n_tiles:
                        continue
                    for hs in range(2):
                        A = np.zeros((16, 16))
                        B = np.zeros((16, 8))
                        for lane in range(32):
                            gid, tid4 = lane >> 2, lane & 3
                            af = [pa[lane, 0, 2 * hs], pa[lane, 1, 2 * hs], pa[lane, 0, 2 * hs + 1],
                                  pa[lane, 1, 2 * hs + 1]]
                            A[gid, 2 * tid4:2 * tid4 + 2] = af[0]
                            A[gid + 8, 2 * tid4:2 * tid4 + 2] = af[1]
                            A[gid, 2 * tid4 + 8:2 * tid4 + 10] = af[2]
                            A[gid + 8, 2 * tid4 + 8:2 * tid4 + 10] = af[3]
                            xi = nt * 8 + gid
                            xv = stg["x"][xi, (4 * w + tid4) ^ ((gid & 1) << 2)]
                            bb = [(xv[0], xv[4]), (xv[1], xv[5]), (xv[2], xv[6]), (xv[3], xv[7])]
                            B[2 * tid4:2 * tid4 + 2, gid] = bb[2 * hs]
                            B[2 * tid4 + 8:2 * tid4 + 10, gid] = bb[2 * hs + 1]
                        D = A @ B
                        for lane in range(32):
                            gid, tid4 = lane >> 2, lane & 3
                            part[lane, nt, 0] += D[gid, 2 * tid4]
                            part[lane, nt, 1] += D[gid, 2 * tid4 + 1]
                            part[lane, nt, 2] += D[gid + 8, 2 * tid4]
                            part[lane, nt, 3] += D[gid + 8, 2 * tid4 + 1]
                if w % WPG == WPG - 1:
                    for lane in range(32):
                        wrow = warp * 16 + (lane >> 2)
                        s0, s1 = stg["s"][wrow, g], stg["s"][wrow + 8, g]
                        acc[warp, lane, :, 0] += part[lane, :, 0] * s0
                        acc[warp, lane, :, 1] += part[lane, :, 1] * s0
                        acc[warp, lane, :, 2] += part[lane, :, 2] * s1
                        acc[warp, lane, :, 3] += part[lane, :, 3] * s1
    for warp, lane, nt, e in itertools.product(range(4), range(32), range(NT), range(4)):
        gid, tid4 = lane >> 2, lane & 3
        tok = m0 + nt * 8 + 2 * tid4 + (e & 1)
        f = rbase + warp * 16 + gid + 8 * (e >> 1)
        if tok >= m:
            continue
        partial[by, tok, f] += acc[warp, lane, nt, e]
        out[tok, f] = 1  # mark written


def acc_emulate(n, k, m, bits, group, sym, MT, splits, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
    s, z = qo.choose_qparams(w, bits, group, sym)
    codes = qo.quantize_to_codes(w, s, z, bits, group, sym)
    qw = qo.pack_int4(codes)
    x = rng.standard_normal((m, k))
    GPT = 1 if group >= KKT else KKT // group
    tiles = k // KKT
    per = (tiles + splits - 1) // splits
    a = dict(n=n, k=k, m=m, group=group, sym=sym, bits=bits, k_per_split=per * KKT)
    nsplit = (tiles + per - 1) // per
    partial = np.zeros((nsplit, m, n))
    mark = np.zeros((m, n))
    for bx in range(n // KROWS):
        for by in range(nsplit):
            for bz in range((m + MT - 1) // MT):
                acc_run_cta(qw, s, z, x, a, bx, by, bz, MT, GPT, partial, mark)
    y = partial.sum(0)
    assert (mark == 1).all()
    # exact: (q - zero) * s with the symmetric bias
    q = qo.unpack_int4(qw, k).astype(np.float64)
    zz = np.repeat(z.astype(np.float64), group, axis=1) if not sym else float(1 << (bits - 1))
    wex = (q - zz) * np.repeat(s.astype(np.float64), group, axis=1)
    want = x @ wex.T
    err = np.abs(y - want).max()
    assert err < 1e-9 * max(1.0, np.abs(want).max()), err
    return err


ACC_CASES = [
    (64, 256, 1, 4, 128, True, 8, 1),
    (64, 256, 5, 4, 64, False, 8, 2),
    (64, 512, 8, 2, 32, True, 8, 3),
    (128, 512, 13, 4, 32, False, 32, 2),
    (64, 768, 31, 4, 256, True, 32, 3),
    (64, 1536, 9, 4, 384, False, 32, 5),
    (64, 512, 45, 4, 32, True, 32, 4),
]


@pytest.mark.parametrize("case", ACC_CASES)
def test_acc_kernel_layout(case):
    acc_emulate(*case, seed=sum(case) % 97)
