// Paged decode attention, sm_100a fast path.
//
// Replaces the gather -> expand -> matmul/softmax/matmul (-> split merge) chain
// of PagedAttention.forward (src/llmopt/attention/paged_attention.py:146-293)
// for 16-bit caches with block_size 16, head_dim 64/128/256 and up to 16 query
// rows per KV head (q_len * group <= 16: decode and short speculative chunks).
//
// Data movement.  One CTA owns `hpc` consecutive KV heads (all heads of the
// cache when there are at most 8) and a range of KV blocks from the split plan
// (plan.cuh).  The cache is described to TMA as the 5-D tensor
// (head_dim, kv_heads, block_size, num_blocks, layers) - the storage order, so
// strides grow with the dimension - and a producer warp issues, per block and
// per 64-dim slice, one box (64 dims, 1 head, 16 tokens) per head for K and
// for V.  The boxes land in shared memory as [head][token][64 dims] rows of
// 128 B with the 128-byte swizzle, so ldmatrix reads of 8 tokens of one head
// hit 8 different bank groups.  Each physical block is read once per CTA for all of
// its KV heads: every GQA group shares the stream.  Blocks whose table entry
// is -1 (or out of range) are not loaded at all.  A ring of `stages` buffers
// with full/empty mbarriers keeps several blocks in flight per SM.
//
// Two-stream mode (streams == 2, used when a rank holds one KV head): the CTA
// keeps the two-head layout and producer warp, but its two consumer warps take
// the same head over two consecutive ranges of the balanced plan (two
// "virtual CTAs"): the producer stages block i of each range into the two head
// slots of ring stage i, so each copy issuer keeps two streams in flight, as
// it does for two heads.
//
// Self-issuing mode (SP, the one-head alternative): the CTA is one warp that
// issues its own K/V copies a ring's depth ahead of the block it is consuming,
// into stages it has already consumed - no producer warp, so about twice as
// many CTAs fit per SM.
//
// Math.  Consumer warp w handles KV head (first + w).  Its query rows (the
// group's heads x q_len, padded to 16) are the A operand of m16n8k16 MMAs:
// S = Q K^T over the 16 tokens (two n-tiles), online softmax in fp32 registers
// (row max/sum via quad shuffles, exp2 on the SFU), then O += P V with P
// re-packed from the S accumulators.  Partials (normalised O, natural-log LSE)
// go to the split workspace; combine.cu merges them.
#include <float.h>

#include <cstdlib>

#include "common.cuh"
#include "kernels.h"

namespace llmopt {
namespace {

constexpr int kBS = 16;            // tokens per KV block on this path
constexpr int kSub = 64;           // dims per TMA box row (128 B, the swizzle span)
constexpr int kSubRowBytes = 128;
constexpr int kMaxBoxHeads = 8;    // consumer warps per CTA
constexpr long long kMaxPrefixBatch = 4096;  // balanced mode keeps prefix[] in smem

struct Smem {
  unsigned char* stages;
  uint64_t* full;
  uint64_t* empty;
  int* meta;
  int* prefix;
};

__device__ __forceinline__ long long find_seq(const int* prefix, long long batch, long long f) {
  long long lo = 0, hi = batch - 1;
  while (lo < hi) {
    const long long mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= f) lo = mid; else hi = mid - 1;
  }
  return lo;
}

template <int D, int Q_DT, int KV_DT>
__device__ __forceinline__ void load_q_frags(const AttnArgs& a, long long s, int kh, int gid,
                                             int tid4, uint32_t (&qa)[D / 16][4]) {
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int r = gid + 8 * half;
    const bool ok = r < a.rows;
    long long base = 0;
    if (ok) {
      const int qi = r / a.group;
      const int gi = r - qi * a.group;
      base = s * a.q_s + (long long)(kh * a.group + gi) * a.q_h + (long long)qi * a.q_t;
    }
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int khalf = 0; khalf < 2; ++khalf) {
        const int d = kk * 16 + khalf * 8 + 2 * tid4;
        float x0 = 0.f, x1 = 0.f;
        if (ok) {
          x0 = load_f32<Q_DT>(a.q, base + d);
          x1 = load_f32<Q_DT>(a.q, base + d + 1);
        }
        qa[kk][half + 2 * khalf] = pack2<KV_DT>(x0, x1);
      }
    }
  }
}

// SP: 12 one-warp CTAs per SM by registers (168 a thread at head_dim 128).
// ST: two-stream mode (never together with SP).
template <int D, int Q_DT, int KV_DT, bool SP, bool ST>
__global__ void __launch_bounds__(SP ? 32 : (kMaxBoxHeads + 1) * 32, SP ? 12 : 1)
    decode_tma_kernel(const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmv, const AttnArgs a, const int hpc,
                      const int nstages) {
  constexpr int streams = ST ? 2 : 1;
  // When the dependent kernel (the combine, or the next decode) may start
  // launching, measured on B200: with a producer warp, right away - the next
  // grid's CTAs then fill SMs as this grid's tail CTAs exit; with self-issuing
  // one-warp CTAs, only as each CTA finishes - released at the start, the
  // combine after it ran 40% slower (298 vs 213 us for decode + combine at the
  // 8-GPU shard shape).
  griddep_wait();
  if (!SP) griddep_launch_dependents();
  constexpr int kSubs = D / kSub;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long batch = a.batch;
  const bool balanced = a.plan.mode == kModeBalanced;
  const int sub_bytes = hpc * kBS * kSubRowBytes;        // one 64-dim slice of one block
  const int half_bytes = kSubs * sub_bytes;              // K (or V) of one block
  const int stage_bytes = 2 * half_bytes;

  extern __shared__ unsigned char smem_raw[];
  Smem sm;
  {
    uintptr_t p = (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023);
    sm.stages = reinterpret_cast<unsigned char*>(p);
    unsigned char* tail = sm.stages + (size_t)nstages * stage_bytes;
    sm.full = reinterpret_cast<uint64_t*>(tail);
    sm.empty = sm.full + nstages;
    sm.meta = reinterpret_cast<int*>(sm.empty + nstages);   // [stage][stream]
    sm.prefix = sm.meta + 2 * nstages;
  }

  // ---- this CTA's block range ------------------------------------------------
  long long lo = 0, hi = 0, mid = 0, fixed_seq = -1;
  if (balanced) {
    // Exclusive prefix sum of per-sequence block counts over the whole batch.
    const int nthreads = blockDim.x;
    const long long chunk = (batch + nthreads - 1) / nthreads;
    const long long s0 = threadIdx.x * chunk;
    const long long s1 = s0 + chunk < batch ? s0 + chunk : batch;
    int local = 0;
    for (long long s = s0; s < s1; ++s) {
      const long long c = load_index(a.ctx, a.ctx_i64, s);
      local += (int)blocks_of(c, kBS, a.table_width);
      if (blockIdx.x == 0 && blockIdx.y == 0 && c > a.table_width * kBS) {
        record_error(a.err, kErrTableWidth);
      }
    }
    // block-wide exclusive scan of `local` (<= 9 warps)
    __shared__ int warp_tot[kMaxBoxHeads + 1];
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    int before = 0;
    for (int w = 0; w < warp; ++w) before += warp_tot[w];
    int run = before + incl - local;
    for (long long s = s0; s < s1; ++s) {
      sm.prefix[s] = run;
      run += (int)blocks_of(load_index(a.ctx, a.ctx_i64, s), kBS, a.table_width);
    }
    if (threadIdx.x == blockDim.x - 1) sm.prefix[batch] = run;
    __syncthreads();
    const long long total = sm.prefix[batch];
    if (blockIdx.x == 0 && blockIdx.y == 0) {
      for (long long s = threadIdx.x; s <= batch; s += blockDim.x) a.prefix[s] = sm.prefix[s];
    }
    // Ranges of this CTA's virtual CTAs: [lo, mid) and [mid, hi) with two
    // streams, [lo, hi) with one.
    const long long v0 = (long long)blockIdx.x * streams;
    lo = range_start(v0, total, a.plan.ctas);
    hi = range_start(v0 + streams, total, a.plan.ctas);
    mid = streams == 2 ? range_start(v0 + 1, total, a.plan.ctas) : hi;
  } else {
    fixed_seq = blockIdx.x / a.plan.splits;
    const int j = blockIdx.x - (int)fixed_seq * a.plan.splits;
    const long long c = load_index(a.ctx, a.ctx_i64, fixed_seq);
    const long long nb = blocks_of(c, kBS, a.table_width);
    if (j == 0 && blockIdx.y == 0 && threadIdx.x == 0 && c > a.table_width * kBS) {
      record_error(a.err, kErrTableWidth);
    }
    lo = (long long)j * a.plan.split_blocks;
    hi = lo + a.plan.split_blocks < nb ? lo + a.plan.split_blocks : nb;
    mid = hi;
  }
  if (lo >= hi) return;  // uniform over the CTA

  if (threadIdx.x == 0) {
    for (int i = 0; i < nstages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], hpc);
    }
    mbar_init_fence();
  }
  __syncthreads();

  const int kh0 = blockIdx.y * (streams == 2 ? 1 : hpc);
  // Stream k covers [s_lo[k], s_lo[k] + s_len[k]); `total` ring steps in all.
  const long long s_lo[2] = {lo, mid};
  const long long s_len[2] = {mid - lo, hi - mid};
  const long long total = streams == 2 ? (s_len[0] > s_len[1] ? s_len[0] : s_len[1]) : hi - lo;

  // Block `idx` of stream k (0-based): its table entry and valid-token count
  // (0: not loaded).  Called by each lane for its own block.
  auto resolve = [&](int k, long long idx, int* id, int* ntok) {
    *id = 0;
    *ntok = 0;
    if (idx >= (streams == 2 ? s_len[k] : total)) return;
    const long long f = s_lo[k] + idx;
    long long s, j;
    if (balanced) {
      s = find_seq(sm.prefix, batch, f);
      j = f - sm.prefix[s];
    } else {
      s = fixed_seq;
      j = f;
    }
    const long long c = load_index(a.ctx, a.ctx_i64, s);
    const long long raw = load_index(a.table, a.table_i64, s * a.table_stride + j);
    const long long left = c - j * kBS;
    const int nt = left < kBS ? (int)left : kBS;
    if (raw < 0) {
      return;
    } else if (raw >= a.num_blocks) {
      record_error(a.err, kErrBlockId);
      return;
    }
    *id = (int)raw;
    *ntok = nt;
  };
  // Fill stage st with block id (ntok > 0) or mark it empty; one thread.  With
  // two streams, block id1 of stream 1 goes to the second head slot.
  auto fill_stage = [&](int st, int id_i, int nt_i, int id1, int nt1) {
    sm.meta[2 * st] = nt_i;
    sm.meta[2 * st + 1] = nt1;
    if (streams == 2) {
      const int one = kBS * kSubRowBytes;  // one 64-dim slice of one head slot
      const unsigned bytes = (unsigned)(((nt_i > 0) + (nt1 > 0)) * 2 * kSubs * one);
      if (bytes == 0) {
        mbar_arrive(&sm.full[st]);
        return;
      }
      unsigned char* kdst = sm.stages + (size_t)st * stage_bytes;
      unsigned char* vdst = kdst + half_bytes;
      mbar_arrive_expect_tx(&sm.full[st], bytes);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int idk = k ? id1 : id_i;
        if ((k ? nt1 : nt_i) <= 0) continue;
#pragma unroll
        for (int sub = 0; sub < kSubs; ++sub) {
          const int off = sub * sub_bytes + k * one;
          tma_load_5d(kdst + off, &tmk, &sm.full[st], sub * kSub, kh0, 0, idk, a.layer);
          tma_load_5d(vdst + off, &tmv, &sm.full[st], sub * kSub, kh0, 0, idk, a.layer);
        }
      }
      return;
    }
    if (nt_i > 0) {
      unsigned char* kdst = sm.stages + (size_t)st * stage_bytes;
      unsigned char* vdst = kdst + half_bytes;
      mbar_arrive_expect_tx(&sm.full[st], (unsigned)stage_bytes);
#pragma unroll
      for (int sub = 0; sub < kSubs; ++sub) {
        for (int hh = 0; hh < hpc; ++hh) {
          const int off = sub * sub_bytes + hh * kBS * kSubRowBytes;
          tma_load_5d(kdst + off, &tmk, &sm.full[st], sub * kSub, kh0 + hh, 0, id_i, a.layer);
          tma_load_5d(vdst + off, &tmv, &sm.full[st], sub * kSub, kh0 + hh, 0, id_i, a.layer);
        }
      }
    } else {
      mbar_arrive(&sm.full[st]);
    }
  };

  // ---- producer warp -----------------------------------------------------------
  if (!SP && warp == hpc) {
    if (lane == 0) {
      prefetch_tensormap(&tmk);
      prefetch_tensormap(&tmv);
    }
    for (long long base = 0; base < total; base += 32) {
      // Each lane resolves one block per stream: table entry and valid tokens.
      int id, ntok, id1 = 0, ntok1 = 0;
      resolve(0, base + lane, &id, &ntok);
      if (streams == 2) resolve(1, base + lane, &id1, &ntok1);
      const int cnt = total - base < 32 ? (int)(total - base) : 32;
      for (int i = 0; i < cnt; ++i) {
        const int id_i = __shfl_sync(0xffffffffu, id, i);
        const int nt_i = __shfl_sync(0xffffffffu, ntok, i);
        const int id1_i = __shfl_sync(0xffffffffu, id1, i);
        const int nt1_i = __shfl_sync(0xffffffffu, ntok1, i);
        if (lane == 0) {
          const long long it = base + i;
          const int st = (int)(it % nstages);
          const long long round = it / nstages;
          if (round > 0 && !mbar_wait(&sm.empty[st], (unsigned)((round - 1) & 1))) {
            record_error(a.err, kErrWaitTimeout | kErrWaitSlot);
          }
          fill_stage(st, id_i, nt_i, id1_i, nt1_i);
        }
        __syncwarp();
      }
    }
    // Do not leave the CTA while copies into its shared memory may be in flight.
    if (lane == 0) {
      const long long first = total > nstages ? total - nstages : 0;
      for (long long it = first; it < total; ++it) {
        if (!mbar_wait(&sm.full[it % nstages], (unsigned)((it / nstages) & 1))) {
          record_error(a.err, kErrWaitTimeout | kErrWaitDrain);
        }
      }
    }
    return;
  }

  // ---- consumer warps: one KV head each, or one stream each ----------------------
  const int kh = streams == 2 ? kh0 : kh0 + warp;
  const int my = streams == 2 ? warp : 0;     // this warp's stream (meta column)
  const int gid = lane >> 2;
  const int tid4 = lane & 3;
  const int mi = lane >> 3;  // which 8x8 matrix this lane addresses in ldmatrix.x4
  const int rr = lane & 7;
  const float scale_log2 = a.scale * kLog2e;
  const bool capped = a.softcap > 0.f;
  const int head_row0 = warp * kBS;  // first smem row of this head inside a slice

  // Self-issuing: blocks [0, issued) have been issued; lane l caches the
  // table entry of block cache_base + l.
  long long issued = 0;
  long long cache_base = -32;
  int c_id = 0, c_nt = 0;
  auto issue_upto = [&](long long limit) {
    if (limit > total) limit = total;
    while (issued < limit) {
      if (issued >= cache_base + 32) {
        cache_base = issued;
        resolve(0, cache_base + lane, &c_id, &c_nt);
      }
      const int k = (int)(issued - cache_base);
      const int id_i = __shfl_sync(0xffffffffu, c_id, k);
      const int nt_i = __shfl_sync(0xffffffffu, c_nt, k);
      // This stage's previous block was consumed by this warp: order its reads
      // (and any zeroing) before the copy that overwrites it.
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      if (lane == 0) fill_stage((int)(issued % nstages), id_i, nt_i, 0, 0);
      __syncwarp();
      ++issued;
    }
  };
  if (SP) {
    if (lane == 0) {
      prefetch_tensormap(&tmk);
      prefetch_tensormap(&tmv);
    }
    issue_upto(nstages);
  }

  long long it = 0;
  long long cur = s_lo[my];
  const long long my_hi = streams == 2 ? s_lo[my] + s_len[my] : hi;
  while (cur < my_hi) {
    long long s, seg_begin, seg_end;
    if (balanced) {
      s = find_seq(sm.prefix, batch, cur);
      seg_begin = sm.prefix[s];
      seg_end = sm.prefix[s + 1] < my_hi ? sm.prefix[s + 1] : my_hi;
    } else {
      s = fixed_seq;
      seg_begin = 0;
      seg_end = hi;
    }
    const long long ctx_s = load_index(a.ctx, a.ctx_i64, s);
    uint32_t qa[D / 16][4];
    load_q_frags<D, Q_DT, KV_DT>(a, s, kh, gid, tid4, qa);
    // Causal limit of my two rows (only used when q_len > 1).
    const long long qpos0 = ctx_s - a.q_len + (gid / a.group);
    const long long qpos1 = ctx_s - a.q_len + ((gid + 8) / a.group);

    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float o[D / 8][4];
#pragma unroll
    for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

    for (long long f = cur; f < seg_end; ++f, ++it) {
      // Self-issuing: keep nstages - 1 blocks in flight beyond this one.
      if (SP) issue_upto(it + nstages);
      const int st = (int)(it % nstages);
      if (!mbar_wait(&sm.full[st], (unsigned)((it / nstages) & 1))) {
        record_error(a.err, kErrWaitTimeout | kErrWaitData);
      }
      const int ntok = sm.meta[2 * st + my];
      if (ntok > 0) {
        unsigned char* kst = sm.stages + (size_t)st * stage_bytes;
        unsigned char* vst = kst + half_bytes;
        if (ntok < kBS) {
          // Slots past the context hold stale data; zero this head's V rows so a
          // zero probability never meets an Inf/NaN there.
          for (int e = lane; e < (kBS - ntok) * kSubs * 8; e += 32) {
            const int t = ntok + e / (kSubs * 8);
            const int rest = e % (kSubs * 8);
            const int sub = rest >> 3;
            const int ch = rest & 7;
            *reinterpret_cast<uint4*>(vst + sub * sub_bytes + (head_row0 + t) * kSubRowBytes +
                                      (ch << 4)) = make_uint4(0u, 0u, 0u, 0u);
          }
          // Order these generic-proxy stores before the TMA (async proxy) that will
          // refill the stage after it is released.
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
        }
        const uint32_t kaddr = smem_addr(kst);
        const uint32_t vaddr = smem_addr(vst);

        // S = Q K^T : two n-tiles of 8 tokens
        float sacc[2][4];
#pragma unroll
        for (int n = 0; n < 2; ++n) sacc[n][0] = sacc[n][1] = sacc[n][2] = sacc[n][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int t = ((mi >> 1) << 3) + rr;
          const int chunk = 2 * kk + (mi & 1);
          const uint32_t addr = kaddr + (chunk >> 3) * sub_bytes + (head_row0 + t) * kSubRowBytes +
                                (((chunk & 7) ^ (t & 7)) << 4);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(addr, b0, b1, b2, b3);
          mma_16816<KV_DT>(sacc[0], qa[kk], b0, b1);
          mma_16816<KV_DT>(sacc[1], qa[kk], b2, b3);
        }

        // scale / softcap / mask, in log2 units
        const long long kbase = (f - seg_begin) * kBS;
        float sc[2][4];
#pragma unroll
        for (int n = 0; n < 2; ++n) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int tok = n * 8 + 2 * tid4 + (e & 1);
            float x = sacc[n][e];
            x = capped ? tanhf(x * a.scale / a.softcap) * (a.softcap * kLog2e) : x * scale_log2;
            bool ok = tok < ntok;
            if (a.q_len > 1) ok = ok && (kbase + tok <= ((e >> 1) ? qpos1 : qpos0));
            sc[n][e] = ok ? x : -INFINITY;
          }
        }
        float mx0 = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
        float mx1 = fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]));
        mx0 = warp_max_xor(warp_max_xor(mx0, 1), 2);
        mx1 = warp_max_xor(warp_max_xor(mx1, 1), 2);
        const float mn0 = fmaxf(m0, mx0);
        const float mn1 = fmaxf(m1, mx1);
        const float mu0 = mn0 == -INFINITY ? 0.f : mn0;
        const float mu1 = mn1 == -INFINITY ? 0.f : mn1;
        const float al0 = fast_exp2(m0 - mu0);
        const float al1 = fast_exp2(m1 - mu1);
        float p[2][4];
#pragma unroll
        for (int n = 0; n < 2; ++n) {
          p[n][0] = fast_exp2(sc[n][0] - mu0);
          p[n][1] = fast_exp2(sc[n][1] - mu0);
          p[n][2] = fast_exp2(sc[n][2] - mu1);
          p[n][3] = fast_exp2(sc[n][3] - mu1);
        }
        l0 = l0 * al0 + (p[0][0] + p[0][1]) + (p[1][0] + p[1][1]);
        l1 = l1 * al1 + (p[0][2] + p[0][3]) + (p[1][2] + p[1][3]);
        m0 = mn0;
        m1 = mn1;
#pragma unroll
        for (int n = 0; n < D / 8; ++n) {
          o[n][0] *= al0;
          o[n][1] *= al0;
          o[n][2] *= al1;
          o[n][3] *= al1;
        }
        const uint32_t pa[4] = {pack2<KV_DT>(p[0][0], p[0][1]), pack2<KV_DT>(p[0][2], p[0][3]),
                                pack2<KV_DT>(p[1][0], p[1][1]), pack2<KV_DT>(p[1][2], p[1][3])};
        // O += P V : pairs of 8-dim n-tiles
#pragma unroll
        for (int np = 0; np < D / 16; ++np) {
          const int t = ((mi & 1) << 3) + rr;
          const int chunk = 2 * np + (mi >> 1);
          const uint32_t addr = vaddr + (chunk >> 3) * sub_bytes + (head_row0 + t) * kSubRowBytes +
                                (((chunk & 7) ^ (t & 7)) << 4);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_trans(addr, b0, b1, b2, b3);
          mma_16816<KV_DT>(o[2 * np], pa, b0, b1);
          mma_16816<KV_DT>(o[2 * np + 1], pa, b2, b3);
        }
      }
      __syncwarp();
      if (!SP && lane == 0) mbar_arrive(&sm.empty[st]);
    }

    // ---- finalize this (sequence, head) partial ------------------------------------
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const long long slot =
        balanced ? s + (long long)blockIdx.x * streams + my
                 : s * a.plan.splits + (blockIdx.x - s * a.plan.splits);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = gid + 8 * half;
      if (r < a.rows) {
        const float l = half ? l1 : l0;
        const float m = half ? m1 : m0;
        const float inv = l > 0.f ? 1.f / l : 0.f;
        const int qi = r / a.group;
        const int qh = kh * a.group + (r - qi * a.group);
        const long long row = (slot * a.num_heads + qh) * a.q_len + qi;
        float* dst = a.part_o + row * D;
#pragma unroll
        for (int n = 0; n < D / 8; ++n) {
          const float2 v = make_float2(o[n][2 * half] * inv, o[n][2 * half + 1] * inv);
          *reinterpret_cast<float2*>(dst + n * 8 + 2 * tid4) = v;
        }
        if (tid4 == 0) a.part_lse[row] = l > 0.f ? (m + log2f(l)) * kLn2 : -INFINITY;
      }
    }
    cur = seg_end;
  }
  // The shorter stream releases the ring steps it has no block for.
  for (; streams == 2 && it < total; ++it) {
    const int st = (int)(it % nstages);
    if (!mbar_wait(&sm.full[st], (unsigned)((it / nstages) & 1))) {
      record_error(a.err, kErrWaitTimeout | kErrWaitData);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[st]);
  }
  if (SP) griddep_launch_dependents();
}

// Two KV heads per CTA (one if the head count is odd).  Measured on B200 for
// the Llama-3-8B decode shape: what limits a CTA is its single TMA-issuing
// producer, so several small CTAs per SM (each with its own producer and a
// 2-stage ring) stream faster than one wide CTA with a deep ring - 8 heads per
// CTA held at ~5.1 TB/s for any ring depth, 2 heads per CTA with 2 stages
// reached ~6.36 TB/s.
int choose_heads_per_cta(int kv_heads, int head_dim) {
  const int max_by_smem = (64 * 1024) / (2 * kBS * head_dim * 2);  // one stage <= 64 KB
  for (int h = 2; h >= 1; h >>= 1) {
    if (h <= max_by_smem && kv_heads % h == 0) return h;
  }
  return 1;
}

template <int D, int Q_DT, int KV_DT>
const void* kernel_ptr(bool sp, bool st) {
  if (sp) return reinterpret_cast<const void*>(&decode_tma_kernel<D, Q_DT, KV_DT, true, false>);
  if (st) return reinterpret_cast<const void*>(&decode_tma_kernel<D, Q_DT, KV_DT, false, true>);
  return reinterpret_cast<const void*>(&decode_tma_kernel<D, Q_DT, KV_DT, false, false>);
}

const void* select_kernel(const AttnArgs& a, bool sp = false, bool st = false) {
#define LLMOPT_DECODE_CASE(DV, QT, KT) \
  if (a.head_dim == DV && a.q_dtype == QT && a.kv_dtype == KT) return kernel_ptr<DV, QT, KT>(sp, st);
#define LLMOPT_DECODE_Q(DV, KT)     \
  LLMOPT_DECODE_CASE(DV, kF32, KT)  \
  LLMOPT_DECODE_CASE(DV, kF16, KT)  \
  LLMOPT_DECODE_CASE(DV, kBF16, KT)
  LLMOPT_DECODE_Q(64, kBF16)
  LLMOPT_DECODE_Q(128, kBF16)
  LLMOPT_DECODE_Q(256, kBF16)
  LLMOPT_DECODE_Q(64, kF16)
  LLMOPT_DECODE_Q(128, kF16)
  LLMOPT_DECODE_Q(256, kF16)
#undef LLMOPT_DECODE_Q
#undef LLMOPT_DECODE_CASE
  return nullptr;
}

size_t smem_bytes_for(int hpc, int head_dim, int stages, long long prefix_entries) {
  const size_t stage = 2ull * hpc * kBS * head_dim * 2;
  return 1024 + stage * stages + stages * (8 + 8 + 2 * 4) + (size_t)prefix_entries * 4 + 16;
}

}  // namespace

bool decode_tma_supported(const AttnArgs& a) {
  if (a.kv_dtype != kBF16 && a.kv_dtype != kF16) return false;
  if (a.block_size != kBS) return false;
  if (a.head_dim != 64 && a.head_dim != 128 && a.head_dim != 256) return false;
  if (a.rows > 16 || a.rows < 1) return false;
  if ((reinterpret_cast<uintptr_t>(a.k_cache) & 15) || (reinterpret_cast<uintptr_t>(a.v_cache) & 15))
    return false;
  if ((long long)a.num_blocks * kBS > 0x7fffffffLL) return false;
  if (a.plan.mode == kModeBalanced && a.batch > kMaxPrefixBatch) return false;
  return select_kernel(a) != nullptr;
}

// Optional tuning overrides (LLMOPT_B200_DECODE_HPC: KV heads per CTA,
// LLMOPT_B200_DECODE_SP: 0/1 self-issuing single-head CTAs,
// LLMOPT_B200_DECODE_STAGES: ring depth); invalid values are ignored.
int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return (v != nullptr && *v != '\0') ? std::atoi(v) : dflt;
}

bool decode_tma_configure(const AttnArgs& a, int sm_count, DecodeLaunch* launch) {
  int hpc = choose_heads_per_cta(a.kv_heads, a.head_dim);
  const int hpc_env = env_int("LLMOPT_B200_DECODE_HPC", 0);
  if (hpc_env >= 1 && hpc_env <= kMaxBoxHeads && a.kv_heads % hpc_env == 0 &&
      2ull * hpc_env * kBS * a.head_dim * 2 <= 64 * 1024) {
    hpc = hpc_env;
  }
  // One KV head (a rank's shard of 8 heads over 8 GPUs): two streams of the
  // balanced plan per CTA in the two-head layout, or (LLMOPT_B200_DECODE_SP=1,
  // and for fixed plans) self-issuing one-warp CTAs.
  bool sp = hpc == 1;
  const int sp_env = env_int("LLMOPT_B200_DECODE_SP", -1);
  if (sp_env == 0 || sp_env == 1) sp = sp_env == 1;
  if (hpc != 1 || a.head_dim > 128) sp = false;   // head_dim 256 would spill at its bound
  int streams = 1;
  if (hpc == 1 && a.plan.mode == kModeBalanced && sp_env != 1 &&
      2ull * 2 * kBS * a.head_dim * 2 <= 64 * 1024) {
    streams = 2;
    sp = false;
  }
  const int box_heads = hpc * streams;          // head slots of the ring layout
  const void* fn = select_kernel(a, sp, streams == 2);
  if (fn == nullptr) return false;
  const long long prefix_entries = a.plan.mode == kModeBalanced ? a.batch + 1 : 0;
  // Double buffering per CTA; parallelism comes from several CTAs per SM.
  int stages = env_int("LLMOPT_B200_DECODE_STAGES", 2);
  if (stages < 2) stages = 2;
  if (stages > 16) stages = 16;
  size_t smem = smem_bytes_for(box_heads, a.head_dim, stages, prefix_entries);
  while (smem > 227 * 1024 && stages > 2) {
    --stages;
    smem = smem_bytes_for(box_heads, a.head_dim, stages, prefix_entries);
  }
  if (smem > 227 * 1024) return false;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess ||
      ensure_max_shared_carveout(fn) != cudaSuccess) {
    return false;
  }
  int occ = 0;
  const int threads = sp ? 32 : (box_heads + 1) * 32;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, threads, smem) != cudaSuccess ||
      occ < 1) {
    return false;
  }
  launch->heads_per_cta = hpc;
  launch->streams = streams;
  launch->self_issue = sp ? 1 : 0;
  launch->stages = stages;
  launch->ctas_per_sm = occ;
  launch->smem_bytes = smem;
  (void)sm_count;
  return true;
}

cudaError_t decode_tma_launch(const AttnArgs& a, const DecodeLaunch& launch,
                              const CUtensorMap& tmk, const CUtensorMap& tmv,
                              cudaStream_t stream) {
  const void* fn = select_kernel(a, launch.self_issue != 0, launch.streams == 2);
  if (fn == nullptr) return cudaErrorInvalidValue;
  const int head_groups = a.kv_heads / launch.heads_per_cta;
  const int streams = launch.streams == 2 ? 2 : 1;
  if (a.plan.mode == kModeBalanced && a.plan.ctas % streams != 0) return cudaErrorInvalidValue;
  const long long gx = a.plan.mode == kModeBalanced ? a.plan.ctas / streams
                                                    : a.batch * (long long)a.plan.splits;
  if (gx <= 0) return cudaSuccess;
  if (gx > 0x7fffffffLL || head_groups > 65535) return cudaErrorInvalidConfiguration;
  dim3 grid((unsigned)gx, (unsigned)head_groups);
  int hpc = launch.heads_per_cta * streams;    // head slots of the ring layout
  dim3 block(launch.self_issue ? 32 : (hpc + 1) * 32);
  int stages = launch.stages;
  void* args[] = {const_cast<CUtensorMap*>(&tmk), const_cast<CUtensorMap*>(&tmv),
                  const_cast<AttnArgs*>(&a), &hpc, &stages};
  return launch_pdl(fn, grid, block, args, launch.smem_bytes, stream);
}

}  // namespace llmopt
