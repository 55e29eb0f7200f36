// Paged decode attention over an e4m3 (FP8) KV cache, sm_100a.
//
// FP8 KV storage is beyond the reference, which only names the dtypes
// (src/llmopt/utils/misc.py:33-34, 57).  The cache keeps the reference's
// [layers, num_blocks, block_size, kv_heads, head_dim] layout with one e4m3
// code per element, plus one fp32 scale per (token, head) row in a
// [layers, num_blocks, kv_heads, block_size] array: value = code * scale.
// The attention semantics are PagedAttention.forward's
// (src/llmopt/attention/paged_attention.py:146-293) on those values, with the
// query rounded to f16.  Half the bytes of a bf16 cache cross HBM per token,
// plus 4 bytes of scale per 128-byte row.
//
// Data movement: the same split plan (plan.cuh), CTA shape (one producer warp,
// one consumer warp per KV head of the CTA) and stage ring as the bf16 kernel
// (decode_tma.cu).  Per block and head the producer issues one TMA box of
// (128 codes, 1 head, 16 tokens) per 128-dim slice of K and of V - rows of 128
// bytes with the 128-byte swizzle, laid out [slice][head][token] - and one
// bulk copy each for the K and V scales of the CTA's heads (contiguous in the
// [.., kv_heads, block_size] scale layout).
//
// Math: m16n8k16 f16 MMAs with fp32 accumulation, transposed against the
// bf16 kernel: the 16 tokens of a block are the M dimension and the query
// rows of the KV head (q_len * group, 4 for Llama-3 decode) the N dimension,
// 8 per n-tile, so a block costs D/16 MMAs for S and D/16 for O instead of
// twice that with rows padded to 16.  e4m3 -> f16 is exact, so the only
// roundings beyond the fp32 reference are the query's (to f16) and the
// probabilities' (to f16).  Fragments come from shared memory in 16-byte
// loads that hit eight different bank groups per quarter warp:
// * S^T = K Q^T: lane (g, t) reads tokens g and g + 8, dims 32t..32t+31 of
//   each 128-dim slice; k-step (slice u, word w) uses dims 128u + 32t + 4w .. +3
//   and the query fragments follow the same dim order (a dot product does not
//   care which k-slot holds which dim).  The token's K scale multiplies the
//   fp32 scores.
// * O^T += V^T P^T: lane (g, t) reads tokens 2t, 2t+1, 2t+8, 2t+9, dims
//   16g..16g+15 of each slice, and byte-permutes token pairs of one dim into
//   the A fragment: m-slots g and g + 8 of m-tile j of slice u are dims
//   128u + 16g + 2j and + 1, so each lane ends with 16 contiguous output dims
//   of its two query rows per slice.  The V scales multiply the probabilities
//   before the f16 cast (the row sums use the unscaled ones), and
//   movmatrix.trans turns the S^T accumulator layout into the B fragments.
// Partials (normalised O, natural-log LSE) go to the split workspace in the
// bf16 kernel's format; combine.cu merges them.
#include <float.h>

#include <cstdlib>

#include "common.cuh"
#include "kernels.h"

namespace llmopt {
namespace {

constexpr int kBS = 16;            // tokens per KV block on this path
constexpr int kSlice = 128;        // dims (= bytes) per TMA box row, the swizzle span
constexpr int kMaxHeads = 8;       // consumer warps per CTA
// head_dim 256 holds twice the accumulators: at most 4 heads (5 warps) per CTA
// lets the register allocator give a thread 255 registers instead of 168.
constexpr int max_heads(int d) { return d == 256 ? 4 : kMaxHeads; }
constexpr long long kMaxPrefixBatch = 4096;

struct Smem {
  unsigned char* stages;  // [stage][K | V][slice][head][token][128 B]
  float* scales;          // [stage][K | V][head][token]
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

// Untiled bulk copy global -> this CTA's shared memory, completing on `bar`
// (both addresses 16-byte aligned, bytes a multiple of 16).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, unsigned bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes),
      "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ uint4 lds128(const unsigned char* p) {
  return *reinterpret_cast<const uint4*>(p);
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Query fragments (the B operand of S^T = K Q^T) in the kernel's dim order:
// n-tile nt holds query rows 8nt..8nt+7 (row 8nt + g in lane g); k-step
// ks = 8u + w covers dims 128u + 32t + 4w + {0,1} (b0) and {2,3} (b1).
template <int D, int Q_DT, int NT>
__device__ __forceinline__ void load_qt_frags(const AttnArgs& a, long long s, int kh, int gid,
                                              int tid4, uint32_t (&qb)[NT][D / 16][2]) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int r = 8 * nt + gid;
    const bool ok = r < a.rows;
    long long base = 0;
    if (ok) {
      const int qi = r / a.group;
      const int gi = r - qi * a.group;
      base = s * a.q_s + (long long)(kh * a.group + gi) * a.q_h + (long long)qi * a.q_t;
    }
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const int d = (ks >> 3) * kSlice + 32 * tid4 + 4 * (ks & 7);
#pragma unroll
      for (int pr = 0; pr < 2; ++pr) {
        float x0 = 0.f, x1 = 0.f;
        if (ok) {
          x0 = load_f32<Q_DT>(a.q, base + d + 2 * pr);
          x1 = load_f32<Q_DT>(a.q, base + d + 2 * pr + 1);
        }
        qb[nt][ks][pr] = pack2<kF16>(x0, x1);
      }
    }
  }
}

// Transpose an 8x8 matrix of 16-bit pairs held in the MMA fragment layout
// (lane holds row lane/4, columns 2(lane%4) and +1) across the warp.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// Register cap per thread.  One n-tile at head_dim 128 fits 112 registers
// without spilling (128 with the self-issue state): 16 one-warp CTAs, or
// three of the default 5-warp CTAs, per SM.
constexpr int reg_cap(int d, int nt, bool sp) {
  return d == 256 ? 255 : (nt == 1 ? (sp ? 128 : 112) : 168);
}

template <int D, int Q_DT, int NT, bool SP>
__global__ void __launch_bounds__(SP ? 32 : (max_heads(D) + 1) * 32) __maxnreg__(reg_cap(D, NT, SP))
    decode_fp8_kernel(const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmv, const AttnArgs a, const int hpc,
                      const int nstages) {
  // Dependent-launch trigger as the bf16 kernel: at the start with a producer
  // warp, at the end for self-issuing one-warp CTAs.
  griddep_wait();
  if (!SP) griddep_launch_dependents();
  constexpr int kSlices = D / kSlice;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long batch = a.batch;
  const bool balanced = a.plan.mode == kModeBalanced;
  const int slice_bytes = hpc * kBS * kSlice;       // one 128-dim slice of one block
  const int half_bytes = kSlices * slice_bytes;     // K (or V) codes of one block
  const int stage_bytes = 2 * half_bytes;
  const int scale_floats = hpc * kBS;               // K (or V) scales of one block

  extern __shared__ unsigned char smem_raw[];
  Smem sm;
  {
    uintptr_t p = (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023);
    sm.stages = reinterpret_cast<unsigned char*>(p);
    sm.scales = reinterpret_cast<float*>(sm.stages + (size_t)nstages * stage_bytes);
    sm.full = reinterpret_cast<uint64_t*>(sm.scales + (size_t)nstages * 2 * scale_floats);
    sm.empty = sm.full + nstages;
    sm.meta = reinterpret_cast<int*>(sm.empty + nstages);
    sm.prefix = sm.meta + nstages;
  }

  // ---- this CTA's block range (the bf16 kernel's plan) ------------------------
  long long lo = 0, hi = 0, fixed_seq = -1;
  if (balanced) {
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
    __shared__ int warp_tot[kMaxHeads + 1];
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
    lo = range_start(blockIdx.x, total, a.plan.ctas);
    hi = range_start(blockIdx.x + 1, total, a.plan.ctas);
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

  const int kh0 = blockIdx.y * hpc;
  const long long total = hi - lo;

  // Block `idx` of this CTA's range: its table entry and valid-token count
  // (ntok 0: not loaded).
  auto resolve = [&](long long idx, int* id, int* ntok) {
    *id = 0;
    *ntok = 0;
    if (idx >= total) return;
    const long long f = lo + idx;
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
    if (raw >= a.num_blocks) {
      record_error(a.err, kErrBlockId);
    } else if (raw >= 0) {
      *id = (int)raw;
      *ntok = left < kBS ? (int)left : kBS;
    }
  };
  // Stage st <- block id (codes of the CTA's heads and their scales); one thread.
  auto fill_stage = [&](int st, int id_i, int nt_i) {
    sm.meta[st] = nt_i;
    if (nt_i > 0) {
      unsigned char* kdst = sm.stages + (size_t)st * stage_bytes;
      unsigned char* vdst = kdst + half_bytes;
      float* sdst = sm.scales + (size_t)st * 2 * scale_floats;
      mbar_arrive_expect_tx(&sm.full[st],
                            (unsigned)(stage_bytes + 2 * scale_floats * sizeof(float)));
#pragma unroll
      for (int sl = 0; sl < kSlices; ++sl) {
        for (int h = 0; h < hpc; ++h) {
          const int off = sl * slice_bytes + h * kBS * kSlice;
          tma_load_5d(kdst + off, &tmk, &sm.full[st], sl * kSlice, kh0 + h, 0, id_i, a.layer);
          tma_load_5d(vdst + off, &tmv, &sm.full[st], sl * kSlice, kh0 + h, 0, id_i, a.layer);
        }
      }
      const long long sidx = (((long long)a.layer * a.num_blocks + id_i) * a.kv_heads + kh0) * kBS;
      bulk_load(sdst, a.k_scale + sidx, (unsigned)(scale_floats * sizeof(float)), &sm.full[st]);
      bulk_load(sdst + scale_floats, a.v_scale + sidx, (unsigned)(scale_floats * sizeof(float)),
                &sm.full[st]);
    } else {
      mbar_arrive(&sm.full[st]);
    }
  };

  // ---- producer warp ------------------------------------------------------------
  if (!SP && warp == hpc) {
    if (lane == 0) {
      prefetch_tensormap(&tmk);
      prefetch_tensormap(&tmv);
    }
    for (long long base = 0; base < total; base += 32) {
      // Each lane resolves one block: its table entry and valid-token count.
      int id, ntok;
      resolve(base + lane, &id, &ntok);
      const int cnt = total - base < 32 ? (int)(total - base) : 32;
      for (int i = 0; i < cnt; ++i) {
        const int id_i = __shfl_sync(0xffffffffu, id, i);
        const int nt_i = __shfl_sync(0xffffffffu, ntok, i);
        if (lane == 0) {
          const long long it = base + i;
          const int st = (int)(it % nstages);
          const long long round = it / nstages;
          if (round > 0 && !mbar_wait(&sm.empty[st], (unsigned)((round - 1) & 1))) {
            record_error(a.err, kErrWaitTimeout | kErrWaitSlot);
          }
          fill_stage(st, id_i, nt_i);
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

  // ---- consumer warps: one KV head each ----------------------------------------
  constexpr int KS = D / 16;   // k-steps of S^T = m-tiles of O^T
  const int hh = warp;
  const int kh = kh0 + hh;
  const int gid = lane >> 2;
  const int tid4 = lane & 3;
  const float scale_log2 = a.scale * kLog2e;
  const bool capped = a.softcap > 0.f;

  // Self-issuing: blocks [0, issued) have been issued; lane l caches the table
  // entry of block cache_base + l.  Every issued block is consumed (waited on)
  // before the warp exits, so no copy is in flight when it returns.
  long long issued = 0;
  long long cache_base = -32;
  int c_id = 0, c_nt = 0;
  auto issue_upto = [&](long long limit) {
    if (limit > total) limit = total;
    while (issued < limit) {
      if (issued >= cache_base + 32) {
        cache_base = issued;
        resolve(cache_base + lane, &c_id, &c_nt);
      }
      const int k = (int)(issued - cache_base);
      const int id_i = __shfl_sync(0xffffffffu, c_id, k);
      const int nt_i = __shfl_sync(0xffffffffu, c_nt, k);
      // The stage's previous block has been read (and its V rows maybe zeroed)
      // by this warp: order those accesses before the copies that overwrite it.
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      if (lane == 0) fill_stage((int)(issued % nstages), id_i, nt_i);
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
  long long cur = lo;
  while (cur < hi) {
    long long s, seg_begin, seg_end;
    if (balanced) {
      s = find_seq(sm.prefix, batch, cur);
      seg_begin = sm.prefix[s];
      seg_end = sm.prefix[s + 1] < hi ? sm.prefix[s + 1] : hi;
    } else {
      s = fixed_seq;
      seg_begin = 0;
      seg_end = hi;
    }
    const long long ctx_s = load_index(a.ctx, a.ctx_i64, s);
    uint32_t qb[NT][KS][2];
    load_qt_frags<D, Q_DT, NT>(a, s, kh, gid, tid4, qb);
    // Causal limit of this lane's rows 8nt + 2t + j (only used when q_len > 1).
    long long qpos[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        qpos[nt][j] = ctx_s - a.q_len + (8 * nt + 2 * tid4 + j) / a.group;
      }
    }

    float m[NT][2], l[NT][2];
    float o[NT][KS][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m[nt][0] = m[nt][1] = -INFINITY;
      l[nt][0] = l[nt][1] = 0.f;
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) o[nt][mt][0] = o[nt][mt][1] = o[nt][mt][2] = o[nt][mt][3] = 0.f;
    }

    for (long long f = cur; f < seg_end; ++f, ++it) {
      // Self-issuing: keep nstages - 1 blocks in flight beyond this one.
      if (SP) issue_upto(it + nstages);
      const int st = (int)(it % nstages);
      if (!mbar_wait(&sm.full[st], (unsigned)((it / nstages) & 1))) {
        record_error(a.err, kErrWaitTimeout | kErrWaitData);
      }
      const int ntok = sm.meta[st];
      if (ntok > 0) {
        unsigned char* kst = sm.stages + (size_t)st * stage_bytes + hh * kBS * kSlice;
        unsigned char* vst = kst + half_bytes;
        const float* kscale = sm.scales + (size_t)st * 2 * scale_floats + hh * kBS;
        const float* vscale = kscale + scale_floats;
        if (ntok < kBS) {
          // Slots past the context hold stale codes (possibly NaN): zero this
          // head's V rows so a zero probability never meets them.
          for (int e = lane; e < (kBS - ntok) * kSlices * 8; e += 32) {
            const int t = ntok + e / (kSlices * 8);
            const int rest = e % (kSlices * 8);
            *reinterpret_cast<uint4*>(vst + (rest >> 3) * slice_bytes + t * kSlice +
                                      ((rest & 7) << 4)) = make_uint4(0u, 0u, 0u, 0u);
          }
          // Order these generic-proxy stores before the TMA that refills the stage.
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
        }

        // S^T = K Q^T: tokens g and g + 8 (A) against the query rows (B)
        float sacc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
#pragma unroll
        for (int sl = 0; sl < kSlices; ++sl) {
          uint4 kv[2][2];
#pragma unroll
          for (int hl = 0; hl < 2; ++hl) {
            const int t = gid + 8 * hl;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              kv[hl][c] = lds128(kst + sl * slice_bytes + t * kSlice +
                                 (((2 * tid4 + c) ^ (t & 7)) << 4));
            }
          }
#pragma unroll
          for (int w = 0; w < 8; ++w) {
            uint32_t af[4];   // token g dims +0,+1 | token g+8 | token g dims +2,+3 | token g+8
            e4m3x4_to_f16x2x2(word_of(kv[0][w >> 2], w & 3), af[0], af[2]);
            e4m3x4_to_f16x2x2(word_of(kv[1][w >> 2], w & 3), af[1], af[3]);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              mma_16816<kF16>(sacc[nt], af, qb[nt][sl * 8 + w][0], qb[nt][sl * 8 + w][1]);
            }
          }
        }

        // K scale, softmax scale / softcap, mask (log2 units); element e of
        // n-tile nt: token g + 8 (e >> 1), query row 8nt + 2t + (e & 1)
        const long long kbase = (f - seg_begin) * kBS;
        const float ksc[2] = {kscale[gid], kscale[gid + 8]};
        const float vsc[2] = {vscale[gid], vscale[gid + 8]};
        uint32_t pb[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          float p[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int tok = gid + 8 * (e >> 1);
            float x = sacc[nt][e] * ksc[e >> 1];
            x = capped ? tanhf(x * a.scale / a.softcap) * (a.softcap * kLog2e) : x * scale_log2;
            bool ok = tok < ntok;
            if (a.q_len > 1) ok = ok && (kbase + tok <= qpos[nt][e & 1]);
            p[e] = ok ? x : -INFINITY;
          }
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            float mx = fmaxf(p[j], p[2 + j]);
            mx = warp_max_xor(warp_max_xor(warp_max_xor(mx, 4), 8), 16);
            const float mn = fmaxf(m[nt][j], mx);
            const float mu = mn == -INFINITY ? 0.f : mn;
            const float al = fast_exp2(m[nt][j] - mu);
            p[j] = fast_exp2(p[j] - mu);
            p[2 + j] = fast_exp2(p[2 + j] - mu);
            l[nt][j] = l[nt][j] * al + (p[j] + p[2 + j]);
            m[nt][j] = mn;
#pragma unroll
            for (int mt = 0; mt < KS; ++mt) {
              o[nt][mt][j] *= al;
              o[nt][mt][2 + j] *= al;
            }
          }
          // V scales into the probabilities (masked tokens stay exactly 0), then
          // the [token][row] 8x8 halves transposed into [row][token] B fragments.
#pragma unroll
          for (int e = 0; e < 4; ++e) p[e] = p[e] > 0.f ? p[e] * vsc[e >> 1] : 0.f;
          pb[nt][0] = movmatrix_trans(pack2<kF16>(p[0], p[1]));   // tokens 2t, 2t+1
          pb[nt][1] = movmatrix_trans(pack2<kF16>(p[2], p[3]));   // tokens 2t+8, 2t+9
        }

        // O^T += V^T P^T: per slice, tokens (2t, 2t+1 | 2t+8, 2t+9) x dims 16g..16g+15
#pragma unroll
        for (int sl = 0; sl < kSlices; ++sl) {
          uint4 rv[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int t = 2 * tid4 + (k & 1) + 8 * (k >> 1);
            rv[k] = lds128(vst + sl * slice_bytes + t * kSlice + ((gid ^ (t & 7)) << 4));
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t lo01 = __byte_perm(word_of(rv[0], q), word_of(rv[1], q), 0x5140);
            const uint32_t lo23 = __byte_perm(word_of(rv[0], q), word_of(rv[1], q), 0x7362);
            const uint32_t hi01 = __byte_perm(word_of(rv[2], q), word_of(rv[3], q), 0x5140);
            const uint32_t hi23 = __byte_perm(word_of(rv[2], q), word_of(rv[3], q), 0x7362);
            // m-tile 2q: dims 16g + 4q (m-slot g) and + 1 (m-slot g + 8);
            // m-tile 2q + 1: dims 16g + 4q + 2 and + 3
            uint32_t a0[4], a1[4];
            e4m3x4_to_f16x2x2(lo01, a0[0], a0[1]);
            e4m3x4_to_f16x2x2(hi01, a0[2], a0[3]);
            e4m3x4_to_f16x2x2(lo23, a1[0], a1[1]);
            e4m3x4_to_f16x2x2(hi23, a1[2], a1[3]);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              mma_16816<kF16>(o[nt][sl * 8 + 2 * q], a0, pb[nt][0], pb[nt][1]);
              mma_16816<kF16>(o[nt][sl * 8 + 2 * q + 1], a1, pb[nt][0], pb[nt][1]);
            }
          }
        }
      }
      __syncwarp();
      if (!SP && lane == 0) mbar_arrive(&sm.empty[st]);
    }

    // ---- finalize this (sequence, head) partial ------------------------------------
    const long long slot =
        balanced ? s + blockIdx.x : s * a.plan.splits + (blockIdx.x - s * a.plan.splits);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float lt = l[nt][j];
        lt += __shfl_xor_sync(0xffffffffu, lt, 4);
        lt += __shfl_xor_sync(0xffffffffu, lt, 8);
        lt += __shfl_xor_sync(0xffffffffu, lt, 16);
        const int r = 8 * nt + 2 * tid4 + j;
        if (r < a.rows) {
          const float inv = lt > 0.f ? 1.f / lt : 0.f;
          const int qi = r / a.group;
          const int qh = kh * a.group + (r - qi * a.group);
          const long long row = (slot * a.num_heads + qh) * a.q_len + qi;
          float* dst = a.part_o + row * D;
#pragma unroll
          for (int sl = 0; sl < kSlices; ++sl) {
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4) {   // dims 16g + 4 v4 .. + 3 of the slice
              const int mt = sl * 8 + 2 * v4;
              const float4 v = make_float4(o[nt][mt][j] * inv, o[nt][mt][2 + j] * inv,
                                           o[nt][mt + 1][j] * inv, o[nt][mt + 1][2 + j] * inv);
              *reinterpret_cast<float4*>(dst + sl * kSlice + 16 * gid + 4 * v4) = v;
            }
          }
          if (gid == 0) {
            a.part_lse[row] = lt > 0.f ? (m[nt][j] + log2f(lt)) * kLn2 : -INFINITY;
          }
        }
      }
    }
    cur = seg_end;
  }
  if (SP) griddep_launch_dependents();
}

template <int D, int Q_DT>
const void* fp8_kernel_ptr(int rows, bool sp) {
  if (sp) {
    return rows <= 8 ? reinterpret_cast<const void*>(&decode_fp8_kernel<D, Q_DT, 1, true>)
                     : reinterpret_cast<const void*>(&decode_fp8_kernel<D, Q_DT, 2, true>);
  }
  return rows <= 8 ? reinterpret_cast<const void*>(&decode_fp8_kernel<D, Q_DT, 1, false>)
                   : reinterpret_cast<const void*>(&decode_fp8_kernel<D, Q_DT, 2, false>);
}

const void* select_fp8_kernel(const AttnArgs& a, bool sp = false) {
#define LLMOPT_FP8_CASE(DV, QT) \
  if (a.head_dim == DV && a.q_dtype == QT) return fp8_kernel_ptr<DV, QT>(a.rows, sp);
  LLMOPT_FP8_CASE(128, kF32)
  LLMOPT_FP8_CASE(128, kF16)
  LLMOPT_FP8_CASE(128, kBF16)
  LLMOPT_FP8_CASE(256, kF32)
  LLMOPT_FP8_CASE(256, kF16)
  LLMOPT_FP8_CASE(256, kBF16)
#undef LLMOPT_FP8_CASE
  return nullptr;
}

size_t fp8_smem_bytes(int hpc, int head_dim, int stages, long long prefix_entries) {
  const size_t stage = 2ull * hpc * kBS * head_dim;          // K + V codes
  const size_t scales = 2ull * hpc * kBS * sizeof(float);    // K + V scales
  return 1024 + (stage + scales) * stages + stages * (8 + 8 + 4) +
         (size_t)prefix_entries * 4 + 16;
}

int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return (v != nullptr && *v != '\0') ? std::atoi(v) : dflt;
}

}  // namespace

bool decode_fp8_supported(const AttnArgs& a) {
  if (a.kv_dtype != kE4M3 || a.block_size != kBS) return false;
  if (a.head_dim != 128 && a.head_dim != 256) return false;
  if (a.rows > 16 || a.rows < 1) return false;
  for (const void* p : {a.k_cache, a.v_cache, static_cast<const void*>(a.k_scale),
                        static_cast<const void*>(a.v_scale)}) {
    if (p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15)) return false;
  }
  if ((long long)a.num_blocks * kBS > 0x7fffffffLL) return false;
  if (a.plan.mode == kModeBalanced && a.batch > kMaxPrefixBatch) return false;
  return select_fp8_kernel(a) != nullptr;
}

// KV heads per CTA, self-issuing one-warp CTAs, ring depth
// (LLMOPT_B200_FP8_HPC / LLMOPT_B200_FP8_SP / LLMOPT_B200_FP8_STAGES override
// them; invalid values are ignored).
bool decode_fp8_configure(const AttnArgs& a, int sm_count, DecodeLaunch* launch) {
  int hpc = a.kv_heads % 4 == 0 ? 4 : (a.kv_heads % 2 == 0 ? 2 : 1);
  const int hpc_env = env_int("LLMOPT_B200_FP8_HPC", 0);
  if (hpc_env >= 1 && hpc_env <= max_heads(a.head_dim) && a.kv_heads % hpc_env == 0) {
    hpc = hpc_env;
  }
  bool sp = hpc == 1;
  const int sp_env = env_int("LLMOPT_B200_FP8_SP", -1);
  if (sp_env == 0 || sp_env == 1) sp = sp_env == 1;
  if (sp) hpc = 1;                      // one warp = one KV head
  const void* fn = select_fp8_kernel(a, sp);
  if (fn == nullptr) return false;
  const long long prefix_entries = a.plan.mode == kModeBalanced ? a.batch + 1 : 0;
  int stages = env_int("LLMOPT_B200_FP8_STAGES", 3);
  if (stages < 2) stages = 2;
  if (stages > 16) stages = 16;
  size_t smem = fp8_smem_bytes(hpc, a.head_dim, stages, prefix_entries);
  while (smem > 227 * 1024 && stages > 2) {
    --stages;
    smem = fp8_smem_bytes(hpc, a.head_dim, stages, prefix_entries);
  }
  if (smem > 227 * 1024) return false;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess ||
      ensure_max_shared_carveout(fn) != cudaSuccess) {
    return false;
  }
  int occ = 0;
  const int threads = sp ? 32 : (hpc + 1) * 32;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, threads, smem) != cudaSuccess ||
      occ < 1) {
    return false;
  }
  launch->heads_per_cta = hpc;
  launch->streams = 1;
  launch->self_issue = sp ? 1 : 0;
  launch->stages = stages;
  launch->ctas_per_sm = occ;
  launch->smem_bytes = smem;
  (void)sm_count;
  return true;
}

cudaError_t decode_fp8_launch(const AttnArgs& a, const DecodeLaunch& launch,
                              const CUtensorMap& tmk, const CUtensorMap& tmv,
                              cudaStream_t stream) {
  const void* fn = select_fp8_kernel(a, launch.self_issue != 0);
  if (fn == nullptr) return cudaErrorInvalidValue;
  const int head_groups = a.kv_heads / launch.heads_per_cta;
  const long long gx =
      a.plan.mode == kModeBalanced ? a.plan.ctas : a.batch * (long long)a.plan.splits;
  if (gx <= 0) return cudaSuccess;
  if (gx > 0x7fffffffLL || head_groups > 65535) return cudaErrorInvalidConfiguration;
  dim3 grid((unsigned)gx, (unsigned)head_groups);
  dim3 block(launch.self_issue ? 32 : (launch.heads_per_cta + 1) * 32);
  int hpc = launch.heads_per_cta;
  int stages = launch.stages;
  void* args[] = {const_cast<CUtensorMap*>(&tmk), const_cast<CUtensorMap*>(&tmv),
                  const_cast<AttnArgs*>(&a), &hpc, &stages};
  return launch_pdl(fn, grid, block, args, launch.smem_bytes, stream);
}

}  // namespace llmopt
