// Chunked-prefill paged attention, two query tiles per CTA in ping-pong
// (sm_100a, tcgen05 tensor cores + TMA).
//
// Replaces PagedAttention.forward for q_len > 1 (src/llmopt/attention/
// paged_attention.py:146-250: gather, h // group expansion, causal mask
// k_pos <= ctx - q_len + i, softmax, P V) when the query rows of one KV head
// form a real dense contraction (q_len * group > 16) on a 16-bit cache, like
// prefill_tc.cu, with a schedule built for the tensor core to stay busy:
//
// * A CTA owns two query tiles of 128 rows (rows ordered [head][token]; tile q
//   holds chunk tokens [t0 + q tq, t0 + (q + 1) tq), tq = 128 / group) of one
//   (sequence, KV head), and walks the keys in tiles of 128 (8 KV blocks).
//   One CTA per SM.
// * Tensor memory (all 512 columns): S of tile q at columns [128 q, 128 q + 128),
//   its probabilities P written by the softmax over the first 64 of them, and
//   O of tile q at [256 + 128 q, 256 + 128 q + head_dim).
// * The MMA thread issues, per key tile j: P0(j) V(j), then S0(j+1) = Q0 K(j+1)^T
//   (tensor-core operations of one thread run in issue order, so the product
//   reads P0(j) before the next S0 overwrites it), then the same for tile 1.
//   While softmax group 0 turns S0 into P0, the tensor core computes P1 V and
//   the next S1, and the other way round: the exponentials of one tile hide
//   behind the matrix products of the other.
// * Optionally a quarter or half of the exponentials run as a polynomial on the
//   FMA pipe (exp2_poly) instead of the special-function unit (measured slower
//   on B200 for this kernel, so off by default).
// * Warps: 0-3 softmax of tile 0, 4-7 softmax of tile 1 (one thread per row =
//   tensor-memory lane, a score row of 128 fp32 values in registers), 8 K
//   loader (Q once, then K tiles through the block table: 5-D map over the
//   cache, one 16-token box per block and 64-dim slice, -1 entries not loaded),
//   9 V loader, 10 MMA issuer (also zeroes V rows that hold no valid key, so a
//   zero probability never meets Inf/NaN).  With 11 warps, three share an SM
//   sub-partition, which caps a thread at 168 registers: the probabilities are
//   packed and stored 32 columns at a time to stay inside it.
// * The O rescale of the lazy online softmax (O is rescaled only when a row's
//   running max grows by more than 2^8) needs no extra wait: S(j) is committed
//   after every earlier product of the MMA thread, P(j-1) V(j-1) included.
// * CTAs take their sequences longest context first (ranked in the kernel for
//   batches of up to kRankBatch), so the long items start in the first wave.
//
// Every wait is bounded (the first that gives up makes the CTA's other waits
// return at once, producers drain what they issued, and the MMA thread waits
// for its products before tensor memory is released).
#include <float.h>

#include <cstdlib>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace llmopt {
namespace {

constexpr int kBS = 16;
constexpr int kM = 128;                   // rows per query tile = TMEM lanes
constexpr int kN = 128;                   // keys per K/V tile
constexpr int kBlocksPerTile = kN / kBS;  // 8
constexpr int kKStages = 2;               // K ring depth
constexpr int kVStages = 3;               // V ring depth (a V stage is held for a whole
                                          // key tile: both tiles' P V products read it)
constexpr int kBitsRing = 8;              // tile valid-block bits, indexed tile % 8
constexpr int kKWarp = 8;
constexpr int kVWarp = 9;
constexpr int kMmaWarp = 10;
constexpr int kThreads = 11 * 32;
constexpr int kQSub = kM * 128;           // 128 rows x 64 dims, 128-byte swizzled (16 KB)
constexpr int kKVSub = kN * 128;          // 128 keys x 64 dims (16 KB)
constexpr int kBlockBytes = kBS * 128;    // one 16-row box (2 KB)
constexpr float kRescaleLog2 = 8.0f;
constexpr uint32_t kTmemCols = 512;
constexpr int kRankBatch = 256;           // longest-first ordering up to this batch

template <int D>
struct Layout {
  static constexpr int kSubs = D / 64;
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + 2 * kSubs * kQSub;
  static constexpr int kV = kK + kKStages * kSubs * kKVSub;
  static constexpr int kBar = kV + kVStages * kSubs * kKVSub;
  static constexpr int kBytes = kBar + 512;
};
static_assert(Layout<128>::kBytes <= 227 * 1024, "shared memory");

struct Bars {
  uint64_t q_full;
  uint64_t k_full[kKStages];
  uint64_t k_empty[kKStages];
  uint64_t v_full[kVStages];
  uint64_t v_empty[kVStages];
  uint64_t bits_full[2];   // s_bits[j % 2] valid for key tile j
  uint64_t s_full[2];      // S(q, j) in TMEM: phase j of tile q's barrier
  uint64_t p_full[2];      // P(q, j) in TMEM (128 arrivals)
  uint64_t o_final[2];     // every P V product of tile q complete
  uint64_t mma_done;       // every product of the CTA complete (before TMEM is freed)
  uint32_t tmem_base;
  uint32_t abort;          // set by the first wait that gives up
  uint32_t tile_bits[kBitsRing];
  uint32_t s_bits[2];
  int seq;
};
static_assert(sizeof(Bars) <= 512, "barrier block");

__device__ __forceinline__ void wait_or_flag(uint64_t* bar, unsigned parity, unsigned* err,
                                             uint32_t* abort) {
  if (*reinterpret_cast<volatile uint32_t*>(abort) != 0u) return;
  if (!mbar_wait(bar, parity)) {
    record_error(err, kErrWaitTimeout | kErrWaitData);
    *reinterpret_cast<volatile uint32_t*>(abort) = 1u;
  }
}

__device__ __forceinline__ void drain_wait(uint64_t* bar, unsigned parity, unsigned* err) {
  if (!mbar_wait(bar, parity)) record_error(err, kErrWaitTimeout | kErrWaitDrain);
}

// Coefficients of a degree-3 polynomial fitted to 2^f on [-0.5, 0.5] by
// iteratively reweighted least squares on the relative error (Lawson's
// algorithm); maximum relative error 8.4e-5 in float32 Horner form, far below
// the 2^-9 step of the 16-bit probabilities it feeds.
constexpr float kP0 = 0.999919593334198f;
constexpr float kP1 = 0.6932621598243713f;
constexpr float kP2 = 0.24271413683891296f;
constexpr float kP3 = 0.055212993174791336f;

// 2^x on the FMA pipe for x <= 2^22: x = n + f with n = round(x) taken from
// the low bits of x + 1.5 * 2^23, 2^f by the polynomial, n added to the
// exponent field.  Inputs below -126 (a masked -inf among them) give exactly
// 0, as the special-function unit does for -inf: a row that has seen no key
// keeps a zero sum and a zero output.
__device__ __forceinline__ float exp2_poly(float x) {
  const float xc = fmaxf(x, -126.f);
  const float t = xc + 12582912.f;
  const float n = t - 12582912.f;
  const float f = xc - n;
  float p = fmaf(kP3, f, kP2);
  p = fmaf(p, f, kP1);
  p = fmaf(p, f, kP0);
  const int ni = __float_as_int(t) - 0x4B400000;
  const float r = __int_as_float(__float_as_int(p) + (ni << 23));
  return x < -126.f ? 0.f : r;
}

// Columns c with (c & 7) >= 8 - POLY use the polynomial (POLY eighths of them).
template <int POLY>
__device__ __forceinline__ float exp2_mixed(float x, int c) {
  return (c & 7) >= 8 - POLY ? exp2_poly(x) : fast_exp2(x);
}

__device__ __forceinline__ long long tile_keys(const AttnArgs& a, long long ctx_s, int t_begin,
                                               int tq) {
  if (t_begin >= a.q_len) return 0;
  const int t_last = (t_begin + tq < a.q_len ? t_begin + tq : a.q_len) - 1;
  long long n = ctx_s - a.q_len + t_last + 1;
  if (n > ctx_s) n = ctx_s;
  if (n > a.table_width * kBS) n = a.table_width * kBS;
  return n < 0 ? 0 : n;
}

template <int D, int KV_DT, int POLY>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_fa_kernel(const __grid_constant__ CUtensorMap tmq,
                      const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmv, const AttnArgs a, int pf) {
  griddep_wait();
  griddep_launch_dependents();
  using L = Layout<D>;
  constexpr int kSubs = L::kSubs;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int group = a.group;
  const int tq = kM / group;                          // chunk tokens per query tile
  const int ctiles = (a.q_len + 2 * tq - 1) / (2 * tq);
  const long long per_seq = (long long)a.kv_heads * ctiles;
  const long long rank = blockIdx.x / per_seq;        // sequence by context length, longest first
  const int rem = (int)(blockIdx.x - rank * per_seq);
  const int ct = ctiles - 1 - rem / a.kv_heads;       // later chunk tiles (more keys) first
  const int kh = rem - (rem / a.kv_heads) * a.kv_heads;
  const int t0 = ct * 2 * tq;

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = smem_raw;
  Bars* bars = reinterpret_cast<Bars*>(sm + L::kBar);
  const bool misaligned = (smem_addr(sm) & 1023u) != 0;
  unsigned char* sQ = sm + L::kQ;
  unsigned char* sK = sm + L::kK;
  unsigned char* sV = sm + L::kV;

  if (threadIdx.x == 0) {
    bars->abort = 0u;
    bars->seq = (int)rank;
    mbar_init(&bars->q_full, 1);
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(&bars->k_full[i], 1);
      mbar_init(&bars->k_empty[i], 1);
    }
    for (int i = 0; i < kVStages; ++i) {
      mbar_init(&bars->v_full[i], 1);
      mbar_init(&bars->v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->bits_full[i], 1);
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], 128);
      mbar_init(&bars->o_final[i], 1);
    }
    mbar_init(&bars->mma_done, 1);
    mbar_init_fence();
  }
  if (warp == 0) {
    tc::tmem_alloc(&bars->tmem_base, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  // Longest context first: the sequence whose rank (descending context length,
  // ties by index) is this CTA's.  Larger batches keep the index order.
  if (a.batch <= kRankBatch && threadIdx.x < a.batch) {
    const long long mine = load_index(a.ctx, a.ctx_i64, threadIdx.x);
    long long r = 0;
    for (long long u = 0; u < a.batch; ++u) {
      const long long other = load_index(a.ctx, a.ctx_i64, u);
      r += (other > mine || (other == mine && u < (long long)threadIdx.x)) ? 1 : 0;
    }
    if (r == rank) bars->seq = (int)threadIdx.x;
  }
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = bars->tmem_base;
  const long long s = bars->seq;

  const long long ctx_s = load_index(a.ctx, a.ctx_i64, s);
  int n_q[2];
  long long keys_q[2];
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    keys_q[q] = tile_keys(a, ctx_s, t0 + q * tq, tq);
    n_q[q] = (int)((keys_q[q] + kN - 1) / kN);
  }
  const int n_tiles = n_q[0] > n_q[1] ? n_q[0] : n_q[1];
  const long long n_keys = keys_q[0] > keys_q[1] ? keys_q[0] : keys_q[1];
  if (rem == 0 && threadIdx.x == 0 && ctx_s > a.table_width * kBS) {
    record_error(a.err, kErrTableWidth);
  }
  if (misaligned) {
    if (threadIdx.x == 0) record_error(a.err, kErrWaitTimeout);
  } else if (warp == kKWarp || warp == kVWarp) {
    // --------------------------------------------------------- TMA producers
    const bool is_k = warp == kKWarp;
    const CUtensorMap* map = is_k ? &tmk : &tmv;
    unsigned char* ring = is_k ? sK : sV;
    uint64_t* full = is_k ? bars->k_full : bars->v_full;
    uint64_t* empty = is_k ? bars->k_empty : bars->v_empty;
    const int stages = is_k ? kKStages : kVStages;
    if (lane == 0) {
      prefetch_tensormap(map);
      if (is_k) {
        prefetch_tensormap(&tmq);
        mbar_arrive_expect_tx(&bars->q_full, (unsigned)(2 * kSubs * kQSub));
#pragma unroll
        for (int q = 0; q < 2; ++q) {
#pragma unroll
          for (int sub = 0; sub < kSubs; ++sub) {
            tc::tma_load_4d(sQ + (q * kSubs + sub) * kQSub, &tmq, &bars->q_full, sub * 64,
                            t0 + q * tq, kh * group, (int)s);
          }
        }
      }
    }
    // Block-table entries for 4 tiles (32 blocks) per warp-wide load; the next
    // group's load is issued before this group's copies.
    constexpr int kTilesPerGroup = 32 / kBlocksPerTile;
    auto load_group = [&](int base, int* id, bool* valid) {
      *id = 0;
      *valid = false;
      const long long b = (long long)base * kBlocksPerTile + lane;
      if (base < n_tiles && b * kBS < n_keys) {
        const long long raw = load_index(a.table, a.table_i64, s * a.table_stride + b);
        if (raw >= 0 && raw < a.num_blocks) {
          *valid = true;
          *id = (int)raw;
        } else if (raw >= a.num_blocks && is_k) {
          record_error(a.err, kErrBlockId);
        }
      }
    };
    // L2 prefetch of the blocks of tile j + pf when tile j is issued (no shared
    // memory, no completion): the later tile copies then mostly hit L2.
    auto prefetch_tile = [&](int jj, int id0, bool v0, int id1, bool v1) {
      const int jt = jj + pf;
      if (pf <= 0 || jt >= kTilesPerGroup * 2) return;
      const bool in_next = jt >= kTilesPerGroup;
      const int id = in_next ? id1 : id0;
      const bool v = in_next ? v1 : v0;
      if (v && lane / kBlocksPerTile == jt % kTilesPerGroup) {
#pragma unroll
        for (int sub = 0; sub < kSubs; ++sub) {
          asm volatile(
              "cp.async.bulk.prefetch.tensor.5d.L2.global.tile [%0, {%1, %2, %3, %4, %5}];" ::"l"(
                  reinterpret_cast<uint64_t>(map)),
              "r"(sub * 64), "r"(kh), "r"(0), "r"(id), "r"(a.layer)
              : "memory");
        }
      }
    };
    int id_cur, id_next;
    bool valid_cur, valid_next;
    int issued = 0;
    load_group(0, &id_cur, &valid_cur);
    for (int base = 0; base < n_tiles; base += kTilesPerGroup) {
      if (*reinterpret_cast<volatile uint32_t*>(&bars->abort) != 0u) break;
      load_group(base + kTilesPerGroup, &id_next, &valid_next);
      const unsigned vmask = __ballot_sync(0xffffffffu, valid_cur);
      const int jn = n_tiles - base < kTilesPerGroup ? n_tiles - base : kTilesPerGroup;
      bool stop = false;
      for (int jj = 0; jj < jn; ++jj) {
        const int j = base + jj;
        const int st = j % stages;
        const unsigned mask = (vmask >> (jj * kBlocksPerTile)) & ((1u << kBlocksPerTile) - 1);
        const unsigned bytes = (unsigned)(__popc(mask) * kSubs * kBlockBytes);
        prefetch_tile(jj, id_cur, valid_cur, id_next, valid_next);
        if (lane == 0 && j >= stages) {
          wait_or_flag(&empty[st], (unsigned)((j / stages - 1) & 1), a.err, &bars->abort);
        }
        stop = __shfl_sync(0xffffffffu,
                           *reinterpret_cast<volatile uint32_t*>(&bars->abort), 0) != 0u;
        if (stop) break;
        if (lane == 0) {
          if (is_k) bars->tile_bits[j % kBitsRing] = mask;
          mbar_arrive_expect_tx(&full[st], bytes);
        }
        issued = j + 1;
        __syncwarp();
        if (valid_cur && lane / kBlocksPerTile == jj) {
          unsigned char* dst = ring + st * kSubs * kKVSub + (lane % kBlocksPerTile) * kBlockBytes;
#pragma unroll
          for (int sub = 0; sub < kSubs; ++sub) {
            tma_load_5d(dst + sub * kKVSub, map, &full[st], sub * 64, kh, 0, id_cur, a.layer);
          }
        }
      }
      if (stop) break;
      id_cur = id_next;
      valid_cur = valid_next;
    }
    if (lane == 0) {
      if (is_k) drain_wait(&bars->q_full, 0, a.err);
      const int first = issued > stages ? issued - stages : 0;
      for (int j = first; j < issued; ++j) {
        drain_wait(&full[j % stages], (unsigned)((j / stages) & 1), a.err);
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------- MMA issuer
    const bool bf16 = KV_DT == kBF16;
    const uint32_t idesc_qk = tc::instr_desc_f16(bf16, kM, kN, false, false);
    const uint32_t idesc_pv = tc::instr_desc_f16(bf16, kM, D, false, true);
    const uint32_t q_addr = smem_addr(sQ);

    // Tile j's K staged: relay its valid-block bits to the softmax warps.
    auto k_ready = [&](int j) {
      wait_or_flag(&bars->k_full[j % kKStages], (unsigned)((j / kKStages) & 1), a.err,
                   &bars->abort);
      if (lane == 0) {
        bars->s_bits[j & 1] = bars->tile_bits[j % kBitsRing];
        mbar_arrive(&bars->bits_full[j & 1]);
      }
      __syncwarp();
    };
    // S(q, j) = Q(q) K(j)^T into tile q's S columns.
    auto qk = [&](int q, int j) {
      if (lane == 0) {
        tc::fence_after_sync();
        const uint32_t k_addr = smem_addr(sK + (j % kKStages) * kSubs * kKVSub);
        const uint32_t qa = q_addr + q * kSubs * kQSub;
        const uint32_t tmem_s = tmem + (uint32_t)(q * 128);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t koff = (kk & 3) * 32;
          tc::mma_f16(tmem_s, tc::smem_desc_sw128(qa + (kk >> 2) * kQSub + koff, 16, 1024),
                      tc::smem_desc_sw128(k_addr + (kk >> 2) * kKVSub + koff, 16, 1024),
                      idesc_qk, kk > 0 ? 1u : 0u);
        }
        tc::commit(&bars->s_full[q]);
      }
      __syncwarp();
    };
    // O(q) += P(q, j) V(j) once the softmax of tile q has written P(q, j).
    auto pv = [&](int q, int j) {
      wait_or_flag(&bars->p_full[q], (unsigned)(j & 1), a.err, &bars->abort);
      if (lane == 0) {
        tc::fence_after_sync();
        const uint32_t v_addr = smem_addr(sV + (j % kVStages) * kSubs * kKVSub);
        const uint32_t tmem_p = tmem + (uint32_t)(q * 128);
        const uint32_t tmem_o = tmem + 256u + (uint32_t)(q * 128);
#pragma unroll
        for (int kk = 0; kk < kN / 16; ++kk) {
          tc::mma_f16_ts(tmem_o, tmem_p + kk * 8,
                         tc::smem_desc_sw128(v_addr + kk * 16 * 128, kKVSub, 1024), idesc_pv,
                         (j > 0 || kk > 0) ? 1u : 0u);
        }
        if (j == n_q[q] - 1) tc::commit(&bars->o_final[q]);
      }
      __syncwarp();
    };
    // Rows of V(j) that hold no valid key are zeroed before any P V reads them.
    auto v_ready = [&](int j) {
      const int st = j % kVStages;
      wait_or_flag(&bars->v_full[st], (unsigned)((j / kVStages) & 1), a.err, &bars->abort);
      const unsigned bits = bars->tile_bits[j % kBitsRing];
      unsigned char* v = sV + st * kSubs * kKVSub;
      bool zeroed = false;
      for (int i = 0; i < kBlocksPerTile; ++i) {
        const long long b = (long long)j * kBlocksPerTile + i;
        int first_bad = 0;
        if ((bits >> i) & 1u) {
          const long long left = ctx_s - b * kBS;
          first_bad = left >= kBS ? kBS : (int)(left > 0 ? left : 0);
        }
        const int nbad = kBS - first_bad;
        if (nbad == 0) continue;
        zeroed = true;
        for (int e = lane; e < nbad * kSubs * 8; e += 32) {
          const int r = first_bad + e / (kSubs * 8);
          const int rest = e % (kSubs * 8);
          const int sub = rest >> 3;
          const int ch = rest & 7;
          *reinterpret_cast<uint4*>(v + sub * kKVSub + (i * kBS + r) * 128 + ch * 16) =
              make_uint4(0u, 0u, 0u, 0u);
        }
      }
      if (zeroed) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
    };

    if (n_tiles > 0) {
      wait_or_flag(&bars->q_full, 0, a.err, &bars->abort);
      k_ready(0);
      if (n_q[0] > 0) qk(0, 0);
      if (n_q[1] > 0) qk(1, 0);
      if (lane == 0) tc::commit(&bars->k_empty[0]);
      __syncwarp();
      for (int j = 0; j < n_tiles; ++j) {
        if (*reinterpret_cast<volatile uint32_t*>(&bars->abort) != 0u) break;
        v_ready(j);
        bool next = false;
        const int last_q = j < n_q[1] ? 1 : 0;     // the last query tile that reads V(j)
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          if (j < n_q[q]) {
            pv(q, j);
            if (q == last_q && lane == 0) tc::commit(&bars->v_empty[j % kVStages]);
            if (j + 1 < n_q[q]) {
              if (!next) {
                k_ready(j + 1);
                next = true;
              }
              qk(q, j + 1);
            }
          }
        }
        if (lane == 0 && next) tc::commit(&bars->k_empty[(j + 1) % kKStages]);
        __syncwarp();
      }
    }
    if (lane == 0) tc::commit(&bars->mma_done);
    __syncwarp();
    drain_wait(&bars->mma_done, 0, a.err);
  } else if (warp < kKWarp) {
    // ------------------------------------------------------------- softmax + epilogue
    const int qt = warp >> 2;                  // query tile of this warp
    const int r = (warp & 3) * 32 + lane;      // row = TMEM lane
    const int g = r / tq;
    const int t = r - g * tq;
    const int tok = t0 + qt * tq + t;
    const bool row_valid = tok < a.q_len;
    const long long qpos = ctx_s - a.q_len + tok;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tmem_s = tmem + (uint32_t)(qt * 128) + lane_off;
    const uint32_t tmem_o = tmem + 256u + (uint32_t)(qt * 128) + lane_off;
    const int my_tiles = n_q[qt];
    const float scale_log2 = a.scale * kLog2e;
    const bool capped = a.softcap > 0.f;
    float m_used = -INFINITY;
    float l = 0.f;

    for (int j = 0; j < my_tiles; ++j) {
      if (*reinterpret_cast<volatile uint32_t*>(&bars->abort) != 0u) break;
      wait_or_flag(&bars->bits_full[j & 1], (unsigned)((j >> 1) & 1), a.err, &bars->abort);
      const unsigned bits = bars->s_bits[j & 1];
      wait_or_flag(&bars->s_full[qt], (unsigned)(j & 1), a.err, &bars->abort);
      tc::fence_after_sync();
      float sv[kN];
#pragma unroll
      for (int c = 0; c < kN / 32; ++c) {
        float tmp[32];
        tc::tmem_ld32(tmem_s + c * 32, tmp);
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[c * 32 + i] = tmp[i];
      }
      tc::tmem_wait_ld();
      const long long kbase = (long long)j * kN;
      const bool full = bits == (1u << kBlocksPerTile) - 1 && kbase + kN <= ctx_s &&
                        kbase + kN - 1 <= qpos;
      if (capped) {
#pragma unroll
        for (int c = 0; c < kN; ++c) {
          sv[c] = tanhf(sv[c] * a.scale / a.softcap) * (a.softcap * kLog2e);
        }
      } else if (!(scale_log2 > 0.f)) {
#pragma unroll
        for (int c = 0; c < kN; ++c) sv[c] *= scale_log2;
      }
      if (!full) {
        const long long lim = qpos < ctx_s - 1 ? qpos : ctx_s - 1;
#pragma unroll
        for (int c = 0; c < kN; ++c) {
          const bool ok = ((bits >> (c / kBS)) & 1u) && kbase + c <= lim;
          sv[c] = ok ? sv[c] : -INFINITY;
        }
      }
      float mx8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx8[i] = sv[i];
#pragma unroll
      for (int c = 8; c < kN; ++c) mx8[c & 7] = fmaxf(mx8[c & 7], sv[c]);
      const float m01 = fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3]));
      const float m23 = fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]));
      const float sl = (capped || !(scale_log2 > 0.f)) ? 1.f : scale_log2;
      const float rowmax = fmaxf(m01, m23) * sl;
      const float m_new = rowmax > m_used + kRescaleLog2 ? rowmax : m_used;
      const float m_sub = m_new == -INFINITY ? 0.f : m_new;
      const bool rescale = j > 0 && m_new != m_used && m_used != -INFINITY;
      const float alpha = rescale ? fast_exp2(m_used - m_new) : 1.f;
      m_used = m_new;
      float sum4[4] = {0.f, 0.f, 0.f, 0.f};
      // P over the first 64 columns of S(j), 32 keys (16 columns) at a time.
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          const int cc = h * 32 + c;
          const float p0 = exp2_mixed<POLY>(fmaf(sv[cc], sl, -m_sub), cc);
          const float p1 = exp2_mixed<POLY>(fmaf(sv[cc + 1], sl, -m_sub), cc + 1);
          sum4[(c >> 1) & 3] += p0 + p1;
          pk[c / 2] = pack2<KV_DT>(p0, p1);
        }
        tc::tmem_st16u(tmem_s + h * 16, pk);
      }
      l = l * alpha + ((sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
      // O rescaled once the scores are dead (fewer live registers).  S(j) was
      // committed after P(j-1) V(j-1), so O is stable; P(j) V(j) is issued only
      // after the arrival below.
      if (rescale) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float o[32];
          tc::tmem_ld32(tmem_o + c * 32, o);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tc::tmem_st32(tmem_o + c * 32, o);
        }
      }
      tc::tmem_wait_st();
      tc::fence_before_sync();
      mbar_arrive(&bars->p_full[qt]);
    }

    if (my_tiles > 0) {
      wait_or_flag(&bars->o_final[qt], 0, a.err, &bars->abort);
      tc::fence_after_sync();
    }
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const int qh = kh * group + g;
    const long long obase = s * a.o_s + (long long)qh * a.o_h + (long long)tok * a.o_t;
    const bool vec_out = a.out_dtype == KV_DT &&
                         (reinterpret_cast<uintptr_t>(a.out) & 15) == 0 && a.o_s % 8 == 0 &&
                         a.o_h % 8 == 0 && a.o_t % 8 == 0;
#pragma unroll
    for (int c = 0; c < D / 32; ++c) {
      float o[32];
      if (my_tiles > 0) {
        tc::tmem_ld32(tmem_o + c * 32, o);
        tc::tmem_wait_ld();
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = l > 0.f ? o[i] * inv : 0.f;
      if (row_valid) {
        if (vec_out) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            const uint4 w = make_uint4(pack2<KV_DT>(o[i], o[i + 1]), pack2<KV_DT>(o[i + 2], o[i + 3]),
                                       pack2<KV_DT>(o[i + 4], o[i + 5]), pack2<KV_DT>(o[i + 6], o[i + 7]));
            *reinterpret_cast<uint4*>(static_cast<unsigned char*>(a.out) +
                                      (obase + c * 32 + i) * 2) = w;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (a.out_dtype == kF32) store_f32<kF32>(a.out, obase + c * 32 + i, o[i]);
            else if (a.out_dtype == kF16) store_f32<kF16>(a.out, obase + c * 32 + i, o[i]);
            else store_f32<kBF16>(a.out, obase + c * 32 + i, o[i]);
          }
        }
      }
    }
    if (row_valid && a.lse != nullptr) {
      a.lse[(s * a.num_heads + qh) * a.q_len + tok] =
          l > 0.f ? (m_used + log2f(l)) * kLn2 : -INFINITY;
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

// Eighths of the exponentials evaluated by the polynomial: none by default
// (measured fastest on B200: the special-function unit is not the limit),
// LLMOPT_B200_FA_POLY=2|4 for a quarter or a half.
int fa_poly() {
  static const int v = [] {
    const char* e = getenv("LLMOPT_B200_FA_POLY");
    if (e == nullptr) return 0;
    const int x = atoi(e);
    return x == 2 || x == 4 ? x : 0;
  }();
  return v;
}

// L2 prefetch distance in key tiles (LLMOPT_B200_FA_PF, 0..4; off by default:
// on B200 a TMA L2 prefetch ahead of the loads did not shorten them).
int fa_prefetch() {
  static const int v = [] {
    const char* e = getenv("LLMOPT_B200_FA_PF");
    const int x = e != nullptr ? atoi(e) : 0;
    return x < 0 ? 0 : (x > 4 ? 4 : x);
  }();
  return v;
}

template <int D, int KV_DT>
const void* fa_ptr() {
  switch (fa_poly()) {
    case 2: return reinterpret_cast<const void*>(&prefill_fa_kernel<D, KV_DT, 2>);
    case 4: return reinterpret_cast<const void*>(&prefill_fa_kernel<D, KV_DT, 4>);
    default: return reinterpret_cast<const void*>(&prefill_fa_kernel<D, KV_DT, 0>);
  }
}

const void* select_fa(const AttnArgs& a) {
  if (a.head_dim == 128 && a.kv_dtype == kBF16) return fa_ptr<128, kBF16>();
  if (a.head_dim == 128 && a.kv_dtype == kF16) return fa_ptr<128, kF16>();
  if (a.head_dim == 64 && a.kv_dtype == kBF16) return fa_ptr<64, kBF16>();
  if (a.head_dim == 64 && a.kv_dtype == kF16) return fa_ptr<64, kF16>();
  return nullptr;
}

}  // namespace

// The ping-pong kernel takes every shape the single-tile prefill kernel takes
// (prefill_tc_supported); it runs when LLMOPT_B200_PREFILL=fa.
bool prefill_fa_enabled() {
  static const int on = [] {
    const char* v = getenv("LLMOPT_B200_PREFILL");
    return (v != nullptr && v[0] == 'f' && v[1] == 'a') ? 1 : 0;
  }();
  return on != 0;
}

bool prefill_fa_usable(const AttnArgs& a) { return select_fa(a) != nullptr; }

cudaError_t prefill_fa_launch(const AttnArgs& a, const CUtensorMap& tmq, const CUtensorMap& tmk,
                              const CUtensorMap& tmv, cudaStream_t stream) {
  const void* fn = select_fa(a);
  if (fn == nullptr) return cudaErrorInvalidValue;
  const size_t smem = a.head_dim == 128 ? Layout<128>::kBytes : Layout<64>::kBytes;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int tq = kM / a.group;
  const long long ctiles = (a.q_len + 2 * tq - 1) / (2 * tq);
  const long long grid = a.batch * a.kv_heads * ctiles;
  if (grid <= 0) return cudaSuccess;
  if (grid > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  int pf = fa_prefetch();
  void* args[] = {const_cast<CUtensorMap*>(&tmq), const_cast<CUtensorMap*>(&tmk),
                  const_cast<CUtensorMap*>(&tmv), const_cast<AttnArgs*>(&a), &pf};
  return launch_pdl(fn, dim3((unsigned)grid), dim3(kThreads), args, smem, stream);
}

}  // namespace llmopt
