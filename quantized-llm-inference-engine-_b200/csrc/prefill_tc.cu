// Chunked-prefill paged attention on the 5th-generation tensor cores (sm_100a).
//
// Replaces PagedAttention.forward for q_len > 1 (src/llmopt/attention/
// paged_attention.py:146-250: gather, h // group expansion, causal mask
// k_pos <= ctx - q_len + i, softmax, P V) when the query rows of one KV head
// form a real dense contraction (q_len * group > 16) on a 16-bit cache.
//
// A CTA owns kQT query tiles of 128 rows of one (sequence, KV head): 128 /
// group consecutive chunk tokens x the group's query heads per tile, rows
// ordered [head][token].  All its tiles read every K/V tile of 64 keys (4 KV
// blocks of 16 tokens) from the same shared-memory stage.  With kQT = 1 two
// CTAs share an SM, so one CTA's tensor-core work overlaps the other's
// softmax (measured faster on B200 than one CTA holding two tiles).  Warps:
//
//   K warp     Q (both tiles) once, then per key tile the 4 blocks' K rows
//              through the block table (5-D map over the cache, one 16-token
//              box per block and 64-dim slice) into a 3-stage ring; table
//              entries for 8 tiles come in with one load per lane, the next
//              group's while this group's copies stream.  -1 entries are not
//              loaded.
//   V warp     the same for V, into its own 2-stage ring (separate issuers, so
//              K of a later tile never queues behind V's wait for a free stage).
//   MMA warp   one thread issues tcgen05.mma kind::f16: S = Q K^T (M=128,
//              N=64, K=head_dim) per query tile into that tile's pair of
//              tensor-memory S buffers, then O += P V (N=head_dim, K=64 keys)
//              with P read from tensor memory (where the softmax left it,
//              over the tile's S buffer) and V as an MN-major shared-memory
//              operand.  Commits signal the softmax warps and free the stages.
//   softmax    4 warps per query tile, one thread per row (= TMEM lane):
//              tcgen05.ld of the S row, mask (block validity, context,
//              causal; skipped for interior tiles), online softmax in fp32
//              with a lazy running max (O in TMEM is rescaled only when the row
//              max grows by more than 2^8, which keeps every exp <= 256), P
//              packed to bf16/fp16 pairs and stored with one tcgen05.st into
//              the first 32 columns of the tile's S buffer.
//   epilogue   O / l from TMEM to the output, plus the natural-log LSE.
//
// Tensor memory (256 columns per query tile): query tile q uses [256 q,
// 256 q + 256): two S buffers of 64 columns and O.  Stale rows (unloaded blocks, slots past the
// context) are zeroed in V before P V so that a zero probability never meets
// an Inf/NaN.  Every wait is bounded; tensor memory is released before the CTA
// exits.
#include <float.h>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace llmopt {
namespace {

constexpr int kBS = 16;
constexpr int kM = 128;                  // query rows per tile = TMEM lanes
constexpr int kQT = 1;                   // query tiles per CTA (2 CTAs per SM)
constexpr int kN = 64;                   // keys per K/V tile
constexpr int kBlocksPerTile = kN / kBS;
constexpr int kKStages = 3;              // K ring depth
constexpr int kVStages = 2;              // V ring depth (V is needed a softmax later)
constexpr int kBitsRing = 8;             // tile valid-block bits, indexed tile % 8
constexpr int kSoftmaxWarps = 4 * kQT;
constexpr int kKWarp = kSoftmaxWarps;
constexpr int kVWarp = kSoftmaxWarps + 1;
constexpr int kMmaWarp = kSoftmaxWarps + 2;
constexpr int kThreads = (kSoftmaxWarps + 3) * 32;
constexpr int kQTile = kM * 128;         // [128 rows x 128 B] swizzled sub-tile (16 KB)
constexpr int kKTile = kN * 128;         // [64 keys x 128 B] swizzled sub-tile (8 KB)
constexpr int kBlockBytes = kBS * 128;   // one 16-row box (2 KB)
constexpr float kRescaleLog2 = 8.0f;
constexpr uint32_t kTmemPerTile = 256;   // S0, S1 (64 columns each), O (head_dim <= 128)
constexpr uint32_t kTmemCols = kTmemPerTile * kQT;
constexpr int kCtasPerSm = 2 / kQT;

template <int D>
struct Layout {
  static constexpr int kSubs = D / 64;
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kQT * kSubs * kQTile;
  static constexpr int kV = kK + kKStages * kSubs * kKTile;
  static constexpr int kBar = kV + kVStages * kSubs * kKTile;
  static constexpr int kBytes = kBar + 512;
};

struct Bars {
  uint64_t q_full;
  uint64_t k_full[kKStages];
  uint64_t k_empty[kKStages];
  uint64_t v_full[kVStages];
  uint64_t v_empty[kVStages];
  uint64_t bits_full[2];           // s_bits[j % 2] valid for tile j
  uint64_t s_full[kQT][2];         // S(q, j) in TMEM: barrier [q][j % 2], phase j / 2
  uint64_t p_full[kQT][2];         // P(q, j) in TMEM
  uint64_t o_done[kQT][2];         // P(q, j) V(j) complete
  uint64_t mma_done;               // every MMA of the CTA complete (before TMEM is freed)
  uint32_t tmem_base;
  uint32_t abort;                  // set by the first wait that gives up
  uint32_t tile_bits[kBitsRing];   // written by the K warp before k_full
  uint32_t s_bits[2];              // relayed by the MMA warp with bits_full
};
static_assert(sizeof(Bars) <= 512, "barrier block");

// Bounded wait.  The first wait of a CTA that gives up records the error and
// makes every later wait of the CTA return at once, so a broken pipeline ends
// within about one wait limit instead of one limit per tile.
__device__ __forceinline__ void wait_or_flag(uint64_t* bar, unsigned parity, unsigned* err,
                                             uint32_t* abort) {
  if (*reinterpret_cast<volatile uint32_t*>(abort) != 0u) return;
  if (!mbar_wait(bar, parity)) {
    record_error(err, kErrWaitTimeout | kErrWaitData);
    *reinterpret_cast<volatile uint32_t*>(abort) = 1u;
  }
}

// Drain wait before a producer exits: bounded, never skipped.
__device__ __forceinline__ void drain_wait(uint64_t* bar, unsigned parity, unsigned* err) {
  if (!mbar_wait(bar, parity)) record_error(err, kErrWaitTimeout | kErrWaitDrain);
}

// Keys visible to the rows of query tile q (its last valid token's causal
// limit, the context and the table row), or 0 when the tile holds no token.
__device__ __forceinline__ long long tile_keys(const AttnArgs& a, long long ctx_s, int t_begin,
                                               int tq) {
  if (t_begin >= a.q_len) return 0;
  const int t_last = (t_begin + tq < a.q_len ? t_begin + tq : a.q_len) - 1;
  long long n = ctx_s - a.q_len + t_last + 1;
  if (n > ctx_s) n = ctx_s;
  if (n > a.table_width * kBS) n = a.table_width * kBS;
  return n < 0 ? 0 : n;
}

template <int D, int KV_DT>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmq,
                      const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmv, const AttnArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  using L = Layout<D>;
  constexpr int kSubs = L::kSubs;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int group = a.group;
  const int tq = kM / group;                          // chunk tokens per query tile
  const int ctiles = (a.q_len + kQT * tq - 1) / (kQT * tq);
  const long long x = blockIdx.x;
  const long long s = x / ((long long)a.kv_heads * ctiles);
  const int rem = (int)(x - s * (long long)a.kv_heads * ctiles);
  const int kh = rem / ctiles;
  const int t0 = (rem - kh * ctiles) * kQT * tq;

  const long long ctx_s = load_index(a.ctx, a.ctx_i64, s);
  int n_tiles_q[kQT];
  int n_tiles = 0;
  long long n_keys = 0;
#pragma unroll
  for (int q = 0; q < kQT; ++q) {
    const long long nk = tile_keys(a, ctx_s, t0 + q * tq, tq);
    n_tiles_q[q] = (int)((nk + kN - 1) / kN);
    if (n_tiles_q[q] > n_tiles) n_tiles = n_tiles_q[q];
    if (nk > n_keys) n_keys = nk;
  }
  if (rem == 0 && threadIdx.x == 0 && ctx_s > a.table_width * kBS) {
    record_error(a.err, kErrTableWidth);
  }

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = smem_raw;
  Bars* bars = reinterpret_cast<Bars*>(sm + L::kBar);
  // The swizzled tiles need a 1024-byte aligned base; refuse to run without it.
  const bool misaligned = (smem_addr(sm) & 1023u) != 0;
  unsigned char* sQ = sm + L::kQ;
  unsigned char* sK = sm + L::kK;
  unsigned char* sV = sm + L::kV;

  if (threadIdx.x == 0) {
    bars->abort = 0u;
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
      for (int q = 0; q < kQT; ++q) {
        mbar_init(&bars->s_full[q][i], 1);
        mbar_init(&bars->p_full[q][i], 128);
        mbar_init(&bars->o_done[q][i], 1);
      }
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
  tc::fence_after_sync();
  const uint32_t tmem = bars->tmem_base;

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
        mbar_arrive_expect_tx(&bars->q_full, (unsigned)(kQT * kSubs * kQTile));
#pragma unroll
        for (int q = 0; q < kQT; ++q) {
#pragma unroll
          for (int sub = 0; sub < kSubs; ++sub) {
            tc::tma_load_4d(sQ + (q * kSubs + sub) * kQTile, &tmq, &bars->q_full, sub * 64,
                            t0 + q * tq, kh * group, (int)s);
          }
        }
      }
    }
    // Block-table entries for 8 tiles (32 blocks) come in with one load per
    // lane, and the next group's load is issued before this group's copies.
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
    int id_cur, id_next;
    bool valid_cur, valid_next;
    int issued = 0;                            // tiles whose copies were issued
    load_group(0, &id_cur, &valid_cur);
    for (int base = 0; base < n_tiles; base += kTilesPerGroup) {
      if (*reinterpret_cast<volatile uint32_t*>(&bars->abort) != 0u) break;
      load_group(base + kTilesPerGroup, &id_next, &valid_next);
      const unsigned vmask = __ballot_sync(0xffffffffu, valid_cur);
      const int jn = n_tiles - base < kTilesPerGroup ? n_tiles - base : kTilesPerGroup;
      for (int jj = 0; jj < jn; ++jj) {
        const int j = base + jj;
        const int st = j % stages;
        const unsigned mask = (vmask >> (jj * kBlocksPerTile)) & ((1u << kBlocksPerTile) - 1);
        const unsigned bytes = (unsigned)(__popc(mask) * kSubs * kBlockBytes);
        // Stage st is free once the tile `stages` earlier has been consumed
        // (its QKs for K, its PVs for V).
        if (lane == 0) {
          if (j >= stages) {
            wait_or_flag(&empty[st], (unsigned)((j / stages - 1) & 1), a.err, &bars->abort);
          }
        }
        // Stop issuing once the CTA gave up (decided by lane 0, shared by the warp).
        const bool stop = __shfl_sync(0xffffffffu,
                                      *reinterpret_cast<volatile uint32_t*>(&bars->abort), 0) != 0u;
        if (stop) break;
        if (lane == 0) {
          if (is_k) bars->tile_bits[j % kBitsRing] = mask;
          mbar_arrive_expect_tx(&full[st], bytes);
        }
        issued = j + 1;
        __syncwarp();
        if (valid_cur && lane / kBlocksPerTile == jj) {
          unsigned char* dst = ring + st * kSubs * kKTile + (lane % kBlocksPerTile) * kBlockBytes;
#pragma unroll
          for (int sub = 0; sub < kSubs; ++sub) {
            tma_load_5d(dst + sub * kKTile, map, &full[st], sub * 64, kh, 0, id_cur, a.layer);
          }
        }
      }
      id_cur = id_next;
      valid_cur = valid_next;
    }
    if (lane == 0) {
      // Drain: no copy may still target this CTA's shared memory at exit.
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

    // S(q, j) = Q(q) K(j)^T for every query tile that still sees tile j; then
    // K stage j % kKStages is released and tile j's valid-block bits relayed.
    auto issue_qk = [&](int j) {
      const int st = j % kKStages;
      wait_or_flag(&bars->k_full[st], (unsigned)((j / kKStages) & 1), a.err, &bars->abort);
      if (lane == 0) {
        bars->s_bits[j & 1] = bars->tile_bits[j % kBitsRing];
        mbar_arrive(&bars->bits_full[j & 1]);
        tc::fence_after_sync();
        const uint32_t k_addr = smem_addr(sK + st * kSubs * kKTile);  // st over the K ring
#pragma unroll
        for (int q = 0; q < kQT; ++q) {
          if (j >= n_tiles_q[q]) continue;
          const uint32_t tmem_s = tmem + q * kTmemPerTile + (uint32_t)((j & 1) * kN);
          const uint32_t qa = q_addr + q * kSubs * kQTile;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t koff = (kk & 3) * 32;
            tc::mma_f16(tmem_s, tc::smem_desc_sw128(qa + (kk >> 2) * kQTile + koff, 16, 1024),
                        tc::smem_desc_sw128(k_addr + (kk >> 2) * kKTile + koff, 16, 1024),
                        idesc_qk, kk > 0 ? 1u : 0u);
          }
          tc::commit(&bars->s_full[q][j & 1]);
        }
        tc::commit(&bars->k_empty[st]);
      }
      __syncwarp();
    };
    // Zero V rows of tile j that hold no valid key, then O(q) += P(q, j) V(j)
    // for every query tile that sees tile j; V stage released after both.
    auto issue_pv = [&](int j) {
      const int st = j % kVStages;
      wait_or_flag(&bars->v_full[st], (unsigned)((j / kVStages) & 1), a.err, &bars->abort);
      const unsigned bits = bars->tile_bits[j % kBitsRing];
      unsigned char* v = sV + st * kSubs * kKTile;
      bool zeroed = false;
      for (int i = 0; i < kBlocksPerTile; ++i) {
        const long long b = (long long)j * kBlocksPerTile + i;
        int first_bad = 0;                       // rows [first_bad, 16) are zeroed
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
          *reinterpret_cast<uint4*>(v + sub * kKTile + (i * kBS + r) * 128 + ch * 16) =
              make_uint4(0u, 0u, 0u, 0u);
        }
      }
      if (zeroed) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      const uint32_t v_addr = smem_addr(v);
#pragma unroll
      for (int q = 0; q < kQT; ++q) {
        if (j >= n_tiles_q[q]) continue;
        // S(q, j) read, P(q, j) written.  The softmax cannot be two phases
        // ahead on this barrier: P(q, j + 2) needs S(q, j + 2), issued only
        // after this wait.
        wait_or_flag(&bars->p_full[q][j & 1], (unsigned)((j >> 1) & 1), a.err, &bars->abort);
        if (lane == 0) {
          tc::fence_after_sync();
          const uint32_t tmem_p = tmem + q * kTmemPerTile + (uint32_t)((j & 1) * kN);
          const uint32_t tmem_o = tmem + q * kTmemPerTile + 2 * kN;
#pragma unroll
          for (int kk = 0; kk < kN / 16; ++kk) {
            tc::mma_f16_ts(tmem_o, tmem_p + kk * 8,
                           tc::smem_desc_sw128(v_addr + kk * 16 * 128, kKTile, 1024), idesc_pv,
                           (j > 0 || kk > 0) ? 1u : 0u);
          }
          tc::commit(&bars->o_done[q][j & 1]);
        }
        __syncwarp();
      }
      if (lane == 0) tc::commit(&bars->v_empty[st]);
      __syncwarp();
    };

    if (n_tiles > 0) {
      wait_or_flag(&bars->q_full, 0, a.err, &bars->abort);
      issue_qk(0);
      if (n_tiles > 1) issue_qk(1);
      for (int j = 0; j < n_tiles; ++j) {
        if (*reinterpret_cast<volatile uint32_t*>(&bars->abort) != 0u) break;
        issue_pv(j);
        if (j + 2 < n_tiles) issue_qk(j + 2);                     // reuses S buffers j % 2
      }
    }
    // No MMA may still write tensor memory when it is freed.
    if (lane == 0) tc::commit(&bars->mma_done);
    __syncwarp();
    drain_wait(&bars->mma_done, 0, a.err);
  } else {
    // ------------------------------------------------------------- softmax + epilogue
    const int qt = warp >> 2;                  // query tile of this warp
    const int r = (warp & 3) * 32 + lane;      // row = TMEM lane
    const int g = r / tq;
    const int t = r - g * tq;
    const int tok = t0 + qt * tq + t;
    const bool row_valid = tok < a.q_len;
    const long long qpos = ctx_s - a.q_len + tok;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tmem_q = tmem + qt * kTmemPerTile;
    const uint32_t tmem_o = tmem_q + 2 * kN;
    const int my_tiles = n_tiles_q[qt];
    const float scale_log2 = a.scale * kLog2e;
    const bool capped = a.softcap > 0.f;
    float m_used = -INFINITY;
    float l = 0.f;

    for (int j = 0; j < my_tiles; ++j) {
      if (*reinterpret_cast<volatile uint32_t*>(&bars->abort) != 0u) break;
      const unsigned par = (unsigned)((j >> 1) & 1);
      wait_or_flag(&bars->bits_full[j & 1], par, a.err, &bars->abort);
      const unsigned bits = bars->s_bits[j & 1];
      wait_or_flag(&bars->s_full[qt][j & 1], par, a.err, &bars->abort);
      tc::fence_after_sync();
      float sv[kN];
#pragma unroll
      for (int c = 0; c < kN / 32; ++c) {
        float tmp[32];
        tc::tmem_ld32(tmem_q + (uint32_t)((j & 1) * kN) + lane_off + c * 32, tmp);
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[c * 32 + i] = tmp[i];
      }
      tc::tmem_wait_ld();
      const long long kbase = (long long)j * kN;
      // Interior tiles (every block loaded, inside the context and at or before
      // this row's causal limit) need no per-key mask.
      const bool full = bits == (1u << kBlocksPerTile) - 1 && kbase + kN <= ctx_s &&
                        kbase + kN - 1 <= qpos;
      if (capped) {
        // tanh soft-cap, in log2 units; monotonic, so masking after it is exact.
#pragma unroll
        for (int c = 0; c < kN; ++c) {
          sv[c] = tanhf(sv[c] * a.scale / a.softcap) * (a.softcap * kLog2e);
        }
      } else if (!(scale_log2 > 0.f)) {
        // A non-positive scale does not commute with max: scale first.
#pragma unroll
        for (int c = 0; c < kN; ++c) sv[c] *= scale_log2;
      }
      if (!full) {
        const long long lim = qpos < ctx_s - 1 ? qpos : ctx_s - 1;   // last visible key
#pragma unroll
        for (int c = 0; c < kN; ++c) {
          const bool ok = ((bits >> (c / kBS)) & 1u) && kbase + c <= lim;
          sv[c] = ok ? sv[c] : -INFINITY;
        }
      }
      // Row max over 8 independent chains (scores are raw unless capped; the
      // positive scale commutes with max and is folded into the exp below).
      float mx8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx8[i] = sv[i];
#pragma unroll
      for (int c = 8; c < kN; ++c) mx8[c & 7] = fmaxf(mx8[c & 7], sv[c]);
      const float m01 = fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3]));
      const float m23 = fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]));
      const float sl = (capped || !(scale_log2 > 0.f)) ? 1.f : scale_log2;  // -> log2 units
      const float rowmax = fmaxf(m01, m23) * sl;
      const float m_new = rowmax > m_used + kRescaleLog2 ? rowmax : m_used;
      const float m_sub = m_new == -INFINITY ? 0.f : m_new;
      float sum8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) sum8[i] = 0.f;
      uint32_t pk[kN / 2];
#pragma unroll
      for (int c = 0; c < kN; c += 2) {
        const float p0 = fast_exp2(fmaf(sv[c], sl, -m_sub));
        const float p1 = fast_exp2(fmaf(sv[c + 1], sl, -m_sub));
        sum8[(c >> 1) & 7] += p0 + p1;
        pk[c / 2] = pack2<KV_DT>(p0, p1);
      }
      const float rowsum = ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) +
                           ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
      // O is rescaled only when the running max moved, and only then does this
      // tile wait for P(j-1)V(j-1) (O stable).  The wait on barrier (j-1) % 2 is
      // unambiguous: P(j-2)V(j-2) completed before S(j) was written, and
      // P(j+1)V(j+1) cannot start before this tile's P exists.
      if (j > 0 && m_new != m_used && m_used != -INFINITY) {
        wait_or_flag(&bars->o_done[qt][(j - 1) & 1], (unsigned)(((j - 1) >> 1) & 1), a.err, &bars->abort);
        tc::fence_after_sync();
        const float alpha = fast_exp2(m_used - m_new);
        l *= alpha;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float o[32];
          tc::tmem_ld32(tmem_o + lane_off + c * 32, o);
          tc::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tc::tmem_st32(tmem_o + lane_off + c * 32, o);
        }
        tc::tmem_wait_st();
      }
      m_used = m_new;
      l += rowsum;
      // P row r over the first 32 columns of its S buffer: S(j) is fully read
      // (wait::ld above), and the P there before was consumed by P(j-2)V(j-2).
      tc::tmem_st32u(tmem_q + (uint32_t)((j & 1) * kN) + lane_off, pk);
      tc::tmem_wait_st();
      tc::fence_before_sync();
      mbar_arrive(&bars->p_full[qt][j & 1]);
    }

    // Every P V done before O is read: the last two tiles' barriers (each has
    // at most that one phase left to complete).
    for (int j = my_tiles > 2 ? my_tiles - 2 : 0; j < my_tiles; ++j) {
      wait_or_flag(&bars->o_done[qt][j & 1], (unsigned)((j >> 1) & 1), a.err, &bars->abort);
    }
    if (my_tiles > 0) tc::fence_after_sync();
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
        tc::tmem_ld32(tmem_o + lane_off + c * 32, o);
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

template <int D, int KV_DT>
const void* prefill_ptr() {
  return reinterpret_cast<const void*>(&prefill_tc_kernel<D, KV_DT>);
}

const void* select_prefill(const AttnArgs& a) {
  if (a.head_dim == 128 && a.kv_dtype == kBF16) return prefill_ptr<128, kBF16>();
  if (a.head_dim == 128 && a.kv_dtype == kF16) return prefill_ptr<128, kF16>();
  if (a.head_dim == 64 && a.kv_dtype == kBF16) return prefill_ptr<64, kBF16>();
  if (a.head_dim == 64 && a.kv_dtype == kF16) return prefill_ptr<64, kF16>();
  return nullptr;
}

size_t prefill_smem(int head_dim) {
  return head_dim == 128 ? Layout<128>::kBytes : Layout<64>::kBytes;
}

}  // namespace

bool prefill_tc_supported(const AttnArgs& a) {
  if (a.kv_dtype != kBF16 && a.kv_dtype != kF16) return false;
  if (a.q_dtype != a.kv_dtype) return false;           // both MMA operands share a type
  if (a.block_size != kBS) return false;
  if (a.head_dim != 64 && a.head_dim != 128) return false;
  if (a.rows <= 16) return false;                       // the decode kernel covers these
  if (a.group < 1 || a.group > kM || kM % a.group != 0) return false;
  // Query tensor map: 16-byte aligned base and strides, unit innermost stride.
  const uintptr_t qp = reinterpret_cast<uintptr_t>(a.q);
  if ((qp & 15) || (a.q_t * 2) % 16 || (a.q_h * 2) % 16 || (a.q_s * 2) % 16) return false;
  if (a.q_t < a.head_dim || a.q_h < 1 || a.q_s < 1) return false;
  if ((reinterpret_cast<uintptr_t>(a.k_cache) & 15) || (reinterpret_cast<uintptr_t>(a.v_cache) & 15))
    return false;
  if ((long long)a.num_blocks * kBS > 0x7fffffffLL) return false;
  if (a.batch > 0x7fffffffLL) return false;
  return select_prefill(a) != nullptr;
}

cudaError_t prefill_tc_launch(const AttnArgs& a, const CUtensorMap& tmq, const CUtensorMap& tmk,
                              const CUtensorMap& tmv, cudaStream_t stream) {
  if (prefill_pair_enabled() && prefill_pair_usable(a)) {
    return prefill_pair_launch(a, tmq, tmk, tmv, stream);
  }
  if (prefill_fa_enabled() && prefill_fa_usable(a)) {
    return prefill_fa_launch(a, tmq, tmk, tmv, stream);
  }
  const void* fn = select_prefill(a);
  if (fn == nullptr) return cudaErrorInvalidValue;
  const size_t smem = prefill_smem(a.head_dim);
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int tq = kM / a.group;
  const long long ctiles = (a.q_len + kQT * tq - 1) / (kQT * tq);
  const long long grid = a.batch * a.kv_heads * ctiles;
  if (grid <= 0) return cudaSuccess;
  if (grid > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  void* args[] = {const_cast<CUtensorMap*>(&tmq), const_cast<CUtensorMap*>(&tmk),
                  const_cast<CUtensorMap*>(&tmv), const_cast<AttnArgs*>(&a)};
  return launch_pdl(fn, dim3((unsigned)grid), dim3(kThreads), args, smem, stream);
}

}  // namespace llmopt
