// Chunked-prefill paged attention on 2-SM tensor-core pairs (sm_100a,
// tcgen05 cta_group::2 + TMA), head_dim 128.
//
// Replaces PagedAttention.forward for q_len > 1 (src/llmopt/attention/
// paged_attention.py:146-250: gather, h // group expansion, causal mask
// k_pos <= ctx - q_len + i, softmax, P V) on the shapes prefill_tc.cu takes,
// with the ping-pong schedule of prefill_fa.cu spread over a cluster of two
// CTAs on two SMs:
//
// * A pair owns two query super-tiles of 256 rows of one (sequence, KV head):
//   super-tile q is the 128-row tile (q, 0) in the even CTA and (q, 1) in the
//   odd CTA, tile (q, c) holding chunk tokens [t0 + (2q + c) tq, + tq),
//   tq = 128 / group, rows ordered [head][token].  Keys are walked in tiles
//   of 128 (8 KV blocks).
// * Every product is one M = 256 tcgen05 MMA issued by one thread of the even
//   CTA: S(q) = Q(q) K^T with each CTA staging HALF of every K tile (keys
//   [64 c, 64 c + 64), K-major) and O(q) += P(q) V with each CTA staging half
//   of every V tile (dims [64 c, 64 c + 64), MN-major).  Each SM therefore
//   keeps half the K/V bytes in flight per unit of tensor work that a
//   one-SM CTA needs - what bounds the one-SM kernels on B200, whose random
//   2 KB paged boxes take microseconds to arrive.
// * Tensor memory of each CTA: S of tile q at columns [128 q, 128 q + 128)
//   (its 128 rows, all 128 keys), P written over its first 64 columns, O of
//   tile q at [256 + 128 q, 384 + 128 q).  The softmax of each CTA works on
//   its own rows exactly as in prefill_fa.cu.
// * Synchronisation across the pair: each CTA's copies complete on its own
//   mbarriers; each CTA's relay warp waits for them, hands the tile's
//   valid-block bits to its softmax warps, cleans the V rows that hold no
//   valid key and arrives on the even CTA's ready barriers; the softmax warps
//   of both CTAs arrive on the even CTA's P barriers; the MMA thread's
//   commits arrive on the barrier at the same offset in both CTAs (multicast
//   commit), which frees both CTAs' ring stages and releases both CTAs'
//   softmax and epilogue.  The MMA thread itself only waits and issues: a
//   shared-memory load right after a burst of MMA issues stalls for
//   microseconds on B200, so it reads nothing else from shared memory.
//
// Every wait is bounded.  The first that gives up sets the abort flag of both
// CTAs (so the pair's other waits return at once), producers drain what they
// issued, the MMA thread waits for its products, and both CTAs meet at a
// cluster barrier before tensor memory is released.
#include <float.h>

#include <cstdlib>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace llmopt {
namespace {

constexpr int kBS = 16;
constexpr int kM = 128;                          // rows per CTA per query tile = TMEM lanes
constexpr int kN = 128;                          // keys per K/V tile
constexpr int kD = 128;                          // head_dim
constexpr int kSubs = kD / 64;                   // 128-byte slices of a K row
constexpr int kBlocksPerTile = kN / kBS;         // 8
constexpr int kHalfBlocks = kBlocksPerTile / 2;  // K blocks staged by each CTA
constexpr int kKStages = 4;
constexpr int kVStages = 6;
constexpr int kBitsRing = 8;
constexpr int kReadyRing = 8;
constexpr int kKWarp = 8;
constexpr int kVWarp = 9;
constexpr int kMmaWarp = 10;
constexpr int kRelayWarp = 11;
constexpr int kThreads = 12 * 32;
constexpr int kQSub = kM * 128;                  // 128 rows x 64 dims (16 KB)
constexpr int kKSub = (kN / 2) * 128;            // 64 keys x 64 dims (8 KB)
constexpr int kKStage = kSubs * kKSub;           // this CTA's half of a K tile (16 KB)
constexpr int kVStage = kN * 128;                // 128 keys x this CTA's 64 dims (16 KB)
constexpr int kBlockBytes = kBS * 128;           // one 16-row box (2 KB)
constexpr float kRescaleLog2 = 8.0f;
constexpr uint32_t kTmemCols = 512;
constexpr int kRankBatch = 256;
constexpr uint16_t kPairMask = 0x3;

constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + 2 * kSubs * kQSub;
constexpr int kOffV = kOffK + kKStages * kKStage;
constexpr int kOffBar = kOffV + kVStages * kVStage;
constexpr int kSmemBytes = kOffBar + 512;
static_assert(kSmemBytes <= 227 * 1024, "shared memory");

struct Bars {
  uint64_t q_full;                 // this CTA's query tiles staged
  uint64_t q_ready;                // (even CTA) Q and K(0) staged in both CTAs: 2 relays
  uint64_t k_full[kKStages];       // this CTA's half of K(j) staged
  uint64_t k_empty[kKStages];      // the products reading the stage are complete
  uint64_t v_full[kVStages];
  uint64_t v_empty[kVStages];
  uint64_t ready[kReadyRing];      // (even) V(j) staged and cleaned and K(j + 1) staged
                                   // in both CTAs: phase j / 8 of ready[j % 8], 2 relays
  uint64_t bits_full[kBitsRing];   // s_bits[j % 8] holds key tile j's valid blocks
  uint64_t s_full[2];              // S(q, j) in tensor memory
  uint64_t p_full[2];              // (even) P(q, j) written: one arrival per softmax warp
  uint64_t o_final[2];             // every P V product of tile q complete
  uint64_t mma_done;               // every product of the pair complete
  uint32_t tmem_base;
  uint32_t abort;
  uint32_t tile_bits[kBitsRing];   // written by the K loader
  uint32_t s_bits[kBitsRing];      // relayed to the softmax warps
  int seq;
};
static_assert(sizeof(Bars) <= 512, "barrier block");

// Wait state of one thread: the pair's abort flags and the error word.
struct PairWait {
  uint32_t* abort;
  uint32_t peer_abort;  // shared::cluster address of the other CTA's flag
  unsigned* err;

  __device__ __forceinline__ bool aborted() const {
    return *reinterpret_cast<volatile uint32_t*>(abort) != 0u;
  }
  // True once the phase completed; false when the pair has given up.  The
  // abort flag is read only once the phase is found incomplete.
  __device__ __forceinline__ bool wait(uint64_t* bar, unsigned parity, unsigned site) const {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const long long t0 = clock64();
    while (!aborted()) {
      if (mbar_try_wait_cluster(bar, parity)) return true;
      if (clock64() - t0 > kWaitLimitCycles) {
        record_error(err, kErrWaitTimeout | site);
        *reinterpret_cast<volatile uint32_t*>(abort) = 1u;
        st_cluster_u32(peer_abort, 1u);
        return false;
      }
    }
    return false;
  }
  __device__ __forceinline__ void drain(uint64_t* bar, unsigned parity) const {
    if (!mbar_wait_cluster(bar, parity)) record_error(err, kErrWaitTimeout | kErrWaitDrain);
  }
};

__device__ __forceinline__ long long tile_keys(const AttnArgs& a, long long ctx_s, int t_begin,
                                               int tq) {
  if (t_begin >= a.q_len) return 0;
  const int t_last = (t_begin + tq < a.q_len ? t_begin + tq : a.q_len) - 1;
  long long n = ctx_s - a.q_len + t_last + 1;
  if (n > ctx_s) n = ctx_s;
  if (n > a.table_width * kBS) n = a.table_width * kBS;
  return n < 0 ? 0 : n;
}

// Zero the rows of this CTA's V stage that hold no valid key (a block the table
// does not name, or positions at or past the context end), so a zero
// probability never meets Inf/NaN left in shared memory; then make the writes
// visible to the tensor core.  The products that read the stage are issued by
// the even CTA, so the proxy fence covers every state space (a CTA-scoped one
// left stale rows visible to the pair's MMAs).  Warp-collective.
__device__ __forceinline__ void clean_v(unsigned char* v, unsigned bits, long long j,
                                        long long ctx_s, int lane) {
  bool zeroed = false;
  for (int i = 0; i < kBlocksPerTile; ++i) {
    const long long b = j * kBlocksPerTile + i;
    int first_bad = 0;
    if ((bits >> i) & 1u) {
      const long long left = ctx_s - b * kBS;
      first_bad = left >= kBS ? kBS : (int)(left > 0 ? left : 0);
    }
    const int nbad = kBS - first_bad;
    if (nbad == 0) continue;
    zeroed = true;
    for (int e = lane; e < nbad * 8; e += 32) {
      const int r = first_bad + (e >> 3);
      *reinterpret_cast<uint4*>(v + (i * kBS + r) * 128 + (e & 7) * 16) =
          make_uint4(0u, 0u, 0u, 0u);
    }
  }
  if (zeroed) asm volatile("fence.proxy.async;" ::: "memory");
  __syncwarp();
}

template <int KV_DT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    prefill_pair_kernel(const __grid_constant__ CUtensorMap tmq,
                        const __grid_constant__ CUtensorMap tmk,
                        const __grid_constant__ CUtensorMap tmv, const AttnArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const bool lead = crank == 0;
  const int group = a.group;
  const int tq = kM / group;                          // chunk tokens per 128-row tile
  const int ctiles = (a.q_len + 4 * tq - 1) / (4 * tq);
  const long long per_seq = (long long)a.kv_heads * ctiles;
  const long long pair = blockIdx.x >> 1;
  const long long rank = pair / per_seq;              // sequence by context length, longest first
  const int rem = (int)(pair - rank * per_seq);
  const int ct = ctiles - 1 - rem / a.kv_heads;       // later chunk tiles (more keys) first
  const int kh = rem - (rem / a.kv_heads) * a.kv_heads;
  const int t0 = ct * 4 * tq;

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = smem_raw;
  Bars* bars = reinterpret_cast<Bars*>(sm + kOffBar);
  const bool misaligned = (smem_addr(sm) & 1023u) != 0;
  unsigned char* sQ = sm + kOffQ;
  unsigned char* sK = sm + kOffK;
  unsigned char* sV = sm + kOffV;

  if (threadIdx.x == 0) {
    bars->abort = 0u;
    bars->seq = (int)rank;
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->q_ready, 2);
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(&bars->k_full[i], 1);
      mbar_init(&bars->k_empty[i], 1);
    }
    for (int i = 0; i < kVStages; ++i) {
      mbar_init(&bars->v_full[i], 1);
      mbar_init(&bars->v_empty[i], 1);
    }
    for (int i = 0; i < kReadyRing; ++i) mbar_init(&bars->ready[i], 2);
    for (int i = 0; i < kBitsRing; ++i) mbar_init(&bars->bits_full[i], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], 8);
      mbar_init(&bars->o_final[i], 1);
    }
    mbar_init(&bars->mma_done, 1);
    mbar_init_fence();
  }
  if (warp == 0) {
    tc::tmem_alloc_pair(&bars->tmem_base, kTmemCols);
    tc::tmem_relinquish_pair();
  }
  __syncthreads();
  // Longest context first (the same ranking in both CTAs of the pair).
  if (a.batch <= kRankBatch && threadIdx.x < a.batch) {
    const long long mine = load_index(a.ctx, a.ctx_i64, threadIdx.x);
    long long r = 0;
    for (long long u = 0; u < a.batch; ++u) {
      const long long other = load_index(a.ctx, a.ctx_i64, u);
      r += (other > mine || (other == mine && u < (long long)threadIdx.x)) ? 1 : 0;
    }
    if (r == rank) bars->seq = (int)threadIdx.x;
  }
  tc::fence_before_sync();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before either arrives on the other's
  tc::fence_after_sync();
  const uint32_t tmem = bars->tmem_base;
  const long long s = bars->seq;
  const PairWait pw{&bars->abort, cluster_addr(&bars->abort, crank ^ 1u), a.err};

  const long long ctx_s = load_index(a.ctx, a.ctx_i64, s);
  int n_q[2];
  long long keys_q[2];
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const long long k0 = tile_keys(a, ctx_s, t0 + 2 * q * tq, tq);
    const long long k1 = tile_keys(a, ctx_s, t0 + (2 * q + 1) * tq, tq);
    keys_q[q] = k0 > k1 ? k0 : k1;
    n_q[q] = (int)((keys_q[q] + kN - 1) / kN);
  }
  const int n_tiles = n_q[0] > n_q[1] ? n_q[0] : n_q[1];
  const long long n_keys = keys_q[0] > keys_q[1] ? keys_q[0] : keys_q[1];
  if (lead && rem == 0 && threadIdx.x == 0 && ctx_s > a.table_width * kBS) {
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
    const int stage_bytes = is_k ? kKStage : kVStage;
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
                            t0 + (2 * q + (int)crank) * tq, kh * group, (int)s);
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
        } else if (raw >= a.num_blocks && is_k && lead) {
          record_error(a.err, kErrBlockId);
        }
      }
    };
    const unsigned own_k = ((1u << kHalfBlocks) - 1u) << (kHalfBlocks * crank);
    int id_cur, id_next;
    bool valid_cur, valid_next;
    int issued = 0;
    load_group(0, &id_cur, &valid_cur);
    for (int base = 0; base < n_tiles; base += kTilesPerGroup) {
      if (pw.aborted()) break;
      load_group(base + kTilesPerGroup, &id_next, &valid_next);
      const unsigned vmask = __ballot_sync(0xffffffffu, valid_cur);
      const int jn = n_tiles - base < kTilesPerGroup ? n_tiles - base : kTilesPerGroup;
      bool stop = false;
      for (int jj = 0; jj < jn; ++jj) {
        const int j = base + jj;
        const int st = j % stages;
        const unsigned mask = (vmask >> (jj * kBlocksPerTile)) & ((1u << kBlocksPerTile) - 1);
        const unsigned bytes = is_k ? (unsigned)(__popc(mask & own_k) * kSubs * kBlockBytes)
                                    : (unsigned)(__popc(mask) * kBlockBytes);
        if (lane == 0 && j >= stages) {
          pw.wait(&empty[st], (unsigned)((j / stages - 1) & 1), kErrWaitSlot);
        }
        stop = __shfl_sync(0xffffffffu, pw.aborted() ? 1u : 0u, 0) != 0u;
        if (stop) break;
        if (lane == 0) {
          if (is_k) bars->tile_bits[j % kBitsRing] = mask;
          mbar_arrive_expect_tx(&full[st], bytes);
        }
        issued = j + 1;
        __syncwarp();
        const int i = lane % kBlocksPerTile;
        if (valid_cur && lane / kBlocksPerTile == jj) {
          unsigned char* stage = ring + st * stage_bytes;
          if (is_k) {
            if ((own_k >> i) & 1u) {
              unsigned char* dst = stage + (i - kHalfBlocks * (int)crank) * kBlockBytes;
#pragma unroll
              for (int sub = 0; sub < kSubs; ++sub) {
                tma_load_5d(dst + sub * kKSub, map, &full[st], sub * 64, kh, 0, id_cur, a.layer);
              }
            }
          } else {
            tma_load_5d(stage + i * kBlockBytes, map, &full[st], 64 * (int)crank, kh, 0, id_cur,
                        a.layer);
          }
        }
      }
      if (stop) break;
      id_cur = id_next;
      valid_cur = valid_next;
    }
    if (lane == 0) {
      if (is_k) pw.drain(&bars->q_full, 0);
      const int first = issued > stages ? issued - stages : 0;
      for (int j = first; j < issued; ++j) {
        pw.drain(&full[j % stages], (unsigned)((j / stages) & 1));
      }
    }
  } else if (warp == kRelayWarp) {
    // ------------------------------------------------------------------ relay
    // Tile j's K staged here: hand its valid-block bits to this CTA's softmax
    // warps; returns the bits.
    auto k_staged = [&](int j) {
      pw.wait(&bars->k_full[j % kKStages], (unsigned)((j / kKStages) & 1), kErrWaitData);
      const unsigned bits = bars->tile_bits[j % kBitsRing];
      if (lane == 0) {
        bars->s_bits[j % kBitsRing] = bits;
        mbar_arrive(&bars->bits_full[j % kBitsRing]);
      }
      return bits;
    };
    // In the order the MMA thread consumes them: Q and K(0), then per tile j
    // V(j) together with K(j + 1).  The ready ring cannot lap the MMA thread:
    // staging K(j + 9) needs the products of tile j + 5, issued only after
    // ready(j + 4) was consumed.
    if (n_tiles > 0) {
      pw.wait(&bars->q_full, 0, kErrWaitData);
      unsigned bits = k_staged(0);
      if (lane == 0) mbar_arrive_cluster(cluster_addr(&bars->q_ready, 0));
      for (int j = 0; j < n_tiles; ++j) {
        if (pw.aborted()) break;
        const int vs = j % kVStages;
        pw.wait(&bars->v_full[vs], (unsigned)((j / kVStages) & 1), kErrWaitData);
        clean_v(sV + vs * kVStage, bits, j, ctx_s, lane);
        if (j + 1 < n_tiles) bits = k_staged(j + 1);
        if (lane == 0) mbar_arrive_cluster(cluster_addr(&bars->ready[j % kReadyRing], 0));
        __syncwarp();
      }
    }
  } else if (warp == kMmaWarp) {
    // ----------------------------------------------- MMA issuer (even CTA only)
    if (lead) {
      const bool bf16 = KV_DT == kBF16;
      const uint32_t idesc_qk = tc::instr_desc_f16(bf16, 2 * kM, kN, false, false);
      const uint32_t idesc_pv = tc::instr_desc_f16(bf16, 2 * kM, kD, false, true);
      // The issuing warp shares its SM sub-partition with two softmax warps,
      // so the loops below carry few instructions per MMA: descriptors are
      // built once and stepped by constants (the start address is bits 0-13,
      // address / 16, and no step carries out of it below 256 KB), and ring
      // stages are counters, not remainders.  Measured: 717 -> 759 TFLOP/s on
      // config 3 for the elected, warp-uniform issue below over `lane == 0`.
      // One lane, elected once, issues every MMA and commit (a commit tracks
      // the MMAs of its own thread); the operands are computed by the whole
      // warp, so they stay warp-uniform.
      const bool issuer = tc::elect_one();
      const uint64_t qdesc = tc::smem_desc_sw128(smem_addr(sQ), 16, 1024);
      const uint64_t kdesc = tc::smem_desc_sw128(smem_addr(sK), 16, 1024);
      const uint64_t vdesc = tc::smem_desc_sw128(smem_addr(sV), kVStage, 1024);
      // S(q, j) = Q(q) K^T over the pair (256 rows x 128 keys), K in stage ks.
      auto qk = [&](int q, int ks) {
        const uint64_t a0 = qdesc + (uint64_t)((q * kSubs * kQSub) >> 4);
        const uint64_t b0 = kdesc + (uint64_t)((ks * kKStage) >> 4);
        const uint32_t tmem_s = tmem + (uint32_t)(q * 128);
        if (issuer) {
          tc::fence_after_sync();
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint32_t koff = (kk & 3) * 32;
            tc::mma_f16_pair(tmem_s, a0 + (uint64_t)(((kk >> 2) * kQSub + koff) >> 4),
                             b0 + (uint64_t)(((kk >> 2) * kKSub + koff) >> 4), idesc_qk,
                             kk > 0 ? 1u : 0u);
          }
          tc::commit_pair(&bars->s_full[q], kPairMask);
        }
        __syncwarp();
      };
      // O(q) += P(q, j) V over the pair (256 rows x 128 dims), V in stage vs.
      auto pv = [&](int q, int vs, bool first, bool last) {
        const uint64_t b0 = vdesc + (uint64_t)((vs * kVStage) >> 4);
        const uint32_t tmem_p = tmem + (uint32_t)(q * 128);
        const uint32_t tmem_o = tmem + 256u + (uint32_t)(q * 128);
        if (issuer) {
          tc::fence_after_sync();
#pragma unroll
          for (int kk = 0; kk < kN / 16; ++kk) {
            tc::mma_f16_ts_pair(tmem_o, tmem_p + kk * 8,
                                b0 + (uint64_t)((kk * 16 * 128) >> 4), idesc_pv,
                                (!first || kk > 0) ? 1u : 0u);
          }
          if (last) tc::commit_pair(&bars->o_final[q], kPairMask);
        }
        __syncwarp();
      };

      // `ok` turns false when a wait gives up; nothing is issued after that.
      bool ok = true;
      if (n_tiles > 0) {
        ok = pw.wait(&bars->q_ready, 0, kErrWaitPeer);
        if (ok && n_q[0] > 0) qk(0, 0);
        if (ok && n_q[1] > 0) qk(1, 0);
        if (issuer) tc::commit_pair(&bars->k_empty[0], kPairMask);
        __syncwarp();
        int ks = 1 % kKStages;      // stage of K(j + 1)
        int vs = 0;                 // stage of V(j)
        int rs = 0;                 // ready-ring slot of tile j
        unsigned rph = 0;           // its phase parity
        for (int j = 0; j < n_tiles && ok; ++j) {
          ok = pw.wait(&bars->ready[rs], rph, kErrWaitPeer);
          bool next = false;
          const int last_q = j < n_q[1] ? 1 : 0;     // the last query tile that reads V(j)
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            if (ok && j < n_q[q]) {
              // Both CTAs' softmax warps have written P(q, j).
              ok = pw.wait(&bars->p_full[q], (unsigned)(j & 1), kErrWaitData);
              if (ok) pv(q, vs, j == 0, j == n_q[q] - 1);
              if (q == last_q && issuer) tc::commit_pair(&bars->v_empty[vs], kPairMask);
              if (ok && j + 1 < n_q[q]) {
                next = true;
                qk(q, ks);
              }
            }
          }
          if (issuer && next) tc::commit_pair(&bars->k_empty[ks], kPairMask);
          __syncwarp();
          ks = ks + 1 == kKStages ? 0 : ks + 1;
          vs = vs + 1 == kVStages ? 0 : vs + 1;
          rs = rs + 1 == kReadyRing ? 0 : rs + 1;
          rph ^= rs == 0 ? 1u : 0u;
        }
      }
      if (issuer) tc::commit_pair(&bars->mma_done, kPairMask);
      __syncwarp();
    }
    // Both CTAs: every product reading this CTA's shared or tensor memory is
    // complete before the pair meets at the final cluster barrier.
    if (lane == 0) pw.drain(&bars->mma_done, 0);
    __syncwarp();
  } else if (warp < kKWarp) {
    // ------------------------------------------------------------- softmax + epilogue
    const int qt = warp >> 2;                  // query tile of this warp
    const int r = (warp & 3) * 32 + lane;      // row = TMEM lane
    const int g = r / tq;
    const int t = r - g * tq;
    const int tok = t0 + (2 * qt + (int)crank) * tq + t;
    const bool row_valid = tok < a.q_len;
    const long long qpos = ctx_s - a.q_len + tok;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tmem_s = tmem + (uint32_t)(qt * 128) + lane_off;
    const uint32_t tmem_o = tmem + 256u + (uint32_t)(qt * 128) + lane_off;
    const uint32_t p_full_lead = cluster_addr(&bars->p_full[qt], 0);
    const int my_tiles = n_q[qt];
    const float scale_log2 = a.scale * kLog2e;
    const bool capped = a.softcap > 0.f;
    float m_used = -INFINITY;
    float l = 0.f;

    for (int j = 0; j < my_tiles; ++j) {
      if (pw.aborted()) break;
      pw.wait(&bars->bits_full[j % kBitsRing], (unsigned)((j / kBitsRing) & 1), kErrWaitData);
      const unsigned bits = bars->s_bits[j % kBitsRing];
      pw.wait(&bars->s_full[qt], (unsigned)(j & 1), kErrWaitData);
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
      // Row maximum: 8 strided chains of three-input maxima.
      float mx8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float acc = max3f(sv[k], sv[k + 8], sv[k + 16]);
#pragma unroll
        for (int i = 3; i + 1 < 16; i += 2) acc = max3f(acc, sv[k + 8 * i], sv[k + 8 * i + 8]);
        mx8[k] = fmaxf(acc, sv[k + 120]);
      }
      const float m01 = max3f(mx8[0], mx8[1], max3f(mx8[2], mx8[3], mx8[4]));
      const float m23 = max3f(mx8[5], mx8[6], mx8[7]);
      const float sl = (capped || !(scale_log2 > 0.f)) ? 1.f : scale_log2;
      const float rowmax = fmaxf(m01, m23) * sl;
      const float m_new = rowmax > m_used + kRescaleLog2 ? rowmax : m_used;
      const float m_sub = m_new == -INFINITY ? 0.f : m_new;
      const bool rescale = j > 0 && m_new != m_used && m_used != -INFINITY;
      const float alpha = rescale ? fast_exp2(m_used - m_new) : 1.f;
      m_used = m_new;
      // P over the first 64 columns of S(j), 32 keys (16 columns) at a time;
      // the exponent arguments in packed two-float arithmetic (per lane the
      // same IEEE fused multiply-add as fmaf).  Packed row sums would spill.
      float sa0 = 0.f, sa1 = 0.f, sb0 = 0.f, sb1 = 0.f;
      const uint64_t sl2 = pack2f(sl, sl);
      const uint64_t nm2 = pack2f(-m_sub, -m_sub);
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          const int cc = h * 32 + c;
          float x0, x1;
          ffma2(x0, x1, sv[cc], sv[cc + 1], sl2, nm2);
          const float p0 = fast_exp2(x0);
          const float p1 = fast_exp2(x1);
          if ((c >> 1) & 1) {
            sb0 += p0;
            sb1 += p1;
          } else {
            sa0 += p0;
            sa1 += p1;
          }
          pk[c / 2] = pack2<KV_DT>(p0, p1);
        }
        tc::tmem_st16u(tmem_s + h * 16, pk);
      }
      l = l * alpha + ((sa0 + sb0) + (sa1 + sb1));
      // O rescaled once the scores are dead.  S(j) was committed after
      // P(j-1) V(j-1), so O is stable; P(j) V(j) is issued only after the
      // arrivals below.
      if (rescale) {
#pragma unroll
        for (int c = 0; c < kD / 32; ++c) {
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
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(p_full_lead);
    }

    if (my_tiles > 0) {
      pw.wait(&bars->o_final[qt], 0, kErrWaitData);
      tc::fence_after_sync();
    }
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const int qh = kh * group + g;
    const long long obase = s * a.o_s + (long long)qh * a.o_h + (long long)tok * a.o_t;
    const bool vec_out = a.out_dtype == KV_DT &&
                         (reinterpret_cast<uintptr_t>(a.out) & 15) == 0 && a.o_s % 8 == 0 &&
                         a.o_h % 8 == 0 && a.o_t % 8 == 0;
#pragma unroll
    for (int c = 0; c < kD / 32; ++c) {
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

  // Neither CTA leaves (or releases tensor memory) while the other may still
  // arrive on its barriers or the pair's products may read its memory.
  tc::fence_before_sync();
  __syncthreads();
  cluster_sync();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc_pair(tmem, kTmemCols);
  }
}

const void* select_pair(const AttnArgs& a) {
  if (a.head_dim != kD) return nullptr;
  if (a.kv_dtype == kBF16) return reinterpret_cast<const void*>(&prefill_pair_kernel<kBF16>);
  if (a.kv_dtype == kF16) return reinterpret_cast<const void*>(&prefill_pair_kernel<kF16>);
  return nullptr;
}

}  // namespace

// The pair kernel takes the head_dim-128 shapes of the single-tile prefill
// kernel (prefill_tc_supported) and is the default for them; LLMOPT_B200_PREFILL
// = tc or fa selects one of the one-SM kernels instead.
bool prefill_pair_enabled() {
  static const int on = [] {
    const char* v = getenv("LLMOPT_B200_PREFILL");
    if (v == nullptr || v[0] == '\0') return 1;
    return (v[0] == 'p' && v[1] == 'a' && v[2] == 'i' && v[3] == 'r') ? 1 : 0;
  }();
  return on != 0;
}

bool prefill_pair_usable(const AttnArgs& a) { return select_pair(a) != nullptr; }

cudaError_t prefill_pair_launch(const AttnArgs& a, const CUtensorMap& tmq,
                                const CUtensorMap& tmk, const CUtensorMap& tmv,
                                cudaStream_t stream) {
  const void* fn = select_pair(a);
  if (fn == nullptr) return cudaErrorInvalidValue;
  cudaError_t e =
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return e;
  const int tq = kM / a.group;
  const long long ctiles = (a.q_len + 4 * tq - 1) / (4 * tq);
  const long long pairs = a.batch * a.kv_heads * ctiles;
  if (pairs <= 0) return cudaSuccess;
  if (2 * pairs > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  void* args[] = {const_cast<CUtensorMap*>(&tmq), const_cast<CUtensorMap*>(&tmk),
                  const_cast<CUtensorMap*>(&tmv), const_cast<AttnArgs*>(&a)};
  return launch_pdl(fn, dim3((unsigned)(2 * pairs)), dim3(kThreads), args, kSmemBytes, stream);
}

}  // namespace llmopt
