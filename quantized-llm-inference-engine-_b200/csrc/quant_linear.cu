// Weight-only quantized linear layer: y = x W^T + b with W held as packed
// 2/4/8-bit codes plus per-group float32 scales and zero points.
//
// Replaces QuantLinear.forward (src/llmopt/quantization/quant_linear.py:93-113),
// which dequantizes the whole weight to the compute dtype (quantizers.py:203-239),
// caches that dense copy and calls F.linear.  Here the codes are read and
// dequantized on the fly by every call, so a forward streams bits/16 of the
// bytes of a 16-bit weight and no dense copy is kept.
//
// Storage (the reference's): qweight uint8 [n, k/2] for 2- and 4-bit codes
// (two per byte, the even column in the low nibble; symmetric codes biased by
// 2^(bits-1)), uint8 [n, k] for asymmetric 8-bit, int8 [n, k] for symmetric
// 8-bit; scales / zeros float32 [n, k / group].  Dequantized value:
// (q - 2^(bits-1)) * s (symmetric, sub-byte), q * s (symmetric 8-bit),
// (q - z) * s (asymmetric), in float32, then cast to the compute dtype.
//
// Kernels:
// * wq_dequant_kernel: the dense weight in the compute dtype, bit-exact with the
//   reference's dequantize.
// * Tensor-core path (f16 / bf16, k % 128 == 0, n % 64 == 0, group 32, 64, 128
//   or a multiple of 128): a CTA owns 64 output features (four warps of 16 rows)
//   and 8 or 32 tokens; a 4-stage cp.async ring brings each 128-column
//   tile's codes, token rows and group constants into shared memory, and each
//   warp builds m16n8k16 A fragments from its 16 rows in registers (weight rows
//   = M, tokens = N: a decode batch pads to 8 tokens, not 16).  Code pairs come
//   out as (code j, code j+4) of each 8-code chunk; the B fragments pair the
//   token values the same way with byte permutes after a 16-byte read.
//   - wq_gemm_acc_kernel, 2- and 4-bit codes: one LOP3 puts two nibbles into
//     the mantissas of a 16-bit pair (128.0 for bf16, 1024.0 for f16, the
//     magic-number trick) and an exact subtraction leaves (q - z).  Each MMA's
//     k-range lies inside one group, so the MMAs sum exact (q - z) x products
//     and the group's scale multiplies the fp32 sum once per group.
//   - wq_gemm_u8_kernel, 8-bit codes: dequantized in float32 (exact), rounded
//     once to the compute dtype, so its weights are the reference's bit for bit.
//   The k range is split across CTAs when n and m alone do not fill the GPU;
//   splits write fp32 partials that wq_reduce_kernel sums (with the bias) in a
//   fixed order.
// * wq_generic_kernel: CUDA cores, fp32 accumulation, any shape and dtype.
#include <cstddef>
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace llmopt {
namespace {

constexpr int kWarps = 4;
constexpr int kRows = 16 * kWarps;   // output features per CTA
constexpr int kKT = 128;             // k per tile
constexpr int kMT = 32;              // tokens per CTA, large batches (4 n-tiles of 8)
constexpr int kMTSmall = 8;          // tokens per CTA up to 8 tokens (one n-tile)
constexpr int kThreads = 32 * kWarps;
constexpr int kChunks = kKT / 8;     // 8-element chunks per token row of a tile

// Physical 16-byte chunk of logical chunk c in token row i of a staged tile.
__device__ __forceinline__ int x_chunk(int i, int c) { return c ^ ((c >> 3) << 1) ^ (i & 1); }

// code value of element e of a row (unpacked, before the offset)
__device__ __forceinline__ float code_at(const QuantLinearArgs& a, long long row, long long e) {
  if (a.bits == 8) {
    const unsigned char b = a.qweight[row * a.k + e];
    return a.symmetric ? (float)(signed char)b : (float)b;
  }
  const unsigned char b = a.qweight[row * (a.k / 2) + (e >> 1)];
  return (float)((e & 1) ? (b >> 4) : (b & 0x0F));
}

// The reference's dequantized weight element in float32 (before the cast).
__device__ __forceinline__ float dequant_at(const QuantLinearArgs& a, long long row, long long e) {
  const long long gi = row * (a.k / a.group) + e / a.group;
  const float q = code_at(a, row, e);
  const float s = a.scales[gi];
  if (a.symmetric) {
    return __fmul_rn(a.bits < 8 ? q - (float)(1 << (a.bits - 1)) : q, s);
  }
  return __fmul_rn(q - a.zeros[gi], s);
}

template <int DT>
__global__ void __launch_bounds__(256) wq_dequant_kernel(const QuantLinearArgs a, void* out) {
  griddep_wait();
  griddep_launch_dependents();
  const long long total = a.n * a.k;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    store_f32<DT>(out, i, dequant_at(a, i / a.k, i % a.k));
  }
}

// CUDA cores: a CTA computes 16 tokens x 64 features; the weight tile is
// dequantized (rounded to the compute dtype, as the reference's dense copy)
// into shared memory once per 32-column step.
template <int DT>
__global__ void __launch_bounds__(256) wq_generic_kernel(const QuantLinearArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  constexpr int TM = 16, TN = 64, TK = 32;
  __shared__ float ws[TN][TK + 1];
  __shared__ float xs[TM][TK + 1];
  const long long m0 = (long long)blockIdx.y * TM;
  const long long n0 = (long long)blockIdx.x * TN;
  const int tid = threadIdx.x;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};     // (token tid / 16, features 4 * (tid % 16) + j)
  const int ti = tid >> 4;
  const int fj = (tid & 15) * 4;
  for (long long k0 = 0; k0 < a.k; k0 += TK) {
    for (int idx = tid; idx < TN * TK; idx += 256) {
      const int r = idx / TK, c = idx % TK;
      float v = 0.f;
      if (n0 + r < a.n && k0 + c < a.k) v = round_through<DT>(dequant_at(a, n0 + r, k0 + c));
      ws[r][c] = v;
    }
    for (int idx = tid; idx < TM * TK; idx += 256) {
      const int r = idx / TK, c = idx % TK;
      float v = 0.f;
      if (m0 + r < a.m && k0 + c < a.k) v = load_f32<DT>(a.x, (m0 + r) * a.ldx + k0 + c);
      xs[r][c] = v;
    }
    __syncthreads();
#pragma unroll 8
    for (int c = 0; c < TK; ++c) {
      const float xv = xs[ti][c];
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = fmaf(xv, ws[fj + j][c], acc[j]);
    }
    __syncthreads();
  }
  const long long tok = m0 + ti;
  if (tok < a.m) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const long long f = n0 + fj + j;
      if (f < a.n) {
        float v = acc[j];
        if (a.bias != nullptr) v += load_f32<DT>(a.bias, f);
        store_f32<DT>(a.out, tok * a.ldo + f, v);
      }
    }
  }
}

// 16-bit pair type of the compute dtype, and its magic-number constants.
template <int DT> struct Pair;
template <> struct Pair<kBF16> {
  using T = __nv_bfloat162;
  static constexpr uint32_t kMagic = 0x43004300u;   // 128.0 in both halves
  static constexpr float kBase = 128.f;
  __device__ static T splat(float v) { return __floats2bfloat162_rn(v, v); }
  __device__ static T pack(float lo, float hi) { return __floats2bfloat162_rn(lo, hi); }
};
template <> struct Pair<kF16> {
  using T = __half2;
  static constexpr uint32_t kMagic = 0x64006400u;   // 1024.0 in both halves
  static constexpr float kBase = 1024.f;
  __device__ static T splat(float v) { return __floats2half2_rn(v, v); }
  __device__ static T pack(float lo, float hi) { return __floats2half2_rn(lo, hi); }
};

template <class T>
__device__ __forceinline__ uint32_t as_u32(const T& v) {
  return *reinterpret_cast<const uint32_t*>(&v);
}
template <class T>
__device__ __forceinline__ T from_u32(uint32_t u) {
  return *reinterpret_cast<const T*>(&u);
}

// Dequantized pairs (code j, code j+4), j = 0..3, of 8 8-bit codes (two words:
// codes 0-3 and 4-7), exact in float32 and rounded once to the compute dtype.
template <int DT>
__device__ __forceinline__ void dequant_chunk8(uint32_t w0, uint32_t w1, uint32_t flip,
                                               float zoff, float s, uint32_t (&p)[4]) {
  using P = Pair<DT>;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t b0 = ((w0 >> (8 * j)) & 0xFFu) ^ flip;
    const uint32_t b1 = ((w1 >> (8 * j)) & 0xFFu) ^ flip;
    const float f0 = __fmul_rn(__int_as_float(0x4B000000 | b0) - zoff, s);
    const float f1 = __fmul_rn(__int_as_float(0x4B000000 | b1) - zoff, s);
    p[j] = as_u32(P::pack(f0, f1));
  }
}

// 16-byte global -> shared copy, L2 only (cp.async.cg); `bytes` of the source
// (0 or 16) are read, the rest of the 16 filled with zeros.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)),
               "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

constexpr int kStages = 4;
constexpr int kMaxGroupsPerTile = kKT / 32;

// ---- 8-bit codes: weights dequantized in float32 -------------------------------
//
// One pipeline stage: the CTA's codes, token tile and group constants of one
// 128-column tile (MT tokens).
template <int MT>
struct Stage8 {
  static constexpr int kRowBytes = kKT;
  unsigned char w[kRows][kRowBytes];        // codes of the CTA's 64 rows
  uint4 x[MT][kChunks];                     // token rows, chunks swizzled by x_chunk()
  float s[kRows][kMaxGroupsPerTile];        // scales of the tile's groups
  float z[kRows][kMaxGroupsPerTile];        // zero points (asymmetric)
};

template <int DT, int MT>
__global__ void __launch_bounds__(kThreads) wq_gemm_u8_kernel(const QuantLinearArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  using P = Pair<DT>;
  using S = Stage8<MT>;
  constexpr int NT = MT / 8;                                   // 8-token n-tiles
  extern __shared__ __align__(16) unsigned char smem_raw[];
  S* st = reinterpret_cast<S*>(smem_raw);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int gid = lane >> 2;
  const int tid4 = lane & 3;
  const long long rbase = (long long)blockIdx.x * kRows;       // the CTA's first row
  const int wrow = warp * 16 + gid;                            // this lane's rows: wrow, +8
  const long long m0 = (long long)blockIdx.z * MT;
  const long long kb = (long long)blockIdx.y * a.k_per_split;
  const long long ke = kb + a.k_per_split < a.k ? kb + a.k_per_split : a.k;
  const int ntiles = (int)((ke - kb) / kKT);
  const long long mrem = a.m - m0;
  const int n_tiles = mrem >= MT ? NT : (int)((mrem + 7) / 8);   // useful 8-token n-tiles
  const long long groups = a.k / a.group;
  const int gpt = a.group >= kKT ? 1 : kKT / a.group;            // groups per tile (<= 4)
  const long long row_bytes = a.k;

  // Stage t <- codes, token tile and group constants of tile t (all threads).
  // A thread's copy slots are the same for every tile: their shared-memory
  // offsets and global addresses are set up once, and a tile only adds its
  // column offset.
  constexpr int kWPieces = kRows * S::kRowBytes / 16;           // 16-byte pieces of codes
  constexpr int kWPer = (kWPieces + kThreads - 1) / kThreads;
  constexpr int kXPer = (MT * kChunks + kThreads - 1) / kThreads;
  const unsigned char* wsrc[kWPer];
  int wdst[kWPer];
#pragma unroll
  for (int q = 0; q < kWPer; ++q) {
    const int i = threadIdx.x + q * kThreads;
    const int r = i / (S::kRowBytes / 16), c = i % (S::kRowBytes / 16);
    wsrc[q] = a.qweight + (rbase + r) * row_bytes + 16 * c;
    wdst[q] = (int)(reinterpret_cast<const unsigned char*>(&st[0].w[r][16 * c]) -
                    reinterpret_cast<const unsigned char*>(&st[0]));
  }
  const unsigned short* xsrc[kXPer];
  int xdst[kXPer], xbytes[kXPer];
#pragma unroll
  for (int q = 0; q < kXPer; ++q) {
    const int i = threadIdx.x + q * kThreads;
    const int r = i / kChunks, c = i % kChunks;
    const bool ok = i < MT * kChunks && m0 + r < a.m;
    xsrc[q] = static_cast<const unsigned short*>(a.x) + (ok ? (m0 + r) * a.ldx + kb + 8 * c : 0);
    xbytes[q] = ok ? 16 : 0;
    xdst[q] = i < MT * kChunks
                  ? (int)(reinterpret_cast<const unsigned char*>(&st[0].x[r][x_chunk(r, c)]) -
                          reinterpret_cast<const unsigned char*>(&st[0]))
                  : -1;
  }
  // group constants: kRows * gpt entries (up to 256: two per thread)
  constexpr int kGPer = (kRows * kMaxGroupsPerTile + kThreads - 1) / kThreads;
  bool has_g[kGPer];
  int gr[kGPer], gj[kGPer];
  const float* ssrc[kGPer];
  const float* zsrc[kGPer];
#pragma unroll
  for (int q = 0; q < kGPer; ++q) {
    const int i = threadIdx.x + q * kThreads;
    has_g[q] = i < kRows * gpt;
    gr[q] = has_g[q] ? i / gpt : 0;
    gj[q] = has_g[q] ? i % gpt : 0;
    ssrc[q] = a.scales + (rbase + gr[q]) * groups + gj[q];
    zsrc[q] = a.zeros != nullptr ? a.zeros + (rbase + gr[q]) * groups + gj[q] : nullptr;
  }
  auto issue = [&](int t) {
    unsigned char* base = reinterpret_cast<unsigned char*>(&st[t % kStages]);
    const long long k0 = kb + (long long)t * kKT;
    const long long wk = k0;
#pragma unroll
    for (int q = 0; q < kWPer; ++q) {
      if (threadIdx.x + q * kThreads < kWPieces) cp_async16(base + wdst[q], wsrc[q] + wk, 16);
    }
    const long long xk = (long long)t * kKT;
#pragma unroll
    for (int q = 0; q < kXPer; ++q) {
      if (xdst[q] >= 0) cp_async16(base + xdst[q], xsrc[q] + (xbytes[q] ? xk : 0), xbytes[q]);
    }
    const long long g0 = k0 / a.group;
    S& s = *reinterpret_cast<S*>(base);
#pragma unroll
    for (int q = 0; q < kGPer; ++q) {
      if (has_g[q]) {
        cp_async4(&s.s[gr[q]][gj[q]], ssrc[q] + g0);
        if (!a.symmetric) cp_async4(&s.z[gr[q]][gj[q]], zsrc[q] + g0);
      }
    }
  };

  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;

#pragma unroll
  for (int t = 0; t < kStages - 1; ++t) {
    if (t < ntiles) issue(t);
    cp_async_commit();
  }

  for (int t = 0; t < ntiles; ++t) {
    cp_async_wait<kStages - 2>();
    __syncthreads();                       // tile t landed; tile t-1's stage is free
    if (t + kStages - 1 < ntiles) issue(t + kStages - 1);
    cp_async_commit();
    const S& s = st[t % kStages];
    // this lane's 32 codes of each row lie in group j = (32 t4) / group of the tile
    const int j = a.group >= kKT ? 0 : (32 * tid4) / a.group;
    // the lane's 32 codes of rows wrow and wrow + 8 (16-byte reads) and their
    // group constants
    uint4 cw[2][2];
    float sf[2], zf[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = wrow + 8 * h;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        cw[h][q] = *reinterpret_cast<const uint4*>(&s.w[r][32 * tid4 + 16 * q]);
      }
      sf[h] = s.s[r][j];
      zf[h] = a.symmetric ? 0.f : s.z[r][j];
    }
#pragma unroll
    for (int w = 0; w < 4; ++w) {          // chunk 4 t4 + w: k-steps 2w, 2w + 1
      uint32_t pa[2][4];                   // [row half][pair (code i, code i+4)]
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        // codes 8w .. 8w+7: words 2w and 2w + 1 of the lane's 32 bytes; symmetric
        // codes are int8, flipped to offset binary (q + 128)
        const uint4& c = cw[h][w >> 1];
        const uint32_t w0 = (w & 1) ? c.z : c.x;
        const uint32_t w1 = (w & 1) ? c.w : c.y;
        const uint32_t flip = a.symmetric ? 0x80u : 0u;
        const float zoff = 8388608.f + (a.symmetric ? 128.f : zf[h]);
        dequant_chunk8<DT>(w0, w1, flip, zoff, sf[h], pa[h]);
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        if (nt < n_tiles) {
          const int i = nt * 8 + gid;
          const uint4 xv = s.x[i][x_chunk(i, 4 * tid4 + w)];     // x0..x7 of the chunk
          // pair (x_i, x_i+4) as the codes: (x0 x4) (x1 x5) (x2 x6) (x3 x7)
          const uint32_t b[4] = {__byte_perm(xv.x, xv.z, 0x5410), __byte_perm(xv.x, xv.z, 0x7632),
                                 __byte_perm(xv.y, xv.w, 0x5410), __byte_perm(xv.y, xv.w, 0x7632)};
#pragma unroll
          for (int hs = 0; hs < 2; ++hs) {   // k-step 2w + hs: pairs 2hs (a0/a1), 2hs+1 (a2/a3)
            const uint32_t af[4] = {pa[0][2 * hs], pa[1][2 * hs], pa[0][2 * hs + 1],
                                    pa[1][2 * hs + 1]};
            mma_16816<DT>(acc[nt], af, b[2 * hs], b[2 * hs + 1]);
          }
        }
      }
    }
  }
  cp_async_wait<0>();

  // c-fragment e of n-tile nt: feature wrow + 8 (e >> 1), token m0 + 8 nt + 2 t4 + (e & 1)
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const long long tok = m0 + nt * 8 + 2 * tid4 + (e & 1);
      const long long f = rbase + wrow + 8 * (e >> 1);
      if (tok >= a.m) continue;
      if (a.partial != nullptr) {
        a.partial[((long long)blockIdx.y * a.m + tok) * a.n + f] = acc[nt][e];
      } else {
        float v = acc[nt][e];
        if (a.bias != nullptr) v += load_f32<DT>(a.bias, f);
        store_f32<DT>(a.out, tok * a.ldo + f, v);
      }
    }
  }
}

// ---- 2- and 4-bit codes: the group scale applied to the fp32 accumulators ------
//
// The k-steps of every MMA are aligned to the groups.  ldmatrix hands lane
// (g, t4) word w (w = 0..3) of a row as the codes of columns 32 w + 8 t4 ..
// 32 w + 8 t4 + 7 of the tile, so the two MMAs of word w cover only the 32
// columns [32 w, 32 w + 32) of the tile, which lie inside one group (groups
// are 32, 64 or 128 columns, or multiples of 128).  Those MMAs therefore run
// on the exact integers (q - z) in the compute dtype (products exact in fp32),
// and the group's scale multiplies the group's fp32 sum once:
// y += s_row * sum_{k in group} (q_k - z) x_k.  Per 8 codes that is one LOP3
// (plus a shift) per pair and one exact subtraction per pair; the scale costs
// one FMA per accumulator per group.
template <int MT, int GPT>
struct StageQ {
  static constexpr int kRowBytes = kKT / 2;   // 64 bytes of codes per row and tile
  // codes; 16-byte piece p of row r sits at piece position p ^ ((r >> 1) & 3),
  // so the eight rows of each ldmatrix phase hit eight different bank groups
  unsigned char w[kRows][kRowBytes];
  // token rows; chunk c of token i sits at chunk position c ^ ((i & 1) << 2)
  uint4 x[MT][kChunks];
  float s[kRows][GPT];                        // scales of the tile's groups
  float z[kRows][GPT];                        // zero points (asymmetric)
};

__device__ __forceinline__ int w_piece_pos(int r, int p) { return p ^ ((r >> 1) & 3); }
__device__ __forceinline__ int x_chunk_pos(int i, int c) { return c ^ ((i & 1) << 2); }

template <int DT, int MT, int GPT>
__global__ void __launch_bounds__(kThreads) wq_gemm_acc_kernel(const QuantLinearArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  using P = Pair<DT>;
  using S = StageQ<MT, GPT>;
  constexpr int NT = MT / 8;                    // 8-token n-tiles
  constexpr int kWordsPerGroup = 4 / GPT;       // 32-column words per group within a tile
  extern __shared__ __align__(16) unsigned char smem_raw[];

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int gid = lane >> 2;
  const int tid4 = lane & 3;
  const long long rbase = (long long)blockIdx.x * kRows;
  const int wrow = warp * 16 + gid;             // this lane's rows: wrow, wrow + 8
  const long long m0 = (long long)blockIdx.z * MT;
  const long long kb = (long long)blockIdx.y * a.k_per_split;
  const long long ke = kb + a.k_per_split < a.k ? kb + a.k_per_split : a.k;
  const int ntiles = (int)((ke - kb) / kKT);
  const long long mrem = a.m - m0;
  const int n_tiles = mrem >= MT ? NT : (int)((mrem + 7) / 8);
  const long long groups = a.k / a.group;
  const long long row_bytes = a.k / 2;
  const int tile0 = (int)(kb / kKT);

  // Copy slots.  Codes: 64 rows x 4 pieces, two per thread (rows tid/4 and
  // tid/4 + 32, piece tid % 4).
  const unsigned char* wsrc = a.qweight + (rbase + (tid >> 2)) * row_bytes + kb / 2 + 16 * (tid & 3);
  const long long wstep = 32 * row_bytes;
  const int wdst = (tid >> 2) * S::kRowBytes + 16 * w_piece_pos(tid >> 2, tid & 3);
  constexpr int kWDstStep = 32 * S::kRowBytes;
  // Token rows: MT x 16 chunks, MT / 8 per thread (tokens tid/16 + 8 q, chunk tid % 16).
  constexpr int kXPer = MT * kChunks / kThreads;
  const int xr0 = tid >> 4;
  const int xc = tid & 15;
  const unsigned short* xsrc =
      static_cast<const unsigned short*>(a.x) + (m0 + xr0) * a.ldx + kb + 8 * xc;
  const long long xstep = 8 * a.ldx;
  const int xdst = (int)offsetof(S, x) + (xr0 * kChunks + x_chunk_pos(xr0, xc)) * 16;
  constexpr int kXDstStep = 8 * kChunks * 16;
  // tokens of this thread's slots that exist: xr0 + 8 q < mrem
  const int x_valid = mrem > xr0 ? (int)((mrem - xr0 + 7) / 8) : 0;
  // Group constants: 64 x GPT entries (row i / GPT, group i % GPT of the tile).
  constexpr int kGPer = (kRows * GPT + kThreads - 1) / kThreads;
  // first group of tile t: (tile0 + t) * GPT, or (tile0 + t) / tpg for groups
  // of tpg tiles; issue() runs for t = 0, 1, 2, ... in order and keeps a cursor
  const int tpg = GPT > 1 ? 1 : a.group / kKT;
  long long g_cur = GPT > 1 ? (long long)tile0 * GPT : tile0 / tpg;
  int g_in = GPT > 1 ? 0 : tile0 % tpg;

  auto issue = [&](int t) {
    unsigned char* base = smem_raw + (size_t)(t % kStages) * sizeof(S);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      cp_async16(base + wdst + q * kWDstStep, wsrc + q * wstep + (long long)t * (kKT / 2), 16);
    }
#pragma unroll
    for (int q = 0; q < kXPer; ++q) {
      const bool ok = q < x_valid;
      // a slot past the last token copies nothing (source size 0) from a valid address
      cp_async16(base + xdst + q * kXDstStep,
                 ok ? xsrc + q * xstep + (long long)t * kKT : static_cast<const unsigned short*>(a.x),
                 ok ? 16 : 0);
    }
    S& sg = *reinterpret_cast<S*>(base);
#pragma unroll
    for (int q = 0; q < kGPer; ++q) {
      const int i = tid + q * kThreads;
      if (i < kRows * GPT) {
        const int r = i / GPT, g = i % GPT;
        const long long gi = (rbase + r) * groups + g_cur + g;
        cp_async4(&sg.s[r][g], a.scales + gi);
        if (!a.symmetric) cp_async4(&sg.z[r][g], a.zeros + gi);
      }
    }
    if (GPT > 1) {
      g_cur += GPT;
    } else if (++g_in == tpg) {
      g_in = 0;
      ++g_cur;
    }
  };

  float acc[NT][4];
  float part[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;

#pragma unroll
  for (int t = 0; t < kStages - 1; ++t) {
    if (t < ntiles) issue(t);
    cp_async_commit();
  }
  // ldmatrix rows: matrix q = lane / 8 is piece q of rows warp*16 + 8h + lane % 8
  const int lr = warp * 16 + (lane & 7);
  const int lm_off = lr * S::kRowBytes + 16 * w_piece_pos(lr, lane >> 3);
  const float zsym = (float)(1 << (a.bits - 1));
  const int xi_pos = gid & 1;                   // parity of every token row this lane reads

  for (int t = 0; t < ntiles; ++t) {
    cp_async_wait<kStages - 2>();
    __syncthreads();                            // tile t landed; tile t-1's stage is free
    if (t + kStages - 1 < ntiles) issue(t + kStages - 1);
    cp_async_commit();
    const unsigned char* base = smem_raw + (size_t)(t % kStages) * sizeof(S);
    const S& sg = *reinterpret_cast<const S*>(base);
    uint32_t cw[2][4];                          // [row half][word w]
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      ldsm_x4(smem_addr(base + lm_off + h * 8 * S::kRowBytes), cw[h][0], cw[h][1], cw[h][2],
              cw[h][3]);
    }
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const int g = w / kWordsPerGroup;
      if (w % kWordsPerGroup == 0) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) part[nt][0] = part[nt][1] = part[nt][2] = part[nt][3] = 0.f;
      }
      uint32_t pa[2][4];                        // [row half][pair (code j, code j+4)]
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float zf = a.symmetric ? zsym : sg.z[wrow + 8 * h][g];
        const typename P::T off2 = P::splat(P::kBase + zf);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t v = ((cw[h][w] >> (4 * j)) & 0x000F000Fu) | P::kMagic;
          pa[h][j] = as_u32(__hsub2(from_u32<typename P::T>(v), off2));
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        if (nt < n_tiles) {
          const uint4 xv = sg.x[nt * 8 + gid][(4 * w + tid4) ^ (xi_pos << 2)];
          const uint32_t b[4] = {__byte_perm(xv.x, xv.z, 0x5410), __byte_perm(xv.x, xv.z, 0x7632),
                                 __byte_perm(xv.y, xv.w, 0x5410), __byte_perm(xv.y, xv.w, 0x7632)};
#pragma unroll
          for (int hs = 0; hs < 2; ++hs) {
            const uint32_t af[4] = {pa[0][2 * hs], pa[1][2 * hs], pa[0][2 * hs + 1],
                                    pa[1][2 * hs + 1]};
            mma_16816<DT>(part[nt], af, b[2 * hs], b[2 * hs + 1]);
          }
        }
      }
      if (w % kWordsPerGroup == kWordsPerGroup - 1) {
        const float s0 = sg.s[wrow][g];
        const float s1 = sg.s[wrow + 8][g];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          acc[nt][0] = fmaf(part[nt][0], s0, acc[nt][0]);
          acc[nt][1] = fmaf(part[nt][1], s0, acc[nt][1]);
          acc[nt][2] = fmaf(part[nt][2], s1, acc[nt][2]);
          acc[nt][3] = fmaf(part[nt][3], s1, acc[nt][3]);
        }
      }
    }
  }
  cp_async_wait<0>();

  // c-fragment e of n-tile nt: feature wrow + 8 (e >> 1), token m0 + 8 nt + 2 t4 + (e & 1)
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const long long tok = m0 + nt * 8 + 2 * tid4 + (e & 1);
      const long long f = rbase + wrow + 8 * (e >> 1);
      if (tok >= a.m) continue;
      if (a.partial != nullptr) {
        a.partial[((long long)blockIdx.y * a.m + tok) * a.n + f] = acc[nt][e];
      } else {
        float v = acc[nt][e];
        if (a.bias != nullptr) v += load_f32<DT>(a.bias, f);
        store_f32<DT>(a.out, tok * a.ldo + f, v);
      }
    }
  }
}

// ---- 2- and 4-bit codes on the 5th-generation tensor cores (opt-in) ------------
//
// For token batches the weight is dequantized once per CTA into shared memory
// and multiplied by tcgen05.mma.  A CTA owns 128 output features (TMEM lanes,
// MMA M) and 64 tokens (MMA N) and walks its k range in 64-column slices:
// * all 128 threads copy a slice's codes (128 rows x 32 bytes), token rows
//   (64 x 128 bytes, in the 128-byte-swizzled K-major layout the MMA reads)
//   and group constants with cp.async into a 4-stage ring;
// * thread r dequantizes row r of the slice as the reference does, (q - z) * s
//   in float32 rounded once to the compute dtype, into a swizzled K-major A
//   tile (two A buffers), so the weights are the reference's bit for bit;
// * one thread issues the slice's four MMAs (K = 16 each) into the fp32
//   accumulator in tensor memory and commits them to an mbarrier.
// Slice t waits only for the MMAs of slice t - 2, which free its A buffer and
// the copy stage it refills, so one slice's dequantization overlaps the MMAs
// of the one before.  The epilogue reads the accumulator with tcgen05.ld
// (thread r = feature r, 32 tokens per load).  Every wait is bounded; a wait
// that gives up sets g_wq_err and the CTA skips the rest of its MMAs.
namespace tc05 {
constexpr int kBM = 128;                    // features per CTA
constexpr int kBN = 64;                     // tokens per CTA
constexpr int kBK = 64;                     // k per slice (one 128-byte row of 16-bit values)
constexpr int kThreads = 128;
constexpr int kStages = 4;
constexpr int kGroups = 2;                  // groups per slice at most (group 32)
constexpr int kATile = kBM * 128;
constexpr int kXTile = kBN * 128;
constexpr int kCodes = kBM * 32;
constexpr int kConsts = kBM * kGroups * 4;
constexpr int kOffA = 0;                    // offsets from the 1024-byte aligned base
constexpr int kOffX = kOffA + 2 * kATile;
constexpr int kOffC = kOffX + kStages * kXTile;
constexpr int kOffS = kOffC + kStages * kCodes;
constexpr int kOffZ = kOffS + kStages * kConsts;
constexpr int kOffBar = kOffZ + kStages * kConsts;
constexpr int kSmem = kOffBar + 64 + 1024;  // barriers, TMEM address, alignment slack
static_assert(kBN % 32 == 0 && kBN >= 32 && kBN <= 256, "TMEM columns / MMA N");
static_assert(kBN * 8 % kThreads == 0, "token-row copy slots");
}  // namespace tc05

__device__ unsigned g_wq_err;               // LLMOPT_DEVERR_* bits of the tcgen05 path

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <int DT>
__global__ void __launch_bounds__(tc05::kThreads) wq_gemm_tc05_kernel(const QuantLinearArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* mma_done = reinterpret_cast<uint64_t*>(base + tc05::kOffBar);   // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + tc05::kOffBar + 16);
  uint32_t* abort_flag = reinterpret_cast<uint32_t*>(base + tc05::kOffBar + 20);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const long long rbase = (long long)blockIdx.x * tc05::kBM;
  const long long m0 = (long long)blockIdx.z * tc05::kBN;
  const long long kb = (long long)blockIdx.y * a.k_per_split;
  const long long ke = kb + a.k_per_split < a.k ? kb + a.k_per_split : a.k;
  const int nslices = (int)((ke - kb) / tc05::kBK);
  const long long mrem = a.m - m0;
  const long long groups = a.k / a.group;
  const long long row_bytes = a.k / 2;
  const int gps = a.group >= tc05::kBK ? 1 : tc05::kBK / a.group;   // groups per slice: 1 or 2
  const int sps = a.group >= tc05::kBK ? a.group / tc05::kBK : 1;   // slices per group
  const int slice0 = (int)(kb / tc05::kBK);

  if (tid == 0) {
    mbar_init(&mma_done[0], 1);
    mbar_init(&mma_done[1], 1);
    *abort_flag = 0u;
    mbar_init_fence();
  }
  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, tc05::kBN);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  auto wait_mma = [&](int slice) {           // bounded; the first give-up aborts the CTA
    if (*reinterpret_cast<volatile uint32_t*>(abort_flag) != 0u) return;
    if (!mbar_wait(&mma_done[slice & 1], (unsigned)((slice >> 1) & 1))) {
      atomicOr(&g_wq_err, kErrWaitTimeout | kErrWaitData);
      *reinterpret_cast<volatile uint32_t*>(abort_flag) = 1u;
    }
  };

  // Copy slots, fixed per thread.  Codes: row tid, its two 16-byte pieces,
  // piece p stored at p ^ ((row >> 2) & 1) so a quarter warp's reads hit eight
  // bank groups.  Token rows: rows tid/8 + 16 q, chunk tid % 8, stored at
  // chunk position chunk ^ (row & 7) (the 128-byte swizzle).
  const unsigned char* csrc = a.qweight + (rbase + tid) * row_bytes + kb / 2;
  const int cdst0 = tid * 32 + 16 * ((tid >> 2) & 1);
  const int cdst1 = tid * 32 + 16 * (1 ^ ((tid >> 2) & 1));
  const int xr0 = tid >> 3;
  const int xc = tid & 7;
  const unsigned short* xsrc =
      static_cast<const unsigned short*>(a.x) + (m0 + xr0) * a.ldx + kb + 8 * xc;
  const int xdst = xr0 * 128 + 16 * (xc ^ (xr0 & 7));
  const float* ssrc = a.scales + (rbase + tid) * groups;
  const float* zsrc = a.zeros != nullptr ? a.zeros + (rbase + tid) * groups : nullptr;
  // first group of slice t: (slice0 + t) * gps, or (slice0 + t) / sps; issue()
  // runs for t = 0, 1, 2, ... in order and keeps a cursor
  long long g_cur = gps > 1 ? (long long)slice0 * gps : slice0 / sps;
  int g_in = gps > 1 ? 0 : slice0 % sps;

  auto issue = [&](int t) {
    const int st = t % tc05::kStages;
    unsigned char* cst = base + tc05::kOffC + st * tc05::kCodes;
    const unsigned char* src = csrc + (long long)t * (tc05::kBK / 2);
    cp_async16(cst + cdst0, src, 16);
    cp_async16(cst + cdst1, src + 16, 16);
    unsigned char* xst = base + tc05::kOffX + st * tc05::kXTile;
#pragma unroll
    for (int q = 0; q < tc05::kBN * 8 / tc05::kThreads; ++q) {
      const bool ok = xr0 + 16 * q < mrem;
      // a row past the last token copies nothing (source size 0) from a valid address
      cp_async16(xst + xdst + q * 16 * 128,
                 ok ? xsrc + 16 * q * a.ldx + (long long)t * tc05::kBK
                    : static_cast<const unsigned short*>(a.x),
                 ok ? 16 : 0);
    }
    float* sst = reinterpret_cast<float*>(base + tc05::kOffS + st * tc05::kConsts) + tid * tc05::kGroups;
    float* zst = reinterpret_cast<float*>(base + tc05::kOffZ + st * tc05::kConsts) + tid * tc05::kGroups;
    for (int g = 0; g < gps; ++g) {
      cp_async4(sst + g, ssrc + g_cur + g);
      if (!a.symmetric) cp_async4(zst + g, zsrc + g_cur + g);
    }
    if (gps > 1) {
      g_cur += gps;
    } else if (++g_in == sps) {
      g_in = 0;
      ++g_cur;
    }
  };

#pragma unroll
  for (int t = 0; t < tc05::kStages - 2; ++t) {
    if (t < nslices) issue(t);
    cp_async_commit();
  }
  const float zsym = (float)(1 << (a.bits - 1));
  const uint32_t idesc = tc::instr_desc_f16(DT == kBF16, tc05::kBM, tc05::kBN, false, false);
  int last_committed = -1;                   // thread 0: the last slice whose MMAs it issued

  for (int t = 0; t < nslices; ++t) {
    cp_async_wait<tc05::kStages - 3>();
    fence_proxy_async_smem();                // the copies, for the tensor core's reads
    __syncthreads();                         // slice t landed for every thread
    if (t >= 2) wait_mma(t - 2);             // frees A[t & 1] and stage (t - 2) % tc05::kStages
    if (t + tc05::kStages - 2 < nslices) issue(t + tc05::kStages - 2);
    cp_async_commit();
    const int st = t % tc05::kStages;
    const unsigned char* cst = base + tc05::kOffC + st * tc05::kCodes;
    const uint4 c0 = *reinterpret_cast<const uint4*>(cst + cdst0);
    const uint4 c1 = *reinterpret_cast<const uint4*>(cst + cdst1);
    const float* sst = reinterpret_cast<const float*>(base + tc05::kOffS + st * tc05::kConsts) + tid * tc05::kGroups;
    const float* zst = reinterpret_cast<const float*>(base + tc05::kOffZ + st * tc05::kConsts) + tid * tc05::kGroups;
    unsigned char* arow = base + tc05::kOffA + (t & 1) * tc05::kATile + tid * 128;
    const uint32_t words[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
    for (int c = 0; c < 8; ++c) {            // 16-byte chunk c of the row: codes 8c .. 8c + 7
      const int g = gps > 1 ? (c >> 2) : 0;  // group 32: chunks 0-3 and 4-7
      const float sc = sst[g];
      const float zoff = 8388608.f + (a.symmetric ? zsym : zst[g]);
      uint32_t pk[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {          // codes 2j (low nibble) and 2j + 1
        const float f0 = __int_as_float(0x4B000000u | ((words[c] >> (8 * j)) & 0xFu)) - zoff;
        const float f1 = __int_as_float(0x4B000000u | ((words[c] >> (8 * j + 4)) & 0xFu)) - zoff;
        pk[j] = as_u32(Pair<DT>::pack(__fmul_rn(f0, sc), __fmul_rn(f1, sc)));
      }
      *reinterpret_cast<uint4*>(arow + 16 * (c ^ (tid & 7))) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
    fence_proxy_async_smem();                // A, for the tensor core's reads
    __syncthreads();
    if (tid == 0 && *reinterpret_cast<volatile uint32_t*>(abort_flag) == 0u) {
      tc::fence_after_sync();
      const uint32_t a_addr = smem_addr(base + tc05::kOffA + (t & 1) * tc05::kATile);
      const uint32_t x_addr = smem_addr(base + tc05::kOffX + st * tc05::kXTile);
#pragma unroll
      for (int kk = 0; kk < tc05::kBK / 16; ++kk) {
        tc::mma_f16(tmem, tc::smem_desc_sw128(a_addr + kk * 32, 16, 1024),
                    tc::smem_desc_sw128(x_addr + kk * 32, 16, 1024), idesc,
                    (t > 0 || kk > 0) ? 1u : 0u);
      }
      tc::commit(&mma_done[t & 1]);
      last_committed = t;
    }
  }
  cp_async_wait<0>();
  // The last committed slice's commit covers every MMA the CTA issued: drained
  // (bounded) even after an abort, before tensor memory is read or freed.
  if (tid == 0 && last_committed >= 0) {
    if (!mbar_wait(&mma_done[last_committed & 1], (unsigned)((last_committed >> 1) & 1))) {
      atomicOr(&g_wq_err, kErrWaitTimeout | kErrWaitDrain);
      *reinterpret_cast<volatile uint32_t*>(abort_flag) = 1u;
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const bool ok = *reinterpret_cast<volatile uint32_t*>(abort_flag) == 0u && nslices > 0;

  // thread tid = feature rbase + tid = TMEM lane tid; columns = tokens m0 ..
  const long long f = rbase + tid;
  const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
  float bias = 0.f;
  if (a.partial == nullptr && a.bias != nullptr) bias = load_f32<DT>(a.bias, f);
#pragma unroll
  for (int cb = 0; cb < tc05::kBN / 32; ++cb) {
    float v[32];
    tc::tmem_ld32(lane_addr + cb * 32, v);
    tc::tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const long long tok = m0 + cb * 32 + j;
      if (tok >= a.m) break;
      const float val = ok ? v[j] : __int_as_float(0x7FC00000);   // NaN after a give-up
      if (a.partial != nullptr) {
        a.partial[((long long)blockIdx.y * a.m + tok) * a.n + f] = val;
      } else {
        store_f32<DT>(a.out, tok * a.ldo + f, val + bias);
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, tc05::kBN);
  }
}

// Sum of the split partials (split order) plus the bias, cast to the compute dtype.
template <int DT>
__global__ void __launch_bounds__(256) wq_reduce_kernel(const QuantLinearArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  const long long total = a.m * a.n;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    float v = 0.f;
    for (int s = 0; s < a.splits; ++s) v += a.partial[(long long)s * total + i];
    const long long tok = i / a.n, f = i % a.n;
    if (a.bias != nullptr) v += load_f32<DT>(a.bias, f);
    store_f32<DT>(a.out, tok * a.ldo + f, v);
  }
}

int groups_per_tile(int group) { return group >= kKT ? 1 : kKT / group; }

// 8 tokens per CTA up to 8 tokens, else 32.  (64-token tiles of the 2/4-bit
// kernel measured slower at 64 tokens: two CTAs per SM, latency-bound.)
int tokens_per_cta(const QuantLinearArgs& a) { return a.m <= kMTSmall ? kMTSmall : kMT; }

template <int DT, int MT>
const void* acc_ptr(int gpt) {
  return gpt == 1   ? reinterpret_cast<const void*>(&wq_gemm_acc_kernel<DT, MT, 1>)
         : gpt == 2 ? reinterpret_cast<const void*>(&wq_gemm_acc_kernel<DT, MT, 2>)
                    : reinterpret_cast<const void*>(&wq_gemm_acc_kernel<DT, MT, 4>);
}

template <int DT>
const void* gemm_ptr(const QuantLinearArgs& a, int mt) {
  if (a.bits == 8) {
    return mt == kMTSmall ? reinterpret_cast<const void*>(&wq_gemm_u8_kernel<DT, kMTSmall>)
                          : reinterpret_cast<const void*>(&wq_gemm_u8_kernel<DT, kMT>);
  }
  const int gpt = groups_per_tile(a.group);
  return mt == kMTSmall ? acc_ptr<DT, kMTSmall>(gpt) : acc_ptr<DT, kMT>(gpt);
}

template <int MT>
size_t acc_smem(int gpt) {
  return kStages * (gpt == 1   ? sizeof(StageQ<MT, 1>)
                    : gpt == 2 ? sizeof(StageQ<MT, 2>)
                               : sizeof(StageQ<MT, 4>));
}

size_t gemm_smem(const QuantLinearArgs& a, int mt) {
  if (a.bits == 8) {
    return kStages * (mt == kMTSmall ? sizeof(Stage8<kMTSmall>) : sizeof(Stage8<kMT>));
  }
  const int gpt = groups_per_tile(a.group);
  return mt == kMTSmall ? acc_smem<kMTSmall>(gpt) : acc_smem<kMT>(gpt);
}

const void* gemm_fn(const QuantLinearArgs& a) {
  const int mt = tokens_per_cta(a);
  return a.x_dtype == kBF16 ? gemm_ptr<kBF16>(a, mt) : gemm_ptr<kF16>(a, mt);
}

// LLMOPT_B200_QUANT_TC05=1 routes 2- and 4-bit token batches (more than 8
// tokens, n % 128 == 0) to wq_gemm_tc05_kernel.  Off by default: that kernel
// has not been run on a GPU yet.
bool tc05_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("LLMOPT_B200_QUANT_TC05");
    return v != nullptr && v[0] == '1';
  }();
  return on;
}

// The tensor-core kernel a call runs and its CTA shape.
struct GemmShape {
  const void* fn;
  int threads;
  size_t smem;
  long long rows;      // output features per CTA
  long long tokens;    // tokens per CTA
};

GemmShape gemm_shape(const QuantLinearArgs& a) {
  if (tc05_enabled() && a.bits < 8 && a.m > kMTSmall && a.n % tc05::kBM == 0 &&
      (a.group == 32 || a.group % tc05::kBK == 0)) {
    const void* fn = a.x_dtype == kBF16
                         ? reinterpret_cast<const void*>(&wq_gemm_tc05_kernel<kBF16>)
                         : reinterpret_cast<const void*>(&wq_gemm_tc05_kernel<kF16>);
    return {fn, tc05::kThreads, (size_t)tc05::kSmem, tc05::kBM, tc05::kBN};
  }
  const int mt = tokens_per_cta(a);
  return {gemm_fn(a), kThreads, gemm_smem(a, mt), kRows, mt};
}

long long grid_blocks(long long work, int threads) {
  long long b = (work + threads - 1) / threads;
  if (b > 148LL * 32) b = 148LL * 32;
  return b < 1 ? 1 : b;
}

}  // namespace

bool quant_linear_tc_supported(const QuantLinearArgs& a) {
  // groups tile the 128-column tiles: 32, 64, 128 or multiples of 128
  const bool groups_ok = a.group % 32 == 0 && (kKT % a.group == 0 || a.group % kKT == 0);
  return (a.x_dtype == kBF16 || a.x_dtype == kF16) && a.k % kKT == 0 && a.n % kRows == 0 &&
         groups_ok && a.ldx % 8 == 0 &&
         (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a.qweight) & 15) == 0;
}

// Splits of the k range: about two full waves of CTAs at the kernel's
// occupancy (one wave leaves a ragged tail when the tile count is not a
// multiple of the slots; more splits cost partial traffic).
int quant_linear_splits(const QuantLinearArgs& a, int sm_count) {
  const GemmShape g = gemm_shape(a);
  const long long ctas = (a.n / g.rows) * ((a.m + g.tokens - 1) / g.tokens);
  const long long tiles = a.k / kKT;
  int occ = 1;
  if (cudaFuncSetAttribute(g.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)g.smem) !=
          cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, g.fn, g.threads, g.smem) !=
          cudaSuccess ||
      occ < 1) {
    occ = 1;
  }
  const long long slots = (long long)occ * sm_count;
  long long splits = (2 * slots + ctas / 2) / (ctas > 0 ? ctas : 1);
  if (splits > tiles) splits = tiles;
  if (splits > 16) splits = 16;
  if (splits < 1) splits = 1;
  return (int)splits;
}

cudaError_t quant_linear_launch(const QuantLinearArgs& a, cudaStream_t stream) {
  if (a.m <= 0 || a.n <= 0) return cudaSuccess;
  void* args[] = {const_cast<QuantLinearArgs*>(&a)};
  if (!quant_linear_tc_supported(a)) {
    const void* fn = a.x_dtype == kBF16 ? reinterpret_cast<const void*>(&wq_generic_kernel<kBF16>)
                     : a.x_dtype == kF16 ? reinterpret_cast<const void*>(&wq_generic_kernel<kF16>)
                                         : reinterpret_cast<const void*>(&wq_generic_kernel<kF32>);
    const long long gx = (a.n + 63) / 64, gy = (a.m + 15) / 16;
    if (gx > 0x7fffffffLL || gy > 65535) return cudaErrorInvalidConfiguration;
    return launch_pdl(fn, dim3((unsigned)gx, (unsigned)gy), dim3(256), args, 0, stream);
  }
  const GemmShape g = gemm_shape(a);
  const long long gx = a.n / g.rows, gz = (a.m + g.tokens - 1) / g.tokens;
  if (gx > 0x7fffffffLL || gz > 65535 || a.splits > 65535) return cudaErrorInvalidConfiguration;
  cudaError_t e =
      cudaFuncSetAttribute(g.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)g.smem);
  if (e != cudaSuccess) return e;
  e = launch_pdl(g.fn, dim3((unsigned)gx, (unsigned)a.splits, (unsigned)gz),
                 dim3((unsigned)g.threads), args, g.smem, stream);
  if (e != cudaSuccess || a.partial == nullptr) return e;
  const void* rfn = a.x_dtype == kBF16 ? reinterpret_cast<const void*>(&wq_reduce_kernel<kBF16>)
                                       : reinterpret_cast<const void*>(&wq_reduce_kernel<kF16>);
  return launch_pdl(rfn, dim3((unsigned)grid_blocks(a.m * a.n, 256)), dim3(256), args, 0,
                    stream);
}

cudaError_t quant_linear_device_errors(unsigned* bits, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(bits, g_wq_err, sizeof(unsigned));
  if (e != cudaSuccess || !clear) return e;
  const unsigned zero = 0u;
  return cudaMemcpyToSymbol(g_wq_err, &zero, sizeof(unsigned));
}

cudaError_t dequantize_launch(const QuantLinearArgs& a, void* out, int out_dtype,
                              cudaStream_t stream) {
  if (a.n <= 0 || a.k <= 0) return cudaSuccess;
  const void* fn = out_dtype == kBF16 ? reinterpret_cast<const void*>(&wq_dequant_kernel<kBF16>)
                   : out_dtype == kF16 ? reinterpret_cast<const void*>(&wq_dequant_kernel<kF16>)
                                       : reinterpret_cast<const void*>(&wq_dequant_kernel<kF32>);
  void* args[] = {const_cast<QuantLinearArgs*>(&a), &out};
  return launch_pdl(fn, dim3((unsigned)grid_blocks(a.n * a.k, 256)), dim3(256), args, 0,
                    stream);
}

}  // namespace llmopt
