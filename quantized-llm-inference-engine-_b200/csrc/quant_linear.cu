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

// ---- 2- and 4-bit codes on the 5th-generation tensor cores ---------------------
//
// A CTA owns 128 output features (the 128 lanes of tensor memory, MMA M) and bn
// tokens (MMA N: the batch rounded up to 16, at most 256; larger batches take
// several token blocks) over a k range of whole 64-column slices.  Each weight
// is dequantized once per CTA and token block, straight into tensor memory as
// the MMA's A operand; the token rows are the B operand in shared memory.
// Warp roles:
// * warps 0-11 dequantize in three sets of four: set h = w / 4 takes the
//   slices s with s % 3 == h, warp w the 32 rows of lane quarter w % 4.
//   Thread r turns its row's 64 codes of a slice into the reference's weights
//   - (q - z) * s in float32, rounded once to the compute dtype - and stores
//   the 32 pairs into a 32-column A slot in tensor memory (tcgen05.st).  Each
//   set owns two slots, so a slot's barriers are only ever waited on by the
//   warps that saw all of its earlier phases;
// * warp 12 loads the codes: one TMA box of 128 rows x 128 bytes (256 columns,
//   128-byte swizzle) per stage of a 4-stage ring, plus the stage's group
//   scales (and zero points) by cp.async completing on the same mbarrier;
// * warp 13 loads the token rows: one TMA box of bn rows x 64 columns per
//   slice (K-major, 128-byte swizzle: the layout the MMA reads);
// * warp 14 issues, from one elected thread, the four tcgen05.mma (K = 16, A
//   from tensor memory) of each slice into the fp32 accumulator and commits
//   them to the barriers that free the A slot and the token slot.
// The dequantize warps then read the accumulator (tcgen05.ld, thread r =
// feature r) and write the output, or the split's fp32 partial.
// (kAInSmem = true instead writes A as K-major, 128-byte-swizzled tiles in
// shared memory for MMAs with both operands there: the same results, 10-30 %
// slower from the extra shared-memory traffic.)
//
// Dequantization without conversions: OR-ing nibble j of a code word (bits
// 4j..4j+3) into the float 2^23 gives 2^23 + q * 16^j exactly; one packed FMA
// by (16^-j, -(2^(23-4j) + c)) leaves q - c exactly (c = 2^(bits-1) for
// symmetric codes, 0 before an asymmetric zero point is subtracted), and one
// packed multiply by the scale rounds the product once, as the reference does.
//
// Every wait is bounded.  A wait that gives up sets g_wq_err and the CTA's
// abort flag; the other roles then stop at their next wait, the loaders wait
// (bounded) for the copies they issued, the MMA issuer's final commit drains
// the MMAs before tensor memory is read or freed, and the CTA writes NaN.
namespace tc05 {
constexpr int kBM = 128;                          // features per CTA
constexpr int kSliceK = 64;                       // k per slice: one A slot, one commit
constexpr int kSliceCols = kSliceK / 2;           // tensor-memory columns of an A slot
constexpr int kXBoxes = kSliceK / 64;             // 64-column token boxes per slice
constexpr int kWords = kSliceK / 8;               // 32-bit code words of a row per slice
constexpr int kQuarters = kSliceK / 32;           // group constants per row per slice
constexpr int kStageK = 256;                      // k per codes stage (128 bytes of a row)
constexpr int kSlicesPerStage = kStageK / kSliceK;
constexpr int kCodeStages = 4;
constexpr bool kAInSmem = false;                  // A tiles in shared memory (else tensor memory)
constexpr int kSlotsPerSet = kAInSmem ? 1 : 2;    // A slots of a set, reused only by it
constexpr int kMaxXSlots = 8;
constexpr int kDqWarps = 12;
constexpr int kSets = kDqWarps / 4;               // slices in flight in the dequantize warps
constexpr int kCodesWarp = kDqWarps;
constexpr int kTokensWarp = kDqWarps + 1;
constexpr int kMmaWarp = kDqWarps + 2;
constexpr int kThreads = (kDqWarps + 3) * 32;
constexpr int kMaxBN = 256;
constexpr int kATile = kBM * 128;                 // one A slot in shared memory: 16 KB
constexpr int kCodeBytes = kBM * kStageK / 2;     // 16 KB per stage
constexpr int kConstBytes = kSlicesPerStage * kQuarters * kBM * 4;   // [slice][32 cols][row]
constexpr int kASlots = kSets * kSlotsPerSet;
constexpr int kXBytes = kAInSmem ? 64 * 1024 : 128 * 1024;   // token-slice ring
constexpr int kOffCodes = 0;                      // offsets from the 1024-byte aligned base
constexpr int kOffA = kOffCodes + kCodeStages * kCodeBytes;
constexpr int kOffX = kOffA + (kAInSmem ? kASlots * kATile : 0);
constexpr int kOffS = kOffX + kXBytes;
constexpr int kOffZ = kOffS + kCodeStages * kConstBytes;
constexpr int kOffBar = kOffZ + kCodeStages * kConstBytes;
constexpr int kBarBytes = 512;
constexpr int kSmem = kOffBar + kBarBytes + 1024; // + alignment slack
// tensor memory: the accumulator [kAccCol, kAccCol + bn), and the A ring in
// columns [0, 256) when it is not in shared memory
constexpr uint32_t kTmemCols = kAInSmem ? 256 : 512;
constexpr int kAccCol = kAInSmem ? 0 : 256;
static_assert(kAccCol + kMaxBN <= (int)kTmemCols, "tensor-memory columns");
static_assert(kSmem <= 227 * 1024, "shared memory");
static_assert(kOffX % 1024 == 0 && kOffS % 1024 == 0 && kOffA % 1024 == 0, "TMA / MMA tiles");
static_assert(kDqWarps % 4 == 0 && kSets <= kSlicesPerStage, "dequantize warp sets");
static_assert(kAInSmem || kASlots * kSliceCols <= kAccCol, "A ring");
static_assert(!kAInSmem || kSliceK == 64, "a shared-memory A slot is one 128-byte swizzle span");

struct Bars {
  uint64_t codes_full[kCodeStages];   // TMA bytes + the 32 cp.async lanes + 1
  uint64_t codes_empty[kCodeStages];  // the dequantize warps
  uint64_t x_full[kMaxXSlots];        // TMA bytes + 1
  uint64_t x_empty[kMaxXSlots];       // MMA commit
  uint64_t a_full[kASlots];           // the 4 dequantize warps of the slice's set
  uint64_t a_empty[kASlots];          // MMA commit
  uint64_t acc_full;                  // MMA commit after the last slice
  uint32_t tmem;
  uint32_t abort;
};
static_assert(sizeof(Bars) <= kBarBytes, "barrier block");

// Tokens per CTA and token-slice ring depth (host and device agree on both).
// A slot of slice s and how many times that slot was used before it: a set
// owns its slots, so the warps that wait on a slot's barriers are the ones that
// saw every one of its earlier phases.
__host__ __device__ constexpr int a_slot(long long s) {
  return (int)(s % kSets) * kSlotsPerSet + (int)((s / kSets) % kSlotsPerSet);
}
__host__ __device__ constexpr long long a_use(long long s) { return s / kSets / kSlotsPerSet; }
__host__ __device__ constexpr int bn_of(long long m) {
  return m >= kMaxBN ? kMaxBN : (int)((m + 15) & ~15LL);
}
__host__ __device__ constexpr int x_slots(int bn) {
  return kXBytes / (bn * 128 * kXBoxes) < kMaxXSlots ? kXBytes / (bn * 128 * kXBoxes)
                                                      : kMaxXSlots;
}
}  // namespace tc05

__device__ unsigned g_wq_err;               // LLMOPT_DEVERR_* bits of the tcgen05 path

__device__ __forceinline__ void fmul2(float& x0, float& x1, float a0, float a1, uint64_t bb) {
  asm("{\n\t.reg .b64 ra, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mul.rn.f32x2 rd, ra, %4;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(x0), "=f"(x1)
      : "f"(a0), "f"(a1), "l"(bb));
}
__device__ __forceinline__ void fadd2(float& x0, float& x1, uint64_t bb) {
  asm("{\n\t.reg .b64 ra;\n\t"
      "mov.b64 ra, {%0, %1};\n\t"
      "add.rn.f32x2 ra, ra, %2;\n\t"
      "mov.b64 {%0, %1}, ra;\n\t}"
      : "+f"(x0), "+f"(x1)
      : "l"(bb));
}

// Constants of one row and group: (16^-j, -(2^(23-4j) + c)) for nibbles j = 0, 1
// and j = 2, 3 of a half-word, the scale pair and the negated zero-point pair.
struct DqConst {
  uint64_t m01, c01, m23, c23;
};
__device__ __forceinline__ DqConst dq_const(float c) {
  return {pack2f(1.f, 0.0625f), pack2f(-(8388608.f + c), -(524288.f + c)),
          pack2f(0.00390625f, 0.000244140625f), pack2f(-(32768.f + c), -(2048.f + c))};
}

// Eight codes (code j in bits 4j..4j+3 of w) -> four 16-bit pairs of weights,
// the lower half holding the even code.
template <int DT, bool SYM>
__device__ __forceinline__ void dequant8(uint32_t w, const DqConst& k, uint64_t ss, uint64_t nz,
                                         uint32_t* out) {
  constexpr uint32_t e = 0x4B000000u;
  const uint32_t u = w >> 16;
  float d[8];
  ffma2(d[0], d[1], __uint_as_float(e | (w & 0xFu)), __uint_as_float(e | (w & 0xF0u)), k.m01,
        k.c01);
  ffma2(d[2], d[3], __uint_as_float(e | (w & 0xF00u)), __uint_as_float(e | (w & 0xF000u)),
        k.m23, k.c23);
  ffma2(d[4], d[5], __uint_as_float(e | (u & 0xFu)), __uint_as_float(e | (u & 0xF0u)), k.m01,
        k.c01);
  ffma2(d[6], d[7], __uint_as_float(e | (u & 0xF00u)), __uint_as_float(e | (u & 0xF000u)),
        k.m23, k.c23);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (!SYM) fadd2(d[2 * i], d[2 * i + 1], nz);
    fmul2(d[2 * i], d[2 * i + 1], d[2 * i], d[2 * i + 1], ss);
    out[i] = pack2<DT>(d[2 * i], d[2 * i + 1]);
  }
}

__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

template <int DT, bool SYM>
__global__ void __launch_bounds__(tc05::kThreads, 1)
    wq_gemm_tc05_kernel(const QuantLinearArgs a, const __grid_constant__ CUtensorMap tm_codes,
                        const __grid_constant__ CUtensorMap tm_x) {
  using namespace tc05;
  griddep_wait();
  griddep_launch_dependents();
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Bars* bars = reinterpret_cast<Bars*>(base + kOffBar);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int bn = bn_of(a.m);
  const int xs = x_slots(bn);
  const long long rbase = (long long)blockIdx.x * kBM;
  const long long m0 = (long long)blockIdx.z * bn;
  const long long kb = (long long)blockIdx.y * a.k_per_split;
  const long long ke = kb + a.k_per_split < a.k ? kb + a.k_per_split : a.k;
  const int nslices = (int)((ke - kb) / kSliceK);
  const int nstages = (nslices + kSlicesPerStage - 1) / kSlicesPerStage;
  const long long groups = a.k / a.group;
  const uint32_t ug = (uint32_t)a.group;                         // k < 2^31 (host check)

  if (threadIdx.x == 0) {
    for (int i = 0; i < kCodeStages; ++i) {
      mbar_init(&bars->codes_full[i], 1 + 32);
      mbar_init(&bars->codes_empty[i], kDqWarps);
    }
    for (int i = 0; i < kMaxXSlots; ++i) {
      mbar_init(&bars->x_full[i], 1);
      mbar_init(&bars->x_empty[i], 1);
    }
    for (int i = 0; i < kASlots; ++i) {
      mbar_init(&bars->a_full[i], 4);
      mbar_init(&bars->a_empty[i], 1);
    }
    mbar_init(&bars->acc_full, 1);
    bars->abort = 0u;
    mbar_init_fence();
  }
  if (warp == 0) {
    tc::tmem_alloc(&bars->tmem, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = bars->tmem;

  volatile uint32_t* abort_flag = &bars->abort;
  // Warp-uniform bounded wait: false once any wait of the CTA has given up.
  auto wait = [&](uint64_t* bar, unsigned parity, unsigned what) -> bool {
    bool ok = mbar_try_wait(bar, parity);
    if (!ok) {
      const long long t0 = clock64();
      while (*abort_flag == 0u) {
        if (mbar_try_wait_sleep(bar, parity, 20000u)) {
          ok = true;
          break;
        }
        if (clock64() - t0 > kWaitLimitCycles) {
          atomicOr(&g_wq_err, kErrWaitTimeout | what);
          *abort_flag = 1u;
          break;
        }
      }
    }
    return __all_sync(0xffffffffu, ok);
  };

  if (warp == kCodesWarp) {
    // ---- codes and group constants, one 256-column stage at a time ----
    if (lane == 0) prefetch_tensormap(&tm_codes);
    int issued = 0;
    for (int st = 0; st < nstages; ++st) {
      const int cs = st % kCodeStages;
      if (st >= kCodeStages &&
          !wait(&bars->codes_empty[cs], (unsigned)((st / kCodeStages - 1) & 1), kErrWaitSlot)) {
        break;
      }
      const long long c0 = kb + (long long)st * kStageK;
      const int in_stage = nslices - st * kSlicesPerStage < kSlicesPerStage
                               ? nslices - st * kSlicesPerStage
                               : kSlicesPerStage;
      if (lane == 0) {
        mbar_arrive_expect_tx(&bars->codes_full[cs], (unsigned)kCodeBytes);
        tc::tma_load_2d(base + kOffCodes + cs * kCodeBytes, &tm_codes, &bars->codes_full[cs],
                        (int)(c0 / 2), (int)rbase);
      }
      // per 32 columns of each slice of the stage, its group's constants:
      // [slice][32 columns][row] floats, so the dequantize warps read them
      // with no group arithmetic
      float* sst = reinterpret_cast<float*>(base + kOffS + cs * kConstBytes);
      float* zst = reinterpret_cast<float*>(base + kOffZ + cs * kConstBytes);
      for (int sub = 0; sub < in_stage; ++sub) {
        for (int hf = 0; hf < kQuarters; ++hf) {
          const uint32_t g = (uint32_t)(c0 + sub * kSliceK + hf * 32) / ug;
          const int o = (sub * kQuarters + hf) * kBM;
#pragma unroll
          for (int j = 0; j < kBM / 32; ++j) {
            const int r = lane + 32 * j;
            const long long gi = (rbase + r) * groups + g;
            cp_async4(sst + o + r, a.scales + gi);
            if (!SYM) cp_async4(zst + o + r, a.zeros + gi);
          }
        }
      }
      cp_async_mbar_arrive_noinc(&bars->codes_full[cs]);
      issued = st + 1;
    }
    // the copies this warp issued land before the CTA can exit
    for (int st = issued - kCodeStages > 0 ? issued - kCodeStages : 0; st < issued; ++st) {
      if (!mbar_wait(&bars->codes_full[st % kCodeStages], (unsigned)((st / kCodeStages) & 1))) {
        if (lane == 0) atomicOr(&g_wq_err, kErrWaitTimeout | kErrWaitDrain);
        *abort_flag = 1u;
      }
    }
  } else if (warp == kTokensWarp) {
    // ---- token rows, one 64-column slice at a time ----
    if (lane == 0) prefetch_tensormap(&tm_x);
    const unsigned boxbytes = (unsigned)bn * 128u;
    int issued = 0, slot = 0, round = 0;
    for (int s = 0; s < nslices; ++s) {
      if (s >= xs && !wait(&bars->x_empty[slot], (unsigned)((round - 1) & 1), kErrWaitSlot)) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(&bars->x_full[slot], boxbytes * kXBoxes);
#pragma unroll
        for (int bx = 0; bx < kXBoxes; ++bx) {
          tc::tma_load_2d(base + kOffX + (slot * kXBoxes + bx) * (int)boxbytes, &tm_x,
                          &bars->x_full[slot], (int)(kb + (long long)s * kSliceK + 64 * bx),
                          (int)m0);
        }
      }
      __syncwarp();
      issued = s + 1;
      if (++slot == xs) {
        slot = 0;
        ++round;
      }
    }
    for (int s = issued - xs > 0 ? issued - xs : 0; s < issued; ++s) {
      if (!mbar_wait(&bars->x_full[s % xs], (unsigned)((s / xs) & 1))) {
        if (lane == 0) atomicOr(&g_wq_err, kErrWaitTimeout | kErrWaitDrain);
        *abort_flag = 1u;
      }
    }
  } else if (warp == kMmaWarp) {
    // ---- MMA issue ----
    const bool issuer = tc::elect_one();
    const uint32_t idesc = tc::instr_desc_f16(DT == kBF16, kBM, bn, false, false);
    const uint32_t x0 = smem_addr(base + kOffX);
    const uint32_t xbox = (uint32_t)bn * 128u;
    int slot = 0, round = 0;
    for (int s = 0; s < nslices; ++s) {
      const int as = a_slot(s);
      if (!wait(&bars->a_full[as], (unsigned)(a_use(s) & 1), kErrWaitData)) break;
      if (!wait(&bars->x_full[slot], (unsigned)(round & 1), kErrWaitData)) break;
      if (issuer) {
        tc::fence_after_sync();
#pragma unroll
        for (int bx = 0; bx < kXBoxes; ++bx) {
          const uint64_t bdesc =
              tc::smem_desc_sw128(x0 + (slot * kXBoxes + bx) * xbox, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            // +32 bytes per K = 16 step: +2 in the descriptor's address field
            if constexpr (kAInSmem) {
              const uint64_t adesc =
                  tc::smem_desc_sw128(smem_addr(base + kOffA + as * kATile), 16, 1024);
              tc::mma_f16(tmem + kAccCol, adesc + 2 * (bx * 4 + kk), bdesc + 2 * kk, idesc,
                          (s > 0 || bx > 0 || kk > 0) ? 1u : 0u);
            } else {
              tc::mma_f16_ts(tmem + kAccCol, tmem + as * kSliceCols + (bx * 4 + kk) * 8,
                             bdesc + 2 * kk, idesc, (s > 0 || bx > 0 || kk > 0) ? 1u : 0u);
            }
          }
        }
        tc::commit(&bars->a_empty[as]);
        tc::commit(&bars->x_empty[slot]);
      }
      __syncwarp();
      if (++slot == xs) {
        slot = 0;
        ++round;
      }
    }
    // covers every MMA this thread issued, also after an abort
    if (issuer) tc::commit(&bars->acc_full);
    __syncwarp();
  } else {
    // ---- dequantize (warps 0 .. kDqWarps - 1) ----
    const int q = warp & 3;                 // lane quarter
    const int h = warp >> 2;                // set: slices s with s % kSets == h
    const int r = q * 32 + lane;            // row of the CTA = tensor-memory lane
    const uint32_t tlane = tmem + ((uint32_t)(q * 32) << 16);
    const float zc = SYM ? (float)(1 << (a.bits - 1)) : 0.f;
    const DqConst kc = dq_const(zc);
    for (int s = h; s < nslices; s += kSets) {
      const int st = s / kSlicesPerStage;
      const int sub = s % kSlicesPerStage;
      const int cs = st % kCodeStages;
      const int in_stage = nslices - st * kSlicesPerStage < kSlicesPerStage
                               ? nslices - st * kSlicesPerStage
                               : kSlicesPerStage;
      // the warp's first slice of the stage waits for it (a set's slices of a
      // stage are kSets apart, so only the first has sub < kSets)
      if (sub < kSets &&
          !wait(&bars->codes_full[cs], (unsigned)((st / kCodeStages) & 1), kErrWaitData)) {
        break;
      }
      // this slice's kSliceK / 2 bytes of row r: 16-byte chunks kQuarters * sub
      // + i, stored at chunk ^ (r % 8) by the 128-byte swizzle
      const unsigned char* crow = base + kOffCodes + cs * kCodeBytes + r * 128;
      uint32_t words[kWords];
#pragma unroll
      for (int i = 0; i < kWords / 4; ++i) {
        const uint4 w =
            *reinterpret_cast<const uint4*>(crow + 16 * ((kQuarters * sub + i) ^ (r & 7)));
        words[4 * i] = w.x;
        words[4 * i + 1] = w.y;
        words[4 * i + 2] = w.z;
        words[4 * i + 3] = w.w;
      }
      const int o = sub * kQuarters * kBM + r;
      const float* sst = reinterpret_cast<const float*>(base + kOffS + cs * kConstBytes) + o;
      const float* zst = reinterpret_cast<const float*>(base + kOffZ + cs * kConstBytes) + o;
      float sc[kQuarters], zp[kQuarters];
#pragma unroll
      for (int i = 0; i < kQuarters; ++i) {
        sc[i] = sst[i * kBM];
        zp[i] = SYM ? 0.f : zst[i * kBM];
      }
      // The warp's last slice of the stage releases it, but only once the math
      // below has consumed the loaded words and constants: an arrival right
      // after the loads let the codes warp refill the stage while shared-memory
      // loads were still in flight, and those returned the next stage's bytes.
      const bool last_in_stage = sub + kSets >= in_stage;
      const int as = a_slot(s);
      if (a_use(s) > 0 &&
          !wait(&bars->a_empty[as], (unsigned)((a_use(s) - 1) & 1), kErrWaitSlot)) {
        break;
      }
      tc::fence_after_sync();
#pragma unroll
      for (int hh = 0; hh < kWords / 8; ++hh) {   // 64 codes -> 32 columns per store
        uint32_t out[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) {         // codes 8c' .. 8c' + 7, c' = 8 hh + c
          const int q4 = (8 * hh + c) / 4;    // its 32-column quarter
          dequant8<DT, SYM>(words[8 * hh + c], kc, pack2f(sc[q4], sc[q4]),
                            pack2f(-zp[q4], -zp[q4]), out + 4 * c);
        }
        if (hh == kWords / 8 - 1 && last_in_stage) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->codes_empty[cs]);
        }
        if constexpr (kAInSmem) {
          // row r of the K-major A tile, 16-byte chunk c at c ^ (r % 8) (the
          // 128-byte swizzle the MMA's descriptor names)
          unsigned char* arow = base + kOffA + as * kATile + r * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            *reinterpret_cast<uint4*>(arow + 16 * ((4 * hh + c) ^ (r & 7))) =
                make_uint4(out[4 * c], out[4 * c + 1], out[4 * c + 2], out[4 * c + 3]);
          }
        } else {
          tc::tmem_st32u(tlane + as * kSliceCols + 32 * hh, out);
        }
      }
      if constexpr (kAInSmem) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // for the MMA's reads
      } else {
        tc::tmem_wait_st();
        tc::fence_before_sync();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->a_full[as]);
    }

    // ---- epilogue: accumulator -> output (or the split's partial) ----
    bool ok = mbar_wait(&bars->acc_full, 0u);
    if (!ok) {
      if (lane == 0) atomicOr(&g_wq_err, kErrWaitTimeout | kErrWaitDrain);
      *abort_flag = 1u;
    }
    ok = __all_sync(0xffffffffu, ok);
    tc::fence_after_sync();
    ok = ok && *abort_flag == 0u && nslices > 0;
    const long long f = rbase + r;
    const long long m_end = m0 + bn < a.m ? m0 + bn : a.m;
    float bias = 0.f;
    if (a.partial == nullptr && a.bias != nullptr) bias = load_f32<DT>(a.bias, f);
    for (int cb = h; cb * 32 < bn; cb += kSets) {
      float v[32];
      tc::tmem_ld32(tlane + kAccCol + cb * 32, v);
      tc::tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const long long tok = m0 + cb * 32 + j;
        if (tok >= m_end) break;
        const float val = ok ? v[j] : __int_as_float(0x7FC00000);   // NaN after a give-up
        if (a.partial != nullptr) {
          a.partial[((long long)blockIdx.y * a.m + tok) * a.n + f] = val;
        } else {
          store_f32<DT>(a.out, tok * a.ldo + f, val + bias);
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
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

// Which 2- and 4-bit calls the tcgen05 kernel takes (n % 128 == 0, groups of
// whole 32-column pieces): batches above kTc05MinTokens tokens by default;
// LLMOPT_B200_QUANT_TC05=1 every batch, =0 none.  (At 1 to 16 tokens the
// mma.sync kernel's 8- and 32-token tiles are as fast or faster: the tcgen05
// kernel's time is its dequantization, the same for any batch up to 256.)
constexpr long long kTc05MinTokens = 16;
bool tc05_enabled(long long m) {
  static const int mode = [] {
    const char* v = std::getenv("LLMOPT_B200_QUANT_TC05");
    return v == nullptr ? -1 : (v[0] == '1' ? 1 : 0);
  }();
  return mode == 1 || (mode < 0 && m > kTc05MinTokens);
}

bool tc05_takes(const QuantLinearArgs& a) {
  // TMA coordinates and the kernel's column arithmetic are 32-bit
  return a.bits < 8 && a.n % tc05::kBM == 0 && a.group % 32 == 0 &&
         a.k < (1LL << 31) && a.n < (1LL << 31) && a.m < (1LL << 31);
}

template <int DT>
const void* tc05_fn(bool sym) {
  return sym ? reinterpret_cast<const void*>(&wq_gemm_tc05_kernel<DT, true>)
             : reinterpret_cast<const void*>(&wq_gemm_tc05_kernel<DT, false>);
}

// The tensor-core kernel a call runs and its CTA shape.
struct GemmShape {
  const void* fn;
  int threads;
  size_t smem;
  long long rows;      // output features per CTA
  long long tokens;    // tokens per CTA
  bool tc05;
};

GemmShape gemm_shape(const QuantLinearArgs& a) {
  if (tc05_enabled(a.m) && tc05_takes(a)) {
    const void* fn = a.x_dtype == kBF16 ? tc05_fn<kBF16>(a.symmetric != 0)
                                        : tc05_fn<kF16>(a.symmetric != 0);
    return {fn, tc05::kThreads, (size_t)tc05::kSmem, tc05::kBM, tc05::bn_of(a.m), true};
  }
  const int mt = tokens_per_cta(a);
  return {gemm_fn(a), kThreads, gemm_smem(a, mt), kRows, mt, false};
}

// tcgen05 kernel, one CTA per SM: the split count that minimizes the waves of
// CTAs times the 128-column tiles per CTA, plus one tile per split for the
// partial write and the reduce.
int tc05_splits(long long ctas, long long tiles, int sms) {
  long long best = -1;
  int best_splits = 1;
  for (long long want = 1; want <= 16 && want <= tiles; ++want) {
    const long long per = (tiles + want - 1) / want;
    const long long used = (tiles + per - 1) / per;
    const long long waves = (ctas * used + sms - 1) / sms;
    const long long cost = waves * per + (used > 1 ? used : 0);
    if (best < 0 || cost < best) {
      best = cost;
      best_splits = (int)used;
    }
  }
  return best_splits;
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
  if (g.tc05) return tc05_splits(ctas, tiles, sm_count);
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
  if (g.tc05) {
    // codes: uint8 [n, k/2], boxes of 128 rows x 128 bytes; token rows: 16-bit
    // [m, ldx], boxes of bn rows x 64 columns (rows past m read as zeros)
    CUtensorMap tm_codes, tm_x;
    if (!tensor_map_2d(&tm_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.qweight, (uint64_t)a.k / 2,
                       (uint64_t)a.n, (uint64_t)a.k / 2, 128, tc05::kBM) ||
        !tensor_map_2d(&tm_x, CU_TENSOR_MAP_DATA_TYPE_UINT16, a.x, (uint64_t)a.k, (uint64_t)a.m,
                       (uint64_t)a.ldx * 2, 64, (uint32_t)g.tokens)) {
      return cudaErrorInvalidValue;
    }
    void* targs[] = {const_cast<QuantLinearArgs*>(&a), &tm_codes, &tm_x};
    e = launch_pdl(g.fn, dim3((unsigned)gx, (unsigned)a.splits, (unsigned)gz),
                   dim3((unsigned)g.threads), targs, g.smem, stream);
  } else {
    e = launch_pdl(g.fn, dim3((unsigned)gx, (unsigned)a.splits, (unsigned)gz),
                   dim3((unsigned)g.threads), args, g.smem, stream);
  }
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
