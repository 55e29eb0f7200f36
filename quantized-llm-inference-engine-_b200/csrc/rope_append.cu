// Rotary position embedding of q and k fused with the K/V append and the cast
// to the cache dtype: the steps of PagedAttentionLayer.forward between the
// projections and attention (src/llmopt/model/layers.py:106-134).
//
// The reference looks the cos/sin rows of the positions up in its tables
// (src/llmopt/model/rotary.py:103-121, after a positions.max().item() host
// sync), casts them to the model dtype, rotates q and k with
// x * cos + rotate_half(x) * sin (rotary.py:16-46) - every product and the sum
// a separate tensor op rounded to the model dtype - then permutes k and v to
// [seq, q_len, kv_heads, head_dim], makes them contiguous and appends them
// with write_decode (q_len == 1) or write (layers.py:118-132).  Here one kernel
// reads the projection outputs once and writes the rotated query plus the
// cache rows, with the same rounding steps (so the results are bit-identical)
// and the same destination rules as kv_cache.cu.
//
// Grid (batch, ceil(q_len / kTokPerCta)); the CTA's warps share the (token,
// row) items of its tokens, a row being one head of q (rotated to q_out), of k
// (rotated to the cache) or of v (copied to the cache).  A position outside
// [-max_pos, max_pos) flags kErrPosition and skips its token (the reference
// raises); negative positions wrap as torch indexing does.
#include <limits.h>

#include "common.cuh"
#include "kernels.h"

namespace llmopt {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kTokPerCta = 8;

__device__ __forceinline__ float load_any(const void* p, int dt, long long i) {
  if (dt == kF32) return static_cast<const float*>(p)[i];
  if (dt == kF16) return __half2float(static_cast<const __half*>(p)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

// One torch op's result in dtype DT: exact for fp32, rounded otherwise.
template <int DT>
__device__ __forceinline__ float op_round(float x) {
  return round_through<DT>(x);
}

// x * cos + rotate_half(x) * sin for the pair (x1, x2) = (x[e], x[e + D/2]):
// out[e] = x1 c1 + (-x2) s1,  out[e + D/2] = x2 c2 + x1 s2, each product and
// the sum rounded to the model dtype (no fused multiply-add).
template <int DT>
__device__ __forceinline__ void rotate_pair(float x1, float x2, float c1, float c2, float s1,
                                            float s2, float* o1, float* o2) {
  const float a1 = op_round<DT>(__fmul_rn(x1, c1));
  const float b1 = op_round<DT>(__fmul_rn(-x2, s1));
  const float a2 = op_round<DT>(__fmul_rn(x2, c2));
  const float b2 = op_round<DT>(__fmul_rn(x1, s2));
  *o1 = op_round<DT>(__fadd_rn(a1, b1));
  *o2 = op_round<DT>(__fadd_rn(a2, b2));
}

// Two consecutive elements of a 16- or 32-bit row as floats (8-byte or 4-byte load).
template <int DT>
__device__ __forceinline__ float2 load2(const void* p, long long i) {
  if constexpr (DT == kF32) {
    return *reinterpret_cast<const float2*>(static_cast<const float*>(p) + i);
  } else if constexpr (DT == kF16) {
    return __half22float2(*reinterpret_cast<const __half2*>(static_cast<const __half*>(p) + i));
  } else {
    return __bfloat1622float2(
        *reinterpret_cast<const __nv_bfloat162*>(static_cast<const __nv_bfloat16*>(p) + i));
  }
}

template <int DT>
__device__ __forceinline__ void store2(void* p, long long i, float x, float y) {
  if constexpr (DT == kF32) {
    *reinterpret_cast<float2*>(static_cast<float*>(p) + i) = make_float2(x, y);
  } else {
    *reinterpret_cast<uint32_t*>(static_cast<typename ElemT<DT>::T*>(p) + i) = pack2<DT>(x, y);
  }
}

__device__ __forceinline__ float2 load2_any(const void* p, int dt, long long i) {
  if (dt == kF32) return *reinterpret_cast<const float2*>(static_cast<const float*>(p) + i);
  if (dt == kF16) return load2<kF16>(p, i);
  return load2<kBF16>(p, i);
}

// Rotates one head row from `src` (model dtype) into `dst` (dtype OUT_DT).
template <int IN_DT, int OUT_DT>
__device__ __forceinline__ void rotate_row(const RopeArgs& a, const void* src_base,
                                           long long src, void* dst_base, long long dst,
                                           long long pos, int lane) {
  const int D = a.head_dim;
  const int half = D / 2;
  const long long trow = pos * D;
  if (a.pairs) {
    for (int e = 2 * lane; e < half; e += 64) {
      const float2 c1 = load2_any(a.cos_t, a.tab_dtype, trow + e);
      const float2 c2 = load2_any(a.cos_t, a.tab_dtype, trow + e + half);
      const float2 s1 = load2_any(a.sin_t, a.tab_dtype, trow + e);
      const float2 s2 = load2_any(a.sin_t, a.tab_dtype, trow + e + half);
      const float2 x1 = load2<IN_DT>(src_base, src + e);
      const float2 x2 = load2<IN_DT>(src_base, src + e + half);
      float o1x, o2x, o1y, o2y;
      rotate_pair<IN_DT>(x1.x, x2.x, op_round<IN_DT>(c1.x), op_round<IN_DT>(c2.x),
                         op_round<IN_DT>(s1.x), op_round<IN_DT>(s2.x), &o1x, &o2x);
      rotate_pair<IN_DT>(x1.y, x2.y, op_round<IN_DT>(c1.y), op_round<IN_DT>(c2.y),
                         op_round<IN_DT>(s1.y), op_round<IN_DT>(s2.y), &o1y, &o2y);
      store2<OUT_DT>(dst_base, dst + e, o1x, o1y);
      store2<OUT_DT>(dst_base, dst + e + half, o2x, o2y);
    }
  } else {
    for (int e = lane; e < half; e += 32) {
      const float c1 = op_round<IN_DT>(load_any(a.cos_t, a.tab_dtype, trow + e));
      const float c2 = op_round<IN_DT>(load_any(a.cos_t, a.tab_dtype, trow + e + half));
      const float s1 = op_round<IN_DT>(load_any(a.sin_t, a.tab_dtype, trow + e));
      const float s2 = op_round<IN_DT>(load_any(a.sin_t, a.tab_dtype, trow + e + half));
      float o1, o2;
      rotate_pair<IN_DT>(load_f32<IN_DT>(src_base, src + e),
                         load_f32<IN_DT>(src_base, src + e + half), c1, c2, s1, s2, &o1, &o2);
      store_f32<OUT_DT>(dst_base, dst + e, o1);
      store_f32<OUT_DT>(dst_base, dst + e + half, o2);
    }
  }
}

constexpr int kRowsPerItem = 8;

// One v head row to the cache (cast only): 16-byte vectors when allowed.
template <int IN_DT, int KV_DT>
__device__ __forceinline__ void copy_v_row(const RopeArgs& a, long long tok, int h,
                                           long long dst, int lane) {
  const int D = a.head_dim;
  const long long src = tok * a.v_row + (long long)h * D;
  const long long out = dst + (long long)h * D;
  if (a.vrow16) {
    using T = typename ElemT<KV_DT>::T;
    const int per = 16 / (int)sizeof(T);
    for (int e = lane * per; e < D; e += 32 * per) {
      *reinterpret_cast<uint4*>(static_cast<T*>(a.v_cache) + out + e) =
          *reinterpret_cast<const uint4*>(static_cast<const T*>(a.v_in) + src + e);
    }
  } else {
    for (int e = lane; e < D; e += 32) {
      store_f32<KV_DT>(a.v_cache, out + e, load_f32<IN_DT>(a.v_in, src + e));
    }
  }
}

// Up to kRowsPerItem rows [r0, r0 + 8) of one token on the paired path
// (head_dim % 4 == 0, head_dim <= 4 * 32 * M): lane l owns the element pairs
// (2l + 64m, 2l + 64m + 1) of each half, m < M.  The token's cos/sin pairs are
// loaded once; each row's two input pairs per m are loaded for all rows first.
template <int IN_DT, int KV_DT, int M>
__device__ __forceinline__ void rotate_rows_paired(const RopeArgs& a, long long s, int i,
                                                   long long tok, long long pos, long long dst,
                                                   int r0, int rows, int lane) {
  const int D = a.head_dim;
  const int half = D / 2;
  const long long trow = pos * D;
  float2 c1[M], c2[M], s1[M], s2[M];
  bool live[M];
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const int e = 2 * lane + 64 * m;
    live[m] = e < half;
    if (live[m]) {
      c1[m] = load2_any(a.cos_t, a.tab_dtype, trow + e);
      c2[m] = load2_any(a.cos_t, a.tab_dtype, trow + e + half);
      s1[m] = load2_any(a.sin_t, a.tab_dtype, trow + e);
      s2[m] = load2_any(a.sin_t, a.tab_dtype, trow + e + half);
      c1[m] = make_float2(op_round<IN_DT>(c1[m].x), op_round<IN_DT>(c1[m].y));
      c2[m] = make_float2(op_round<IN_DT>(c2[m].x), op_round<IN_DT>(c2[m].y));
      s1[m] = make_float2(op_round<IN_DT>(s1[m].x), op_round<IN_DT>(s1[m].y));
      s2[m] = make_float2(op_round<IN_DT>(s2[m].x), op_round<IN_DT>(s2[m].y));
    }
  }
  // Loads of every rotated row of the item first.
  float2 x1[kRowsPerItem][M], x2[kRowsPerItem][M];
#pragma unroll
  for (int j = 0; j < kRowsPerItem; ++j) {
    const int r = r0 + j;
    const bool rq = r < a.num_heads;
    const bool rk = !rq && r < a.num_heads + a.kv_heads && dst >= 0;
    const void* base = rq ? a.q_in : a.k_in;
    const long long src = rq ? tok * a.q_row + (long long)r * D
                             : tok * a.k_row + (long long)(r - a.num_heads) * D;
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const int e = 2 * lane + 64 * m;
      if ((rq || rk) && r < rows && live[m]) {
        x1[j][m] = load2<IN_DT>(base, src + e);
        x2[j][m] = load2<IN_DT>(base, src + e + half);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kRowsPerItem; ++j) {
    const int r = r0 + j;
    if (r >= rows) break;
    if (r < a.num_heads + a.kv_heads) {
      const bool rq = r < a.num_heads;
      if (!rq && dst < 0) continue;
#pragma unroll
      for (int m = 0; m < M; ++m) {
        if (!live[m]) continue;
        const int e = 2 * lane + 64 * m;
        float o1x, o2x, o1y, o2y;
        rotate_pair<IN_DT>(x1[j][m].x, x2[j][m].x, c1[m].x, c2[m].x, s1[m].x, s2[m].x, &o1x,
                           &o2x);
        rotate_pair<IN_DT>(x1[j][m].y, x2[j][m].y, c1[m].y, c2[m].y, s1[m].y, s2[m].y, &o1y,
                           &o2y);
        if (rq) {
          const long long out = s * a.qo_s + (long long)r * a.qo_h + (long long)i * a.qo_t;
          store2<IN_DT>(a.q_out, out + e, o1x, o1y);
          store2<IN_DT>(a.q_out, out + e + half, o2x, o2y);
        } else {
          const long long out = dst + (long long)(r - a.num_heads) * D;
          store2<KV_DT>(a.k_cache, out + e, o1x, o1y);
          store2<KV_DT>(a.k_cache, out + e + half, o2x, o2y);
        }
      }
    } else if (dst >= 0) {
      copy_v_row<IN_DT, KV_DT>(a, tok, r - a.num_heads - a.kv_heads, dst, lane);
    }
  }
}

// M: element pairs per lane of the paired path (1: head_dim <= 128, 2: <= 256),
// 0: the element-wise path.  Separate kernels, so the common M = 1 carries no
// registers of the others.
template <int IN_DT, int KV_DT, int M>
__global__ void __launch_bounds__(kThreads, 3) rope_append_kernel(const RopeArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  const long long s = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long bs = a.block_size;
  const long long W = a.table_width;
  const int D = a.head_dim;
  const int half = D / 2;
  const bool decode = a.q_len == 1;

  // ---- where this sequence's rows go (kv_cache.cu's write / write_decode) ----
  const long long start = load_index(a.offsets, a.off_i64, s);
  long long stop_col = LLONG_MAX;
  long long dec_dst = -1;  // write_decode: row offset in the cache, -1 if not written
  if (!decode) {
    const long long c0 = floordiv(start, bs);
    const long long c_last = floordiv(start + a.q_len - 1, bs);
    __shared__ unsigned long long first_stop;
    if (threadIdx.x == 0) first_stop = ULLONG_MAX;
    __syncthreads();
    for (long long c = c0 + threadIdx.x; c <= c_last; c += kThreads) {
      unsigned reason = 0;
      bool stop = false;
      if (c >= W) {
        stop = true;
      } else if (c < -W) {
        stop = true;
        reason = 2;
      } else {
        const long long id =
            load_index(a.table, a.table_i64, s * a.table_stride + (c < 0 ? c + W : c));
        if (id < 0) {
          stop = true;
        } else if (id >= a.num_blocks) {
          stop = true;
          reason = 1;
        }
      }
      if (stop) atomicMin(&first_stop, (unsigned long long)(4 * (c - c0) + reason));
    }
    __syncthreads();
    const unsigned long long key = first_stop;
    stop_col = key == ULLONG_MAX ? LLONG_MAX : c0 + (long long)(key >> 2);
    if (threadIdx.x == 0 && blockIdx.y == 0 && key != ULLONG_MAX) {
      const unsigned reason = (unsigned)(key & 3);
      if (reason == 1) record_error(a.err, kErrBlockId);
      if (reason == 2) record_error(a.err, kErrTableWidth);
    }
  } else {
    const long long col = floordiv(start, bs);
    if (col < -W || col >= W) {
      if (threadIdx.x == 0) record_error(a.err, kErrTableWidth);
    } else {
      long long id =
          load_index(a.table, a.table_i64, s * a.table_stride + (col < 0 ? col + W : col));
      if (id < 0 || id >= a.num_blocks) id = 0;   // paged_cache.py:257-259
      // A later sequence writing the same row of block 0 wins (index_put).
      if (id != 0 || !block0_row_taken_later(a.table, a.table_i64, a.table_stride, W,
                                             a.offsets, a.off_i64, bs, a.num_blocks, s,
                                             a.batch, floormod(start, bs), lane)) {
        dec_dst = (((long long)a.layer * a.num_blocks + id) * bs + floormod(start, bs)) *
                  (long long)a.kv_heads * D;
      }
    }
  }

  const int t0 = blockIdx.y * kTokPerCta;
  const int ntok = a.q_len - t0 < kTokPerCta ? a.q_len - t0 : kTokPerCta;
  const int rows = a.num_heads + 2 * a.kv_heads;
  const int groups = (rows + kRowsPerItem - 1) / kRowsPerItem;
  // Work item = (token, group of kRowsPerItem consecutive rows): the token's
  // position, cache row and cos/sin values are loaded once per item, and the
  // item's rows issue all their loads before any of them is rotated.
  for (int item = warp; item < ntok * groups; item += kWarps) {
    const int ti = item / groups;
    const int r0 = (item - ti * groups) * kRowsPerItem;
    const int i = t0 + ti;
    const long long tok = s * a.q_len + i;
    long long pos = load_index(a.positions, a.pos_i64, tok);
    if (pos >= a.max_pos || pos < -a.max_pos) {
      if (lane == 0 && r0 == 0) record_error(a.err, kErrPosition);
      continue;
    }
    if (pos < 0) pos += a.max_pos;
    long long dst = -1;                            // this token's cache row
    if (r0 + kRowsPerItem > a.num_heads) {
      if (decode) {
        dst = dec_dst;
      } else {
        const long long p = start + i;
        const long long c = floordiv(p, bs);
        if (c < stop_col) {
          const long long id =
              load_index(a.table, a.table_i64, s * a.table_stride + (c < 0 ? c + W : c));
          dst = (((long long)a.layer * a.num_blocks + id) * bs + floormod(p, bs)) *
                (long long)a.kv_heads * D;
        }
      }
    }
    if constexpr (M > 0) {
      rotate_rows_paired<IN_DT, KV_DT, M>(a, s, i, tok, pos, dst, r0, rows, lane);
    } else {
      for (int r = r0; r < r0 + kRowsPerItem && r < rows; ++r) {
        if (r >= a.num_heads && dst < 0) continue;
        if (r < a.num_heads) {
          rotate_row<IN_DT, IN_DT>(a, a.q_in, tok * a.q_row + (long long)r * D, a.q_out,
                                   s * a.qo_s + (long long)r * a.qo_h + (long long)i * a.qo_t,
                                   pos, lane);
        } else if (r < a.num_heads + a.kv_heads) {
          const int h = r - a.num_heads;
          rotate_row<IN_DT, KV_DT>(a, a.k_in, tok * a.k_row + (long long)h * D, a.k_cache,
                                   dst + (long long)h * D, pos, lane);
        } else {
          copy_v_row<IN_DT, KV_DT>(a, tok, r - a.num_heads - a.kv_heads, dst, lane);
        }
      }
    }
  }
}

template <int IN_DT, int KV_DT>
const void* rope_ptr(int m) {
  if (m == 1) return reinterpret_cast<const void*>(&rope_append_kernel<IN_DT, KV_DT, 1>);
  if (m == 2) return reinterpret_cast<const void*>(&rope_append_kernel<IN_DT, KV_DT, 2>);
  return reinterpret_cast<const void*>(&rope_append_kernel<IN_DT, KV_DT, 0>);
}

const void* select_rope(int in_dt, int kv_dt, int m) {
#define LLMOPT_ROPE_CASE(I, K) \
  if (in_dt == I && kv_dt == K) return rope_ptr<I, K>(m);
  LLMOPT_ROPE_CASE(kF32, kF32)
  LLMOPT_ROPE_CASE(kF32, kF16)
  LLMOPT_ROPE_CASE(kF32, kBF16)
  LLMOPT_ROPE_CASE(kF16, kF32)
  LLMOPT_ROPE_CASE(kF16, kF16)
  LLMOPT_ROPE_CASE(kF16, kBF16)
  LLMOPT_ROPE_CASE(kBF16, kF32)
  LLMOPT_ROPE_CASE(kBF16, kF16)
  LLMOPT_ROPE_CASE(kBF16, kBF16)
#undef LLMOPT_ROPE_CASE
  return nullptr;
}

}  // namespace

cudaError_t rope_append_launch(const RopeArgs& a, cudaStream_t stream) {
  if (a.batch <= 0 || a.q_len <= 0) return cudaSuccess;
  const int half = a.head_dim / 2;
  const int m = !a.pairs ? 0 : half <= 64 ? 1 : half <= 128 ? 2 : 0;
  const void* fn = select_rope(a.in_dtype, a.kv_dtype, m);
  if (fn == nullptr) return cudaErrorInvalidValue;
  const long long gy = (a.q_len + kTokPerCta - 1) / kTokPerCta;
  if (a.batch > 0x7fffffffLL || gy > 65535) return cudaErrorInvalidConfiguration;
  void* args[] = {const_cast<RopeArgs*>(&a)};
  return launch_pdl(fn, dim3((unsigned)a.batch, (unsigned)gy), dim3(kThreads), args, 0, stream);
}

}  // namespace llmopt
