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
constexpr int kTokPerCta = 4;

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

template <int IN_DT, int KV_DT>
__global__ void __launch_bounds__(kThreads) rope_append_kernel(const RopeArgs a) {
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
      dec_dst = (((long long)a.layer * a.num_blocks + id) * bs + floormod(start, bs)) *
                (long long)a.kv_heads * D;
    }
  }

  const int t0 = blockIdx.y * kTokPerCta;
  const int ntok = a.q_len - t0 < kTokPerCta ? a.q_len - t0 : kTokPerCta;
  const int rows = a.num_heads + 2 * a.kv_heads;
  for (int item = warp; item < ntok * rows; item += kWarps) {
    const int ti = item / rows;
    const int r = item - ti * rows;
    const int i = t0 + ti;
    const long long tok = s * a.q_len + i;
    long long pos = load_index(a.positions, a.pos_i64, tok);
    if (pos >= a.max_pos || pos < -a.max_pos) {
      if (lane == 0 && r == 0) record_error(a.err, kErrPosition);
      continue;
    }
    if (pos < 0) pos += a.max_pos;
    long long dst = -1;                            // cache row of this token
    if (r >= a.num_heads) {
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
      if (dst < 0) continue;
    }
    if (r < a.num_heads) {
      // q head r -> q_out[s, r, i, :]
      const long long src = tok * a.q_row + (long long)r * D;
      const long long out = s * a.qo_s + (long long)r * a.qo_h + (long long)i * a.qo_t;
      for (int e = lane; e < half; e += 32) {
        const float c1 = op_round<IN_DT>(load_any(a.cos_t, a.tab_dtype, pos * D + e));
        const float c2 = op_round<IN_DT>(load_any(a.cos_t, a.tab_dtype, pos * D + e + half));
        const float s1 = op_round<IN_DT>(load_any(a.sin_t, a.tab_dtype, pos * D + e));
        const float s2 = op_round<IN_DT>(load_any(a.sin_t, a.tab_dtype, pos * D + e + half));
        float o1, o2;
        rotate_pair<IN_DT>(load_f32<IN_DT>(a.q_in, src + e), load_f32<IN_DT>(a.q_in, src + e + half),
                           c1, c2, s1, s2, &o1, &o2);
        store_f32<IN_DT>(a.q_out, out + e, o1);
        store_f32<IN_DT>(a.q_out, out + e + half, o2);
      }
    } else if (r < a.num_heads + a.kv_heads) {
      // k head -> cache: rotated in the model dtype, then cast to the cache dtype
      const int h = r - a.num_heads;
      const long long src = tok * a.k_row + (long long)h * D;
      const long long out = dst + (long long)h * D;
      for (int e = lane; e < half; e += 32) {
        const float c1 = op_round<IN_DT>(load_any(a.cos_t, a.tab_dtype, pos * D + e));
        const float c2 = op_round<IN_DT>(load_any(a.cos_t, a.tab_dtype, pos * D + e + half));
        const float s1 = op_round<IN_DT>(load_any(a.sin_t, a.tab_dtype, pos * D + e));
        const float s2 = op_round<IN_DT>(load_any(a.sin_t, a.tab_dtype, pos * D + e + half));
        float o1, o2;
        rotate_pair<IN_DT>(load_f32<IN_DT>(a.k_in, src + e), load_f32<IN_DT>(a.k_in, src + e + half),
                           c1, c2, s1, s2, &o1, &o2);
        store_f32<KV_DT>(a.k_cache, out + e, o1);
        store_f32<KV_DT>(a.k_cache, out + e + half, o2);
      }
    } else {
      // v head -> cache, cast only
      const int h = r - a.num_heads - a.kv_heads;
      const long long src = tok * a.v_row + (long long)h * D;
      const long long out = dst + (long long)h * D;
      for (int e = lane; e < D; e += 32) {
        store_f32<KV_DT>(a.v_cache, out + e, load_f32<IN_DT>(a.v_in, src + e));
      }
    }
  }
}

template <int IN_DT, int KV_DT>
const void* rope_ptr() {
  return reinterpret_cast<const void*>(&rope_append_kernel<IN_DT, KV_DT>);
}

const void* select_rope(int in_dt, int kv_dt) {
#define LLMOPT_ROPE_CASE(I, K) \
  if (in_dt == I && kv_dt == K) return rope_ptr<I, K>();
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
  const void* fn = select_rope(a.in_dtype, a.kv_dtype);
  if (fn == nullptr) return cudaErrorInvalidValue;
  const long long gy = (a.q_len + kTokPerCta - 1) / kTokPerCta;
  if (a.batch > 0x7fffffffLL || gy > 65535) return cudaErrorInvalidConfiguration;
  void* args[] = {const_cast<RopeArgs*>(&a)};
  return launch_pdl(fn, dim3((unsigned)a.batch, (unsigned)gy), dim3(kThreads), args, 0, stream);
}

}  // namespace llmopt
