// KV append (write / write_decode) and the padded gather, bit-exact with the
// reference's PagedKVCache (src/llmopt/cache/paged_cache.py:175-312).
//
// A token row of the cache, [kv_heads, head_dim] at (layer, block, slot), is
// contiguous, so each append is a row copy fused with the cast to the cache
// dtype (round-to-nearest-even, as torch's .to()).  One warp moves one row
// with 16-byte stores when every address allows it.
#include <limits.h>

#include "common.cuh"
#include "kernels.h"

namespace llmopt {
namespace {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int kRowsPerCta = 16;       // gather: positions per CTA
constexpr int kWriteRowsPerCta = 4;   // write: one token row per warp, many CTAs in flight

template <int DT>
struct Vec8 {
  // 8 elements of DT
  using T = typename ElemT<DT>::T;
  T v[8];
};

template <int IN_DT, int OUT_DT>
__device__ __forceinline__ void copy8(const void* src, long long si, void* dst, long long di) {
  float x[8];
  if constexpr (IN_DT == kF32) {
    const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(src) + si);
    const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(src) + si + 4);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
  } else {
    const uint4 raw = *reinterpret_cast<const uint4*>(
        static_cast<const typename ElemT<IN_DT>::T*>(src) + si);
    if constexpr (IN_DT == OUT_DT) {
      *reinterpret_cast<uint4*>(static_cast<typename ElemT<OUT_DT>::T*>(dst) + di) = raw;
      return;
    }
    const typename ElemT<IN_DT>::T* e = reinterpret_cast<const typename ElemT<IN_DT>::T*>(&raw);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if constexpr (IN_DT == kF16) x[k] = __half2float(e[k]);
      else x[k] = __bfloat162float(e[k]);
    }
  }
  if constexpr (OUT_DT == kF32) {
    float* d = static_cast<float*>(dst) + di;
    *reinterpret_cast<float4*>(d) = make_float4(x[0], x[1], x[2], x[3]);
    *reinterpret_cast<float4*>(d + 4) = make_float4(x[4], x[5], x[6], x[7]);
  } else {
    Vec8<OUT_DT> o;
#pragma unroll
    for (int k = 0; k < 8; ++k) o.v[k] = from_f32<OUT_DT>(x[k]);
    *reinterpret_cast<uint4*>(static_cast<typename ElemT<OUT_DT>::T*>(dst) + di) =
        *reinterpret_cast<const uint4*>(&o);
  }
}

template <int IN_DT, int OUT_DT>
__device__ __forceinline__ void copy1(const void* src, long long si, void* dst, long long di) {
  if constexpr (IN_DT == OUT_DT) {
    static_cast<typename ElemT<OUT_DT>::T*>(dst)[di] =
        static_cast<const typename ElemT<IN_DT>::T*>(src)[si];
  } else {
    store_f32<OUT_DT>(dst, di, load_f32<IN_DT>(src, si));
  }
}

// Copy one token row [kv_heads, head_dim] (source head stride `sh`) by one warp.
template <int IN_DT, int OUT_DT>
__device__ __forceinline__ void copy_row(const void* src, long long sbase, long long sh,
                                         void* dst, long long dbase, int kvh, int d, int vec,
                                         int lane) {
  const int n = kvh * d;
  if (vec == 8) {
    for (int e = lane * 8; e < n; e += 32 * 8) {
      const int h = e / d;
      const int k = e - h * d;
      copy8<IN_DT, OUT_DT>(src, sbase + (long long)h * sh + k, dst, dbase + e);
    }
  } else {
    for (int e = lane; e < n; e += 32) {
      const int h = e / d;
      const int k = e - h * d;
      copy1<IN_DT, OUT_DT>(src, sbase + (long long)h * sh + k, dst, dbase + e);
    }
  }
}

// Quantize one token row [kv_heads, head_dim] (head_dim <= 256) to e4m3 by one
// warp: per head, amax over the row (NaN ignored), scale = amax / 448 (1 if
// that is not positive), code = e4m3(x / scale) with both steps rounded to
// nearest.  `scale_idx` is head 0's scale; heads are block_size apart.
template <int IN_DT>
__device__ __forceinline__ void quantize_row(const void* src, long long sbase, long long sh,
                                             uint8_t* dst, long long dbase, float* scales,
                                             long long scale_idx, long long scale_step, int kvh,
                                             int d, int lane) {
  for (int h = 0; h < kvh; ++h) {
    float x[8];
    float amax = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int e = lane + 32 * k;
      x[k] = e < d ? load_f32<IN_DT>(src, sbase + (long long)h * sh + e) : 0.f;
      amax = fmaxf(amax, fabsf(x[k]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = e4m3_row_scale(amax);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int e = lane + 32 * k;
      if (e < d) dst[dbase + (long long)h * d + e] = f32_to_e4m3(__fdiv_rn(x[k], scale));
    }
    if (lane == 0) scales[scale_idx + (long long)h * scale_step] = scale;
  }
}

// Append one token row of K or V: cast copy, or e4m3 quantization with scales.
template <int IN_DT, int OUT_DT>
__device__ __forceinline__ void append_row(const KvWriteArgs& a, const void* src, long long sbase,
                                           long long sh, void* cache, float* scales,
                                           long long id, long long slot, int lane) {
  const long long row_elems = (long long)a.kv_heads * a.head_dim;
  const long long bs = a.block_size;
  const long long blk = (long long)a.layer * a.num_blocks + id;
  if constexpr (OUT_DT == kE4M3) {
    quantize_row<IN_DT>(src, sbase, sh, static_cast<uint8_t*>(cache), (blk * bs + slot) * row_elems,
                        scales, blk * a.kv_heads * bs + slot, bs, a.kv_heads, a.head_dim, lane);
  } else {
    copy_row<IN_DT, OUT_DT>(src, sbase, sh, cache, (blk * bs + slot) * row_elems, a.kv_heads,
                            a.head_dim, a.vec, lane);
  }
}

// write(): grid (batch, ceil(q_len / kWriteRowsPerCta)).
template <int IN_DT, int OUT_DT>
__global__ void __launch_bounds__(kThreads) kv_write_kernel(const KvWriteArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  const long long s = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long bs = a.block_size;
  const long long W = a.table_width;
  const long long start = load_index(a.offsets, a.off_i64, s);
  const long long c0 = floordiv(start, bs);
  const long long c_last = floordiv(start + a.q_len - 1, bs);

  // The walk of _write_one (paged_cache.py:213-232) stops at the first column
  // past the row (normal end), at a -1 entry (normal end), or where torch would
  // raise (column < -W, id >= num_blocks).  key = 4 * (col - c0) + reason.
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
      const long long id = load_index(a.table, a.table_i64, s * a.table_stride + (c < 0 ? c + W : c));
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
  const long long stop_col = key == ULLONG_MAX ? LLONG_MAX : c0 + (long long)(key >> 2);
  if (threadIdx.x == 0 && blockIdx.y == 0 && key != ULLONG_MAX) {
    const unsigned reason = (unsigned)(key & 3);
    if (reason == 1) record_error(a.err, kErrBlockId);
    if (reason == 2) record_error(a.err, kErrTableWidth);
  }

  const int t0 = blockIdx.y * kWriteRowsPerCta;
  const int t1 = t0 + kWriteRowsPerCta < a.q_len ? t0 + kWriteRowsPerCta : a.q_len;
  for (int i = t0 + warp; i < t1; i += kWarps) {
    const long long pos = start + i;
    const long long c = floordiv(pos, bs);
    if (c >= stop_col) continue;
    const long long id = load_index(a.table, a.table_i64, s * a.table_stride + (c < 0 ? c + W : c));
    const long long slot = floormod(pos, bs);
    append_row<IN_DT, OUT_DT>(a, a.keys, s * a.k_s + (long long)i * a.k_t, a.k_h, a.k_cache,
                              a.k_scale, id, slot, lane);
    append_row<IN_DT, OUT_DT>(a, a.values, s * a.v_s + (long long)i * a.v_t, a.v_h, a.v_cache,
                              a.v_scale, id, slot, lane);
  }
}

// write_decode(): one warp pair per sequence (warp 0: K, warp 1: V).
template <int IN_DT, int OUT_DT>
__global__ void __launch_bounds__(64) kv_write_decode_kernel(const KvWriteArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  const long long s = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long bs = a.block_size;
  const long long W = a.table_width;
  const long long off = load_index(a.offsets, a.off_i64, s);
  const long long col = floordiv(off, bs);          // paged_cache.py:252
  if (col < -W || col >= W) {                       // torch would raise IndexError
    if (threadIdx.x == 0) record_error(a.err, kErrTableWidth);
    return;
  }
  long long id = load_index(a.table, a.table_i64, s * a.table_stride + (col < 0 ? col + W : col));
  if (id < 0 || id >= a.num_blocks) id = 0;         // paged_cache.py:257-259
  const long long slot = floormod(off, bs);         // paged_cache.py:253
  if (id == 0 && block0_row_taken_later(a.table, a.table_i64, a.table_stride, W, a.offsets,
                                        a.off_i64, bs, a.num_blocks, s, a.batch, slot, lane)) {
    return;                                         // a later sequence's row wins
  }
  if (warp == 0) {
    append_row<IN_DT, OUT_DT>(a, a.keys, s * a.k_s, a.k_h, a.k_cache, a.k_scale, id, slot, lane);
  } else {
    append_row<IN_DT, OUT_DT>(a, a.values, s * a.v_s, a.v_h, a.v_cache, a.v_scale, id, slot,
                              lane);
  }
}

// gather(): grid (batch, ceil(max_len / kRowsPerCta)); one warp per position.
template <int DT>
__global__ void __launch_bounds__(kThreads) gather_kernel(const GatherArgs a, int vec) {
  griddep_wait();
  griddep_launch_dependents();
  const long long s = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long bs = a.block_size;
  const long long ctx_s = load_index(a.ctx, a.ctx_i64, s);
  const long long row_elems = (long long)a.kv_heads * a.head_dim;
  const long long t0 = (long long)blockIdx.y * kRowsPerCta;
  const long long t1 = t0 + kRowsPerCta < a.max_len ? t0 + kRowsPerCta : a.max_len;
  for (long long t = t0 + warp; t < t1; t += kWarps) {
    const long long col = t / bs;                   // paged_cache.py:289 (< width, host-checked)
    const long long id = load_index(a.table, a.table_i64, s * a.table_stride + col);
    bool ok = id >= 0 && t < ctx_s;                 // paged_cache.py:293-295
    if (id >= a.num_blocks) {
      if (lane == 0) record_error(a.err, kErrBlockId);
      ok = false;
    }
    const long long dst = (s * a.max_len + t) * row_elems;
    const long long src = ok ? (((long long)a.layer * a.num_blocks + id) * bs + (t - col * bs)) * row_elems : 0;
    if (lane == 0) a.valid[s * a.max_len + t] = ok ? 1 : 0;
    using T = typename ElemT<DT>::T;
    const T* kc = static_cast<const T*>(a.k_cache);
    const T* vc = static_cast<const T*>(a.v_cache);
    T* ok_ = static_cast<T*>(a.out_k);
    T* ov = static_cast<T*>(a.out_v);
    const int per = 16 / (int)sizeof(T);
    if (vec) {
      for (long long e = (long long)lane * per; e < row_elems; e += 32LL * per) {
        uint4 kx = make_uint4(0u, 0u, 0u, 0u), vx = kx;
        if (ok) {
          kx = *reinterpret_cast<const uint4*>(kc + src + e);
          vx = *reinterpret_cast<const uint4*>(vc + src + e);
        }
        *reinterpret_cast<uint4*>(ok_ + dst + e) = kx;
        *reinterpret_cast<uint4*>(ov + dst + e) = vx;
      }
    } else {
      for (long long e = lane; e < row_elems; e += 32) {
        T kx = T(0.f), vx = T(0.f);
        if (ok) {
          kx = kc[src + e];
          vx = vc[src + e];
        }
        ok_[dst + e] = kx;
        ov[dst + e] = vx;
      }
    }
  }
}

// gather() of an e4m3 cache: the padded rows come out dequantised to fp32
// (code value * row scale, one rounding), zero where invalid.
__global__ void __launch_bounds__(kThreads) gather_e4m3_kernel(const GatherArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  const long long s = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long bs = a.block_size;
  const long long ctx_s = load_index(a.ctx, a.ctx_i64, s);
  const long long row_elems = (long long)a.kv_heads * a.head_dim;
  const long long t0 = (long long)blockIdx.y * kRowsPerCta;
  const long long t1 = t0 + kRowsPerCta < a.max_len ? t0 + kRowsPerCta : a.max_len;
  const uint8_t* kc = static_cast<const uint8_t*>(a.k_cache);
  const uint8_t* vc = static_cast<const uint8_t*>(a.v_cache);
  float* ok_ = static_cast<float*>(a.out_k);
  float* ov = static_cast<float*>(a.out_v);
  for (long long t = t0 + warp; t < t1; t += kWarps) {
    const long long col = t / bs;                   // paged_cache.py:289 (< width, host-checked)
    const long long id = load_index(a.table, a.table_i64, s * a.table_stride + col);
    bool ok = id >= 0 && t < ctx_s;                 // paged_cache.py:293-295
    if (id >= a.num_blocks) {
      if (lane == 0) record_error(a.err, kErrBlockId);
      ok = false;
    }
    const long long slot = t - col * bs;
    const long long blk = ok ? (long long)a.layer * a.num_blocks + id : 0;
    const long long src = (blk * bs + slot) * row_elems;
    const long long dst = (s * a.max_len + t) * row_elems;
    if (lane == 0) a.valid[s * a.max_len + t] = ok ? 1 : 0;
    for (long long e = lane; e < row_elems; e += 32) {
      float kx = 0.f, vx = 0.f;
      if (ok) {
        const long long sidx = (blk * a.kv_heads + e / a.head_dim) * bs + slot;
        kx = e4m3_to_f32(kc[src + e]) * a.k_scale[sidx];
        vx = e4m3_to_f32(vc[src + e]) * a.v_scale[sidx];
      }
      ok_[dst + e] = kx;
      ov[dst + e] = vx;
    }
  }
}

template <int IN_DT, int OUT_DT>
const void* write_ptr(bool decode) {
  return decode ? reinterpret_cast<const void*>(&kv_write_decode_kernel<IN_DT, OUT_DT>)
                : reinterpret_cast<const void*>(&kv_write_kernel<IN_DT, OUT_DT>);
}

const void* select_write(int in_dt, int out_dt, bool decode) {
#define LLMOPT_WRITE_CASE(I, O) \
  if (in_dt == I && out_dt == O) return write_ptr<I, O>(decode);
  LLMOPT_WRITE_CASE(kF32, kF32)
  LLMOPT_WRITE_CASE(kF32, kF16)
  LLMOPT_WRITE_CASE(kF32, kBF16)
  LLMOPT_WRITE_CASE(kF16, kF32)
  LLMOPT_WRITE_CASE(kF16, kF16)
  LLMOPT_WRITE_CASE(kF16, kBF16)
  LLMOPT_WRITE_CASE(kBF16, kF32)
  LLMOPT_WRITE_CASE(kBF16, kF16)
  LLMOPT_WRITE_CASE(kBF16, kBF16)
  LLMOPT_WRITE_CASE(kF32, kE4M3)
  LLMOPT_WRITE_CASE(kF16, kE4M3)
  LLMOPT_WRITE_CASE(kBF16, kE4M3)
#undef LLMOPT_WRITE_CASE
  return nullptr;
}

}  // namespace

cudaError_t kv_write_launch(const KvWriteArgs& a, cudaStream_t stream) {
  if (a.batch <= 0 || a.q_len <= 0) return cudaSuccess;
  const void* fn = select_write(a.in_dtype, a.kv_dtype, false);
  if (fn == nullptr) return cudaErrorInvalidValue;
  const long long gy = (a.q_len + kWriteRowsPerCta - 1) / kWriteRowsPerCta;
  if (a.batch > 0x7fffffffLL || gy > 65535) return cudaErrorInvalidConfiguration;
  void* args[] = {const_cast<KvWriteArgs*>(&a)};
  return launch_pdl(fn, dim3((unsigned)a.batch, (unsigned)gy), dim3(kThreads), args, 0,
                          stream);
}

cudaError_t kv_write_decode_launch(const KvWriteArgs& a, cudaStream_t stream) {
  if (a.batch <= 0) return cudaSuccess;
  const void* fn = select_write(a.in_dtype, a.kv_dtype, true);
  if (fn == nullptr) return cudaErrorInvalidValue;
  if (a.batch > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  void* args[] = {const_cast<KvWriteArgs*>(&a)};
  return launch_pdl(fn, dim3((unsigned)a.batch), dim3(64), args, 0, stream);
}

cudaError_t gather_launch(const GatherArgs& a, cudaStream_t stream) {
  if (a.batch <= 0 || a.max_len <= 0) return cudaSuccess;
  const long long gy = (a.max_len + kRowsPerCta - 1) / kRowsPerCta;
  if (a.batch > 0x7fffffffLL || gy > 65535) return cudaErrorInvalidConfiguration;
  if (a.kv_dtype == kE4M3) {
    void* args[] = {const_cast<GatherArgs*>(&a)};
    return launch_pdl(reinterpret_cast<const void*>(&gather_e4m3_kernel),
                      dim3((unsigned)a.batch, (unsigned)gy), dim3(kThreads), args, 0, stream);
  }
  const int esize = a.kv_dtype == kF32 ? 4 : 2;
  const long long row_bytes = (long long)a.kv_heads * a.head_dim * esize;
  int vec = (row_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(a.k_cache) & 15) == 0 &&
             (reinterpret_cast<uintptr_t>(a.v_cache) & 15) == 0 &&
             (reinterpret_cast<uintptr_t>(a.out_k) & 15) == 0 &&
             (reinterpret_cast<uintptr_t>(a.out_v) & 15) == 0)
                ? 1
                : 0;
  const void* fn = nullptr;
  switch (a.kv_dtype) {
    case kF32: fn = reinterpret_cast<const void*>(&gather_kernel<kF32>); break;
    case kF16: fn = reinterpret_cast<const void*>(&gather_kernel<kF16>); break;
    case kBF16: fn = reinterpret_cast<const void*>(&gather_kernel<kBF16>); break;
    default: return cudaErrorInvalidValue;
  }
  void* args[] = {const_cast<GatherArgs*>(&a), &vec};
  return launch_pdl(fn, dim3((unsigned)a.batch, (unsigned)gy), dim3(kThreads), args, 0,
                          stream);
}

}  // namespace llmopt
