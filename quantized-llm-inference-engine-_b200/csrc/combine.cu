// Split-K combine and merge_states.
//
// combine_kernel folds the split partials of each (sequence, head, query row)
// with the exact log-sum-exp rule of merge_states
// (src/llmopt/attention/paged_attention.py:30-55), done in one pass over all
// partials instead of the reference's sequential pairwise chain (:287-290):
//   lse = M + log(sum_p exp(lse_p - M)),  out = sum_p exp(lse_p - lse) * out_p
// with M = max_p lse_p.  A row whose partials are all -inf (every key masked)
// gets out = 0 and lse = -inf, which is what the reference's nan_to_num
// produces (:291-293).  One warp per output row; lanes own head_dim slices.
#include <float.h>

#include "common.cuh"
#include "kernels.h"

namespace llmopt {
namespace {

constexpr int kWarpsPerCta = 4;
constexpr int kMaxDimPerLane = 8;  // head_dim <= 256

struct SlotRange {
  long long first;   // fixed: first slot; balanced: first CTA
  long long count;   // fixed: number of slots; balanced: CTAs to scan
  long long p_lo, p_hi, total;  // balanced: the sequence's block range and T
};

__device__ __forceinline__ bool balanced_touch(long long c, const SlotRange& r, long long ctas) {
  const long long a0 = range_start(c, r.total, ctas);
  const long long a1 = range_start(c + 1, r.total, ctas);
  const long long lo = a0 > r.p_lo ? a0 : r.p_lo;
  const long long hi = a1 < r.p_hi ? a1 : r.p_hi;
  return lo < hi;
}

// One warp per output row.  Lanes first evaluate the row's partials in
// parallel (validity, LSE, max, weight), then every lane accumulates its VEC
// contiguous dims of the row from each partial in turn - loads that do not
// depend on each other, so many stay in flight even when a long sequence has
// dozens of partials.  VEC == 0 is the scalar path for head_dim % 32 != 0.
// Merges one output row; `emit(d0, vals, n)` stores n consecutive dims from d0.
template <int VEC, class Emit>
__device__ __forceinline__ void combine_row(const AttnArgs& a, long long row, int lane,
                                            Emit&& emit);

template <int O_DT, int VEC>
__global__ void __launch_bounds__(kWarpsPerCta * 32) combine_kernel(const AttnArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * kWarpsPerCta + warp;
  const long long nrows = a.batch * a.num_heads * (long long)a.q_len;
  if (row >= nrows) return;
  const int qi = (int)(row % a.q_len);
  const long long sh = row / a.q_len;
  const int h = (int)(sh % a.num_heads);
  const long long s = sh / a.num_heads;
  const long long obase = s * a.o_s + (long long)h * a.o_h + (long long)qi * a.o_t;
  combine_row<VEC>(a, row, lane, [&](int d0, const float* v, int n) {
    for (int k = 0; k < n; ++k) store_f32<O_DT>(a.out, obase + d0 + k, v[k]);
  });
}

// Arrival of one CTA at the cross-rank barrier that closes a gathered call.
// The CTA's stores (local and over NVLink) are ordered before its arrival by
// the barrier plus thread 0's system-scope fence (fences are cumulative).  The
// last CTA of this rank then writes `epoch` into its slot of every rank's
// flags (release: a fence, then relaxed stores) and polls its own flags until
// every rank's slot has reached `epoch` (then an acquire fence): after that
// every rank's rows are in this rank's gathered output.  The wait gives up
// after kWaitLimitCycles and records kErrWaitTimeout instead of hanging.
__device__ __forceinline__ void peer_barrier(const PeerArgs& p, unsigned* err) {
  __syncthreads();
  if (threadIdx.x != 0) return;
  __threadfence_system();
  const unsigned arrived = atomicAdd(p.counter, 1u);
  if (arrived != gridDim.x - 1) return;
  // One release fence covers every flag store after it (fence + relaxed
  // stores is a release pattern), so the stores to the peers are issued back
  // to back instead of each waiting for the previous one to be acknowledged.
  __threadfence_system();
  for (int r = 0; r < p.world; ++r) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p.flags[r] + p.rank), "r"(p.epoch)
                 : "memory");
  }
  const unsigned* mine = p.flags[p.rank];
  const long long t0 = clock64();
  bool timed_out = false;
  for (int r = 0; r < p.world && !timed_out; ++r) {
    while (true) {
      unsigned v;
      asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine + r) : "memory");
      if ((int)(v - p.epoch) >= 0) break;
      if (clock64() - t0 > kWaitLimitCycles) {
        record_error(err, kErrWaitTimeout | kErrWaitPeer);
        timed_out = true;
        break;
      }
    }
  }
  // Acquire side of the pattern: the peers' rows are visible to this grid's
  // completion (and so to every later kernel on the stream) after this fence.
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  *p.counter = 0u;
}

// n (1, 2, 4 or 8) consecutive output values as one store where the width allows.
template <int O_DT>
__device__ __forceinline__ void store_run(void* base, long long idx, const float* v, int n) {
  if constexpr (O_DT == kF32) {
    float* dst = static_cast<float*>(base) + idx;
    if (n == 4) {
      *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
      return;
    }
    if (n == 8) {
      reinterpret_cast<float4*>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
      reinterpret_cast<float4*>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
      return;
    }
  } else {
    unsigned short* dst = static_cast<unsigned short*>(base) + idx;
    if (n == 2 || n == 4 || n == 8) {
      unsigned w[4];
      for (int k = 0; k < n / 2; ++k) w[k] = pack2<O_DT>(v[2 * k], v[2 * k + 1]);
      if (n == 2) *reinterpret_cast<unsigned*>(dst) = w[0];
      if (n == 4) *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
      if (n == 8) *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
      return;
    }
  }
  for (int k = 0; k < n; ++k) store_f32<O_DT>(base, idx + k, v[k]);
}

// Combine + all-gather: each merged row goes to every rank's gathered output
// at head rank * num_heads + h ([H_total, batch, q_len, head_dim]), then the
// peer barrier, so when the kernel ends this rank's gathered output is whole.
template <int O_DT, int VEC>
__global__ void __launch_bounds__(kWarpsPerCta * 32)
    combine_gather_kernel(const AttnArgs a, const PeerArgs p) {
  griddep_wait();
  griddep_launch_dependents();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * kWarpsPerCta + warp;
  const long long nrows = a.batch * a.num_heads * (long long)a.q_len;
  if (row < nrows) {
    const int qi = (int)(row % a.q_len);
    const long long sh = row / a.q_len;
    const int h = (int)(sh % a.num_heads);
    const long long s = sh / a.num_heads;
    const long long gh = (long long)p.rank * a.num_heads + h;
    const long long gbase = ((gh * a.batch + s) * a.q_len + qi) * (long long)a.head_dim;
    combine_row<VEC>(a, row, lane, [&](int d0, const float* v, int n) {
      for (int r = 0; r < p.world; ++r) store_run<O_DT>(p.out[r], gbase + d0, v, n);
    });
  }
  peer_barrier(p, a.err);
}

// This rank's contiguous slice of its gathered output, copied to every peer
// at the same offset in units of T (uint4 when the slice allows, else 2 bytes).
template <class T>
__global__ void __launch_bounds__(256) push_gather_kernel(const AttnArgs a, const PeerArgs p,
                                                          long long off_units,
                                                          long long n_units) {
  griddep_wait();
  griddep_launch_dependents();
  const T* src = static_cast<const T*>(p.out[p.rank]) + off_units;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n_units;
       i += (long long)gridDim.x * blockDim.x) {
    const T v = src[i];
    for (int r = 0; r < p.world; ++r) {
      if (r != p.rank) static_cast<T*>(p.out[r])[off_units + i] = v;
    }
  }
  peer_barrier(p, a.err);
}

template <int VEC, class Emit>
__device__ __forceinline__ void combine_row(const AttnArgs& a, long long row, int lane,
                                            Emit&& emit) {
  const int qi = (int)(row % a.q_len);
  const long long sh = row / a.q_len;
  const int h = (int)(sh % a.num_heads);
  const long long s = sh / a.num_heads;
  const int D = a.head_dim;

  SlotRange r{0, 0, 0, 0, 0};
  const bool balanced = a.plan.mode == kModeBalanced;
  if (balanced) {
    r.p_lo = a.prefix[s];
    r.p_hi = a.prefix[s + 1];
    r.total = a.prefix[a.batch];
    if (r.p_hi > r.p_lo) {
      r.first = range_owner(r.p_lo, r.total, a.plan.ctas);
      r.count = range_owner(r.p_hi - 1, r.total, a.plan.ctas) - r.first + 1;
    }
  } else {
    const long long ctx_s = load_index(a.ctx, a.ctx_i64, s);
    const long long nb = blocks_of(ctx_s, a.block_size, a.table_width);
    long long cnt = (nb + a.plan.split_blocks - 1) / a.plan.split_blocks;
    if (cnt > a.plan.splits) cnt = a.plan.splits;
    r.first = s * a.plan.splits;
    r.count = cnt;
  }
  // Partial i of this row: its row index in the workspace, or -1 if that CTA
  // did not touch the sequence (balanced plan) or saw only masked keys.
  auto partial_row = [&](long long i, float* lse) -> long long {
    if (i >= r.count) return -1;
    if (balanced && !balanced_touch(r.first + i, r, a.plan.ctas)) return -1;
    const long long slot = balanced ? s + (r.first + i) : r.first + i;
    const long long prow = (slot * a.num_heads + h) * a.q_len + qi;
    *lse = a.part_lse[prow];
    return *lse == -INFINITY ? -1 : prow;
  };

  float mx = -INFINITY;
  for (long long i = lane; i < r.count; i += 32) {
    float l;
    if (partial_row(i, &l) >= 0) mx = fmaxf(mx, l);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));

  constexpr int kAcc = VEC > 0 ? VEC : kMaxDimPerLane;
  float acc[kAcc];
#pragma unroll
  for (int k = 0; k < kAcc; ++k) acc[k] = 0.f;
  float wsum = 0.f;
  if (mx != -INFINITY) {
    for (long long base = 0; base < r.count; base += 32) {
      float l = -INFINITY, w = 0.f;
      long long prow = partial_row(base + lane, &l);
      if (prow >= 0) w = expf(l - mx);
      wsum += w;
      const int n = r.count - base < 32 ? (int)(r.count - base) : 32;
#pragma unroll 4
      for (int k = 0; k < n; ++k) {
        const float wk = __shfl_sync(0xffffffffu, w, k);
        const long long pk = __shfl_sync(0xffffffffu, prow, k);
        if (wk == 0.f) continue;  // warp-uniform
        const float* src = a.part_o + pk * D;
        if constexpr (VEC == 4) {
          const float4 v = *reinterpret_cast<const float4*>(src + lane * 4);
          acc[0] = fmaf(wk, v.x, acc[0]);
          acc[1] = fmaf(wk, v.y, acc[1]);
          acc[2] = fmaf(wk, v.z, acc[2]);
          acc[3] = fmaf(wk, v.w, acc[3]);
        } else if constexpr (VEC == 2) {
          const float2 v = *reinterpret_cast<const float2*>(src + lane * 2);
          acc[0] = fmaf(wk, v.x, acc[0]);
          acc[1] = fmaf(wk, v.y, acc[1]);
        } else if constexpr (VEC == 8) {
          const float4 v0 = *reinterpret_cast<const float4*>(src + lane * 8);
          const float4 v1 = *reinterpret_cast<const float4*>(src + lane * 8 + 4);
          acc[0] = fmaf(wk, v0.x, acc[0]);
          acc[1] = fmaf(wk, v0.y, acc[1]);
          acc[2] = fmaf(wk, v0.z, acc[2]);
          acc[3] = fmaf(wk, v0.w, acc[3]);
          acc[4] = fmaf(wk, v1.x, acc[4]);
          acc[5] = fmaf(wk, v1.y, acc[5]);
          acc[6] = fmaf(wk, v1.z, acc[6]);
          acc[7] = fmaf(wk, v1.w, acc[7]);
        } else if constexpr (VEC == 1) {
          acc[0] = fmaf(wk, src[lane], acc[0]);
        } else {
#pragma unroll
          for (int kk = 0; kk < kMaxDimPerLane; ++kk) {
            const int d = lane + 32 * kk;
            if (d < D) acc[kk] = fmaf(wk, src[d], acc[kk]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  if constexpr (VEC > 0) {
    float v[VEC];
#pragma unroll
    for (int k = 0; k < VEC; ++k) v[k] = acc[k] * inv;
    emit(lane * VEC, v, VEC);
  } else {
#pragma unroll
    for (int kk = 0; kk < kMaxDimPerLane; ++kk) {
      const int d = lane + 32 * kk;
      if (d < D) {
        const float v = acc[kk] * inv;
        emit(d, &v, 1);
      }
    }
  }
  if (a.lse != nullptr && lane == 0) {
    a.lse[row] = wsum > 0.f ? mx + logf(wsum) : -INFINITY;
  }
}

// torch.logaddexp semantics: equal infinities return themselves, otherwise
// max + log1p(exp(-|a - b|)) (NaN propagates).
__device__ __forceinline__ float logaddexp_f(float x, float y) {
  const float m = fmaxf(x, y);
  if (isinf(m) && x == y) return m;
  if (isnan(x) || isnan(y)) return x + y;
  return m + log1pf(expf(-fabsf(x - y)));
}

template <int O_DT, int L_DT>
__global__ void merge_states_kernel(const void* o1, const void* o2, const void* l1,
                                    const void* l2, void* out, void* lse_out, long long rows,
                                    int head_dim) {
  griddep_wait();
  griddep_launch_dependents();
  const long long n = rows * head_dim;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / head_dim;
    const float a1 = load_f32<L_DT>(l1, r);
    const float a2 = load_f32<L_DT>(l2, r);
    const float m = logaddexp_f(a1, a2);
    const float w1 = expf(a1 - m);
    const float w2 = expf(a2 - m);
    store_f32<O_DT>(out, i, load_f32<O_DT>(o1, i) * w1 + load_f32<O_DT>(o2, i) * w2);
    if (i - r * head_dim == 0 && lse_out != nullptr) store_f32<L_DT>(lse_out, r, m);
  }
}

template <int O_DT, int L_DT>
const void* merge_ptr() {
  return reinterpret_cast<const void*>(&merge_states_kernel<O_DT, L_DT>);
}

}  // namespace

cudaError_t combine_launch(const AttnArgs& a, cudaStream_t stream) {
  const long long nrows = a.batch * a.num_heads * (long long)a.q_len;
  if (nrows <= 0) return cudaSuccess;
  const long long grid = (nrows + kWarpsPerCta - 1) / kWarpsPerCta;
  if (grid > 0x7fffffffLL || a.head_dim > 32 * kMaxDimPerLane) return cudaErrorInvalidValue;
  const int vec = (a.head_dim % 32 == 0 && a.head_dim <= 256) ? a.head_dim / 32 : 0;
  const void* fn = nullptr;
#define LLMOPT_COMBINE_CASE(DT)                                                   \
  if (a.out_dtype == DT) {                                                        \
    switch (vec) {                                                                \
      case 1: fn = reinterpret_cast<const void*>(&combine_kernel<DT, 1>); break;  \
      case 2: fn = reinterpret_cast<const void*>(&combine_kernel<DT, 2>); break;  \
      case 4: fn = reinterpret_cast<const void*>(&combine_kernel<DT, 4>); break;  \
      case 8: fn = reinterpret_cast<const void*>(&combine_kernel<DT, 8>); break;  \
      default: fn = reinterpret_cast<const void*>(&combine_kernel<DT, 0>); break; \
    }                                                                             \
  }
  LLMOPT_COMBINE_CASE(kF32)
  LLMOPT_COMBINE_CASE(kF16)
  LLMOPT_COMBINE_CASE(kBF16)
#undef LLMOPT_COMBINE_CASE
  if (fn == nullptr) return cudaErrorInvalidValue;
  void* args[] = {const_cast<AttnArgs*>(&a)};
  return launch_pdl(fn, dim3((unsigned)grid), dim3(kWarpsPerCta * 32), args, 0, stream);
}

cudaError_t combine_gather_launch(const AttnArgs& a, const PeerArgs& p, cudaStream_t stream) {
  const long long nrows = a.batch * a.num_heads * (long long)a.q_len;
  if (nrows <= 0) return cudaSuccess;
  const long long grid = (nrows + kWarpsPerCta - 1) / kWarpsPerCta;
  if (grid > 0x7fffffffLL || a.head_dim > 32 * kMaxDimPerLane) return cudaErrorInvalidValue;
  const int vec = (a.head_dim % 32 == 0 && a.head_dim <= 256) ? a.head_dim / 32 : 0;
  const void* fn = nullptr;
#define LLMOPT_GATHER_CASE(DT)                                                           \
  if (a.out_dtype == DT) {                                                               \
    switch (vec) {                                                                       \
      case 1: fn = reinterpret_cast<const void*>(&combine_gather_kernel<DT, 1>); break;  \
      case 2: fn = reinterpret_cast<const void*>(&combine_gather_kernel<DT, 2>); break;  \
      case 4: fn = reinterpret_cast<const void*>(&combine_gather_kernel<DT, 4>); break;  \
      case 8: fn = reinterpret_cast<const void*>(&combine_gather_kernel<DT, 8>); break;  \
      default: fn = reinterpret_cast<const void*>(&combine_gather_kernel<DT, 0>); break; \
    }                                                                                    \
  }
  LLMOPT_GATHER_CASE(kF32)
  LLMOPT_GATHER_CASE(kF16)
  LLMOPT_GATHER_CASE(kBF16)
#undef LLMOPT_GATHER_CASE
  if (fn == nullptr) return cudaErrorInvalidValue;
  void* args[] = {const_cast<AttnArgs*>(&a), const_cast<PeerArgs*>(&p)};
  return launch_pdl(fn, dim3((unsigned)grid), dim3(kWarpsPerCta * 32), args, 0, stream);
}

cudaError_t push_gather_launch(const AttnArgs& a, const PeerArgs& p, int elem_bytes,
                               cudaStream_t stream) {
  const long long slice = a.batch * a.num_heads * (long long)a.q_len * a.head_dim * elem_bytes;
  const long long off = (long long)p.rank * slice;
  const bool wide = slice % 16 == 0 && off % 16 == 0;
  const int unit = wide ? 16 : 2;
  const long long n_units = slice / unit;
  long long grid = (n_units + 255) / 256;
  if (grid > 4096) grid = 4096;
  if (grid < 1) grid = 1;
  long long off_units = off / unit;
  void* args[] = {const_cast<AttnArgs*>(&a), const_cast<PeerArgs*>(&p), &off_units, const_cast<long long*>(&n_units)};
  const void* fn = wide ? reinterpret_cast<const void*>(&push_gather_kernel<uint4>)
                        : reinterpret_cast<const void*>(&push_gather_kernel<unsigned short>);
  return launch_pdl(fn, dim3((unsigned)grid), dim3(256), args, 0, stream);
}

cudaError_t merge_states_launch(const void* o1, const void* o2, const void* l1, const void* l2,
                                void* out, void* lse_out, long long rows, int head_dim,
                                int o_dtype, int lse_dtype, cudaStream_t stream) {
  const long long n = rows * head_dim;
  if (n <= 0) return cudaSuccess;
  const void* fn = nullptr;
#define LLMOPT_MERGE_CASE(OT, LT) \
  if (o_dtype == OT && lse_dtype == LT) fn = merge_ptr<OT, LT>();
  LLMOPT_MERGE_CASE(kF32, kF32)
  LLMOPT_MERGE_CASE(kF16, kF32)
  LLMOPT_MERGE_CASE(kBF16, kF32)
  LLMOPT_MERGE_CASE(kF16, kF16)
  LLMOPT_MERGE_CASE(kBF16, kBF16)
  LLMOPT_MERGE_CASE(kF32, kF16)
  LLMOPT_MERGE_CASE(kF32, kBF16)
#undef LLMOPT_MERGE_CASE
  if (fn == nullptr) return cudaErrorInvalidValue;
  long long blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  void* args[] = {const_cast<void**>(&o1), const_cast<void**>(&o2), const_cast<void**>(&l1),
                  const_cast<void**>(&l2), &out, &lse_out, &rows, &head_dim};
  return launch_pdl(fn, dim3((unsigned)blocks), dim3(256), args, 0, stream);
}

}  // namespace llmopt
