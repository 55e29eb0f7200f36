// Paged attention, general path (CUDA cores, fp32 arithmetic).
//
// Covers every shape the tensor-core paths do not: fp32 caches (where the
// 1e-5 relative bar rules out 16-bit operands), head_dim up to 256 of any
// size, any block_size, any group size and q_len (chunked prefill included).
// Semantics are those of PagedAttention.forward
// (src/llmopt/attention/paged_attention.py:146-293): positions whose table
// entry is -1 are masked (paged_cache.py:293-295), query row i of a sequence
// sits at context - q_len + i and sees keys at or before it (:212-229), the
// query is rounded to the cache dtype first (:242), and a fully masked row
// yields 0 (:249, :293).
//
// Grid: x = (sequence, split) of the fixed split plan, y = KV head,
// z = tile of 16 query rows (the group's heads x q_len).  Each CTA walks its
// split's keys in tiles of 32 tokens through shared memory, keeps an online
// softmax per row, and writes a normalised partial + LSE for combine.cu.
//
// e4m3 caches: a K/V element is its code's value times the row's fp32 scale
// (one float product, as the gather's dequantisation), and the query is
// rounded to f16, the operand precision of the fp8 tensor-core decode.
#include <float.h>

#include "common.cuh"
#include "kernels.h"

namespace llmopt {
namespace {

constexpr int kThreads = 128;
constexpr int RT = kGenericRowTile;
constexpr int KT = kGenericKeyTile;

size_t generic_smem(int d) {
  return sizeof(float) * ((size_t)RT * d + (size_t)KT * (d + 1) + (size_t)KT * d +
                          (size_t)RT * (KT + 1) + (size_t)RT * d + 3 * RT) +
         2 * sizeof(long long) * KT + 16;
}

template <int KV_DT, int Q_DT>
__global__ void __launch_bounds__(kThreads) attn_generic_kernel(const AttnArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  const int D = a.head_dim;
  const int tid = threadIdx.x;
  extern __shared__ float sm[];
  float* Qs = sm;                       // [RT][D]
  float* Ks = Qs + RT * D;              // [KT][D+1]
  float* Vs = Ks + KT * (D + 1);        // [KT][D]
  float* S = Vs + KT * D;               // [RT][KT+1]
  float* Os = S + RT * (KT + 1);        // [RT][D]
  float* mrow = Os + RT * D;            // [RT]
  float* lrow = mrow + RT;              // [RT]
  float* arow = lrow + RT;              // [RT]
  long long* tok_off = reinterpret_cast<long long*>(
      (reinterpret_cast<uintptr_t>(arow + RT) + 7) & ~uintptr_t(7));  // [KT]
  long long* tok_sidx = tok_off + KT;   // [KT] scale index (e4m3 caches)
  // The query's rounding: the cache dtype (q.to(k.dtype)), f16 for e4m3.
  constexpr int QR = KV_DT == kE4M3 ? kF16 : KV_DT;

  const long long s = blockIdx.x / a.plan.splits;
  const int j = blockIdx.x - (int)(s * a.plan.splits);
  const int kh = blockIdx.y;
  const int r0 = blockIdx.z * RT;
  const int nrows = a.rows - r0 < RT ? a.rows - r0 : RT;

  const long long ctx_s = load_index(a.ctx, a.ctx_i64, s);
  const long long nb = blocks_of(ctx_s, a.block_size, a.table_width);
  if (j == 0 && kh == 0 && blockIdx.z == 0 && tid == 0 &&
      ctx_s > a.table_width * (long long)a.block_size) {
    record_error(a.err, kErrTableWidth);
  }
  const long long blk_lo = (long long)j * a.plan.split_blocks;
  const long long blk_hi = blk_lo + a.plan.split_blocks < nb ? blk_lo + a.plan.split_blocks : nb;
  if (blk_lo >= blk_hi) return;
  const long long tok_lo = blk_lo * a.block_size;
  long long tok_hi = blk_hi * a.block_size;
  if (tok_hi > ctx_s) tok_hi = ctx_s;

  for (int idx = tid; idx < RT * D; idx += kThreads) {
    const int rr = idx / D;
    const int d = idx - rr * D;
    float v = 0.f;
    if (rr < nrows) {
      const int r = r0 + rr;
      const int qi = r / a.group;
      const int qh = kh * a.group + (r - qi * a.group);
      v = round_through<QR>(
          load_f32<Q_DT>(a.q, s * a.q_s + (long long)qh * a.q_h + (long long)qi * a.q_t + d));
    }
    Qs[idx] = v;
    Os[idx] = 0.f;
  }
  if (tid < RT) {
    mrow[tid] = -INFINITY;
    lrow[tid] = 0.f;
  }
  const long long row_elems = (long long)a.kv_heads * D;
  const long long layer_base = (long long)a.layer * a.num_blocks * a.block_size * row_elems;
  __syncthreads();

  for (long long kp0 = tok_lo; kp0 < tok_hi; kp0 += KT) {
    if (tid < KT) {
      const long long pos = kp0 + tid;
      long long off = -1, sidx = 0;
      if (pos < tok_hi) {
        const long long col = pos / a.block_size;
        const long long id = load_index(a.table, a.table_i64, s * a.table_stride + col);
        if (id >= 0 && id < a.num_blocks) {
          const long long slot = pos - col * a.block_size;
          off = layer_base + (id * a.block_size + slot) * row_elems + (long long)kh * D;
          sidx = (((long long)a.layer * a.num_blocks + id) * a.kv_heads + kh) * a.block_size +
                 slot;
        } else if (id >= a.num_blocks) {
          record_error(a.err, kErrBlockId);
        }
      }
      tok_off[tid] = off;
      tok_sidx[tid] = sidx;
    }
    __syncthreads();
    for (int idx = tid; idx < KT * D; idx += kThreads) {
      const int t = idx / D;
      const int d = idx - t * D;
      const long long off = tok_off[t];
      float kv = 0.f, vv = 0.f;
      if (off >= 0) {
        if constexpr (KV_DT == kE4M3) {
          const long long si = tok_sidx[t];
          kv = e4m3_to_f32(static_cast<const uint8_t*>(a.k_cache)[off + d]) * a.k_scale[si];
          vv = e4m3_to_f32(static_cast<const uint8_t*>(a.v_cache)[off + d]) * a.v_scale[si];
        } else {
          kv = load_f32<KV_DT>(a.k_cache, off + d);
          vv = load_f32<KV_DT>(a.v_cache, off + d);
        }
      }
      Ks[t * (D + 1) + d] = kv;
      Vs[t * D + d] = vv;
    }
    __syncthreads();
    for (int pidx = tid; pidx < RT * KT; pidx += kThreads) {
      const int rr = pidx / KT;
      const int t = pidx - rr * KT;
      float acc = 0.f;
      const float* qrow = Qs + rr * D;
      const float* krow = Ks + t * (D + 1);
      for (int d = 0; d < D; ++d) acc = fmaf(qrow[d], krow[d], acc);
      float x = acc * a.scale;
      if (a.softcap > 0.f) x = tanhf(x / a.softcap) * a.softcap;
      bool ok = rr < nrows && tok_off[t] >= 0;
      if (ok && a.q_len > 1) {
        const int qi = (r0 + rr) / a.group;
        ok = kp0 + t <= ctx_s - a.q_len + qi;
      }
      S[rr * (KT + 1) + t] = ok ? x : -INFINITY;
    }
    __syncthreads();
    if (tid < RT) {
      float* srow = S + tid * (KT + 1);
      float mx = -INFINITY;
      for (int t = 0; t < KT; ++t) mx = fmaxf(mx, srow[t]);
      const float mold = mrow[tid];
      const float mnew = fmaxf(mold, mx);
      const float mu = mnew == -INFINITY ? 0.f : mnew;
      const float al = expf(mold - mu);
      float sum = 0.f;
      for (int t = 0; t < KT; ++t) {
        const float p = expf(srow[t] - mu);
        srow[t] = p;
        sum += p;
      }
      lrow[tid] = lrow[tid] * al + sum;
      mrow[tid] = mnew;
      arow[tid] = al;
    }
    __syncthreads();
    for (int idx = tid; idx < RT * D; idx += kThreads) {
      const int rr = idx / D;
      const int d = idx - rr * D;
      float acc = Os[idx] * arow[rr];
      const float* prow = S + rr * (KT + 1);
      for (int t = 0; t < KT; ++t) acc = fmaf(prow[t], Vs[t * D + d], acc);
      Os[idx] = acc;
    }
    __syncthreads();
  }

  const long long slot = blockIdx.x;  // fixed plan: s * splits + j
  for (int idx = tid; idx < nrows * D; idx += kThreads) {
    const int rr = idx / D;
    const int d = idx - rr * D;
    const int r = r0 + rr;
    const int qi = r / a.group;
    const int qh = kh * a.group + (r - qi * a.group);
    const float l = lrow[rr];
    a.part_o[((slot * a.num_heads + qh) * a.q_len + qi) * D + d] = l > 0.f ? Os[idx] / l : 0.f;
  }
  if (tid < nrows) {
    const int r = r0 + tid;
    const int qi = r / a.group;
    const int qh = kh * a.group + (r - qi * a.group);
    const float l = lrow[tid];
    a.part_lse[(slot * a.num_heads + qh) * a.q_len + qi] =
        l > 0.f ? mrow[tid] + logf(l) : -INFINITY;
  }
}

template <int KV_DT, int Q_DT>
const void* generic_ptr() {
  return reinterpret_cast<const void*>(&attn_generic_kernel<KV_DT, Q_DT>);
}

const void* select_generic(const AttnArgs& a) {
#define LLMOPT_GENERIC_CASE(KT_, QT_) \
  if (a.kv_dtype == KT_ && a.q_dtype == QT_) return generic_ptr<KT_, QT_>();
  LLMOPT_GENERIC_CASE(kF32, kF32)
  LLMOPT_GENERIC_CASE(kF32, kF16)
  LLMOPT_GENERIC_CASE(kF32, kBF16)
  LLMOPT_GENERIC_CASE(kF16, kF32)
  LLMOPT_GENERIC_CASE(kF16, kF16)
  LLMOPT_GENERIC_CASE(kF16, kBF16)
  LLMOPT_GENERIC_CASE(kBF16, kF32)
  LLMOPT_GENERIC_CASE(kBF16, kF16)
  LLMOPT_GENERIC_CASE(kBF16, kBF16)
  LLMOPT_GENERIC_CASE(kE4M3, kF32)
  LLMOPT_GENERIC_CASE(kE4M3, kF16)
  LLMOPT_GENERIC_CASE(kE4M3, kBF16)
#undef LLMOPT_GENERIC_CASE
  return nullptr;
}

}  // namespace

bool generic_supported(const AttnArgs& a) {
  return a.head_dim >= 1 && a.head_dim <= 256 && a.plan.mode == kModeFixed &&
         select_generic(a) != nullptr;
}

cudaError_t generic_launch(const AttnArgs& a, cudaStream_t stream) {
  const void* fn = select_generic(a);
  if (fn == nullptr) return cudaErrorInvalidValue;
  const size_t smem = generic_smem(a.head_dim);
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const long long gx = a.batch * (long long)a.plan.splits;
  const long long gz = (a.rows + RT - 1) / RT;
  if (gx <= 0 || gz <= 0) return cudaSuccess;
  if (gx > 0x7fffffffLL || a.kv_heads > 65535 || gz > 65535) return cudaErrorInvalidConfiguration;
  dim3 grid((unsigned)gx, (unsigned)a.kv_heads, (unsigned)gz);
  void* args[] = {const_cast<AttnArgs*>(&a)};
  return launch_pdl(fn, grid, dim3(kThreads), args, smem, stream);
}

}  // namespace llmopt
