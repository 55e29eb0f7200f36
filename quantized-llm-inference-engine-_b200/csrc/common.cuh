// Shared device helpers for the paged-KV kernels (sm_100a).
//
// * element conversions with torch's rounding (round-to-nearest-even casts);
// * thin inline-PTX wrappers for mbarriers, TMA tile loads, ldmatrix and the
//   m16n8k16 tensor-core MMA used by the decode kernel;
// * bounded waits: every spin on an mbarrier gives up after kWaitLimitCycles,
//   records LLMOPT_DEVERR_WAIT_TIMEOUT and lets the kernel finish.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace llmopt {

// kE4M3: float8_e4m3fn KV storage with one fp32 scale per (token, head) row
// (value = e4m3 * scale); caches only.
enum DType : int { kF32 = 0, kF16 = 1, kBF16 = 2, kE4M3 = 3 };

// Largest finite e4m3 magnitude: a row's scale maps its amax onto it.
constexpr float kE4M3Max = 448.f;

constexpr unsigned kErrBlockId = 1u;
constexpr unsigned kErrTableWidth = 2u;
constexpr unsigned kErrWaitTimeout = 4u;
constexpr unsigned kErrPosition = 8u;       // rotary position outside the table (token skipped)
// Which wait gave up (set together with kErrWaitTimeout).
constexpr unsigned kErrWaitData = 0x100u;   // consumer waiting for a staged tile
constexpr unsigned kErrWaitSlot = 0x200u;   // producer waiting for a free ring slot
constexpr unsigned kErrWaitDrain = 0x400u;  // producer waiting for its last copies
constexpr unsigned kErrWaitPeer = 0x800u;   // cross-rank barrier of a gathered call

// About one second at B200 clocks: a wait that long means a lost producer.
constexpr long long kWaitLimitCycles = 2000000000LL;

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ void record_error(unsigned* err, unsigned bits) {
  if (err != nullptr) atomicOr(err, bits);
}

// ---------------------------------------------------------------------------
// element types
// ---------------------------------------------------------------------------
template <int DT> struct ElemT;
template <> struct ElemT<kF32> { using T = float; };
template <> struct ElemT<kF16> { using T = __half; };
template <> struct ElemT<kBF16> { using T = __nv_bfloat16; };

template <int DT>
__device__ __forceinline__ float load_f32(const void* base, long long idx) {
  if constexpr (DT == kF32) {
    return static_cast<const float*>(base)[idx];
  } else if constexpr (DT == kF16) {
    return __half2float(static_cast<const __half*>(base)[idx]);
  } else {
    return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[idx]);
  }
}

// float -> storage type, round-to-nearest-even (torch's .to(dtype) for finite
// values and infinities; subnormals are kept, not flushed).
template <int DT>
__device__ __forceinline__ typename ElemT<DT>::T from_f32(float x) {
  if constexpr (DT == kF32) {
    return x;
  } else if constexpr (DT == kF16) {
    return __float2half_rn(x);
  } else {
    return __float2bfloat16_rn(x);
  }
}

// Round a float to storage type DT and widen it back (q.to(k.dtype) in fp32 math).
template <int DT>
__device__ __forceinline__ float round_through(float x) {
  if constexpr (DT == kF32) {
    return x;
  } else if constexpr (DT == kF16) {
    return __half2float(__float2half_rn(x));
  } else {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
}

template <int DT>
__device__ __forceinline__ void store_f32(void* base, long long idx, float x) {
  static_cast<typename ElemT<DT>::T*>(base)[idx] = from_f32<DT>(x);
}

// Two floats packed into one 32-bit register of 16-bit elements (low = first).
template <int DT>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (DT == kF16) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// ---- float8 e4m3 (cuda_fp8.h conversions, hardware cvt on sm_100a) --------
// Two e4m3 bytes (low byte first) -> two f16 in one register; exact, since every
// e4m3 value is an f16 value.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t pair) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)pair, __NV_E4M3);
  return (uint32_t)h.x | ((uint32_t)h.y << 16);
}

// Four e4m3 bytes -> two f16 pairs: bytes (0, 1) into lo, (2, 3) into hi.  The
// word is split into its 16-bit halves in PTX so each conversion reads a half
// register directly.
__device__ __forceinline__ void e4m3x4_to_f16x2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t.reg .b16 l, h;\n\t"
      "mov.b32 {l, h}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, l;\n\t"
      "cvt.rn.f16x2.e4m3x2 %1, h;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(w));
}

__device__ __forceinline__ float e4m3_to_f32(uint8_t b) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3);
  return __half2float(__half(h));
}

// Round-to-nearest-even to e4m3, saturating to +-448 (NaN stays NaN).  The
// inputs here are already scaled into [-448, 448] (up to one rounding step),
// where this equals torch's non-saturating .to(torch.float8_e4m3fn).
__device__ __forceinline__ uint8_t f32_to_e4m3(float x) {
  return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}

// Scale of a row with largest magnitude amax: amax / 448, or 1 when that is
// not a positive number (an all-zero row, underflow, NaN).
__device__ __forceinline__ float e4m3_row_scale(float amax) {
  const float s = __fdiv_rn(amax, kE4M3Max);
  return s > 0.f ? s : 1.f;
}

__device__ __forceinline__ long long load_index(const void* p, int is64, long long i) {
  return is64 ? static_cast<const long long*>(p)[i]
              : static_cast<long long>(static_cast<const int*>(p)[i]);
}

// Python floor division / modulo (the reference's torch.div(..., "floor") and %).
__device__ __forceinline__ long long floordiv(long long a, long long b) {
  long long q = a / b;
  return (a % b != 0 && ((a < 0) != (b < 0))) ? q - 1 : q;
}
__device__ __forceinline__ long long floormod(long long a, long long b) {
  long long r = a % b;
  return (r != 0 && ((r < 0) != (b < 0))) ? r + b : r;
}

// write_decode's destination of sequence s (paged_cache.py:252-259): block
// id (an id < 0 or >= num_blocks goes to block 0) and slot; false when the
// table column is outside the row (nothing is written).
__device__ __forceinline__ bool decode_target(const void* table, int table_i64,
                                              long long table_stride, long long width,
                                              const void* offsets, int off_i64, long long bs,
                                              long long num_blocks, long long s,
                                              long long* block, long long* slot) {
  const long long off = load_index(offsets, off_i64, s);
  const long long col = floordiv(off, bs);
  if (col < -width || col >= width) return false;
  long long id = load_index(table, table_i64, s * table_stride + (col < 0 ? col + width : col));
  if (id < 0 || id >= num_blocks) id = 0;
  *block = id;
  *slot = floormod(off, bs);
  return true;
}

// True when a later sequence of the batch writes the same row of block 0.
// The reference's write_decode is one index_put, where the last of repeated
// indices wins; repeats arise by design only at block 0 (the redirect of
// invalid ids), so only rows of block 0 are checked.  Warp-collective.
__device__ __forceinline__ bool block0_row_taken_later(const void* table, int table_i64,
                                                       long long table_stride, long long width,
                                                       const void* offsets, int off_i64,
                                                       long long bs, long long num_blocks,
                                                       long long s, long long batch,
                                                       long long slot, int lane) {
  bool hit = false;
  for (long long s2 = s + 1 + lane; s2 < batch; s2 += 32) {
    long long b2, t2;
    if (decode_target(table, table_i64, table_stride, width, offsets, off_i64, bs, num_blocks,
                      s2, &b2, &t2) &&
        b2 == 0 && t2 == slot) {
      hit = true;
    }
  }
  return __any_sync(0xffffffffu, hit);
}

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// The same, suspending the thread until the phase completes or about `ns`
// nanoseconds pass (a suspended warp issues nothing).
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, unsigned parity, unsigned ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity; false after the limit.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitLimitCycles) return false;
  }
  return true;
}

// ---- thread-block clusters -------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The shared::cluster address of `local`'s offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(local)), "r"(rank));
  return r;
}
// Arrive on an mbarrier of any CTA of the cluster; the caller's earlier writes
// are released at cluster scope.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(
                   bar_cluster_addr)
               : "memory");
}
// Arrive on an mbarrier of any CTA of the cluster with the default (CTA-scope)
// release: for arrivals that publish tensor-memory writes, which the
// tcgen05 fences around the barrier order, not generic memory.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr)
               : "memory");
}
__device__ __forceinline__ void st_cluster_u32(uint32_t cluster_address, uint32_t v) {
  asm volatile("st.relaxed.cluster.shared::cluster.u32 [%0], %1;" ::"r"(cluster_address), "r"(v)
               : "memory");
}
// One test of a phase, acquiring at cluster scope (for barriers other CTAs
// arrive on).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity; false after the limit.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, unsigned parity) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait_cluster(bar, parity)) {
    if (clock64() - t0 > kWaitLimitCycles) return false;
  }
  return true;
}
// All threads of every CTA of the cluster meet (release / acquire).
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// 5-D TMA tile load into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3), "r"(c4)
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                              uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D = A * B + D for one m16n8k16 tile with fp32 accumulators.
template <int DT>
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  if constexpr (DT == kF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// Programmatic dependent launch: block until the previous kernel in the stream
// has finished and its writes are visible.  Every kernel here calls it before
// touching global memory, so launches can overlap the previous kernel's tail.
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
// Let the next kernel in the stream start launching; it still waits for this
// grid's completion (and memory visibility) in its own griddep_wait().
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// 2^x on the special-function unit (MUFU.EX2); exact 0 for -inf.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed two-lane fp32 fused multiply-add (sm_100): per lane exactly the
// IEEE operation of fmaf, at one issue for two.
// (b, b) and (c, c) come pre-packed (pack2f), built once outside the loop.
__device__ __forceinline__ uint64_t pack2f(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void ffma2(float& x0, float& x1, float a0, float a1, uint64_t bb,
                                      uint64_t cc) {
  asm("{\n\t.reg .b64 ra, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "fma.rn.f32x2 rd, ra, %4, %5;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(x0), "=f"(x1)
      : "f"(a0), "f"(a1), "l"(bb), "l"(cc));
}
// max(a, b, c) in one instruction (NaN operands ignored, as fmaxf does).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ float warp_max_xor(float v, int mask) {
  return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, mask));
}

}  // namespace llmopt
