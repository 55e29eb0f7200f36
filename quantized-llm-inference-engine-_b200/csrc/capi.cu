// extern "C" entry points declared in include/llmopt_b200.h: argument checks,
// split planning, TMA descriptor cache and kernel dispatch.  Apart from the
// llmopt_peer_* buffer routines, no entry point allocates device memory or
// synchronises the stream.
#include <nvtx3/nvToolsExt.h>
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <tuple>

#include "../../include/llmopt_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace llmopt {

namespace {
std::mutex g_carveout_mu;
std::set<std::pair<int, const void*>> g_carveout_done;
}  // namespace

// Every kernel of this library asks for the largest shared-memory carveout.
// An SM changes its L1 / shared split only when idle; with programmatic
// dependent launch the next kernel's CTAs are placed while the previous
// kernel's CTAs are still resident, so a small-shared kernel (combine, KV
// append) left at the default split would cap how many decode / prefill CTAs
// fit on that SM for the whole of their run - a one-wave grid then runs
// partly as a second wave.
cudaError_t ensure_max_shared_carveout(const void* fn) {
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(g_carveout_mu);
  if (g_carveout_done.count({device, fn})) return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess) g_carveout_done.insert({device, fn});
  return e;
}

cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, void** args, size_t smem,
                       cudaStream_t stream) {
  static const bool enabled = [] {
    const char* v = std::getenv("LLMOPT_B200_PDL");
    return !(v != nullptr && v[0] == '0');
  }();
  cudaError_t ce = ensure_max_shared_carveout(fn);
  if (ce != cudaSuccess) return ce;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = enabled ? 1 : 0;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace llmopt

namespace {

using namespace llmopt;

thread_local std::string g_last_error;

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int ok() {
  g_last_error.clear();
  return LLMOPT_OK;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(LLMOPT_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool valid_dtype(int dt) { return dt == kF32 || dt == kF16 || dt == kBF16; }

// ---- device properties ---------------------------------------------------------
std::mutex g_dev_mu;
std::map<int, int> g_sm_count;

int sm_count_of(int device) {
  std::lock_guard<std::mutex> lock(g_dev_mu);
  auto it = g_sm_count.find(device);
  if (it != g_sm_count.end()) return it->second;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) {
    n = 148;
  }
  g_sm_count[device] = n;
  return n;
}

int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) d = 0;
  return d;
}

// ---- TMA descriptors -------------------------------------------------------------
// One 5-D descriptor per cache tensor: (head_dim, kv_heads, block_size,
// num_blocks, layers), box (64, 1, block_size, 1, 1), 128-byte swizzle.
using TmaKey = std::tuple<uintptr_t, int, int, int, int, int, int, int>;
std::mutex g_tma_mu;
std::map<TmaKey, CUtensorMap> g_tma_cache;

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  return fn;
}

bool kv_tensor_map(const void* base, int dtype, int layers, int num_blocks, int block_size,
                   int kv_heads, int head_dim, CUtensorMap* out, std::string* why) {
  const TmaKey key{reinterpret_cast<uintptr_t>(base), dtype, layers, num_blocks, block_size,
                   kv_heads, head_dim, 0};
  {
    std::lock_guard<std::mutex> lock(g_tma_mu);
    auto it = g_tma_cache.find(key);
    if (it != g_tma_cache.end()) {
      *out = it->second;
      return true;
    }
  }
  auto encode = tensor_map_encoder();
  if (encode == nullptr) {
    *why = "cuTensorMapEncodeTiled unavailable";
    return false;
  }
  // e4m3 codes: one byte per element, boxes of 128 dims (the swizzle span).
  const bool e4m3 = dtype == kE4M3;
  const cuuint64_t es = e4m3 ? 1 : 2;
  cuuint64_t dims[5] = {(cuuint64_t)head_dim, (cuuint64_t)kv_heads, (cuuint64_t)block_size,
                        (cuuint64_t)num_blocks, (cuuint64_t)layers};
  cuuint64_t strides[4] = {es * head_dim, es * head_dim * kv_heads,
                           es * head_dim * kv_heads * block_size,
                           es * head_dim * kv_heads * block_size * (cuuint64_t)num_blocks};
  cuuint32_t box[5] = {e4m3 ? 128u : 64u, 1, (cuuint32_t)block_size, 1, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUtensorMap map;
  std::memset(&map, 0, sizeof(map));
  CUresult r = encode(&map,
                      e4m3            ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                      : dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                      5, const_cast<void*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[96];
    snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (%d)", (int)r);
    *why = buf;
    return false;
  }
  std::lock_guard<std::mutex> lock(g_tma_mu);
  if (g_tma_cache.size() > 512) g_tma_cache.clear();
  g_tma_cache[key] = map;
  *out = map;
  return true;
}

}  // namespace

bool llmopt::tensor_map_2d(CUtensorMap* out, CUtensorMapDataType dtype, const void* base,
                           uint64_t inner, uint64_t outer, uint64_t row_bytes,
                           uint32_t box_inner, uint32_t box_outer) {
  auto encode = tensor_map_encoder();
  if (encode == nullptr) return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  std::memset(out, 0, sizeof(*out));
  return encode(out, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

namespace {

// Per-call descriptor of the query for the prefill kernel: (head_dim, q_len,
// num_heads, batch), box (64, 128 / group tokens, group heads, 1).
bool query_tensor_map(const AttnArgs& a, CUtensorMap* out, std::string* why) {
  auto encode = tensor_map_encoder();
  if (encode == nullptr) {
    *why = "cuTensorMapEncodeTiled unavailable";
    return false;
  }
  const cuuint64_t es = 2;
  cuuint64_t dims[4] = {(cuuint64_t)a.head_dim, (cuuint64_t)a.q_len, (cuuint64_t)a.num_heads,
                        (cuuint64_t)a.batch};
  cuuint64_t strides[3] = {es * (cuuint64_t)a.q_t, es * (cuuint64_t)a.q_h,
                           es * (cuuint64_t)a.q_s};
  cuuint32_t box[4] = {64, (cuuint32_t)(kPrefillRows / a.group), (cuuint32_t)a.group, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  std::memset(out, 0, sizeof(*out));
  CUresult r = encode(out,
                      a.q_dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                      4, const_cast<void*>(a.q), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[96];
    snprintf(buf, sizeof(buf), "query cuTensorMapEncodeTiled failed (%d)", (int)r);
    *why = buf;
    return false;
  }
  return true;
}

// ---- split planning and workspace layout ------------------------------------------
constexpr long long kAlign = 256;
constexpr int kMaxBalancedCtasPerSm = 16;
constexpr long long kMaxBalancedBatch = 4096;

long long round_up(long long x, long long a) { return (x + a - 1) / a * a; }

struct WsLayout {
  long long prefix_off, lse_off, o_off, total;
};

WsLayout layout_for(long long batch, long long slots, int num_heads, int q_len, int head_dim) {
  WsLayout w;
  w.prefix_off = 0;
  w.lse_off = round_up(4 * (batch + 1), kAlign);
  w.o_off = w.lse_off + round_up(4 * slots * num_heads * (long long)q_len, kAlign);
  w.total = w.o_off + round_up(4 * slots * num_heads * (long long)q_len * head_dim, kAlign);
  return w;
}

SplitPlan fixed_plan(long long batch, long long width, long long split_blocks) {
  SplitPlan p{};
  p.mode = kModeFixed;
  const long long w = width > 0 ? width : 1;
  if (split_blocks < 1) split_blocks = 1;
  if (split_blocks > w) split_blocks = w;
  p.split_blocks = (int)split_blocks;
  p.splits = (int)((w + split_blocks - 1) / split_blocks);
  p.ctas = 0;
  p.slots = batch * p.splits;
  return p;
}

// Fixed plan for an explicit split_tokens (> 0: chunk size; < 0: one chunk).
SplitPlan explicit_plan(long long batch, long long width, int block_size, long long split_tokens) {
  if (split_tokens < 0) return fixed_plan(batch, width, width);
  return fixed_plan(batch, width, (split_tokens + block_size - 1) / block_size);
}

// Automatic fixed plan for the CUDA-core path: about two waves of CTAs.
SplitPlan generic_auto_plan(long long batch, long long width, int kv_heads, int rows, int sms) {
  const long long row_tiles = (rows + kGenericRowTile - 1) / kGenericRowTile;
  const long long per_split = batch * kv_heads * row_tiles;
  long long splits = per_split > 0 ? (2LL * sms + per_split - 1) / per_split : 1;
  const long long w = width > 0 ? width : 1;
  if (splits > w) splits = w;
  if (splits < 1) splits = 1;
  return fixed_plan(batch, width, (w + splits - 1) / splits);
}

struct Choice {
  bool tma = false;      // decode_tma_kernel + combine
  bool prefill = false;  // prefill_tc_kernel (no combine)
  DecodeLaunch launch{};
  SplitPlan plan{};
  CUtensorMap tmk, tmv, tmq;
};

// Pick the kernel and split plan.  Returns LLMOPT_OK or an error code.
int choose(AttnArgs& a, long long split_tokens, int device, bool encode_maps, Choice* c) {
  const int sms = sm_count_of(device);
  const bool e4m3 = a.kv_dtype == kE4M3;
  // Dense chunked prefill: tensor-core tiles over whole sequences, no split-K.
  if (!e4m3 && prefill_tc_supported(a)) {
    bool maps = true;
    if (encode_maps) {
      std::string why;
      maps = query_tensor_map(a, &c->tmq, &why) &&
             kv_tensor_map(a.k_cache, a.kv_dtype, a.num_layers, a.num_blocks, a.block_size,
                           a.kv_heads, a.head_dim, &c->tmk, &why) &&
             kv_tensor_map(a.v_cache, a.kv_dtype, a.num_layers, a.num_blocks, a.block_size,
                           a.kv_heads, a.head_dim, &c->tmv, &why);
    }
    if (maps) {
      c->prefill = true;
      c->tma = false;
      c->plan = fixed_plan(a.batch, a.table_width, a.table_width);
      c->plan.slots = 0;
      return LLMOPT_OK;
    }
  }
  // Fast path first: it supports the balanced plan (auto) and fixed plans.
  AttnArgs probe = a;
  if (split_tokens == LLMOPT_SPLIT_AUTO && a.batch <= kMaxBalancedBatch) {
    probe.plan.mode = kModeBalanced;
  } else if (split_tokens == LLMOPT_SPLIT_AUTO) {
    probe.plan = generic_auto_plan(a.batch, a.table_width, a.kv_heads, a.rows, sms);
  } else {
    probe.plan = explicit_plan(a.batch, a.table_width, a.block_size, split_tokens);
  }
  const bool fast = e4m3 ? decode_fp8_supported(probe) && decode_fp8_configure(probe, sms, &c->launch)
                         : decode_tma_supported(probe) && decode_tma_configure(probe, sms, &c->launch);
  if (fast) {
    bool maps = true;
    if (encode_maps) {
      std::string why;
      maps = kv_tensor_map(a.k_cache, a.kv_dtype, a.num_layers, a.num_blocks, a.block_size,
                           a.kv_heads, a.head_dim, &c->tmk, &why) &&
             kv_tensor_map(a.v_cache, a.kv_dtype, a.num_layers, a.num_blocks, a.block_size,
                           a.kv_heads, a.head_dim, &c->tmv, &why);
    }
    if (maps) {
      c->tma = true;
      c->plan = probe.plan;
      if (c->plan.mode == kModeBalanced) {
        const int head_groups = a.kv_heads / c->launch.heads_per_cta;
        int occ = c->launch.ctas_per_sm;
        if (occ > kMaxBalancedCtasPerSm) occ = kMaxBalancedCtasPerSm;
        long long ctas = (long long)sms * occ / head_groups;
        if (ctas < 1) ctas = 1;
        if (!e4m3 && c->launch.streams == 2) ctas *= 2;  // plan ranges, two per CTA
        c->plan.ctas = (int)ctas;
        c->plan.split_blocks = 0;
        c->plan.splits = 0;
        c->plan.slots = a.batch + ctas;
      }
      return LLMOPT_OK;
    }
  }
  c->tma = false;
  c->plan = split_tokens == LLMOPT_SPLIT_AUTO
                ? generic_auto_plan(a.batch, a.table_width, a.kv_heads, a.rows, sms)
                : explicit_plan(a.batch, a.table_width, a.block_size, split_tokens);
  AttnArgs g = a;
  g.plan = c->plan;
  if (!generic_supported(g)) {
    return fail(LLMOPT_ERR_UNSUPPORTED, "no kernel for head_dim=%d q_dtype=%d kv_dtype=%d",
                a.head_dim, a.q_dtype, a.kv_dtype);
  }
  return LLMOPT_OK;
}

// Upper bound of the workspace over every plan `choose` can return.
long long workspace_bound(long long batch, int num_heads, int kv_heads, int head_dim, int q_len,
                          int block_size, long long width, long long split_tokens, int sms) {
  const int rows = q_len * (num_heads / (kv_heads > 0 ? kv_heads : 1));
  long long slots = 0;
  if (split_tokens == LLMOPT_SPLIT_AUTO) {
    slots = generic_auto_plan(batch, width, kv_heads, rows, sms).slots;
    if (batch <= kMaxBalancedBatch) {
      const long long bal = batch + (long long)sms * kMaxBalancedCtasPerSm;
      if (bal > slots) slots = bal;
    }
  } else {
    slots = explicit_plan(batch, width, block_size, split_tokens).slots;
  }
  return layout_for(batch, slots, num_heads, q_len, head_dim).total;
}

}  // namespace

namespace {
// NVTX range around a C-ABI call, so the entry points appear by name on
// Nsight timelines (header-only NVTX 3; a no-op unless a tool is attached).
struct Range {
  explicit Range(const char* name) { nvtxRangePushA(name); }
  ~Range() { nvtxRangePop(); }
  Range(const Range&) = delete;
  Range& operator=(const Range&) = delete;
};
}  // namespace
#define LLMOPT_RANGE(name) Range llmopt_range_(name)

extern "C" {

const char* llmopt_b200_version(void) { return "llmopt-b200 0.1.0 (sm_100a)"; }

int llmopt_b200_abi_version(void) { return LLMOPT_B200_ABI_VERSION; }

const char* llmopt_status_string(int status) {
  switch (status) {
    case LLMOPT_OK: return "ok";
    case LLMOPT_ERR_INVALID_ARGUMENT: return "invalid argument";
    case LLMOPT_ERR_UNSUPPORTED: return "unsupported dtype or shape";
    case LLMOPT_ERR_WORKSPACE: return "workspace too small";
    case LLMOPT_ERR_CUDA: return "CUDA error";
    case LLMOPT_ERR_INDEX: return "index out of range";
    default: return "unknown status";
  }
}

const char* llmopt_last_error(void) { return g_last_error.c_str(); }

int llmopt_paged_attention_workspace_size(int device, int64_t batch, int32_t num_heads,
                                          int32_t num_kv_heads, int32_t head_dim, int32_t q_len,
                                          int32_t block_size, int64_t table_width,
                                          int32_t kv_dtype, int64_t split_tokens,
                                          size_t* bytes) {
  (void)kv_dtype;
  if (bytes == nullptr) return fail(LLMOPT_ERR_INVALID_ARGUMENT, "bytes is null");
  if (batch < 0 || num_heads < 1 || num_kv_heads < 1 || head_dim < 1 || q_len < 0 ||
      block_size < 1 || table_width < 0) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "invalid shape");
  }
  if (num_heads % num_kv_heads != 0) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "num_heads must be divisible by num_kv_heads");
  }
  if (batch == 0 || q_len == 0) {
    *bytes = 0;
    return ok();
  }
  *bytes = (size_t)workspace_bound(batch, num_heads, num_kv_heads, head_dim, q_len, block_size,
                                   table_width, split_tokens, sm_count_of(device));
  return ok();
}

int llmopt_paged_attention(const void* query, int32_t q_dtype, int64_t q_s, int64_t q_h,
                           int64_t q_t, const void* key_cache, const void* value_cache,
                           int32_t kv_dtype, int32_t num_layers, int32_t num_blocks,
                           int32_t block_size, int32_t num_kv_heads, int32_t head_dim,
                           int32_t layer_idx, const void* block_table, int32_t table_is_i64,
                           int64_t table_width, int64_t table_stride, const void* context_lens,
                           int32_t ctx_is_i64, void* out, int32_t out_dtype, int64_t o_s,
                           int64_t o_h, int64_t o_t, float* lse, int64_t batch, int32_t num_heads,
                           int32_t q_len, float scale, float softcap, int64_t split_tokens,
                           void* workspace, size_t workspace_bytes, uint32_t* err,
                           void* stream) {
  LLMOPT_RANGE("llmopt_paged_attention");
  return llmopt_paged_attention_phase(
      query, q_dtype, q_s, q_h, q_t, key_cache, value_cache, kv_dtype, num_layers, num_blocks,
      block_size, num_kv_heads, head_dim, layer_idx, block_table, table_is_i64, table_width,
      table_stride, context_lens, ctx_is_i64, out, out_dtype, o_s, o_h, o_t, lse, batch,
      num_heads, q_len, scale, softcap, split_tokens, workspace, workspace_bytes, err, stream,
      LLMOPT_PHASE_ALL);
}

namespace {

// Body of llmopt_paged_attention_phase; with `peers` the combine phase also
// delivers the output to every rank of the head-sharded group.
int phase_impl(const void* query, int32_t q_dtype, int64_t q_s, int64_t q_h, int64_t q_t,
               const void* key_cache, const void* value_cache, int32_t kv_dtype,
               int32_t num_layers, int32_t num_blocks, int32_t block_size,
               int32_t num_kv_heads, int32_t head_dim, int32_t layer_idx,
               const void* block_table, int32_t table_is_i64, int64_t table_width,
               int64_t table_stride, const void* context_lens, int32_t ctx_is_i64, void* out,
               int32_t out_dtype, int64_t o_s, int64_t o_h, int64_t o_t, float* lse,
               int64_t batch, int32_t num_heads, int32_t q_len, float scale, float softcap,
               int64_t split_tokens, void* workspace, size_t workspace_bytes, uint32_t* err,
               void* stream, int32_t phases, const PeerArgs* peers,
               const float* k_scale = nullptr, const float* v_scale = nullptr) {
  if (phases < 1 || phases > LLMOPT_PHASE_ALL) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "phases must be 1, 2 or 3");
  }
  // e4m3 caches come with their scales (llmopt_paged_attention_scaled only).
  const bool kv_ok = k_scale != nullptr ? kv_dtype == kE4M3 : valid_dtype(kv_dtype);
  if (!valid_dtype(q_dtype) || !kv_ok || !valid_dtype(out_dtype)) {
    return fail(LLMOPT_ERR_UNSUPPORTED, "unsupported dtype (q=%d kv=%d out=%d)", q_dtype,
                kv_dtype, out_dtype);
  }
  if (kv_dtype == kE4M3 && (v_scale == nullptr || head_dim > 256)) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "e4m3 cache needs both scale arrays, head_dim <= 256");
  }
  if (num_heads < 1 || num_kv_heads < 1 || num_heads % num_kv_heads != 0) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "num_heads must be divisible by num_kv_heads");
  }
  if (batch < 0 || q_len < 0 || num_layers < 1 || num_blocks < 1 || block_size < 1 ||
      head_dim < 1 || table_width < 0) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "invalid shape");
  }
  if (layer_idx < 0 || layer_idx >= num_layers) {
    return fail(LLMOPT_ERR_INDEX, "layer_idx %d out of range [0, %d)", layer_idx, num_layers);
  }
  if (head_dim > 256) {
    return fail(LLMOPT_ERR_UNSUPPORTED, "head_dim %d > 256", head_dim);
  }
  if (batch == 0 || q_len == 0) return ok();
  if (!query || !key_cache || !value_cache || !out || !context_lens ||
      (!block_table && table_width > 0)) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "null pointer argument");
  }
  if (table_width > 0 && table_stride < table_width) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "table_stride < table_width");
  }
  AttnArgs a{};
  a.q = query;
  a.q_s = q_s;
  a.q_h = q_h;
  a.q_t = q_t;
  a.q_dtype = q_dtype;
  a.k_cache = key_cache;
  a.v_cache = value_cache;
  a.kv_dtype = kv_dtype;
  a.num_layers = num_layers;
  a.num_blocks = num_blocks;
  a.block_size = block_size;
  a.kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.layer = layer_idx;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.table = block_table;
  a.table_i64 = table_is_i64 ? 1 : 0;
  a.table_width = table_width;
  a.table_stride = table_stride;
  a.ctx = context_lens;
  a.ctx_i64 = ctx_is_i64 ? 1 : 0;
  a.batch = batch;
  a.num_heads = num_heads;
  a.q_len = q_len;
  a.group = num_heads / num_kv_heads;
  a.rows = q_len * a.group;
  a.scale = scale;
  a.softcap = softcap;
  a.out = out;
  a.out_dtype = out_dtype;
  a.o_s = o_s;
  a.o_h = o_h;
  a.o_t = o_t;
  a.lse = lse;
  a.err = err;

  const int device = current_device();
  Choice c;
  int st = choose(a, split_tokens, device, true, &c);
  if (st != LLMOPT_OK) return st;
  a.plan = c.plan;
  const WsLayout w = layout_for(batch, a.plan.slots, num_heads, q_len, head_dim);
  if (workspace == nullptr || (long long)workspace_bytes < w.total) {
    return fail(LLMOPT_ERR_WORKSPACE, "workspace of %zu bytes < %lld needed", workspace_bytes,
                w.total);
  }
  if (reinterpret_cast<uintptr_t>(workspace) % 16 != 0) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "workspace must be 16-byte aligned");
  }
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  a.prefix = reinterpret_cast<int*>(ws + w.prefix_off);
  a.part_lse = reinterpret_cast<float*>(ws + w.lse_off);
  a.part_o = reinterpret_cast<float*>(ws + w.o_off);

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (phases & LLMOPT_PHASE_SPLIT) {
    cudaError_t e = c.prefill ? prefill_tc_launch(a, c.tmq, c.tmk, c.tmv, s)
                    : c.tma   ? (kv_dtype == kE4M3 ? decode_fp8_launch(a, c.launch, c.tmk, c.tmv, s)
                                                   : decode_tma_launch(a, c.launch, c.tmk, c.tmv, s))
                              : generic_launch(a, s);
    if (e != cudaSuccess) {
      return cuda_fail(e, c.prefill ? "prefill_tc launch"
                          : c.tma   ? "decode_tma launch"
                                    : "generic launch");
    }
  }
  if ((phases & LLMOPT_PHASE_COMBINE) && peers != nullptr) {
    const int elem = out_dtype == kF32 ? 4 : 2;
    cudaError_t e = c.prefill ? push_gather_launch(a, *peers, elem, s)
                              : combine_gather_launch(a, *peers, s);
    if (e != cudaSuccess) return cuda_fail(e, c.prefill ? "push_gather launch" : "combine_gather launch");
  } else if ((phases & LLMOPT_PHASE_COMBINE) && !c.prefill) {
    cudaError_t e = combine_launch(a, s);
    if (e != cudaSuccess) return cuda_fail(e, "combine launch");
  }
  return ok();
}

}  // namespace

int llmopt_paged_attention_phase(const void* query, int32_t q_dtype, int64_t q_s, int64_t q_h,
                                 int64_t q_t, const void* key_cache, const void* value_cache,
                                 int32_t kv_dtype, int32_t num_layers, int32_t num_blocks,
                                 int32_t block_size, int32_t num_kv_heads, int32_t head_dim,
                                 int32_t layer_idx, const void* block_table,
                                 int32_t table_is_i64, int64_t table_width,
                                 int64_t table_stride, const void* context_lens,
                                 int32_t ctx_is_i64, void* out, int32_t out_dtype, int64_t o_s,
                                 int64_t o_h, int64_t o_t, float* lse, int64_t batch,
                                 int32_t num_heads, int32_t q_len, float scale, float softcap,
                                 int64_t split_tokens, void* workspace, size_t workspace_bytes,
                                 uint32_t* err, void* stream, int32_t phases) {
  LLMOPT_RANGE("llmopt_paged_attention_phase");
  return phase_impl(query, q_dtype, q_s, q_h, q_t, key_cache, value_cache, kv_dtype, num_layers,
                    num_blocks, block_size, num_kv_heads, head_dim, layer_idx, block_table,
                    table_is_i64, table_width, table_stride, context_lens, ctx_is_i64, out,
                    out_dtype, o_s, o_h, o_t, lse, batch, num_heads, q_len, scale, softcap,
                    split_tokens, workspace, workspace_bytes, err, stream, phases, nullptr);
}

int llmopt_paged_attention_scaled(
    const void* query, int32_t q_dtype, int64_t q_s, int64_t q_h, int64_t q_t,
    const void* key_cache, const void* value_cache, int32_t kv_dtype, const float* key_scale,
    const float* value_scale, int32_t num_layers, int32_t num_blocks, int32_t block_size,
    int32_t num_kv_heads, int32_t head_dim, int32_t layer_idx, const void* block_table,
    int32_t table_is_i64, int64_t table_width, int64_t table_stride, const void* context_lens,
    int32_t ctx_is_i64, void* out, int32_t out_dtype, int64_t o_s, int64_t o_h, int64_t o_t,
    float* lse, int64_t batch, int32_t num_heads, int32_t q_len, float scale, float softcap,
    int64_t split_tokens, void* workspace, size_t workspace_bytes, uint32_t* err, void* stream,
    int32_t phases) {
  LLMOPT_RANGE("llmopt_paged_attention_scaled");
  if (kv_dtype != kE4M3 || key_scale == nullptr || value_scale == nullptr) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT,
                "llmopt_paged_attention_scaled takes an e4m3 cache and both scale arrays");
  }
  return phase_impl(query, q_dtype, q_s, q_h, q_t, key_cache, value_cache, kv_dtype, num_layers,
                    num_blocks, block_size, num_kv_heads, head_dim, layer_idx, block_table,
                    table_is_i64, table_width, table_stride, context_lens, ctx_is_i64, out,
                    out_dtype, o_s, o_h, o_t, lse, batch, num_heads, q_len, scale, softcap,
                    split_tokens, workspace, workspace_bytes, err, stream, phases, nullptr,
                    key_scale, value_scale);
}

// ---- head-sharded groups: peer memory and the gathered entry -----------------
static_assert(sizeof(cudaIpcMemHandle_t) == LLMOPT_PEER_HANDLE_BYTES, "IPC handle size");
static_assert(kMaxPeers == LLMOPT_MAX_PEERS, "peer count");

namespace {

// Runs fn with `device` current and restores the caller's device afterwards.
int on_device(int32_t device, const std::function<int()>& fn) {
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  const int st = fn();
  cudaSetDevice(prev);
  return st;
}

}  // namespace

int llmopt_peer_alloc(int32_t device, size_t bytes, void** ptr, void* handle) {
  if (ptr == nullptr || handle == nullptr || bytes == 0) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "peer_alloc needs bytes > 0, ptr and handle");
  }
  *ptr = nullptr;
  return on_device(device, [&]() -> int {
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(peer buffer)");
    e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) {
      e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), p);
    }
    if (e != cudaSuccess) {
      cudaFree(p);
      return cuda_fail(e, "peer buffer setup");
    }
    *ptr = p;
    return ok();
  });
}

int llmopt_peer_open(int32_t device, const void* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "peer_open needs handle and ptr");
  }
  *ptr = nullptr;
  return on_device(device, [&]() -> int {
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
    *ptr = p;
    return ok();
  });
}

int llmopt_peer_close(int32_t device, void* ptr) {
  if (ptr == nullptr) return ok();
  return on_device(device, [&]() -> int {
    cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? ok() : cuda_fail(e, "cudaIpcCloseMemHandle");
  });
}

int llmopt_peer_free(int32_t device, void* ptr) {
  if (ptr == nullptr) return ok();
  return on_device(device, [&]() -> int {
    cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? ok() : cuda_fail(e, "cudaFree(peer buffer)");
  });
}

int llmopt_paged_attention_gather(
    const void* query, int32_t q_dtype, int64_t q_s, int64_t q_h, int64_t q_t,
    const void* key_cache, const void* value_cache, int32_t kv_dtype, int32_t num_layers,
    int32_t num_blocks, int32_t block_size, int32_t num_kv_heads, int32_t head_dim,
    int32_t layer_idx, const void* block_table, int32_t table_is_i64, int64_t table_width,
    int64_t table_stride, const void* context_lens, int32_t ctx_is_i64,
    void* const* gathered, uint32_t* const* flags, int32_t world, int32_t rank, uint32_t epoch,
    int32_t out_dtype, float* lse, int64_t batch, int32_t num_heads, int32_t q_len, float scale,
    float softcap, int64_t split_tokens, void* workspace, size_t workspace_bytes,
    uint32_t* err, void* stream, int32_t phases) {
  LLMOPT_RANGE("llmopt_paged_attention_gather");
  if (world < 1 || world > LLMOPT_MAX_PEERS || rank < 0 || rank >= world) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "rank %d of world %d (at most %d ranks)", rank,
                world, LLMOPT_MAX_PEERS);
  }
  if (gathered == nullptr || flags == nullptr) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "null peer array");
  }
  PeerArgs p{};
  for (int r = 0; r < world; ++r) {
    if (gathered[r] == nullptr || flags[r] == nullptr) {
      return fail(LLMOPT_ERR_INVALID_ARGUMENT, "null peer pointer for rank %d", r);
    }
    if (reinterpret_cast<uintptr_t>(gathered[r]) % 16 != 0 ||
        reinterpret_cast<uintptr_t>(flags[r]) % 16 != 0) {
      return fail(LLMOPT_ERR_INVALID_ARGUMENT, "peer buffers must be 16-byte aligned");
    }
    p.out[r] = gathered[r];
    p.flags[r] = flags[r];
  }
  p.counter = flags[rank] + LLMOPT_MAX_PEERS;
  p.epoch = epoch;
  p.world = world;
  p.rank = rank;
  const int64_t o_t = head_dim;
  const int64_t o_s = (int64_t)q_len * head_dim;
  const int64_t o_h = batch * o_s;
  const size_t elem = out_dtype == kF32 ? 4 : 2;
  unsigned char* own = static_cast<unsigned char*>(gathered[rank]) +
                       (size_t)rank * num_heads * (size_t)o_h * elem;
  return phase_impl(query, q_dtype, q_s, q_h, q_t, key_cache, value_cache, kv_dtype, num_layers,
                    num_blocks, block_size, num_kv_heads, head_dim, layer_idx, block_table,
                    table_is_i64, table_width, table_stride, context_lens, ctx_is_i64, own,
                    out_dtype, o_s, o_h, o_t, lse, batch, num_heads, q_len, scale, softcap,
                    split_tokens, workspace, workspace_bytes, err, stream, phases, &p);
}

// ---- weight-only quantized linear ---------------------------------------------
namespace {

// Checks shared by the quantized-linear entry points; fills the kernel args.
int quant_args(const void* qweight, int32_t bits, int32_t group_size, int32_t symmetric,
               const float* scales, const float* zeros, int64_t n, int64_t k,
               QuantLinearArgs* a) {
  if (bits != 2 && bits != 4 && bits != 8) {
    return fail(LLMOPT_ERR_UNSUPPORTED, "bits must be 2, 4 or 8 (got %d)", bits);
  }
  if (n < 1 || k < 1 || group_size < 1 || k % group_size != 0 || (bits < 8 && k % 2 != 0)) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT,
                "invalid shape: n=%lld k=%lld group_size=%d (k must be a multiple of the "
                "group size, and even for 2/4-bit codes)",
                (long long)n, (long long)k, group_size);
  }
  if (qweight == nullptr || scales == nullptr || (!symmetric && zeros == nullptr)) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "null pointer argument");
  }
  *a = QuantLinearArgs{};
  a->qweight = static_cast<const unsigned char*>(qweight);
  a->bits = bits;
  a->group = group_size;
  a->symmetric = symmetric ? 1 : 0;
  a->scales = scales;
  a->zeros = zeros;
  a->n = n;
  a->k = k;
  return LLMOPT_OK;
}

// Split of the k range (whole 128-column tiles) for the tensor-core path.
void plan_quant_splits(QuantLinearArgs* a, int sms) {
  a->splits = 1;
  a->k_per_split = a->k;
  if (!quant_linear_tc_supported(*a)) return;
  const long long tiles = a->k / 128;
  int want = quant_linear_splits(*a, sms);
  // LLMOPT_B200_QUANT_SPLITS=n fixes the split count (tuning measurements).
  static const int forced = [] {
    const char* v = std::getenv("LLMOPT_B200_QUANT_SPLITS");
    return v != nullptr ? std::atoi(v) : 0;
  }();
  if (forced > 0) want = forced < (int)tiles ? forced : (int)tiles;
  const long long per = (tiles + want - 1) / want;
  a->k_per_split = per * 128;
  a->splits = (int)((tiles + per - 1) / per);
}

// fp32 workspace bytes of a planned call.
size_t quant_workspace_bytes(const QuantLinearArgs& a) {
  return a.splits > 1 ? (size_t)a.splits * (size_t)a.m * (size_t)a.n * sizeof(float) : 0;
}

}  // namespace

int llmopt_quant_linear_workspace_size(int device, int64_t m, int64_t n, int64_t k,
                                       int32_t bits, int32_t group_size, int32_t x_dtype,
                                       size_t* bytes) {
  if (bytes == nullptr) return fail(LLMOPT_ERR_INVALID_ARGUMENT, "bytes is null");
  *bytes = 0;
  if (m < 0) return fail(LLMOPT_ERR_INVALID_ARGUMENT, "m < 0");
  if (!valid_dtype(x_dtype)) return fail(LLMOPT_ERR_UNSUPPORTED, "unsupported dtype %d", x_dtype);
  QuantLinearArgs a{};
  static const float kDummy[4] = {};
  const int st = quant_args(kDummy, bits, group_size, 1, kDummy, kDummy, n, k, &a);
  if (st != LLMOPT_OK) return st;
  if (m == 0) return ok();
  // Size for 16-byte aligned operands (an unaligned call runs without splits).
  alignas(16) static const unsigned char kAligned[16] = {};
  a.x = kAligned;
  a.qweight = kAligned;
  a.x_dtype = x_dtype;
  a.m = m;
  a.ldx = k;
  plan_quant_splits(&a, sm_count_of(device));
  *bytes = quant_workspace_bytes(a);
  return ok();
}

int llmopt_quant_linear(const void* x, int32_t x_dtype, int64_t m, int64_t ldx,
                        const void* qweight, int32_t bits, int32_t group_size,
                        int32_t symmetric, const float* scales, const float* zeros, int64_t n,
                        int64_t k, const void* bias, void* out, int64_t ldo, void* workspace,
                        size_t workspace_bytes, void* stream) {
  LLMOPT_RANGE("llmopt_quant_linear");
  if (!valid_dtype(x_dtype)) return fail(LLMOPT_ERR_UNSUPPORTED, "unsupported dtype %d", x_dtype);
  QuantLinearArgs a{};
  int st = quant_args(qweight, bits, group_size, symmetric, scales, zeros, n, k, &a);
  if (st != LLMOPT_OK) return st;
  if (m < 0 || ldx < k || ldo < n) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "invalid shape: m=%lld ldx=%lld ldo=%lld",
                (long long)m, (long long)ldx, (long long)ldo);
  }
  if (m == 0) return ok();
  if (x == nullptr || out == nullptr) return fail(LLMOPT_ERR_INVALID_ARGUMENT, "null pointer argument");
  a.x = x;
  a.x_dtype = x_dtype;
  a.m = m;
  a.ldx = ldx;
  a.bias = bias;
  a.out = out;
  a.ldo = ldo;
  plan_quant_splits(&a, sm_count_of(current_device()));
  const size_t need = quant_workspace_bytes(a);
  if (need > 0) {
    if (workspace == nullptr || workspace_bytes < need) {
      return fail(LLMOPT_ERR_WORKSPACE, "workspace of %zu bytes < %zu needed", workspace_bytes,
                  need);
    }
    if (reinterpret_cast<uintptr_t>(workspace) % 16 != 0) {
      return fail(LLMOPT_ERR_INVALID_ARGUMENT, "workspace must be 16-byte aligned");
    }
    a.partial = static_cast<float*>(workspace);
  }
  cudaError_t e = quant_linear_launch(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "quant_linear launch");
  return ok();
}

int llmopt_dequantize(const void* qweight, int32_t bits, int32_t group_size, int32_t symmetric,
                      const float* scales, const float* zeros, int64_t n, int64_t k, void* out,
                      int32_t out_dtype, void* stream) {
  LLMOPT_RANGE("llmopt_dequantize");
  if (!valid_dtype(out_dtype)) return fail(LLMOPT_ERR_UNSUPPORTED, "unsupported dtype %d", out_dtype);
  QuantLinearArgs a{};
  int st = quant_args(qweight, bits, group_size, symmetric, scales, zeros, n, k, &a);
  if (st != LLMOPT_OK) return st;
  if (out == nullptr) return fail(LLMOPT_ERR_INVALID_ARGUMENT, "null pointer argument");
  cudaError_t e = dequantize_launch(a, out, out_dtype, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dequantize launch");
  return ok();
}

int llmopt_quant_linear_device_errors(int32_t clear, uint32_t* bits) {
  if (bits == nullptr) return fail(LLMOPT_ERR_INVALID_ARGUMENT, "bits is null");
  unsigned v = 0u;
  cudaError_t e = quant_linear_device_errors(&v, clear != 0);
  if (e != cudaSuccess) return cuda_fail(e, "quant_linear device errors");
  *bits = v;
  return ok();
}

int llmopt_merge_states(const void* o1, const void* o2, const void* l1, const void* l2,
                        void* out, void* lse_out, int64_t rows, int32_t head_dim,
                        int32_t o_dtype, int32_t lse_dtype, void* stream) {
  LLMOPT_RANGE("llmopt_merge_states");
  if (!valid_dtype(o_dtype) || !valid_dtype(lse_dtype)) {
    return fail(LLMOPT_ERR_UNSUPPORTED, "unsupported dtype");
  }
  if (rows < 0 || head_dim < 0) return fail(LLMOPT_ERR_INVALID_ARGUMENT, "invalid shape");
  if (rows == 0 || head_dim == 0) return ok();
  if (!o1 || !o2 || !l1 || !l2 || !out) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "null pointer argument");
  }
  cudaError_t e = merge_states_launch(o1, o2, l1, l2, out, lse_out, rows, head_dim, o_dtype,
                                      lse_dtype, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    return e == cudaErrorInvalidValue
               ? fail(LLMOPT_ERR_UNSUPPORTED, "unsupported dtype pair (o=%d lse=%d)", o_dtype,
                      lse_dtype)
               : cuda_fail(e, "merge_states launch");
  }
  return ok();
}

static int check_cache_args(int kv_dtype, int num_layers, int num_blocks, int block_size,
                            int num_kv_heads, int head_dim, int layer_idx, int64_t table_width,
                            int64_t table_stride) {
  if (!valid_dtype(kv_dtype)) return fail(LLMOPT_ERR_UNSUPPORTED, "unsupported cache dtype");
  if (num_layers < 1 || num_blocks < 1 || block_size < 1 || num_kv_heads < 1 || head_dim < 1 ||
      table_width < 0) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "invalid cache shape");
  }
  if (layer_idx < 0 || layer_idx >= num_layers) {
    return fail(LLMOPT_ERR_INDEX, "layer_idx %d out of range [0, %d)", layer_idx, num_layers);
  }
  if (table_width > 0 && table_stride < table_width) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "table_stride < table_width");
  }
  return LLMOPT_OK;
}

static int vector_width(const void* src_k, const void* src_v, int in_dtype, const void* k_cache,
                        const void* v_cache, int head_dim, std::initializer_list<int64_t> strides) {
  (void)in_dtype;
  if (head_dim % 8 != 0) return 1;
  for (const void* p : {src_k, src_v, k_cache, v_cache}) {
    if (reinterpret_cast<uintptr_t>(p) % 16 != 0) return 1;
  }
  for (int64_t s : strides) {
    if (s % 8 != 0) return 1;
  }
  return 8;
}

static int kv_write_impl(const void* keys, const void* values, int32_t in_dtype, int64_t k_s,
                         int64_t k_t, int64_t k_h, int64_t v_s, int64_t v_t, int64_t v_h,
                         void* key_cache, void* value_cache, int32_t kv_dtype, float* key_scale,
                         float* value_scale, int32_t num_layers, int32_t num_blocks,
                         int32_t block_size, int32_t num_kv_heads, int32_t head_dim,
                         int32_t layer_idx, const void* block_table, int32_t table_is_i64,
                         int64_t table_width, int64_t table_stride, const void* token_offsets,
                         int32_t off_is_i64, int64_t batch, int32_t q_len, uint32_t* err,
                         void* stream) {
  if (!valid_dtype(in_dtype)) return fail(LLMOPT_ERR_UNSUPPORTED, "unsupported input dtype");
  int st = check_cache_args(kv_dtype == kE4M3 ? kF32 : kv_dtype, num_layers, num_blocks,
                            block_size, num_kv_heads, head_dim, layer_idx, table_width,
                            table_stride);
  if (st != LLMOPT_OK) return st;
  if (batch < 0 || q_len < 0) return fail(LLMOPT_ERR_INVALID_ARGUMENT, "invalid shape");
  if (batch == 0 || q_len == 0) return ok();
  if (!keys || !values || !key_cache || !value_cache || !token_offsets ||
      (!block_table && table_width > 0)) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "null pointer argument");
  }
  KvWriteArgs a{};
  a.keys = keys;
  a.values = values;
  a.in_dtype = in_dtype;
  a.k_s = k_s;
  a.k_t = k_t;
  a.k_h = k_h;
  a.v_s = v_s;
  a.v_t = v_t;
  a.v_h = v_h;
  a.k_cache = key_cache;
  a.v_cache = value_cache;
  a.kv_dtype = kv_dtype;
  a.num_layers = num_layers;
  a.num_blocks = num_blocks;
  a.block_size = block_size;
  a.kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.layer = layer_idx;
  a.table = block_table;
  a.table_i64 = table_is_i64 ? 1 : 0;
  a.table_width = table_width;
  a.table_stride = table_stride;
  a.offsets = token_offsets;
  a.off_i64 = off_is_i64 ? 1 : 0;
  a.batch = batch;
  a.q_len = q_len;
  a.err = err;
  a.k_scale = key_scale;
  a.v_scale = value_scale;
  a.vec = vector_width(keys, values, in_dtype, key_cache, value_cache, head_dim,
                       {k_s, k_t, k_h, v_s, v_t, v_h});
  if (table_width == 0) return ok();  // every walk ends before its first column
  cudaError_t e = kv_write_launch(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "kv_write launch");
  return ok();
}

// Arguments every e4m3 entry point checks.
static int check_e4m3(int32_t kv_dtype, const void* key_scale, const void* value_scale,
                      int32_t head_dim) {
  if (kv_dtype != kE4M3) return fail(LLMOPT_ERR_UNSUPPORTED, "scaled entry points take e4m3 caches");
  if (key_scale == nullptr || value_scale == nullptr) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "null scale array");
  }
  if (head_dim > 256) return fail(LLMOPT_ERR_UNSUPPORTED, "e4m3 caches need head_dim <= 256");
  return LLMOPT_OK;
}

int llmopt_kv_write(const void* keys, const void* values, int32_t in_dtype, int64_t k_s,
                    int64_t k_t, int64_t k_h, int64_t v_s, int64_t v_t, int64_t v_h,
                    void* key_cache, void* value_cache, int32_t kv_dtype, int32_t num_layers,
                    int32_t num_blocks, int32_t block_size, int32_t num_kv_heads,
                    int32_t head_dim, int32_t layer_idx, const void* block_table,
                    int32_t table_is_i64, int64_t table_width, int64_t table_stride,
                    const void* token_offsets, int32_t off_is_i64, int64_t batch, int32_t q_len,
                    uint32_t* err, void* stream) {
  LLMOPT_RANGE("llmopt_kv_write");
  if (!valid_dtype(kv_dtype)) return fail(LLMOPT_ERR_UNSUPPORTED, "unsupported cache dtype");
  return kv_write_impl(keys, values, in_dtype, k_s, k_t, k_h, v_s, v_t, v_h, key_cache,
                       value_cache, kv_dtype, nullptr, nullptr, num_layers, num_blocks,
                       block_size, num_kv_heads, head_dim, layer_idx, block_table, table_is_i64,
                       table_width, table_stride, token_offsets, off_is_i64, batch, q_len, err,
                       stream);
}

int llmopt_kv_write_scaled(const void* keys, const void* values, int32_t in_dtype, int64_t k_s,
                           int64_t k_t, int64_t k_h, int64_t v_s, int64_t v_t, int64_t v_h,
                           void* key_cache, void* value_cache, int32_t kv_dtype,
                           float* key_scale, float* value_scale, int32_t num_layers,
                           int32_t num_blocks, int32_t block_size, int32_t num_kv_heads,
                           int32_t head_dim, int32_t layer_idx, const void* block_table,
                           int32_t table_is_i64, int64_t table_width, int64_t table_stride,
                           const void* token_offsets, int32_t off_is_i64, int64_t batch,
                           int32_t q_len, uint32_t* err, void* stream) {
  LLMOPT_RANGE("llmopt_kv_write_scaled");
  const int st = check_e4m3(kv_dtype, key_scale, value_scale, head_dim);
  if (st != LLMOPT_OK) return st;
  return kv_write_impl(keys, values, in_dtype, k_s, k_t, k_h, v_s, v_t, v_h, key_cache,
                       value_cache, kv_dtype, key_scale, value_scale, num_layers, num_blocks,
                       block_size, num_kv_heads, head_dim, layer_idx, block_table, table_is_i64,
                       table_width, table_stride, token_offsets, off_is_i64, batch, q_len, err,
                       stream);
}

static int kv_write_decode_impl(const void* keys, const void* values, int32_t in_dtype,
                                int64_t k_s, int64_t k_h, int64_t v_s, int64_t v_h,
                                void* key_cache, void* value_cache, int32_t kv_dtype,
                                float* key_scale, float* value_scale, int32_t num_layers,
                                int32_t num_blocks, int32_t block_size, int32_t num_kv_heads,
                                int32_t head_dim, int32_t layer_idx, const void* block_table,
                                int32_t table_is_i64, int64_t table_width, int64_t table_stride,
                                const void* token_offsets, int32_t off_is_i64, int64_t batch,
                                uint32_t* err, void* stream) {
  if (!valid_dtype(in_dtype)) return fail(LLMOPT_ERR_UNSUPPORTED, "unsupported input dtype");
  int st = check_cache_args(kv_dtype == kE4M3 ? kF32 : kv_dtype, num_layers, num_blocks,
                            block_size, num_kv_heads, head_dim, layer_idx, table_width,
                            table_stride);
  if (st != LLMOPT_OK) return st;
  if (batch < 0) return fail(LLMOPT_ERR_INVALID_ARGUMENT, "invalid shape");
  if (batch == 0) return ok();
  if (table_width == 0) return fail(LLMOPT_ERR_INDEX, "empty block table");
  if (!keys || !values || !key_cache || !value_cache || !token_offsets || !block_table) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "null pointer argument");
  }
  KvWriteArgs a{};
  a.keys = keys;
  a.values = values;
  a.in_dtype = in_dtype;
  a.k_s = k_s;
  a.k_t = 0;
  a.k_h = k_h;
  a.v_s = v_s;
  a.v_t = 0;
  a.v_h = v_h;
  a.k_cache = key_cache;
  a.v_cache = value_cache;
  a.kv_dtype = kv_dtype;
  a.num_layers = num_layers;
  a.num_blocks = num_blocks;
  a.block_size = block_size;
  a.kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.layer = layer_idx;
  a.table = block_table;
  a.table_i64 = table_is_i64 ? 1 : 0;
  a.table_width = table_width;
  a.table_stride = table_stride;
  a.offsets = token_offsets;
  a.off_i64 = off_is_i64 ? 1 : 0;
  a.batch = batch;
  a.q_len = 1;
  a.err = err;
  a.k_scale = key_scale;
  a.v_scale = value_scale;
  a.vec = vector_width(keys, values, in_dtype, key_cache, value_cache, head_dim,
                       {k_s, k_h, v_s, v_h});
  cudaError_t e = kv_write_decode_launch(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "kv_write_decode launch");
  return ok();
}

int llmopt_kv_write_decode(const void* keys, const void* values, int32_t in_dtype, int64_t k_s,
                           int64_t k_h, int64_t v_s, int64_t v_h, void* key_cache,
                           void* value_cache, int32_t kv_dtype, int32_t num_layers,
                           int32_t num_blocks, int32_t block_size, int32_t num_kv_heads,
                           int32_t head_dim, int32_t layer_idx, const void* block_table,
                           int32_t table_is_i64, int64_t table_width, int64_t table_stride,
                           const void* token_offsets, int32_t off_is_i64, int64_t batch,
                           uint32_t* err, void* stream) {
  LLMOPT_RANGE("llmopt_kv_write_decode");
  if (!valid_dtype(kv_dtype)) return fail(LLMOPT_ERR_UNSUPPORTED, "unsupported cache dtype");
  return kv_write_decode_impl(keys, values, in_dtype, k_s, k_h, v_s, v_h, key_cache, value_cache,
                              kv_dtype, nullptr, nullptr, num_layers, num_blocks, block_size,
                              num_kv_heads, head_dim, layer_idx, block_table, table_is_i64,
                              table_width, table_stride, token_offsets, off_is_i64, batch, err,
                              stream);
}

int llmopt_kv_write_decode_scaled(const void* keys, const void* values, int32_t in_dtype,
                                  int64_t k_s, int64_t k_h, int64_t v_s, int64_t v_h,
                                  void* key_cache, void* value_cache, int32_t kv_dtype,
                                  float* key_scale, float* value_scale, int32_t num_layers,
                                  int32_t num_blocks, int32_t block_size, int32_t num_kv_heads,
                                  int32_t head_dim, int32_t layer_idx, const void* block_table,
                                  int32_t table_is_i64, int64_t table_width,
                                  int64_t table_stride, const void* token_offsets,
                                  int32_t off_is_i64, int64_t batch, uint32_t* err,
                                  void* stream) {
  LLMOPT_RANGE("llmopt_kv_write_decode_scaled");
  const int st = check_e4m3(kv_dtype, key_scale, value_scale, head_dim);
  if (st != LLMOPT_OK) return st;
  return kv_write_decode_impl(keys, values, in_dtype, k_s, k_h, v_s, v_h, key_cache, value_cache,
                              kv_dtype, key_scale, value_scale, num_layers, num_blocks,
                              block_size, num_kv_heads, head_dim, layer_idx, block_table,
                              table_is_i64, table_width, table_stride, token_offsets, off_is_i64,
                              batch, err, stream);
}

static int gather_impl(const void* key_cache, const void* value_cache, int32_t kv_dtype,
                       const float* key_scale, const float* value_scale, int32_t num_layers,
                       int32_t num_blocks, int32_t block_size, int32_t num_kv_heads,
                       int32_t head_dim, int32_t layer_idx, const void* block_table,
                       int32_t table_is_i64, int64_t table_width, int64_t table_stride,
                       const void* context_lens, int32_t ctx_is_i64, int64_t batch,
                       int64_t max_len, void* out_keys, void* out_values, uint8_t* valid,
                       uint32_t* err, void* stream) {
  int st = check_cache_args(kv_dtype == kE4M3 ? kF32 : kv_dtype, num_layers, num_blocks,
                            block_size, num_kv_heads, head_dim, layer_idx, table_width,
                            table_stride);
  if (st != LLMOPT_OK) return st;
  if (batch < 0 || max_len < 0) return fail(LLMOPT_ERR_INVALID_ARGUMENT, "invalid shape");
  if (batch == 0 || max_len == 0) return ok();
  if (max_len > table_width * (int64_t)block_size) {
    return fail(LLMOPT_ERR_INDEX, "max_len %lld exceeds table width %lld x block_size %d",
                (long long)max_len, (long long)table_width, block_size);
  }
  if (!key_cache || !value_cache || !block_table || !context_lens || !out_keys || !out_values ||
      !valid) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "null pointer argument");
  }
  GatherArgs a{};
  a.k_cache = key_cache;
  a.v_cache = value_cache;
  a.kv_dtype = kv_dtype;
  a.num_layers = num_layers;
  a.num_blocks = num_blocks;
  a.block_size = block_size;
  a.kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.layer = layer_idx;
  a.table = block_table;
  a.table_i64 = table_is_i64 ? 1 : 0;
  a.table_width = table_width;
  a.table_stride = table_stride;
  a.ctx = context_lens;
  a.ctx_i64 = ctx_is_i64 ? 1 : 0;
  a.batch = batch;
  a.max_len = max_len;
  a.out_k = out_keys;
  a.out_v = out_values;
  a.valid = valid;
  a.err = err;
  a.k_scale = key_scale;
  a.v_scale = value_scale;
  cudaError_t e = gather_launch(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gather launch");
  return ok();
}

int llmopt_paged_gather(const void* key_cache, const void* value_cache, int32_t kv_dtype,
                        int32_t num_layers, int32_t num_blocks, int32_t block_size,
                        int32_t num_kv_heads, int32_t head_dim, int32_t layer_idx,
                        const void* block_table, int32_t table_is_i64, int64_t table_width,
                        int64_t table_stride, const void* context_lens, int32_t ctx_is_i64,
                        int64_t batch, int64_t max_len, void* out_keys, void* out_values,
                        uint8_t* valid, uint32_t* err, void* stream) {
  LLMOPT_RANGE("llmopt_paged_gather");
  if (!valid_dtype(kv_dtype)) return fail(LLMOPT_ERR_UNSUPPORTED, "unsupported cache dtype");
  return gather_impl(key_cache, value_cache, kv_dtype, nullptr, nullptr, num_layers, num_blocks,
                     block_size, num_kv_heads, head_dim, layer_idx, block_table, table_is_i64,
                     table_width, table_stride, context_lens, ctx_is_i64, batch, max_len,
                     out_keys, out_values, valid, err, stream);
}

int llmopt_paged_gather_scaled(const void* key_cache, const void* value_cache, int32_t kv_dtype,
                               const float* key_scale, const float* value_scale,
                               int32_t num_layers, int32_t num_blocks, int32_t block_size,
                               int32_t num_kv_heads, int32_t head_dim, int32_t layer_idx,
                               const void* block_table, int32_t table_is_i64,
                               int64_t table_width, int64_t table_stride,
                               const void* context_lens, int32_t ctx_is_i64, int64_t batch,
                               int64_t max_len, float* out_keys, float* out_values,
                               uint8_t* valid, uint32_t* err, void* stream) {
  LLMOPT_RANGE("llmopt_paged_gather_scaled");
  const int st = check_e4m3(kv_dtype, key_scale, value_scale, head_dim);
  if (st != LLMOPT_OK) return st;
  return gather_impl(key_cache, value_cache, kv_dtype, key_scale, value_scale, num_layers,
                     num_blocks, block_size, num_kv_heads, head_dim, layer_idx, block_table,
                     table_is_i64, table_width, table_stride, context_lens, ctx_is_i64, batch,
                     max_len, out_keys, out_values, valid, err, stream);
}

}  // extern "C"


extern "C" int llmopt_rope_kv_append(
    const void* q_proj, const void* k_proj, const void* v_proj, int32_t in_dtype, int64_t q_row,
    int64_t k_row, int64_t v_row, const void* positions, int32_t pos_is_i64,
    const void* cos_table, const void* sin_table, int32_t table_dtype, int64_t max_positions,
    void* q_out, int64_t qo_s, int64_t qo_h, int64_t qo_t, void* key_cache, void* value_cache,
    int32_t kv_dtype, int32_t num_layers, int32_t num_blocks, int32_t block_size,
    int32_t num_kv_heads, int32_t head_dim, int32_t layer_idx, const void* block_table,
    int32_t table_is_i64, int64_t table_width, int64_t table_stride, const void* token_offsets,
    int32_t off_is_i64, int64_t batch, int32_t num_heads, int32_t q_len, uint32_t* err,
    void* stream) {
  LLMOPT_RANGE("llmopt_rope_kv_append");
  if (!valid_dtype(in_dtype) || !valid_dtype(table_dtype)) {
    return fail(LLMOPT_ERR_UNSUPPORTED, "unsupported input or table dtype");
  }
  int st = check_cache_args(kv_dtype, num_layers, num_blocks, block_size, num_kv_heads, head_dim,
                            layer_idx, table_width, table_stride);
  if (st != LLMOPT_OK) return st;
  if (head_dim % 2 != 0) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "head_dim must be even for rotary embeddings");
  }
  if (num_heads < 1 || num_heads % num_kv_heads != 0) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "num_heads must be divisible by num_kv_heads");
  }
  if (batch < 0 || q_len < 0 || max_positions < 1) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "invalid shape");
  }
  if (batch == 0 || q_len == 0) return ok();
  if (table_width == 0) return fail(LLMOPT_ERR_INDEX, "empty block table");
  if (!q_proj || !k_proj || !v_proj || !positions || !cos_table || !sin_table || !q_out ||
      !key_cache || !value_cache || !block_table || !token_offsets) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "null pointer argument");
  }
  if (q_row < (int64_t)num_heads * head_dim || k_row < (int64_t)num_kv_heads * head_dim ||
      v_row < (int64_t)num_kv_heads * head_dim) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "projection row stride shorter than a row");
  }
  RopeArgs a{};
  a.q_in = q_proj;
  a.k_in = k_proj;
  a.v_in = v_proj;
  a.in_dtype = in_dtype;
  a.q_row = q_row;
  a.k_row = k_row;
  a.v_row = v_row;
  a.positions = positions;
  a.pos_i64 = pos_is_i64 ? 1 : 0;
  a.cos_t = cos_table;
  a.sin_t = sin_table;
  a.tab_dtype = table_dtype;
  a.max_pos = max_positions;
  a.q_out = q_out;
  a.qo_s = qo_s;
  a.qo_h = qo_h;
  a.qo_t = qo_t;
  a.k_cache = key_cache;
  a.v_cache = value_cache;
  a.kv_dtype = kv_dtype;
  a.num_layers = num_layers;
  a.num_blocks = num_blocks;
  a.block_size = block_size;
  a.kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.layer = layer_idx;
  a.table = block_table;
  a.table_i64 = table_is_i64 ? 1 : 0;
  a.table_width = table_width;
  a.table_stride = table_stride;
  a.offsets = token_offsets;
  a.off_i64 = off_is_i64 ? 1 : 0;
  a.batch = batch;
  a.num_heads = num_heads;
  a.q_len = q_len;
  a.err = err;
  // Paired accesses: 2 elements (4 bytes for 16-bit, 8 for fp32) at every
  // row start, pair offset and table row.
  {
    const int es = in_dtype == kF32 ? 4 : 2;
    const int ts = table_dtype == kF32 ? 4 : 2;
    auto al = [](const void* p, int n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; };
    const bool even = head_dim % 4 == 0 && q_row % 2 == 0 && k_row % 2 == 0 && qo_s % 2 == 0 &&
                      qo_h % 2 == 0 && qo_t % 2 == 0;
    a.pairs = even && al(q_proj, 2 * es) && al(k_proj, 2 * es) && al(q_out, 2 * es) &&
              al(key_cache, 2 * (kv_dtype == kF32 ? 4 : 2)) && al(cos_table, 2 * ts) &&
              al(sin_table, 2 * ts) ? 1 : 0;
    const int per = kv_dtype == kF32 ? 4 : 8;
    a.vrow16 = in_dtype == kv_dtype && head_dim % per == 0 && v_row % per == 0 &&
               al(v_proj, 16) && al(value_cache, 16) ? 1 : 0;
  }
  cudaError_t e = rope_append_launch(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rope_append launch");
  return ok();
}

extern "C" int llmopt_decode_step_advance(const int64_t* updates, int64_t capacity,
                                          int32_t* block_table, int64_t table_width,
                                          int64_t table_stride, int64_t* context_lens,
                                          int64_t* token_offsets, int64_t* positions,
                                          int64_t max_rows, int64_t batch, uint32_t* err,
                                          void* stream) {
  LLMOPT_RANGE("llmopt_decode_step_advance");
  if (capacity < 0 || table_width < 1 || table_stride < table_width || max_rows < 1 ||
      batch < 0 || batch > max_rows) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "invalid step-state shape");
  }
  if (!updates || !block_table || !context_lens || !token_offsets || !positions) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "null pointer argument");
  }
  StepArgs a{};
  a.updates = reinterpret_cast<const long long*>(updates);
  a.capacity = capacity;
  a.table = block_table;
  a.table_width = table_width;
  a.table_stride = table_stride;
  a.ctx = reinterpret_cast<long long*>(context_lens);
  a.offsets = reinterpret_cast<long long*>(token_offsets);
  a.positions = reinterpret_cast<long long*>(positions);
  a.max_rows = max_rows;
  a.batch = batch;
  a.err = err;
  cudaError_t e = step_advance_launch(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "step_advance launch");
  return ok();
}
// ---------------------------------------------------------------------------
// llmopt_paged_attention_noalloc: paged attention whose split-K scratch is a
// fixed array compiled into this library instead of caller-provided memory.
//
// It exists for callers that cannot allocate device memory at the point where
// they run attention: serving processes that hand nearly all HBM to the KV
// block pool at start-up (llmopt sizes the pool from gpu_memory_utilization)
// and forbid allocations afterwards, and foreign-language hosts (C, Go, Java
// through this C ABI) that have no device allocator of their own to carve a
// workspace from.  The caller still passes every input and output.
//
// The scratch lives in device global memory: LLMOPT_NOALLOC_SCRATCH_BYTES per
// GPU, held by every GPU that loads this code until the process exits.  Host
// code must not use the array's name as a device address (in host code it is
// only a stand-in); the address is looked up with cudaGetSymbolAddress, with
// the device current, by the first call in each CUDA context (a device's
// primary context, a context that replaced it after cudaDeviceReset, or a
// caller's own context) - so make the first call on each device before any
// stream capture.
// Every call on a device shares the one array and it keeps whatever the last
// call left there: calls that can overlap on the GPU (different streams, or
// several host threads) race on it and must be serialised by the caller.
// Nothing in it has to start at zero: each call writes every scratch byte it
// later reads.  Shapes whose scratch would exceed the array are rejected with
// LLMOPT_ERR_WORKSPACE before anything is launched.  No cudaMalloc, cudaFree
// or other allocating routine is called.
// ---------------------------------------------------------------------------
namespace {

constexpr int kNoAllocMaxContexts = 64;
static __device__ __align__(256) unsigned char g_noalloc_scratch[LLMOPT_NOALLOC_SCRATCH_BYTES];
std::mutex g_noalloc_mu;
// (context id, device address of g_noalloc_scratch in that context)
unsigned long long g_noalloc_ctx[kNoAllocMaxContexts] = {};
void* g_noalloc_addr[kNoAllocMaxContexts] = {};
int g_noalloc_used = 0;

// The unique id (cuCtxGetId) of the calling thread's current CUDA context, or
// 0 when no context is current or the driver does not expose the call.  Unlike
// a device ordinal, an id is never reused: a context that replaced another
// (after cudaDeviceReset, or a caller's own non-primary context) gets its own.
unsigned long long current_context_id() {
  static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
  static PFN_cuCtxGetId_v12000 get_id = nullptr;
  static bool resolved = false;
  if (!resolved) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    }
    p = nullptr;
    q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
    }
    resolved = true;
  }
  if (get_current == nullptr || get_id == nullptr) return 0;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  unsigned long long id = 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of g_noalloc_scratch in the current context.  Looked up with
// cudaGetSymbolAddress (which allocates nothing) on the first call in each
// context and remembered by context id; without an id it is looked up on every
// call.
int noalloc_scratch(void** addr) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  unsigned long long id = current_context_id();
  for (int i = 0; id != 0 && i < g_noalloc_used; ++i) {
    if (g_noalloc_ctx[i] == id) {
      *addr = g_noalloc_addr[i];
      return LLMOPT_OK;
    }
  }
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr) {
    return cuda_fail(e == cudaSuccess ? cudaErrorInvalidSymbol : e,
                     "cudaGetSymbolAddress(scratch)");
  }
  if (id == 0) id = current_context_id();  // the lookup made the primary context current
  if (id != 0 && g_noalloc_used < kNoAllocMaxContexts) {
    g_noalloc_ctx[g_noalloc_used] = id;
    g_noalloc_addr[g_noalloc_used] = p;
    ++g_noalloc_used;
  }
  *addr = p;
  return LLMOPT_OK;
}

}  // namespace

extern "C" int llmopt_paged_attention_noalloc(
    const void* query, int32_t q_dtype, int64_t q_s, int64_t q_h, int64_t q_t,
    const void* key_cache, const void* value_cache, int32_t kv_dtype, int32_t num_layers,
    int32_t num_blocks, int32_t block_size, int32_t num_kv_heads, int32_t head_dim,
    int32_t layer_idx, const void* block_table, int32_t table_is_i64, int64_t table_width,
    int64_t table_stride, const void* context_lens, int32_t ctx_is_i64, void* out,
    int32_t out_dtype, int64_t o_s, int64_t o_h, int64_t o_t, float* lse, int64_t batch,
    int32_t num_heads, int32_t q_len, float scale, float softcap, int64_t split_tokens,
    uint32_t* err, void* stream) {
  LLMOPT_RANGE("llmopt_paged_attention_noalloc");
  if (batch <= 0 || q_len <= 0) {
    // Nothing to launch; the regular entry validates the remaining arguments.
    return llmopt_paged_attention(query, q_dtype, q_s, q_h, q_t, key_cache, value_cache,
                                  kv_dtype, num_layers, num_blocks, block_size, num_kv_heads,
                                  head_dim, layer_idx, block_table, table_is_i64, table_width,
                                  table_stride, context_lens, ctx_is_i64, out, out_dtype, o_s,
                                  o_h, o_t, lse, batch, num_heads, q_len, scale, softcap,
                                  split_tokens, nullptr, 0, err, stream);
  }
  if (num_heads < 1 || num_kv_heads < 1 || num_heads % num_kv_heads != 0 || head_dim < 1 ||
      block_size < 1 || table_width < 0) {
    return fail(LLMOPT_ERR_INVALID_ARGUMENT, "invalid shape");
  }
  if (!valid_dtype(q_dtype) || !valid_dtype(kv_dtype) || !valid_dtype(out_dtype)) {
    return fail(LLMOPT_ERR_UNSUPPORTED, "unsupported dtype (q=%d kv=%d out=%d)", q_dtype,
                kv_dtype, out_dtype);
  }
  // Size the scratch for the plan the regular entry will pick, and refuse
  // shapes that do not fit before anything is launched.
  AttnArgs a{};
  a.q = query;
  a.q_s = q_s;
  a.q_h = q_h;
  a.q_t = q_t;
  a.q_dtype = q_dtype;
  a.k_cache = key_cache;
  a.v_cache = value_cache;
  a.kv_dtype = kv_dtype;
  a.num_layers = num_layers;
  a.num_blocks = num_blocks;
  a.block_size = block_size;
  a.kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.table_width = table_width;
  a.batch = batch;
  a.num_heads = num_heads;
  a.q_len = q_len;
  a.group = num_heads / num_kv_heads;
  a.rows = q_len * a.group;
  a.table = block_table;
  a.table_i64 = table_is_i64;
  a.table_stride = table_stride;
  a.ctx = context_lens;
  a.ctx_i64 = ctx_is_i64;
  const int device = current_device();
  // The same plan the regular entry picks, tensor maps included (a shape whose
  // maps cannot be encoded falls back to a plan that may need more scratch).
  Choice c;
  int st = choose(a, split_tokens, device, true, &c);
  if (st != LLMOPT_OK) return st;
  const long long need = layout_for(batch, c.plan.slots, num_heads, q_len, head_dim).total;
  if (need > (long long)LLMOPT_NOALLOC_SCRATCH_BYTES) {
    return fail(LLMOPT_ERR_WORKSPACE,
                "llmopt_paged_attention_noalloc: this shape needs %lld bytes of split-K scratch "
                "but the built-in scratch holds %lld; use llmopt_paged_attention with a "
                "caller-provided workspace, or fewer sequences/splits per call",
                need, (long long)LLMOPT_NOALLOC_SCRATCH_BYTES);
  }
  void* scratch = nullptr;
  st = noalloc_scratch(&scratch);
  if (st != LLMOPT_OK) return st;
  return llmopt_paged_attention(query, q_dtype, q_s, q_h, q_t, key_cache, value_cache, kv_dtype,
                                num_layers, num_blocks, block_size, num_kv_heads, head_dim,
                                layer_idx, block_table, table_is_i64, table_width, table_stride,
                                context_lens, ctx_is_i64, out, out_dtype, o_s, o_h, o_t, lse,
                                batch, num_heads, q_len, scale, softcap, split_tokens, scratch,
                                (size_t)LLMOPT_NOALLOC_SCRATCH_BYTES, err, stream);
}
