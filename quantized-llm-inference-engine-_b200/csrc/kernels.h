// Internal launch interface between the C ABI (capi.cu) and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "plan.cuh"

namespace llmopt {

// cudaLaunchKernel with programmatic stream serialization, so the launch of a
// kernel overlaps the tail of the previous one (each kernel starts with
// griddepcontrol.wait).  LLMOPT_B200_PDL=0 turns it off.
// Sets the largest shared-memory carveout on `fn` (once per device).
cudaError_t ensure_max_shared_carveout(const void* fn);
cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, void** args, size_t smem,
                       cudaStream_t stream);

// Everything the attention kernels read, in one POD passed by value.
struct AttnArgs {
  // query [batch, num_heads, q_len, head_dim]
  const void* q;
  long long q_s, q_h, q_t;
  int q_dtype;
  // cache [layers, num_blocks, block_size, kv_heads, head_dim]
  const void* k_cache;
  const void* v_cache;
  int kv_dtype;
  int num_layers, num_blocks, block_size, kv_heads, head_dim, layer;
  // kE4M3 caches: fp32 scale per (token, head) row, [layers, num_blocks, kv_heads, block_size]
  const float* k_scale;
  const float* v_scale;
  // block table / context
  const void* table;
  int table_i64;
  long long table_width, table_stride;
  const void* ctx;
  int ctx_i64;
  // shape
  long long batch;
  int num_heads, q_len, group, rows;  // rows = q_len * group (query rows per KV head)
  float scale, softcap;
  // partition + workspace
  SplitPlan plan;
  int* prefix;        // [batch + 1] block prefix sums (balanced mode)
  float* part_lse;    // [slots, num_heads, q_len]
  float* part_o;      // [slots, num_heads, q_len, head_dim]
  // output
  void* out;
  int out_dtype;
  long long o_s, o_h, o_t;
  float* lse;         // optional [batch, num_heads, q_len]
  unsigned* err;
};

// Fast decode path: TMA-staged blocks + m16n8k16 tensor-core tiles.
struct DecodeLaunch {
  int heads_per_cta;  // KV heads one CTA stages per block (box height)
  int self_issue;     // 1: one-warp CTAs that issue their own copies (heads_per_cta == 1)
  int streams;        // 2: two balanced ranges of one head per CTA (plan.ctas counts ranges)
  int stages;         // shared-memory ring depth
  int ctas_per_sm;
  size_t smem_bytes;
};

bool decode_tma_supported(const AttnArgs& a);
// Fills `launch` (occupancy, smem) for this shape; false if it cannot run here.
bool decode_tma_configure(const AttnArgs& a, int sm_count, DecodeLaunch* launch);
cudaError_t decode_tma_launch(const AttnArgs& a, const DecodeLaunch& launch,
                              const CUtensorMap& tmk, const CUtensorMap& tmv,
                              cudaStream_t stream);

// The same split-K decode over an e4m3 cache (decode_fp8.cu): TMA-staged code
// blocks and scales, dequantised in registers into f16 m16n8k16 tiles.
bool decode_fp8_supported(const AttnArgs& a);
bool decode_fp8_configure(const AttnArgs& a, int sm_count, DecodeLaunch* launch);
cudaError_t decode_fp8_launch(const AttnArgs& a, const DecodeLaunch& launch,
                              const CUtensorMap& tmk, const CUtensorMap& tmv,
                              cudaStream_t stream);

// Chunked prefill on tcgen05 tensor cores (q_len * group > 16, 16-bit cache and
// query of the same dtype, head_dim 64/128, block_size 16).  Writes the final
// output and LSE itself: no split partials, no combine.
bool prefill_tc_supported(const AttnArgs& a);
cudaError_t prefill_tc_launch(const AttnArgs& a, const CUtensorMap& tmq, const CUtensorMap& tmk,
                              const CUtensorMap& tmv, cudaStream_t stream);
constexpr int kPrefillRows = 128;  // query rows per prefill query tile
// The same shapes on the two-query-tile ping-pong kernel (prefill_fa.cu), which
// prefill_tc_launch uses when LLMOPT_B200_PREFILL=fa.
bool prefill_fa_enabled();
bool prefill_fa_usable(const AttnArgs& a);
cudaError_t prefill_fa_launch(const AttnArgs& a, const CUtensorMap& tmq, const CUtensorMap& tmk,
                              const CUtensorMap& tmv, cudaStream_t stream);
// head_dim 128 on 2-SM tensor-core pairs (prefill_pair.cu), which
// prefill_tc_launch uses for those shapes unless LLMOPT_B200_PREFILL names
// another kernel (tc or fa).
bool prefill_pair_enabled();
bool prefill_pair_usable(const AttnArgs& a);
cudaError_t prefill_pair_launch(const AttnArgs& a, const CUtensorMap& tmq,
                                const CUtensorMap& tmk, const CUtensorMap& tmv,
                                cudaStream_t stream);

// Generic path: any dtype / head_dim <= 256 / block size / q_len (CUDA cores).
constexpr int kGenericRowTile = 16;
constexpr int kGenericKeyTile = 32;
bool generic_supported(const AttnArgs& a);
cudaError_t generic_launch(const AttnArgs& a, cudaStream_t stream);

// Merge of split partials into the output (+ optional LSE).
cudaError_t combine_launch(const AttnArgs& a, cudaStream_t stream);

// Peers of a head-sharded group for the fused combine + all-gather.  Every
// rank's gathered output is [world * num_heads, batch, q_len, head_dim]
// (num_heads = this rank's heads); rank r owns heads [r*num_heads, (r+1)*num_heads).
constexpr int kMaxPeers = 8;
struct PeerArgs {
  void* out[kMaxPeers];          // each rank's gathered output (device pointers, peer-mapped)
  unsigned* flags[kMaxPeers];    // each rank's arrival flags: u32[kMaxPeers], slot = source rank
  unsigned* counter;             // this rank's CTA arrival counter (0 between calls)
  unsigned epoch;                // written to every peer's flag slot by this call
  int world;
  int rank;
};
// Combine that stores each merged row into every rank's gathered output over
// NVLink, then barriers with the peers through their flags (bounded wait).
cudaError_t combine_gather_launch(const AttnArgs& a, const PeerArgs& p, cudaStream_t stream);
// Copies this rank's slice of its gathered output (already written by a
// kernel that stores the output directly) to every peer, then the same barrier.
cudaError_t push_gather_launch(const AttnArgs& a, const PeerArgs& p, int elem_bytes,
                               cudaStream_t stream);

// merge_states
cudaError_t merge_states_launch(const void* o1, const void* o2, const void* l1, const void* l2,
                                void* out, void* lse_out, long long rows, int head_dim,
                                int o_dtype, int lse_dtype, cudaStream_t stream);

// KV cache writes and gather.
struct KvWriteArgs {
  const void* keys;
  const void* values;
  int in_dtype;
  long long k_s, k_t, k_h, v_s, v_t, v_h;
  void* k_cache;
  void* v_cache;
  int kv_dtype;
  int num_layers, num_blocks, block_size, kv_heads, head_dim, layer;
  float* k_scale;  // kE4M3: [layers, num_blocks, kv_heads, block_size]
  float* v_scale;
  const void* table;
  int table_i64;
  long long table_width, table_stride;
  const void* offsets;
  int off_i64;
  long long batch;
  int q_len;
  unsigned* err;
  int vec;  // elements per vector access (8 when every address allows 16-byte stores, else 1)
};

cudaError_t kv_write_launch(const KvWriteArgs& a, cudaStream_t stream);
cudaError_t kv_write_decode_launch(const KvWriteArgs& a, cudaStream_t stream);

// Rotary embedding of q and k fused with the K/V append (the attention layer's
// step before attention).
struct RopeArgs {
  const void* q_in;              // [tokens, heads * head_dim] rows, model dtype
  const void* k_in;              // [tokens, kv_heads * head_dim]
  const void* v_in;
  int in_dtype;
  long long q_row, k_row, v_row; // token-row strides (elements)
  const void* positions;         // [tokens] = [batch * q_len]
  int pos_i64;
  const void* cos_t;             // [max_pos, head_dim]
  const void* sin_t;
  int tab_dtype;
  long long max_pos;
  void* q_out;                   // rotated query, model dtype, strides (seq, head, token)
  long long qo_s, qo_h, qo_t;
  void* k_cache;
  void* v_cache;
  int kv_dtype;
  int num_layers, num_blocks, block_size, kv_heads, head_dim, layer;
  const void* table;
  int table_i64;
  long long table_width, table_stride;
  const void* offsets;
  int off_i64;
  long long batch;
  int num_heads;
  int q_len;
  unsigned* err;
  int pairs;   // 1: head_dim % 4 == 0 and every row/table address allows 2-element accesses
  int vrow16;  // 1: v rows move as 16-byte vectors (same dtype, 16-byte aligned rows)
};
cudaError_t rope_append_launch(const RopeArgs& a, cudaStream_t stream);

// Device-resident decode step metadata (step_state.cu).
struct StepArgs {
  const long long* updates;   // [1 + 4 * capacity]: count, then (op, row, a, b) records
  long long capacity;
  int* table;                 // [max_rows, table_stride] int32 block table
  long long table_width, table_stride;
  long long* ctx;             // [max_rows] context lengths (committed + this step)
  long long* offsets;         // [max_rows] write offsets of the step
  long long* positions;       // [max_rows] positions of the step (q_len 1)
  long long max_rows;
  long long batch;            // active rows [0, batch)
  unsigned* err;
};
cudaError_t step_advance_launch(const StepArgs& a, cudaStream_t stream);

// Weight-only quantized linear (quant_linear.cu): out = x W^T + bias with W as
// packed codes + per-group fp32 scales / zeros (the reference's QuantizedTensor).
struct QuantLinearArgs {
  const void* x;                   // [m, k] compute dtype, row stride ldx
  int x_dtype;
  long long m, ldx;
  const unsigned char* qweight;    // [n, k/2] (2/4-bit, nibbles) or [n, k] (8-bit)
  int bits, group, symmetric;
  const float* scales;             // [n, k / group]
  const float* zeros;
  long long n, k;
  const void* bias;                // [n] compute dtype, or null
  void* out;                       // [m, n] compute dtype, row stride ldo
  long long ldo;
  float* partial;                  // [splits, m, n] when the k range is split, else null
  int splits;
  long long k_per_split;           // multiple of 128
};
bool quant_linear_tc_supported(const QuantLinearArgs& a);
int quant_linear_splits(const QuantLinearArgs& a, int sm_count);
cudaError_t quant_linear_launch(const QuantLinearArgs& a, cudaStream_t stream);
// LLMOPT_DEVERR_* bits recorded by the quantized-linear kernels' bounded waits
// on the current device (read, and cleared when `clear`).
cudaError_t quant_linear_device_errors(unsigned* bits, bool clear);
// 2-D tensor map for TMA tile loads: `inner` elements per row (contiguous),
// `outer` rows `row_bytes` apart, boxes of box_inner x box_outer, 128-byte
// swizzle, zero fill outside the tensor.  False when the driver's encoder is
// unavailable or rejects the arguments.
bool tensor_map_2d(CUtensorMap* out, CUtensorMapDataType dtype, const void* base,
                   uint64_t inner, uint64_t outer, uint64_t row_bytes, uint32_t box_inner,
                   uint32_t box_outer);
cudaError_t dequantize_launch(const QuantLinearArgs& a, void* out, int out_dtype,
                              cudaStream_t stream);

struct GatherArgs {
  const void* k_cache;
  const void* v_cache;
  int kv_dtype;
  int num_layers, num_blocks, block_size, kv_heads, head_dim, layer;
  const float* k_scale;  // kE4M3: outputs are dequantised fp32
  const float* v_scale;
  const void* table;
  int table_i64;
  long long table_width, table_stride;
  const void* ctx;
  int ctx_i64;
  long long batch, max_len;
  void* out_k;
  void* out_v;
  unsigned char* valid;
  unsigned* err;
};
cudaError_t gather_launch(const GatherArgs& a, cudaStream_t stream);

}  // namespace llmopt
