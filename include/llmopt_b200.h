/*
 * llmopt_b200.h - C ABI of the B200-native paged-KV hot path.
 *
 * Every entry point takes plain device pointers, element strides and sizes,
 * plus the CUDA stream to launch on.  Nothing here allocates device memory:
 * split-K scratch ("workspace") is passed in by the caller, sized with
 * llmopt_paged_attention_workspace_size().  Functions never throw; they return
 * an llmopt_status and leave a human-readable message in llmopt_last_error()
 * (thread-local).  Kernels that find a bad index at run time (a block id
 * outside the pool, a context longer than its block-table row) skip the
 * access and OR a LLMOPT_DEVERR_* bit into the optional device word `err`.
 *
 * Cache layout (identical to the reference's PagedKVCache storage,
 * src/llmopt/cache/paged_cache.py:171-173): key_cache and value_cache are
 * contiguous [num_layers, num_blocks, block_size, num_kv_heads, head_dim].
 * Block tables are [batch, table_width] (int32 or int64, row stride
 * table_stride elements, -1 padded); context_lens / token_offsets are [batch]
 * (int32 or int64).
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   llmopt_paged_attention  <- PagedAttention.forward
 *                              src/llmopt/attention/paged_attention.py:146-187
 *   llmopt_merge_states     <- merge_states  paged_attention.py:30-55
 *   llmopt_kv_write         <- PagedKVCache.write  src/llmopt/cache/paged_cache.py:175-232
 *   llmopt_kv_write_decode  <- PagedKVCache.write_decode  paged_cache.py:234-261
 *   llmopt_paged_gather     <- PagedKVCache.gather  paged_cache.py:263-312
 *   llmopt_decode_step_advance <- ModelRunner._build_decode + _finalize
 *                              src/llmopt/engine/model_runner.py:169-230 (device-resident)
 *   llmopt_rope_kv_append   <- the rotary + append statements of
 *                              PagedAttentionLayer.forward  src/llmopt/model/layers.py:106-134
 *                              (RotaryEmbedding.forward, apply_rotary_pos_emb
 *                              src/llmopt/model/rotary.py:16-46, 103-121)
 *   llmopt_quant_linear     <- QuantLinear.forward  src/llmopt/quantization/quant_linear.py:93-113
 *   llmopt_dequantize       <- QuantizedTensor.dequantize / dequantize
 *                              src/llmopt/quantization/quantizers.py:203-239
 *   llmopt_*_scaled         <- the same operations on an FP8 (e4m3) cache; the
 *                              reference only names the float8 dtypes
 *                              (src/llmopt/utils/misc.py:33-34, 57) and has no
 *                              fp8 attention of its own.
 */
#ifndef LLMOPT_B200_H_
#define LLMOPT_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LLMOPT_API __attribute__((visibility("default")))
#else
#define LLMOPT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define LLMOPT_B200_ABI_VERSION 1

/* Element types (torch.float32 / float16 / bfloat16; float8_e4m3fn for
 * caches through the *_scaled entry points only). */
enum {
  LLMOPT_DTYPE_F32 = 0,
  LLMOPT_DTYPE_F16 = 1,
  LLMOPT_DTYPE_BF16 = 2,
  LLMOPT_DTYPE_E4M3 = 3
};

/* Return codes. The Python layer maps them to the reference's exception types. */
enum {
  LLMOPT_OK = 0,
  LLMOPT_ERR_INVALID_ARGUMENT = 1, /* ValueError */
  LLMOPT_ERR_UNSUPPORTED = 2,      /* ValueError: dtype/shape not supported   */
  LLMOPT_ERR_WORKSPACE = 3,        /* RuntimeError: workspace too small        */
  LLMOPT_ERR_CUDA = 4,             /* RuntimeError: CUDA launch/driver error   */
  LLMOPT_ERR_INDEX = 5             /* IndexError                               */
};

/* Bits a kernel ORs into the optional `err` word (uint32 in device memory). */
#define LLMOPT_DEVERR_BLOCK_ID 1u      /* block id >= num_blocks (access skipped)     */
#define LLMOPT_DEVERR_TABLE_WIDTH 2u   /* position beyond the block-table row         */
#define LLMOPT_DEVERR_WAIT_TIMEOUT 4u  /* a bounded on-device wait gave up            */
#define LLMOPT_DEVERR_POSITION 8u      /* rotary position outside the table (skipped)  */
/* Set together with LLMOPT_DEVERR_WAIT_TIMEOUT: which wait gave up. */
#define LLMOPT_DEVERR_WAIT_DATA 0x100u  /* a consumer waiting for a staged K/V tile     */
#define LLMOPT_DEVERR_WAIT_SLOT 0x200u  /* the copy issuer waiting for a free slot      */
#define LLMOPT_DEVERR_WAIT_DRAIN 0x400u /* the copy issuer waiting for its last copies  */
#define LLMOPT_DEVERR_WAIT_PEER 0x800u  /* the cross-rank barrier of a gathered call    */

/* split_tokens argument of the attention entry points. */
#define LLMOPT_SPLIT_AUTO 0LL  /* balanced split-K chosen from context and SM count */
#define LLMOPT_SPLIT_NONE (-1LL) /* one split per sequence (split_kv=False)        */
/* split_tokens > 0: each sequence cut into chunks of at most split_tokens
 * tokens, rounded up to whole blocks (PagedAttentionConfig.split_size). */

/* Library identification; callable without a GPU. */
LLMOPT_API const char* llmopt_b200_version(void);
LLMOPT_API int llmopt_b200_abi_version(void);
LLMOPT_API const char* llmopt_status_string(int status);
/* Message of the last failing call on this thread ("" if none). */
LLMOPT_API const char* llmopt_last_error(void);

/*
 * Bytes of split-K workspace llmopt_paged_attention needs for these shapes on
 * `device` (the CUDA ordinal).  Pass the same arguments as the call.
 */
LLMOPT_API int llmopt_paged_attention_workspace_size(int device, int64_t batch, int32_t num_heads,
                                          int32_t num_kv_heads, int32_t head_dim, int32_t q_len,
                                          int32_t block_size, int64_t table_width,
                                          int32_t kv_dtype, int64_t split_tokens,
                                          size_t* bytes);

/*
 * Paged attention over the block-addressed cache: decode (q_len == 1) and
 * chunked prefill (q_len > 1, causal within the chunk, full over the prefix:
 * query i of sequence s sits at position context_lens[s] - q_len + i).
 * Replaces PagedAttention.forward (paged_attention.py:146-187).
 *
 *   query  [batch, num_heads, q_len, head_dim], element strides (q_s, q_h, q_t),
 *          head_dim contiguous; rounded to the cache dtype before the dot
 *          products, as the reference's q.to(k.dtype).
 *   out    same shape, element strides (o_s, o_h, o_t), dtype out_dtype.
 *   lse    optional fp32 [batch, num_heads, q_len] contiguous: natural-log
 *          sum-exp of the masked, scaled (and soft-capped) scores; -inf for a
 *          fully masked row (whose output is 0, as the reference's nan_to_num).
 *   softcap > 0 applies tanh(s / softcap) * softcap after scaling.
 *   Query head h reads KV head h / (num_heads / num_kv_heads).
 */
LLMOPT_API int llmopt_paged_attention(const void* query, int32_t q_dtype, int64_t q_s, int64_t q_h,
                           int64_t q_t,
                           const void* key_cache, const void* value_cache, int32_t kv_dtype,
                           int32_t num_layers, int32_t num_blocks, int32_t block_size,
                           int32_t num_kv_heads, int32_t head_dim, int32_t layer_idx,
                           const void* block_table, int32_t table_is_i64, int64_t table_width,
                           int64_t table_stride,
                           const void* context_lens, int32_t ctx_is_i64,
                           void* out, int32_t out_dtype, int64_t o_s, int64_t o_h, int64_t o_t,
                           float* lse,
                           int64_t batch, int32_t num_heads, int32_t q_len, float scale,
                           float softcap, int64_t split_tokens,
                           void* workspace, size_t workspace_bytes, uint32_t* err,
                           void* stream);

/*
 * The two halves of llmopt_paged_attention, for callers that time or schedule
 * them separately: LLMOPT_PHASE_SPLIT runs the split-K attention kernel (its
 * partial states go to the workspace), LLMOPT_PHASE_COMBINE merges them into
 * out / lse.  Issue SPLIT then COMBINE on one stream with identical arguments
 * and workspace; LLMOPT_PHASE_ALL is llmopt_paged_attention itself.
 */
#define LLMOPT_PHASE_SPLIT 1
#define LLMOPT_PHASE_COMBINE 2
#define LLMOPT_PHASE_ALL 3
LLMOPT_API int llmopt_paged_attention_phase(const void* query, int32_t q_dtype, int64_t q_s,
                           int64_t q_h, int64_t q_t,
                           const void* key_cache, const void* value_cache, int32_t kv_dtype,
                           int32_t num_layers, int32_t num_blocks, int32_t block_size,
                           int32_t num_kv_heads, int32_t head_dim, int32_t layer_idx,
                           const void* block_table, int32_t table_is_i64, int64_t table_width,
                           int64_t table_stride,
                           const void* context_lens, int32_t ctx_is_i64,
                           void* out, int32_t out_dtype, int64_t o_s, int64_t o_h, int64_t o_t,
                           float* lse,
                           int64_t batch, int32_t num_heads, int32_t q_len, float scale,
                           float softcap, int64_t split_tokens,
                           void* workspace, size_t workspace_bytes, uint32_t* err,
                           void* stream, int32_t phases);

/*
 * llmopt_paged_attention without a workspace argument.  No counterpart in the
 * reference: it is an addition of this library for callers that cannot
 * allocate device memory where they run attention - serving processes that
 * give nearly all HBM to the KV block pool at start-up and may not allocate
 * afterwards, and hosts calling this C ABI from other languages with no device
 * allocator of their own.  Inputs and outputs are still the caller's.
 *
 * The split-K scratch is a fixed array of LLMOPT_NOALLOC_SCRATCH_BYTES compiled
 * into the library, held in device memory by every GPU that loads it until the
 * process exits.  The first call in each CUDA context looks up the array's
 * address there, with the device current, and keeps it by the context's unique
 * id, so a context that replaces another (after cudaDeviceReset, or a caller's
 * own non-primary context) gets its own lookup; make the first call on each
 * device before any stream capture.  All calls on
 * a device share the array and it keeps the last call's contents, so calls
 * that may overlap on the GPU (other streams, other threads) race and must be
 * serialised by the caller.  A shape needing more scratch than the array holds
 * returns LLMOPT_ERR_WORKSPACE without launching anything.  The function never
 * calls cudaMalloc, cudaFree or any other allocating routine.
 */
#define LLMOPT_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
LLMOPT_API int llmopt_paged_attention_noalloc(const void* query, int32_t q_dtype, int64_t q_s,
                           int64_t q_h, int64_t q_t,
                           const void* key_cache, const void* value_cache, int32_t kv_dtype,
                           int32_t num_layers, int32_t num_blocks, int32_t block_size,
                           int32_t num_kv_heads, int32_t head_dim, int32_t layer_idx,
                           const void* block_table, int32_t table_is_i64, int64_t table_width,
                           int64_t table_stride,
                           const void* context_lens, int32_t ctx_is_i64,
                           void* out, int32_t out_dtype, int64_t o_s, int64_t o_h, int64_t o_t,
                           float* lse,
                           int64_t batch, int32_t num_heads, int32_t q_len, float scale,
                           float softcap, int64_t split_tokens, uint32_t* err, void* stream);

/* ---- head-sharded groups (one process per GPU) ---------------------------
 * No llmopt counterpart: llmopt runs on one device.  With KV heads split over
 * `world` GPUs (rank r owns query heads [r*H, (r+1)*H) of H*world), the only
 * exchange is an all-gather of the attention output.  These entry points do
 * it inside the combine kernel: each merged row is stored straight into every
 * rank's gathered output over NVLink, and the kernel ends with a bounded
 * cross-rank barrier on flags in peer memory.
 *
 * Peer buffers are plain cudaMalloc allocations shared between processes with
 * CUDA IPC: llmopt_peer_alloc returns the local pointer and a
 * LLMOPT_PEER_HANDLE_BYTES handle to send to the other ranks (any host
 * channel), llmopt_peer_open maps a peer's handle, llmopt_peer_close unmaps
 * it, llmopt_peer_free releases a local buffer (after every peer closed it).
 * These allocate and synchronise; call them at set-up, not per step.
 */
#define LLMOPT_PEER_HANDLE_BYTES 64
#define LLMOPT_MAX_PEERS 8
/* Bytes of a rank's flag buffer: LLMOPT_MAX_PEERS arrival slots + a CTA counter. */
#define LLMOPT_PEER_FLAGS_BYTES 64
LLMOPT_API int llmopt_peer_alloc(int32_t device, size_t bytes, void** ptr, void* handle);
LLMOPT_API int llmopt_peer_open(int32_t device, const void* handle, void** ptr);
LLMOPT_API int llmopt_peer_close(int32_t device, void* ptr);
LLMOPT_API int llmopt_peer_free(int32_t device, void* ptr);

/* llmopt_paged_attention_phase for this rank's heads, whose COMBINE phase also
 * performs the all-gather.  gathered[r] / flags[r] are rank r's gathered
 * output ([world*num_heads, batch, q_len, head_dim] of out_dtype, head-major)
 * and flag buffer (LLMOPT_PEER_FLAGS_BYTES, zeroed before first use), as
 * mapped in this process; gathered[rank] / flags[rank] are this rank's own.
 * Every rank makes the same sequence of calls with the same shapes, each with
 * an `epoch` one above its previous call, modulo 2^32 (starting at 1; 0
 * follows 0xFFFFFFFF: arrivals are compared by serial-number arithmetic, so
 * the count may wrap, as long as ranks stay within 2^31 calls of each other).
 * When the COMBINE
 * kernel ends, this rank's gathered output holds every rank's heads.  Peers
 * write a call's rows into gathered[] while this rank may still be reading
 * the previous call's: alternate two gathered buffers between calls.  A peer
 * that never arrives makes the barrier give up after about a second with
 * LLMOPT_DEVERR_WAIT_TIMEOUT set in `err`.  Everything else (workspace, lse of
 * this rank's heads, split_tokens, phases) is as in llmopt_paged_attention_phase. */
LLMOPT_API int llmopt_paged_attention_gather(
    const void* query, int32_t q_dtype, int64_t q_s, int64_t q_h, int64_t q_t,
    const void* key_cache, const void* value_cache, int32_t kv_dtype, int32_t num_layers,
    int32_t num_blocks, int32_t block_size, int32_t num_kv_heads, int32_t head_dim,
    int32_t layer_idx, const void* block_table, int32_t table_is_i64, int64_t table_width,
    int64_t table_stride, const void* context_lens, int32_t ctx_is_i64,
    void* const* gathered, uint32_t* const* flags, int32_t world, int32_t rank, uint32_t epoch,
    int32_t out_dtype, float* lse, int64_t batch, int32_t num_heads, int32_t q_len, float scale,
    float softcap, int64_t split_tokens, void* workspace, size_t workspace_bytes,
    uint32_t* err, void* stream, int32_t phases);

/*
 * Exact log-sum-exp merge of two partial attention states.  Replaces
 * merge_states (paged_attention.py:30-55).  o1/o2/out are contiguous
 * [rows, head_dim] of o_dtype; l1/l2/lse_out contiguous [rows] of lse_dtype.
 * Same IEEE behaviour as torch.logaddexp (two -inf inputs give NaN outputs).
 */
LLMOPT_API int llmopt_merge_states(const void* o1, const void* o2, const void* l1, const void* l2,
                        void* out, void* lse_out, int64_t rows, int32_t head_dim,
                        int32_t o_dtype, int32_t lse_dtype, void* stream);

/*
 * Chunked-prefill KV append.  Replaces PagedKVCache.write + _write_one
 * (paged_cache.py:175-232): for each sequence, rows keys[s, i] land at
 * position token_offsets[s] + i; the walk stops at the first -1 table entry or
 * the end of the row.  keys/values [batch, q_len, num_kv_heads, head_dim]
 * with element strides (seq, token, head), head_dim contiguous, cast to the
 * cache dtype with round-to-nearest-even.
 */
LLMOPT_API int llmopt_kv_write(const void* keys, const void* values, int32_t in_dtype,
                    int64_t k_s, int64_t k_t, int64_t k_h, int64_t v_s, int64_t v_t, int64_t v_h,
                    void* key_cache, void* value_cache, int32_t kv_dtype,
                    int32_t num_layers, int32_t num_blocks, int32_t block_size,
                    int32_t num_kv_heads, int32_t head_dim, int32_t layer_idx,
                    const void* block_table, int32_t table_is_i64, int64_t table_width,
                    int64_t table_stride, const void* token_offsets, int32_t off_is_i64,
                    int64_t batch, int32_t q_len, uint32_t* err, void* stream);

/*
 * Single-token decode append.  Replaces PagedKVCache.write_decode
 * (paged_cache.py:234-261): row s lands in table column floor(off/bs) (a
 * negative column wraps, as torch indexing does) at slot off mod bs; a block
 * id < 0 or >= num_blocks is written to block 0, which is the reference's
 * behaviour.  keys/values [batch, num_kv_heads, head_dim], strides (seq, head).
 */
LLMOPT_API int llmopt_kv_write_decode(const void* keys, const void* values, int32_t in_dtype,
                           int64_t k_s, int64_t k_h, int64_t v_s, int64_t v_h,
                           void* key_cache, void* value_cache, int32_t kv_dtype,
                           int32_t num_layers, int32_t num_blocks, int32_t block_size,
                           int32_t num_kv_heads, int32_t head_dim, int32_t layer_idx,
                           const void* block_table, int32_t table_is_i64, int64_t table_width,
                           int64_t table_stride, const void* token_offsets, int32_t off_is_i64,
                           int64_t batch, uint32_t* err, void* stream);

/*
 * Padded gather of a batch's KV.  Replaces PagedKVCache.gather
 * (paged_cache.py:263-312).  out_keys/out_values contiguous
 * [batch, max_len, num_kv_heads, head_dim] in the cache dtype (zero where
 * invalid); valid contiguous [batch, max_len] uint8.  max_len must not exceed
 * table_width * block_size (the reference raises IndexError there).
 */
LLMOPT_API int llmopt_paged_gather(const void* key_cache, const void* value_cache, int32_t kv_dtype,
                        int32_t num_layers, int32_t num_blocks, int32_t block_size,
                        int32_t num_kv_heads, int32_t head_dim, int32_t layer_idx,
                        const void* block_table, int32_t table_is_i64, int64_t table_width,
                        int64_t table_stride, const void* context_lens, int32_t ctx_is_i64,
                        int64_t batch, int64_t max_len, void* out_keys, void* out_values,
                        uint8_t* valid, uint32_t* err, void* stream);

/*
 * Rotary embedding of q and k fused with the K/V append: the statements of
 * PagedAttentionLayer.forward between the projections and attention
 * (layers.py:106-134).  q_proj [batch * q_len, num_heads * head_dim], k_proj /
 * v_proj [batch * q_len, num_kv_heads * head_dim] (rows of tokens, row strides
 * q_row / k_row / v_row, unit inner stride, dtype in_dtype = the model dtype);
 * positions [batch * q_len]; cos_table / sin_table [max_positions, head_dim]
 * (table_dtype; RotaryEmbedding.cos_cached / sin_cached).  The cos/sin rows are
 * cast to in_dtype, q and k rotated as x * cos + rotate_half(x) * sin with each
 * product and the sum rounded to in_dtype (bit-identical to the reference's
 * tensor ops); the rotated query goes to q_out (in_dtype, strides (seq, head,
 * token) of a [batch, num_heads, q_len, head_dim] view), the rotated k and the
 * v rows to the cache at the offsets, cast to kv_dtype, with the rules of
 * llmopt_kv_write_decode when q_len == 1 and llmopt_kv_write otherwise.
 * head_dim must be even.  A position >= max_positions or < -max_positions
 * skips its token and sets LLMOPT_DEVERR_POSITION (the reference raises
 * ValueError after a host sync; no sync happens here).
 */
LLMOPT_API int llmopt_rope_kv_append(
    const void* q_proj, const void* k_proj, const void* v_proj, int32_t in_dtype, int64_t q_row,
    int64_t k_row, int64_t v_row, const void* positions, int32_t pos_is_i64,
    const void* cos_table, const void* sin_table, int32_t table_dtype, int64_t max_positions,
    void* q_out, int64_t qo_s, int64_t qo_h, int64_t qo_t, void* key_cache, void* value_cache,
    int32_t kv_dtype, int32_t num_layers, int32_t num_blocks, int32_t block_size,
    int32_t num_kv_heads, int32_t head_dim, int32_t layer_idx, const void* block_table,
    int32_t table_is_i64, int64_t table_width, int64_t table_stride, const void* token_offsets,
    int32_t off_is_i64, int64_t batch, int32_t num_heads, int32_t q_len, uint32_t* err,
    void* stream);

/*
 * Decode-step metadata kept on the device.  Replaces the per-step host build
 * of ModelRunner._build_decode + _finalize (model_runner.py:169-230): for a
 * decode step the reference gives each request position = token offset =
 * committed tokens, context length = committed + 1 and its block ids (-1
 * padded) as a table row.  Here block_table [max_rows, table_width] (row
 * stride table_stride, int32), context_lens, token_offsets and positions
 * ([max_rows] int64) live on the device; updates (device memory, int64) is
 * [count, then count records (op, row, a, b)], capacity records at most,
 * applied in order:
 *   LLMOPT_STEP_SET_BLOCK  table[row][a] = b
 *   LLMOPT_STEP_ADMIT      row holds a new sequence with a committed tokens:
 *                          context_lens[row] = a, table row set to -1
 *   LLMOPT_STEP_MOVE       row takes row a's table row and context length
 * then every row r < batch advances: token_offsets[r] = positions[r] =
 * context_lens[r]; context_lens[r] += 1.  One launch, no host sync; the count
 * is read on the device, so a captured graph replays with any update count.
 * Bad rows or columns are skipped and flag LLMOPT_DEVERR_TABLE_WIDTH.
 */
#define LLMOPT_STEP_SET_BLOCK 0
#define LLMOPT_STEP_ADMIT 1
#define LLMOPT_STEP_MOVE 2
LLMOPT_API int llmopt_decode_step_advance(const int64_t* updates, int64_t capacity,
                                          int32_t* block_table, int64_t table_width,
                                          int64_t table_stride, int64_t* context_lens,
                                          int64_t* token_offsets, int64_t* positions,
                                          int64_t max_rows, int64_t batch, uint32_t* err,
                                          void* stream);

/*
 * FP8 KV storage.  An e4m3 cache is key_cache / value_cache in the usual
 * [num_layers, num_blocks, block_size, num_kv_heads, head_dim] layout holding
 * float8_e4m3fn codes, plus key_scale / value_scale: contiguous fp32
 * [num_layers, num_blocks, num_kv_heads, block_size] (head-major within a
 * block, so one head's scales for a block are 64 contiguous bytes).  Element
 * value = code * scale of its (token, head) row.  The appends quantize each
 * (token, head) row on its own: scale = amax(|row|) / 448 (NaN ignored; 1 when
 * not positive), code = e4m3(x / scale), both rounded to nearest even (the
 * code rounding is torch's .to(torch.float8_e4m3fn)).  Attention reads the
 * cache as those values with the query rounded to f16; outputs, LSE, splits,
 * workspace and errors as llmopt_paged_attention_phase.  Gather returns the
 * dequantized values as fp32.  Caches and scales 16-byte aligned, head_dim
 * <= 256; the tensor-core decode covers block_size 16, head_dim 128 or 256
 * and q_len * group <= 16, everything else runs on CUDA cores.
 */
LLMOPT_API int llmopt_kv_write_scaled(const void* keys, const void* values, int32_t in_dtype,
                    int64_t k_s, int64_t k_t, int64_t k_h, int64_t v_s, int64_t v_t, int64_t v_h,
                    void* key_cache, void* value_cache, int32_t kv_dtype,
                    float* key_scale, float* value_scale,
                    int32_t num_layers, int32_t num_blocks, int32_t block_size,
                    int32_t num_kv_heads, int32_t head_dim, int32_t layer_idx,
                    const void* block_table, int32_t table_is_i64, int64_t table_width,
                    int64_t table_stride, const void* token_offsets, int32_t off_is_i64,
                    int64_t batch, int32_t q_len, uint32_t* err, void* stream);

LLMOPT_API int llmopt_kv_write_decode_scaled(const void* keys, const void* values,
                    int32_t in_dtype, int64_t k_s, int64_t k_h, int64_t v_s, int64_t v_h,
                    void* key_cache, void* value_cache, int32_t kv_dtype,
                    float* key_scale, float* value_scale,
                    int32_t num_layers, int32_t num_blocks, int32_t block_size,
                    int32_t num_kv_heads, int32_t head_dim, int32_t layer_idx,
                    const void* block_table, int32_t table_is_i64, int64_t table_width,
                    int64_t table_stride, const void* token_offsets, int32_t off_is_i64,
                    int64_t batch, uint32_t* err, void* stream);

LLMOPT_API int llmopt_paged_attention_scaled(const void* query, int32_t q_dtype, int64_t q_s,
                    int64_t q_h, int64_t q_t, const void* key_cache, const void* value_cache,
                    int32_t kv_dtype, const float* key_scale, const float* value_scale,
                    int32_t num_layers, int32_t num_blocks, int32_t block_size,
                    int32_t num_kv_heads, int32_t head_dim, int32_t layer_idx,
                    const void* block_table, int32_t table_is_i64, int64_t table_width,
                    int64_t table_stride, const void* context_lens, int32_t ctx_is_i64,
                    void* out, int32_t out_dtype, int64_t o_s, int64_t o_h, int64_t o_t,
                    float* lse, int64_t batch, int32_t num_heads, int32_t q_len, float scale,
                    float softcap, int64_t split_tokens, void* workspace,
                    size_t workspace_bytes, uint32_t* err, void* stream, int32_t phases);

LLMOPT_API int llmopt_paged_gather_scaled(const void* key_cache, const void* value_cache,
                    int32_t kv_dtype, const float* key_scale, const float* value_scale,
                    int32_t num_layers, int32_t num_blocks, int32_t block_size,
                    int32_t num_kv_heads, int32_t head_dim, int32_t layer_idx,
                    const void* block_table, int32_t table_is_i64, int64_t table_width,
                    int64_t table_stride, const void* context_lens, int32_t ctx_is_i64,
                    int64_t batch, int64_t max_len, float* out_keys, float* out_values,
                    uint8_t* valid, uint32_t* err, void* stream);

/*
 * Weight-only quantized linear layer.  Replaces QuantLinear.forward
 * (src/llmopt/quantization/quant_linear.py:93-113: dequantize the packed weight
 * to the compute dtype, quantizers.py:203-239, then F.linear) by one fused
 * kernel that reads the packed codes on every call (no dense copy is kept).
 *
 *   x       [m, k] compute dtype (f32 / f16 / bf16), row stride ldx
 *   qweight the reference's QuantizedTensor.qweight: uint8 [n, k/2] for 2- and
 *           4-bit codes (two per byte, even column in the low nibble, symmetric
 *           codes biased by 2^(bits-1)); uint8 [n, k] (asymmetric) or int8 [n, k]
 *           (symmetric) for 8-bit
 *   scales, zeros  float32 [n, k / group_size] (zeros unused and may be null
 *           when symmetric)
 *   bias    [n] compute dtype, or null;  out [m, n] compute dtype, stride ldo
 * The weight element is (q - offset) * s or (q - z) * s in float32 rounded to
 * the compute dtype, as the reference's dequantize.  16-bit compute dtypes
 * with k % 128 == 0, n % 64 == 0, group_size 32, 64, 128 or a multiple of
 * 128, and 16-byte aligned x / qweight run on tensor cores; everything else
 * runs on CUDA cores.  On tensor cores, 2- and 4-bit codes are not rounded
 * weight by weight: the MMAs sum the exact products (q - z) * x of each group
 * in fp32 and the group's scale multiplies that sum, which is at least as
 * accurate as the reference's weights rounded to the compute dtype; 8-bit
 * weights are the reference's bit for bit.  Zero points must be whole numbers,
 * as the reference's quantizers round them: the kernels subtract them exactly
 * only then (a fractional zero point is rounded to an integer; the Python layer
 * refuses one with ValueError).  The workspace (fp32
 * split-k partials) is sized by llmopt_quant_linear_workspace_size for the
 * same m, n, k.
 */
LLMOPT_API int llmopt_quant_linear_workspace_size(int device, int64_t m, int64_t n, int64_t k,
                    int32_t bits, int32_t group_size, int32_t x_dtype, size_t* bytes);
LLMOPT_API int llmopt_quant_linear(const void* x, int32_t x_dtype, int64_t m, int64_t ldx,
                    const void* qweight, int32_t bits, int32_t group_size, int32_t symmetric,
                    const float* scales, const float* zeros, int64_t n, int64_t k,
                    const void* bias, void* out, int64_t ldo, void* workspace,
                    size_t workspace_bytes, void* stream);
/* The dense weight [n, k] in out_dtype, bit-exact with the reference's
 * dequantize (QuantizedTensor.dequantize().to(dtype), quantizers.py:231-239). */
LLMOPT_API int llmopt_dequantize(const void* qweight, int32_t bits, int32_t group_size,
                    int32_t symmetric, const float* scales, const float* zeros, int64_t n,
                    int64_t k, void* out, int32_t out_dtype, void* stream);
/* LLMOPT_DEVERR_* bits that the quantized-linear kernels' bounded waits recorded
 * on the current device since the last clear (synchronous read; cleared when
 * `clear` is non-zero).  Only the tcgen05 path, enabled by
 * LLMOPT_B200_QUANT_TC05=1, waits on the device; its outputs are NaN where a
 * wait gave up. */
LLMOPT_API int llmopt_quant_linear_device_errors(int32_t clear, uint32_t* bits);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* LLMOPT_B200_H_ */
