// Split-K partition of the paged attention work, shared by the attention
// kernels (which produce partial states) and the combine kernel (which merges
// them).  Units are KV blocks; a sequence with context c owns
// nb = min(ceil(c / block_size), table_width) blocks (positions past the table
// row are never visited and are flagged LLMOPT_DEVERR_TABLE_WIDTH).
//
// Two modes:
//
// * kModeBalanced: the blocks of the whole batch, concatenated in sequence
//   order (prefix[s] = blocks before sequence s, T = prefix[batch]), are cut
//   into `ctas` equal ranges [floor(c*T/ctas), floor((c+1)*T/ctas)).  A range
//   may cover the tail of one sequence and the head of the next; every
//   (sequence, CTA) pair it touches becomes one partial in slot s + c, which
//   is unique because both indices grow along the concatenated order.
//   Every CTA streams the same number of blocks, whatever the context mix.
// * kModeFixed: sequence s is cut into chunks of `split_blocks` blocks; CTA
//   (s, j) = blockIdx s * splits + j writes slot s * splits + j.  This is
//   PagedAttentionConfig.split_size (rounded up to whole blocks), or one chunk
//   per sequence when split_kv is off.
#pragma once

#include <stdint.h>

namespace llmopt {

enum SplitMode : int { kModeFixed = 0, kModeBalanced = 1 };

struct SplitPlan {
  int mode;
  int ctas;          // kModeBalanced: number of ranges (CTAs along x)
  int split_blocks;  // kModeFixed: blocks per chunk
  int splits;        // kModeFixed: chunks per sequence (grid x = batch * splits)
  long long slots;   // partial slots to reserve
};

__host__ __device__ __forceinline__ long long range_start(long long c, long long total,
                                                          long long ctas) {
  return (c * total) / ctas;
}

// The CTA whose balanced range contains block f (0 <= f < total).
__host__ __device__ __forceinline__ long long range_owner(long long f, long long total,
                                                          long long ctas) {
  return ((f + 1) * ctas - 1) / total;
}

__host__ __device__ __forceinline__ long long blocks_of(long long ctx, int block_size,
                                                        long long width) {
  if (ctx <= 0) return 0;
  long long nb = (ctx + block_size - 1) / block_size;
  return nb < width ? nb : width;
}

}  // namespace llmopt
