// Device-resident decode step metadata: the block table, context lengths,
// write offsets and positions of every running sequence stay on the GPU and
// one launch per step applies the host's scheduling decisions and advances
// every row by one token.
//
// The reference rebuilds these tensors each step on the host
// (ModelRunner._build_decode + _finalize, src/llmopt/engine/model_runner.py:
// 169-230: a Python loop over requests, torch.full of the table, one small
// host-to-device copy per table row and one per vector).  For a decode step
// its values per request are: position = offset = committed tokens,
// context length = committed + 1, table row = the request's block ids, -1
// padded.  Here the committed count lives in context_lens from the previous
// step, so the advance is offset = position = context, context += 1; the host
// only sends what changed (a block appended, a sequence admitted or moved),
// packed as [count, op, row, a, b, op, row, a, b, ...] int64 in device memory.
// Because the count is read on the device, a captured CUDA graph of the whole
// decode step replays with any number of updates up to the buffer capacity.
#include "common.cuh"
#include "kernels.h"

namespace llmopt {
namespace {

constexpr int kThreads = 256;

// ops (also in include/llmopt_b200.h)
constexpr long long kOpSetBlock = 0;  // table[row][a] = b
constexpr long long kOpAdmit = 1;     // row holds a new sequence with a committed tokens: ctx = a, row = -1
constexpr long long kOpMove = 2;      // row takes row a's table row and context (compaction)

__global__ void __launch_bounds__(kThreads) step_advance_kernel(const StepArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  const long long n = a.updates[0] < a.capacity ? a.updates[0] : a.capacity;
  if (threadIdx.x == 0 && a.updates[0] > a.capacity) record_error(a.err, kErrTableWidth);
  const long long W = a.table_width;
  // Updates in order: each is applied by the whole CTA, barriers between them.
  for (long long u = 0; u < n; ++u) {
    const long long* rec = a.updates + 1 + 4 * u;
    const long long op = rec[0], row = rec[1], x = rec[2], y = rec[3];
    const bool row_ok = row >= 0 && row < a.max_rows;
    if (op == kOpSetBlock) {
      if (threadIdx.x == 0) {
        if (row_ok && x >= 0 && x < W) {
          a.table[row * a.table_stride + x] = (int)y;
        } else {
          record_error(a.err, kErrTableWidth);
        }
      }
    } else if (op == kOpAdmit) {
      if (row_ok) {
        for (long long c = threadIdx.x; c < W; c += kThreads) a.table[row * a.table_stride + c] = -1;
        if (threadIdx.x == 0) a.ctx[row] = x;
      } else if (threadIdx.x == 0) {
        record_error(a.err, kErrTableWidth);
      }
    } else if (op == kOpMove) {
      if (row_ok && x >= 0 && x < a.max_rows) {
        for (long long c = threadIdx.x; c < W; c += kThreads) {
          a.table[row * a.table_stride + c] = a.table[x * a.table_stride + c];
        }
        if (threadIdx.x == 0) a.ctx[row] = a.ctx[x];
      } else if (threadIdx.x == 0) {
        record_error(a.err, kErrTableWidth);
      }
    } else if (threadIdx.x == 0) {
      record_error(a.err, kErrTableWidth);
    }
    __syncthreads();
  }
  // The step: every active row writes its next token at its committed length.
  for (long long r = threadIdx.x; r < a.batch; r += kThreads) {
    const long long c = a.ctx[r];
    a.offsets[r] = c;
    a.positions[r] = c;
    a.ctx[r] = c + 1;
  }
}

}  // namespace

cudaError_t step_advance_launch(const StepArgs& a, cudaStream_t stream) {
  void* args[] = {const_cast<StepArgs*>(&a)};
  return launch_pdl(reinterpret_cast<const void*>(&step_advance_kernel), dim3(1), dim3(kThreads),
                    args, 0, stream);
}

}  // namespace llmopt
