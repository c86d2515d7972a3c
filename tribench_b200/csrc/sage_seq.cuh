// sage_seq.cuh — where one sequence of a batch lives in the token axis of a tensor.
//
// Dense batches: sequence b is batch entry b, rows [0, S). Variable-length batches (packed
// sequences): every tensor has batch extent 1 and sequence b owns rows [cu[b], cu[b+1]) of the
// token axis, cu being the batch's prefix sums of lengths (flash-attention's cu_seqlens).
#pragma once

namespace sage {

struct SeqSpan {
  int base;   // first token row of the sequence
  int len;    // rows
  int batch;  // batch coordinate of the tensors (b, or 0 for packed sequences)
};

// Lengths are clamped so that a malformed cu array (decreasing, out of range, longer than the
// max_len the launch was sized for) never reaches rows or scale blocks outside the buffers.
__device__ __forceinline__ SeqSpan seq_span(const int* cu, int b, int max_len, int tokens) {
  if (cu == nullptr) return {0, max_len, b};
  const int s0 = cu[b];
  if (s0 < 0 || s0 > tokens) return {0, 0, 0};
  const int len = min(min(cu[b + 1] - s0, max_len), tokens - s0);
  return {s0, max(len, 0), 0};
}

}  // namespace sage
