// qargmax.cuh — row-wise argmax of fp16 logits as packed 64-bit keys.
//
// The engines of the reference only ever take argmax over the lm_head's
// logits (greedy decoding: src/engine/paged_engine.py:146-147,202-203,
// graphed_decode_engine.py:114-115).  With the lm_head column-sharded, each
// rank reduces its [M, N/P] logits to one key per row and the ranks
// exchange 8 bytes per row instead of the logits themselves.
//
// key = (ord(h) << 32) | (0xFFFFFFFF - column), column = col_offset + n,
// where ord maps fp16 bits to an unsigned order-preserving code
// (negatives: ~bits; non-negatives: bits | 0x8000; -0 as +0, NaN largest).  The largest key is the
// largest value and, among equal values, the smallest column — the index
// torch.argmax returns ("the first maximal value").  Keys from different
// shards combine with a plain max.
#pragma once

#include "ql_common.cuh"

namespace ql {
namespace amax {

__device__ __forceinline__ unsigned long long row_key(unsigned short bits, long long column) {
  // -0 counts as +0, and every NaN as the largest value (torch.argmax
  // treats NaN as maximal)
  if (bits == 0x8000u) bits = 0;
  if ((bits & 0x7FFFu) > 0x7C00u) bits = 0x7FFFu;
  const unsigned ord = (bits & 0x8000u) ? (unsigned)(~bits & 0xFFFFu) : (unsigned)(bits | 0x8000u);
  return ((unsigned long long)ord << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)column);
}

__device__ __forceinline__ unsigned long long umax64(unsigned long long a, unsigned long long b) {
  return a > b ? a : b;
}

// grid (chunks, M); each CTA reduces columns [chunk*span, +span) of one row
// and merges its key into keys[m] with a 64-bit atomic max (keys zeroed by
// the caller's stream beforehand).  vec: rows 16-byte aligned and N % 8 == 0.
__global__ void __launch_bounds__(256) argmax_rows_kernel(const __half* x, long long ldx, int N, int span,
                                                          long long col_offset, int vec,
                                                          unsigned long long* keys) {
  griddep_wait();   // the logits come from the kernel before (programmatic dependent launch)
  const int m = blockIdx.y;
  const int c0 = blockIdx.x * span;
  const int c1 = min(N, c0 + span);
  const unsigned short* row = reinterpret_cast<const unsigned short*>(x + (long long)m * ldx);
  unsigned long long best = 0ull;
  if (vec) {
    for (int c = c0 + (int)threadIdx.x * 8; c < c1; c += 256 * 8) {
      const uint4 v = *reinterpret_cast<const uint4*>(row + c);
      const unsigned w[4] = {v.x, v.y, v.z, v.w};
      #pragma unroll
      for (int j = 0; j < 4; ++j) {
        best = umax64(best, row_key((unsigned short)(w[j] & 0xFFFFu), col_offset + c + 2 * j));
        best = umax64(best, row_key((unsigned short)(w[j] >> 16), col_offset + c + 2 * j + 1));
      }
    }
  } else {
    for (int c = c0 + (int)threadIdx.x; c < c1; c += 256) best = umax64(best, row_key(row[c], col_offset + c));
  }
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = umax64(best, __shfl_xor_sync(0xffffffffu, best, o));
  __shared__ unsigned long long red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = red[0];
    for (int w = 1; w < 8; ++w) b = umax64(b, red[w]);
    atomicMax(keys + m, b);
  }
}

}  // namespace amax
}  // namespace ql
