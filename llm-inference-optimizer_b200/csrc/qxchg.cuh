// qxchg.cuh — sharded-lm_head argmax in one kernel: local reduction plus a
// push exchange of the per-row keys over NVLink peer memory.
//
// Every rank owns an exchange buffer (plain device memory shared with the
// other ranks of the node through CUDA IPC):
//   [0, KB)             keys[2][world][max_m] u64: by epoch parity, by source rank
//   then                scratch[max_m] u64: this rank's running row maxima
//   then                state: counter u32 (CTAs arrived), epoch u32 (calls done)
// Only the owner touches scratch and state; peers write keys.
//
// One launch (grid (chunks, M)): each CTA reduces its column chunk of one
// row to a 48-bit key (qargmax.cuh) and merges it into scratch with a 64-bit
// atomic max; the last CTA to arrive stores, for every row, the key tagged
// with the call's epoch in bits 48..63 into keys[e & 1][rank][m] of every
// rank's buffer — one 8-byte store each, which a reader sees whole, so no
// fence or separate flag is needed — then polls (bounded) its own buffer
// until every rank's slot carries the epoch, and writes out[m] = the column
// of the largest key.  A rank can be at most one call ahead of another (it
// needs everybody's keys of the call before), so two banks by epoch parity
// are enough.  Ranks must make the same sequence of calls.
#pragma once

#include "qargmax.cuh"

namespace ql {
namespace xchg {

constexpr int kMaxRanks = 8;

struct Layout {
  size_t keys, scratch, state, total;
};
__host__ __device__ inline Layout layout(int world, int max_m) {
  Layout l;
  l.keys = 0;
  l.scratch = l.keys + (size_t)2 * world * max_m * 8;
  l.state = l.scratch + (size_t)max_m * 8;
  l.total = (l.state + 8 + 255) / 256 * 256;
  return l;
}

struct Params {
  const __half* x;
  long long ldx;
  int M, N, span, vec;
  long long col_offset;
  int rank, world, max_m;
  unsigned char* peer[kMaxRanks];   // exchange buffer of every rank (peer[rank] = own)
  long long* out;                   // [M] argmax columns
  unsigned* err;
};

__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long* p) {
  return *reinterpret_cast<const volatile unsigned long long*>(p);
}
__device__ __forceinline__ void st_volatile_u64(unsigned long long* p, unsigned long long v) {
  *reinterpret_cast<volatile unsigned long long*>(p) = v;
}
constexpr unsigned long long kKeyMask = 0xFFFFFFFFFFFFull;   // the 48 key bits

__global__ void __launch_bounds__(256) argmax_exchange_kernel(const Params p) {
  const Layout L = layout(p.world, p.max_m);
  unsigned char* own = p.peer[p.rank];
  unsigned long long* scratch = reinterpret_cast<unsigned long long*>(own + L.scratch);
  unsigned* counter = reinterpret_cast<unsigned*>(own + L.state);
  unsigned* epoch_done = counter + 1;
  __shared__ unsigned long long red[8];
  __shared__ int is_last;

  // the logits come from the kernel before (launched with programmatic
  // dependent launch, this kernel is resident early and waits here)
  griddep_wait();

  // ---- local reduction of this CTA's chunk of row m
  const int m = blockIdx.y;
  const int c0 = blockIdx.x * p.span;
  const int c1 = min(p.N, c0 + p.span);
  const unsigned short* row = reinterpret_cast<const unsigned short*>(p.x + (long long)m * p.ldx);
  unsigned long long best = 0ull;
  if (p.vec) {
    for (int c = c0 + (int)threadIdx.x * 8; c < c1; c += 256 * 8) {
      const uint4 v = *reinterpret_cast<const uint4*>(row + c);
      const unsigned w[4] = {v.x, v.y, v.z, v.w};
      #pragma unroll
      for (int j = 0; j < 4; ++j) {
        best = amax::umax64(best, amax::row_key((unsigned short)(w[j] & 0xFFFFu), p.col_offset + c + 2 * j));
        best = amax::umax64(best, amax::row_key((unsigned short)(w[j] >> 16), p.col_offset + c + 2 * j + 1));
      }
    }
  } else {
    for (int c = c0 + (int)threadIdx.x; c < c1; c += 256) best = amax::umax64(best, amax::row_key(row[c], p.col_offset + c));
  }
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = amax::umax64(best, __shfl_xor_sync(0xffffffffu, best, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = red[0];
    for (int w = 1; w < 8; ++w) b = amax::umax64(b, red[w]);
    atomicMax(scratch + m, b);
    __threadfence();
    const unsigned total = gridDim.x * gridDim.y;
    is_last = atomicAdd(counter, 1u) == total - 1;
    if (is_last) __threadfence();
  }
  __syncthreads();
  if (!is_last) return;

  // ---- last CTA: push tagged keys, wait for every rank's, combine
  const unsigned e = *reinterpret_cast<volatile unsigned*>(epoch_done) + 1u;
  const int bank = (int)(e & 1u);
  const unsigned long long tag = (unsigned long long)((e & 0x7FFFu) | 0x8000u) << 48;   // never 0
  for (int q = 0; q < p.world; ++q) {
    unsigned long long* dst =
        reinterpret_cast<unsigned long long*>(p.peer[q] + L.keys) + ((size_t)bank * p.world + p.rank) * p.max_m;
    for (int i = threadIdx.x; i < p.M; i += blockDim.x) st_volatile_u64(dst + i, tag | ld_volatile_u64(scratch + i));
  }
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(own + L.keys) + (size_t)bank * p.world * p.max_m;
  for (int i = threadIdx.x; i < p.M; i += blockDim.x) {
    unsigned long long b = 0ull;
    for (int q = 0; q < p.world; ++q) {
      const unsigned long long* slot = keys + (size_t)q * p.max_m + i;
      unsigned long long v = ld_volatile_u64(slot);
      if ((v & ~kKeyMask) != tag) {               // bounded wait for rank q's key of this call
        const long long t0 = clock64();
        while (((v = ld_volatile_u64(slot)) & ~kKeyMask) != tag) {
          if (clock64() - t0 > kWaitBudgetCycles) {
            atomicCAS(p.err, 0u, kDevErrPeerWait);
            break;
          }
          __nanosleep(32);
        }
      }
      b = amax::umax64(b, v & kKeyMask);
    }
    p.out[i] = (long long)(0xFFFFFFFFu - (unsigned)(b & 0xFFFFFFFFull));
    scratch[i] = 0ull;                       // ready for the next call
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    *counter = 0u;
    *reinterpret_cast<volatile unsigned*>(epoch_done) = e;
  }
}

}  // namespace xchg
}  // namespace ql
