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
//
// The decode GEMV (qgemv.cuh) runs the same protocol from its own epilogue
// (keys of the fp16-rounded outputs, no logits written): `Ctx` is the part
// both kernels share and `publish_and_combine` the last CTA's step.
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

// What a kernel needs to take part in one exchange.
struct Ctx {
  unsigned char* peer[kMaxRanks];   // exchange buffer of every rank (peer[rank] = own)
  long long* out;                   // [M] argmax columns
  long long col_offset;             // global column of this rank's first column
  int rank, world, max_m;
};

struct Params {
  const __half* x;
  long long ldx;
  int M, N, span, vec;
  Ctx c;
  unsigned* err;
};

__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long* p) {
  return *reinterpret_cast<const volatile unsigned long long*>(p);
}
__device__ __forceinline__ void st_volatile_u64(unsigned long long* p, unsigned long long v) {
  *reinterpret_cast<volatile unsigned long long*>(p) = v;
}
constexpr unsigned long long kKeyMask = 0xFFFFFFFFFFFFull;   // the 48 key bits

// Calls completed so far on this rank's buffer (read once the kernel
// before has finished: only the last CTA of a call changes it, at its end).
__device__ __forceinline__ unsigned epochs_done(const Ctx& c) {
  const Layout L = layout(c.world, c.max_m);
  return *reinterpret_cast<const volatile unsigned*>(c.peer[c.rank] + L.state + 4);
}

// This rank's row maxima (scratch) are complete: push them, tagged with the
// call's epoch, into every rank's bank, wait (bounded) for every rank's,
// write the argmax columns and reset scratch, the CTA counter and the epoch
// for the next call (one rank: the columns straight from scratch).  Run by
// all `nthr` threads of the last CTA; `bar` synchronises them; `done` =
// epochs_done() read earlier in the kernel.
template <class Bar>
__device__ __forceinline__ void publish_and_combine(const Ctx& c, int M, int tid, int nthr, unsigned* err, Bar bar,
                                                    unsigned done) {
  const Layout L = layout(c.world, c.max_m);
  unsigned char* own = c.peer[c.rank];
  unsigned long long* scratch = reinterpret_cast<unsigned long long*>(own + L.scratch);
  unsigned* counter = reinterpret_cast<unsigned*>(own + L.state);
  unsigned* epoch_done = counter + 1;
  const unsigned e = done + 1u;
  if (c.world == 1) {
    for (int i = tid; i < M; i += nthr) {
      const unsigned long long b = ld_volatile_u64(scratch + i) & kKeyMask;
      c.out[i] = (long long)(0xFFFFFFFFu - (unsigned)(b & 0xFFFFFFFFull));
      scratch[i] = 0ull;
    }
    bar();
    if (tid == 0) {
      *counter = 0u;
      *reinterpret_cast<volatile unsigned*>(epoch_done) = e;
    }
    return;
  }
  const int bank = (int)(e & 1u);
  const unsigned long long tag = (unsigned long long)((e & 0x7FFFu) | 0x8000u) << 48;   // never 0
  for (int q = 0; q < c.world; ++q) {
    unsigned long long* dst =
        reinterpret_cast<unsigned long long*>(c.peer[q] + L.keys) + ((size_t)bank * c.world + c.rank) * c.max_m;
    for (int i = tid; i < M; i += nthr) st_volatile_u64(dst + i, tag | ld_volatile_u64(scratch + i));
  }
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(own + L.keys) + (size_t)bank * c.world * c.max_m;
  for (int i = tid; i < M; i += nthr) {
    unsigned long long b = 0ull;
    for (int q = 0; q < c.world; ++q) {
      const unsigned long long* slot = keys + (size_t)q * c.max_m + i;
      unsigned long long v = ld_volatile_u64(slot);
      if ((v & ~kKeyMask) != tag) {               // bounded wait for rank q's key of this call
        const long long t0 = clock64();
        while (((v = ld_volatile_u64(slot)) & ~kKeyMask) != tag) {
          if (clock64() - t0 > kWaitBudgetCycles) {
            atomicCAS(err, 0u, kDevErrPeerWait);
            break;
          }
          __nanosleep(32);
        }
      }
      b = amax::umax64(b, v & kKeyMask);
    }
    c.out[i] = (long long)(0xFFFFFFFFu - (unsigned)(b & 0xFFFFFFFFull));
    scratch[i] = 0ull;                       // ready for the next call
  }
  bar();
  if (tid == 0) {
    *counter = 0u;
    *reinterpret_cast<volatile unsigned*>(epoch_done) = e;
  }
}

// This CTA's contribution is in scratch: count the CTA in; true for the
// last one to arrive (which then sees every CTA's atomics).  Thread 0 only.
__device__ __forceinline__ bool arrive_last(const Ctx& c, unsigned total) {
  const Layout L = layout(c.world, c.max_m);
  unsigned* counter = reinterpret_cast<unsigned*>(c.peer[c.rank] + L.state);
  return atomic_add_acq_rel_gpu(counter, 1u) == total - 1;
}

__device__ __forceinline__ unsigned long long* scratch_of(const Ctx& c) {
  return reinterpret_cast<unsigned long long*>(c.peer[c.rank] + layout(c.world, c.max_m).scratch);
}

__global__ void __launch_bounds__(256) argmax_exchange_kernel(const Params p) {
  unsigned long long* scratch = scratch_of(p.c);
  __shared__ unsigned long long red[8];
  __shared__ int is_last;
  __shared__ unsigned done_s;

  // the logits come from the kernel before (launched with programmatic
  // dependent launch, this kernel is resident early and waits here)
  griddep_wait();
  const unsigned done = threadIdx.x == 0 ? epochs_done(p.c) : 0u;   // off the tail's critical path

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
        best = amax::umax64(best, amax::row_key((unsigned short)(w[j] & 0xFFFFu), p.c.col_offset + c + 2 * j));
        best = amax::umax64(best, amax::row_key((unsigned short)(w[j] >> 16), p.c.col_offset + c + 2 * j + 1));
      }
    }
  } else {
    for (int c = c0 + (int)threadIdx.x; c < c1; c += 256) best = amax::umax64(best, amax::row_key(row[c], p.c.col_offset + c));
  }
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = amax::umax64(best, __shfl_xor_sync(0xffffffffu, best, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = red[0];
    for (int w = 1; w < 8; ++w) b = amax::umax64(b, red[w]);
    atomicMax(scratch + m, b);
    is_last = arrive_last(p.c, gridDim.x * gridDim.y);
    done_s = done;
  }
  __syncthreads();
  if (!is_last) return;

  // ---- last CTA: push tagged keys, wait for every rank's, combine
  publish_and_combine(p.c, p.M, (int)threadIdx.x, (int)blockDim.x, p.err, [] { __syncthreads(); }, done_s);
}

}  // namespace xchg
}  // namespace ql
