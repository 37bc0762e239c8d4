// qgather.cuh — all-gather of a column-sharded layer's fp16 outputs over
// NVLink peer memory, one kernel per rank, no NCCL.
//
// The output [M, N] is `groups` blocks of ng = N / groups columns (one block
// for an lm_head, two for a fused [gate | up] projection); rank q owns the
// columns [q*b, min(ng, (q+1)*b)) of every block, b = ceil(ng / world).
//
// Every rank owns a gather buffer (plain device memory shared with the other
// ranks of the node through CUDA IPC, zero-filled at allocation):
//   [0, 8192)   ready[kMaxRanks][kMaxCtas] u32: ready[q][c] = the last call
//               whose chunk c of rank q's columns CTA c of rank q has
//               completely stored into this buffer (written by rank q)
//   [8192, 8200) state: counter u32 (CTAs arrived), epoch u32 (calls done);
//               only the owner touches them
//   [8448, ...) data[2][max_m][ldb] fp16, ldb = N rounded up to 8: the other
//               ranks' columns of a call, by epoch parity, at their global
//               positions
//   then        lines[2][line_rows][ldb / 4] 16-byte lines for small calls:
//               two u64 words {2 fp16 | tag << 32}, tag = the call's epoch
//
// One launch per rank and call, after the rank's own columns are in `out`
// (or in `src`, then they are copied into `out` too).  Small calls (at most
// kLineMaxPayload bytes of output) travel as tagged lines: every 16-byte
// store carries 8 bytes of columns and the epoch twice, a reader polls each
// word (bounded) until both tags read e, so neither side needs a fence, a
// counter or a flag — twice the bytes on NVLink, a few microseconds less
// latency (used only when every rank owns columns: each rank then waits for
// every peer's lines of a call).  Larger calls go through the banks, chunk
// by chunk: the G CTAs of a launch (the same G on every rank: it depends
// only on the shapes) split each rank's columns into G contiguous chunks of
// units, and CTA c of every rank handles chunk c of every rank's columns:
//   1. CTA c stores chunk c of this rank's columns into data[e & 1] of every
//      peer (16-byte stores when the shapes allow), makes them visible
//      system-wide (one fence.acq_rel.sys) and then writes ready[rank][c] =
//      e into every peer's buffer (relaxed system-scope stores);
//   2. it takes the peers in turn: one thread polls its own ready[q][c]
//      (bounded, acquire) until it has reached e, then the CTA copies chunk
//      c of q's columns from its own data[e & 1] into `out`.
// No CTA waits for the other CTAs of its rank, so the copies out of the
// bank start chunk by chunk as the peers' chunks land.  (Measured on two
// B200s, M = 16 / 64 of a 151936-wide output: one flag per rank, set by the
// last CTA to finish, went out ~4.5 us after the median CTA's fence; pulling
// the chunks over NVLink instead of pushing them was 7-12 % slower.)
// Every CTA waits for every peer's ready[q][c] in every call, whether or
// not chunk c holds columns.  A rank finishes call e + 1 only once CTA c of
// every peer has published ready[q][c] = e + 1, which that CTA does in its
// call e + 1, after the peer's call e — and with it the peer's copies out
// of bank e & 1 — has completed; so when this rank stores call e + 2 into a
// peer's bank e & 1, that peer no longer reads call e there.  Two banks are
// therefore enough.  The same bound means a peer's ready[q][c] may already
// be at e + 1 (it has moved on to the other bank), so the wait is for it to
// have reached e (wrap-safe: (int)(flag - e) >= 0), not to equal it.  The grid
// is at most one CTA per SM, so all CTAs of a rank are resident together.
// Ranks must make the same sequence of calls with the same shapes and
// equally aligned buffers (the alignment picks the protocol).  A wait that runs out sets
// kDevErrPeerWait in the device error word and the kernel carries on (the
// affected columns are then stale).
#pragma once

#include "ql_common.cuh"

namespace ql {
namespace gather {

constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 256;   // CTAs of one gather launch (ready flags per rank)
constexpr long long kLineMaxPayload = 4ll << 20;   // bytes of output [M, N] fp16 sent as tagged lines
constexpr int kBatch = 4;    // loads a thread keeps in flight before its stores (push and copy loops)

struct Layout {
  size_t flags, state, data, lines, total;
  long long ldb;
  int line_rows;   // rows the line banks hold
};
__host__ __device__ inline Layout layout(int max_m, long long n) {
  Layout l;
  l.flags = 0;
  l.state = (size_t)kMaxRanks * kMaxCtas * 4;
  l.data = l.state + 256;
  l.ldb = (n + 7) / 8 * 8;
  l.lines = (l.data + (size_t)2 * max_m * l.ldb * 2 + 255) / 256 * 256;
  const long long fit = kLineMaxPayload / (2 * l.ldb);
  l.line_rows = (int)(fit < 1 ? 0 : (fit < max_m ? fit : max_m));
  l.total = (l.lines + (size_t)2 * l.line_rows * l.ldb * 4 + 255) / 256 * 256;
  return l;
}

struct Params {
  const __half* src;      // this rank's columns [M, groups*w] (ld lds), or nullptr: already in out
  long long lds;
  __half* out;            // [M, ldo]
  long long ldo;
  long long ng, block;    // columns per group; shard width per group
  int M, groups, rank, world, max_m;
  int cw;                 // columns per unit of the flagged protocol: 8 when ng and block are
                          // multiples of 8, else 1 (shapes only: the same on every rank)
  int vec;                // 16-byte accesses (cw == 8, 16-byte aligned pointers and strides)
  int lines;              // tagged-line protocol (4-aligned offsets, widths, strides; M <= line_rows)
  unsigned char* peer[kMaxRanks];   // gather buffer of every rank (peer[rank] = own)
  unsigned* err;
};

// One release fence, then plain (relaxed, system-scope) flag stores: each
// st.release would wait for the stores before it — the earlier flags to
// other GPUs included — to be acknowledged over NVLink.
__device__ __forceinline__ void fence_release_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void st_relaxed_sys(unsigned* p, unsigned v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// A peer's flag has reached call e (it may already be at e + 1, never
// further: see the header); wrap-safe over the 32-bit epoch.
__device__ __forceinline__ bool flag_reached(unsigned flag, unsigned e) { return (int)(flag - e) >= 0; }

// Columns of rank q within one group.
__device__ __forceinline__ long long shard_width(const Params& p, int q) {
  const long long c0 = (long long)q * p.block;
  return c0 >= p.ng ? 0 : min(p.block, p.ng - c0);
}

// A line is two 8-byte words {2 fp16 | tag << 32}; each word is one
// naturally aligned 64-bit element, read and written whole (single-copy
// atomic), so a word whose tag reads e carries this call's columns.
__device__ __forceinline__ void st_line(uint4* p, unsigned long long a, unsigned long long b) {
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ld_line(const uint4* p, unsigned long long& a, unsigned long long& b) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Unit i of rank q's [M, groups*w] slice (units of `vw` columns; i <
// M*groups*wu) -> its row m, its column j within the slice and its global
// column col, both in units.
__device__ __forceinline__ void locate(int groups, long long ngu, long long bu, int q, long long wu, long long i,
                                       int& m, long long& j, long long& col) {
  const long long per_row = (long long)groups * wu;
  m = (int)(i / per_row);
  j = i - (long long)m * per_row;
  const long long g = j / wu;
  col = g * ngu + (long long)q * bu + (j - g * wu);
}

// Tagged-line protocol (units of 4 columns): push this rank's columns as
// lines into every peer's bank e & 1, count the CTA in (the last one
// advances the epoch), then read every peer's lines of this call as they
// arrive.  A thread whose wait runs out records the error and stops waiting.
__device__ __forceinline__ void gather_lines(const Params& p, const Layout& L, unsigned e, unsigned* counter,
                                             unsigned* epoch_done) {
  const long long nthr = (long long)gridDim.x * blockDim.x;
  const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long ngu = p.ng / 4, bu = p.block / 4, ldl = L.ldb / 4;
  const size_t bank = (size_t)(e & 1u) * L.line_rows * ldl;
  {
    const long long wu = shard_width(p, p.rank) / 4;
    const long long units = (long long)p.M * p.groups * wu;
    const unsigned long long tag = (unsigned long long)e << 32;
    for (long long i0 = tid; i0 < units; i0 += kBatch * nthr) {
      // kBatch loads in flight per thread before any store
      uint2 v[kBatch];
      int mm[kBatch];
      long long cc[kBatch];
      #pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const long long i = i0 + u * nthr;
        mm[u] = -1;
        if (i < units) {
          long long j;
          locate(p.groups, ngu, bu, p.rank, wu, i, mm[u], j, cc[u]);
          v[u] = p.src ? *reinterpret_cast<const uint2*>(p.src + (long long)mm[u] * p.lds + j * 4)
                       : *reinterpret_cast<const uint2*>(p.out + (long long)mm[u] * p.ldo + cc[u] * 4);
        }
      }
      #pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        if (mm[u] < 0) continue;
        if (p.src) *reinterpret_cast<uint2*>(p.out + (long long)mm[u] * p.ldo + cc[u] * 4) = v[u];
        const unsigned long long wa = tag | v[u].x, wb = tag | v[u].y;
        for (int k = 1; k < p.world; ++k) {
          const int q = (p.rank + k) % p.world;
          st_line(reinterpret_cast<uint4*>(p.peer[q] + L.lines) + bank + (long long)mm[u] * ldl + cc[u], wa, wb);
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(counter, 1u) == gridDim.x - 1) {
    *reinterpret_cast<volatile unsigned*>(counter) = 0u;     // every CTA has read the epoch
    *reinterpret_cast<volatile unsigned*>(epoch_done) = e;
  }
  const uint4* lines = reinterpret_cast<const uint4*>(p.peer[p.rank] + L.lines) + bank;
  bool waiting = true;
  for (int k = 1; k < p.world; ++k) {
    const int q = (p.rank + k) % p.world;
    const long long wu = shard_width(p, q) / 4;
    const long long units = (long long)p.M * p.groups * wu;
    for (long long i0 = tid; i0 < units; i0 += kBatch * nthr) {
      unsigned long long wa[kBatch], wb[kBatch];
      int mm[kBatch];
      long long cc[kBatch];
      #pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const long long i = i0 + u * nthr;
        mm[u] = -1;
        if (i < units) {
          long long j;
          locate(p.groups, ngu, bu, q, wu, i, mm[u], j, cc[u]);
          ld_line(lines + (long long)mm[u] * ldl + cc[u], wa[u], wb[u]);
        }
      }
      #pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        if (mm[u] < 0) continue;
        const uint4* src = lines + (long long)mm[u] * ldl + cc[u];
        if (((unsigned)(wa[u] >> 32) != e || (unsigned)(wb[u] >> 32) != e) && waiting) {
          const long long t0 = clock64();
          for (;;) {
            ld_line(src, wa[u], wb[u]);
            if ((unsigned)(wa[u] >> 32) == e && (unsigned)(wb[u] >> 32) == e) break;
            if (clock64() - t0 > kWaitBudgetCycles) {
              atomicCAS(p.err, 0u, kDevErrPeerWait);
              waiting = false;
              break;
            }
            __nanosleep(32);
          }
        }
        *reinterpret_cast<uint2*>(p.out + (long long)mm[u] * p.ldo + cc[u] * 4) =
            make_uint2((unsigned)wa[u], (unsigned)wb[u]);
      }
    }
  }
}

__global__ void __launch_bounds__(512) allgather_kernel(const Params p) {
  __shared__ unsigned done_s;
  griddep_wait();   // this rank's columns come from the kernel before

  const Layout L = layout(p.max_m, (long long)p.groups * p.ng);
  unsigned char* own = p.peer[p.rank];
  unsigned* flags = reinterpret_cast<unsigned*>(own + L.flags);
  unsigned* counter = reinterpret_cast<unsigned*>(own + L.state);
  unsigned* epoch_done = counter + 1;
  if (threadIdx.x == 0) done_s = *reinterpret_cast<volatile unsigned*>(epoch_done);
  __syncthreads();
  const unsigned e = done_s + 1u;
  if (p.lines) {
    gather_lines(p, L, e, counter, epoch_done);
    return;
  }
  const size_t bank = (size_t)(e & 1u) * p.max_m * L.ldb;
  const long long ngu = p.ng / p.cw, bu = p.block / p.cw;
  // chunk c of rank q's columns: units [c * U / G, (c + 1) * U / G) of its
  // [M, groups*w] slice, U = M * groups * w / cw.  cw, G and the shard
  // widths depend on the shapes alone, so every rank splits rank q's
  // columns the same way.
  auto chunk = [&](int q, long long& wu, long long& u0, long long& u1) {
    wu = shard_width(p, q) / p.cw;
    const long long units = (long long)p.M * p.groups * wu;
    u0 = units * blockIdx.x / gridDim.x;
    u1 = units * (blockIdx.x + 1) / gridDim.x;
  };

  // ---- 1. this rank's chunk into every peer's bank (and into out if staged)
  {
    long long wu, u0, u1;
    chunk(p.rank, wu, u0, u1);
    if (p.vec) {
      for (long long i0 = u0 + threadIdx.x; i0 < u1; i0 += kBatch * blockDim.x) {
        uint4 v[kBatch];
        int mm[kBatch];
        long long cc[kBatch];
        #pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const long long i = i0 + u * blockDim.x;
          mm[u] = -1;
          if (i < u1) {
            long long j;
            locate(p.groups, ngu, bu, p.rank, wu, i, mm[u], j, cc[u]);
            cc[u] *= 8;
            v[u] = p.src ? *reinterpret_cast<const uint4*>(p.src + (long long)mm[u] * p.lds + j * 8)
                         : __ldcg(reinterpret_cast<const uint4*>(p.out + (long long)mm[u] * p.ldo + cc[u]));
          }
        }
        #pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          if (mm[u] < 0) continue;
          if (p.src) *reinterpret_cast<uint4*>(p.out + (long long)mm[u] * p.ldo + cc[u]) = v[u];
          for (int k = 1; k < p.world; ++k) {
            const int q = (p.rank + k) % p.world;
            __half* dst = reinterpret_cast<__half*>(p.peer[q] + L.data) + bank + (long long)mm[u] * L.ldb + cc[u];
            *reinterpret_cast<uint4*>(dst) = v[u];
          }
        }
      }
    } else {
      for (long long i = u0 + threadIdx.x; i < u1; i += blockDim.x) {
        int m;
        long long j, col;
        locate(p.groups, ngu, bu, p.rank, wu, i, m, j, col);
        for (int t = 0; t < p.cw; ++t) {
          const long long jj = j * p.cw + t, cl = col * p.cw + t;
          const __half v = p.src ? p.src[(long long)m * p.lds + jj] : p.out[(long long)m * p.ldo + cl];
          if (p.src) p.out[(long long)m * p.ldo + cl] = v;
          for (int k = 1; k < p.world; ++k) {
            const int q = (p.rank + k) % p.world;
            reinterpret_cast<__half*>(p.peer[q] + L.data)[bank + (long long)m * L.ldb + cl] = v;
          }
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // release: every thread's peer stores (ordered before this thread's by
    // the barrier) become visible system-wide before any of the flags
    fence_release_sys();
    for (int k = 1; k < p.world; ++k) {
      const int q = (p.rank + k) % p.world;
      st_relaxed_sys(reinterpret_cast<unsigned*>(p.peer[q] + L.flags) + p.rank * kMaxCtas + blockIdx.x, e);
    }
    // the epoch advances once every CTA has read it (local bookkeeping only)
    if (atomicAdd(counter, 1u) == gridDim.x - 1) {
      *reinterpret_cast<volatile unsigned*>(counter) = 0u;
      *reinterpret_cast<volatile unsigned*>(epoch_done) = e;
    }
  }

  // ---- 2. peers in turn: wait for their chunk c, copy it out of the bank
  for (int k = 1; k < p.world; ++k) {
    const int q = (p.rank + k) % p.world;
    long long wu, u0, u1;
    chunk(q, wu, u0, u1);
    if (threadIdx.x == 0) {
      const unsigned* f = flags + q * kMaxCtas + blockIdx.x;
      if (!flag_reached(ld_acquire_sys(f), e)) {
        const long long t0 = clock64();
        while (!flag_reached(ld_acquire_sys(f), e)) {
          if (clock64() - t0 > kWaitBudgetCycles) {
            atomicCAS(p.err, 0u, kDevErrPeerWait);
            break;
          }
          __nanosleep(64);
        }
      }
    }
    __syncthreads();
    const __half* data = reinterpret_cast<const __half*>(own + L.data) + bank;
    if (p.vec) {
      for (long long i0 = u0 + threadIdx.x; i0 < u1; i0 += kBatch * blockDim.x) {
        uint4 v[kBatch];
        int mm[kBatch];
        long long cc[kBatch];
        #pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const long long i = i0 + u * blockDim.x;
          mm[u] = -1;
          if (i < u1) {
            long long j;
            locate(p.groups, ngu, bu, q, wu, i, mm[u], j, cc[u]);
            cc[u] *= 8;
            v[u] = __ldcg(reinterpret_cast<const uint4*>(data + (long long)mm[u] * L.ldb + cc[u]));
          }
        }
        #pragma unroll
        for (int u = 0; u < kBatch; ++u)
          if (mm[u] >= 0) *reinterpret_cast<uint4*>(p.out + (long long)mm[u] * p.ldo + cc[u]) = v[u];
      }
    } else {
      for (long long i = u0 + threadIdx.x; i < u1; i += blockDim.x) {
        int m;
        long long j, col;
        locate(p.groups, ngu, bu, q, wu, i, m, j, col);
        for (int t = 0; t < p.cw; ++t) {
          const long long cl = col * p.cw + t;
          p.out[(long long)m * p.ldo + cl] = __ldcg(data + (long long)m * L.ldb + cl);
        }
      }
    }
  }
}

}  // namespace gather
}  // namespace ql
