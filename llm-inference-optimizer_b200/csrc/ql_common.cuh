// ql_common.cuh — device helpers shared by the qlinear kernels (sm_100a).
//
// Inline-PTX wrappers for mbarriers, TMA bulk-tensor loads, programmatic
// dependent launch, named barriers and mma.sync, plus the register-level
// decoders that turn packed int4 / int8 weights into exact fp16 pairs.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace ql {

// ------------------------------------------------------------------ errors
// Device-global error word.  A kernel whose bounded wait runs out stores a
// code here (first writer wins), lets its in-flight copies and tensor-core
// operations finish, and returns without trapping.
enum DeviceError : unsigned {
  kDevErrNone = 0,
  kDevErrFullWait = 1,      // consumer waited too long for a TMA stage
  kDevErrEmptyWait = 2,     // producer waited too long for a free stage
  kDevErrMmaWait = 3,       // tensor-core completion wait ran out
  kDevErrTmem = 4,          // TMEM allocation failed
  kDevErrPeerWait = 5,      // another rank's exchange data never arrived
};

// Budget of any single bounded wait, in SM clock cycles.  %clock64 is
// per-SM and monotonic: 4e9 cycles is about 2 s at the 1.965 GHz boost
// clock, and longer when the clock is lower.
constexpr long long kWaitBudgetCycles = 4000000000ll;

// ------------------------------------------------------------ addressing
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// --------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  // make the initialised barriers visible to the async (TMA) proxy
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait on the phase with the given parity.  Returns false when the
// budget runs out (the first code is recorded in the device error word) or,
// when `abort` is given, as soon as *abort is non-zero (another warp of the
// same CTA has given up).  The error word is only written here, never read,
// so an error left behind by an earlier launch cannot end this one's waits.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned* err_word, unsigned code,
                                          const volatile int* abort = nullptr) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (;;) {
    #pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (abort != nullptr && *abort != 0) return false;
    if (clock64() - t0 > kWaitBudgetCycles) {
      atomicCAS(err_word, 0u, code);
      return false;
    }
  }
}

// ------------------------------------------------------- arrival counters
// Fetch-and-add with acquire-release semantics at GPU scope: the caller's
// (and, through a preceding CTA barrier, its CTA's) writes are released
// before the add, and the reads that follow see what the earlier arrivals
// released.  One instruction instead of fence + atomic + fence.
__device__ __forceinline__ unsigned atomic_add_acq_rel_gpu(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// -------------------------------------------------------------------- TMA
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* tm) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// 2-D tiled bulk-tensor load global -> shared, completion on an mbarrier.
// Plain per-CTA loads only (nothing shared across a cluster).
__device__ __forceinline__ void tma_load_2d(uint32_t smem_dst, const CUtensorMap* tm, int x, int y,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// 3-D tiled bulk-tensor load global -> shared, completion on an mbarrier.
__device__ __forceinline__ void tma_load_3d(uint32_t smem_dst, const CUtensorMap* tm, int x, int y, int z,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// ---------------------------------------------- programmatic dependent launch
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------- named barriers
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------------ memory ops
__device__ __forceinline__ float lds_f16_as_f32(uint32_t addr) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return __half2float(__ushort_as_half(v));
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}
__device__ __forceinline__ uint4 ldg_cg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// ------------------------------------------------------------- tensor ops
// D(16x8,f32) += A(16x16,f16,row) * B(16x8,f16,col)
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ------------------------------------------------------- weight decoders
// All decoders build fp16 values with the exponent of 1024 ("magic number"
// construction: 0x6400 | v is the half 1024 + v for 0 <= v < 1024) and
// subtract the offset in half precision.  Every intermediate is an integer
// below 2048, so each result is the exact small integer.
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t bits) {
  uint32_t r;
  // r = (a & mask) | bits   (truth table 0xEA)
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(bits));
  return r;
}
__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
  __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
  __half2 r = __hfma2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b),
                      *reinterpret_cast<__half2*>(&c));
  return *reinterpret_cast<uint32_t*>(&r);
}

constexpr uint32_t kH2Magic = 0x64006400u;     // (1024, 1024)
constexpr uint32_t kH2_1032 = 0x64086408u;     // (1032, 1032): 1024 + 8
constexpr uint32_t kH2_1152 = 0x64806480u;     // (1152, 1152): 1024 + 128
constexpr uint32_t kH2_1_16 = 0x2C002C00u;     // (1/16, 1/16)
constexpr uint32_t kH2_m72 = 0xD480D480u;      // (-72, -72): 64 + 8

// Split-half int4 (the reference's layout).  u holds 4 consecutive packed
// bytes b0..b3 of one group; their low nibbles are k = j..j+3 and their high
// nibbles k = j+64..j+67.  Outputs are (q-8) as half2 pairs:
//   lo01 = (k j,   k j+1)     lo23 = (k j+2,  k j+3)
//   hi01 = (k j+64, k j+65)   hi23 = (k j+66, k j+67)
__device__ __forceinline__ void dec_w4_split(uint32_t u, uint32_t& lo01, uint32_t& lo23,
                                             uint32_t& hi01, uint32_t& hi23) {
  const uint32_t t0 = __byte_perm(u, 0u, 0x1100);   // byte0 = b0, byte2 = b1
  const uint32_t t1 = __byte_perm(u, 0u, 0x3322);   // byte0 = b2, byte2 = b3
  lo01 = h2_sub(lop3_and_or(t0, 0x000F000Fu, kH2Magic), kH2_1032);
  lo23 = h2_sub(lop3_and_or(t1, 0x000F000Fu, kH2Magic), kH2_1032);
  // (1024 + 16 h) / 16 - 72 = h - 8
  hi01 = h2_fma(lop3_and_or(t0, 0x00F000F0u, kH2Magic), kH2_1_16, kH2_m72);
  hi23 = h2_fma(lop3_and_or(t1, 0x00F000F0u, kH2Magic), kH2_1_16, kH2_m72);
}

// The same nibbles decoded without byte permutes, for activations staged in
// a permuted k order (stage_x_perm):
//   split-half: u = bytes b0..b3 (k j..j+3 low, k j+64.. high nibbles) ->
//     lo02 = (k0, k2), lo13 = (k1, k3), hi02 = (k64, k66), hi13 = (k65, k67)
//   adjacent:   u = k 0..7 -> p04 = (k0, k4), p15 = (k1, k5), p26, p37
// Exact: the same integer values as the decoders above, in another order.
__device__ __forceinline__ void dec_w4_split_perm(uint32_t u, uint32_t& lo02, uint32_t& lo13,
                                                  uint32_t& hi02, uint32_t& hi13) {
  const uint32_t v = u >> 8;
  lo02 = h2_sub(lop3_and_or(u, 0x000F000Fu, kH2Magic), kH2_1032);
  lo13 = h2_sub(lop3_and_or(v, 0x000F000Fu, kH2Magic), kH2_1032);
  hi02 = h2_fma(lop3_and_or(u, 0x00F000F0u, kH2Magic), kH2_1_16, kH2_m72);
  hi13 = h2_fma(lop3_and_or(v, 0x00F000F0u, kH2Magic), kH2_1_16, kH2_m72);
}
__device__ __forceinline__ void dec_w4_adjacent_perm(uint32_t u, uint32_t& p04, uint32_t& p15,
                                                     uint32_t& p26, uint32_t& p37) {
  const uint32_t v = u >> 8;
  p04 = h2_sub(lop3_and_or(u, 0x000F000Fu, kH2Magic), kH2_1032);
  p15 = h2_fma(lop3_and_or(u, 0x00F000F0u, kH2Magic), kH2_1_16, kH2_m72);
  p26 = h2_sub(lop3_and_or(v, 0x000F000Fu, kH2Magic), kH2_1032);
  p37 = h2_fma(lop3_and_or(v, 0x00F000F0u, kH2Magic), kH2_1_16, kH2_m72);
}
// Activation words (8 halves, k 0..7) in the order the permuted decoders
// pair them: split-half (k0,k2)(k1,k3)(k4,k6)(k5,k7); adjacent
// (k0,k4)(k1,k5)(k2,k6)(k3,k7).
template <int LAYOUT>
__device__ __forceinline__ uint4 stage_x_perm(uint4 v) {
  uint4 r;
  if (LAYOUT == 0) {
    r.x = __byte_perm(v.x, v.y, 0x5410);
    r.y = __byte_perm(v.x, v.y, 0x7632);
    r.z = __byte_perm(v.z, v.w, 0x5410);
    r.w = __byte_perm(v.z, v.w, 0x7632);
  } else {
    r.x = __byte_perm(v.x, v.z, 0x5410);
    r.y = __byte_perm(v.x, v.z, 0x7632);
    r.z = __byte_perm(v.y, v.w, 0x5410);
    r.w = __byte_perm(v.y, v.w, 0x7632);
  }
  return r;
}

// Adjacent-pair int4: byte i holds k = 2i (low nibble) and 2i+1 (high).
// u = bytes b0..b3 -> k 0..7; outputs p01 = (k0,k1), p23, p45, p67.
__device__ __forceinline__ void dec_w4_adjacent(uint32_t u, uint32_t& p01, uint32_t& p23,
                                                uint32_t& p45, uint32_t& p67) {
  const uint32_t v = u >> 4;
  p01 = h2_sub(lop3_and_or(__byte_perm(u, v, 0x4400), 0x000F000Fu, kH2Magic), kH2_1032);
  p23 = h2_sub(lop3_and_or(__byte_perm(u, v, 0x5511), 0x000F000Fu, kH2Magic), kH2_1032);
  p45 = h2_sub(lop3_and_or(__byte_perm(u, v, 0x6622), 0x000F000Fu, kH2Magic), kH2_1032);
  p67 = h2_sub(lop3_and_or(__byte_perm(u, v, 0x7733), 0x000F000Fu, kH2Magic), kH2_1032);
}

// int8: u = 4 signed bytes (k 0..3) -> p01 = (k0,k1), p23 = (k2,k3), exact.
__device__ __forceinline__ void dec_w8(uint32_t u, uint32_t& p01, uint32_t& p23) {
  const uint32_t v = u ^ 0x80808080u;                      // b + 128 in 0..255
  p01 = h2_sub(__byte_perm(v, 0x64646464u, 0x4140), kH2_1152);
  p23 = h2_sub(__byte_perm(v, 0x64646464u, 0x4342), kH2_1152);
}

__device__ __forceinline__ float2 h2_to_f2(uint32_t h) {
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

}  // namespace ql
