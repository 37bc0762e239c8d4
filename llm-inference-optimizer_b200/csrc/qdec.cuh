// qdec.cuh — small-batch (decode-shaped) dequant-fused linear on the 5th-gen
// tensor cores: tcgen05.mma with the decoded weights in TMEM.
//
// Replaces the reference's Triton kernels for small M
// (_w8a16_matmul_kernel, src/kernels/w8a16_matmul_triton.py:39-86;
//  _w4a16_matmul_kernel, src/kernels/w4a16_matmul_triton.py:62-117).
//
// Why not mma.sync: at M <= 8 a warp-level m16n8k16 spends 7/8 of its work
// on padding, and on B200 the legacy tensor pipe takes about 8 SM cycles per
// m16n8k16, which caps an int4 GEMV (16 of them per 2 KB of packed weights)
// near 4.6 TB/s.  tcgen05 has no such cap; what remains is decoding the
// weights, which this kernel does with five instructions per eight int4.
//
// Swap-AB: D[n, m] = sum_k W[n, k] * x[m, k].  A CTA owns 128 weight rows
// (UMMA M = 128; thread = row = TMEM lane) and a range of 128-k blocks
// (gridDim.z K-splits form one thread-block cluster and reduce through
// distributed shared memory); the batch is the UMMA N side (BN = 16 or 32).
//   * warp 0 (one thread): TMA producer.  Stage i = the tile's packed rows
//     for 128-k block i (64 B per row for int4 with 64-byte swizzle, 128 B
//     for int8 with 128-byte swizzle).  Weights do not depend on the kernel
//     before (programmatic dependent launch): the first ring-full is issued
//     before anything else.
//   * warps 2-9: two sets of four warps (one per TMEM lane quarter); set h
//     decodes the blocks g with g % 2 == h into TMEM A slots (64 columns =
//     128 k as fp16 pairs), runs that block's epilogue and, for the first
//     blocks, does so before waiting for the kernel before.
//   * warp 1 (one thread): issues tcgen05.mma.cta_group::1.kind::f16 (A from
//     TMEM, B = the activations in shared memory by descriptor, fp32 D in
//     TMEM), eight K=16 steps per block, and commits each block back.
//
// Decode without the offset subtraction.  int4 code q (0..15, weight q - 8):
// (v & 0x000F000F) | 0x6400 is the fp16 pair (1024 + q_a, 1024 + q_b) and
// (v & 0x00F000F0) | 0x6400 is (1024 + 16 q_a, 1024 + 16 q_b), one lop3 each;
// v >> 8 gives the other two bytes.  The activations that meet high nibbles
// are staged times 1/16 (exact in fp16), so a block's partial is
//     D = sum_lo (1024 + q) x + sum_hi (64 + q) x
//       = sum (q - 8) x + 1032 S_lo + 72 S_hi,
// with S_lo / S_hi the sums of the block's activations that meet low / high
// nibbles (computed once per CTA while staging).  The epilogue subtracts
// that and applies the block's group scale in fp32, in the same order as
// the reference kernel (partial of one 128-group times its scale,
// w4a16_matmul_triton.py:107-110).  int8: byte b gives 1152 + b with one
// xor and a byte permute; D - 1152 * sum(x), times the row scale at the end
// (w8a16_matmul_triton.py:74-76).  The pairs a decode produces are in a
// permuted k order (k, k+2), (k+1, k+3) for int4; the activations are staged
// in the same order, so each product meets its own activation.
//
// Bounded waits everywhere (ql_common.cuh); a wait that gives up records the
// device error word, the CTA stops, drains its copies and MMAs and frees
// its TMEM.
#pragma once

#include "qgemm.cuh"

namespace ql {
namespace dec {

constexpr int kRows = 128;       // weight rows per CTA = UMMA M = TMEM lanes
constexpr int kThreads = 320;    // producer, MMA, 8 decode/epilogue warps
constexpr int kDecThreads = 256;
constexpr int kNA = 3;           // A slots (64 TMEM columns each)
constexpr uint32_t kACol = 64;   // first A column; D uses columns [0, 64)
constexpr uint32_t kTmemCols = 256;
constexpr int kMaxSplits = 16;
constexpr int kMaxStages = 8;

struct Params {
  const __half* x;        // [M, ldx]
  const void* scale;      // int4: [K/128, lds] f16; int8: [N] f32 / f16
  const void* bias;       // [N] or nullptr
  __half* out;            // [M, ldo]
  long long ldx, lds, ldo;
  int M, N, K;
  int nkb;                // 128-k blocks of K
  int kb_split;           // blocks per K-split (gridDim.z splits)
  int stages;             // shared-memory ring depth (<= kMaxStages)
  int scale_f32, bias_f32;
  unsigned* err;
};

// Shared-memory carve-up (byte offsets from the 1024-aligned base), the same
// on host and device.
struct Smem {
  size_t ring, xs, sums, scl, comb, recv, bars, total;
};
template <int WBITS, int BN>
struct Tile {
  static constexpr int kWStage = kRows * (WBITS == 4 ? 64 : 128);   // packed bytes of one 128-k block
  static constexpr int kAtom = BN * 128;                             // 64 k x BN rows of fp16 (SW128)
  static constexpr uint32_t kDCols = WBITS == 4 ? 2 * BN : BN;       // int4: one partial per decode set
  static_assert(kDCols <= kACol, "D columns overlap the A slots");
  static_assert(kACol + kNA * 64 <= kTmemCols, "A slots exceed the allocation");
};
__host__ __device__ inline size_t al(size_t v, size_t a) { return (v + a - 1) / a * a; }
template <int WBITS, int BN>
__host__ __device__ inline Smem smem_plan(int stages, int kb_split, int ks) {
  using T = Tile<WBITS, BN>;
  Smem s;
  s.ring = 0;
  s.xs = al((size_t)stages * T::kWStage, 1024);
  s.sums = s.xs + (size_t)kb_split * 2 * T::kAtom;
  s.scl = al(s.sums + (size_t)kb_split * 2 * BN * 4, 16);
  s.comb = al(s.scl + (WBITS == 4 ? (size_t)kb_split * kRows * 4 : 0), 16);
  s.recv = al(s.comb + (size_t)BN * kRows * 4, 16);
  const size_t recv_bytes = ks > 1 ? (size_t)((BN * kRows + ks - 1) / ks) * ks * 4 : 0;
  s.bars = al(s.recv + recv_bytes, 16);
  s.total = 1024 /* base alignment */ + s.bars + 256;
  return s;
}

// 32 consecutive TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ uint4 h2x4_mul(uint4 v, uint32_t s) {
  v.x = gemm::h2_mul(v.x, s);
  v.y = gemm::h2_mul(v.y, s);
  v.z = gemm::h2_mul(v.z, s);
  v.w = gemm::h2_mul(v.w, s);
  return v;
}
__device__ __forceinline__ float sum8_f16(uint4 v) {
  const float2 a = h2_to_f2(v.x), b = h2_to_f2(v.y), c = h2_to_f2(v.z), d = h2_to_f2(v.w);
  return ((a.x + a.y) + (b.x + b.y)) + ((c.x + c.y) + (d.x + d.y));
}
// Sum over the 8 lanes of an aligned lane octet (fixed order: deterministic).
__device__ __forceinline__ float octet_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  return v;
}

template <int WBITS, int LAYOUT, int BN>
__global__ void __launch_bounds__(kThreads, 2)
    qdec_kernel(const __grid_constant__ CUtensorMap tmap_w, const Params p) {
  using T = Tile<WBITS, BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int S = p.stages;
  const int ks = (int)gridDim.z;
  const int n0 = (int)blockIdx.x * kRows;
  const int kb0 = (int)blockIdx.z * p.kb_split;
  const int G = min(p.kb_split, p.nkb - kb0);          // 128-k blocks of this CTA (>= 1)
  const Smem L = smem_plan<WBITS, BN>(S, p.kb_split, ks);
  uint8_t* ring = smem + L.ring;
  uint8_t* xs = smem + L.xs;                           // B operand: [2G atoms][BN rows][128 B] SW128
  float* sums = reinterpret_cast<float*>(smem + L.sums);   // [2G][BN] activation sums per atom
  float* scl = reinterpret_cast<float*>(smem + L.scl);     // int4: [G][128] group scales of the rows
  float* comb = reinterpret_cast<float*>(smem + L.comb);   // [BN][128] second decode set's partials
  float* recv = reinterpret_cast<float*>(smem + L.recv);   // split-K receive buffer
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* wfree = full + kMaxStages;
  uint64_t* afull = wfree + kMaxStages;
  uint64_t* afree = afull + kNA;
  uint64_t* dfull = afree + kNA;     // [2]: int4 per decode set; int8 uses [0] once
  uint64_t* dfree = dfull + 2;       // [2]
  uint64_t* xready = dfree + 2;
  uint64_t* dall = xready + 1;       // every MMA of the CTA has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dall + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full + s, 1);
      mbar_init(wfree + s, 4);
    }
    for (int a = 0; a < kNA; ++a) {
      mbar_init(afull + a, 4);
      mbar_init(afree + a, 1);
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(dfull + h, 1);
      mbar_init(dfree + h, 4);
    }
    mbar_init(xready, 1);
    mbar_init(dall, 1);
    *abort = 0;
    fence_barrier_init();
    // the first ring-full of weights: no dependency on the kernel before
    prefetch_tmap(&tmap_w);
    const uint64_t pol = l2_policy_evict_first();
    for (int i = 0; i < min(S, G); ++i) {
      mbar_arrive_expect_tx(full + i, (uint32_t)T::kWStage);
      tma_load_3d(smem_u32(ring + (size_t)i * T::kWStage), &tmap_w, 0, kb0 + i, n0, full + i, pol);
    }
  }
  if (warp == 1) gemm::tmem_alloc(smem_u32(tmem_slot), kTmemCols);
  gemm::tc_fence_before();
  __syncthreads();
  gemm::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      int issued = min(S, G);
      for (int i = S; i < G; ++i) {
        const int s = i % S;
        if (!mbar_wait(wfree + s, ((i / S) - 1) & 1, p.err, kDevErrEmptyWait, abort)) {
          *abort = 1;
          break;
        }
        mbar_arrive_expect_tx(full + s, (uint32_t)T::kWStage);
        tma_load_3d(smem_u32(ring + (size_t)s * T::kWStage), &tmap_w, 0, kb0 + i, n0, full + s, pol);
        issued = i + 1;
      }
      // every issued copy lands before the CTA may exit (only the last
      // stage issued on each slot can still be in flight)
      for (int s = 0; s < min(issued, S); ++s) {
        const int last = s + ((issued - 1 - s) / S) * S;
        mbar_wait(full + s, (last / S) & 1, p.err, kDevErrFullWait);
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = gemm::idesc_f16<BN>();
      bool ok = mbar_wait(xready, 0, p.err, kDevErrMmaWait, abort);
      for (int g = 0; ok && g < G; ++g) {
        const int a = g % kNA, h = g & 1;
        if (!mbar_wait(afull + a, (g / kNA) & 1, p.err, kDevErrMmaWait, abort) ||
            (WBITS == 4 && g >= 2 && !mbar_wait(dfree + h, ((g >> 1) - 1) & 1, p.err, kDevErrMmaWait, abort))) {
          ok = false;
          break;
        }
        gemm::tc_fence_after();
        const uint32_t d = tmem + (WBITS == 4 ? (uint32_t)(h * BN) : 0u);
        const uint32_t at = tmem + kACol + 64u * (uint32_t)a;
        const uint32_t xb = smem_u32(xs) + (uint32_t)(g * 2 * T::kAtom);
        #pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint64_t bd = gemm::desc_sw128(xb + (uint32_t)((j >> 2) * T::kAtom + (j & 3) * 32));
          const uint32_t acc = WBITS == 4 ? (j > 0 ? 1u : 0u) : ((g > 0 || j > 0) ? 1u : 0u);
          gemm::tc_mma_ts(d, at + 8u * (uint32_t)j, bd, idesc, acc);
        }
        gemm::tc_commit(afree + a);
        if (WBITS == 4) gemm::tc_commit(dfull + h);
      }
      if (!ok) *abort = 1;
      if (WBITS == 8) gemm::tc_commit(dfull);
      // no MMA may be in flight when the TMEM is released, on the error path too
      gemm::tc_commit(dall);
      mbar_wait(dall, 0, p.err, kDevErrMmaWait);
    }
  } else {
    // ------------------------------------------------ decode + epilogue
    const int quarter = warp & 3;                     // TMEM lane quarter of this warp
    const int set = (warp - 2) >> 2;                  // decode set: blocks g with g % 2 == set
    const int r = quarter * 32 + lane;                // weight row within the tile = TMEM lane
    const int n = n0 + r;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const int dtid = (int)threadIdx.x - 64;           // 0..255
    const int dwarp = dtid >> 5;

    // int4 group scales of the tile's rows (static data: before the wait)
    if (WBITS == 4) {
      const __half* sc = static_cast<const __half*>(p.scale);
      for (int idx = dtid; idx < G * kRows; idx += kDecThreads) {
        const int g = idx >> 7, rr = idx & (kRows - 1);
        scl[idx] = (n0 + rr < p.N) ? __half2float(sc[(long long)(kb0 + g) * p.lds + n0 + rr]) : 0.f;
      }
    }

    // decode block g into A slot g % kNA (this set's four warps): the packed
    // row goes to registers, the ring stage is released, then the low and
    // high halves (64 k each) are decoded and stored in two passes
    auto decode = [&](int g) -> bool {
      const int s = g % S;
      if (!__all_sync(0xffffffffu, mbar_wait(full + s, (g / S) & 1, p.err, kDevErrFullWait, abort))) return false;
      const uint32_t stg = smem_u32(ring + (size_t)s * T::kWStage);
      const int a = g % kNA;
      const uint32_t at = tmem + lane_base + kACol + 64u * (uint32_t)a;
      uint32_t cols[32];
      if (WBITS == 4) {
        // 64 bytes of row r (64-byte swizzle: chunk q at q ^ ((r >> 1) & 3))
        uint32_t w[16];
        #pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 v = lds128(stg + (uint32_t)(r * 64) + (uint32_t)((q ^ ((r >> 1) & 3)) << 4));
          w[4 * q] = v.x; w[4 * q + 1] = v.y; w[4 * q + 2] = v.z; w[4 * q + 3] = v.w;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(wfree + s);      // the packed stage is in registers
        if (g >= kNA &&
            !__all_sync(0xffffffffu, mbar_wait(afree + a, ((g / kNA) - 1) & 1, p.err, kDevErrFullWait, abort)))
          return false;
        gemm::tc_fence_after();
        #pragma unroll
        for (int j = 0; j < 16; ++j) {               // low nibbles: k = 4j .. 4j+3
          cols[2 * j] = lop3_and_or(w[j], 0x000F000Fu, kH2Magic);
          cols[2 * j + 1] = lop3_and_or(w[j] >> 8, 0x000F000Fu, kH2Magic);
        }
        tmem_st32(at, cols);
        #pragma unroll
        for (int j = 0; j < 16; ++j) {               // high nibbles: k = 64 + 4j ..
          cols[2 * j] = lop3_and_or(w[j], 0x00F000F0u, kH2Magic);
          cols[2 * j + 1] = lop3_and_or(w[j] >> 8, 0x00F000F0u, kH2Magic);
        }
        tmem_st32(at + 32u, cols);
      } else {
        // 128 bytes of row r (128-byte swizzle: chunk q at q ^ (r & 7)):
        // chunks 0-3 = k 0..63, chunks 4-7 = k 64..127, natural order
        if (g >= kNA &&
            !__all_sync(0xffffffffu, mbar_wait(afree + a, ((g / kNA) - 1) & 1, p.err, kDevErrFullWait, abort)))
          return false;
        gemm::tc_fence_after();
        #pragma unroll
        for (int pass = 0; pass < 2; ++pass) {
          uint4 v[4];
          #pragma unroll
          for (int q = 0; q < 4; ++q)
            v[q] = lds128(stg + (uint32_t)(r * 128) + (uint32_t)(((4 * pass + q) ^ (r & 7)) << 4));
          if (pass == 1) {
            __syncwarp();
            if (lane == 0) mbar_arrive(wfree + s);
          }
          #pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t wd[4] = {v[q].x ^ 0x80808080u, v[q].y ^ 0x80808080u, v[q].z ^ 0x80808080u,
                                    v[q].w ^ 0x80808080u};
            #pragma unroll
            for (int e = 0; e < 4; ++e) {
              cols[8 * q + 2 * e] = __byte_perm(wd[e], 0x64646464u, 0x4140);
              cols[8 * q + 2 * e + 1] = __byte_perm(wd[e], 0x64646464u, 0x4342);
            }
          }
          tmem_st32(at + 32u * (uint32_t)pass, cols);
        }
      }
      gemm::tmem_st_wait();
      gemm::tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(afull + a);
      return true;
    };

    bool ok = true;
    int gnext = set;                              // next block of this set to decode
    for (; ok && gnext < G && gnext < kNA; gnext += 2) ok = decode(gnext);
    if (!ok) *abort = 1;

    // ---- activations: staged once the kernel before has completed
    griddep_wait();
    {
      const int M = p.M;
      const int natoms = 2 * G;
      const uint32_t k16 = 0x2C002C00u;           // (1/16, 1/16)
      if (WBITS == 4 && LAYOUT == 1) {
        // adjacent pairs: block g, 16-k run c -> lo chunk c (even k) and hi chunk c (odd k, / 16)
        const int total = M * G * 8;
        for (int base = dwarp * 32; base < total; base += kDecThreads) {
          const int idx = base + lane;
          const bool act = idx < total;
          const int m = act ? idx / (G * 8) : 0;
          const int rem = idx - m * G * 8;
          const int g = rem >> 3, c = rem & 7;
          const int k = (kb0 + g) * 128 + 16 * c;
          uint4 a = make_uint4(0u, 0u, 0u, 0u), b = a;
          if (act && k < p.K) {
            const __half* src = p.x + (long long)m * p.ldx + k;
            a = ldg_cg_v4(src);
            b = ldg_cg_v4(src + 8);
          }
          uint4 lo, hi;
          lo.x = __byte_perm(a.x, a.z, 0x5410); lo.y = __byte_perm(a.y, a.w, 0x5410);
          lo.z = __byte_perm(b.x, b.z, 0x5410); lo.w = __byte_perm(b.y, b.w, 0x5410);
          hi.x = __byte_perm(a.x, a.z, 0x7632); hi.y = __byte_perm(a.y, a.w, 0x7632);
          hi.z = __byte_perm(b.x, b.z, 0x7632); hi.w = __byte_perm(b.y, b.w, 0x7632);
          const float slo = octet_sum(sum8_f16(lo)), shi = octet_sum(sum8_f16(hi));
          if (act) {
            const uint32_t off = (uint32_t)(m * 128) + (uint32_t)((c ^ (m & 7)) << 4);
            *reinterpret_cast<uint4*>(xs + (size_t)(2 * g) * T::kAtom + off) = lo;
            *reinterpret_cast<uint4*>(xs + (size_t)(2 * g + 1) * T::kAtom + off) = h2x4_mul(hi, k16);
            if (c == 0) {
              sums[(2 * g) * BN + m] = slo;
              sums[(2 * g + 1) * BN + m] = shi;
            }
          }
        }
      } else {
        // one 16-byte chunk c of atom b (64 k) per lane; 8 lanes per (row, atom)
        const int total = M * natoms * 8;
        for (int base = dwarp * 32; base < total; base += kDecThreads) {
          const int idx = base + lane;
          const bool act = idx < total;
          const int m = act ? idx / (natoms * 8) : 0;
          const int rem = idx - m * natoms * 8;
          const int b = rem >> 3, c = rem & 7;
          const int k = (kb0 + (b >> 1)) * 128 + (b & 1) * 64 + 8 * c;
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (act && k < p.K) v = ldg_cg_v4(p.x + (long long)m * p.ldx + k);
          if (WBITS == 4) v = stage_x_perm<0>(v);      // the decode's (k, k+2), (k+1, k+3) order
          const float sm = octet_sum(sum8_f16(v));
          if (act) {
            if (WBITS == 4 && (b & 1)) v = h2x4_mul(v, k16);
            *reinterpret_cast<uint4*>(xs + (size_t)b * T::kAtom + (uint32_t)(m * 128) +
                                      (uint32_t)((c ^ (m & 7)) << 4)) = v;
            if (c == 0) sums[b * BN + m] = sm;
          }
        }
      }
      fence_proxy_async_smem();                     // generic-proxy stores -> tcgen05.mma reads
      named_bar_sync(1, kDecThreads);
      if (dtid == 0) mbar_arrive(xready);
    }
    griddep_launch_dependents();

    // ---- blocks of this set: epilogue in order, then decode ahead.  The
    // epilogue of block g frees this set's D columns for the MMAs of block
    // g + 2, so it goes first; the decode runs up to kNA blocks ahead of the
    // MMAs (each A slot is reused once the MMAs of the block kNA earlier are
    // done).
    float acc[BN];
    #pragma unroll
    for (int m = 0; m < BN; ++m) acc[m] = 0.f;
    const int M = p.M;
    int kth = 0;                                   // blocks of this set finished
    for (int g = set; ok && g < G; g += 2, ++kth) {
      if (WBITS == 4) {
        if (!__all_sync(0xffffffffu, mbar_wait(dfull + set, kth & 1, p.err, kDevErrMmaWait, abort))) {
          ok = false;
          break;
        }
        gemm::tc_fence_after();
        const float s = scl[g * kRows + r];
        #pragma unroll
        for (int c8 = 0; c8 < BN / 8; ++c8) {
          if (8 * c8 >= M) break;                  // warp-uniform
          uint32_t v[8];
          gemm::tmem_ld8(tmem + lane_base + (uint32_t)(set * BN + 8 * c8), v);
          #pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int m = 8 * c8 + j;
            if (m < M) {
              const float cm = fmaf(1032.f, sums[(2 * g) * BN + m], 72.f * sums[(2 * g + 1) * BN + m]);
              acc[m] = fmaf(__uint_as_float(v[j]) - cm, s, acc[m]);
            }
          }
        }
        gemm::tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dfree + set);
      }
      if (gnext < G) {
        ok = decode(gnext);
        gnext += 2;
      }
    }
    // int8 has no per-block epilogue: the loop above only decodes; finish
    // the decode of this set's remaining blocks
    for (; ok && gnext < G; gnext += 2) ok = decode(gnext);
    if (!ok) *abort = 1;

    // ---- this CTA's partial of row r: set 1 hands its sums to set 0
    if (WBITS == 4 && set == 1) {
      #pragma unroll
      for (int m = 0; m < BN; ++m)
        if (m < M) comb[m * kRows + r] = acc[m];
    }
    named_bar_sync(1, kDecThreads);
    if (set == 0) {
      if (WBITS == 4) {
        #pragma unroll
        for (int m = 0; m < BN; ++m)
          if (m < M) acc[m] += comb[m * kRows + r];
      } else {
        // one accumulator over every block: subtract 1152 * sum(x), row scale
        const bool fine = __all_sync(0xffffffffu, mbar_wait(dfull, 0, p.err, kDevErrMmaWait, abort));
        gemm::tc_fence_after();
        const float s8 = n < p.N ? (p.scale_f32 ? static_cast<const float*>(p.scale)[n]
                                                : __half2float(static_cast<const __half*>(p.scale)[n]))
                                 : 0.f;
        #pragma unroll
        for (int c8 = 0; c8 < BN / 8; ++c8) {
          if (8 * c8 >= M || !fine) break;          // warp-uniform
          uint32_t v[8];
          gemm::tmem_ld8(tmem + lane_base + (uint32_t)(8 * c8), v);
          #pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int m = 8 * c8 + j;
            if (m < M) {
              float sx = 0.f;
              for (int b = 0; b < 2 * G; ++b) sx += sums[b * BN + m];
              acc[m] = (__uint_as_float(v[j]) - 1152.f * sx) * s8;
            }
          }
        }
      }
      if (ks == 1) {
        if (n < p.N) {
          const float bv = p.bias ? (p.bias_f32 ? static_cast<const float*>(p.bias)[n]
                                                : __half2float(static_cast<const __half*>(p.bias)[n]))
                                  : 0.f;
          #pragma unroll
          for (int m = 0; m < BN; ++m)
            if (m < M) p.out[(long long)m * p.ldo + n] = __float2half_rn(acc[m] + bv);
        }
      } else {
        // split-K: element e = m * 128 + r belongs to member e / sz, which
        // sums it; remote store into its receive buffer, slot of this rank
        const int E = M * kRows;
        const int sz = (E + ks - 1) / ks;
        const uint32_t me = gemm::cluster_rank();
        const uint32_t rbuf = smem_u32(recv);
        #pragma unroll
        for (int m = 0; m < BN; ++m) {
          if (m < M) {
            const int e = m * kRows + r;
            const int owner = e / sz;
            gemm::st_dsmem_f32(gemm::dsmem_addr(rbuf + (uint32_t)(me * sz + (e - owner * sz)) * 4u, (uint32_t)owner),
                               acc[m]);
          }
        }
      }
    }
  }

  if (ks > 1) {
    // ------------------------------------------------ cluster reduction
    gemm::cluster_sync_all();                   // every member's slices are in this CTA's buffer
    if (warp >= 2) {
      const int E = p.M * kRows;
      const int sz = (E + ks - 1) / ks;
      const int me = (int)gemm::cluster_rank();
      const int e0 = me * sz, e1 = min(E, e0 + sz);
      for (int e = e0 + (int)threadIdx.x - 64; e < e1; e += kDecThreads) {
        float v = 0.f;
        for (int q = 0; q < ks; ++q) v += recv[q * sz + (e - e0)];   // rank order
        const int nn = n0 + (e & (kRows - 1));
        const int m = e >> 7;
        if (nn < p.N) {
          const float bv = p.bias ? (p.bias_f32 ? static_cast<const float*>(p.bias)[nn]
                                                : __half2float(static_cast<const __half*>(p.bias)[nn]))
                                  : 0.f;
          p.out[(long long)m * p.ldo + nn] = __float2half_rn(v + bv);
        }
      }
    }
  }

  gemm::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    gemm::tc_fence_after();
    gemm::tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace dec
}  // namespace ql
