// qgemm.cuh — prefill-shaped (larger M) dequant-fused GEMM on the 5th-gen
// tensor cores (tcgen05 / TMEM).
//
// Replaces the reference's Triton kernels for large M
// (_w8a16_matmul_kernel, src/kernels/w8a16_matmul_triton.py:39-86;
//  _w4a16_matmul_kernel, src/kernels/w4a16_matmul_triton.py:62-117).
//
// "Swap-AB" formulation: D[n, m] = sum_k W[n, k] * x[m, k], so the
// dequantized weights are the MMA's A operand (M = 128 weight rows per CTA)
// and the activations are the B operand (N = BN activation rows per CTA).
//   * warp 0 (one thread): TMA producer (the first ring-full of weight
//     stages is issued before waiting for the kernel before).  Per 128-k stage it loads the
//     packed weight tile (128 rows x 64 B int4 / 128 B int8, 64/128-byte
//     swizzle, a 3-D view of the rows) and the activation tile (BN rows x
//     128 k as two 128-byte-swizzled K-major atoms), each completing on its
//     own barrier: the decode of the first stages (up to the A slots in
//     TMEM) runs while the kernel before finishes, and only the MMAs wait
//     for the activations.
//   * warps 2-9 (256 threads; thread = weight row = TMEM lane, two warps per
//     lane quarter, each decoding one half of the stage's 128 k): read the
//     row's packed bytes, decode them to fp16 in registers (int4: times the
//     fp16 group scale, one rounding per weight; int8: exact) and write them
//     into TMEM with tcgen05.st — the A operand never touches shared memory,
//     which keeps shared-memory bandwidth for the activations.
//   * warp 1 (one thread): issues tcgen05.mma.cta_group::1.kind::f16
//     (A from TMEM, B from shared memory by descriptor, fp32 accumulator
//     in TMEM) and tcgen05.commit's the stage back to producer/dequant.
//     Activation tiles of up to 64 rows add a second issuer (warp 10) that
//     takes the odd stages into a second accumulator: measured on B200, a
//     thread issuing K = 16 MMAs back to back gets one through every ~57
//     cycles or more whatever N is, while two issuers together reach ~40
//     (N = 16) to ~64 (N = 128, the dense peak).  The epilogue adds the two
//     accumulators in a fixed order.
//   * epilogue (warps 2-9, each half of the activation columns): tcgen05.ld
//     of the accumulator(s), int8 row scale and bias in fp32, fp16 store (32
//     consecutive n per warp per activation row).
//   * split-K (grids with fewer tiles than SMs): the K-splits of one tile
//     are one thread-block cluster (cluster dims 1 x 1 x splits, at most 16);
//     every member sums a 1/splits slice of the tile in rank order
//     (deterministic) and stores it.  Narrow activation tiles (16/32 rows)
//     push: each CTA stores its partial's elements straight into the
//     receive buffer of the member that sums them, and one cluster barrier
//     publishes them.  Wider tiles pull: each CTA parks its partial in its
//     drained stage ring, the cluster meets, the members read the slices
//     they sum through distributed shared memory, and a second barrier keeps
//     every CTA resident until its partial has been read.  No workspace, no
//     atomics, no L2 round trip.
// Per-CTA TMA loads only (no multicast); every mbarrier wait is bounded, and
// every thread reaches the cluster barriers after its bounded waits.
#pragma once

#include "ql_common.cuh"

namespace ql {
namespace gemm {

constexpr int kTileN = 128;     // weight rows per CTA = UMMA M
constexpr int kBK = 128;        // k per stage = 8 MMAs of K=16
// Warps: 0 producer, 1 MMA issuer, 2-9 dequant/epilogue, and (activation
// tiles of up to 64 rows) 10 the second MMA issuer; Layout::kThreads.
constexpr int kIssuer1Warp = 10;

struct Params {
  const void* scale;      // int8: [N] f32/f16; int4: [K/128, lds] f16
  const void* bias;       // [N] or nullptr
  __half* out;            // [M, ldo]
  long long lds, ldo;
  int M, N, K;
  int nk;                 // number of 128-k stages of K
  int nk_split;           // stages per K-split (gridDim.z splits = cluster size)
  int stages;             // shared-memory ring depth
  int scale_f32, bias_f32;
  // SwiGLU mode (nh > 0): the weight is a stacked [gate; up] of 2*nh rows
  // and out[M, nh] = silu(x gate^T) * (x up^T).  Tile x then holds gate
  // rows [64x, 64x + 64) in its TMEM lanes 0-63 and the matching up rows
  // in lanes 64-127 (two 64-row weight boxes per stage), so both factors of
  // an output meet in one CTA.  Unsplit launches and pull-mode K-splits.
  int nh;
  unsigned* err;
};

// Weight row held in TMEM lane r of tile `tile` (-1: past the weight).
__device__ __forceinline__ int tile_row(const Params& p, int tile, int r) {
  if (p.nh == 0) {
    const int n = tile * kTileN + r;
    return n < p.N ? n : -1;
  }
  const int c = tile * (kTileN / 2) + (r & (kTileN / 2 - 1));   // output column
  if (c >= p.nh) return -1;
  return r < kTileN / 2 ? c : p.nh + c;
}

// Largest K-split = thread-block cluster size (beyond the portable 8: the
// kernels are marked for non-portable cluster sizes, which B200 runs up to 16).
constexpr int kMaxSplits = 16;

template <int WBITS, int BN>
struct Layout {
  static constexpr int kWStage = kTileN * (WBITS == 4 ? 64 : 128);
  static constexpr int kXAtom = BN * 128;           // 64 k x BN rows of fp16
  static constexpr int kXStage = 2 * kXAtom;
  static constexpr int kStage = kXStage + kWStage;  // multiple of 1024
  // A (dequantized weight) stages in TMEM, 64 columns each from kACol: the
  // narrow tiles' accumulator leaves room for three, so the decode runs
  // three stages ahead of the MMAs (and, before the dependency wait, of
  // the activations)
  static constexpr int kASlots = BN <= 32 ? 3 : 2;
  static constexpr uint32_t kACol = BN <= 32 ? 64 : BN <= 128 ? 128 : 256;  // first A column
  static constexpr uint32_t kTmemCols = kACol + kASlots * 64 <= 256 ? 256 : 512;
  // second MMA issuer and accumulator (columns [BN, 2 BN), below kACol)
  static constexpr bool kTwoIssuers = BN <= 64;
  static constexpr int kThreads = kTwoIssuers ? 352 : 320;
  static_assert((kTwoIssuers ? 2 * BN : BN) <= (int)kACol, "accumulators overlap the A slots");
  // mbarriers (wfull, xfull, wfree, xfree per stage, afull / afree per A
  // slot, dfull), TMEM address and abort flag in the 256 bytes after the ring
  static_assert((4 * 6 + 2 * kASlots + 1) * 8 + 8 <= 256, "barrier area");
  // Split-K reduction: narrow tiles push their partial into the members'
  // receive buffers (one cluster barrier); wide tiles park it in the
  // drained ring and the members pull (two barriers, no extra memory).
  static constexpr bool kPush = BN <= 32;   // measured: 64-row tiles pull faster
  // receive buffer [splits][ceil(BN*128/splits)] fp32 (push mode)
  static constexpr size_t kRecvBytes = (((size_t)BN * kTileN + kMaxSplits) * 4 + 1023) / 1024 * 1024;
  __host__ __device__ static constexpr size_t kRecvOffset(int stages) { return (size_t)stages * kStage + 256; }
  static size_t smem_bytes(int stages, bool split = false) {
    return 1024 + (size_t)stages * kStage + 256 + (split && kPush ? kRecvBytes : 0);
  }
  // pull mode: the fp32 partial [BN][128] is parked in the drained ring
  static bool partial_fits(int stages) { return kPush || (size_t)BN * kTileN * 4 <= (size_t)stages * kStage; }
};

// ------------------------------------------------------ cluster helpers
// Arrive (release) and wait (acquire) on the cluster barrier; not .aligned,
// so the threads of a warp may arrive at different times.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// Address of the same shared-memory offset in cluster member `rank`.
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void st_dsmem_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// ----------------------------------------------------------- tcgen05 ops
__device__ __forceinline__ void tmem_alloc(uint32_t slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16, fp32 accumulate
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 8 consecutive fp32 accumulator columns of this thread's TMEM lane, not
// waited (tmem_ld_wait before use).
__device__ __forceinline__ void tmem_ld8_async(uint32_t taddr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(taddr)
               : "memory");
}
// 8 consecutive fp32 accumulator columns of this thread's TMEM lane, waited.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(taddr)
               : "memory");
  tmem_ld_wait();
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), version 1.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor: kind::f16, A/B fp16, fp32 accumulator, both
// K-major, M = 128, N = BN.
template <int BN>
__device__ __forceinline__ uint32_t idesc_f16() {
  return (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kTileN >> 4) << 24);
}

__device__ __forceinline__ uint32_t h2_mul(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// Sums elements [e0, e1) of the tile's partial ([column m][row r] fp32 in
// every member's shared memory at `base`) over the ks members in rank order
// and stores them with scale and bias.  EB elements per thread per batch,
// all of up to KS members' values in flight together.
template <int WBITS, int EB, int KS>
__device__ __forceinline__ void reduce_slice(const Params& p, uint32_t base, int ks, int e0, int e1, int tid,
                                             int n0, int m0) {
  constexpr int kStride = 256;   // the 8 epilogue warps
  #pragma unroll 1
  for (int eb = e0 + tid; eb < e1; eb += EB * kStride) {
    float t[EB][KS];
    #pragma unroll
    for (int q = 0; q < KS; ++q) {
      const uint32_t peer = q < ks ? dsmem_addr(base, (uint32_t)q) : 0u;
      #pragma unroll
      for (int u = 0; u < EB; ++u) {
        const int e = eb + u * kStride;
        t[u][q] = (q < ks && e < e1) ? ld_dsmem_f32(peer + (uint32_t)e * 4u) : 0.f;
      }
    }
    #pragma unroll
    for (int u = 0; u < EB; ++u) {
      const int e = eb + u * kStride;
      float acc = 0.f;
      #pragma unroll
      for (int q = 0; q < KS; ++q) acc += t[u][q];                 // rank order; padding adds +0
      const int nn = n0 + (e & (kTileN - 1));
      const int m = m0 + (e >> 7);
      if (e < e1 && nn < p.N && m < p.M) {
        float s8 = 1.f, b = 0.f;
        if (WBITS == 8)
          s8 = p.scale_f32 ? static_cast<const float*>(p.scale)[nn]
                           : __half2float(static_cast<const __half*>(p.scale)[nn]);
        if (p.bias)
          b = p.bias_f32 ? static_cast<const float*>(p.bias)[nn]
                         : __half2float(static_cast<const __half*>(p.bias)[nn]);
        p.out[(long long)m * p.ldo + nn] = __float2half_rn(fmaf(acc, s8, b));
      }
    }
  }
}

// SwiGLU mode of the pull reduction: pairs [q0, q1) of the tile, pair
// q = m*64 + c joining gate element m*128 + c and up element m*128 + 64 + c;
// each is summed over the ks members in rank order, finished with its own
// scale and bias, and silu(gate) * up is stored once (fp32, one rounding).
template <int WBITS, int EB, int KS>
__device__ __forceinline__ void reduce_pairs(const Params& p, uint32_t base, int ks, int q0, int q1, int tid,
                                             int tile, int m0) {
  constexpr int kStride = 256;
  constexpr int kHalfRows = kTileN / 2;
  #pragma unroll 1
  for (int qb = q0 + tid; qb < q1; qb += EB * kStride) {
    float tg[EB][KS], tu[EB][KS];
    #pragma unroll
    for (int q = 0; q < KS; ++q) {
      const uint32_t peer = q < ks ? dsmem_addr(base, (uint32_t)q) : 0u;
      #pragma unroll
      for (int u = 0; u < EB; ++u) {
        const int pq = qb + u * kStride;
        const int e = (pq / kHalfRows) * kTileN + (pq % kHalfRows);
        const bool ok = q < ks && pq < q1;
        tg[u][q] = ok ? ld_dsmem_f32(peer + (uint32_t)e * 4u) : 0.f;
        tu[u][q] = ok ? ld_dsmem_f32(peer + (uint32_t)(e + kHalfRows) * 4u) : 0.f;
      }
    }
    #pragma unroll
    for (int u = 0; u < EB; ++u) {
      const int pq = qb + u * kStride;
      float gv = 0.f, uv = 0.f;
      #pragma unroll
      for (int q = 0; q < KS; ++q) {                 // rank order; padding adds +0
        gv += tg[u][q];
        uv += tu[u][q];
      }
      const int c = tile * kHalfRows + (pq % kHalfRows);
      const int m = m0 + pq / kHalfRows;
      if (pq < q1 && c < p.nh && m < p.M) {
        float sg = 1.f, su = 1.f, bg = 0.f, bu = 0.f;
        if (WBITS == 8) {
          sg = p.scale_f32 ? static_cast<const float*>(p.scale)[c]
                           : __half2float(static_cast<const __half*>(p.scale)[c]);
          su = p.scale_f32 ? static_cast<const float*>(p.scale)[p.nh + c]
                           : __half2float(static_cast<const __half*>(p.scale)[p.nh + c]);
        }
        if (p.bias) {
          bg = p.bias_f32 ? static_cast<const float*>(p.bias)[c]
                          : __half2float(static_cast<const __half*>(p.bias)[c]);
          bu = p.bias_f32 ? static_cast<const float*>(p.bias)[p.nh + c]
                          : __half2float(static_cast<const __half*>(p.bias)[p.nh + c]);
        }
        gv = fmaf(gv, sg, bg);
        uv = fmaf(uv, su, bu);
        p.out[(long long)m * p.ldo + c] = __float2half_rn(gv / (1.f + __expf(-gv)) * uv);
      }
    }
  }
}

template <int WBITS, int LAYOUT, int BN>
__global__ void __launch_bounds__(Layout<WBITS, BN>::kThreads, 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                 const Params p) {
  using L = Layout<WBITS, BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int S = p.stages;
  // wfull: the stage's packed weights have landed (dequant waits); xfull:
  // its activation tile has (the MMA waits).  Separate, so that the decode
  // of the first stages does not wait for the activations, which only
  // follow the dependency wait.
  uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + (size_t)S * L::kStage);
  uint64_t* xfull = wfull + S;
  uint64_t* wfree = xfull + S;
  uint64_t* xfree = wfree + S;
  uint64_t* afull = xfree + S;
  uint64_t* afree = afull + L::kASlots;
  uint64_t* dfull = afree + L::kASlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dfull + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);   // a wait of this CTA gave up

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kTileN;
  const int m0 = blockIdx.y * BN;
  // this CTA's K-split: stages [kbeg, kbeg + nk)
  const int kbeg = blockIdx.z * p.nk_split;
  const int nk = min(p.nk - kbeg, p.nk_split);
  // MMA issuers: issuer q takes stages q, q + nissuers, ... into the
  // accumulator at TMEM column q * BN
  const int nissuers = (L::kTwoIssuers && nk > 1) ? 2 : 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(wfull + s, 1);
      mbar_init(xfull + s, 1);
      mbar_init(wfree + s, 8);
      mbar_init(xfree + s, 1);
    }
    for (int a = 0; a < L::kASlots; ++a) {
      mbar_init(afull + a, 8);
      mbar_init(afree + a, 1);
    }
    mbar_init(dfull, nissuers);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), L::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  griddep_launch_dependents();

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tmap(&tmap_x);
      prefetch_tmap(&tmap_w);
      const uint64_t pol_w = l2_policy_evict_last();   // reused by every activation tile
      const uint64_t pol_x = l2_policy_evict_last();   // reused by every weight tile
      // one 128-row box, or (SwiGLU mode) the gate and up halves as two
      // 64-row boxes (the map's box is then 64 rows high)
      auto load_w = [&](uint8_t* st, int kstage, uint64_t* bar) {
        if (p.nh == 0) {
          tma_load_3d(smem_u32(st + L::kXStage), &tmap_w, 0, kstage, n0, bar, pol_w);
        } else {
          const int c0 = blockIdx.x * (kTileN / 2);
          tma_load_3d(smem_u32(st + L::kXStage), &tmap_w, 0, kstage, c0, bar, pol_w);
          tma_load_3d(smem_u32(st + L::kXStage + L::kWStage / 2), &tmap_w, 0, kstage, p.nh + c0, bar, pol_w);
        }
      };
      // The weights of the first ring-full of stages do not depend on the
      // kernel before (programmatic dependent launch): they stream while it
      // finishes; the activations follow once it has.
      const int pre = min(S, nk);
      for (int i = 0; i < pre; ++i) {
        uint8_t* st = smem + (size_t)i * L::kStage;
        mbar_arrive_expect_tx(wfull + i, L::kWStage);
        load_w(st, kbeg + i, wfull + i);
      }
      griddep_wait();
      for (int i = 0; i < pre; ++i) {
        uint8_t* st = smem + (size_t)i * L::kStage;
        mbar_arrive_expect_tx(xfull + i, L::kXStage);
        tma_load_2d(smem_u32(st), &tmap_x, (kbeg + i) * kBK, m0, xfull + i, pol_x);
        tma_load_2d(smem_u32(st + L::kXAtom), &tmap_x, (kbeg + i) * kBK + 64, m0, xfull + i, pol_x);
      }
      int issued = pre;
      bool xissued_last = true;     // the last issued stage's activations went out too
      for (int i = pre; i < nk; ++i) {
        const int s = i % S;
        const uint32_t par = ((i / S) - 1) & 1;
        uint8_t* st = smem + (size_t)s * L::kStage;
        if (!mbar_wait(wfree + s, par, p.err, kDevErrEmptyWait, abort)) {
          *abort = 1;
          break;
        }
        mbar_arrive_expect_tx(wfull + s, L::kWStage);
        load_w(st, kbeg + i, wfull + s);
        // stage i's weights are in flight; should its activation slot never
        // free, the drain below waits for the weights alone
        const bool xok = mbar_wait(xfree + s, par, p.err, kDevErrEmptyWait, abort);
        if (xok) {
          mbar_arrive_expect_tx(xfull + s, L::kXStage);
          tma_load_2d(smem_u32(st), &tmap_x, (kbeg + i) * kBK, m0, xfull + s, pol_x);
          tma_load_2d(smem_u32(st + L::kXAtom), &tmap_x, (kbeg + i) * kBK + 64, m0, xfull + s, pol_x);
        }
        issued = i + 1;
        if (!xok) {
          *abort = 1;
          xissued_last = false;
          break;
        }
      }
      // every issued copy lands before the CTA can exit (only the last
      // stage of each slot can still be in flight)
      for (int s = 0; s < min(issued, S); ++s) {
        const int last = s + ((issued - 1 - s) / S) * S;
        mbar_wait(wfull + s, (last / S) & 1, p.err, kDevErrFullWait);
        if (xissued_last || last != issued - 1) mbar_wait(xfull + s, (last / S) & 1, p.err, kDevErrFullWait);
      }
    }
  } else if (warp == 1 || warp == kIssuer1Warp) {
    // -------------------------------------------------------- MMA issuers
    const int q = warp == 1 ? 0 : 1;
    if (lane == 0 && q < nissuers) {
      const uint32_t idesc = idesc_f16<BN>();
      const uint32_t d_tmem = tmem + (uint32_t)(q * BN);
      for (int i = q; i < nk; i += nissuers) {
        const int s = i % S, a = i % L::kASlots;
        if (!mbar_wait(xfull + s, (i / S) & 1, p.err, kDevErrMmaWait, abort) ||
            !mbar_wait(afull + a, (i / L::kASlots) & 1, p.err, kDevErrMmaWait, abort)) {
          *abort = 1;
          break;
        }
        tc_fence_after();
        const uint32_t xs = smem_u32(smem + (size_t)s * L::kStage);
        const uint32_t a_tmem = tmem + L::kACol + 64u * a;
        #pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint64_t bd = desc_sw128(xs + (uint32_t)((j >> 2) * L::kXAtom + (j & 3) * 32));
          tc_mma_ts(d_tmem, a_tmem + 8u * j, bd, idesc, (i > q || j > 0) ? 1u : 0u);
        }
        tc_commit(xfree + s);
        tc_commit(afree + a);
      }
      // dfull tracks every MMA issued above (one arrival per issuer);
      // waiting for it here means no MMA is in flight when the TMEM is
      // released, on the error path too
      tc_commit(dfull);
      mbar_wait(dfull, 0, p.err, kDevErrMmaWait);
    }
  } else {
    // ------------------------------------------------ dequant + epilogue
    const int quarter = warp & 3;                 // TMEM lane quarter of this warp
    const int half = (warp - 2) >> 2;             // which 64 k of the stage (and half of the columns)
    const int r = quarter * 32 + lane;            // weight row within the tile = TMEM lane
    const int n = tile_row(p, blockIdx.x, r);     // its row in the weight, -1 past it
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const __half* sc4 = static_cast<const __half*>(p.scale);
    // int4 group scale of this row for stage i (0 past N), two stages ahead
    auto load_scale = [&](int i) -> __half {
      return (WBITS == 4 && i < nk && n >= 0) ? sc4[(long long)(kbeg + i) * p.lds + n] : __float2half(0.f);
    };
    __half s_next = load_scale(0), s_next2 = load_scale(1);
    for (int i = 0; i < nk; ++i) {
      const int s = i % S, a = i % L::kASlots;
      const __half s_cur = s_next;
      s_next = s_next2;
      s_next2 = load_scale(i + 2);
      // warp-uniform outcome: tcgen05.st below is warp-collective
      if (!__all_sync(0xffffffffu, mbar_wait(wfull + s, (i / S) & 1, p.err, kDevErrFullWait, abort))) {
        *abort = 1;
        break;
      }
      const uint32_t wrow = smem_u32(smem + (size_t)s * L::kStage + L::kXStage);
      uint32_t cols[32];                          // columns 32*half .. +32 of the A stage: k = 64*half ..
      if (WBITS == 4) {
        const uint32_t s2 = (uint32_t)__half_as_ushort(s_cur) * 0x00010001u;
        if (LAYOUT == 0) {
          // all 64 bytes of row r (64-byte swizzle: chunk q at q ^ ((r >> 1) & 3)); half 0 takes the
          // low nibbles (k = 4w..4w+3), half 1 the high nibbles (k = 64+4w..)
          uint32_t wd[16];
          #pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 v = lds128(wrow + r * 64 + ((q ^ ((r >> 1) & 3)) << 4));
            wd[4 * q] = v.x; wd[4 * q + 1] = v.y; wd[4 * q + 2] = v.z; wd[4 * q + 3] = v.w;
          }
          // the branch is per warp (uniform) and outside the unrolled loops
          if (half == 0) {
            #pragma unroll
            for (int w = 0; w < 16; ++w) {
              const uint32_t t0 = __byte_perm(wd[w], 0u, 0x1100), t1 = __byte_perm(wd[w], 0u, 0x3322);
              cols[2 * w] = h2_mul(h2_sub(lop3_and_or(t0, 0x000F000Fu, kH2Magic), kH2_1032), s2);
              cols[2 * w + 1] = h2_mul(h2_sub(lop3_and_or(t1, 0x000F000Fu, kH2Magic), kH2_1032), s2);
            }
          } else {
            #pragma unroll
            for (int w = 0; w < 16; ++w) {
              const uint32_t t0 = __byte_perm(wd[w], 0u, 0x1100), t1 = __byte_perm(wd[w], 0u, 0x3322);
              cols[2 * w] = h2_mul(h2_fma(lop3_and_or(t0, 0x00F000F0u, kH2Magic), kH2_1_16, kH2_m72), s2);
              cols[2 * w + 1] = h2_mul(h2_fma(lop3_and_or(t1, 0x00F000F0u, kH2Magic), kH2_1_16, kH2_m72), s2);
            }
          }
        } else {
          // bytes 32*half .. +32 of row r: k = 64*half + 8w' .. +7
          #pragma unroll
          for (int q2 = 0; q2 < 2; ++q2) {
            const int q = 2 * half + q2;
            const uint4 v = lds128(wrow + r * 64 + ((q ^ ((r >> 1) & 3)) << 4));
            const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
            #pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int w = 4 * q2 + e;
              uint32_t p01, p23, p45, p67;
              dec_w4_adjacent(wd[e], p01, p23, p45, p67);
              cols[4 * w] = h2_mul(p01, s2);
              cols[4 * w + 1] = h2_mul(p23, s2);
              cols[4 * w + 2] = h2_mul(p45, s2);
              cols[4 * w + 3] = h2_mul(p67, s2);
            }
          }
        }
      } else {
        // bytes 64*half .. +64 of row r (128-byte swizzle: chunk q at q ^ (r & 7)); k = 64*half + 4w'..
        #pragma unroll
        for (int q2 = 0; q2 < 4; ++q2) {
          const int q = 4 * half + q2;
          const uint4 v = lds128(wrow + r * 128 + ((q ^ (r & 7)) << 4));
          dec_w8(v.x, cols[8 * q2 + 0], cols[8 * q2 + 1]);
          dec_w8(v.y, cols[8 * q2 + 2], cols[8 * q2 + 3]);
          dec_w8(v.z, cols[8 * q2 + 4], cols[8 * q2 + 5]);
          dec_w8(v.w, cols[8 * q2 + 6], cols[8 * q2 + 7]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(wfree + s);       // packed tile consumed
      if (i >= L::kASlots &&
          !__all_sync(0xffffffffu, mbar_wait(afree + a, ((i / L::kASlots) - 1) & 1, p.err, kDevErrFullWait, abort))) {
        *abort = 1;
        break;
      }
      tc_fence_after();
      const uint32_t a_taddr = tmem + lane_base + L::kACol + 64u * a + 32u * half;
      #pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        uint32_t v8[8];
        #pragma unroll
        for (int e = 0; e < 8; ++e) v8[e] = cols[8 * c8 + e];
        tmem_st8(a_taddr + 8u * c8, v8);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(afull + a);
    }

    // epilogue: this warp stores activation columns [half*BN/2, (half+1)*BN/2)
    mbar_wait(dfull, 0, p.err, kDevErrMmaWait);
    tc_fence_after();
    // 8 accumulator columns of this lane: D0, or D0 + D1 (fixed order)
    auto ld_acc = [&](uint32_t taddr, uint32_t (&v)[8]) {
      if (nissuers == 2) {
        uint32_t u[8];
        tmem_ld8_async(taddr, v);
        tmem_ld8_async(taddr + (uint32_t)BN, u);
        tmem_ld_wait();
        #pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(u[j]));
      } else {
        tmem_ld8(taddr, v);
      }
    };
    float sc8 = 1.f, bv = 0.f;
    if (n >= 0) {
      if (WBITS == 8)
        sc8 = p.scale_f32 ? static_cast<const float*>(p.scale)[n]
                          : __half2float(static_cast<const __half*>(p.scale)[n]);
      if (p.bias)
        bv = p.bias_f32 ? static_cast<const float*>(p.bias)[n]
                        : __half2float(static_cast<const __half*>(p.bias)[n]);
    }
    constexpr int kHalfCols = BN / 2;
    if (gridDim.z == 1 && p.nh > 0) {
      // SwiGLU, unsplit: every epilogue warp parks its finished fp32 values
      // in the drained ring as [gate | up][column m][row c] (lanes 0-63 hold
      // gate rows, 64-127 the matching up rows), the warps meet, and all
      // 256 threads combine the pairs: silu and product in fp32, one
      // rounding to fp16, 64 consecutive output columns per activation row
      float* buf = reinterpret_cast<float*>(smem);
      constexpr int kHalfRows = kTileN / 2;
      const int sel = r >= kHalfRows ? 1 : 0, hr = r & (kHalfRows - 1);
      #pragma unroll 1
      for (int c0 = half * kHalfCols; c0 < (half + 1) * kHalfCols; c0 += 8) {
        uint32_t v[8];
        ld_acc(tmem + lane_base + (uint32_t)c0, v);
        #pragma unroll
        for (int j = 0; j < 8; ++j)
          buf[(sel * BN + c0 + j) * kHalfRows + hr] = fmaf(__uint_as_float(v[j]), sc8, bv);
      }
      named_bar_sync(1, 256);
      #pragma unroll 4
      for (int idx = (int)threadIdx.x - 64; idx < BN * kHalfRows; idx += 256) {
        const int ml = idx / kHalfRows, c = idx % kHalfRows;
        const int col = blockIdx.x * kHalfRows + c, m = m0 + ml;
        if (col < p.nh && m < p.M) {
          const float gv = buf[idx], uv = buf[BN * kHalfRows + idx];
          p.out[(long long)m * p.ldo + col] = __float2half_rn(gv / (1.f + __expf(-gv)) * uv);
        }
      }
    } else if (gridDim.z == 1) {
      #pragma unroll 1
      for (int c0 = half * kHalfCols; c0 < (half + 1) * kHalfCols; c0 += 8) {
        uint32_t v[8];
        ld_acc(tmem + lane_base + (uint32_t)c0, v);
        if (n >= 0) {
          #pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int m = m0 + c0 + j;
            if (m < p.M) p.out[(long long)m * p.ldo + n] = __float2half_rn(fmaf(__uint_as_float(v[j]), sc8, bv));
          }
        }
      }
    } else if (L::kPush) {
      // Split-K, push: element e = m*128 + r of the partial belongs to
      // member e / sz, which sums it; store it straight into that member's
      // receive buffer, slot of this CTA's rank (remote stores, no reply)
      const int ks = (int)gridDim.z;
      const int sz = (BN * kTileN + ks - 1) / ks;
      const uint32_t me = cluster_rank();
      const uint32_t recv = smem_u32(smem + L::kRecvOffset(S));
      int e = half * kHalfCols * kTileN + r;
      int owner = e / sz, off = e - owner * sz;
      #pragma unroll 1
      for (int c0 = half * kHalfCols; c0 < (half + 1) * kHalfCols; c0 += 8) {
        uint32_t v[8];
        ld_acc(tmem + lane_base + (uint32_t)c0, v);
        #pragma unroll
        for (int j = 0; j < 8; ++j) {
          st_dsmem_f32(dsmem_addr(recv + (uint32_t)(me * sz + off) * 4u, (uint32_t)owner), __uint_as_float(v[j]));
          off += kTileN;                     // next column, same row
          while (off >= sz) {
            off -= sz;
            ++owner;
          }
        }
      }
    } else {
      // Split-K, pull: park the fp32 partial in this CTA's drained ring as
      // [column m][row r] (consecutive rows -> consecutive banks).  Every
      // TMA copy has landed and every MMA and decode read of the ring is
      // done once dfull has fired.
      float* part = reinterpret_cast<float*>(smem);
      #pragma unroll 1
      for (int c0 = half * kHalfCols; c0 < (half + 1) * kHalfCols; c0 += 8) {
        uint32_t v[8];
        ld_acc(tmem + lane_base + (uint32_t)c0, v);
        #pragma unroll
        for (int j = 0; j < 8; ++j) part[(c0 + j) * kTileN + r] = __uint_as_float(v[j]);
      }
    }
  }

  if (gridDim.z > 1 && L::kPush) {
    // ------------------------------------------ cluster reduction (push)
    cluster_sync_all();                 // every member's slices are in this CTA's receive buffer
    if (warp >= 2 && warp < kIssuer1Warp) {
      const int ks = (int)gridDim.z;
      constexpr int E = BN * kTileN;
      const int sz = (E + ks - 1) / ks;
      const uint32_t me = cluster_rank();
      const int e0 = (int)me * sz, e1 = min(E, e0 + sz);
      const float* recv = reinterpret_cast<const float*>(smem + L::kRecvOffset(S));
      for (int e = e0 + (int)threadIdx.x - 64; e < e1; e += 256) {
        float acc = 0.f;
        for (int q = 0; q < ks; ++q) acc += recv[q * sz + (e - e0)];   // rank order
        const int nn = n0 + (e & (kTileN - 1));
        const int m = m0 + (e >> 7);
        if (nn < p.N && m < p.M) {
          float s8 = 1.f, b = 0.f;
          if (WBITS == 8)
            s8 = p.scale_f32 ? static_cast<const float*>(p.scale)[nn]
                             : __half2float(static_cast<const __half*>(p.scale)[nn]);
          if (p.bias)
            b = p.bias_f32 ? static_cast<const float*>(p.bias)[nn]
                           : __half2float(static_cast<const __half*>(p.bias)[nn]);
          p.out[(long long)m * p.ldo + nn] = __float2half_rn(fmaf(acc, s8, b));
        }
      }
    }
    // nothing touches this CTA's shared memory after the barrier: no second one
  } else if (gridDim.z > 1) {
    // ------------------------------------------ cluster reduction (pull)
    cluster_sync_all();                 // every member's partial is in its shared memory
    if (warp >= 2 && warp < kIssuer1Warp) {
      const int ks = (int)gridDim.z;
      const uint32_t me = cluster_rank();
      constexpr int E = BN * kTileN;
      const int e0 = (int)(me * E / ks), e1 = (int)((me + 1) * E / ks);
      // all members' values of a batch of elements are loaded before any is
      // summed (one remote round trip per batch): 8 elements x up to 4
      // members, or 2 elements x up to 16 (32 registers, so that the narrow
      // tiles still run two CTAs per SM)
      if (p.nh > 0) {
        constexpr int P = BN * kTileN / 2;          // gate/up pairs of the tile
        const int q0 = (int)(me * P / ks), q1 = (int)((me + 1) * P / ks);
        if (ks <= 4)
          reduce_pairs<WBITS, 4, 4>(p, smem_u32(smem), ks, q0, q1, (int)threadIdx.x - 64, blockIdx.x, m0);
        else
          reduce_pairs<WBITS, 1, kMaxSplits>(p, smem_u32(smem), ks, q0, q1, (int)threadIdx.x - 64, blockIdx.x, m0);
      } else if (ks <= 4) {
        reduce_slice<WBITS, 8, 4>(p, smem_u32(smem), ks, e0, e1, (int)threadIdx.x - 64, n0, m0);
      } else {
        reduce_slice<WBITS, 2, kMaxSplits>(p, smem_u32(smem), ks, e0, e1, (int)threadIdx.x - 64, n0, m0);
      }
    }
    cluster_sync_all();                 // no member leaves while its partial may still be read
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::kTmemCols);
  }
}

}  // namespace gemm
}  // namespace ql
