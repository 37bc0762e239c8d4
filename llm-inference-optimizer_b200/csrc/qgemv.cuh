// qgemv.cuh — decode-shaped (small M) dequant-fused GEMV / skinny GEMM.
//
// Replaces the reference's Triton kernels for small M
// (_w8a16_matmul_kernel, src/kernels/w8a16_matmul_triton.py:39-86;
//  _w4a16_matmul_kernel, src/kernels/w4a16_matmul_triton.py:62-117).
//
// Work decomposition
//   * A "tile" is 16 consecutive weight rows (output columns n); a "block" is
//     `tpc` consecutive tiles.  The grid is persistent along N: CTA x runs
//     blocks x, x + gridDim.x, ... of one K-split (gridDim.y) and one batch
//     chunk (gridDim.z).  A k-block is 128 bytes of every row (256 k for
//     int4, 128 k for int8); a split covers `kb_per_split` k-blocks.
//   * Weights stream through shared memory in stages of one tile x
//     `kb_stage` k-blocks, each stage ONE 3-D TMA box over the rows viewed as
//     [N][kbytes/C][C] (C = 128, 64, 32 or 16 bytes; boxes past the row end
//     or past N read as zero).  For int4 the stage also carries the tile's
//     fp16 group scales for those k-blocks (a second, 2-D box), so nothing
//     but TMA touches the weight-side data.  One producer thread issues the
//     stages of all the CTA's blocks in order, running ahead across block
//     boundaries as far as the ring allows, and issues before the kernel
//     waits for its predecessor (programmatic dependent launch): weights
//     and scales do not depend on it.
//   * Every tile position has its own P = stages/tpc ring slots, so each
//     slot is consumed by one tile's warps, in order (a slot shared by
//     several tiles could be awaited by a faster tile one phase early,
//     which mbarrier parity cannot tell apart).
//   * Consumer warps: `wpt` warps per tile split each stage's k-blocks.  A
//     warp loads 16-byte chunks of rows g and g+8, decodes them in registers
//     to exact fp16 integers and issues mma.sync m16n8k16 with the weights
//     as the 16-row A operand and the activations (the CTA's x slice,
//     staged once in shared memory) as the n8 operand ("swap-AB": the batch
//     is the narrow side).  Odd rows load the two 64-byte halves of a
//     k-block in the opposite order to even rows, so each quarter-warp
//     touches all 32 banks once.  fp32 accumulation; the int4 group scale
//     multiplies each 128-k group partial in fp32, the int8 row scale
//     multiplies the sum once at the end — as in the reference kernels.
//   * Per block, the warps of a tile reduce through shared memory in a
//     fixed order.  With more than one K-split, each CTA writes an fp32
//     partial to its own workspace slot and the last CTA to arrive (atomic
//     counter) sums the slots in slot order, applies scale/bias and zeroes
//     slots and counter, so the result is deterministic and the workspace
//     stays zeroed.
//   * Greedy-head mode (amax.out set, K unsplit, M <= 8): instead of storing the
//     outputs, each tile turns its fp16-rounded outputs into argmax keys
//     (qargmax.cuh), the CTA keeps the per-row maximum in shared memory and
//     merges it into the exchange buffer's scratch once; the last CTA of the
//     grid runs the exchange over NVLink (qxchg.cuh) and writes the argmax
//     columns.  One launch per rank for logits-free greedy decoding.
#pragma once

#include "qxchg.cuh"

namespace ql {
namespace gemv {

constexpr int kTileRows = 16;
constexpr int kBlockBytes = 128;    // k-block width
// At most 8 consumer warps + 1 producer warp, so that two CTAs fit on an SM
// by registers: the next kernel's CTAs can then start streaming their
// weights (programmatic dependent launch) while this kernel finishes.
constexpr int kMaxConsumerWarps = 8;
constexpr int kMaxThreads = (kMaxConsumerWarps + 1) * 32;

struct Params {
  const __half* x;        // [M, ldx]
  const void* scale;      // int8: [N] (f32 or f16); int4: [K/128, lds] f16
  const void* bias;       // [N] or nullptr
  __half* out;            // [M, ldo]
  long long ldx, lds, ldo;
  int M, N, K;
  int kbytes;             // valid bytes of one weight row: K/2 (int4) or K (int8)
  int nkb;                // ceil(kbytes / 128)
  int kb_per_split;
  int ks;                 // number of K-splits (gridDim.y)
  int nblk;               // blocks of tpc tiles along N (gridDim.x <= nblk)
  int tpc;                // tiles per block
  int wpt;                // consumer warps per tile
  int kb_stage;           // k-blocks per stage (divides kb_per_split or covers it)
  int stages;             // ring depth (stages resident at once), a multiple of tpc
  int chunk;              // C: bytes of the innermost tensor-map dimension
  int x_stride;           // halves per staged x row
  int x_rows;             // staged x rows = min(8*MT, M)
  int scale_tma;          // int4: scales arrive with each stage (else staged per block)
  int scale_f32;          // int8 scale dtype
  int bias_f32;           // bias dtype
  int early_weights;      // stream weights before griddepcontrol.wait
  int swiglu_n;           // > 0: rows [0, n) are gate and [n, 2n) up rows of one stacked
                          // weight; a block pairs tpc/2 gate tiles with the matching up
                          // tiles and stores silu(gate) * up, [M, n] (ks == 1 only)
  uint32_t* counters;     // [gridDim.z * nblk] (ks > 1)
  float* partials;        // [gridDim.z][nblk][ks][mc][tpc*16] (ks > 1)
  xchg::Ctx amax;         // amax.out != nullptr: greedy-head mode (ks == 1, swiglu_n == 0)
  unsigned* err;          // device error word
};

// Bytes of one ring stage: weights, then (int4 with scale_tma) the scale box
// [2*kb_stage groups][16 rows] fp16, padded to 128 bytes.
__host__ __device__ inline uint32_t stage_weight_bytes(int kb_stage) {
  return (uint32_t)(kTileRows * kb_stage * kBlockBytes);
}
__host__ __device__ inline uint32_t stage_scale_bytes(int wbits, int scale_tma, int kb_stage) {
  return (wbits == 4 && scale_tma) ? (uint32_t)((2 * kb_stage * kTileRows * 2 + 127) / 128 * 128) : 0u;
}

// Shared-memory carve-up, identical on host and device.
struct Smem {
  size_t ring, red, x, sc, bars, total;
};
__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
__host__ __device__ inline Smem smem_layout(int wbits, int mc, int x_rows, int tpc, int wpt, int stages,
                                            int kb_stage, int x_stride, int kb_per_split, int scale_tma) {
  Smem s;
  s.ring = (size_t)stages * (stage_weight_bytes(kb_stage) + stage_scale_bytes(wbits, scale_tma, kb_stage));
  s.red = align_up((size_t)tpc * wpt * kTileRows * mc * 4, 128);
  s.x = align_up((size_t)x_rows * x_stride * 2, 16);
  s.sc = (wbits == 4 && !scale_tma) ? align_up((size_t)kb_per_split * 2 * tpc * kTileRows * 4, 16) : 0;
  // mbarriers, last_flag + abort, the CTA's row maxima (greedy-head mode)
  s.bars = align_up((size_t)2 * stages * 8 + 16 + (size_t)8 * mc, 16);
  s.total = 128 /* base alignment slack */ + s.ring + s.red + s.x + s.sc + s.bars;
  return s;
}

template <int WBITS>
__device__ __forceinline__ float finish_value(const Params& p, float v, int n) {
  if (WBITS == 8) {
    const float s = p.scale_f32 ? static_cast<const float*>(p.scale)[n]
                                : __half2float(static_cast<const __half*>(p.scale)[n]);
    v *= s;
  }
  if (p.bias) {
    v += p.bias_f32 ? static_cast<const float*>(p.bias)[n]
                    : __half2float(static_cast<const __half*>(p.bias)[n]);
  }
  return v;
}

// B fragments (activations) of one 64-byte k-step for MT batch tiles: the
// two 16-element runs of row t*8+g that this lane's weights multiply.  Lanes
// of rows past the batch read row 0 instead: an mma output column depends
// only on its own B column, and those columns are never stored — so no
// predicate and no zeroing in the hot loop.
template <int MT>
__device__ __forceinline__ void load_b(uint32_t (&b0)[MT][8], uint32_t (&b1)[MT][8], uint32_t xs_s,
                                       int x_stride, int g, int mvalid, int e0, int e1) {
  #pragma unroll
  for (int t = 0; t < MT; ++t) {
    const int row = t * 8 + g < mvalid ? t * 8 + g : 0;
    const uint32_t xr = xs_s + (uint32_t)(row * x_stride) * 2u;
    const uint4 v0 = lds128(xr + e0 * 2);
    const uint4 v1 = lds128(xr + e0 * 2 + 16);
    const uint4 v2 = lds128(xr + e1 * 2);
    const uint4 v3 = lds128(xr + e1 * 2 + 16);
    b0[t][0] = v0.x; b0[t][1] = v0.y; b0[t][2] = v0.z; b0[t][3] = v0.w;
    b0[t][4] = v1.x; b0[t][5] = v1.y; b0[t][6] = v1.z; b0[t][7] = v1.w;
    b1[t][0] = v2.x; b1[t][1] = v2.y; b1[t][2] = v2.z; b1[t][3] = v2.w;
    b1[t][4] = v3.x; b1[t][5] = v3.y; b1[t][6] = v3.z; b1[t][7] = v3.w;
  }
}

__device__ __forceinline__ void u4_to_words(const uint4& v, uint32_t (&w)[4]) {
  w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
}

// NS consecutive 64-byte k-steps (h0, h0+1, ...) of k-block `i` of one tile,
// all loaded before any is computed so that their shared-memory loads and
// mma chains overlap.  Every k-step keeps two independent accumulator
// chains per batch tile.  `rowA`/`rowB` are the shared addresses of this
// k-block's 128 bytes in rows g and g+8; `odd` = g & 1.  int4: sA[h] / sB[h]
// are the group scales of rows g / g+8 for the k-block's group h (0, 1).
template <int WBITS, int LAYOUT, int MT, int NS>
__device__ __forceinline__ void ksteps(float (&acc)[2][MT][4], uint32_t rowA, uint32_t rowB, int i, int h0,
                                       int c, int g, bool odd, uint32_t xs_s, int x_stride, int mvalid,
                                       const float (&sA)[2], const float (&sB)[2]) {
  uint32_t wA[NS][4], wB[NS][4];
  if (NS == 2) {
    // even rows read half 0 then 1, odd rows half 1 then 0: a quarter-warp
    // (two rows x four chunks) then covers all eight 16-byte bank groups
    const uint32_t c0 = (uint32_t)(((odd ? 1 : 0) * 4 + c) << 4);
    const uint32_t c1 = (uint32_t)(((odd ? 0 : 1) * 4 + c) << 4);
    const uint4 a0 = lds128(rowA + c0), a1 = lds128(rowA + c1);
    const uint4 b0 = lds128(rowB + c0), b1 = lds128(rowB + c1);
    u4_to_words(odd ? a1 : a0, wA[0]);
    u4_to_words(odd ? a0 : a1, wA[NS - 1]);
    u4_to_words(odd ? b1 : b0, wB[0]);
    u4_to_words(odd ? b0 : b1, wB[NS - 1]);
  } else {
    const uint32_t co = (uint32_t)((h0 * 4 + c) << 4);
    u4_to_words(lds128(rowA + co), wA[0]);
    u4_to_words(lds128(rowB + co), wB[0]);
  }
  if (WBITS == 4) {
    uint32_t bx0[NS][MT][8], bx1[NS][MT][8];
    #pragma unroll
    for (int n = 0; n < NS; ++n) {
      const int kg = (i * 2 + h0 + n) * 128;     // first k of the group (relative to the split)
      // split-half: low nibbles k = kg+16c.., high nibbles k = kg+64+16c..
      // adjacent:   k = kg+32c .. kg+32c+31
      const int e0 = LAYOUT == 0 ? kg + 16 * c : kg + 32 * c;
      const int e1 = LAYOUT == 0 ? kg + 64 + 16 * c : kg + 32 * c + 16;
      load_b<MT>(bx0[n], bx1[n], xs_s, x_stride, g, mvalid, e0, e1);
    }
    float part[NS][2][MT][4];
    #pragma unroll
    for (int n = 0; n < NS; ++n)
      #pragma unroll
      for (int u = 0; u < 2; ++u)
        #pragma unroll
        for (int t = 0; t < MT; ++t) part[n][u][t][0] = part[n][u][t][1] = part[n][u][t][2] = part[n][u][t][3] = 0.f;
    #pragma unroll
    for (int j = 0; j < 4; ++j) {
      #pragma unroll
      for (int n = 0; n < NS; ++n) {
        if (LAYOUT == 0) {
          // permuted decode: the staged activations are in the matching order
          uint32_t al01, al23, ah01, ah23, bl01, bl23, bh01, bh23;
          dec_w4_split_perm(wA[n][j], al01, al23, ah01, ah23);
          dec_w4_split_perm(wB[n][j], bl01, bl23, bh01, bh23);
          #pragma unroll
          for (int t = 0; t < MT; ++t) {
            mma_16816(part[n][0][t], al01, bl01, al23, bl23, bx0[n][t][2 * j], bx0[n][t][2 * j + 1]);
            mma_16816(part[n][1][t], ah01, bh01, ah23, bh23, bx1[n][t][2 * j], bx1[n][t][2 * j + 1]);
          }
        } else {
          uint32_t a01, a23, a45, a67, b01, b23, b45, b67;
          dec_w4_adjacent_perm(wA[n][j], a01, a23, a45, a67);
          dec_w4_adjacent_perm(wB[n][j], b01, b23, b45, b67);
          const int jj = (j & 1) * 4;
          #pragma unroll
          for (int t = 0; t < MT; ++t) {
            const uint32_t* bx = j < 2 ? bx0[n][t] : bx1[n][t];
            mma_16816(part[n][0][t], a01, b01, a23, b23, bx[jj], bx[jj + 1]);
            mma_16816(part[n][1][t], a45, b45, a67, b67, bx[jj + 2], bx[jj + 3]);
          }
        }
      }
    }
    #pragma unroll
    for (int n = 0; n < NS; ++n) {
      const float a_s = sA[h0 + n], b_s = sB[h0 + n];
      #pragma unroll
      for (int t = 0; t < MT; ++t) {
        acc[n & 1][t][0] = fmaf(part[n][0][t][0] + part[n][1][t][0], a_s, acc[n & 1][t][0]);
        acc[n & 1][t][1] = fmaf(part[n][0][t][1] + part[n][1][t][1], a_s, acc[n & 1][t][1]);
        acc[n & 1][t][2] = fmaf(part[n][0][t][2] + part[n][1][t][2], b_s, acc[n & 1][t][2]);
        acc[n & 1][t][3] = fmaf(part[n][0][t][3] + part[n][1][t][3], b_s, acc[n & 1][t][3]);
      }
    }
  } else {
    // int8: k = i*128 + (h0+n)*64 + 16c + 4j + {0..3}
    uint32_t bx[NS][MT][8];
    #pragma unroll
    for (int n = 0; n < NS; ++n) {
      const int e0 = i * kBlockBytes + (h0 + n) * 64 + 16 * c;
      #pragma unroll
      for (int t = 0; t < MT; ++t) {
        const int row = t * 8 + g < mvalid ? t * 8 + g : 0;   // see load_b
        const uint32_t xr = xs_s + (uint32_t)(row * x_stride) * 2u;
        const uint4 v0 = lds128(xr + e0 * 2);
        const uint4 v1 = lds128(xr + e0 * 2 + 16);
        bx[n][t][0] = v0.x; bx[n][t][1] = v0.y; bx[n][t][2] = v0.z; bx[n][t][3] = v0.w;
        bx[n][t][4] = v1.x; bx[n][t][5] = v1.y; bx[n][t][6] = v1.z; bx[n][t][7] = v1.w;
      }
    }
    #pragma unroll
    for (int j = 0; j < 4; ++j) {
      #pragma unroll
      for (int n = 0; n < NS; ++n) {
        uint32_t a01, a23, b01, b23;
        dec_w8(wA[n][j], a01, a23);
        dec_w8(wB[n][j], b01, b23);
        #pragma unroll
        for (int t = 0; t < MT; ++t)
          mma_16816(acc[j & 1][t], a01, b01, a23, b23, bx[n][t][2 * j], bx[n][t][2 * j + 1]);
      }
    }
  }
}


// MT = number of n8 batch tiles per CTA (mc = 8*MT batch rows per grid.z slice).
template <int WBITS, int LAYOUT, int MT>
__global__ void __launch_bounds__(kMaxThreads, 2)
    qgemv_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_s,
                 const Params p) {
  constexpr int MC = 8 * MT;
  constexpr int EPK = WBITS == 4 ? 256 : 128;      // k elements per k-block
  constexpr int NS = MT == 1 ? 2 : 1;              // k-steps decoded together
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);

  const int tpc = p.tpc, wpt = p.wpt, stages = p.stages, kb_stage = p.kb_stage;
  const int ncw = tpc * wpt;                 // consumer warps
  const int nct = ncw * 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows_cta = tpc * kTileRows;      // power of two
  const int rows_log2 = 31 - __clz(rows_cta);
  const bool scale_tma = WBITS == 4 && p.scale_tma != 0;
  const uint32_t w_bytes = stage_weight_bytes(kb_stage);
  const uint32_t stage_bytes = w_bytes + stage_scale_bytes(WBITS, p.scale_tma, kb_stage);
  // bytes the TMA actually delivers per stage (the scale box is not padded)
  const uint32_t stage_tx = w_bytes + (scale_tma ? (uint32_t)(2 * kb_stage * kTileRows * 2) : 0u);

  const Smem L = smem_layout(WBITS, MC, p.x_rows, tpc, wpt, stages, kb_stage, p.x_stride, p.kb_per_split,
                             p.scale_tma);
  uint8_t* ring = smem;
  float* red = reinterpret_cast<float*>(smem + L.ring);                    // [tpc][wpt][MC][16]
  __half* xs = reinterpret_cast<__half*>(smem + L.ring + L.red);
  float* ssc = reinterpret_cast<float*>(smem + L.ring + L.red + L.x);       // per-block scales (fallback)
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.ring + L.red + L.x + L.sc);
  uint64_t* empty = full + stages;
  int* last_flag = reinterpret_cast<int*>(empty + stages);
  volatile int* abort = last_flag + 1;    // set once a wait of this CTA gives up
  unsigned long long* amax_s = reinterpret_cast<unsigned long long*>(empty + stages + 2);   // [MC]
  const bool greedy = MT == 1 && p.amax.out != nullptr;   // host: greedy-head plans have MT == 1

  const int split = blockIdx.y, mchunk = blockIdx.z;
  const int kb0 = split * p.kb_per_split;
  const int kbc = min(p.kb_per_split, p.nkb - kb0);
  const int nkc = (kbc + kb_stage - 1) / kb_stage;   // k-chunks (stages per tile per block)
  const int m0 = mchunk * MC;
  // Ring slots per tile: the q-th stage of tile position tt (q = it*nkc + kc
  // for block iteration it, k-chunk kc) lives in slot tt*P + q%P and is that
  // slot's phase q/P.
  const int P = stages / tpc;
  const int nit = (p.nblk - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;   // blocks of this CTA
  // first weight row of tile position tt of block blk
  const int half_tiles = tpc >> 1;
  auto tile_row = [&](int blk, int t) -> int {
    if (p.swiglu_n == 0) return blk * rows_cta + t * kTileRows;
    return t < half_tiles ? (blk * half_tiles + t) * kTileRows
                          : p.swiglu_n + (blk * half_tiles + t - half_tiles) * kTileRows;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, wpt);
    }
    *abort = 0;
    fence_barrier_init();
  }
  __syncthreads();

  // ------------------------------------------------------------ producer
  // Stages are issued in the order (block iteration, k-chunk, tile).
  if (warp == ncw) {
    if (lane == 0) {
      prefetch_tmap(&tmap_w);
      if (scale_tma) prefetch_tmap(&tmap_s);
      // weights are read once unless several batch chunks share them
      const uint64_t pol = gridDim.z > 1 ? l2_policy_evict_last() : l2_policy_evict_first();
      if (!p.early_weights) griddep_wait();
      const int per_kb = kBlockBytes / p.chunk;
      const int total = nit * nkc * tpc;
      int issued = 0;
      for (int st = 0; st < total; ++st) {
        const int q = st / tpc, tt = st - q * tpc;
        const int it = q / nkc, kc = q - it * nkc;
        const int s = tt * P + q % P;
        if (q >= P && !mbar_wait(empty + s, ((q / P) - 1) & 1, p.err, kDevErrEmptyWait, abort)) {
          *abort = 1;
          break;
        }
        const int row = tile_row((int)blockIdx.x + it * (int)gridDim.x, tt);
        const int kbg = kb0 + kc * kb_stage;               // first k-block of the stage
        uint8_t* dst = ring + (size_t)s * stage_bytes;
        mbar_arrive_expect_tx(full + s, stage_tx);
        tma_load_3d(smem_u32(dst), &tmap_w, 0, kbg * per_kb, row, full + s, pol);
        if (scale_tma) tma_load_2d(smem_u32(dst + w_bytes), &tmap_s, row, kbg * 2, full + s, pol);
        issued = st + 1;
      }
      // Keep the CTA resident until every issued copy has landed, whatever
      // the consumers did (in normal operation they have waited for all of
      // them anyway).  A slot is re-filled only after its previous stage
      // was consumed, so only the last stage issued on each slot can still
      // be in flight.
      for (int tt = 0; tt < tpc && tt < issued; ++tt) {
        const int q_last = (issued - 1 - tt) / tpc;            // last stage issued for tile tt
        for (int j = 0; j < P && j <= q_last; ++j) {
          const int q = q_last - (q_last - j) % P;             // last stage issued on slot tt*P+j
          mbar_wait(full + tt * P + j, (q / P) & 1, p.err, kDevErrFullWait);
        }
      }
    }
    return;
  }

  // ----------------------------------------------------------- consumers
  const int ctid = threadIdx.x;
  const int tt = warp / wpt, w = warp - tt * wpt;
  const int g = lane >> 2, c = lane & 3;

  // int4 group scales of one block's rows -> fp32 in shared memory, when
  // they do not come with the stages (scale rows not 16-byte aligned).
  auto stage_scales = [&](int blk) {
    const int G = p.K / 128;
    const int g0 = kb0 * 2;
    const int ng = min(kbc * 2, G - g0);
    const __half* sc = static_cast<const __half*>(p.scale);
    for (int idx = ctid; idx < (ng << rows_log2); idx += nct) {
      const int gl = idx >> rows_log2, r = idx & (rows_cta - 1);
      const int n = tile_row(blk, r >> 4) + (r & 15);
      ssc[idx] = n < p.N ? __half2float(sc[(long long)(g0 + gl) * p.lds + n]) : 0.f;
    }
  };
  // scales are static like the weights: the first block's are loaded
  // before the dependency wait
  if (WBITS == 4 && !scale_tma) stage_scales(blockIdx.x);

  griddep_wait();   // x (and out / workspace) may belong to the previous kernel
  // greedy head: the exchange's epoch, read now rather than in the tail
  const unsigned xchg_done = (greedy && ctid == 0) ? xchg::epochs_done(p.amax) : 0u;

  const int mvalid = min(MC, p.M - m0);
  // x slice [m0, m0+mvalid) x [kx0, kx0 + kbc*EPK) -> shared memory, once per
  // CTA (every block of the CTA uses the same slice); k past K reads as
  // zero.  Rows >= mvalid are never read.
  {
    // Up to 8 16-byte loads in flight per thread before any is stored (one
    // after another they would be serial L2 round trips on the critical
    // path): 8 of a thread's vectors of a single row, or one vector of up
    // to 8 rows.
    const int kx0 = kb0 * EPK;
    const int nvec = kbc * EPK / 8;
    if (mvalid == 1) {
      const __half* xrow = p.x + (long long)m0 * p.ldx + kx0;
      for (int v0 = ctid; v0 < nvec; v0 += 8 * nct) {
        uint4 val[8];
        #pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int v = v0 + u * nct;
          val[u] = make_uint4(0u, 0u, 0u, 0u);
          if (v < nvec && kx0 + v * 8 < p.K) val[u] = ldg_cg_v4(xrow + v * 8);
        }
        #pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int v = v0 + u * nct;
          if (v < nvec) {
            uint4 w = val[u];
            if (WBITS == 4) w = stage_x_perm<LAYOUT>(w);   // k order of the permuted int4 decode
            *reinterpret_cast<uint4*>(xs + v * 8) = w;
          }
        }
      }
    } else {
      for (int v = ctid; v < nvec; v += nct) {
        const bool in_k = kx0 + v * 8 < p.K;
        #pragma unroll
        for (int r0 = 0; r0 < MC; r0 += 8) {
          uint4 val[8];
          #pragma unroll
          for (int u = 0; u < 8; ++u) {
            val[u] = make_uint4(0u, 0u, 0u, 0u);
            if (r0 + u < mvalid && in_k) val[u] = ldg_cg_v4(p.x + (long long)(m0 + r0 + u) * p.ldx + kx0 + v * 8);
          }
          #pragma unroll
          for (int u = 0; u < 8; ++u) {
            if (r0 + u < mvalid) {
              uint4 w = val[u];
              if (WBITS == 4) w = stage_x_perm<LAYOUT>(w);   // k order of the permuted int4 decode
              *reinterpret_cast<uint4*>(xs + (r0 + u) * p.x_stride + v * 8) = w;
            }
          }
        }
      }
    }
    if (greedy)
      for (int i = ctid; i < MC; i += nct) amax_s[i] = 0ull;
  }
  named_bar_sync(1, nct);
  griddep_launch_dependents();

  const uint32_t ring_s = smem_u32(ring);
  const uint32_t xs_s = smem_u32(xs);
  const int valid_bytes = p.kbytes - kb0 * kBlockBytes;
  const bool odd = (g & 1) != 0;
  const uint32_t rowA_off = (uint32_t)(g * kb_stage * kBlockBytes);
  const uint32_t rowB_off = (uint32_t)((g + 8) * kb_stage * kBlockBytes);
  const int nout = mvalid << rows_log2;   // (m, r) pairs of a block, r fastest

  for (int it = 0; it < nit; ++it) {
    const int blk = (int)blockIdx.x + it * (int)gridDim.x;
    const int row0 = blk * rows_cta;
    if (it > 0 && WBITS == 4 && !scale_tma) {
      stage_scales(blk);
      named_bar_sync(1, nct);
    }

    float acc[2][MT][4];
    #pragma unroll
    for (int u = 0; u < 2; ++u)
      #pragma unroll
      for (int t = 0; t < MT; ++t) acc[u][t][0] = acc[u][t][1] = acc[u][t][2] = acc[u][t][3] = 0.f;

    for (int kc = 0; kc < nkc; ++kc) {
      const int q = it * nkc + kc;
      const int s = tt * P + q % P;
      // warp-uniform outcome: mma.sync below needs the whole warp
      if (!__all_sync(0xffffffffu, mbar_wait(full + s, (q / P) & 1, p.err, kDevErrFullWait, abort))) {
        *abort = 1;   // stop here without releasing the slot; the producer drains its copies
        break;
      }
      const uint32_t tile_s = ring_s + (uint32_t)s * stage_bytes;
      const uint32_t sst = tile_s + w_bytes + (uint32_t)g * 2u;   // this lane's row in the scale box
      const int kb_lo = kc * kb_stage;
      const int kb_hi = min(kb_stage, kbc - kb_lo);
      for (int kbl = w; kbl < kb_hi; kbl += wpt) {
        const int i = kb_lo + kbl;                          // k-block within the split
        const uint32_t rowA = tile_s + rowA_off + (uint32_t)(kbl * kBlockBytes);
        const uint32_t rowB = tile_s + rowB_off + (uint32_t)(kbl * kBlockBytes);
        const int rem = valid_bytes - i * kBlockBytes;       // > 0
        float sA[2] = {0.f, 0.f}, sB[2] = {0.f, 0.f};
        if (WBITS == 4) {
          if (scale_tma) {
            // stage scale box: [group within the stage][16 rows] fp16
            const uint32_t s0 = sst + (uint32_t)(kbl * 2 * kTileRows * 2);
            sA[0] = lds_f16_as_f32(s0);
            sB[0] = lds_f16_as_f32(s0 + 16);
            sA[1] = lds_f16_as_f32(s0 + kTileRows * 2);
            sB[1] = lds_f16_as_f32(s0 + kTileRows * 2 + 16);
          } else {
            const float* scr = ssc + tt * kTileRows + g;
            sA[0] = scr[(i * 2) * rows_cta];
            sB[0] = scr[(i * 2) * rows_cta + 8];
            if (rem > 64) {
              sA[1] = scr[(i * 2 + 1) * rows_cta];
              sB[1] = scr[(i * 2 + 1) * rows_cta + 8];
            }
          }
        }
        if (rem > 64) {
          if (NS == 2) {
            ksteps<WBITS, LAYOUT, MT, 2>(acc, rowA, rowB, i, 0, c, g, odd, xs_s, p.x_stride, mvalid, sA, sB);
          } else {
            ksteps<WBITS, LAYOUT, MT, 1>(acc, rowA, rowB, i, 0, c, g, odd, xs_s, p.x_stride, mvalid, sA, sB);
            ksteps<WBITS, LAYOUT, MT, 1>(acc, rowA, rowB, i, 1, c, g, odd, xs_s, p.x_stride, mvalid, sA, sB);
          }
        } else {
          ksteps<WBITS, LAYOUT, MT, 1>(acc, rowA, rowB, i, 0, c, g, odd, xs_s, p.x_stride, mvalid, sA, sB);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + s);
    }

    // -------------------------------------------------- block epilogue
    {
      float* mine = red + (size_t)(tt * wpt + w) * MC * kTileRows;
      #pragma unroll
      for (int t = 0; t < MT; ++t) {
        const int mm = t * 8 + 2 * c;
        mine[(mm + 0) * kTileRows + g] = acc[0][t][0] + acc[1][t][0];
        mine[(mm + 1) * kTileRows + g] = acc[0][t][1] + acc[1][t][1];
        mine[(mm + 0) * kTileRows + g + 8] = acc[0][t][2] + acc[1][t][2];
        mine[(mm + 1) * kTileRows + g + 8] = acc[0][t][3] + acc[1][t][3];
      }
    }

    if (p.swiglu_n > 0) {
      // gate tile t and up tile t + tpc/2 live in different warps: the CTA
      // meets, then every (row, column) pair is finished and stored once,
      // silu and product in fp32, one rounding to fp16
      named_bar_sync(1, nct);
      const int hrows = half_tiles * kTileRows;
      for (int idx = ctid; idx < mvalid * hrows; idx += nct) {
        const int m = idx / hrows, r = idx - m * hrows;
        const int t = r >> 4, rr = r & 15;
        float gv = 0.f, uv = 0.f;
        for (int w2 = 0; w2 < wpt; ++w2) {
          gv += red[((t * wpt + w2) * MC + m) * kTileRows + rr];
          uv += red[(((t + half_tiles) * wpt + w2) * MC + m) * kTileRows + rr];
        }
        const int n = blk * hrows + r;                       // output column = gate row
        if (n < p.swiglu_n) {
          gv = finish_value<WBITS>(p, gv, n);
          uv = finish_value<WBITS>(p, uv, p.swiglu_n + n);
          p.out[(long long)(m0 + m) * p.ldo + n] = __float2half_rn(gv / (1.f + __expf(-gv)) * uv);
        }
      }
      named_bar_sync(1, nct);   // red (and the block scales) are reused next block
    } else if (p.ks == 1) {
      // Only the warps of one tile meet here (named barrier 2 + tt), so
      // tiles finish their blocks independently.
      if (wpt > 1) named_bar_sync(2 + tt, wpt * 32); else __syncwarp();
      if (greedy) {
        // keys of the fp16-rounded outputs (what argmax over the stored
        // logits would see); max over the tile's 16 rows within each half
        // warp, then into the CTA's row maxima
        for (int b = w * 32; b < mvalid * kTileRows; b += wpt * 32) {   // warp-uniform
          const int idx = b + lane;
          unsigned long long key = 0ull;
          if (idx < mvalid * kTileRows) {
            const int m = idx >> 4, rr = idx & 15;
            float v = 0.f;
            for (int w2 = 0; w2 < wpt; ++w2) v += red[((tt * wpt + w2) * MC + m) * kTileRows + rr];
            const int n = row0 + tt * kTileRows + rr;
            if (n < p.N) {
              const __half h = __float2half_rn(finish_value<WBITS>(p, v, n));
              key = amax::row_key(__half_as_ushort(h), p.amax.col_offset + n);
            }
          }
          #pragma unroll
          for (int o = 8; o > 0; o >>= 1) key = amax::umax64(key, __shfl_xor_sync(0xffffffffu, key, o));
          if ((lane & 15) == 0 && idx < mvalid * kTileRows) atomicMax(amax_s + (idx >> 4), key);
        }
      } else {
        for (int idx = w * 32 + lane; idx < mvalid * kTileRows; idx += wpt * 32) {
          const int m = idx >> 4, rr = idx & 15;
          float v = 0.f;
          for (int w2 = 0; w2 < wpt; ++w2) v += red[((tt * wpt + w2) * MC + m) * kTileRows + rr];
          const int n = row0 + tt * kTileRows + rr;
          if (n < p.N) p.out[(long long)(m0 + m) * p.ldo + n] = __float2half_rn(finish_value<WBITS>(p, v, n));
        }
      }
      if (wpt > 1) named_bar_sync(2 + tt, wpt * 32); else __syncwarp();   // red is reused next block
      if (WBITS == 4 && !scale_tma) named_bar_sync(1, nct);               // so are the block scales
    } else {
      named_bar_sync(1, nct);
      // ------------------------------------- cross-CTA split-K reduction
      const int slot_elems = MC << rows_log2;
      const size_t tile_id = (size_t)mchunk * p.nblk + blk;
      float* slots = p.partials + tile_id * p.ks * slot_elems;
      {
        float* mine = slots + (size_t)split * slot_elems;
        for (int idx = ctid; idx < nout; idx += nct) {
          const int m = idx >> rows_log2, r = idx & (rows_cta - 1);
          const int t = r >> 4, rr = r & 15;
          float v = 0.f;
          for (int w2 = 0; w2 < wpt; ++w2) v += red[((t * wpt + w2) * MC + m) * kTileRows + rr];
          mine[idx] = v;
        }
      }
      named_bar_sync(1, nct);
      if (ctid == 0) {
        // one thread releases the CTA's partials (cumulative over the
        // barrier) and, if it arrives last, acquires the other splits'
        const unsigned old = atomic_add_acq_rel_gpu(p.counters + tile_id, 1u);
        const int last = old == (unsigned)(p.ks - 1);
        *last_flag = last;
      }
      named_bar_sync(1, nct);
      if (*last_flag) {
        for (int idx = ctid; idx < nout; idx += nct) {
          // slots in order, 8 independent loads in flight at a time
          float v = 0.f;
          int s2 = 0;
          for (; s2 + 8 <= p.ks; s2 += 8) {
            float t[8];
            #pragma unroll
            for (int j = 0; j < 8; ++j) t[j] = __ldcg(slots + (size_t)(s2 + j) * slot_elems + idx);
            #pragma unroll
            for (int j = 0; j < 8; ++j) v += t[j];
          }
          for (; s2 < p.ks; ++s2) v += __ldcg(slots + (size_t)s2 * slot_elems + idx);
          for (s2 = 0; s2 < p.ks; ++s2) __stcg(slots + (size_t)s2 * slot_elems + idx, 0.f);   // leave it zeroed
          const int m = idx >> rows_log2, r = idx & (rows_cta - 1);
          const int n = row0 + r;
          if (n < p.N) p.out[(long long)(m0 + m) * p.ldo + n] = __float2half_rn(finish_value<WBITS>(p, v, n));
        }
        if (ctid == 0) p.counters[tile_id] = 0u;     // leave the workspace zeroed
      }
      named_bar_sync(1, nct);   // red, the block scales and last_flag are reused by the next block
    }
  }

  if (greedy) {
    // the CTA's row maxima -> this rank's scratch; the last CTA of the grid
    // exchanges the keys with the other ranks and writes the columns
    named_bar_sync(1, nct);
    unsigned long long* scratch = xchg::scratch_of(p.amax);
    for (int i = ctid; i < mvalid; i += nct) atomicMax(scratch + m0 + i, amax_s[i]);
    named_bar_sync(1, nct);
    if (ctid == 0) {
      *last_flag = xchg::arrive_last(p.amax, gridDim.x * gridDim.y * gridDim.z) ? 1 : 0;
      amax_s[0] = xchg_done;            // hand the epoch to the other threads (row maxima are merged)
    }
    named_bar_sync(1, nct);
    if (*last_flag)
      xchg::publish_and_combine(p.amax, p.M, ctid, nct, p.err, [&] { named_bar_sync(1, nct); },
                                (unsigned)amax_s[0]);
  }
}

}  // namespace gemv
}  // namespace ql
