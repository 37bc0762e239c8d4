// qformat.cuh — portable linear kernel and the weight-format kernels.
//
//  * qlinear_generic_kernel: CUDA-core fp32 path for shapes the TMA kernels
//    cannot take (int8 rows whose byte length is not a multiple of 16,
//    misaligned pointers or strides).  One warp per output column n, lanes
//    stride K, warp-shuffle reduction.  Same math as the reference kernels.
//  * unpack / dequantize: bit-exact with unpack_int4 / dequantize_int4 /
//    dequantized_weight; the dequantizers run the same register decoders as
//    the GEMV/GEMM kernels, so they double as a device-side check of them.
//  * quantize: QuantizedLinearInt8/Int4.from_linear on the device,
//    bit-exact (IEEE division, round-half-even rint, fp16 RN scale).
#pragma once

#include "ql_common.cuh"

namespace ql {
namespace fmt {

__device__ __forceinline__ int nibble_at(const uint8_t* row, int k, int layout) {
  if (layout == 0) {
    const int gi = k >> 7, j = k & 127;
    const uint8_t b = row[gi * 64 + (j & 63)];
    return j < 64 ? (b & 0xF) : (b >> 4);
  }
  const uint8_t b = row[k >> 1];
  return (k & 1) ? (b >> 4) : (b & 0xF);
}

// ------------------------------------------------------------- generic
struct GenericParams {
  const __half* x;
  const void* w;          // int8 [N, ldw] or packed uint8 [N, ldw]
  const void* scale;      // int8: [N] f32/f16; int4: [K/128, lds] f16
  const void* bias;
  __half* out;
  long long ldx, ldw, lds, ldo;
  int M, N, K;
  int scale_f32, bias_f32, layout;
};

template <int WBITS>
__global__ void __launch_bounds__(256) qlinear_generic_kernel(const GenericParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * 8 + warp;
  if (n >= p.N) return;
  const int mbeg = blockIdx.y * 8, mend = min(p.M, mbeg + 8);
  const uint8_t* wrow = static_cast<const uint8_t*>(p.w) + (long long)n * p.ldw;
  for (int m0 = mbeg; m0 < mend; m0 += 4) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k = lane; k < p.K; k += 32) {
      float wv;
      if (WBITS == 8) {
        wv = static_cast<float>(reinterpret_cast<const int8_t*>(wrow)[k]);
      } else {
        const float s = __half2float(static_cast<const __half*>(p.scale)[(long long)(k >> 7) * p.lds + n]);
        wv = static_cast<float>(nibble_at(wrow, k, p.layout) - 8) * s;
      }
      #pragma unroll
      for (int mi = 0; mi < 4; ++mi)
        if (m0 + mi < mend) acc[mi] = fmaf(__half2float(p.x[(long long)(m0 + mi) * p.ldx + k]), wv, acc[mi]);
    }
    #pragma unroll
    for (int mi = 0; mi < 4; ++mi) {
      float v = acc[mi];
      #pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      acc[mi] = v;
    }
    if (lane == 0) {
      for (int mi = 0; mi < 4 && m0 + mi < mend; ++mi) {
        float v = acc[mi];
        if (WBITS == 8)
          v *= p.scale_f32 ? static_cast<const float*>(p.scale)[n]
                           : __half2float(static_cast<const __half*>(p.scale)[n]);
        if (p.bias)
          v += p.bias_f32 ? static_cast<const float*>(p.bias)[n]
                          : __half2float(static_cast<const __half*>(p.bias)[n]);
        p.out[(long long)(m0 + mi) * p.ldo + n] = __float2half_rn(v);
      }
    }
  }
}

// -------------------------------------------------------------- unpack
__global__ void unpack_int4_kernel(const uint8_t* packed, int layout, uint8_t* out, int N, int K,
                                   long long ldw) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)N * K) return;
  const int n = (int)(idx / K), k = (int)(idx - (long long)n * K);
  out[idx] = (uint8_t)nibble_at(packed + (long long)n * ldw, k, layout);
}

// ---------------------------------------------------------- dequantize
// One thread per 4 packed bytes (8 weights), through the GEMV decoders.
__global__ void dequant_int4_kernel(const uint8_t* packed, int layout, const __half* scales, float* out,
                                    int N, int K, long long ldw, long long lds, int vec_ok) {
  const int words = K / 8;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)N * words) return;
  const int n = (int)(idx / words), wi = (int)(idx - (long long)n * words);
  const uint8_t* row = packed + (long long)n * ldw;
  float* orow = out + (long long)n * K;
  uint32_t u;
  if (vec_ok) {
    u = *reinterpret_cast<const uint32_t*>(row + 4 * wi);
  } else {
    u = (uint32_t)row[4 * wi] | ((uint32_t)row[4 * wi + 1] << 8) | ((uint32_t)row[4 * wi + 2] << 16) |
        ((uint32_t)row[4 * wi + 3] << 24);
  }
  if (layout == 0) {
    const int b = 4 * wi, gi = b >> 6, j = b & 63;
    const int klo = gi * 128 + j, khi = klo + 64;
    const float s = __half2float(scales[(long long)gi * lds + n]);
    uint32_t lo01, lo23, hi01, hi23;
    dec_w4_split(u, lo01, lo23, hi01, hi23);
    const float2 a = h2_to_f2(lo01), bb = h2_to_f2(lo23), cc = h2_to_f2(hi01), d = h2_to_f2(hi23);
    orow[klo + 0] = a.x * s;  orow[klo + 1] = a.y * s;
    orow[klo + 2] = bb.x * s; orow[klo + 3] = bb.y * s;
    orow[khi + 0] = cc.x * s; orow[khi + 1] = cc.y * s;
    orow[khi + 2] = d.x * s;  orow[khi + 3] = d.y * s;
  } else {
    const int k0 = 8 * wi, gi = k0 >> 7;
    const float s = __half2float(scales[(long long)gi * lds + n]);
    uint32_t p01, p23, p45, p67;
    dec_w4_adjacent(u, p01, p23, p45, p67);
    const float2 a = h2_to_f2(p01), bb = h2_to_f2(p23), cc = h2_to_f2(p45), d = h2_to_f2(p67);
    orow[k0 + 0] = a.x * s;  orow[k0 + 1] = a.y * s;
    orow[k0 + 2] = bb.x * s; orow[k0 + 3] = bb.y * s;
    orow[k0 + 4] = cc.x * s; orow[k0 + 5] = cc.y * s;
    orow[k0 + 6] = d.x * s;  orow[k0 + 7] = d.y * s;
  }
}

// One thread per 4 int8 weights (the tail of a row with K % 4 != 0 is done
// element-wise by the same thread that owns the last full word).
__global__ void dequant_int8_kernel(const int8_t* wq, const void* scale, int scale_f32, float* out, int N,
                                    int K, long long ldw, int vec_ok) {
  const int words = (K + 3) / 4;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)N * words) return;
  const int n = (int)(idx / words), wi = (int)(idx - (long long)n * words);
  const int8_t* row = wq + (long long)n * ldw;
  float* orow = out + (long long)n * K;
  const float s = scale_f32 ? static_cast<const float*>(scale)[n]
                            : __half2float(static_cast<const __half*>(scale)[n]);
  const int k0 = 4 * wi;
  if (k0 + 4 <= K) {
    uint32_t u;
    if (vec_ok) {
      u = *reinterpret_cast<const uint32_t*>(row + k0);
    } else {
      u = (uint32_t)(uint8_t)row[k0] | ((uint32_t)(uint8_t)row[k0 + 1] << 8) |
          ((uint32_t)(uint8_t)row[k0 + 2] << 16) | ((uint32_t)(uint8_t)row[k0 + 3] << 24);
    }
    uint32_t p01, p23;
    dec_w8(u, p01, p23);
    const float2 a = h2_to_f2(p01), b = h2_to_f2(p23);
    orow[k0 + 0] = a.x * s; orow[k0 + 1] = a.y * s;
    orow[k0 + 2] = b.x * s; orow[k0 + 3] = b.y * s;
  } else {
    for (int k = k0; k < K; ++k) orow[k] = static_cast<float>(row[k]) * s;
  }
}

// ------------------------------------------------------------ quantize
// int8, one block (256 threads) per row: scale = max(amax/127, 1e-8),
// q = rint(w / scale) clamped to [-127, 127].
__global__ void __launch_bounds__(256) quantize_int8_kernel(const __half* w, long long ldw, int K, int8_t* wq,
                                                             float* scale) {
  const int n = blockIdx.x;
  const __half* row = w + (long long)n * ldw;
  float amax = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) amax = fmaxf(amax, fabsf(__half2float(row[k])));
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float s = fmaxf(__fdiv_rn(red[0], 127.0f), 1e-8f);
  if (threadIdx.x == 0) scale[n] = s;
  int8_t* orow = wq + (long long)n * K;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    float q = rintf(__fdiv_rn(__half2float(row[k]), s));
    q = fminf(fmaxf(q, -127.f), 127.f);
    orow[k] = static_cast<int8_t>(q);
  }
}

// int4, one warp per (row, group of 128): scale = max(amax/7, 1e-5) rounded
// to fp16, q = rint(w / float(scale16)) clamped to [qmin, 7], nibble q+8.
__global__ void __launch_bounds__(128) quantize_int4_kernel(const __half* w, long long ldw, int K, int qmin,
                                                             int layout, uint8_t* packed, __half* scales,
                                                             int N) {
  const int G = K / 128;
  const int gi = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (gi >= G) return;
  for (int n = blockIdx.y; n < N; n += gridDim.y) {   // rows: grid-stride (gridDim.y <= 65535)
    const __half* src = w + (long long)n * ldw + gi * 128 + lane * 4;
    float v[4];
    float amax = 0.f;
    #pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[i] = __half2float(src[i]);
      amax = fmaxf(amax, fabsf(v[i]));
    }
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const __half s16 = __float2half_rn(fmaxf(__fdiv_rn(amax, 7.0f), 1e-5f));
    const float s = __half2float(s16);
    uint32_t q[4];
    #pragma unroll
    for (int i = 0; i < 4; ++i) {
      float r = rintf(__fdiv_rn(v[i], s));
      r = fminf(fmaxf(r, (float)qmin), 7.f);
      q[i] = static_cast<uint32_t>(static_cast<int>(r) + 8);
    }
    uint8_t* prow = packed + (long long)n * (K / 2) + gi * 64;
    if (layout == 0) {
      // byte j = q[j] | q[j+64] << 4: lanes 0..15 hold k 0..63, lanes 16..31 hold k 64..127
      uint32_t hi[4];
      #pragma unroll
      for (int i = 0; i < 4; ++i) hi[i] = __shfl_down_sync(0xffffffffu, q[i], 16);
      if (lane < 16) {
        uint32_t word = 0;
        #pragma unroll
        for (int i = 0; i < 4; ++i) word |= (q[i] | (hi[i] << 4)) << (8 * i);
        *reinterpret_cast<uint32_t*>(prow + lane * 4) = word;
      }
    } else {
      const uint32_t b0 = q[0] | (q[1] << 4), b1 = q[2] | (q[3] << 4);
      prow[lane * 2] = static_cast<uint8_t>(b0);
      prow[lane * 2 + 1] = static_cast<uint8_t>(b1);
    }
    if (lane == 0) scales[(long long)gi * N + n] = s16;
  }
}

// out[m, n] = silu(y[m, n]) * y[m, n + nh] for the [M, 2nh] product of a
// stacked gate+up weight (fp32 math, one rounding); grid-stride.  y lives in
// the caller's workspace, which must be left zero-filled (split-K scratch
// shares it), so every element is cleared after it is read.
__global__ void __launch_bounds__(256) swiglu_kernel(__half* y, long long ldy, int M, int nh, __half* out,
                                                     long long ldo, int vec) {
  griddep_wait();   // y comes from the kernel before
  griddep_launch_dependents();
  const __half zero = __float2half(0.f);
  if (vec) {
    // 8 columns per thread: 16-byte loads of gate and up, 16-byte stores
    const int nv = nh / 8;
    const long long total = (long long)M * nv;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
      const int m = (int)(i / nv), n = (int)(i - (long long)m * nv) * 8;
      uint4* gp = reinterpret_cast<uint4*>(y + (long long)m * ldy + n);
      uint4* up = reinterpret_cast<uint4*>(y + (long long)m * ldy + nh + n);
      const uint4 gv = *gp, uv = *up;
      *gp = make_uint4(0u, 0u, 0u, 0u);
      *up = make_uint4(0u, 0u, 0u, 0u);
      const __half* gh = reinterpret_cast<const __half*>(&gv);
      const __half* uh = reinterpret_cast<const __half*>(&uv);
      uint4 ov;
      __half* oh = reinterpret_cast<__half*>(&ov);
      #pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float g = __half2float(gh[j]);
        oh[j] = __float2half_rn(g / (1.f + __expf(-g)) * __half2float(uh[j]));
      }
      *reinterpret_cast<uint4*>(out + (long long)m * ldo + n) = ov;
    }
    return;
  }
  const long long total = (long long)M * nh;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(i / nh), n = (int)(i - (long long)m * nh);
    __half* gp = y + (long long)m * ldy + n;
    const float g = __half2float(*gp);
    const float u = __half2float(gp[nh]);
    *gp = zero;
    gp[nh] = zero;
    out[(long long)m * ldo + n] = __float2half_rn(g / (1.f + __expf(-g)) * u);
  }
}

}  // namespace fmt
}  // namespace ql
