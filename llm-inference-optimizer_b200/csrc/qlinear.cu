// qlinear.cu — C ABI of libqlinear.so (declared in include/qlinear.h).
//
// Host side of the B200 weight-only quantized linear layer: argument
// checks, the shape-based kernel plan (fixed heuristic, no autotuning, so a
// first call can be recorded into a CUDA graph), TMA descriptor encoding and
// the launches.  Every entry point returns a status and allocates nothing.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/qlinear.h"
#include "ql_common.cuh"
#include "qargmax.cuh"
#include "qxchg.cuh"
#include "qgather.cuh"
#include "qformat.cuh"
#include "qdec.cuh"
#include "qgemm.cuh"
#include "qgemv.cuh"

#define QL_VERSION_MAJOR 0
#define QL_VERSION_MINOR 1
#define QL_VERSION_PATCH 0

// Device-global error word written by bounded waits that run out.
__device__ unsigned g_ql_device_error;

// Fixed split-K scratch of ql_w4a16_linear_static_ws: one array per device,
// shared by every call of that entry point on the device.
static __device__ __align__(256) unsigned char g_ql_static_ws[QL_STATIC_WS_BYTES];

namespace {

constexpr int kMaxDevices = 64;
constexpr size_t kSmemOptin = 232448;   // 227 KB dynamic shared memory per block on sm_100

struct DeviceInfo {
  std::once_flag once;
  int status = QL_OK;
  int sms = 0;
  unsigned* err_word = nullptr;
};
DeviceInfo g_dev[kMaxDevices];

int init_device(int dev) {
  int major = 0, minor = 0, sms = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    return QL_ERR_CUDA;
  }
  if (major != 10) return QL_ERR_DEVICE;   // built for sm_100a only
  g_dev[dev].sms = sms;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_ql_device_error) != cudaSuccess) {
    cudaGetLastError();
    return QL_ERR_CUDA;
  }
  g_dev[dev].err_word = static_cast<unsigned*>(p);
  return QL_OK;
}

// Returns the current device's info, or nullptr with *status set.
DeviceInfo* current_device(int* status) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    *status = QL_ERR_DEVICE;
    return nullptr;
  }
  DeviceInfo& d = g_dev[dev];
  std::call_once(d.once, [&] { d.status = init_device(dev); });
  *status = d.status;
  return d.status == QL_OK ? &d : nullptr;
}

// ------------------------------------------------------- tensor maps
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// Weight rows viewed as a 3-D uint8 tensor [rows][kbytes/C][C]: a box of
// (C, kb_stage*128/C, 16) is 16 runs of kb_stage*128 contiguous bytes.
// C is the largest of 128/64/32/16 dividing the row length, so the middle
// dimension ends exactly at the row end and anything past it reads as zero.
int weight_chunk(uint64_t kbytes) {
  for (int c : {128, 64, 32, 16})
    if (kbytes % c == 0) return c;
  return 0;
}

int make_weight_map(CUtensorMap* tm, const void* base, uint64_t kbytes, uint64_t rows, uint64_t row_stride,
                    int chunk, int kb_stage) {
  auto fn = encode_fn();
  if (!fn) return QL_ERR_DEVICE;
  cuuint64_t dims[3] = {(cuuint64_t)chunk, kbytes / chunk, rows};
  cuuint64_t strides[2] = {(cuuint64_t)chunk, row_stride};
  cuuint32_t box[3] = {(cuuint32_t)chunk, (cuuint32_t)(kb_stage * 128 / chunk), 16};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? QL_OK : QL_ERR_UNSUPPORTED;
}

// int4 group scales [G][lds] fp16 as a 2-D map (inner dimension n), box
// (16 rows, 2*kb_stage groups): the scales of one tile for one stage.
int make_scale_map(CUtensorMap* tm, const void* base, uint64_t N, uint64_t G, uint64_t lds, int kb_stage) {
  auto fn = encode_fn();
  if (!fn) return QL_ERR_DEVICE;
  cuuint64_t dims[2] = {N, G};
  cuuint64_t strides[1] = {lds * 2};
  cuuint32_t box[2] = {16, (cuuint32_t)(2 * kb_stage)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? QL_OK : QL_ERR_UNSUPPORTED;
}

// Activations [rows][K] fp16 as a 2-D map, box (64 k, box_rows), 128-byte
// swizzle: the K-major canonical layout the tensor-core B operand reads.
int make_act_map(CUtensorMap* tm, const void* base, uint64_t K, uint64_t rows, uint64_t ld_elems, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return QL_ERR_DEVICE;
  cuuint64_t dims[2] = {K, rows};
  cuuint64_t strides[1] = {ld_elems * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? QL_OK : QL_ERR_UNSUPPORTED;
}

// Packed weight rows as [N][kbytes/C][C] with one C-byte stage per row per
// box (C = 64 for int4, 128 for int8) and the matching swizzle.
int make_gemm_weight_map(CUtensorMap* tm, const void* base, uint64_t kbytes, uint64_t rows, uint64_t row_stride,
                         int chunk, int box_rows = 128) {
  auto fn = encode_fn();
  if (!fn) return QL_ERR_DEVICE;
  cuuint64_t dims[3] = {(cuuint64_t)chunk, kbytes / chunk, rows};
  cuuint64_t strides[2] = {(cuuint64_t)chunk, row_stride};
  cuuint32_t box[3] = {(cuuint32_t)chunk, 1, (cuuint32_t)box_rows};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, chunk == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? QL_OK : QL_ERR_UNSUPPORTED;
}

// ------------------------------------------------------------- launch
// cluster_z > 1: thread-block clusters of 1 x 1 x cluster_z CTAs.
template <typename Kern, typename... Args>
int launch_ex(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, int cluster_z,
              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_z > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 1;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = (unsigned)cluster_z;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return QL_ERR_CUDA;
  }
  return QL_OK;
}

template <typename Kern, typename... Args>
int launch(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, Args... args) {
  return launch_ex(kernel, grid, block, smem, s, pdl, 1, args...);
}

// Raise the dynamic shared-memory limit of a kernel once per device.
template <typename Kern>
int allow_smem(Kern kernel, int slot) {
  static std::atomic<unsigned char> done[kMaxDevices][16];
  int dev = 0;
  cudaGetDevice(&dev);
  if (done[dev][slot].load(std::memory_order_acquire)) return QL_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemOptin) !=
      cudaSuccess) {
    cudaGetLastError();
    return QL_ERR_CUDA;
  }
  done[dev][slot].store(1, std::memory_order_release);
  return QL_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ------------------------------------------------------------- GEMV plan
struct GemvPlan {
  int tpc = 0, wpt = 0, ks = 0, kbps = 0, stages = 0, kb_stage = 0, chunk = 0, mt = 0, mchunks = 0;
  int x_stride = 0, x_rows = 0, nblk = 0, gx = 0, nkb = 0, scale_tma = 0;
  size_t smem = 0, ws_bytes = 0;
  double cost = 0;
};

size_t gemv_ws_bytes(const GemvPlan& p) {
  if (p.ks <= 1) return 0;
  const size_t counters = ((size_t)p.nblk * p.mchunks * 4 + 255) / 256 * 256;
  const size_t partials = (size_t)p.nblk * p.mchunks * p.ks * (8 * p.mt) * (p.tpc * 16) * 4;
  return counters + partials;
}

// Optional override for tuning sweeps: QLINEAR_GEMV_PLAN="tpc,ks" (ks = 0
// lets the planner choose).  When the variable is set at the first call it
// is re-read on every call (so a sweep can change it); otherwise never again.
void plan_override(int* tpc, int* ks) {
  static std::atomic<int> mode{-1};   // -1 unknown, 0 unset, 1 tuning
  int m = mode.load(std::memory_order_relaxed);
  if (m < 0) {
    m = std::getenv("QLINEAR_GEMV_PLAN") ? 1 : 0;
    mode.store(m, std::memory_order_relaxed);
  }
  *tpc = *ks = -1;
  if (m == 0) return;
  const char* e = std::getenv("QLINEAR_GEMV_PLAN");
  if (e && std::sscanf(e, "%d,%d", tpc, ks) != 2) *tpc = *ks = -1;
}

// Fixed, shape-based plan (no autotuning).  The grid is persistent along N:
// with more blocks than resident CTAs, each CTA runs R = ceil(blocks / CTAs)
// blocks back to back while its producer keeps the ring full.  Cost model:
// HBM bandwidth is shared by the active CTAs and limited by the bytes they
// keep in flight (ring depth / latency) and by a per-SM cap; the decode
// arithmetic is issue-bound at a fixed rate; the first data arrives after a
// fixed latency; each block pays an epilogue and split-K a reduction.
constexpr size_t kSmemShared = 110 * 1024;   // two CTAs per SM fit under this
// dynamic shared memory at which two CTAs still share an SM (228 KB per SM,
// 1 KB reserved per CTA)
constexpr size_t kSmemTwoPerSm = 233472 / 2 - 1024;
// Largest activation slice a CTA stages.  Measured: raising it to 176 KB
// (8 rows of an 8960-wide K unsplit) made the planner pick slower plans.
constexpr size_t kXStageMax = 96 * 1024;

bool plan_gemv(int wbits, int64_t M, int64_t N, int64_t K, int sms, size_t ws_avail, int scale_tma,
               GemvPlan* out, int64_t pair_n = 0) {
  const int mt = M <= 8 ? 1 : 2;
  const int mc = 8 * mt;
  const int64_t kbytes = wbits == 4 ? K / 2 : K;
  const int nkb = (int)cdiv(kbytes, 128);
  const int epk = wbits == 4 ? 256 : 128;
  // pair_n > 0 (fused gate+up): N = 2 * pair_n stacked rows, blocks pair
  // gate tiles with up tiles, no K-split
  const int64_t NT = pair_n > 0 ? 2 * cdiv(pair_n, 16) : cdiv(N, 16);
  const int x_rows = (int)std::min<int64_t>(mc, M);
  const int mchunks = (int)cdiv(M, mc);
  if (mchunks > 65535) return false;
  const int chunk = weight_chunk((uint64_t)kbytes);
  if (chunk == 0) return false;
  const int stma = wbits == 4 ? scale_tma : 0;
  // model constants (B200): HBM bandwidth, loaded latency, per-SM stream
  // cap, first-data latency, per-block epilogue, split-K reduction, and the
  // decode issue cost (warp instructions per 2 KB k-block of one tile)
  const double bw_total = 6.5e12, lat = 1.0e-6, bw_sm_max = 120e9, t_fill = 1.5e-6, t_blk = 0.25e-6,
               t_red = 1.0e-6, t_red_blk = 0.5e-6, issue_rate = 2.5 * 1.9e9, bw_x_sm = 480e9;
  const double ipk = (wbits == 4 ? 325.0 : 221.0) * (mt == 2 ? 1.3 : 1.0);
  int o_tpc, o_ks;
  plan_override(&o_tpc, &o_ks);

  GemvPlan best;
  best.cost = 1e30;
  bool found = false;
  for (int tpc : {1, 2, 4, 8}) {
    if (o_tpc > 0 && tpc != o_tpc) continue;
    if (o_tpc <= 0 && tpc > 1 && (int64_t)(tpc / 2) * 16 >= N) continue;
    if (pair_n > 0 && tpc < 2) continue;
    const int64_t nblk = pair_n > 0 ? cdiv(cdiv(pair_n, 16), tpc / 2) : cdiv(NT, tpc);
    if (nblk > INT_MAX / 2) continue;
    int last_kbps = -1;
    for (int ks = 1; ks <= nkb; ++ks) {
      const int kbps = (int)cdiv(nkb, ks);
      if (kbps == last_kbps) continue;
      last_kbps = kbps;
      const int ks_eff = (int)cdiv(nkb, kbps);
      if (o_ks > 0 && ks_eff != o_ks) continue;
      if (pair_n > 0 && ks_eff != 1) continue;
      if (ks_eff > 65535) continue;
      GemvPlan p;
      p.tpc = tpc;
      p.ks = ks_eff;
      p.kbps = kbps;
      p.mt = mt;
      p.mchunks = mchunks;
      p.nblk = (int)nblk;
      p.nkb = nkb;
      p.chunk = chunk;
      p.scale_tma = stma;
      p.x_stride = kbps * epk + 8;
      p.x_rows = x_rows;
      p.wpt = std::min(kbps, ql::gemv::kMaxConsumerWarps / tpc);
      if ((size_t)x_rows * p.x_stride * 2 > kXStageMax) continue;
      p.ws_bytes = gemv_ws_bytes(p);
      if (p.ws_bytes > ws_avail) continue;
      const ql::gemv::Smem base =
          ql::gemv::smem_layout(wbits, mc, x_rows, tpc, p.wpt, 0, 1, p.x_stride, kbps, stma);
      const size_t fixed = base.total + 2 * 8 * 64;
      const double per_x = (double)ks_eff * mchunks;   // CTAs per block column
      for (int per_sm : {2, 1}) {
        const size_t budget = per_sm == 2 ? kSmemShared : kSmemOptin;
        if (budget <= fixed) continue;
        // blocks per CTA and grid width
        const double slots_x = std::max(1.0, std::floor((double)sms * per_sm / per_x));
        const int64_t R = cdiv(nblk, (int64_t)slots_x);
        const int64_t gx = cdiv(nblk, R);
        // stages: the largest k-chunk that still leaves every tile at least
        // two ring slots (one when a tile has a single stage in total)
        int kbs = 0, P = 0;
        for (int nkc = 1; nkc <= kbps; ++nkc) {
          const int kb = (int)cdiv(kbps, nkc);
          if (kb * 128 / chunk > 256 || (stma && 2 * kb > 256)) continue;   // TMA box extents
          const int nkc_eff = (int)cdiv(kbps, kb);
          const size_t stage_bytes =
              ql::gemv::stage_weight_bytes(kb) + ql::gemv::stage_scale_bytes(wbits, stma, kb);
          const int fit = (int)std::min<size_t>(64, (budget - fixed) / stage_bytes);
          const int64_t per_tile_total = (int64_t)nkc_eff * R;
          const int Pc = (int)std::min<int64_t>(std::min(fit / tpc, 16), per_tile_total);
          if (Pc >= std::min<int64_t>(2, per_tile_total)) {
            kbs = kb;
            P = Pc;
            break;
          }
        }
        if (P == 0) continue;
        GemvPlan q = p;
        q.kb_stage = kbs;
        q.stages = P * tpc;
        q.gx = (int)gx;
        q.smem = ql::gemv::smem_layout(wbits, mc, x_rows, tpc, q.wpt, q.stages, kbs, q.x_stride, kbps, stma).total;
        if (q.smem > kSmemOptin) continue;
        const int resident = q.smem <= kSmemShared ? 2 : 1;
        const double ctas = (double)gx * per_x;
        const double active = std::min(ctas, (double)sms * resident);
        const double stage_b = (double)(16 * kbs * 128);
        const double inflight = active * std::max(1, P - 1) * tpc * stage_b;
        const double bw = std::min(bw_total, inflight / lat);
        const double bw_cta = std::min(bw / active, bw_sm_max / resident);
        // weights of the CTA's blocks, its x slice (staged once, from L2 at a
        // per-SM rate) and, with split-K, the fp32 partials written and read
        const double bytes_cta = (double)R * tpc * 16 * kbps * 128 +
                                 (ks_eff > 1 ? (double)R * mc * tpc * 16 * 4 * 2.0 : 0.0);
        const double x_cta = (double)x_rows * kbps * epk * 2;
        const double t_mem = bytes_cta / bw_cta + x_cta / bw_x_sm;
        const double tiles_kb = (double)NT * nkb * mchunks;   // 2 KB units, all CTAs
        const double t_comp = tiles_kb * ipk / (std::min<double>(ctas, sms) * issue_rate);
        // The stream and the decode overlap only partly at these sizes (a CTA
        // holds few stages): both terms count.  Split-K: a reduction at the
        // end and per block an arrival round trip (one acquire-release
        // atomic).  Constants fitted to forced-plan sweeps on B200 over the
        // config-1/2 shapes at M = 1, 4, 8 and the 14336/4096 projections
        // (the x slice is staged with 8 loads in flight per thread: fast).
        q.cost = t_fill + t_mem + t_comp + R * t_blk + (ks_eff > 1 ? t_red + R * t_red_blk : 0.0);
        // measured on B200: a warp should own 3..8 k-blocks of a tile's split
        // (fewer: the block epilogue dominates; more: the tile's stages drain
        // too slowly to keep its ring slots turning over)
        const double kb_per_warp = (double)kbps / q.wpt;
        if (kb_per_warp < 3.0) q.cost *= 1.0 + 0.1 * (3.0 - kb_per_warp);
        if (kb_per_warp > 8.0) q.cost *= 1.0 + 0.03 * (kb_per_warp - 8.0);
        if (tpc == 8) q.cost *= 1.4;   // measured: 8-tile blocks are always slower than 4-tile ones
        if (q.cost < best.cost * 0.999) {
          best = q;
          found = true;
        }
      }
    }
  }
  if (found) *out = best;
  return found;
}

template <int WBITS, int LAYOUT, int MT>
int launch_gemv_t(const GemvPlan& pl, const CUtensorMap& tm, const CUtensorMap& tms, const ql::gemv::Params& prm,
                  cudaStream_t s, bool pdl) {
  auto kern = ql::gemv::qgemv_kernel<WBITS, LAYOUT, MT>;
  const int slot = (WBITS == 4 ? 0 : 8) + LAYOUT * 4 + MT;
  int st = allow_smem(kern, slot);
  if (st != QL_OK) return st;
  dim3 grid(pl.gx, pl.ks, pl.mchunks);
  dim3 block((pl.tpc * pl.wpt + 1) * 32);
  return launch(kern, grid, block, pl.smem, s, pdl, tm, tms, prm);
}

struct LinearArgs {
  int wbits;
  const void* x;
  const void* w;
  int layout;
  const void* scale;
  int scale_dtype;
  const void* bias;
  int bias_dtype;
  void* out;
  int64_t M, N, K, ldx, ldw, lds, ldo;
  void* ws;
  size_t ws_bytes;
  unsigned flags;
  cudaStream_t stream;
  int64_t swiglu_n = 0;   // > 0: fused gate+up, N = 2 * swiglu_n stacked weight rows
  const ql::xchg::Ctx* amax = nullptr;   // greedy head: argmax columns instead of outputs
  bool no_tcdec = false;                 // keep the dispatch off the small-batch tensor-core kernel
};

int run_generic(const LinearArgs& a) {
  ql::fmt::GenericParams p;
  p.x = static_cast<const __half*>(a.x);
  p.w = a.w;
  p.scale = a.scale;
  p.bias = a.bias;
  p.out = static_cast<__half*>(a.out);
  p.ldx = a.ldx;
  p.ldw = a.ldw;
  p.lds = a.lds;
  p.ldo = a.ldo;
  p.M = (int)a.M;
  p.N = (int)a.N;
  p.K = (int)a.K;
  p.scale_f32 = a.scale_dtype == QL_DTYPE_F32;
  p.bias_f32 = a.bias_dtype == QL_DTYPE_F32;
  p.layout = a.layout;
  dim3 grid((unsigned)cdiv(a.N, 8), (unsigned)cdiv(a.M, 8));
  if (grid.y > 65535) return QL_ERR_BAD_SHAPE;
  if (a.wbits == 8) return launch(ql::fmt::qlinear_generic_kernel<8>, grid, dim3(256), 0, a.stream, false, p);
  return launch(ql::fmt::qlinear_generic_kernel<4>, grid, dim3(256), 0, a.stream, false, p);
}

int run_generic(const LinearArgs& a);

// A fused gate+up call the decode kernel has no plan for.
constexpr int kNoPlan = 1;

int run_gemv(const LinearArgs& a, DeviceInfo* dev) {
  GemvPlan pl;
  const size_t avail = a.ws ? a.ws_bytes : 0;
  // int4 scales travel with the weight stages (TMA) when their rows are
  // 16-byte aligned; otherwise every block stages them with plain loads
  const int scale_tma = (a.wbits == 4 && aligned16(a.scale) && a.lds % 8 == 0) ? 1 : 0;
  // no decode plan fits (e.g. a tall K with many batch rows and no
  // workspace for split-K): the portable kernel takes it
  if (!plan_gemv(a.wbits, a.M, a.N, a.K, dev->sms, avail, scale_tma, &pl, a.swiglu_n))
    return a.swiglu_n > 0 ? kNoPlan : run_generic(a);
  if (pl.stages < pl.tpc || pl.stages % pl.tpc != 0 || pl.gx < 1 || pl.gx > pl.nblk)
    return QL_ERR_UNSUPPORTED;
  CUtensorMap tm, tms;
  std::memset(&tms, 0, sizeof(tms));
  const uint64_t kbytes = a.wbits == 4 ? (uint64_t)a.K / 2 : (uint64_t)a.K;
  int st = make_weight_map(&tm, a.w, kbytes, (uint64_t)a.N, (uint64_t)a.ldw, pl.chunk, pl.kb_stage);
  if (st != QL_OK) return st;
  if (pl.scale_tma) {
    st = make_scale_map(&tms, a.scale, (uint64_t)a.N, (uint64_t)(a.K / 128), (uint64_t)a.lds, pl.kb_stage);
    if (st != QL_OK) return st;
  }
  ql::gemv::Params p;
  p.x = static_cast<const __half*>(a.x);
  p.scale = a.scale;
  p.bias = a.bias;
  p.out = static_cast<__half*>(a.out);
  p.ldx = a.ldx;
  p.lds = a.lds;
  p.ldo = a.ldo;
  p.M = (int)a.M;
  p.N = (int)a.N;
  p.K = (int)a.K;
  p.kbytes = (int)kbytes;
  p.nkb = pl.nkb;
  p.kb_per_split = pl.kbps;
  p.ks = pl.ks;
  p.tpc = pl.tpc;
  p.wpt = pl.wpt;
  p.stages = pl.stages;
  p.kb_stage = pl.kb_stage;
  p.chunk = pl.chunk;
  p.x_stride = pl.x_stride;
  p.x_rows = pl.x_rows;
  p.nblk = pl.nblk;
  p.scale_tma = pl.scale_tma;
  p.scale_f32 = a.scale_dtype == QL_DTYPE_F32;
  p.bias_f32 = a.bias_dtype == QL_DTYPE_F32;
  const bool pdl = (a.flags & QL_FLAG_PDL) != 0;
  p.early_weights = pdl ? 1 : 0;
  p.swiglu_n = (int)a.swiglu_n;
  std::memset(&p.amax, 0, sizeof(p.amax));
  if (a.amax) {
    if (pl.ks != 1 || pl.mt != 1 || a.swiglu_n > 0) return QL_ERR_UNSUPPORTED;
    p.amax = *a.amax;
  }
  p.err = dev->err_word;
  if (pl.ks > 1) {
    const size_t counters = ((size_t)pl.nblk * pl.mchunks * 4 + 255) / 256 * 256;
    p.counters = static_cast<uint32_t*>(a.ws);
    p.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(a.ws) + counters);
  } else {
    p.counters = nullptr;
    p.partials = nullptr;
  }
  if (a.wbits == 8) {
    return pl.mt == 1 ? launch_gemv_t<8, 0, 1>(pl, tm, tms, p, a.stream, pdl)
                      : launch_gemv_t<8, 0, 2>(pl, tm, tms, p, a.stream, pdl);
  }
  if (a.layout == QL_W4_LAYOUT_SPLIT_HALF)
    return pl.mt == 1 ? launch_gemv_t<4, 0, 1>(pl, tm, tms, p, a.stream, pdl)
                      : launch_gemv_t<4, 0, 2>(pl, tm, tms, p, a.stream, pdl);
  return pl.mt == 1 ? launch_gemv_t<4, 1, 1>(pl, tm, tms, p, a.stream, pdl)
                    : launch_gemv_t<4, 1, 2>(pl, tm, tms, p, a.stream, pdl);
}

// ------------------------------------------------------------- GEMM plan
// Activation rows per CTA (int4 tiles at 256 when the batch fills them:
// three 72 KB stages fit; int8 stays at 128).  The K-split is chosen at
// launch (launch_gemm_t): the splits of a tile are one thread-block cluster
// and reduce through distributed shared memory, so no workspace is
// involved.
struct GemmPlan {
  int bn = 0;
  int64_t tiles = 0;
  size_t ws_bytes = 0;   // always 0: K-splits reduce inside their cluster
  int stage_cap = 0;     // > 0: ring depth at most this (two CTAs per SM)
};

// Optional override for tuning sweeps: QLINEAR_GEMM_PLAN="ks,stages" (0 =
// the planner's choice), read like QLINEAR_GEMV_PLAN.
void gemm_override(int* ks, int* stages) {
  static std::atomic<int> mode{-1};
  int m = mode.load(std::memory_order_relaxed);
  if (m < 0) {
    m = std::getenv("QLINEAR_GEMM_PLAN") ? 1 : 0;
    mode.store(m, std::memory_order_relaxed);
  }
  *ks = *stages = 0;
  if (m == 0) return;
  const char* e = std::getenv("QLINEAR_GEMM_PLAN");
  if (e && std::sscanf(e, "%d,%d", ks, stages) != 2) *ks = *stages = 0;
}

GemmPlan plan_gemm(int wbits, int64_t M, int64_t N, int64_t K, int sms) {
  GemmPlan g;
  // int8 stages carry twice the weight bytes, so its widest tile is 192
  // rows (three 64 KB stages) where int4 takes 256 (three 72 KB stages);
  // measured: the 192-row int8 tile pays off from M = 1024 (at 512 its 1.4
  // waves lose to the 128-row tile's 1.9)
  g.bn = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : wbits == 4 ? 256 : M >= 1024 ? 192 : 128;
  // int8 beyond 128 rows: 128-row activation tiles with a two-stage ring,
  // so that two CTAs share each SM and one's decode, prologue and epilogue
  // overlap the other's MMAs (measured, config 3 int8: 12 cases 3.56 ->
  // 3.13 ms in all; 1536->8960 at M 8192 704 -> 871 TFLOP/s, 14336->4096
  // 1057 -> 1136; one CTA per SM with the 192/128-row tiles before).  The
  // int4 tiles lose with it (their 256-row tile feeds the MMAs better).
  if (wbits == 8 && M > 128) {
    g.bn = 128;
    g.stage_cap = 2;
  }
  g.tiles = cdiv(N, ql::gemm::kTileN) * cdiv(M, g.bn);
  (void)K;
  (void)sms;
  return g;   // the K-split is chosen at launch, from the kernel's cluster occupancy
}

// How many clusters of cz CTAs of qgemm_kernel<WBITS, LAYOUT, BN> (with
// `smem` dynamic bytes) fit on the device at once; 0 when the query fails.
// Cached per instantiation, device and size (for the default ring depth).
template <int WBITS, int LAYOUT, int BN>
int max_active_clusters(int cz, size_t smem, bool cacheable) {
  auto kern = ql::gemm::qgemm_kernel<WBITS, LAYOUT, BN>;
  static std::atomic<int> cache[kMaxDevices][ql::gemm::kMaxSplits + 1];
  int dev = 0;
  cudaGetDevice(&dev);
  if (cacheable && dev < kMaxDevices) {
    const int c = cache[dev][cz].load(std::memory_order_relaxed);
    if (c > 0) return c - 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, (unsigned)cz);
  cfg.blockDim = dim3(ql::gemm::Layout<WBITS, BN>::kThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = (unsigned)cz;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  if (cacheable && dev < kMaxDevices) cache[dev][cz].store(n + 1, std::memory_order_relaxed);
  return n;
}

// CTAs of qgemm_kernel<WBITS, LAYOUT, BN> that share one SM, by shared
// memory (whole carveout), registers and tensor memory.  The cluster
// occupancy query above counts clusters as if one CTA held an SM (measured
// on B200: 74 two-CTA clusters for 16- to 64-row tiles alike), while the
// narrow tiles run two per SM; the launch plan scales by this.
template <int WBITS, int LAYOUT, int BN>
int ctas_per_sm(size_t smem) {
  using L = ql::gemm::Layout<WBITS, BN>;
  static std::atomic<int> cache[kMaxDevices];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < kMaxDevices) {
    const int c = cache[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int smem_sm = 0, reserved = 0;
  cudaFuncAttributes fa;
  if (cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) != cudaSuccess ||
      cudaFuncGetAttributes(&fa, ql::gemm::qgemm_kernel<WBITS, LAYOUT, BN>) != cudaSuccess) {
    cudaGetLastError();
    return 1;
  }
  int n = (int)((size_t)smem_sm / (smem + (size_t)reserved));
  n = std::min(n, 65536 / std::max(1, fa.numRegs * ql::gemm::Layout<WBITS, BN>::kThreads));
  n = std::min(n, (int)(512 / L::kTmemCols));
  n = std::max(1, n);
  if (dev < kMaxDevices) cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

// Ring depth and K-split of one tensor-core launch.  The split is the
// largest cluster (at most kMaxSplits CTAs, at least two stages each) for
// which a cluster per tile fits on the GPU at once: more splits shorten
// each CTA's K loop, a second wave would double it.
struct GemmLaunch {
  int stages = 0, ks = 1, nk_split = 0, clusters_fit = 0;
  size_t smem = 0;
  int stages_unsplit = 0;     // the plan without a K-split (fallback)
  size_t smem_unsplit = 0;
};

template <int WBITS, int LAYOUT, int BN>
int gemm_launch_plan(int64_t tiles, int nk, GemmLaunch* g, int stage_cap = 0) {
  using L = ql::gemm::Layout<WBITS, BN>;
  auto kern = ql::gemm::qgemm_kernel<WBITS, LAYOUT, BN>;
  int S = (int)std::min<size_t>(6, (kSmemOptin - 1024 - 256) / L::kStage);
  int o_ks, o_stages;
  gemm_override(&o_ks, &o_stages);
  if (o_stages > 0) S = std::min(S, o_stages);
  if (stage_cap > 0) S = std::min(S, stage_cap);
  // a capped or overridden ring plans its K-split as one CTA per SM and
  // skips the occupancy cache (kept for the default ring depth)
  const bool default_ring = o_stages <= 0 && stage_cap <= 0;
  if (S < 3 && BN > 128) return QL_ERR_UNSUPPORTED;
  if (S < 2) return QL_ERR_UNSUPPORTED;
  static std::atomic<unsigned char> done[kMaxDevices];
  int dev = 0;
  cudaGetDevice(&dev);
  if (!done[dev].load(std::memory_order_acquire)) {
    // the whole unified L1/shared array as shared memory, so that two CTAs
    // of the narrow tiles share an SM; clusters of up to 16 K-splits
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemOptin) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared) !=
            cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
      cudaGetLastError();
      return QL_ERR_CUDA;
    }
    done[dev].store(1, std::memory_order_release);
  }
  // split launches (push mode) carry a receive buffer; the narrow tiles
  // give up ring stages rather than the second CTA on the SM
  int S_split = S;
  while (S_split > 2 && L::smem_bytes(S_split, true) > kSmemOptin) --S_split;
  if (BN <= 32)
    while (S_split > 2 && L::smem_bytes(S_split, true) > kSmemTwoPerSm) --S_split;
  g->stages = S_split;
  g->smem = L::smem_bytes(S_split, true);
  int ks = 1;
  if (L::smem_bytes(S_split, true) <= kSmemOptin && L::partial_fits(S_split)) {
    if (o_ks > 0) {
      ks = std::min(std::min(o_ks, ql::gemm::kMaxSplits), nk);
    } else {
      const int per_sm = default_ring ? ctas_per_sm<WBITS, LAYOUT, BN>(g->smem) : 1;
      int sms = 0;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      for (int c = std::min(ql::gemm::kMaxSplits, nk / 2); c >= 2; --c) {
        // with two CTAs per SM the query's one-per-SM packing is pessimistic:
        // measured, 70 clusters of 4 of the 32-row tile run as one wave
        int fit = max_active_clusters<WBITS, LAYOUT, BN>(c, g->smem, default_ring) * per_sm;
        if (per_sm > 1) fit = std::max(fit, (int)(0.95 * sms * per_sm / c));
        if (tiles <= fit) {
          ks = c;
          g->clusters_fit = fit;
          break;
        }
      }
      // Narrow tiles (two CTAs per SM): two CTAs on one SM share its issue
      // slots for the decode, so a split that keeps one CTA per SM wins
      // unless it leaves each CTA more than 1.4x the stages.  Measured on
      // 12 tiles of 8960->1536 (70 stages) at M 32 / 16: 10 splits of 7
      // stages 8.0 / 7.1 us against 14 of 5 (two CTAs on some SMs) 9.0 /
      // 8.1 us; on 28 tiles of 4096->3584 (32 stages): 8 splits of 4
      // stages 6.9 us against 5 of 7 stages 7.8 us.
      if (per_sm > 1 && ks > 1) {
        for (int c = std::min(ql::gemm::kMaxSplits, nk / 2); c >= 2; --c) {
          if (tiles * c > (int64_t)(0.95 * sms)) continue;
          if ((double)cdiv(nk, c) <= 1.4 * (double)cdiv(nk, ks)) {
            ks = c;
            g->clusters_fit = (int)(0.95 * sms) / c;
          }
          break;
        }
      }
    }
  }
  g->nk_split = (int)cdiv(nk, ks);
  g->ks = (int)cdiv(nk, g->nk_split);
  g->stages_unsplit = S;
  g->smem_unsplit = L::smem_bytes(S);
  if (g->ks == 1) {
    g->stages = S;
    g->smem = L::smem_bytes(S);
  }
  return QL_OK;
}

template <int WBITS, int LAYOUT, int BN>
int launch_gemm_t(const LinearArgs& a, const CUtensorMap& tx, const CUtensorMap& tw, ql::gemm::Params prm,
                  int64_t tiles, int stage_cap) {
  GemmLaunch g;
  int st = gemm_launch_plan<WBITS, LAYOUT, BN>(tiles, prm.nk, &g, stage_cap);
  if (st != QL_OK) return st;
  if (prm.nh > 0 && ql::gemm::Layout<WBITS, BN>::kPush && g.ks > 1) {
    // SwiGLU mode has no push-mode reduction: the narrow tiles run unsplit
    g.ks = 1;
    g.nk_split = prm.nk;
    g.stages = g.stages_unsplit;
    g.smem = g.smem_unsplit;
  }
  prm.stages = g.stages;
  prm.nk_split = g.nk_split;
  // (SwiGLU mode: 64 output columns per tile, cdiv(N / 2, 64) = cdiv(N, 128) tiles)
  dim3 grid((unsigned)cdiv(a.N, ql::gemm::kTileN), (unsigned)cdiv(a.M, BN), (unsigned)g.ks);
  if (grid.y > 65535 || grid.z > 65535) return QL_ERR_BAD_SHAPE;
  const bool pdl = (a.flags & QL_FLAG_PDL) != 0;
  st = launch_ex(ql::gemm::qgemm_kernel<WBITS, LAYOUT, BN>, grid, dim3(ql::gemm::Layout<WBITS, BN>::kThreads), g.smem, a.stream, pdl,
                 g.ks, tx, tw, prm);
  if (st == QL_ERR_CUDA && g.ks > 1) {
    // a cluster launch the device refuses (resources taken by other work,
    // a different partitioning): the same product unsplit
    prm.stages = g.stages_unsplit;
    prm.nk_split = prm.nk;
    grid.z = 1;
    st = launch_ex(ql::gemm::qgemm_kernel<WBITS, LAYOUT, BN>, grid, dim3(ql::gemm::Layout<WBITS, BN>::kThreads), g.smem_unsplit,
                   a.stream, pdl, 1, tx, tw, prm);
  }
  return st;
}

// The launch plan of the tensor-core kernel for (wbits, layout, M, N, K).
int gemm_plan_query(int wbits, int layout, int64_t M, int64_t N, int64_t K, int sms, GemmPlan* gp, GemmLaunch* gl) {
  *gp = plan_gemm(wbits, M, N, K, sms);
  const int nk = (int)(K / 128);
  const int bn = gp->bn;
#define QL_GEMM_PLAN_CASE(W, LY, B) return gemm_launch_plan<W, LY, B>(gp->tiles, nk, gl, gp->stage_cap)
  if (wbits == 8) {
    switch (bn) {
      case 16: QL_GEMM_PLAN_CASE(8, 0, 16);
      case 32: QL_GEMM_PLAN_CASE(8, 0, 32);
      case 64: QL_GEMM_PLAN_CASE(8, 0, 64);
      case 128: QL_GEMM_PLAN_CASE(8, 0, 128);
      default: QL_GEMM_PLAN_CASE(8, 0, 192);
    }
  }
  if (layout == QL_W4_LAYOUT_SPLIT_HALF) {
    switch (bn) {
      case 16: QL_GEMM_PLAN_CASE(4, 0, 16);
      case 32: QL_GEMM_PLAN_CASE(4, 0, 32);
      case 64: QL_GEMM_PLAN_CASE(4, 0, 64);
      case 128: QL_GEMM_PLAN_CASE(4, 0, 128);
      default: QL_GEMM_PLAN_CASE(4, 0, 256);
    }
  }
  switch (bn) {
    case 16: QL_GEMM_PLAN_CASE(4, 1, 16);
    case 32: QL_GEMM_PLAN_CASE(4, 1, 32);
    case 64: QL_GEMM_PLAN_CASE(4, 1, 64);
    case 128: QL_GEMM_PLAN_CASE(4, 1, 128);
    default: QL_GEMM_PLAN_CASE(4, 1, 256);
  }
#undef QL_GEMM_PLAN_CASE
}

// Tensor-core path eligibility: int4 always (K % 128 == 0); int8 needs
// K % 128 == 0 so a stage is one 128-byte run of every row.
bool gemm_ok(const LinearArgs& a) {
  const int64_t kbytes = a.wbits == 4 ? a.K / 2 : a.K;
  return a.K % 128 == 0 && kbytes % (a.wbits == 4 ? 64 : 128) == 0 && a.N <= INT_MAX && a.M <= 65535LL * 128;
}

template <int WBITS, int LAYOUT>
int run_gemm_layout(const LinearArgs& a, DeviceInfo* dev, const GemmPlan& g) {
  const int bn = g.bn;
  const uint64_t kbytes = WBITS == 4 ? (uint64_t)a.K / 2 : (uint64_t)a.K;
  CUtensorMap tx, tw;
  int st = make_act_map(&tx, a.x, (uint64_t)a.K, (uint64_t)a.M, (uint64_t)a.ldx, bn);
  if (st != QL_OK) return st;
  // SwiGLU mode loads the gate and up halves of a tile as two 64-row boxes
  st = make_gemm_weight_map(&tw, a.w, kbytes, (uint64_t)a.N, (uint64_t)a.ldw, WBITS == 4 ? 64 : 128,
                            a.swiglu_n > 0 ? ql::gemm::kTileN / 2 : ql::gemm::kTileN);
  if (st != QL_OK) return st;
  ql::gemm::Params p;
  p.scale = a.scale;
  p.bias = a.bias;
  p.out = static_cast<__half*>(a.out);
  p.lds = a.lds;
  p.ldo = a.ldo;
  p.M = (int)a.M;
  p.N = (int)a.N;
  p.K = (int)a.K;
  p.nk = (int)(a.K / 128);
  p.nk_split = p.nk;
  p.stages = 0;
  p.scale_f32 = a.scale_dtype == QL_DTYPE_F32;
  p.bias_f32 = a.bias_dtype == QL_DTYPE_F32;
  p.nh = (int)a.swiglu_n;
  p.err = dev->err_word;
  switch (bn) {
    case 16: return launch_gemm_t<WBITS, LAYOUT, 16>(a, tx, tw, p, g.tiles, g.stage_cap);
    case 32: return launch_gemm_t<WBITS, LAYOUT, 32>(a, tx, tw, p, g.tiles, g.stage_cap);
    case 64: return launch_gemm_t<WBITS, LAYOUT, 64>(a, tx, tw, p, g.tiles, g.stage_cap);
    case 128: return launch_gemm_t<WBITS, LAYOUT, 128>(a, tx, tw, p, g.tiles, g.stage_cap);
    case 192: return launch_gemm_t<WBITS, LAYOUT, WBITS == 4 ? 256 : 192>(a, tx, tw, p, g.tiles, g.stage_cap);
    default: return launch_gemm_t<WBITS, LAYOUT, WBITS == 4 ? 256 : 192>(a, tx, tw, p, g.tiles, g.stage_cap);
  }
}

int run_gemm(const LinearArgs& a, DeviceInfo* dev) {
  const GemmPlan g = plan_gemm(a.wbits, a.M, a.N, a.K, dev->sms);
  if (a.wbits == 8) return run_gemm_layout<8, 0>(a, dev, g);
  if (a.layout == QL_W4_LAYOUT_SPLIT_HALF) return run_gemm_layout<4, 0>(a, dev, g);
  return run_gemm_layout<4, 1>(a, dev, g);
}

// ------------------------------------------- small-batch tensor-core kernel
// qdec_kernel<WBITS, LAYOUT, BN> (csrc/qdec.cuh): 128 weight rows per CTA,
// BN = 16 or 32 activation rows, the K range split over a thread-block
// cluster when the tiles alone do not fill two CTAs per SM.
struct DecPlan {
  int bn = 0, ks = 1, kb_split = 0, stages = 0;
  int64_t tiles = 0;
  size_t smem = 0;
};

// Shapes the kernel takes: fast-path operands (checked by the caller), M <=
// 32, K a multiple of 128 (a stage is one 128-k block of every row).
bool dec_shape_ok(int wbits, int64_t M, int64_t N, int64_t K) {
  (void)wbits;
  return M >= 1 && M <= 32 && K >= 128 && K % 128 == 0 && N >= 1 && N <= INT_MAX && K <= INT_MAX;
}

// Optional override for tuning sweeps: QLINEAR_TCDEC_KS=<splits> (read like
// QLINEAR_GEMV_PLAN: re-read on every call when set at the first call).
int tcdec_override() {
  static std::atomic<int> mode{-1};
  int m = mode.load(std::memory_order_relaxed);
  if (m < 0) {
    m = std::getenv("QLINEAR_TCDEC_KS") ? 1 : 0;
    mode.store(m, std::memory_order_relaxed);
  }
  if (m == 0) return 0;
  const char* e = std::getenv("QLINEAR_TCDEC_KS");
  int v = 0;
  if (!e || std::sscanf(e, "%d", &v) != 1) return 0;
  return v;
}

template <int WBITS, int BN>
bool plan_dec_budget(int64_t N, int64_t K, int sms, size_t budget, DecPlan* d) {
  const int nkb = (int)(K / 128);
  const int64_t tiles = cdiv(N, ql::dec::kRows);
  const int kmax = std::min(ql::dec::kMaxSplits, nkb);
  // K-split: enough CTAs for two per SM when the tiles alone are fewer; more
  // splits when the activation tile would leave the ring shallower than 4
  int ks0 = (int)std::max<int64_t>(1, std::min<int64_t>(2 * sms / tiles, kmax));
  const int o = tcdec_override();
  if (o > 0) ks0 = std::min(o, kmax);
  bool found = false;
  for (int ks = ks0; ks <= kmax; ++ks) {
    const int kbs = (int)cdiv(nkb, ks);
    const int ke = (int)cdiv(nkb, kbs);
    // the deepest ring (up to 8 stages) that keeps two CTAs per SM
    for (int S = std::min(ql::dec::kMaxStages, kbs); S >= std::min(2, kbs); --S) {
      const size_t smem = ql::dec::smem_plan<WBITS, BN>(S, kbs, ke).total;
      if (smem > budget) continue;
      if (!found || S > d->stages) {
        d->bn = BN;
        d->ks = ke;
        d->kb_split = kbs;
        d->stages = S;
        d->tiles = tiles;
        d->smem = smem;
        found = true;
      }
      break;
    }
    if (found && (d->stages >= std::min(4, d->kb_split) || o > 0)) break;
  }
  return found;
}

// Two CTAs per SM where the activation tile allows, else one.
template <int WBITS, int BN>
bool plan_dec_t(int64_t N, int64_t K, int sms, DecPlan* d) {
  return plan_dec_budget<WBITS, BN>(N, K, sms, kSmemTwoPerSm, d) ||
         plan_dec_budget<WBITS, BN>(N, K, sms, kSmemOptin, d);
}

bool plan_dec(int wbits, int64_t M, int64_t N, int64_t K, int sms, DecPlan* d) {
  if (!dec_shape_ok(wbits, M, N, K)) return false;
  if (wbits == 4) return M <= 16 ? plan_dec_t<4, 16>(N, K, sms, d) : plan_dec_t<4, 32>(N, K, sms, d);
  return M <= 16 ? plan_dec_t<8, 16>(N, K, sms, d) : plan_dec_t<8, 32>(N, K, sms, d);
}

// Where the dispatch sends a plain linear to the small-batch tensor-core
// kernel: nowhere, measured.  On B200 one tcgen05.mma with the weights as
// the TMEM A operand (M = 128, K = 16) takes about 125 SM cycles whatever N
// is (timestamped inside the kernel: 8 K-steps of a 128-k block take ~1000
// cycles, the same with the steps spread over four independent
// accumulators), i.e. ~16 fp16 weights per SM cycle: ~2 TB/s of int4 at any
// batch size up to 32, below the mma.sync decode kernel (3.3 TB/s on the
// 1536 -> 151936 lm_head at M = 1) and, from 24 rows, the prefill GEMM.  The
// kernel stays reachable with QL_FLAG_FORCE_TCDEC.
bool use_tcdec(int wbits, int64_t M, int64_t N, int64_t K) {
  (void)wbits;
  (void)M;
  (void)N;
  (void)K;
  return false;
}

template <int WBITS, int LAYOUT, int BN>
int launch_dec_t(const LinearArgs& a, const DecPlan& d, const CUtensorMap& tw, const ql::dec::Params& prm) {
  auto kern = ql::dec::qdec_kernel<WBITS, LAYOUT, BN>;
  static std::atomic<unsigned char> done[kMaxDevices];
  int dev = 0;
  cudaGetDevice(&dev);
  if (!done[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemOptin) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared) !=
            cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
      cudaGetLastError();
      return QL_ERR_CUDA;
    }
    done[dev].store(1, std::memory_order_release);
  }
  dim3 grid((unsigned)d.tiles, 1, (unsigned)d.ks);
  return launch_ex(kern, grid, dim3(ql::dec::kThreads), d.smem, a.stream,
                   (a.flags & QL_FLAG_PDL) != 0, d.ks, tw, prm);
}

int run_dec(const LinearArgs& a, DeviceInfo* dev) {
  DecPlan d;
  if (!plan_dec(a.wbits, a.M, a.N, a.K, dev->sms, &d)) return QL_ERR_UNSUPPORTED;
  if (d.tiles > INT_MAX) return QL_ERR_BAD_SHAPE;
  const uint64_t kbytes = a.wbits == 4 ? (uint64_t)a.K / 2 : (uint64_t)a.K;
  CUtensorMap tw;
  int st = make_gemm_weight_map(&tw, a.w, kbytes, (uint64_t)a.N, (uint64_t)a.ldw, a.wbits == 4 ? 64 : 128);
  if (st != QL_OK) return st;
  ql::dec::Params p;
  p.x = static_cast<const __half*>(a.x);
  p.scale = a.scale;
  p.bias = a.bias;
  p.out = static_cast<__half*>(a.out);
  p.ldx = a.ldx;
  p.lds = a.lds;
  p.ldo = a.ldo;
  p.M = (int)a.M;
  p.N = (int)a.N;
  p.K = (int)a.K;
  p.nkb = (int)(a.K / 128);
  p.kb_split = d.kb_split;
  p.stages = d.stages;
  p.scale_f32 = a.scale_dtype == QL_DTYPE_F32;
  p.bias_f32 = a.bias_dtype == QL_DTYPE_F32;
  p.err = dev->err_word;
  if (a.wbits == 8) return d.bn == 16 ? launch_dec_t<8, 0, 16>(a, d, tw, p) : launch_dec_t<8, 0, 32>(a, d, tw, p);
  if (a.layout == QL_W4_LAYOUT_SPLIT_HALF)
    return d.bn == 16 ? launch_dec_t<4, 0, 16>(a, d, tw, p) : launch_dec_t<4, 0, 32>(a, d, tw, p);
  return d.bn == 16 ? launch_dec_t<4, 1, 16>(a, d, tw, p) : launch_dec_t<4, 1, 32>(a, d, tw, p);
}

// Where the tensor-core GEMM replaces the decode kernel (measured on B200:
// forced-path sweeps of both over M = 8..64 on the config-1 to 4 shapes and
// their 8-way column shards).  The decode kernel re-decodes the weights for
// every 16-row batch chunk, so the GEMM takes every layer from 17 rows —
// except small layers (at most 4 Mi weights, K < 4096: q/k/v/o of
// 1.5B-class models), whose weights stay in L2 across the chunks: the decode kernel
// keeps those up to 64 rows from 17 (int8) / 48 (int4) rows (1536x1536 /
// 1536x2048 at M 64: int8 6.3 / 6.3 us against the GEMM's 6.9 / 7.3, int4
// 6.4 / 6.3 against 6.6 / 7.0), while int4 small layers at least 1024 wide
// take the GEMM from 16 rows (4.1 / 4.3 against 4.3 / 4.4 us).  From 12
// rows the GEMM also takes K >= 4096 (4096x3584 at M 16: 6.9 against 12.4
// us; the decode kernel needs a K-split there), tall-K layers (K >= 3N;
// from 8 rows when K >= 8192: 8960x1536 at M 8, 7.1 against 7.6 us) and
// int4 layers wider than 16384
// (1536x18992 at M 16: 11.6 against 12.8 us).  Below 12 rows the decode
// kernel keeps the rest, which also keeps the one-launch greedy head there.
bool use_gemm(int wbits, int64_t M, int64_t N, int64_t K) {
  const bool small = N * K <= (int64_t)1 << 22 && K < 4096;
  if (small && M <= 64 && M >= (wbits == 8 ? 17 : 48)) return false;
  if (small && wbits == 4 && M >= 16 && N >= 1024) return true;
  if (M > 16) return true;
  if (M < 8) return false;
  if (K >= 3 * N && (M >= 12 || K >= 8192)) return true;
  if (M < 12) return false;
  return K >= 4096 || (wbits == 4 && N >= 16384);
}

// Argument checks shared by the linear entry points; out_cols = the
// columns of `out` (N, or N/2 for the fused gate+up).  QL_OK + *empty when
// there is nothing to do.
int check_args(const LinearArgs& a, int64_t out_cols, bool* empty) {
  *empty = false;
  if (!a.x || !a.w || !a.scale || !a.out) {
    if (a.M == 0 || a.N == 0) {
      *empty = true;
      return QL_OK;
    }
    return QL_ERR_NULL_POINTER;
  }
  if (a.M < 0 || a.N < 0 || a.K < 0) return QL_ERR_BAD_SHAPE;
  if (a.M > INT_MAX || a.N > INT_MAX || a.K > INT_MAX) return QL_ERR_BAD_SHAPE;
  if (a.wbits == 4 && a.K % 128 != 0) return QL_ERR_BAD_SHAPE;
  if (a.M == 0 || a.N == 0) {
    *empty = true;
    return QL_OK;
  }
  const int64_t wrow = a.wbits == 4 ? a.K / 2 : a.K;
  if (a.ldx < a.K || a.ldw < wrow || a.ldo < out_cols) return QL_ERR_BAD_STRIDE;
  if (a.wbits == 4 && a.lds < a.N) return QL_ERR_BAD_STRIDE;
  if (a.scale_dtype != QL_DTYPE_F32 && a.scale_dtype != QL_DTYPE_F16) return QL_ERR_UNSUPPORTED;
  if (a.wbits == 4 && a.scale_dtype != QL_DTYPE_F16) return QL_ERR_UNSUPPORTED;
  if (a.bias && a.bias_dtype != QL_DTYPE_F16 && a.bias_dtype != QL_DTYPE_F32) return QL_ERR_UNSUPPORTED;
  if (a.wbits == 4 && a.layout != QL_W4_LAYOUT_SPLIT_HALF && a.layout != QL_W4_LAYOUT_ADJACENT)
    return QL_ERR_UNSUPPORTED;
  return QL_OK;
}

bool fast_path_ok(const LinearArgs& a) {
  const int64_t wrow = a.wbits == 4 ? a.K / 2 : a.K;
  return a.K > 0 && aligned16(a.x) && a.ldx % 8 == 0 && a.K % 8 == 0 && aligned16(a.w) && a.ldw % 16 == 0 &&
         wrow % 16 == 0;
}

int run_linear(const LinearArgs& a) {
  if (!a.x || !a.w || !a.scale || !a.out) {
    if (a.M == 0 || a.N == 0) return QL_OK;
    return QL_ERR_NULL_POINTER;
  }
  if (a.M < 0 || a.N < 0 || a.K < 0) return QL_ERR_BAD_SHAPE;
  if (a.M > INT_MAX || a.N > INT_MAX || a.K > INT_MAX) return QL_ERR_BAD_SHAPE;
  if (a.wbits == 4 && a.K % 128 != 0) return QL_ERR_BAD_SHAPE;
  if (a.M == 0 || a.N == 0) return QL_OK;
  const int64_t wrow = a.wbits == 4 ? a.K / 2 : a.K;
  if (a.ldx < a.K || a.ldw < wrow || a.ldo < a.N) return QL_ERR_BAD_STRIDE;
  if (a.wbits == 4 && a.lds < a.N) return QL_ERR_BAD_STRIDE;
  if (a.scale_dtype != QL_DTYPE_F32 && a.scale_dtype != QL_DTYPE_F16) return QL_ERR_UNSUPPORTED;
  if (a.wbits == 4 && a.scale_dtype != QL_DTYPE_F16) return QL_ERR_UNSUPPORTED;
  if (a.bias && a.bias_dtype != QL_DTYPE_F16 && a.bias_dtype != QL_DTYPE_F32) return QL_ERR_UNSUPPORTED;
  if (a.wbits == 4 && a.layout != QL_W4_LAYOUT_SPLIT_HALF && a.layout != QL_W4_LAYOUT_ADJACENT)
    return QL_ERR_UNSUPPORTED;
  int st;
  DeviceInfo* dev = current_device(&st);
  if (!dev) return st;
  const bool fast_ok = a.K > 0 && aligned16(a.x) && a.ldx % 8 == 0 && a.K % 8 == 0 && aligned16(a.w) &&
                       a.ldw % 16 == 0 && wrow % 16 == 0;
  if (a.flags & QL_FLAG_FORCE_GEMM) {
    if (!fast_ok || !gemm_ok(a)) return QL_ERR_UNSUPPORTED;
    return run_gemm(a, dev);
  }
  if (a.flags & QL_FLAG_FORCE_TCDEC) {
    if (!fast_ok || !dec_shape_ok(a.wbits, a.M, a.N, a.K) || !gemm_ok(a)) return QL_ERR_UNSUPPORTED;
    return run_dec(a, dev);
  }
  if ((a.flags & QL_FLAG_FORCE_GENERIC) || !fast_ok) return run_generic(a);
  if (!(a.flags & QL_FLAG_FORCE_GEMV) && !a.no_tcdec && use_tcdec(a.wbits, a.M, a.N, a.K) && gemm_ok(a)) {
    const int st = run_dec(a, dev);
    if (st != QL_ERR_UNSUPPORTED) return st;
  }
  if (!(a.flags & QL_FLAG_FORCE_GEMV) && use_gemm(a.wbits, a.M, a.N, a.K) && gemm_ok(a)) return run_gemm(a, dev);
  return run_gemv(a, dev);
}

// Fused gate+up with SwiGLU: weights are 2n stacked rows (gate, then up),
// out[M, n] = silu(x @ gate^T) * (x @ up^T).  The decode kernel does it in
// its epilogue when the dispatch picks it and it has a K-unsplit plan, the
// tensor-core kernel in its epilogue when the dispatch picks that (tiles of
// 64 gate rows and the matching 64 up rows); otherwise (unaligned operands,
// forced portable kernel, no unsplit decode plan) the [M, 2n] product goes
// through the workspace and an elementwise kernel applies SwiGLU.
size_t swiglu_temp_bytes(int64_t M, int64_t n) { return ((size_t)M * 2 * n * 2 + 255) / 256 * 256; }

bool swiglu_fused_plan(int wbits, int64_t M, int64_t n, int64_t K, int sms) {
  if (use_gemm(wbits, M, 2 * n, K)) return false;
  GemvPlan pl;
  return plan_gemv(wbits, M, 2 * n, K, sms, 0, 0, &pl, n) && plan_gemv(wbits, M, 2 * n, K, sms, 0, 1, &pl, n);
}

int run_swiglu(const LinearArgs& a) {
  const int64_t n = a.swiglu_n;
  if (n <= 0 || a.N != 2 * n) return QL_ERR_BAD_SHAPE;
  bool empty;
  int st = check_args(a, n, &empty);
  if (st != QL_OK || empty) return st;
  DeviceInfo* dev = current_device(&st);
  if (!dev) return st;
  const bool fast_ok = fast_path_ok(a);
  if (fast_ok && !(a.flags & (QL_FLAG_FORCE_GEMM | QL_FLAG_FORCE_GENERIC)) &&
      ((a.flags & QL_FLAG_FORCE_GEMV) || !use_gemm(a.wbits, a.M, a.N, a.K))) {
    st = run_gemv(a, dev);
    if (st != kNoPlan) return st;
  }
  if (fast_ok && !(a.flags & (QL_FLAG_FORCE_GEMV | QL_FLAG_FORCE_GENERIC | QL_FLAG_FORCE_TCDEC)) &&
      gemm_ok(a) && ((a.flags & QL_FLAG_FORCE_GEMM) || use_gemm(a.wbits, a.M, a.N, a.K)))
    return run_gemm(a, dev);   // the tensor-core kernel's SwiGLU epilogue (a.swiglu_n > 0)
  const size_t temp = swiglu_temp_bytes(a.M, n);
  if (!a.ws || a.ws_bytes < temp) return QL_ERR_WORKSPACE;
  LinearArgs b = a;
  b.swiglu_n = 0;
  b.out = a.ws;
  b.ldo = 2 * n;
  b.ws = a.ws_bytes > temp ? static_cast<uint8_t*>(a.ws) + temp : nullptr;
  b.ws_bytes = a.ws_bytes - temp;
  st = run_linear(b);
  if (st != QL_OK) return st;
  // 8 columns per thread where n, ldo and out allow 16-byte accesses (the
  // temporary is 256-byte aligned with a row stride of 2n)
  const int vec = n % 8 == 0 && a.ldo % 8 == 0 && aligned16(a.out) && aligned16(a.ws);
  const long long total = a.M * n / (vec ? 8 : 1);
  const unsigned blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>(cdiv(total, 256), 65535LL * 8));
  return launch(ql::fmt::swiglu_kernel, dim3(blocks), dim3(256), 0, a.stream, (a.flags & QL_FLAG_PDL) != 0,
                static_cast<__half*>(a.ws), (long long)(2 * n), (int)a.M, (int)n,
                static_cast<__half*>(a.out), (long long)a.ldo, vec);
}

// Exchange context of one call; QL_OK or the status for bad arguments.
int make_xchg_ctx(ql::xchg::Ctx* c, int64_t col_offset, int rank, int world, int max_m, void* const* peers,
                  int64_t* out) {
  if (!peers || !out) return QL_ERR_NULL_POINTER;
  if (world < 1 || world > QL_XCHG_MAX_RANKS || rank < 0 || rank >= world || max_m < 1 || max_m > 65535 ||
      col_offset < 0)
    return QL_ERR_BAD_SHAPE;
  std::memset(c, 0, sizeof(*c));
  for (int q = 0; q < world; ++q) {
    c->peer[q] = static_cast<unsigned char*>(peers[q]);
    if (!c->peer[q]) return QL_ERR_NULL_POINTER;
  }
  c->out = reinterpret_cast<long long*>(out);
  c->col_offset = col_offset;
  c->rank = rank;
  c->world = world;
  c->max_m = max_m;
  return QL_OK;
}

// Greedy head in one launch: the decode kernel with an unsplit K turns its
// outputs into argmax keys and runs the exchange itself.  Shapes that take
// the tensor-core path, have more than 8 rows, or have no unsplit decode plan, are
// QL_ERR_UNSUPPORTED (the caller runs the linear, then ql_argmax_exchange_f16).
bool greedy_fused_plan(int wbits, int64_t M, int64_t N, int64_t K, int sms, int scale_tma) {
  if (use_gemm(wbits, M, N, K)) return false;
  GemvPlan pl;
  return plan_gemv(wbits, M, N, K, sms, 0, scale_tma, &pl) && pl.ks == 1 && pl.mt == 1;
}

int run_linear_argmax(const LinearArgs& a0, int64_t col_offset, int rank, int world, int max_m, void* const* peers,
                      int64_t* out_ids) {
  if (!a0.x || !a0.w || !a0.scale) return QL_ERR_NULL_POINTER;
  ql::xchg::Ctx c;
  int st = make_xchg_ctx(&c, col_offset, rank, world, max_m, peers, out_ids);
  if (st != QL_OK) return st;
  if (a0.M < 1 || a0.M > max_m || a0.N < 1 || a0.N > INT_MAX || a0.K < 1 || a0.K > INT_MAX ||
      col_offset + a0.N > 0xFFFFFFFFLL)
    return QL_ERR_BAD_SHAPE;
  LinearArgs a = a0;
  a.ldo = a.N;
  a.out = const_cast<void*>(a.x);   // never written in greedy-head mode; satisfies the common checks
  bool empty;
  st = check_args(a, a.N, &empty);
  if (st != QL_OK) return st;
  if (!fast_path_ok(a)) return QL_ERR_UNSUPPORTED;
  DeviceInfo* dev = current_device(&st);
  if (!dev) return st;
  const int scale_tma = (a.wbits == 4 && aligned16(a.scale) && a.lds % 8 == 0) ? 1 : 0;
  if (!greedy_fused_plan(a.wbits, a.M, a.N, a.K, dev->sms, scale_tma)) return QL_ERR_UNSUPPORTED;
  a.ws = nullptr;
  a.ws_bytes = 0;
  a.amax = &c;
  return run_gemv(a, dev);
}

}  // namespace

// ======================================================================
extern "C" {

int ql_w8a16_linear(const void* x, int x_dtype, const void* w_q, const void* scale, int scale_dtype,
                    const void* bias, int bias_dtype, void* out, int64_t M, int64_t N, int64_t K, int64_t ldx,
                    int64_t ldw, int64_t ldo, void* workspace, size_t workspace_bytes, unsigned flags,
                    void* stream) {
  if (x_dtype != QL_DTYPE_F16) return QL_ERR_UNSUPPORTED;
  LinearArgs a{8, x, w_q, 0, scale, scale_dtype, bias, bias_dtype, out, M, N, K, ldx, ldw, 0, ldo,
               workspace, workspace_bytes, flags, static_cast<cudaStream_t>(stream)};
  return run_linear(a);
}

int ql_w4a16_linear(const void* x, int x_dtype, const void* w_packed, int layout, const void* scales,
                    const void* bias, int bias_dtype, void* out, int64_t M, int64_t N, int64_t K, int64_t ldx,
                    int64_t ldw, int64_t lds, int64_t ldo, void* workspace, size_t workspace_bytes,
                    unsigned flags, void* stream) {
  if (x_dtype != QL_DTYPE_F16) return QL_ERR_UNSUPPORTED;
  LinearArgs a{4, x, w_packed, layout, scales, QL_DTYPE_F16, bias, bias_dtype, out, M, N, K, ldx, ldw, lds,
               ldo, workspace, workspace_bytes, flags, static_cast<cudaStream_t>(stream)};
  return run_linear(a);
}

int ql_w8a16_linear_argmax(const void* x, int x_dtype, const void* w_q, const void* scale, int scale_dtype,
                           const void* bias, int bias_dtype, int64_t M, int64_t N, int64_t K, int64_t ldx, int64_t ldw,
                           int64_t col_offset, int rank, int world, int max_m, void* const* peers, int64_t* out_ids,
                           unsigned flags, void* stream) {
  if (x_dtype != QL_DTYPE_F16) return QL_ERR_UNSUPPORTED;
  LinearArgs a{8, x, w_q, 0, scale, scale_dtype, bias, bias_dtype, nullptr, M, N, K, ldx, ldw, 0, N,
               nullptr, 0, flags, static_cast<cudaStream_t>(stream)};
  return run_linear_argmax(a, col_offset, rank, world, max_m, peers, out_ids);
}

int ql_w4a16_linear_argmax(const void* x, int x_dtype, const void* w_packed, int layout, const void* scales,
                           const void* bias, int bias_dtype, int64_t M, int64_t N, int64_t K, int64_t ldx, int64_t ldw,
                           int64_t lds, int64_t col_offset, int rank, int world, int max_m, void* const* peers,
                           int64_t* out_ids, unsigned flags, void* stream) {
  if (x_dtype != QL_DTYPE_F16) return QL_ERR_UNSUPPORTED;
  LinearArgs a{4, x, w_packed, layout, scales, QL_DTYPE_F16, bias, bias_dtype, nullptr, M, N, K, ldx, ldw, lds,
               N, nullptr, 0, flags, static_cast<cudaStream_t>(stream)};
  return run_linear_argmax(a, col_offset, rank, world, max_m, peers, out_ids);
}

int ql_linear_argmax_supported(int wbits, int64_t M, int64_t N, int64_t K) {
  if ((wbits != 4 && wbits != 8) || M < 1 || N < 1 || K < 1 || M > INT_MAX || N > INT_MAX || K > INT_MAX) return 0;
  if (wbits == 4 && K % 128 != 0) return 0;
  int st;
  DeviceInfo* dev = current_device(&st);
  if (!dev) return 0;
  // int4 scales may or may not qualify for TMA (alignment): both plans must be unsplit
  return greedy_fused_plan(wbits, M, N, K, dev->sms, 0) && (wbits == 8 || greedy_fused_plan(wbits, M, N, K, dev->sms, 1))
             ? 1 : 0;
}

int ql_w8a16_gate_up_silu(const void* x, int x_dtype, const void* w_q, const void* scale, int scale_dtype,
                          const void* bias, int bias_dtype, void* out, int64_t M, int64_t N, int64_t K,
                          int64_t ldx, int64_t ldw, int64_t ldo, void* workspace, size_t workspace_bytes,
                          unsigned flags, void* stream) {
  if (x_dtype != QL_DTYPE_F16) return QL_ERR_UNSUPPORTED;
  if (N <= 0 || N > INT_MAX / 2) return N == 0 ? QL_OK : QL_ERR_BAD_SHAPE;
  LinearArgs a{8, x, w_q, 0, scale, scale_dtype, bias, bias_dtype, out, M, 2 * N, K, ldx, ldw, 2 * N,
               ldo, workspace, workspace_bytes, flags, static_cast<cudaStream_t>(stream), N};
  return run_swiglu(a);
}

int ql_w4a16_gate_up_silu(const void* x, int x_dtype, const void* w_packed, int layout, const void* scales,
                          const void* bias, int bias_dtype, void* out, int64_t M, int64_t N, int64_t K,
                          int64_t ldx, int64_t ldw, int64_t lds, int64_t ldo, void* workspace,
                          size_t workspace_bytes, unsigned flags, void* stream) {
  if (x_dtype != QL_DTYPE_F16) return QL_ERR_UNSUPPORTED;
  if (N <= 0 || N > INT_MAX / 2) return N == 0 ? QL_OK : QL_ERR_BAD_SHAPE;
  LinearArgs a{4, x, w_packed, layout, scales, QL_DTYPE_F16, bias, bias_dtype, out, M, 2 * N, K, ldx, ldw, lds,
               ldo, workspace, workspace_bytes, flags, static_cast<cudaStream_t>(stream), N};
  return run_swiglu(a);
}

static size_t swiglu_workspace_size(int wbits, int64_t M, int64_t N, int64_t K);

size_t ql_w8a16_gate_up_silu_workspace_size(int64_t M, int64_t N, int64_t K) {
  return swiglu_workspace_size(8, M, N, K);
}
size_t ql_w4a16_gate_up_silu_workspace_size(int64_t M, int64_t N, int64_t K) {
  return swiglu_workspace_size(4, M, N, K);
}

static size_t workspace_size(int wbits, int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0 || (wbits == 4 && K % 128 != 0)) return 0;
  int st;
  DeviceInfo* dev = current_device(&st);
  if (!dev) return 0;
  // enough for the kernel the dispatch picks; for the decode kernel, the
  // larger of its two int4 scale paths (a forced tensor-core call with less
  // workspace than its split-K needs simply runs unsplit)
  if (K % 128 == 0 && use_gemm(wbits, M, N, K)) return plan_gemm(wbits, M, N, K, dev->sms).ws_bytes;
  size_t bytes = 0;
  for (int stma : {0, 1}) {
    GemvPlan pl;
    if (plan_gemv(wbits, M, N, K, dev->sms, SIZE_MAX, stma, &pl)) bytes = std::max(bytes, pl.ws_bytes);
  }
  return bytes;
}

size_t ql_w8a16_workspace_size(int64_t M, int64_t N, int64_t K) { return workspace_size(8, M, N, K); }

static size_t swiglu_workspace_size(int wbits, int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0 || (wbits == 4 && K % 128 != 0)) return 0;
  int st;
  DeviceInfo* dev = current_device(&st);
  if (!dev) return 0;
  if (swiglu_fused_plan(wbits, M, N, K, dev->sms)) return 0;
  return swiglu_temp_bytes(M, N) + workspace_size(wbits, M, 2 * N, K);
}

int ql_gemv_plan(int wbits, int64_t M, int64_t N, int64_t K, size_t workspace_bytes, int64_t* fields,
                 int nfields) {
  if (!fields || nfields < 12) return QL_ERR_NULL_POINTER;
  if ((wbits != 4 && wbits != 8) || M <= 0 || N <= 0 || K <= 0 || (wbits == 4 && K % 128 != 0))
    return QL_ERR_BAD_SHAPE;
  int st;
  DeviceInfo* dev = current_device(&st);
  const int sms = dev ? dev->sms : 148;   // without a device: the B200 SM count
  GemvPlan pl;
  if (!plan_gemv(wbits, M, N, K, sms, workspace_bytes, 1, &pl)) return QL_ERR_UNSUPPORTED;
  const int64_t v[13] = {pl.tpc, pl.wpt, pl.ks, pl.kbps, pl.stages, pl.mt, pl.mchunks,
                         (int64_t)pl.gx * pl.ks * pl.mchunks, (int64_t)pl.smem, (int64_t)pl.ws_bytes,
                         pl.kb_stage, pl.chunk, (int64_t)(pl.cost * 1e9)};
  for (int i = 0; i < std::min(nfields, 13); ++i) fields[i] = v[i];
  return QL_OK;
}
size_t ql_w4a16_workspace_size(int64_t M, int64_t N, int64_t K) { return workspace_size(4, M, N, K); }

int ql_tcdec_plan(int wbits, int64_t M, int64_t N, int64_t K, int64_t* fields, int nfields) {
  if (!fields || nfields < 7) return QL_ERR_NULL_POINTER;
  if ((wbits != 4 && wbits != 8) || M <= 0 || N <= 0 || K <= 0) return QL_ERR_BAD_SHAPE;
  int st;
  DeviceInfo* dev = current_device(&st);
  const int sms = dev ? dev->sms : 148;   // without a device: the B200 SM count
  DecPlan d;
  if (!plan_dec(wbits, M, N, K, sms, &d)) return QL_ERR_UNSUPPORTED;
  const int64_t v[7] = {d.bn, d.ks, d.kb_split, d.stages, (int64_t)d.smem, d.tiles,
                        use_tcdec(wbits, M, N, K) ? 1 : 0};
  for (int i = 0; i < 7; ++i) fields[i] = v[i];
  return QL_OK;
}

int ql_gemm_plan(int wbits, int layout, int64_t M, int64_t N, int64_t K, int64_t* fields, int nfields) {
  if (!fields || nfields < 8) return QL_ERR_NULL_POINTER;
  if ((wbits != 4 && wbits != 8) || M <= 0 || N <= 0 || K <= 0 || K % 128 != 0 || M > 65535LL * 128 ||
      N > INT_MAX)
    return QL_ERR_BAD_SHAPE;
  if (wbits == 4 && layout != QL_W4_LAYOUT_SPLIT_HALF && layout != QL_W4_LAYOUT_ADJACENT) return QL_ERR_UNSUPPORTED;
  int st;
  DeviceInfo* dev = current_device(&st);
  if (!dev) return st;
  GemmPlan gp;
  GemmLaunch gl;
  st = gemm_plan_query(wbits, layout, M, N, K, dev->sms, &gp, &gl);
  if (st != QL_OK) return st;
  const int64_t v[8] = {gp.bn, gl.ks, gl.nk_split, gl.stages, (int64_t)gl.smem, gp.tiles, gp.tiles * gl.ks,
                        gl.clusters_fit};
  for (int i = 0; i < 8; ++i) fields[i] = v[i];
  return QL_OK;
}

int ql_w8a16_dequantize(const void* w_q, const void* scale, int scale_dtype, float* out, int64_t N, int64_t K,
                        int64_t ldw, void* stream) {
  if (N == 0 || K == 0) return QL_OK;
  if (!w_q || !scale || !out) return QL_ERR_NULL_POINTER;
  if (N < 0 || K < 0 || N > INT_MAX || K > INT_MAX) return QL_ERR_BAD_SHAPE;
  if (ldw < K) return QL_ERR_BAD_STRIDE;
  if (scale_dtype != QL_DTYPE_F32 && scale_dtype != QL_DTYPE_F16) return QL_ERR_UNSUPPORTED;
  int st;
  if (!current_device(&st)) return st;
  const int vec_ok = (reinterpret_cast<uintptr_t>(w_q) % 4 == 0) && ldw % 4 == 0;
  const long long total = N * ((K + 3) / 4);
  const unsigned blocks = (unsigned)cdiv(total, 256);
  return launch(ql::fmt::dequant_int8_kernel, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream),
                false, static_cast<const int8_t*>(w_q), scale, (int)(scale_dtype == QL_DTYPE_F32), out, (int)N,
                (int)K, (long long)ldw, vec_ok);
}

int ql_w4a16_dequantize(const void* w_packed, int layout, const void* scales, float* out, int64_t N, int64_t K,
                        int64_t ldw, int64_t lds, void* stream) {
  if (N == 0 || K == 0) return QL_OK;
  if (!w_packed || !scales || !out) return QL_ERR_NULL_POINTER;
  if (N < 0 || K < 0 || K % 128 != 0 || N > INT_MAX || K > INT_MAX) return QL_ERR_BAD_SHAPE;
  if (ldw < K / 2 || lds < N) return QL_ERR_BAD_STRIDE;
  if (layout != QL_W4_LAYOUT_SPLIT_HALF && layout != QL_W4_LAYOUT_ADJACENT) return QL_ERR_UNSUPPORTED;
  int st;
  if (!current_device(&st)) return st;
  const int vec_ok = (reinterpret_cast<uintptr_t>(w_packed) % 4 == 0) && ldw % 4 == 0;
  const long long total = N * (K / 8);
  const unsigned blocks = (unsigned)cdiv(total, 256);
  return launch(ql::fmt::dequant_int4_kernel, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream),
                false, static_cast<const uint8_t*>(w_packed), layout, static_cast<const __half*>(scales), out,
                (int)N, (int)K, (long long)ldw, (long long)lds, vec_ok);
}

int ql_w4a16_unpack(const void* w_packed, int layout, uint8_t* out, int64_t N, int64_t K, int64_t ldw,
                    void* stream) {
  if (N == 0 || K == 0) return QL_OK;
  if (!w_packed || !out) return QL_ERR_NULL_POINTER;
  if (N < 0 || K < 0 || K % 2 != 0 || N > INT_MAX || K > INT_MAX) return QL_ERR_BAD_SHAPE;
  if (layout == QL_W4_LAYOUT_SPLIT_HALF && K % 128 != 0) return QL_ERR_BAD_SHAPE;
  if (ldw < K / 2) return QL_ERR_BAD_STRIDE;
  if (layout != QL_W4_LAYOUT_SPLIT_HALF && layout != QL_W4_LAYOUT_ADJACENT) return QL_ERR_UNSUPPORTED;
  int st;
  if (!current_device(&st)) return st;
  const long long total = N * K;
  return launch(ql::fmt::unpack_int4_kernel, dim3((unsigned)cdiv(total, 256)), dim3(256), 0,
                static_cast<cudaStream_t>(stream), false, static_cast<const uint8_t*>(w_packed), layout, out,
                (int)N, (int)K, (long long)ldw);
}

int ql_w8a16_quantize(const void* w, int64_t N, int64_t K, int64_t ldw, int8_t* w_q, float* scale,
                      void* stream) {
  if (N == 0) return QL_OK;
  if (!w || !w_q || !scale) return QL_ERR_NULL_POINTER;
  if (N < 0 || K < 0 || N > INT_MAX || K > INT_MAX) return QL_ERR_BAD_SHAPE;
  if (ldw < K) return QL_ERR_BAD_STRIDE;
  int st;
  if (!current_device(&st)) return st;
  return launch(ql::fmt::quantize_int8_kernel, dim3((unsigned)N), dim3(256), 0,
                static_cast<cudaStream_t>(stream), false, static_cast<const __half*>(w), (long long)ldw, (int)K,
                w_q, scale);
}

int ql_w4a16_quantize(const void* w, int64_t N, int64_t K, int64_t ldw, int qmin, int layout, uint8_t* w_packed,
                      void* scales, void* stream) {
  if (N == 0 || K == 0) return QL_OK;
  if (!w || !w_packed || !scales) return QL_ERR_NULL_POINTER;
  if (N < 0 || K < 0 || K % 128 != 0 || N > INT_MAX || K > INT_MAX) return QL_ERR_BAD_SHAPE;
  if (ldw < K) return QL_ERR_BAD_STRIDE;
  if (qmin < -8 || qmin > 0) return QL_ERR_UNSUPPORTED;
  if (layout != QL_W4_LAYOUT_SPLIT_HALF && layout != QL_W4_LAYOUT_ADJACENT) return QL_ERR_UNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(w_packed) % 4 != 0) return QL_ERR_UNSUPPORTED;
  int st;
  if (!current_device(&st)) return st;
  const int G = (int)(K / 128);
  return launch(ql::fmt::quantize_int4_kernel, dim3((unsigned)cdiv(G, 4), (unsigned)std::min<int64_t>(N, 65535)),
                dim3(128), 0,
                static_cast<cudaStream_t>(stream), false, static_cast<const __half*>(w), (long long)ldw, (int)K,
                qmin, layout, w_packed, static_cast<__half*>(scales), (int)N);
}

int ql_argmax_rows_f16(const void* x, int64_t M, int64_t N, int64_t ldx, int64_t col_offset, uint64_t* keys,
                       void* stream) {
  if (M == 0) return QL_OK;
  if (!x || !keys) return QL_ERR_NULL_POINTER;
  if (M < 0 || N <= 0 || M > 65535 || N > INT_MAX || col_offset < 0 || col_offset + N > 0xFFFFFFFFLL)
    return QL_ERR_BAD_SHAPE;
  if (ldx < N) return QL_ERR_BAD_STRIDE;
  int st;
  if (!current_device(&st)) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(keys, 0, (size_t)M * sizeof(uint64_t), s) != cudaSuccess) {
    cudaGetLastError();
    return QL_ERR_CUDA;
  }
  const int vec = aligned16(x) && ldx % 8 == 0 && N % 8 == 0;
  const int span = 8192;   // columns per CTA
  return launch(ql::amax::argmax_rows_kernel, dim3((unsigned)cdiv(N, span), (unsigned)M), dim3(256), 0, s, true,
                static_cast<const __half*>(x), (long long)ldx, (int)N, span, (long long)col_offset, vec,
                reinterpret_cast<unsigned long long*>(keys));
}

size_t ql_xchg_buffer_bytes(int world, int max_m) {
  if (world < 1 || world > QL_XCHG_MAX_RANKS || max_m < 1 || max_m > 65535) return 0;
  return ql::xchg::layout(world, max_m).total;
}

int ql_xchg_alloc(size_t bytes, void** buffer, void* ipc_handle) {
  if (!buffer || !ipc_handle) return QL_ERR_NULL_POINTER;
  if (bytes == 0) return QL_ERR_BAD_SHAPE;
  int st;
  if (!current_device(&st)) return st;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return QL_ERR_CUDA;
  }
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(p);
    return QL_ERR_CUDA;
  }
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(ipc_handle, &h, sizeof(h));
  *buffer = p;
  return QL_OK;
}

int ql_xchg_free(void* buffer) {
  if (!buffer) return QL_OK;
  if (cudaFree(buffer) != cudaSuccess) {
    cudaGetLastError();
    return QL_ERR_CUDA;
  }
  return QL_OK;
}

int ql_xchg_open(const void* ipc_handle, void** peer_buffer) {
  if (!ipc_handle || !peer_buffer) return QL_ERR_NULL_POINTER;
  int st;
  if (!current_device(&st)) return st;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return QL_ERR_CUDA;
  }
  *peer_buffer = p;
  return QL_OK;
}

int ql_xchg_close(void* peer_buffer) {
  if (!peer_buffer) return QL_OK;
  if (cudaIpcCloseMemHandle(peer_buffer) != cudaSuccess) {
    cudaGetLastError();
    return QL_ERR_CUDA;
  }
  return QL_OK;
}

int ql_argmax_exchange_f16(const void* x, int64_t M, int64_t N, int64_t ldx, int64_t col_offset, int rank, int world,
                           int max_m, void* const* peers, int64_t* out, void* stream) {
  if (!x || !peers || !out) return QL_ERR_NULL_POINTER;
  if (world < 1 || world > QL_XCHG_MAX_RANKS || rank < 0 || rank >= world) return QL_ERR_BAD_SHAPE;
  if (M < 1 || M > max_m || max_m > 65535 || N <= 0 || N > INT_MAX || col_offset < 0 ||
      col_offset + N > 0xFFFFFFFFLL)
    return QL_ERR_BAD_SHAPE;
  if (ldx < N) return QL_ERR_BAD_STRIDE;
  int st;
  DeviceInfo* dev = current_device(&st);
  if (!dev) return st;
  ql::xchg::Params p;
  p.x = static_cast<const __half*>(x);
  p.ldx = ldx;
  p.M = (int)M;
  p.N = (int)N;
  p.span = 8192;
  p.vec = aligned16(x) && ldx % 8 == 0 && N % 8 == 0;
  st = make_xchg_ctx(&p.c, col_offset, rank, world, max_m, peers, out);
  if (st != QL_OK) return st;
  p.err = dev->err_word;
  return launch(ql::xchg::argmax_exchange_kernel, dim3((unsigned)cdiv(N, p.span), (unsigned)M), dim3(256), 0,
                static_cast<cudaStream_t>(stream), true, p);
}

size_t ql_gather_buffer_bytes(int max_m, int64_t N) {
  if (max_m < 1 || max_m > 65535 || N < 1 || N > INT_MAX) return 0;
  return ql::gather::layout(max_m, N).total;
}

int ql_allgather_f16(const void* src, int64_t lds, void* out, int64_t ldo, int64_t M, int64_t N, int groups,
                     int64_t block, int rank, int world, int max_m, void* const* peers, unsigned flags,
                     void* stream) {
  if (!out || !peers) return QL_ERR_NULL_POINTER;
  if (world < 1 || world > QL_XCHG_MAX_RANKS || rank < 0 || rank >= world) return QL_ERR_BAD_SHAPE;
  if (groups < 1 || M < 1 || M > max_m || max_m > 65535 || N < 1 || N > INT_MAX || N % groups != 0)
    return QL_ERR_BAD_SHAPE;
  const int64_t ng = N / groups;
  if (block < 1 || block * world < ng) return QL_ERR_BAD_SHAPE;   // the shards must cover a block
  const int64_t c0 = (int64_t)rank * block;
  const int64_t w = c0 >= ng ? 0 : std::min<int64_t>(block, ng - c0);
  if (ldo < N) return QL_ERR_BAD_STRIDE;
  if (src && lds < groups * w) return QL_ERR_BAD_STRIDE;
  for (int q = 0; q < world; ++q)
    if (!peers[q]) return QL_ERR_NULL_POINTER;
  if (world == 1 && !src) return QL_OK;   // nothing to move
  int st;
  DeviceInfo* dev = current_device(&st);
  if (!dev) return st;
  ql::gather::Params p{};
  p.src = static_cast<const __half*>(src);
  p.lds = lds;
  p.out = static_cast<__half*>(out);
  p.ldo = ldo;
  p.ng = ng;
  p.block = block;
  p.M = (int)M;
  p.groups = groups;
  p.rank = rank;
  p.world = world;
  p.max_m = max_m;
  p.cw = ng % 8 == 0 && block % 8 == 0 ? 8 : 1;
  p.vec = p.cw == 8 && aligned16(out) && ldo % 8 == 0 && (!src || (aligned16(src) && lds % 8 == 0));
  // small calls as tagged lines (8-byte column runs: 4-aligned offsets,
  // widths and strides), the rest through the flagged banks.  Lines only
  // when every rank owns columns: a reader waits for the lines of each peer
  // that has some, and those waits are what keep every rank within one call
  // of the others (a rank with none would never be waited for)
  const ql::gather::Layout L = ql::gather::layout(max_m, N);
  p.lines = world > 1 && (int64_t)(world - 1) * block < ng && M <= L.line_rows &&
            M * N * 2 <= ql::gather::kLineMaxPayload &&
            (reinterpret_cast<uintptr_t>(out) & 7u) == 0 && ldo % 4 == 0 && ng % 4 == 0 && block % 4 == 0 &&
            (!src || ((reinterpret_cast<uintptr_t>(src) & 7u) == 0 && lds % 4 == 0));
  for (int q = 0; q < world; ++q) p.peer[q] = static_cast<unsigned char*>(peers[q]);
  p.err = dev->err_word;
  // one CTA per SM at most (every CTA waits on the peers: all must be
  // resident together), fewer when there is little to move.  The flagged
  // protocol's grid depends on the shapes alone: CTA c of every rank
  // handles chunk c of every rank's columns.
  const int64_t units = M * N / (p.lines ? 4 : p.cw);
  const int grid = (int)std::max<int64_t>(
      1, std::min<int64_t>(std::min(dev->sms, ql::gather::kMaxCtas), cdiv(units, 512 * 4)));
  return launch(ql::gather::allgather_kernel, dim3((unsigned)grid), dim3(512), 0, static_cast<cudaStream_t>(stream),
                (flags & QL_FLAG_PDL) != 0, p);
}

// Once per device, with that device current: the host-side name of
// g_ql_static_ws is only a stand-in, so its device address is looked up
// here and checked.  The array is zero when the module loads; the set-up
// clears it once more on the first caller's stream and waits for that
// clear, so calls made later on any stream find it zeroed.
struct StaticWs {
  std::once_flag once;
  int status = QL_OK;
  void* ptr = nullptr;
};
static StaticWs g_static_ws[kMaxDevices];

int ql_w4a16_linear_static_ws(const void* x, int x_dtype, const void* w_packed, int layout, const void* scales,
                              const void* bias, int bias_dtype, void* out, int64_t M, int64_t N, int64_t K,
                              int64_t ldx, int64_t ldw, int64_t lds, int64_t ldo, unsigned flags, void* stream) {
  if (x_dtype != QL_DTYPE_F16) return QL_ERR_UNSUPPORTED;
  int st;
  DeviceInfo* dev = current_device(&st);
  if (!dev) return st;
  if (workspace_size(4, M, N, K) > QL_STATIC_WS_BYTES) return QL_ERR_WORKSPACE;
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) {
    cudaGetLastError();
    return QL_ERR_CUDA;
  }
  StaticWs& w = g_static_ws[d];
  std::call_once(w.once, [&] {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_ql_static_ws) != cudaSuccess || ptr == nullptr) {
      cudaGetLastError();
      w.status = QL_ERR_CUDA;
      return;
    }
    if (cudaMemsetAsync(ptr, 0, QL_STATIC_WS_BYTES, static_cast<cudaStream_t>(stream)) != cudaSuccess ||
        cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) {
      cudaGetLastError();
      w.status = QL_ERR_CUDA;
      return;
    }
    w.ptr = ptr;
  });
  if (w.status != QL_OK) return w.status;
  LinearArgs a{4, x, w_packed, layout, scales, QL_DTYPE_F16, bias, bias_dtype, out, M, N, K, ldx, ldw, lds,
               ldo, w.ptr, (size_t)QL_STATIC_WS_BYTES, flags, static_cast<cudaStream_t>(stream)};
  a.no_tcdec = true;   // the decode kernel with its split-K scratch, as the size check above assumes
  return run_linear(a);
}

const char* ql_strerror(int status) {
  switch (status) {
    case QL_OK: return "ok";
    case QL_ERR_NULL_POINTER: return "qlinear: a required pointer is NULL";
    case QL_ERR_BAD_SHAPE: return "qlinear: unsupported or invalid shape";
    case QL_ERR_BAD_STRIDE: return "qlinear: leading dimension smaller than the row length";
    case QL_ERR_UNSUPPORTED: return "qlinear: dtype, layout, flag or alignment not supported by this build";
    case QL_ERR_WORKSPACE: return "qlinear: workspace too small";
    case QL_ERR_CUDA: return "qlinear: CUDA runtime call failed";
    case QL_ERR_DEVICE: return "qlinear: no usable sm_100 device (this library is built for B200 / sm_100a)";
    case QL_ERR_DEVICE_TIMEOUT: return "qlinear: a kernel gave up a bounded wait";
    default: return "qlinear: unknown status";
  }
}

int ql_version(void) { return (QL_VERSION_MAJOR << 16) | (QL_VERSION_MINOR << 8) | QL_VERSION_PATCH; }

int ql_device_error(int* code_out) {
  if (!code_out) return QL_ERR_NULL_POINTER;
  int st;
  if (!current_device(&st)) return st;
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, g_ql_device_error, sizeof(v)) != cudaSuccess) {
    cudaGetLastError();
    return QL_ERR_CUDA;
  }
  *code_out = (int)v;
  return QL_OK;
}

int ql_clear_device_error(void) {
  int st;
  if (!current_device(&st)) return st;
  const unsigned zero = 0;
  if (cudaMemcpyToSymbol(g_ql_device_error, &zero, sizeof(zero)) != cudaSuccess) {
    cudaGetLastError();
    return QL_ERR_CUDA;
  }
  return QL_OK;
}

}  // extern "C"
