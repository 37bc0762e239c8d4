/*
 * qlinear.h — C ABI of libqlinear.so, the B200 (sm_100a) weight-only
 * quantized linear layer (W8A16 and W4A16, group 128).
 *
 * This is the drop-in boundary for the quantized-linear path of
 * SriramL1/LLM-inference-optimizer.  Each entry point replaces one function
 * of the reference (paths relative to the reference repository root):
 *
 *   ql_w8a16_linear        <- w8a16_linear          src/kernels/w8a16_matmul_triton.py:102-134
 *                             (kernel _w8a16_matmul_kernel, :39-86)
 *   ql_w4a16_linear        <- w4a16_linear          src/kernels/w4a16_matmul_triton.py:134-170
 *                             (kernel _w4a16_matmul_kernel, :62-117)
 *   ql_w8a16_dequantize    <- QuantizedLinearInt8.dequantized_weight  src/quantization/int8.py:52-53
 *   ql_w4a16_dequantize    <- dequantize_int4       src/kernels/w4a16_matmul_triton.py:173-178
 *   ql_w4a16_unpack        <- unpack_int4           src/kernels/w4a16_matmul_triton.py:52-58
 *   ql_w8a16_quantize      <- QuantizedLinearInt8.from_linear  src/quantization/int8.py:44-50
 *   ql_w4a16_quantize      <- QuantizedLinearInt4.from_linear  src/quantization/int4.py:37-49
 *                             (+ pack_int4, w4a16_matmul_triton.py:42-49)
 *
 * Conventions
 *   - Plain pointers and sizes only.  All pointers are device pointers on the
 *     current CUDA device unless stated otherwise; `stream` is a cudaStream_t
 *     (NULL = legacy default stream).  Every call is asynchronous on `stream`,
 *     allocates nothing, never synchronises the device, and is safe to record
 *     into a CUDA graph (no host-side sync, no lazy compilation).
 *   - Matrices are row-major with the leading dimension given in ELEMENTS
 *     (bytes for packed int4 rows).  The reduction dimension K is contiguous.
 *   - Every function returns a status (QL_OK = 0, negative on error) and never
 *     aborts; ql_strerror() turns a status into a message.  Argument errors
 *     are detected on the host before anything is launched.
 *   - The reference's Python asserts (w8a16_matmul_triton.py:110-113,
 *     w4a16_matmul_triton.py:142-148) stay in the Python wrapper; this layer
 *     re-checks what it needs for memory safety.
 */
#ifndef QLINEAR_H_
#define QLINEAR_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ----------------------------------------------------------------- status */
#define QL_OK                   0
#define QL_ERR_NULL_POINTER    -1   /* a required pointer is NULL                       */
#define QL_ERR_BAD_SHAPE       -2   /* negative size, K % 128 != 0 for int4, ...          */
#define QL_ERR_BAD_STRIDE      -3   /* leading dimension smaller than the row            */
#define QL_ERR_UNSUPPORTED     -4   /* dtype / layout / flag this build does not handle  */
#define QL_ERR_WORKSPACE       -5   /* workspace too small for the requested plan        */
#define QL_ERR_CUDA            -6   /* a CUDA runtime call failed (launch, attribute)    */
#define QL_ERR_DEVICE          -7   /* no usable sm_100 device / driver entry point      */
#define QL_ERR_DEVICE_TIMEOUT  -8   /* a kernel gave up a bounded wait (see below)       */

/* ------------------------------------------------------------------ dtypes */
#define QL_DTYPE_F16   0
#define QL_DTYPE_F32   1
#define QL_DTYPE_BF16  2

/* ---------------------------------------------------- int4 packing layouts */
/* The reference's layout: inside each group of 128 along K, byte j (0..63)
 * holds element j in the low nibble and element j+64 in the high nibble
 * (w4a16_matmul_triton.py:10-20, 42-49).  Nibbles are offset-binary q+8.  */
#define QL_W4_LAYOUT_SPLIT_HALF  0
/* Adjacent pairs: byte i holds k = 2i (low nibble) and k = 2i+1 (high).   */
#define QL_W4_LAYOUT_ADJACENT    1

/* ------------------------------------------------------------------- flags */
/* Launch with programmatic dependent launch: the kernel starts streaming its
 * weights (and int4 scales) before the preceding kernel in the stream has
 * finished, and waits for it only before reading x / writing out / using the
 * workspace.  Valid whenever the weight and scale buffers are not written by
 * the kernels queued just before this call (true for inference).           */
#define QL_FLAG_PDL             0x1u
/* Force the tensor-core GEMM (prefill) path regardless of M.  Test hook.   */
#define QL_FLAG_FORCE_GEMM      0x2u
/* Force the decode (GEMV / skinny) path regardless of M.  Test hook.        */
#define QL_FLAG_FORCE_GEMV      0x4u
/* Force the portable CUDA-core path (any shape / alignment).  Test hook.    */
#define QL_FLAG_FORCE_GENERIC   0x8u
/* Force the small-batch tensor-core kernel (tcgen05, decoded weights in
 * TMEM; M <= 32, K % 128 == 0); QL_ERR_UNSUPPORTED where it cannot run.
 * Test hook.                                                                */
#define QL_FLAG_FORCE_TCDEC     0x10u

/* ------------------------------------------------------------------ linear */
/*
 * out[M, N] = x[M, K] @ (w_q[N, K] * scale[N])^T (+ bias[N]),
 * fp32 accumulation, fp16 output (the dtype of x).
 *   x        fp16 [M, ldx]           (x_dtype must be QL_DTYPE_F16)
 *   w_q      int8 [N, ldw]
 *   scale    [N], scale_dtype QL_DTYPE_F32 (reference) or QL_DTYPE_F16
 *   bias     [N] or NULL, bias_dtype QL_DTYPE_F16 or QL_DTYPE_F32
 *   out      fp16 [M, ldo]
 *   workspace / workspace_bytes: optional scratch for the decode kernel's
 *     split-K (the tensor-core kernel reduces its K-splits inside a
 *     thread-block cluster and needs none).  Must be zero-filled before its
 *     first use; every call leaves it zero-filled.  With NULL (or too small)
 *     the decode kernel is planned without split-K, which is always valid
 *     but can be slower for tall-K shapes.  Calls that share one workspace
 *     must not run concurrently (use one per stream).
 */
int ql_w8a16_linear(const void* x, int x_dtype,
                    const void* w_q,
                    const void* scale, int scale_dtype,
                    const void* bias, int bias_dtype,
                    void* out,
                    int64_t M, int64_t N, int64_t K,
                    int64_t ldx, int64_t ldw, int64_t ldo,
                    void* workspace, size_t workspace_bytes,
                    unsigned flags, void* stream);

/*
 * out[M, N] = x[M, K] @ dequant(w_packed, scales)^T (+ bias[N]),
 * dequant = (nibble - 8) * scales[k / 128, n], fp32 accumulation.
 *   w_packed uint8 [N, ldw] (ldw in bytes, >= K/2), layout as above
 *   scales   fp16 [K/128, lds]  (lds >= N)
 *   K must be a multiple of 128.
 */
int ql_w4a16_linear(const void* x, int x_dtype,
                    const void* w_packed, int layout,
                    const void* scales,
                    const void* bias, int bias_dtype,
                    void* out,
                    int64_t M, int64_t N, int64_t K,
                    int64_t ldx, int64_t ldw, int64_t lds, int64_t ldo,
                    void* workspace, size_t workspace_bytes,
                    unsigned flags, void* stream);

/* Workspace bytes the fastest plan for (M, N, K) needs on the current device
 * (0 when that plan needs none).  Deterministic for a given device. */
size_t ql_w8a16_workspace_size(int64_t M, int64_t N, int64_t K);
size_t ql_w4a16_workspace_size(int64_t M, int64_t N, int64_t K);

/* The decode-kernel plan the library would use for (wbits, M, N, K) with a
 * workspace of `workspace_bytes` (SIZE_MAX = unlimited) and 16-byte aligned
 * int4 scale rows, for tuning and tests.  fields[0..11] = tiles of 16 rows
 * per block, consumer warps per tile, K-splits, 128-byte k-blocks per split,
 * ring stages, batch tiles of 8 per CTA, batch chunks, CTAs launched (each
 * runs one or more blocks), dynamic shared bytes, workspace bytes, k-blocks
 * per stage, bytes of the innermost tensor-map dimension (nfields >= 12), and
 * with nfields >= 13 the planner's cost estimate in ns.  Has no
 * counterpart in the reference (its Triton configs are fixed in
 * _pick_config, w8a16_matmul_triton.py:89-99). */
int ql_gemv_plan(int wbits, int64_t M, int64_t N, int64_t K, size_t workspace_bytes,
                 int64_t* fields, int nfields);

/* The tensor-core kernel's launch plan for (wbits, layout, M, N, K) on the
 * current device (K % 128 == 0), for tuning and tests: fields[0..7] =
 * activation rows per tile, K-splits (= thread-block cluster size; the
 * splits of a tile reduce through distributed shared memory), 128-k stages
 * per split, shared-memory ring stages, dynamic shared bytes, tiles, CTAs,
 * clusters of that size the device holds at once (0 without a split)
 * (nfields >= 8).  No counterpart in the reference. */
int ql_gemm_plan(int wbits, int layout, int64_t M, int64_t N, int64_t K, int64_t* fields, int nfields);

/* The small-batch tensor-core kernel's plan for (wbits, M, N, K) on the
 * current device: fields[0..6] = activation rows per tile (16 or 32),
 * K-splits (= cluster size), 128-k blocks per split, ring stages, dynamic
 * shared bytes, 128-row weight tiles, 1 if the dispatch sends this shape to
 * it (nfields >= 7).  QL_ERR_UNSUPPORTED when the kernel cannot take the
 * shape.  No counterpart in the reference. */
int ql_tcdec_plan(int wbits, int64_t M, int64_t N, int64_t K, int64_t* fields, int nfields);

/* ----------------------------------------------- no-allocation variant */
/* Size of the fixed scratch array behind ql_w4a16_linear_static_ws. */
#define QL_STATIC_WS_BYTES (2u * 1024u * 1024u)
/*
 * ql_w4a16_linear without a workspace argument: the split-K scratch comes
 * from one fixed QL_STATIC_WS_BYTES array compiled into the library, so the
 * call needs no device memory beyond the caller's inputs and outputs.  No
 * counterpart in the reference (its Triton launcher needs no scratch).
 * It exists for callers that cannot allocate device memory when they call
 * in and have no spare buffer to hand over: code embedded in a host
 * program or framework that owns every device allocation, or a serving
 * loop where a cudaMalloc/cudaFree (which can synchronise the whole
 * device) is not acceptable in the request path.
 *   - It never calls cudaMalloc, cudaFree or any allocating routine.
 *   - Shapes whose fastest plan needs more scratch than QL_STATIC_WS_BYTES
 *     return QL_ERR_WORKSPACE and launch nothing.
 *   - The first call on a device looks up the array's device address,
 *     clears it on `stream` and waits for the clear (so later calls on any
 *     stream see it zeroed); make that first call before any stream capture.
 *   - All calls on a device share the array.  Each call leaves it zeroed for
 *     the next, but calls that overlap on the GPU (e.g. on two streams) race.
 */
int ql_w4a16_linear_static_ws(const void* x, int x_dtype,
                              const void* w_packed, int layout,
                              const void* scales,
                              const void* bias, int bias_dtype,
                              void* out,
                              int64_t M, int64_t N, int64_t K,
                              int64_t ldx, int64_t ldw, int64_t lds, int64_t ldo,
                              unsigned flags, void* stream);

/* -------------------------------------------------------- format helpers */
/* out_f32[N, K] = w_q * scale (fp32), bit-exact with the reference. */
int ql_w8a16_dequantize(const void* w_q, const void* scale, int scale_dtype,
                        float* out, int64_t N, int64_t K, int64_t ldw,
                        void* stream);
/* out_f32[N, K] = (nibble - 8) * scales (fp32), bit-exact with the reference.
 * Uses the same register-level nibble decoder as the GEMV/GEMM kernels. */
int ql_w4a16_dequantize(const void* w_packed, int layout, const void* scales,
                        float* out, int64_t N, int64_t K, int64_t ldw, int64_t lds,
                        void* stream);
/* out_u8[N, K] = the raw nibbles (0..15) in logical k order. */
int ql_w4a16_unpack(const void* w_packed, int layout, uint8_t* out,
                    int64_t N, int64_t K, int64_t ldw, void* stream);

/* On-device quantizers, bit-exact with the reference's from_linear.
 *   ql_w8a16_quantize: w fp16 [N, K] -> w_q int8 [N, K], scale fp32 [N]
 *   ql_w4a16_quantize: w fp16 [N, K] -> packed uint8 [N, K/2] (layout),
 *                      scales fp16 [K/128, N]; q clamped to [qmin, 7]
 *                      (reference: qmin = -7). */
int ql_w8a16_quantize(const void* w, int64_t N, int64_t K, int64_t ldw,
                      int8_t* w_q, float* scale, void* stream);
int ql_w4a16_quantize(const void* w, int64_t N, int64_t K, int64_t ldw,
                      int qmin, int layout, uint8_t* w_packed, void* scales,
                      void* stream);

/* ----------------------------------------------------- fused gate+up SwiGLU */
/* out[M, N] = silu(x @ gate^T) * (x @ up^T) from ONE quantized weight of 2N
 * stacked rows (rows 0..N-1 = gate_proj, N..2N-1 = up_proj; for int4 the
 * scales are [K/128, lds >= 2N], for int8 scale[2N]; bias [2N] or NULL).
 * Replaces the two projections and the activation of the reference's MLP
 * forward, act_fn(gate_proj(x)) * up_proj(x) (HF Qwen2MLP; the reference
 * fuses only the elementwise part, src/kernels/fused_swiglu_triton.py:21-53).
 * The decode kernel and the tensor-core kernel apply SwiGLU in their
 * epilogues (fp32, one rounding) and never store the [M, 2N] product; only
 * unaligned operands, a forced portable kernel or a decode kernel without a
 * K-unsplit plan send the product through the workspace (size from the
 * *_workspace_size functions; 0 when the decode kernel's fused path runs)
 * and an elementwise kernel. */
int ql_w8a16_gate_up_silu(const void* x, int x_dtype,
                          const void* w_q, const void* scale, int scale_dtype,
                          const void* bias, int bias_dtype,
                          void* out,
                          int64_t M, int64_t N, int64_t K,
                          int64_t ldx, int64_t ldw, int64_t ldo,
                          void* workspace, size_t workspace_bytes,
                          unsigned flags, void* stream);
int ql_w4a16_gate_up_silu(const void* x, int x_dtype,
                          const void* w_packed, int layout,
                          const void* scales,
                          const void* bias, int bias_dtype,
                          void* out,
                          int64_t M, int64_t N, int64_t K,
                          int64_t ldx, int64_t ldw, int64_t lds, int64_t ldo,
                          void* workspace, size_t workspace_bytes,
                          unsigned flags, void* stream);
size_t ql_w8a16_gate_up_silu_workspace_size(int64_t M, int64_t N, int64_t K);
size_t ql_w4a16_gate_up_silu_workspace_size(int64_t M, int64_t N, int64_t K);

/* ------------------------------------------------------------------ argmax */
/* Row-wise argmax of fp16 logits x[M, ldx] (N columns) as packed keys:
 *   keys[m] = max over n of (ord(x[m, n]) << 32) | (0xFFFFFFFF - (col_offset + n))
 * with ord the order-preserving code of the fp16 bits, so the largest key is
 * the largest logit and, among equal logits, the smallest column — the
 * index torch.argmax returns.  Keys of column shards (each passing its first
 * column as col_offset) combine with a max; column = 0xFFFFFFFF - low 32
 * bits.  keys[M] (uint64, device) is overwritten.  Requires
 * col_offset + N <= 2^32 - 1.  Replaces, for a sharded lm_head, the
 * all-gather of the logits that the reference's greedy decode reduces with
 * argmax (src/engine/paged_engine.py:146-147, graphed_decode_engine.py:114-115). */
int ql_argmax_rows_f16(const void* x, int64_t M, int64_t N, int64_t ldx, int64_t col_offset,
                       uint64_t* keys, void* stream);

/* ---------------------------------------------- sharded argmax over NVLink */
/* One launch per rank computes the row argmax of its logit shard and
 * exchanges the per-row keys (as ql_argmax_rows_f16) with the other ranks of
 * the node by plain stores into their exchange buffers over NVLink, then
 * waits (bounded) for theirs and writes out[m] = the global argmax column.
 * Replaces the all-gather of the logits before the reference's greedy
 * argmax (src/engine/paged_engine.py:146-147); no NCCL call.  All ranks
 * must make the same sequence of calls with the same M.
 *
 * Exchange buffers: each rank allocates one (ql_xchg_alloc, sized by
 * ql_xchg_buffer_bytes for the world size and the largest M), shares the
 * 64-byte IPC handle with the others, and opens theirs (ql_xchg_open);
 * peers[q] is rank q's buffer as seen from this rank (peers[rank] = own).
 * A peer wait that runs out records QL_DEVICE_ERROR_PEER_WAIT (5) in the
 * device error word. */
#define QL_XCHG_MAX_RANKS 8
size_t ql_xchg_buffer_bytes(int world, int max_m);
int ql_xchg_alloc(size_t bytes, void** buffer, void* ipc_handle /* 64 bytes out */);
int ql_xchg_free(void* buffer);
int ql_xchg_open(const void* ipc_handle /* 64 bytes */, void** peer_buffer);
int ql_xchg_close(void* peer_buffer);
int ql_argmax_exchange_f16(const void* x, int64_t M, int64_t N, int64_t ldx, int64_t col_offset,
                           int rank, int world, int max_m, void* const* peers, int64_t* out,
                           void* stream);

/* Greedy head in ONE launch per rank: the quantized linear (arguments as
 * ql_w{8,4}a16_linear, minus out/ldo/workspace) of this rank's column shard
 * followed by the exchange above, fused — the decode kernel turns its
 * fp16-rounded outputs into argmax keys in its epilogue and its last CTA
 * runs the exchange; no logits are written.  out_ids[m] = the global argmax
 * column, identical to ql_w{8,4}a16_linear + ql_argmax_exchange_f16.
 * Shapes with more than 8 rows, that need a K-split, or with unaligned
 * operands return QL_ERR_UNSUPPORTED without launching:
 * ql_linear_argmax_supported(wbits, M, N, K) tells in advance (1 = fused). */
int ql_w8a16_linear_argmax(const void* x, int x_dtype, const void* w_q, const void* scale, int scale_dtype,
                           const void* bias, int bias_dtype, int64_t M, int64_t N, int64_t K,
                           int64_t ldx, int64_t ldw, int64_t col_offset, int rank, int world, int max_m,
                           void* const* peers, int64_t* out_ids, unsigned flags, void* stream);
int ql_w4a16_linear_argmax(const void* x, int x_dtype, const void* w_packed, int layout, const void* scales,
                           const void* bias, int bias_dtype, int64_t M, int64_t N, int64_t K,
                           int64_t ldx, int64_t ldw, int64_t lds, int64_t col_offset, int rank, int world,
                           int max_m, void* const* peers, int64_t* out_ids, unsigned flags, void* stream);
int ql_linear_argmax_supported(int wbits, int64_t M, int64_t N, int64_t K);

/* ------------------------------------- sharded outputs: all-gather over NVLink */
/* All-gather of a column-sharded layer's fp16 outputs, one launch per rank,
 * no NCCL: the B200 build's replacement for the all-gather that a
 * column-sharded lm_head / gate+up projection needs (the reference runs one
 * GPU; its unsharded output is QuantizedLinearInt{8,4}.forward, int8.py:62,
 * int4.py:61).  The output out [M, ldo] holds `groups` blocks of
 * N / groups columns; rank q owns columns [q*block, min(N/groups,
 * (q+1)*block)) of every block.  This rank's columns are either already in
 * `out` (src = NULL) or in src [M, groups*w] (lds; w = this rank's width per
 * block: gate columns, then up columns), then copied into out as well.
 * Outputs of up to 4 MiB are pushed into every peer's gather buffer over
 * NVLink as lines whose 8-byte words carry the call's epoch; larger ones are
 * pushed into the peers' banks chunk by chunk, each chunk published to the
 * peer by a ready flag (one release fence, then relaxed system-scope flag
 * stores), and each rank copies a peer's chunk out of its own bank once
 * that flag has reached the call.  The kernel waits (bounded) for
 * every peer's columns: on completion out holds all N columns on every
 * rank.  All ranks make the same sequence of calls with the same shapes and
 * equally aligned buffers.  Gather buffers: ql_gather_buffer_bytes(max_m, N) bytes, allocated
 * and shared with ql_xchg_alloc / ql_xchg_open / ql_xchg_close /
 * ql_xchg_free as the exchange buffers above (peers[rank] = own).  A wait
 * that runs out records QL_DEVICE_ERROR_PEER_WAIT. */
size_t ql_gather_buffer_bytes(int max_m, int64_t N);
int ql_allgather_f16(const void* src, int64_t lds, void* out, int64_t ldo, int64_t M, int64_t N, int groups,
                     int64_t block, int rank, int world, int max_m, void* const* peers, unsigned flags,
                     void* stream);

/* ------------------------------------------------------------- diagnostics */
const char* ql_strerror(int status);
/* Version as (major << 16) | (minor << 8) | patch. */
int ql_version(void);
/* Device error codes (ql_device_error). */
#define QL_DEVICE_ERROR_FULL_WAIT   1   /* a consumer waited too long for a weight stage  */
#define QL_DEVICE_ERROR_EMPTY_WAIT  2   /* the producer waited too long for a free stage  */
#define QL_DEVICE_ERROR_MMA_WAIT    3   /* a tensor-core completion wait ran out          */
#define QL_DEVICE_ERROR_TMEM        4   /* tensor-memory allocation failed                */
#define QL_DEVICE_ERROR_PEER_WAIT   5   /* another rank's keys / columns never arrived    */
/* Kernels never trap: a bounded wait that runs out records a code in a
 * device-global word, and the kernel lets its copies in flight land and
 * returns early.  These read (and clear)
 * that word on the current device; they synchronise the device. */
int ql_device_error(int* code_out);
int ql_clear_device_error(void);

#ifdef __cplusplus
}
#endif
#endif /* QLINEAR_H_ */
