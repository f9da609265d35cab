/*
 * llm_kernels_b200.h — C ABI of the sm_100a (B200) llm_kernels inference op set.
 *
 * Every entry point takes plain device pointers, 64-bit sizes/strides (in ELEMENTS), a dtype
 * code where the op is type-generic, and a cudaStream_t passed as `void*` (NULL = legacy
 * default stream).  Compute calls are asynchronous on that stream and return an lk_status
 * code; argument errors are detected on the host before anything is launched.  Outputs and
 * scratch are caller-provided.  One exception allocates: the first int8 GEMM or
 * lk_rmsnorm_linear call on a (device, stream) whose problem splits its last round of tiles
 * allocates that stream's split workspace with cudaMalloc (which may synchronise the device)
 * and keeps it until exit; see lk_int8_gemm_dequant.  lk_rmsnorm_linear_noalloc never
 * allocates.  lk_device_status / lk_clear_device_status synchronise the device.
 *
 * Device-side failures (a pipeline wait that ran out of time) do not trap: the kernel records
 * the failure in a device status word and unwinds.  lk_device_status() reads that word
 * (it synchronises the device) and lk_clear_device_status() resets it.
 *
 * Outputs are caller-allocated.  The reference allocated them inside its wrappers
 * (kernels/flash_attn/flash_attn_fwd.py:136, kernels/int8_gemm/int8_gemm.py:122,
 * csrc/bindings.cpp:53); the Python layer of this library does the same on top of this ABI.
 */
#ifndef LLM_KERNELS_B200_H
#define LLM_KERNELS_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define LK_API __attribute__((visibility("default")))
#else
#define LK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------------------------ */
typedef enum {
  LK_OK = 0,
  LK_ERR_INVALID_ARG = 1,   /* null pointer, bad shape, mismatched sizes                        */
  LK_ERR_UNSUPPORTED = 2,   /* dtype / head dim / layout this build does not implement           */
  LK_ERR_CUDA = 3,          /* a CUDA runtime or driver call failed (see lk_last_cuda_error)    */
  LK_ERR_TIMEOUT = 4,       /* a device-side pipeline wait ran out (from lk_device_status)      */
  LK_ERR_ALIGNMENT = 5,     /* pointer or stride not 16-byte aligned where TMA needs it          */
  LK_ERR_SCRATCH_LIMIT = 6  /* problem larger than a no-allocation entry point's fixed scratch   */
} lk_status;

/* ---- dtype codes ------------------------------------------------------------------------- */
typedef enum { LK_F32 = 0, LK_F16 = 1, LK_BF16 = 2, LK_I8 = 3, LK_I32 = 4 } lk_dtype;

/* Human-readable name of a status code (static string). */
LK_API const char* lk_status_string(int status);

/* The cudaError_t of the last LK_ERR_CUDA returned on this host thread (0 if none). */
LK_API int lk_last_cuda_error(void);

/* ABI version: (major << 16) | minor. */
LK_API int lk_version(void);

/* Makes `device` the current device for this library's calls on the calling host thread.
 * Entry points given a non-NULL stream bind to that stream's device themselves; calls on the
 * legacy default stream (NULL) run on the device set here (default 0). */
LK_API int lk_set_device(int device);

/* Synchronises the current device, then copies its status word into out4 (may be NULL):
 * out4[0] = lk_status of the first device failure (0 = none), out4[1] = failure site id,
 * out4[2] = blockIdx.x, out4[3] = threadIdx.x of the thread that recorded it.
 * Returns out4[0] (or LK_ERR_CUDA). */
LK_API int lk_device_status(int* out4);

/* ---- failure-path test hooks (no counterpart in the reference, which has no device-side
 * error path: kernels/flash_attn/flash_attn_fwd.py:132-135 only asserts on the host) ------ *
 * They let a test make one bounded device wait run out on purpose and check that the kernel
 * records LK_ERR_TIMEOUT, unwinds (in-flight copies and MMAs drained, tensor memory freed)
 * and leaves the context usable.  Nothing faults: the hooks only withhold one copy or one
 * counter update, so a consumer's bounded wait ends with an error status. */

/* Limit of every bounded device wait on the current device, in nanoseconds (<= 0 restores the
 * default of one second).  Synchronous. */
LK_API int lk_debug_set_wait_limit(int64_t ns);

/* Arms a one-shot injection, taken by the next launch of the named kernel in this process:
 *   LK_INJECT_FA_DROP_LOAD        flash attention: the TMA producer of CTA `block` skips ring
 *                                 item `item` (K_j = 2j, V_j = 2j+1): no copy, no arrive;
 *   LK_INJECT_GEMM_DROP_LOAD      one-CTA GEMM (problems with fewer 256x256 tiles than SM
 *                                 pairs): the producer of CTA `block` skips its `item`-th stage;
 *   LK_INJECT_SPLIT_SKIP_PUBLISH  CTA-pair GEMM split tail: the writer warp of leftover tile
 *                                 `item`, warp slot 0, never publishes its partial;
 *   LK_INJECT_REQUANT_SKIP_PUBLISH  re-quantising GEMM: in CTA `block`, the epilogue warp of
 *                                 TMEM quadrant 0 never publishes its row maxima for its
 *                                 `item`-th tile, so that row block's codes warps wait in vain.
 * kind LK_INJECT_NONE disarms. */
typedef enum {
  LK_INJECT_NONE = 0,
  LK_INJECT_FA_DROP_LOAD = 1,
  LK_INJECT_GEMM_DROP_LOAD = 2,
  LK_INJECT_SPLIT_SKIP_PUBLISH = 3,
  LK_INJECT_REQUANT_SKIP_PUBLISH = 4
} lk_inject;
LK_API int lk_debug_inject(int kind, int block, int item);

/* Resets the current device's status word to 0 (synchronous), and re-zeroes the counters of
 * every split workspace of the device, which a launch that gave up may have left non-zero.
 * After a non-zero status, results of launches up to this call are not to be trusted. */
LK_API int lk_clear_device_status(void);

/* ---- quantize_symmetric ------------------------------------------------------------------ *
 * Replaces kernels/int8_gemm/int8_gemm.py:146-161 (quantize_symmetric).
 * Per-row symmetric absmax quantisation of x[rows, cols] (last dim contiguous, row stride
 * x_ld elements; x_dtype LK_F32 / LK_F16 / LK_BF16):
 *     scale[r] = fp32(max_c |x[r,c]|) / 127          (IEEE division, NaN-propagating max)
 *     q[r,c]   = clamp(rint(x[r,c] / scale[r]), -128, 127)  (IEEE division, ties to even;
 *                a NaN quotient gives 0, as the reference's CPU cast does)
 * q is int8 with row stride q_ld; scale is fp32[rows]. */
LK_API int lk_quantize_symmetric(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t x_ld,
                          int8_t* q, int64_t q_ld, float* scale, void* stream);

/* ---- int8 GEMM with fused dequant --------------------------------------------------------- *
 * Replaces kernels/int8_gemm/int8_gemm.py:98-138 (int8_gemm_dequant_fwd) and its kernel
 * kernels/int8_gemm/int8_gemm.py:33-90.
 *     acc[m,n] = sum_k A[m,k] * B(k,n)              (exact int32)
 *     C[m,n]   = fp16( (fp32(acc[m,n]) * scale_a[m]) * scale_b[n] )   (two RN multiplies)
 * A is int8 [M,K] row-major with row stride lda.  b_layout selects B's storage:
 *     0 = [K,N] row-major, row stride ldb (the reference's layout, int8_gemm.py:100),
 *     1 = [N,K] row-major, row stride ldb (a weight's natural layout; no transpose copy).
 * C is fp16 [M,N] row-major with row stride ldc.
 * Requirements: K % 16 == 0; lda, ldb, ldc and the base pointers 16-byte aligned.
 * Memory: when a problem's 256 x 256 tiles do not fill whole rounds of SM pairs, the leftover
 * tiles are split along K through a workspace the library allocates once per (device, stream)
 * on first need (~19 MB on a 148-SM part) and keeps; a call captured into a CUDA graph before
 * its stream has one runs unsplit.  Calls on one stream share it (they never overlap); calls
 * on different streams use different workspaces. */
LK_API int lk_int8_gemm_dequant(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, int b_layout,
                         const float* scale_a, const float* scale_b, void* C, int64_t ldc,
                         int64_t M, int64_t N, int64_t K, void* stream);

/* The same GEMM followed by the next layer's activation quantisation, in one kernel: replaces
 * the pair `C = int8_gemm_dequant_fwd(...)`; `q, s = quantize_symmetric(C)` of the reference's
 * int8 linear chain (llm_kernels/__init__.py:111-118 feeding the next Int8Linear), i.e. the
 * quantise-fused decoder path of notebooks/dev_walkthrough.ipynb:264-337.
 *     q[m,n], q_scale[m] = quantize_symmetric(C)[m,n]   bit for bit (C as fp16, as above)
 * The epilogue rounds each output to fp16, the tiles of a row combine their max |C| through
 * `workspace`, and each tile then writes its codes; C itself is written only when C != NULL.
 * q is int8 [M,N] row-major, row stride ldq (a multiple of 16, base 16-byte aligned).
 * workspace: lk_int8_gemm_requant_workspace_bytes(M) bytes of device memory on the current
 * device, 256-byte aligned (any contents; the call clears what must start at zero on its
 * stream), not shared with a concurrent call: 4(M + M/32) bytes of row maxima and counters
 * plus 128 KB per SM where each epilogue warp parks one tile's fp16 values until its row
 * block's maximum is known (~19 MB on a 148-SM B200).
 * LK_ERR_UNSUPPORTED when N > 256 * (SM count / 2) (18944 on a 148-SM B200). */
LK_API int64_t lk_int8_gemm_requant_workspace_bytes(int64_t M);
LK_API int lk_int8_gemm_dequant_requant(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, int b_layout,
                                 const float* scale_a, const float* scale_b, void* C, int64_t ldc, int8_t* q,
                                 int64_t ldq, float* q_scale, void* workspace, int64_t M, int64_t N, int64_t K,
                                 void* stream);

/* Same GEMM, writing the raw int32 accumulator (C int32 [M,N], row stride ldc) instead of the
 * dequantised fp16.  Exists so the accumulator can be checked bit for bit. */
LK_API int lk_int8_gemm_i32(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, int b_layout,
                     int32_t* C, int64_t ldc, int64_t M, int64_t N, int64_t K, void* stream);

/* Column-sharded layer with the gather fused into the epilogue.  Computes this rank's
 * [M, N] column block of dequant(A x B) exactly as lk_int8_gemm_dequant and stores every
 * element into each of dsts[0 .. num_dst) at columns [col_offset, col_offset + N) of an
 * fp16 matrix with row pitch ldc -- typically the replicated [M, N_total] outputs of all ranks,
 * peers' buffers mapped with lk_peer_open, so the all-gather of the reference's optional
 * tensor-parallel mode (an Int8Linear, llm_kernels/__init__.py:82-121, split by output
 * columns) happens tile by tile inside the GEMM over NVLink instead of as a separate
 * collective.  dsts is a host array of device pointers valid on the stream's device.
 * 1 <= num_dst <= 8; ldc and col_offset multiples of 8; every dsts[d] and scale_b 16-byte
 * aligned.
 * The caller orders the launch against the destinations' other users (e.g. a small NCCL
 * all-reduce before and after, as llm_kernels.sharding does). */
LK_API int lk_int8_gemm_dequant_scatter(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, int b_layout,
                                 const float* scale_a, const float* scale_b, void* const* dsts, int num_dst,
                                 int64_t ldc, int64_t col_offset, int64_t M, int64_t N, int64_t K, void* stream);

/* The same column-sharded layer with the gather done by the NVSwitch: multicast_dst is an
 * NVLink multicast address (CUDA multicast object, e.g. torch symmetric memory's
 * multicast_ptr) bound to every rank's replicated [M, N_total] fp16 output, row pitch ldc.
 * Each epilogue chunk is stored once with multimem.st and the switch writes it to all ranks,
 * so a rank sends its block over NVLink once instead of once per peer.  Replaces, like
 * lk_int8_gemm_dequant_scatter, the GEMM + all-gather of a column-split Int8Linear
 * (llm_kernels/__init__.py:82-121); no counterpart in the reference, which has no
 * multi-GPU code.  N % 32 == 0, ldc and col_offset multiples of 8, multicast_dst and scale_b
 * 16-byte aligned.  The caller orders the launch against the outputs' other users on every
 * rank (a barrier before and after). */
LK_API int lk_int8_gemm_dequant_multicast(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, int b_layout,
                                   const float* scale_a, const float* scale_b, void* multicast_dst, int64_t ldc,
                                   int64_t col_offset, int64_t M, int64_t N, int64_t K, void* stream);

/* ---- peer buffers (CUDA IPC) -------------------------------------------------------------- *
 * lk_peer_export writes an LK_PEER_HANDLE_BYTES-byte handle for the allocation holding ptr
 * (on `device`) and ptr's byte offset inside it; another process passes both to lk_peer_open,
 * which maps the allocation on its own `device` (peer access enabled on first use) and returns
 * a pointer that kernels on that device can load from and store to.  lk_peer_close releases
 * it.  Buffers carved out of one allocation share a handle: each (device, handle) is mapped
 * once per process and counted, and its last lk_peer_close unmaps it.  A process cannot open
 * its own handles.  No counterpart in the reference (its only multi-GPU path is the
 * benchmark harness). */
#define LK_PEER_HANDLE_BYTES 64
LK_API int lk_peer_export(int device, const void* ptr, void* handle_out, int64_t* offset_out);
LK_API int lk_peer_open(int device, const void* handle, int64_t offset, void** ptr_out);
LK_API int lk_peer_close(int device, void* ptr, int64_t offset);

/* ---- flash attention forward ------------------------------------------------------------ *
 * Replaces kernels/flash_attn/flash_attn_fwd.py:131-156 (flash_attn_forward) and its two
 * kernels (flash_attn_fwd.py:6-64 non-causal, :67-128 causal).
 *     O[b,h,m,:] = sum_n softmax_n(scale * <Q[b,h,m,:], K[b,h,n,:]>) V[b,h,n,:]
 * causal != 0 masks keys n > m (top-left aligned, flash_attn_fwd.py:118).
 * dtype LK_F16 or LK_BF16 for all four tensors; head dim D in {64, 128}; M, N >= 1 arbitrary
 * (no tile-multiple requirement).  Strides are in elements, 4 per tensor in (b, h, row, d)
 * order; the d stride must be 1 and the others multiples of 8 elements.  softmax_scale <= 0
 * selects D^-0.5 (the reference's hard-coded scale, flash_attn_fwd.py:50). */
LK_API int lk_flash_attn_fwd(const void* q, const void* k, const void* v, void* o, int dtype,
                      int64_t B, int64_t H, int64_t M, int64_t N, int64_t D,
                      const int64_t* q_strides, const int64_t* k_strides,
                      const int64_t* v_strides, const int64_t* o_strides,
                      int causal, float softmax_scale, void* stream);

/* Grouped-query / multi-query attention: K and V hold H_kv heads (H % H_kv == 0) and query
 * head h attends to K/V head h / (H / H_kv) -- the reference's GroupedQueryAttention
 * (experiments/attention_ablation.py:107-141, K/V heads repeat_interleave'd at :125-127) and,
 * with H_kv = 1, MultiQueryAttention (:70-104, one K/V head expanded at :87-88), without
 * materialising the repeated K/V.  k_strides/v_strides index the H_kv-head tensors; all else
 * as lk_flash_attn_fwd, which is this call with H_kv = H. */
LK_API int lk_flash_attn_fwd_gqa(const void* q, const void* k, const void* v, void* o, int dtype,
                          int64_t B, int64_t H, int64_t H_kv, int64_t M, int64_t N, int64_t D,
                          const int64_t* q_strides, const int64_t* k_strides,
                          const int64_t* v_strides, const int64_t* o_strides,
                          int causal, float softmax_scale, void* stream);

/* ---- flash attention: forward with log-sum-exp, and backward ----------------------------- *
 * Replace the reference's training path kernels/flash_attn/flash_attn_bwd.py: its forward
 * that also writes L (flash_attn_fwd_with_lse_kernel, :39-119), its backward kernel (:127-237)
 * and the Delta pre-pass of FlashAttnFunction.backward (:293).  (Those reference kernels cannot
 * run as written -- the head dimension D they use at :85 and :190 is never defined -- so they
 * fix the formulas, not a tested behaviour.)
 *
 * lk_flash_attn_fwd_lse is lk_flash_attn_fwd_gqa that also writes, for every query row,
 *     lse[(b*H + h) * lse_ld + m] = ln( sum_{visible n} exp(scale * <Q[b,h,m,:], K[b,h,n,:]>) )
 * (the reference's L_i = m_i + log(l_i), flash_attn_bwd.py:118-119), fp32, lse_ld >= M.
 *
 * lk_flash_attn_bwd computes, for O = softmax(scale Q K^T [causal mask]) V and its upstream
 * gradient dO (Q, O, dO, dQ [B, H, M, D]; K, V, dK, dV [B, H_kv, N, D], H_kv dividing H, query
 * head h attending to K/V head h / (H / H_kv); dK, dV sum over the query heads sharing a head):
 *     dV = P^T dO,  dS = P * (dO V^T - Delta),  dQ = scale dS K,  dK = scale dS^T Q,
 * with P recomputed from lse (as written by lk_flash_attn_fwd_lse for the same Q, K, scale and
 * mask) and Delta_m = sum_d dO[m,d] O[m,d], which it writes into the caller's `delta` scratch
 * first.  Three kernels on `stream`: the Delta pass, a dK/dV pass over key tiles and a dQ pass
 * over query tiles (no atomics: repeated calls give identical bits).
 *   lse, delta: fp32 [B*H][lse_ld]; lse_ld a multiple of 4 and >= M rounded up to a multiple of
 *               128 (whole 128-row tiles are read; values past M are ignored), 16-byte aligned.
 *   strides:    32 element strides, (b, h, row, d) for q, k, v, o, dout, dq, dk, dv in that
 *               order; d strides 1, the others multiples of 8; o, dout, dq, dk, dv 16-byte
 *               aligned (read / written with 16-byte vectors).
 * dtype LK_F16 or LK_BF16, D in {64, 128}, M, N >= 1 arbitrary, softmax_scale <= 0 = D^-0.5. */
LK_API int lk_flash_attn_fwd_lse(const void* q, const void* k, const void* v, void* o, float* lse, int64_t lse_ld,
                                 int dtype, int64_t B, int64_t H, int64_t H_kv, int64_t M, int64_t N, int64_t D,
                                 const int64_t* q_strides, const int64_t* k_strides,
                                 const int64_t* v_strides, const int64_t* o_strides,
                                 int causal, float softmax_scale, void* stream);
LK_API int lk_flash_attn_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
                             const float* lse, int64_t lse_ld, void* dq, void* dk, void* dv, float* delta,
                             int dtype, int64_t B, int64_t H, int64_t H_kv, int64_t M, int64_t N, int64_t D,
                             const int64_t* strides, int causal, float softmax_scale, void* stream);

/* ---- fused RMSNorm + Linear --------------------------------------------------------------- *
 * Replaces csrc/fused_rmsnorm_linear.cu:105-120 (launch_fused_rmsnorm_linear) behind
 * csrc/bindings.cpp:26-67, and the fallback kernels/fused_rmsnorm_linear/fused_ops.py:27-37:
 *     y[r,:] = rsqrt(mean_k x[r,k]^2 + eps) * ( (x[r,:] * w_norm) @ w_lin^T )
 *
 * lk_rmsnorm_linear_fold writes w_fold[n,k] = dtype(w_lin[n,k] * w_norm[k]) — the RMSNorm gain
 * folded into the weight, a weight-side transform done once per weight version (w_norm may be
 * LK_F32, LK_F16 or LK_BF16; w_lin and w_fold are `dtype`).
 *
 * lk_rmsnorm_linear runs two kernels on `stream`: a row kernel that writes
 * row_rstd[r] = rsqrt(mean_k x[r,k]^2 + eps) (fp32 scratch, `rows` floats), and one tcgen05
 * GEMM x @ w_fold^T whose epilogue multiplies row r by row_rstd[r].  The GEMM is launched as a
 * programmatic dependent of the row kernel: only its epilogue waits for row_rstd.
 * dtype LK_F16 or LK_BF16 for x, w_fold and y.  x [rows, d_in] and y [rows, d_out] are
 * row-major with row strides x_ld, y_ld (elements); w_fold is [d_out, d_in] contiguous.
 * Requirements: d_in % 8 == 0, x_ld % 8 == 0, 16-byte aligned base pointers.
 * Memory: large problems may take the same per-(device, stream) split workspace as the int8
 * GEMM (see there); lk_rmsnorm_linear_noalloc never does. */
LK_API int lk_rmsnorm_linear_fold(const void* w_norm, int w_norm_dtype, const void* w_lin, void* w_fold,
                                  int dtype, int64_t d_in, int64_t d_out, void* stream);
LK_API int lk_rmsnorm_linear(const void* x, int64_t x_ld, const void* w_fold, void* y, int64_t y_ld,
                             int dtype, int64_t rows, int64_t d_in, int64_t d_out, float eps,
                             float* row_rstd, void* stream);

/* One-call form with the reference launcher's argument list (csrc/fused_rmsnorm_linear.cu:105:
 * X, W_norm, W_lin, Y, eps, B, D_in, D_out, stream) plus the dtype and two caller-owned scratch
 * buffers: w_fold (D_out * D_in elements of dtype, rewritten on every call) and row_rstd
 * (B floats).  W_norm has the same dtype as X. */
LK_API int lk_fused_rmsnorm_linear(const void* X, const void* W_norm, const void* W_lin, void* Y,
                                   float eps, int64_t B, int64_t D_in, int64_t D_out, int dtype,
                                   void* w_fold, float* row_rstd, void* stream);

/* lk_rmsnorm_linear without the row_rstd scratch argument.  No counterpart in the reference.
 *
 * For callers that cannot allocate device memory when they call the op: an engine that
 * plans every device buffer ahead of time and hands kernels only those buffers, or a
 * plugin host that gives its plugins no allocator.  Such callers still provide x, w_fold
 * (from lk_rmsnorm_linear_fold) and y; the per-row rsqrt scratch lives in a fixed array
 * inside this library, 65536 fp32 values (256 KiB) that every GPU loading the library holds
 * until the process exits.  rows > 65536 returns LK_ERR_SCRATCH_LIMIT before any launch.
 * The entry point itself calls no allocating function.
 *
 * The first call on each device looks up the array's device address (cudaGetSymbolAddress)
 * and caches it with the device's current context (a call after a device reset looks it up
 * again); make that first call before any stream capture begins.  All calls on a
 * device share the one array, so calls that can overlap on the GPU (different streams
 * without ordering between them) race on it; calls on one stream are ordered and safe.
 * Nothing in the array needs to start at zero: each call overwrites every value it reads. */
LK_API int lk_rmsnorm_linear_noalloc(const void* x, int64_t x_ld, const void* w_fold, void* y,
                                     int64_t y_ld, int dtype, int64_t rows, int64_t d_in,
                                     int64_t d_out, float eps, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LLM_KERNELS_B200_H */
