/*
 * tileops_b200.h — C ABI of libtileops_b200.so, the sm_100a kernels behind the
 * TileOps quantized-linear facade (AWQ W4A16, INT8 W8A8, FP8 e4m3, symmetric INT8).
 *
 * Conventions shared by every entry point:
 *   - Pointers are CUDA device pointers on the current device; sizes are int64 element
 *     counts; tensors are dense row-major unless a stride argument says otherwise.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Every call is
 *     asynchronous and stream-ordered; nothing is synchronised inside the library.
 *   - The library never allocates device memory. Kernels that need scratch take a
 *     caller-owned `workspace` of at least the size its `*_workspace_size` query returns.
 *   - Return value: TO_OK (0) or a negative TO_E* status; to_last_error_string() gives the
 *     text of the calling thread's last failure. The Python facade maps TO_EINVAL to
 *     ValueError, TO_EUNSUPPORTED to NotImplementedError / TypeError and the rest to
 *     RuntimeError, the exception types the reference raises.
 *
 * Each declaration names the reference function (path within the TileOps project,
 * file:line) whose arithmetic it reproduces. In the reference these run as PyTorch
 * tensor expressions or TileLang kernels reached through
 * tileops/runtime/_infra.py:492 (dispatch_compile_quant) and
 * tileops/runtime/__init__.py:446,488 (invoke_quant_kernel, invoke_per_token_quant_int8_kernel).
 */
#ifndef TILEOPS_B200_H_
#define TILEOPS_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TO_API __attribute__((visibility("default")))
#else
#define TO_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------------- */
#define TO_OK 0
#define TO_EINVAL (-1)       /* bad shape / value argument           -> ValueError        */
#define TO_EUNSUPPORTED (-2) /* dtype or option this build rejects    -> TypeError / NIE   */
#define TO_ECUDA (-3)        /* CUDA runtime / launch failure         -> RuntimeError      */
#define TO_ETIMEOUT (-4)     /* a bounded device wait gave up         -> RuntimeError      */
#define TO_ENOSPACE (-5)     /* workspace smaller than *_workspace_size                     */

/* ---- dtype codes ------------------------------------------------------------------- */
#define TO_F32 0
#define TO_F16 1
#define TO_BF16 2
#define TO_I8 3
#define TO_E4M3 4 /* float8_e4m3fn (OCP e4m3, finite-only, max 448) */
#define TO_I32 5
#define TO_I64 6

/* ---- library / device ---------------------------------------------------------------- */
TO_API const char* to_version(void);
/* Text of the calling thread's most recent failure ("" if none). */
TO_API const char* to_last_error_string(void);
/* TO_OK when `device` is an sm_100 (B200-class) GPU, else TO_EUNSUPPORTED. */
TO_API int to_device_check(int device);
/* Reads (and with clear != 0 resets) the device-side error word that kernels with bounded
 * waits set when a wait gives up: 0 = no error. Synchronises the current device. */
TO_API int to_device_error_word(int* value, int clear);
/* Device buffers shared between the processes of one node (plumbing for the gathering GEMM,
 * no reference counterpart): to_ipc_alloc allocates `bytes` on the current device and writes
 * its 64-byte CUDA IPC handle; to_ipc_open maps a peer's handle into this process (peer access
 * enabled on demand); to_ipc_close unmaps it; to_ipc_free releases an own buffer. */
TO_API int to_ipc_alloc(size_t bytes, void** ptr, void* handle);
TO_API int to_ipc_open(const void* handle, void** ptr);
TO_API int to_ipc_close(void* ptr);
TO_API int to_ipc_free(void* ptr);
/* Self-test of the bounded waits (library extension, no reference counterpart). One warp waits
 * on a shared-memory mbarrier through the same bounded wait the GEMM pipelines use, with a
 * limit of limit_us microseconds (1 .. 1000000). arrive != 0: the barrier is arrived at first
 * and the wait completes. arrive == 0: nothing arrives, the wait gives up after the limit,
 * records 1 (wait timeout) in the device error word and the kernel returns; the context stays
 * usable. out (device memory, 2 x u64) receives {completed ? 1 : 0, nanoseconds waited}.
 * Asynchronous on stream. */
TO_API int to_wait_limit_selftest(int limit_us, int arrive, unsigned long long* out, void* stream);
/* Launch overlap for the streaming small-M AWQ kernels, the 2-CTA W8A8 kernel, to_gemv and
 * to_peer_barrier (programmatic dependent launch; the GEMV's A counts as its weights): with
 * enable = 1, a launch may start reading its weights, zeros and scales while the previous
 * kernel in the stream is still running; x is read and y written only after that kernel has
 * completed. Use it for chains of layers whose weights no kernel in the stream writes (a
 * decode loop); leave it off (the default) when a kernel that writes the weights, such as
 * to_awq_pack, may be the immediately preceding launch. enable < 0 only queries. Returns the
 * previous setting. Process-wide. No reference counterpart (a launch-policy extension). */
TO_API int to_set_launch_overlap(int enable);

/* ---- symmetric INT8 (tileops/quant.py) ------------------------------------------------
 * q = clamp(round_half_even(float(x) / scale), -128, 127);  y = out_dtype(float(q) * scale).
 * Per-channel: x is viewed as [outer, channels, inner] (the channel axis is `dim`), one
 * fp32 scale per channel, output in the same layout as the input (no permute copies). */
/* replaces tileops/quant.py:53 quantize_per_tensor (kernel backend/cuda/quant.py:32) */
TO_API int to_quant_per_tensor_i8(const void* x, int x_dtype, const float* scale, int8_t* q,
                           int64_t n, void* stream);
/* replaces tileops/quant.py:96 dequantize_per_tensor (kernel backend/cuda/quant.py:49) */
TO_API int to_dequant_per_tensor_i8(const int8_t* q, const float* scale, void* y, int y_dtype,
                             int64_t n, void* stream);
/* replaces tileops/quant.py:144 quantize_per_channel (kernel backend/cuda/quant.py:65) */
TO_API int to_quant_per_channel_i8(const void* x, int x_dtype, const float* scale, int8_t* q,
                            int64_t outer, int64_t channels, int64_t inner, void* stream);
/* replaces tileops/quant.py:193 dequantize_per_channel (kernel backend/cuda/quant.py:87) */
TO_API int to_dequant_per_channel_i8(const int8_t* q, const float* scale, void* y, int y_dtype,
                              int64_t outer, int64_t channels, int64_t inner, void* stream);

/* ---- dynamic quantisation (tileops/quant_int8.py, tileops/quant_fp8.py) ---------------- */
/* Bytes of workspace the tensor-wide quantisers need (one amax word, padded). */
TO_API size_t to_input_quant_workspace_size(void);
/* replaces tileops/quant_int8.py:29 input_to_int8. Arithmetic in x_dtype exactly as the
 * reference's tensor expression: s = dtype(dtype(1/amax) * 127); q = trunc(clamp(x*s)).
 * Writes q [n] and dq_scale[0] = 1/float(s). */
TO_API int to_input_to_int8(const void* x, int x_dtype, int64_t n, int8_t* q, float* dq_scale,
                     void* workspace, size_t workspace_bytes, void* stream);
/* replaces tileops/quant_fp8.py:52 input_to_float8 (e4m3fn; same arithmetic with 448). */
TO_API int to_input_to_fp8(const void* x, int x_dtype, int64_t n, void* q, float* dq_scale,
                    void* workspace, size_t workspace_bytes, void* stream);
/* No counterpart in the reference. Same result as to_input_to_fp8, for callers that cannot
 * hand the library a device workspace: runtimes that reserve all device memory for their own
 * pool at start-up, so a cudaMalloc during serving fails or fragments it, and foreign-language
 * bindings that only pass tensor pointers and have no device allocator of their own. Its
 * scratch (33 KB per GPU, held until the process exits) is built into the library, which caps
 * n at 134,217,728 elements (TO_EINVAL beyond). It allocates nothing. The first call on each
 * device looks up the scratch address with that device current; make that first call before
 * any stream capture. The looked-up address is kept for the life of the process, so the entry
 * must not be used after cudaDeviceReset (or anything else that destroys the device's primary
 * context) in the same process. All calls share the one scratch buffer: calls that overlap on
 * the GPU (several streams or host threads at once) race and must be serialised. */
TO_API int to_input_to_fp8_noalloc(const void* x, int x_dtype, int64_t n, void* q,
                                   float* dq_scale, void* stream);
/* replaces tileops/quant_int8.py:109 per_token_group_quant_int8 and :54 per_token_quant_int8
 * (group_size = K). x is [n_groups, group_size] contiguous; scales[g] = max(absmax,eps)/127. */
TO_API int to_per_token_group_quant_i8(const void* x, int x_dtype, int64_t n_groups,
                                int64_t group_size, float eps, int8_t* q, float* scales,
                                void* stream);
/* replaces tileops/quant_fp8.py:83 per_token_group_quant_fp8 (via _quantize_groups_fp8 :66).
 * ue8m0 != 0 rounds each scale up to a power of two (quant_fp8.py:48). When cm_rows > 0 the
 * scales are written in the layout the reference's column_major_scales option returns,
 * s_flat.reshape(..., cm_groups, cm_rows).transpose(-2, -1).contiguous() (quant_fp8.py:129-136):
 * within each batch of cm_rows x cm_groups scales, flat scale t goes to row t % cm_rows,
 * column t / cm_rows of a contiguous [cm_rows, cm_groups] array. */
TO_API int to_per_token_group_quant_fp8(const void* x, int x_dtype, int64_t n_groups,
                                 int64_t group_size, float eps, int ue8m0, int64_t cm_rows,
                                 int64_t cm_groups, void* q, float* scales, void* stream);
/* Library extension: per_token_group_quant_fp8 of a 2-D x [rows, cols] (e4m3fn) with the scales
 * in the TMA-aligned column-major layout the reference leaves unimplemented (its
 * tma_aligned_scales option raises, quant_fp8.py:94-98): the scale of row r, group j at
 * scales[j * scales_ld + r], scales_ld >= rows rounded up to a multiple of 4 (16-byte columns).
 * Codes and scale values as per_token_group_quant_fp8. */
TO_API int to_per_token_group_quant_fp8_tma(const void* x, int x_dtype, int64_t rows,
                                            int64_t cols, int64_t group_size, float eps,
                                            int ue8m0, void* q, float* scales, int64_t scales_ld,
                                            void* stream);
/* The same two quantisers with dtype = torch.float8_e4m3fnuz (quant_fp8.py:52, :83 with that
 * dtype): codes in the e4m3fnuz encoding (exponent bias 8, max 240, no negative zero, NaN 0x80).
 * The tensor-wide form scales to finfo(e4m3fnuz).max = 240 and clamps to +-240; the group form
 * uses get_fp8_min_max's +-224 (quant_fp8.py:42-43). Every NaN code is 0x80. No sm_100 GEMM
 * consumes these codes; they are for exchange with e4m3fnuz consumers. */
TO_API int to_input_to_fp8_fnuz(const void* x, int x_dtype, int64_t n, void* q, float* dq_scale,
                                void* workspace, size_t workspace_bytes, void* stream);
TO_API int to_per_token_group_quant_fp8_fnuz(const void* x, int x_dtype, int64_t n_groups,
                                             int64_t group_size, float eps, int ue8m0,
                                             int64_t cm_rows, int64_t cm_groups, void* q,
                                             float* scales, void* stream);

/* ---- block dequantisation ------------------------------------------------------------- */
/* replaces tileops/quant_int8.py:136 block_dequant: y[n,k] = float(q[n,k]) * s[n/bn, k/bk]. */
TO_API int to_block_dequant_i8(const int8_t* q, const float* s, float* y, int64_t n, int64_t k,
                        int64_t block_n, int64_t block_k, void* stream);
/* replaces tileops/quant_fp8.py:143 block_dequant (e4m3fn input). */
TO_API int to_block_dequant_fp8(const void* q, const float* s, float* y, int64_t n, int64_t k,
                         int64_t block_n, int64_t block_k, void* stream);
/* replaces tileops/quant_fp8.py:143 block_dequant for e4m3fnuz input (0x80 reads as NaN). */
TO_API int to_block_dequant_fp8_fnuz(const void* q, const float* s, float* y, int64_t n,
                                     int64_t k, int64_t block_n, int64_t block_k, void* stream);

/* ---- AWQ W4A16 (tileops/quant_awq.py) --------------------------------------------------
 * Packed layout: eight 4-bit values per 32-bit word; logical column 8c+i sits in nibble
 * ORDER[i] of word c with ORDER = (0,4,1,5,2,6,3,7) (quant_awq.py:22). */
/* replaces quant_awq.py:55 pack_awq_int4: in [rows, 8*cols8] (TO_I32 or TO_I64), out [rows, cols8]. */
TO_API int to_awq_pack(const void* unpacked, int in_dtype, int32_t* packed, int64_t rows,
                int64_t cols8, void* stream);
/* replaces quant_awq.py:41 unpack_awq_int4: in [rows, cols8] (TO_I32 or TO_I64, low 32 bits
 * used), out int64 [rows, 8*cols8]. */
TO_API int to_awq_unpack(const void* packed, int in_dtype, int64_t* out, int64_t rows, int64_t cols8,
                  void* stream);
/* replaces quant_awq.py:68 awq_dequantize_triton: out[k,n] = s_dtype((w-z) * s) with
 * qweight [K, N/8], scales [K/G, N] (s_dtype F16/BF16/F32), qzeros [K/G, N/8]. */
TO_API int to_awq_dequant(const int32_t* qweight, const void* scales, int s_dtype,
                   const int32_t* qzeros, void* out, int64_t K, int64_t N, int64_t group_size,
                   void* stream);
/* replaces quant_awq.py:112 awq_gemm_triton: y [M,N] = x [M,K] @ dequant(W), x and y in
 * s_dtype (the facade casts x first, as the reference does), fp32 accumulation. 1-32 tokens
 * run the stream-K decode kernel (1-2 tokens on small layers the streaming GEMV); 33-128 tokens
 * the stream-K tcgen05 kernel on long-K layers of few column tiles, else the register-MMA
 * kernel or the tcgen05 tile GEMM, which takes all larger M. The stream-K kernels need a
 * workspace of to_awq_gemm_workspace_size(M, K, N, group_size) bytes (16-byte aligned; 0 when
 * no kernel for these shapes needs one) for the partial sums of column tiles split over SMs;
 * calls that share a workspace must not overlap on the GPU. */
TO_API size_t to_awq_gemm_workspace_size(int64_t M, int64_t K, int64_t N, int64_t group_size);
TO_API int to_awq_gemm(const void* x, const int32_t* qweight, const void* scales, int s_dtype,
                const int32_t* qzeros, void* y, int64_t M, int64_t K, int64_t N,
                int64_t group_size, void* workspace, size_t workspace_bytes, void* stream);
/* to_awq_gemm with x rows ldx elements apart (ldx >= K, a multiple of 8): a slice of a wider
 * activation, such as the first K columns of a fused qkv output, read in place. Runs where
 * to_awq_gemm would use the decode kernel; TO_EUNSUPPORTED (nothing launched, no error recorded)
 * for other shapes: make x contiguous and call to_awq_gemm. Library extension. */
TO_API int to_awq_gemm_strided(const void* x, int64_t ldx, const int32_t* qweight,
                               const void* scales, int s_dtype, const int32_t* qzeros, void* y,
                               int64_t M, int64_t K, int64_t N, int64_t group_size,
                               void* workspace, size_t workspace_bytes, void* stream);
/* Library extension for N-sharded layers (no reference counterpart; it fuses to_awq_gemm on a
 * rank's column slice with the all-gather that follows it). The group's `world` ranks each
 * hold N = N_full / world output columns of qweight/scales/qzeros; this rank computes its
 * [M, N] slice (1-32 tokens on the decode kernel, more on the tensor-core kernel) and stores
 * it straight into the [M, N * world] output of every rank, y_ranks[r] (host array of device
 * pointers valid on this device: its own buffer and the peers' buffers mapped with
 * to_ipc_open), at columns [rank * N, (rank + 1) * N). Workspace as for to_awq_gemm with the
 * rank's (M, K, N). The stores have completed when the kernel has; the caller orders the
 * peers' reads after every rank's kernel (to_peer_barrier) and must not reuse a buffer a peer
 * may still read. TO_EUNSUPPORTED (nothing launched) for shapes outside both kernels: run
 * to_awq_gemm and an all-gather instead. */
TO_API int to_awq_gemm_gather(const void* x, const int32_t* qweight, const void* scales,
                              int s_dtype, const int32_t* qzeros, void* const* y_ranks,
                              int world, int rank, int64_t M, int64_t K, int64_t N,
                              int64_t group_size, void* workspace, size_t workspace_bytes,
                              void* stream);
/* Library extension: the gate_up linear of an MLP block with its gated activation (no
 * reference counterpart; it fuses to_awq_gemm with tileops/fused.py:97 silu_and_mul or :107
 * gelu_and_mul). qweight/scales/qzeros hold the gate and up columns interleaved in blocks of 8
 * (block 2j = gate columns 8j..8j+7, block 2j + 1 = up columns 8j..8j+7; N = 2F, N % 16 == 0);
 * y[M, F] = act(gate) * up, act TO_ACT_SILU or TO_ACT_GELU_TANH, equal to to_awq_gemm on the
 * un-interleaved weights followed by the activation kernel on its two halves (each GEMM output
 * rounded to the scales' dtype first). The decode kernel (3-32 tokens) and the stream-K kernel
 * apply it in their epilogue on the shapes to_awq_gemm routes to them; other shapes (and 1-2
 * tokens, whose next layer streams faster after a separate activation launch) run the GEMM
 * into the workspace and the activation after it.
 * Bit for bit it is to_awq_gemm on these weights followed by the activation. The workspace is
 * to_awq_gemm_act_workspace_size(M, K, N, group_size) bytes, 16-byte aligned. */
#define TO_ACT_SILU 0
#define TO_ACT_GELU_TANH 1
TO_API size_t to_awq_gemm_act_workspace_size(int64_t M, int64_t K, int64_t N,
                                             int64_t group_size);
TO_API int to_awq_gemm_act(const void* x, const int32_t* qweight, const void* scales, int s_dtype,
                           const int32_t* qzeros, void* y, int64_t M, int64_t K, int64_t N,
                           int64_t group_size, int act, void* workspace, size_t workspace_bytes,
                           void* stream);
/* to_awq_gemm_act on a rank's column slice (N = this rank's interleaved columns) with the
 * all-gather inside the decode kernel, as to_awq_gemm_gather: this rank's [M, N/2] activation
 * slice goes into every rank's [M, N/2 * world] output at columns [rank N/2, (rank + 1) N/2).
 * Workspace as for to_awq_gemm with the rank's (M, K, N). Shapes of the decode and stream-K
 * kernels only; TO_EUNSUPPORTED (nothing launched) otherwise: run to_awq_gemm_act and an
 * all-gather instead. */
TO_API int to_awq_gemm_act_gather(const void* x, const int32_t* qweight, const void* scales,
                                  int s_dtype, const int32_t* qzeros, void* const* y_ranks,
                                  int world, int rank, int64_t M, int64_t K, int64_t N,
                                  int64_t group_size, int act, void* workspace,
                                  size_t workspace_bytes, void* stream);
/* Rank barrier on the GPU (no reference counterpart; the completion step of the gathering
 * GEMMs). Each rank owns a flag array of to_peer_flags_bytes() bytes, zeroed, in memory the
 * others map with to_ipc_open, and an 8-byte counter in its own device memory, zeroed.
 * flag_ranks[r] is rank r's array as seen from this process. The kernel raises this rank's
 * slot in every array to the next count and waits until every rank's slot in its own array
 * has reached it; work queued after it on `stream` sees every rank's earlier stores. Every
 * rank runs the same sequence of barriers; a wait that reaches the library's limit records a
 * timeout in the device error word instead of hanging. With launch overlap on
 * (to_set_launch_overlap) the barrier starts when the previous kernel in the stream completes
 * and lets the next kernel begin streaming its weights during the flag exchange; that
 * kernel's activations and output still wait for the barrier. */
TO_API size_t to_peer_flags_bytes(void);
TO_API int to_peer_barrier(unsigned long long* const* flag_ranks, int world, int rank,
                           unsigned long long* counter, void* stream);

/* ---- W8A8 block-scaled GEMMs --------------------------------------------------------------
 * C[m,n] = sum_kb  (sum_{k in kb} A[m,k]*B[n,k]) * a_s[m,kb] * b_s[n/block_n, kb]
 * A [M,K] row-major, B [N,K] row-major ("NT"), a_s [M, ceil(K/block_k)],
 * b_s [ceil(N/block_n), ceil(K/block_k)], C [M,N] in c_dtype (F32/F16/BF16).
 * bias (optional, c_dtype, [N]) is added after the rounding to c_dtype and rounded again,
 * the order of `output + bias` in apply_w8a8_block_*_linear. */
/* replaces tileops/quant_int8.py:180 w8a8_block_int8_matmul. acc_out (optional, int32
 * [M,N]) receives the exact integer dot products sum_k A[m,k]*B[n,k]. */
TO_API int to_w8a8_i8_gemm(const int8_t* a, const int8_t* b, const float* a_s, const float* b_s,
                    void* c, int c_dtype, const void* bias, int32_t* acc_out, int64_t M,
                    int64_t N, int64_t K, int64_t block_n, int64_t block_k, void* stream);
/* replaces tileops/quant_fp8.py:188 w8a8_block_fp8_matmul (A, B e4m3fn; fp32 accumulation). */
TO_API int to_w8a8_fp8_gemm(const void* a, const void* b, const float* a_s, const float* b_s,
                     void* c, int c_dtype, const void* bias, int64_t M, int64_t N, int64_t K,
                     int64_t block_n, int64_t block_k, void* stream);

/* ---- dense GEMM and GEMV (tileops/blas/gemm.py, tileops/blas/gemv.py) ---------------------
 * replaces tileops/blas/gemm.py:31 gemm (and its mm alias, :71): C [M,N] = A [M,K] @ B [K,N],
 * all row-major, dtype F32, F16 or BF16 for A, B and C, fp32 accumulation, C rounded once. 16-bit
 * operands run on the tcgen05 tiles when K % 8 == 0, N % 64 == 0 and the pointers are 16-byte
 * aligned; other shapes, alignments and fp32 on 64 x 64 SIMT tiles. */
TO_API int to_gemm(const void* a, const void* b, void* c, int dtype, int64_t M, int64_t N,
                   int64_t K, void* stream);
/* replaces tileops/blas/gemv.py:22 gemv (and its mv alias, :60): y [M] = A [M,K] @ x [K], A
 * row-major, dtype F32, F16 or BF16 for A, x and y, fp32 accumulation, y rounded once. Any M, K
 * (K = 0 writes zeros); 16-byte loads when K * sizeof(dtype) % 16 == 0 and A, x are 16-byte
 * aligned. */
TO_API int to_gemv(const void* a, const void* x, void* y, int dtype, int64_t M, int64_t K,
                   void* stream);

/* ---- gated activations (tileops/fused.py) -----------------------------------------------
 * C = act(A) * B element-wise over [rows, cols] views with unit column stride and row strides
 * lda, ldb, ldc (elements; a flat tensor of n elements is rows = 1, cols = n). dtype F32, F16
 * or BF16 for all three. Arithmetic in fp32; act(A) is rounded to dtype, then the product. */
/* replaces tileops/fused.py:97 silu_and_mul (kernel tileops/backend/cuda/fused.py:17):
 * act(x) = x * sigmoid(x). */
TO_API int to_silu_and_mul(const void* a, const void* b, void* c, int dtype, int64_t rows,
                           int64_t cols, int64_t lda, int64_t ldb, int64_t ldc, void* stream);
/* replaces tileops/fused.py:107 gelu_and_mul (kernel tileops/backend/cuda/fused.py:32):
 * act(x) = 0.5 x (1 + tanh(0.7978845608028654 (x + 0.044715 x^3))). */
TO_API int to_gelu_and_mul(const void* a, const void* b, void* c, int dtype, int64_t rows,
                           int64_t cols, int64_t lda, int64_t ldb, int64_t ldc, void* stream);
/* Library extension (no reference counterpart; it fuses the two): the gated activation of
 * to_silu_and_mul / to_gelu_and_mul (act TO_ACT_SILU or TO_ACT_GELU_TANH) quantised per token
 * group as tileops/quant_fp8.py:83 per_token_group_quant_fp8 (q_dtype TO_E4M3; ue8m0 and
 * column_major as there) or tileops/quant_int8.py:109 per_token_group_quant_int8 (TO_I8), without
 * writing the activation: q [rows, cols] codes, scales [rows, cols / group_size] (column_major:
 * the reference's column-major layout). Each activation value is rounded to dtype first, so the
 * result equals the activation kernel followed by the quantiser, bit for bit. */
TO_API int to_act_and_mul_group_quant(const void* a, const void* b, int dtype, int64_t rows,
                                      int64_t cols, int64_t lda, int64_t ldb, int act,
                                      int64_t group_size, float eps, int ue8m0, int column_major,
                                      int q_dtype, void* q, float* scales, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TILEOPS_B200_H_ */
