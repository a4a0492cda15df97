/*
 * b200q — C ABI of the B200 (sm_100a) quantized DiT-linear kernels.
 *
 * Every entry point takes raw device pointers, element strides and sizes, and
 * the cudaStream_t to launch on (passed as void*; NULL = legacy default stream).
 * Nothing here allocates device memory: outputs and scratch words are owned by
 * the caller.  Calls are asynchronous (no device synchronisation) and return
 * B200Q_OK or an error code; b200q_status_string() names it.  Shapes/strides
 * are validated on the host before any launch.
 *
 * Each declaration cites the reference interface it replaces (paths inside
 * luix93/ComfyUI-AppleSilicon-Optimized).
 */
#ifndef B200Q_H_
#define B200Q_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B200Q_API __attribute__((visibility("default")))
#else
#define B200Q_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define B200Q_OK 0
#define B200Q_ERR_INVALID 1     /* bad pointer / shape / stride / dtype argument */
#define B200Q_ERR_UNSUPPORTED 2 /* device is not sm_100 or feature not built     */
#define B200Q_ERR_CUDA 3        /* a CUDA runtime/driver call failed             */
#define B200Q_ERR_WORKSPACE 4   /* caller-provided workspace too small           */

/* element types */
#define B200Q_BF16 0
#define B200Q_F16 1
#define B200Q_F32 2
#define B200Q_I32 3

/* bias types (B200Q_BIAS_NONE = no bias) */
#define B200Q_BIAS_NONE 0
#define B200Q_BIAS_BF16 1
#define B200Q_BIAS_F16 2
#define B200Q_BIAS_F32 3

/* epilogue activations */
#define B200Q_ACT_NONE 0
#define B200Q_ACT_GELU_TANH 1
#define B200Q_ACT_GELU_ERF 2

/* FP8 encodings */
#define B200Q_FP8_E4M3 0
#define B200Q_FP8_E5M2 1

B200Q_API int b200q_version(void);
B200Q_API const char* b200q_status_string(int status);
/* Number of kernels this library has launched in this process. */
B200Q_API uint64_t b200q_launch_count(void);
/* Reads (and optionally clears) the device-side status word of the current
 * device: bit 0 = a pipeline wait timed out, bit 1 = bad argument.  Synchronous. */
B200Q_API int b200q_get_device_status(unsigned int* status, int reset);

/* Per-token INT8 activation quantization, bit-exact to the reference's
 * i8_quant_rowwise (_patches/int8_ext/int8_gemm.mm:2332, kernel body :1346-1381).
 * x [M,K] bf16/f16 (x_dtype B200Q_BF16/B200Q_F16) row stride ldx elements;
 * q [M,K] int8 row stride ldq; scales [M] fp32. */
B200Q_API int b200q_quant_rowwise_i8(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx,
                           int8_t* q, int64_t ldq, float* scales, void* stream);

/* Convrot rotation fused into the per-token INT8 quant: each 256-wide group of a
 * row is multiplied by comfy_kitchen's regular Hadamard (H4 (x) H4 (x) H4 (x) H4
 * / 16), rounded once to x's dtype, then quantized exactly as
 * b200q_quant_rowwise_i8.  Replaces the convrot branch of _quant_cached
 * (_patches/int8_linear_kernel_mps.py:97-140: _build_hadamard + _rotate_activation
 * + i8_quant_rowwise) and the rotation of i8_merge_rot_quant
 * (_patches/int8_ext/int8_gemm.mm:1409-1505).  The fp32 butterfly order follows
 * the latter, so like it the result can differ from the eager bf16 Hadamard
 * matmul by a last-ulp rotation flip on rare ties.  groupsize must be 256 and
 * K a multiple of it, K <= B200Q_CONVROT_MAX_K (B200Q_ERR_UNSUPPORTED otherwise). */
#define B200Q_CONVROT_MAX_K 65536
B200Q_API int b200q_quant_rowwise_i8_convrot(const void* x, int x_dtype, int64_t M, int64_t K,
                                             int64_t ldx, int groupsize, int8_t* q, int64_t ldq,
                                             float* scales, void* stream);

/* Exact int8 x int8 -> int32 NT GEMM, C[M,N] = A[M,K] . W[N,K]^T.
 * Replaces i8_matmul2d_nt (_patches/int8_ext/int8_gemm.mm:1655) and the
 * torch._int_mm seam (_patches/int_mm_mps.py:90). */
B200Q_API int b200q_i8_matmul_nt(const int8_t* a, int64_t lda, const int8_t* w, int64_t ldw, int32_t* c,
                       int64_t ldc, int64_t M, int64_t N, int64_t K, void* stream);

/* INT8 W8A8 GEMM with the reference's fused dequant epilogue:
 *   out[m,n] = T( T(float(C[m,n]) * (col_scale[n] * row_scale[m])) + bias[n] )
 * (T = bf16 or f16, two RNE roundings; bias is in T or NULL).  col_scale_numel is
 * N (channelwise) or 1 (tensorwise weight scale).  act != B200Q_ACT_NONE applies
 * the activation to that result and rounds once more: T(act(out)).  Replaces i8_matmul2d_nt_fused
 * (int8_gemm.mm:1709) and i8_matmul2d_nt_fused_cs (int8_gemm.mm:1823). */
B200Q_API int b200q_i8_matmul_nt_dequant(const int8_t* a, int64_t lda, const int8_t* w, int64_t ldw,
                               const float* row_scale, const float* col_scale,
                               int64_t col_scale_numel, const void* bias, int act, void* out,
                               int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t K,
                               void* stream);

/* Per-token quant + INT8 GEMM + dequant epilogue in one call (the comfy
 * int8_tensorwise Linear: _patches/int8_linear_kernel_mps.py:218 _int8_linear_kernel).
 * x [M,K] bf16/f16; q_scratch [M,K] int8 and scale_scratch [M] fp32 receive the
 * quantized activation (they stay valid after the call, as the reference's
 * activation cache expects). */
B200Q_API int b200q_i8_linear(const void* x, int x_dtype, int64_t ldx, const int8_t* w, int64_t ldw,
                    const float* col_scale, int64_t col_scale_numel, const void* bias, int act,
                    void* out, int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t K,
                    int8_t* q_scratch, float* scale_scratch, void* stream);

/* FP8 (e4m3 x e4m3) scaled GEMM, out = act(((A.W^T) * scale_a * scale_b * scale_result)
 * + bias) in fp32, one rounding to out_dtype (bf16/f16/f32).  scale_a numel 1 or M,
 * scale_b numel 1 or N, any scale may be NULL.  W is [N,K] row-major, i.e. the
 * column-major [K,N] `other` operand of torch._scaled_mm consumed in place.
 * Replaces _mps_scaled_mm / _fast_route (_patches/scaled_mm_fp8.py:123-207) and
 * fp8fp8_matmul2d_nt (_patches/fp8_ext/fp8_matmul2d.mm:229). */
B200Q_API int b200q_fp8_scaled_mm(const uint8_t* a, int64_t lda, const uint8_t* w, int64_t ldw,
                        const float* scale_a, int64_t scale_a_numel, const float* scale_b,
                        int64_t scale_b_numel, const float* scale_result, const void* bias,
                        int bias_dtype, int act, void* out, int out_dtype, int64_t ldo,
                        int64_t M, int64_t N, int64_t K, void* stream);

/* b200q_fp8_scaled_mm (bf16/f16 output) that also writes max |out| over the
 * stored outputs to *amax_bits (float bits, overwritten), so that the next
 * layer's per-tensor FP8 quant of this output (b200q_fp8_quant_from_amax) skips
 * its amax pass: on the CTA-pair route the epilogue takes the max while
 * storing.  No reference counterpart (the reference quantizes FP8 activations
 * upstream of torch._scaled_mm, _patches/scaled_mm_fp8.py:149). */
B200Q_API int b200q_fp8_scaled_mm_amax(const uint8_t* a, int64_t lda, const uint8_t* w,
                                       int64_t ldw, const float* scale_a, int64_t scale_a_numel,
                                       const float* scale_b, int64_t scale_b_numel,
                                       const float* scale_result, const void* bias,
                                       int bias_dtype, int act, void* out, int out_dtype,
                                       int64_t ldo, int64_t M, int64_t N, int64_t K,
                                       unsigned int* amax_bits, void* stream);

/* Per-tensor e4m3 quant of x given its amax (float bits, e.g. from
 * b200q_fp8_scaled_mm_amax): the same scale and codes as
 * b200q_fp8_quant_tensorwise without its amax pass. */
B200Q_API int b200q_fp8_quant_from_amax(const void* x, int x_dtype, int64_t M, int64_t K,
                                        int64_t ldx, const unsigned int* amax_bits, uint8_t* q,
                                        int64_t ldq, float* scale, void* stream);

/* Column-parallel (N-split) b200q_fp8_scaled_mm with its all-gather fused in:
 * this rank holds the weight rows of output columns [c0, c0 + N) and computes
 * them for all M tokens; `out` and each of the n_peer_outs (<= 7) peer_outs[i]
 * point at column c0 of a full-width [M, N_total] output with row stride ldo
 * (this rank's copy and the other ranks' copies, the latter mapped from them
 * with b200q_ipc_import).  Each output block is written to every copy (on the
 * CTA-pair route straight from the epilogue's shared-memory staging block over
 * NVLink; otherwise the GEMM writes `out` and one 2-D copy per peer follows on
 * the stream).  bf16/f16 output only.  The peers' copies are complete once the
 * peers' calls have finished: synchronise the ranks (e.g. a one-element NCCL
 * all-reduce on this stream) before reading columns other ranks own.  The
 * reference is single-GPU; this serves the optional N-split of the Wan-shaped
 * block (its token rows, _patches/int8_linear_kernel_mps.py:75-94, are the
 * default split, which needs no communication). */
B200Q_API int b200q_fp8_scaled_mm_allgather(const uint8_t* a, int64_t lda, const uint8_t* w,
                                            int64_t ldw, const float* scale_a, int64_t scale_a_numel,
                                            const float* scale_b, int64_t scale_b_numel,
                                            const float* scale_result, const void* bias,
                                            int bias_dtype, int act, void* out,
                                            void* const* peer_outs, int n_peer_outs, int out_dtype,
                                            int64_t ldo, int64_t M, int64_t N, int64_t K,
                                            void* stream);

/* Peer mappings for b200q_fp8_scaled_mm_allgather (no reference counterpart).
 * export: the 64-byte CUDA IPC handle of the device allocation holding dev_ptr
 * and dev_ptr's byte offset in it.  import (in another process): maps that
 * allocation (peer access enabled lazily) and returns the pointer at the offset
 * plus the mapping's base for b200q_ipc_close. */
B200Q_API int b200q_ipc_export(const void* dev_ptr, void* handle_out, uint64_t* offset_out);
B200Q_API int b200q_ipc_import(const void* handle, uint64_t offset, void** dev_ptr_out,
                               void** base_out);
B200Q_API int b200q_ipc_close(void* base);

/* Per-tensor FP8 activation quantization: amax = max|x|, scale = max(amax/448, 1e-30),
 * q = e4m3 saturating RNE of x/scale.  amax_scratch: one caller-owned device word
 * (overwritten).  No reference counterpart (comfy's quant ops produce the e4m3
 * activation upstream of torch._scaled_mm, _patches/scaled_mm_fp8.py:149). */
B200Q_API int b200q_fp8_quant_tensorwise(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx,
                               uint8_t* q, int64_t ldq, float* scale, unsigned int* amax_scratch,
                               void* stream);

/* INT8 GEMM + dequant epilogue (as b200q_i8_matmul_nt_dequant, no activation)
 * storing straight into attention layout: column kind*H*D + h*D + d of token
 * row m = b*S + s (S = M / batch) goes to {q,k,v}_out[((b*H + h)*S + s)*D + d]
 * (kind 0/1/2), i.e. three [batch, H, S, D] tensors instead of one [M, 3*H*D].
 * N must be 3*heads*head_dim, head_dim % 32 == 0, outputs 16-byte aligned.
 * Replaces i8_matmul2d_nt_fused_cs_qkv (_patches/int8_ext/int8_gemm.mm:2028,
 * epilogue :445-474), whose layout is the batch = 1 case. */
B200Q_API int b200q_i8_matmul_nt_dequant_qkv(const int8_t* a, int64_t lda, const int8_t* w,
                                             int64_t ldw, const float* row_scale,
                                             const float* col_scale, int64_t col_scale_numel,
                                             const void* bias, void* q_out, void* k_out,
                                             void* v_out, int out_dtype, int64_t heads,
                                             int64_t head_dim, int64_t batch, int64_t M,
                                             int64_t N, int64_t K, void* stream);

/* b200q_i8_matmul_nt_dequant_qkv (bf16 out, head_dim 128) with Q and K
 * RMS-normalized and rotated in the epilogue before the store, as
 * b200q_rms_rope_partial would do afterwards: y = bf16((x * rsqrt(sum(x^2)/128 +
 * eps)) * w) with q_weight / k_weight [128] fp32, then split-half RoPE on the
 * first 2*rot_half dims with freqs [batch*seq, rot_half, 2, 2] bf16.  rot_half % 8
 * == 0, 2*rot_half <= 128 (0: norm only); V is stored unnormalized.  Needs the
 * TMA path (K % 16 == 0, lda/ldw % 16 == 0, 16-byte aligned a, w, outputs,
 * freqs and weights).  Replaces i8_matmul2d_nt_fused_cs_qkv_rms_rope
 * (_patches/int8_ext/int8_gemm.mm:2111, epilogue :672-862), batch 1 there. */
B200Q_API int b200q_i8_matmul_nt_dequant_qkv_rms_rope(
    const int8_t* a, int64_t lda, const int8_t* w, int64_t ldw, const float* row_scale,
    const float* col_scale, int64_t col_scale_numel, const void* bias, void* q_out, void* k_out,
    void* v_out, int64_t heads, int64_t batch, const void* freqs, int64_t rot_half,
    const float* q_weight, const float* k_weight, float eps, int64_t M, int64_t N, int64_t K,
    void* stream);

/* In place on bf16 q, k [batch, heads, seq, head_dim] (contiguous): per row
 * RMSNorm y = bf16((x * rsqrt(sum(x^2)/D + eps)) * w) with fp32 weights
 * q_weight/k_weight [D], then split-half RoPE on the first 2*rot_half dims with
 * the bf16 rotation-matrix table freqs [batch*seq, rot_half, 2, 2] (diagonal
 * product rounded, then the off-diagonal product added with one rounding).
 * head_dim % 32 == 0, <= 256; rot_half = 0 skips RoPE.  q, k 8-byte aligned,
 * weights 16-byte aligned, freqs 16-byte aligned when rot_half % 4 == 0.  Replaces
 * rms_rope_attention_partial (_patches/dit_ext/dit_kernels.mm:825-874, 1677). */
B200Q_API int b200q_rms_rope_partial(void* q, void* k, const void* freqs, const float* q_weight,
                                     const float* k_weight, int64_t batch, int64_t heads,
                                     int64_t seq, int64_t head_dim, int64_t rot_half, float eps,
                                     void* stream);

/* ---- SwiGLU between FC1 and FC2 (bf16 only, as the reference).
 * A "wide" tensor is [M, 2F] bf16 with gate = columns [0, F), up = [F, 2F);
 * act = bf16(bf16(silu(gate)) * up), silu(a) = a / (1 + exp(-a)) in fp32 with
 * exp correctly rounded.  The convrot variants rotate every 256-wide group of
 * act (radix-4 Hadamard butterflies in fp32, then * 2^-4 and one bf16 rounding),
 * exactly as b200q_quant_rowwise_i8_convrot does for a plain activation. */
#define B200Q_SWIGLU_MAX_F 65536

/* act [M, F] of a wide tensor (row stride ldx >= 2F).  Replaces silu_mul_split
 * (_patches/dit_ext/dit_kernels.mm:724-737) behind _swiglu_activation
 * (_patches/int8_linear_kernel_mps.py:693-705). */
B200Q_API int b200q_silu_mul_split(const void* x, int64_t ldx, int64_t M, int64_t F, void* out,
                                   int64_t ldo, void* stream);

/* Rotated act [M, F] (F % 256 == 0).  Replaces i8_swiglu_rot
 * (_patches/int8_ext/int8_gemm.mm:1521-1555, host :2593-2624). */
B200Q_API int b200q_i8_swiglu_rot(const void* x, int64_t ldx, int64_t M, int64_t F, void* out,
                                  int64_t ldo, void* stream);

/* Per-token INT8 codes q [M, F] + scales [M] of act (rotate = 1: of the rotated
 * act) in one pass, the rotated act never written.  Replaces the FC2 pre-pass
 * i8_swiglu_rot -> i8_quant_rowwise of _try_int8_swiglu_forward
 * (_patches/int8_linear_kernel_mps.py:757-766) and, with rotate = 0,
 * _swiglu_activation -> rowwise quant (:771-773). */
B200Q_API int b200q_i8_swiglu_quant(const void* x, int64_t ldx, int64_t M, int64_t F, int rotate,
                                    int8_t* q, int64_t ldq, float* scales, void* stream);

/* FC1 of the bridge: INT8 GEMM of a [M, K] with w [N2 = 2F, K] (rows [gate; up],
 * the checkpoint's layout) and the channelwise two-rounding dequant (+ bf16 bias
 * [2F]) of b200q_i8_matmul_nt_dequant, followed in the same epilogue by
 * act = swiglu(gate, up) -> act_out [M, F] bf16.  The [M, 2F] output is never
 * formed.  Needs the TMA path (K % 16 == 0, lda/ldw % 16 == 0, 16-byte aligned
 * a and w; B200Q_ERR_INVALID otherwise).  Replaces i8_matmul2d_nt_fused_cs ->
 * silu_mul_split (_patches/int8_linear_kernel_mps.py:643-654). */
B200Q_API int b200q_i8_matmul_nt_dequant_swiglu(const int8_t* a, int64_t lda, const int8_t* w,
                                                int64_t ldw, const float* row_scale,
                                                const float* col_scale, int64_t col_scale_numel,
                                                const void* bias, void* act_out, int64_t ldo,
                                                int64_t M, int64_t N2, int64_t K, void* stream);

/* The FC1 -> SwiGLU (-> convrot) -> FC2-quant bridge: per block of tile_rows
 * rows (0 = all), b200q_i8_matmul_nt_dequant_swiglu into act_scratch
 * ([tile_rows or M, F] bf16, caller-owned) then the per-token quant of act
 * (rotate = 1: convrot, F % 256 == 0 and F <= B200Q_CONVROT_MAX_K) into
 * q [M, F] (row stride ldq) and scales [M].  Replaces i8_mlp_bridge_prequant
 * (_patches/int8_ext/int8_gemm.mm:2377-2537), which is rotate = 1. */
B200Q_API int b200q_i8_mlp_bridge_prequant(const int8_t* a, int64_t lda, const int8_t* w1,
                                           int64_t ldw, const float* row_scale,
                                           const float* col_scale, int64_t col_scale_numel,
                                           const void* bias, int64_t M, int64_t N2, int64_t K,
                                           int rotate, int64_t tile_rows, void* act_scratch,
                                           int8_t* q, int64_t ldq, float* scales, void* stream);

/* Fused quant prologue: the activation quantization runs inside the GEMM launch
 * (idle warps quantize 128-row bands while the tensor cores work; the TMA
 * producer waits for a band's rows before loading them), so there is no separate
 * quant kernel and no kernel boundary between quant and GEMM.
 *
 * `sync` is a caller-owned device buffer of at least b200q_prologue_sync_bytes(M)
 * bytes, 16-byte aligned, ALL ZERO before the first call.  Every call leaves it
 * all zero again when its kernels finish, so calls ordered on one stream (and
 * CUDA-graph replays) can reuse it; calls that may overlap on the GPU need
 * separate buffers. */
B200Q_API size_t b200q_prologue_sync_bytes(int64_t M);

/* b200q_i8_linear with the per-token quant fused into the GEMM launch (one
 * launch).  Same arguments and results as b200q_i8_linear (q_scratch and
 * scale_scratch receive the codes and scales), plus the sync buffer.  Replaces
 * _int8_linear_kernel (_patches/int8_linear_kernel_mps.py:218-263): the
 * reference's i8_quant_rowwise (_patches/int8_ext/int8_gemm.mm:2332) followed by
 * i8_matmul2d_nt_fused_cs (:1823).  Shapes the TMA path cannot take (K % 16 != 0,
 * unaligned weight) fall back to the two-launch route inside the call. */
B200Q_API int b200q_i8_linear_fused(const void* x, int x_dtype, int64_t ldx, const int8_t* w,
                                    int64_t ldw, const float* col_scale, int64_t col_scale_numel,
                                    const void* bias, int act, void* out, int out_dtype,
                                    int64_t ldo, int64_t M, int64_t N, int64_t K,
                                    int8_t* q_scratch, float* scale_scratch, unsigned int* sync,
                                    size_t sync_bytes, void* stream);

/* FP8 W8A8 linear from a bf16/f16 activation: per-tensor e4m3 quant of x
 * (b200q_fp8_quant_tensorwise semantics) fused into b200q_fp8_scaled_mm with
 * scale_a = the activation scale.  Two launches: an amax reduction over x, then
 * the GEMM whose prologue quantizes.  q_scratch [M,K] receives the codes and
 * scale_out (one fp32) the activation scale.  Replaces the activation-quant +
 * torch._scaled_mm pair that reaches _mps_scaled_mm (_patches/scaled_mm_fp8.py:149). */
B200Q_API int b200q_fp8_linear_fused(const void* x, int x_dtype, int64_t ldx, const uint8_t* w,
                                     int64_t ldw, const float* scale_b, int64_t scale_b_numel,
                                     const float* scale_result, const void* bias, int bias_dtype,
                                     int act, void* out, int out_dtype, int64_t ldo, int64_t M,
                                     int64_t N, int64_t K, uint8_t* q_scratch, float* scale_out,
                                     unsigned int* sync, size_t sync_bytes, void* stream);

/* Bytes of device workspace b200q_w8a16_linear needs for this shape (0 = none). */
B200Q_API size_t b200q_w8a16_workspace_size(int64_t M, int64_t N, int64_t K);

/* FP8 weight-only linear: out = act((X . decode(W)^T) * w_scale + bias), fp32
 * accumulation, one rounding to out_dtype.  X [M,K] bf16/f16, W [N,K] e4m3 bytes,
 * w_scale one fp32 or NULL, bias bf16/f16/f32 or NULL.  Replaces w8a16_bias_bf16 /
 * w8a16_f32 (_patches/fp8s_ext/w8a16_gemm.mm:286-314), fp8_matmul2d_nt
 * (_patches/fp8_ext/fp8_matmul2d.mm:312) and _w8a16_forward
 * (_patches/linear_fp8_w8a16.py:151). */
B200Q_API int b200q_w8a16_linear(const void* x, int x_dtype, int64_t ldx, const uint8_t* w, int64_t ldw,
                       const float* w_scale, const void* bias, int bias_dtype, int act,
                       void* out, int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t K,
                       void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free variant of b200q_w8a16_linear (same arguments minus the
 * workspace).  No counterpart in the reference: it exists for callers that
 * cannot allocate device memory themselves -- a host that reaches this library
 * only through the C ABI with buffers it registered up front (no device
 * allocator of its own), or a runtime with a fixed device-memory budget in which
 * every allocation must be planned before the model runs.  Its scratch (the
 * small-M planes route's activation planes, or the split-K partials and tile
 * counters of the weight-stationary kernel) lives in a static device array of
 * B200Q_NOALLOC_SCRATCH_BYTES that every GPU loading this library holds until
 * exit.  The route is the one b200q_w8a16_linear would take without the
 * decoded-weight route; when that route's scratch exceeds the array the call
 * returns B200Q_ERR_TOO_LARGE and launches nothing (invalid arguments give
 * B200Q_ERR_INVALID first).  The first call on each device (and again after a
 * device reset re-creates its context) looks up the array's device address;
 * make that first call before any stream capture.  All calls share the array:
 * calls whose kernels overlap on the GPU (other streams, other threads) race on
 * it and must be serialised by the caller.  Never calls cudaMalloc/cudaFree. */
#define B200Q_NOALLOC_SCRATCH_BYTES (16u << 20)
#define B200Q_ERR_TOO_LARGE 5   /* needs more scratch than the static buffer */
B200Q_API int b200q_w8a16_linear_noalloc(const void* x, int x_dtype, int64_t ldx, const uint8_t* w,
                                         int64_t ldw, const float* w_scale, const void* bias,
                                         int bias_dtype, int act, void* out, int out_dtype,
                                         int64_t ldo, int64_t M, int64_t N, int64_t K,
                                         void* stream);

/* Exact FP8 -> bf16/f16/f32 decode of n contiguous codes.  Replaces decode_fp8
 * (_patches/_common.py:249-273). */
B200Q_API int b200q_fp8_decode(const uint8_t* src, int64_t n, int fp8_kind, void* dst, int out_dtype,
                     void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200Q_H_ */
