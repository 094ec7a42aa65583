/*
 * lunara_b200.h -- C ABI of the B200 (sm_100a) kernel library behind Lunara's
 * KernelSpec kinds (GEMM, ATTENTION, SOFTMAX, LAYERNORM, ELEMENTWISE) and the
 * index graph ops (Gather / Slice / Reshape).
 *
 * Conventions shared by every entry point
 *   - Pointers are device pointers owned by the caller (torch owns every
 *     buffer); no entry point allocates device memory.
 *   - Work is enqueued asynchronously on `stream` (a cudaStream_t, NULL = the
 *     legacy default stream) in the caller's current device context (the CUDA
 *     primary context shared with torch).
 *   - The return value is a lunara_status. On failure a message is kept in a
 *     thread-local buffer readable with lunara_last_error_string().
 *   - Strides and leading dimensions are in elements, not bytes.
 *
 * The reference reaches each kernel through a generated Triton launcher
 * (`{name}_launch`); the entry points below replace those launchers one for
 * one. Citations are paths inside the reference project.
 */
#ifndef LUNARA_B200_H
#define LUNARA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum lunara_status {
  LUNARA_OK = 0,
  LUNARA_ERR_INVALID_ARG = 1,  /* bad shape, stride, pointer or enum value */
  LUNARA_ERR_UNSUPPORTED = 2,  /* valid request this build has no kernel for */
  LUNARA_ERR_LAUNCH = 3,       /* CUDA returned an error at launch time */
  LUNARA_ERR_DEVICE = 4        /* a kernel recorded a device-side error */
} lunara_status;

typedef enum lunara_dtype {
  LUNARA_F16 = 0,
  LUNARA_BF16 = 1,
  LUNARA_F32 = 2
} lunara_dtype;

/* Activations of KernelSpec.activation (lunara/codegen/triton_emitter.py:82-89)
 * and of the ELEMENTWISE bodies (triton_emitter.py:452-458), plus the tanh-form
 * GELU of the BERT encoder block. */
typedef enum lunara_activation {
  LUNARA_ACT_NONE = 0,
  LUNARA_ACT_RELU = 1,
  LUNARA_ACT_GELU_ERF = 2,
  LUNARA_ACT_GELU_TANH = 3,
  LUNARA_ACT_SIGMOID = 4,
  LUNARA_ACT_TANH = 5
} lunara_activation;

typedef enum lunara_binary_op {
  LUNARA_BIN_ADD = 0,
  LUNARA_BIN_MUL = 1
} lunara_binary_op;

/* Layout of the GEMM B operand. */
typedef enum lunara_b_layout {
  LUNARA_B_KN = 0, /* B[K,N] row-major, ldb >= N: the reference launcher's B (triton_emitter.py:155-159) */
  LUNARA_B_NK = 1  /* B stored as [N,K] row-major, ldb >= K: a Linear weight (C = A * B^T) */
} lunara_b_layout;

/* Optional tile request for the GEMM (the sm_100a counterpart of TileConfig,
 * triton_emitter.py:44-56). Zero fields mean "choose automatically".
 *   block_n : tcgen05 MMA N: 64, 128, 192 or 256 for 128-row tiles of one
 *             CTA; 128, 192 (B as [N,K] only) or 256 for 256-row tiles of a
 *             CTA pair
 *   stages  : shared-memory pipeline depth (2..8)
 *   num_ctas: persistent grid size (0 = every SM / SM pair)
 *   cta_pair: 1 = single-CTA tiles, 2 = CTA-pair tiles (cta_group::2),
 *             0 = choose from the problem shape */
typedef struct lunara_gemm_config {
  int32_t block_n;
  int32_t stages;
  int32_t num_ctas;
  int32_t cta_pair;
} lunara_gemm_config;

/* GEMM: C[M,N] = act(A[M,K] * B + bias[N]) + residual[M,N]
 * A row-major (lda >= K); B per b_layout; C and residual row-major.
 * bias and residual may be NULL. fp32 accumulation; output rounded once.
 * f16/bf16 run on tcgen05 tensor cores when the TMA alignment rules hold
 * (16-byte aligned bases, leading dimensions multiples of 8); other shapes
 * and f32 run a CUDA-core kernel.
 * Replaces: the GEMM kernel and `{name}_launch(A, B, C, bias=None)`,
 * lunara/codegen/triton_emitter.py:107-175 (bias/act epilogue 145-147,
 * emit_gemm 178-193); the residual add fuses the post-LN block's skip
 * connection (lunara/passes/operator_fusion.cpp:71-94, FuseGemmEpilogue). */
int lunara_gemm(const void* A, const void* B, void* C, const void* bias, const void* residual, int64_t M, int64_t N,
                int64_t K, int64_t lda, int64_t ldb, int64_t ldc, int64_t ldr, int b_layout, int dtype, int activation,
                const lunara_gemm_config* config, void* stream);

/* GEMM with the post-LN residual block's LayerNorm fused into the epilogue:
 *   Y[M,N] = LayerNorm(A[M,K] * B + bias[N] + residual[M,N]) * gamma[N] + beta[N]
 * A, B, bias and residual as for lunara_gemm (no activation); the sum is
 * rounded once to the output type (the value lunara_gemm would store), then
 * normalised with fp32 statistics over exactly N columns (population
 * variance, eps added to it). bias and residual may be NULL; Y may not alias
 * A, B or residual. Each row's N columns are computed by one cluster of
 * G = N / slice CTAs (slice 128, 192 or 256 columns, 2 <= G <= 8) that
 * exchange row statistics through distributed shared memory, so no [M, N]
 * intermediate is written. Requires f16/bf16, the TMA rules of lunara_gemm,
 * and 16-byte aligned Y, residual, bias, gamma and beta with ldy and ldr
 * multiples of 8; otherwise returns LUNARA_ERR_UNSUPPORTED (and launches
 * nothing): run lunara_gemm into a buffer, then lunara_layernorm.
 * config: block_n = slice width request, stages = ring depth, num_ctas = grid
 * (0 = as many clusters as fit); cta_pair is ignored.
 * Replaces: the out_proj + layernorm_attn and ffn2 + layernorm_ffn kernel
 * pairs of the reference's block kernel list (lunara/driver.py:275-283),
 * fused as its FusionOptions.fuse_layernorm ("fuse LayerNorm into preceding
 * matmul", lunara/passes/operator_fusion.h:19-20) and FuseGemmEpilogue
 * (lunara/passes/operator_fusion.cpp:71-94) intend. */
int lunara_gemm_layernorm(const void* A, const void* B, void* Y, const void* bias, const void* residual,
                          const void* gamma, const void* beta, int64_t M, int64_t N, int64_t K, int64_t lda,
                          int64_t ldb, int64_t ldy, int64_t ldr, int b_layout, int dtype, float eps,
                          const lunara_gemm_config* config, void* stream);

/* Scaled-dot-product attention, O = softmax(Q K^T * scale [+ causal mask]) V.
 * Q [B,H,Sq,D], K and V [B,H,Skv,D], O [B,H,Sq,D] given by 4-entry element
 * strides (batch, head, seq, dim); the dim stride must be 1. Causal masking
 * keeps key j for query i when i >= j (top-left aligned).
 * f16/bf16 with D == 64 run on tcgen05; other cases run a CUDA-core kernel.
 * Replaces: the flash-attention kernel and `{name}_launch(Q, K, V, causal)`,
 * lunara/codegen/triton_emitter.py:212-317 (scale 1/sqrt(D) at 302, causal
 * mask at 265-268). */
int lunara_attention(const void* Q, const void* K, const void* V, void* O, int64_t B, int64_t H, int64_t Sq,
                     int64_t Skv, int64_t D, const int64_t* q_strides, const int64_t* k_strides,
                     const int64_t* v_strides, const int64_t* o_strides, float scale, int causal, int dtype,
                     void* stream);

/* LayerNorm over the last dimension: Y = (X - mean) / sqrt(var + eps) * gamma + beta,
 * X and Y [M,N] row-major (leading dimension N), gamma/beta [N] in the same dtype.
 * Statistics in fp32 over exactly N elements (population variance).
 * Replaces: lunara/codegen/triton_emitter.py:382-411. */
int lunara_layernorm(const void* X, const void* gamma, const void* beta, void* Y, int64_t M, int64_t N, float eps,
                     int dtype, void* stream);

/* Row softmax over the last dimension of X [M,N] row-major into Y.
 * Replaces: lunara/codegen/triton_emitter.py:341-364. */
int lunara_softmax(const void* X, void* Y, int64_t M, int64_t N, int dtype, void* stream);

/* Elementwise unary activation over n contiguous elements (in place allowed).
 * Replaces: lunara/codegen/triton_emitter.py:432-458 (`{name}_launch(X)`). */
int lunara_eltwise_unary(int activation, const void* X, void* Y, int64_t n, int dtype, void* stream);

/* Elementwise binary op over n contiguous elements: Out = X op Y. */
int lunara_eltwise_binary(int op, const void* X, const void* Y, void* Out, int64_t n, int dtype, void* stream);

/* Fused bias-add + activation: Y[r,c] = act(X[r,c] + bias[c]) over X [rows,cols]
 * row-major (the ELEMENTWISE kind with KernelSpec.has_bias). */
int lunara_bias_act(const void* X, const void* bias, void* Y, int64_t rows, int64_t cols, int activation, int dtype,
                    void* stream);

/* Gather rows: dst[i,:] = src[index[i],:] for a [src_rows, row_bytes] byte
 * matrix and int64 indices; bit-exact. An out-of-range index records a
 * device error (read with lunara_device_error) and its row is zero-filled.
 * Replaces: the Gather graph op, lunara/frontend/graph_ir.h:23. */
int lunara_gather(const void* src, const int64_t* index, void* dst, int64_t n_index, int64_t src_rows,
                  int64_t row_bytes, void* stream);

/* Strided copy into a contiguous destination: dst[i0..] = src[sum(i_k*src_strides[k])],
 * ndim <= 8, strides in elements, elem_bytes in {1,2,4,8}; bit-exact.
 * Slice is this copy from an offset source pointer with the sliced sizes and
 * stepped strides; Reshape/Transpose of a non-contiguous view is this copy.
 * Replaces: the Slice / Reshape / Transpose graph ops, lunara/frontend/graph_ir.h:23. */
int lunara_copy_strided(const void* src, void* dst, int ndim, const int64_t* sizes, const int64_t* src_strides,
                        int64_t elem_bytes, void* stream);

/* Slice along every dimension of a row-major contiguous source:
 * dst = src[starts[k] : starts[k] + dst_sizes[k]*steps[k] : steps[k]] for each k. */
int lunara_slice(const void* src, void* dst, int ndim, const int64_t* src_sizes, const int64_t* starts,
                 const int64_t* steps, const int64_t* dst_sizes, int64_t elem_bytes, void* stream);

/* Split a fused QKV projection [B,S,3,H,D] into three [B,H,S,D] tensors
 * (the QKV split + head reshape of the encoder block); bit-exact. */
int lunara_qkv_split(const void* qkv, void* q, void* k, void* v, int64_t B, int64_t S, int64_t H, int64_t D,
                     int64_t elem_bytes, void* stream);

/* Message of the last failing call on this host thread ("" if none). */
const char* lunara_last_error_string(void);

/* Synchronizes `stream`, then returns the device error word (0 = none) and
 * clears it when `clear` is non-zero. Codes: 0x1xx GEMM, 0x2xx attention
 * (a bounded wait ran out), 0x301 gather index out of range, 0x4xx the
 * self-tests of lunara_b200_selftest.h.
 * The word is one per device and sticky: a kernel on any stream of the
 * current device sets it (the first failure wins) and it stays set until a
 * caller clears it. Only `stream` is synchronized, so a caller that launched
 * on several streams synchronizes all of them (or the device) first; two
 * threads reading and clearing it at the same time may both see one error. */
int lunara_device_error(void* stream, int clear);

/* Number of SMs of the current device, as the kernels size their grids. */
int lunara_num_sms(void);

/* Library ABI version (major * 10000 + minor * 100 + patch). */
int lunara_version(void);

#ifdef __cplusplus
}
#endif

#endif /* LUNARA_B200_H */
