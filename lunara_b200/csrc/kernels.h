// Internal launcher prototypes shared between the kernel translation units and
// the C-ABI layer (abi.cu). Launchers validate nothing beyond what their
// kernel needs; argument checking happens in abi.cu.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <utility>

namespace lunara {

int device_num_sms();

// Launch with programmatic stream serialization: the kernel may be scheduled
// before its predecessor in the stream has finished and waits for it in
// pdl_wait() (common.cuh). Used for every kernel of the hot path.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// As launch_pdl, for a kernel launched in clusters of `cluster` CTAs along x.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, unsigned cluster, size_t smem,
                               cudaStream_t s, Args&&... args) {
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Device address of the library's error word on the current device (cached
// per device); nullptr when the symbol cannot be resolved.
unsigned int* device_error_word();

cudaError_t launch_layernorm(const void* X, const void* gamma, const void* beta, void* Y, int64_t M, int64_t N,
                             float eps, int dtype, cudaStream_t stream);

cudaError_t launch_softmax(const void* X, void* Y, int64_t M, int64_t N, int dtype, cudaStream_t stream);

cudaError_t launch_eltwise_unary(int act, const void* X, void* Y, int64_t n, int dtype, cudaStream_t stream);
cudaError_t launch_eltwise_binary(int op, const void* X, const void* Yin, void* Out, int64_t n, int dtype,
                                  cudaStream_t stream);
cudaError_t launch_bias_act(const void* X, const void* bias, void* Y, int64_t rows, int64_t cols, int act, int dtype,
                            cudaStream_t stream);

cudaError_t launch_gather(const void* src, const int64_t* index, void* dst, int64_t n_index, int64_t src_rows,
                          int64_t row_bytes, cudaStream_t stream);
// Single-launch QKV split for 16-byte-aligned head rows; sets *handled to
// false (and launches nothing) when the shape or alignment needs the general
// strided copy instead.
cudaError_t launch_qkv_split(const void* qkv, void* q, void* k, void* v, int64_t B, int64_t S, int64_t H,
                             int64_t D, int64_t elem_bytes, cudaStream_t stream, bool* handled);
cudaError_t launch_copy_strided(const void* src, void* dst, int ndim, const int64_t* sizes,
                                const int64_t* src_strides, int64_t elem_bytes, cudaStream_t stream);

struct GemmArgs {
  const void* A;
  const void* B;
  void* C;
  const void* bias;
  const void* residual;
  int64_t M, N, K;
  int64_t lda, ldb, ldc, ldr;
  int b_layout;  // lunara_b_layout
  int dtype;     // lunara_dtype
  int act;       // lunara_activation
  int block_n;   // 0 = auto
  int stages;    // 0 = auto
  int num_ctas;  // 0 = auto
  int cta_pair;  // 0 = auto, 1 = single-CTA tiles, 2 = CTA-pair (cta_group::2) tiles
};

// True when the tcgen05/TMA path accepts the shapes, strides and pointers.
bool gemm_tc_supported(const GemmArgs& g);
cudaError_t launch_gemm_tcgen05(const GemmArgs& g, cudaStream_t stream);

// GEMM + bias + residual + LayerNorm over the N columns of each row, N split
// over a cluster of 2..8 CTAs (N = G * block_n, block_n 128 / 192 / 256).
// gemm_ln_block_n returns the slice width for N (0 when none fits).
int gemm_ln_block_n(int64_t N, int requested);
bool gemm_ln_supported(const GemmArgs& g, const void* gamma, const void* beta);
cudaError_t launch_gemm_layernorm(const GemmArgs& g, const void* gamma, const void* beta, float eps,
                                  cudaStream_t stream);
cudaError_t launch_gemm_simt(const GemmArgs& g, cudaStream_t stream);

struct AttnArgs {
  const void* Q;
  const void* K;
  const void* V;
  void* O;
  int64_t B, H, Sq, Skv, D;
  int64_t qs[4], ks[4], vs[4], os[4];  // element strides (batch, head, seq, dim)
  float scale;
  int causal;
  int dtype;
};

bool attention_tc_supported(const AttnArgs& a);
// Sets *handled to false (and launches nothing) when the driver refuses one of
// the tensor maps; the caller then runs the CUDA-core kernel.
cudaError_t launch_attention_tcgen05(const AttnArgs& a, cudaStream_t stream, bool* handled);
cudaError_t launch_attention_simt(const AttnArgs& a, cudaStream_t stream);

// Resolves cuTensorMapEncodeTiled through the runtime's driver entry point
// (the library does not link libcuda directly). Returns nullptr on failure.
void* tensor_map_encoder();

}  // namespace lunara
