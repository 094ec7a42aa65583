// C ABI of the kernel library (declared in include/lunara_b200.h).
//
// Each entry point validates its arguments on the host, picks the kernel
// (tcgen05 path when its layout rules hold, CUDA-core path otherwise; there is
// no CPU path), enqueues it on the caller's stream and returns a status code.
// Failures keep a message in a thread-local buffer. The runtime API is used
// throughout, so every launch runs in the primary context shared with torch.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "../../include/lunara_b200.h"
#include "kernels.h"

namespace lunara {

__device__ unsigned int g_device_error_word = 0;

namespace {

thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int ok() {
  g_last_error[0] = '\0';
  return LUNARA_OK;
}

int from_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return ok();
  return fail(LUNARA_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
}

bool valid_dtype(int d) { return d == LUNARA_F16 || d == LUNARA_BF16 || d == LUNARA_F32; }
bool valid_act(int a) { return a >= LUNARA_ACT_NONE && a <= LUNARA_ACT_TANH; }

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned int* g_err_ptr[kMaxDevices] = {};
int g_sms[kMaxDevices] = {};
void* g_encoder = nullptr;
bool g_encoder_tried = false;

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

}  // namespace

int device_num_sms() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 148;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_sms[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sms[dev] = n;
  }
  return g_sms[dev];
}

unsigned int* device_error_word() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_err_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error_word) != cudaSuccess) return nullptr;
    g_err_ptr[dev] = static_cast<unsigned int*>(p);
  }
  return g_err_ptr[dev];
}

void* tensor_map_encoder() {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_encoder_tried) {
    g_encoder_tried = true;
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encoder = fn;
  }
  return g_encoder;
}

}  // namespace lunara

using namespace lunara;

extern "C" {

int lunara_version(void) { return 10000; }

const char* lunara_last_error_string(void) { return g_last_error; }

int lunara_num_sms(void) { return device_num_sms(); }

int lunara_device_error(void* stream, int clear) {
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return -fail(LUNARA_ERR_LAUNCH, "lunara_device_error: %s", cudaGetErrorString(e));
  unsigned int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_device_error_word, sizeof(v));
  if (e != cudaSuccess) return -fail(LUNARA_ERR_LAUNCH, "lunara_device_error: %s", cudaGetErrorString(e));
  if (clear && v != 0) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_device_error_word, &zero, sizeof(zero));
    if (e != cudaSuccess) return -fail(LUNARA_ERR_LAUNCH, "lunara_device_error: %s", cudaGetErrorString(e));
  }
  return static_cast<int>(v);
}

int lunara_gemm(const void* A, const void* B, void* C, const void* bias, const void* residual, int64_t M, int64_t N,
                int64_t K, int64_t lda, int64_t ldb, int64_t ldc, int64_t ldr, int b_layout, int dtype, int activation,
                const lunara_gemm_config* config, void* stream) {
  if (!valid_dtype(dtype)) return fail(LUNARA_ERR_INVALID_ARG, "lunara_gemm: bad dtype %d", dtype);
  if (!valid_act(activation)) return fail(LUNARA_ERR_INVALID_ARG, "lunara_gemm: bad activation %d", activation);
  if (b_layout != LUNARA_B_KN && b_layout != LUNARA_B_NK)
    return fail(LUNARA_ERR_INVALID_ARG, "lunara_gemm: bad b_layout %d", b_layout);
  if (M < 0 || N < 0 || K < 0) return fail(LUNARA_ERR_INVALID_ARG, "lunara_gemm: negative shape");
  if (M >= (int64_t{1} << 31) || N >= (int64_t{1} << 31))
    return fail(LUNARA_ERR_UNSUPPORTED, "lunara_gemm: M and N must be below 2^31");
  if (M == 0 || N == 0) return ok();
  if (A == nullptr && K > 0) return fail(LUNARA_ERR_INVALID_ARG, "lunara_gemm: A is NULL");
  if (B == nullptr && K > 0) return fail(LUNARA_ERR_INVALID_ARG, "lunara_gemm: B is NULL");
  if (C == nullptr) return fail(LUNARA_ERR_INVALID_ARG, "lunara_gemm: C is NULL");
  if (lda < K || ldc < N) return fail(LUNARA_ERR_INVALID_ARG, "lunara_gemm: lda < K or ldc < N");
  if (b_layout == LUNARA_B_KN ? ldb < N : ldb < K)
    return fail(LUNARA_ERR_INVALID_ARG, "lunara_gemm: ldb too small for the B layout");
  if (residual != nullptr && ldr < N) return fail(LUNARA_ERR_INVALID_ARG, "lunara_gemm: ldr < N");
  GemmArgs g{};
  g.A = A;
  g.B = B;
  g.C = C;
  g.bias = bias;
  g.residual = residual;
  g.M = M;
  g.N = N;
  g.K = K;
  g.lda = lda;
  g.ldb = ldb;
  g.ldc = ldc;
  g.ldr = ldr;
  g.b_layout = b_layout;
  g.dtype = dtype;
  g.act = activation;
  if (config != nullptr) {
    g.block_n = config->block_n;
    g.stages = config->stages;
    g.num_ctas = config->num_ctas;
    g.cta_pair = config->cta_pair;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (gemm_tc_supported(g)) return from_cuda(launch_gemm_tcgen05(g, s), "lunara_gemm(tcgen05)");
  return from_cuda(launch_gemm_simt(g, s), "lunara_gemm(simt)");
}

int lunara_gemm_layernorm(const void* A, const void* B, void* Y, const void* bias, const void* residual,
                          const void* gamma, const void* beta, int64_t M, int64_t N, int64_t K, int64_t lda,
                          int64_t ldb, int64_t ldy, int64_t ldr, int b_layout, int dtype, float eps,
                          const lunara_gemm_config* config, void* stream) {
  if (!valid_dtype(dtype)) return fail(LUNARA_ERR_INVALID_ARG, "lunara_gemm_layernorm: bad dtype %d", dtype);
  if (b_layout != LUNARA_B_KN && b_layout != LUNARA_B_NK)
    return fail(LUNARA_ERR_INVALID_ARG, "lunara_gemm_layernorm: bad b_layout %d", b_layout);
  if (M < 0 || N <= 0 || K < 0) return fail(LUNARA_ERR_INVALID_ARG, "lunara_gemm_layernorm: bad shape");
  if (!(eps >= 0.0f)) return fail(LUNARA_ERR_INVALID_ARG, "lunara_gemm_layernorm: eps must be >= 0");
  if (M == 0) return ok();
  if (!A || !B || !Y || !gamma || !beta) return fail(LUNARA_ERR_INVALID_ARG, "lunara_gemm_layernorm: NULL tensor");
  if (lda < K || ldy < N) return fail(LUNARA_ERR_INVALID_ARG, "lunara_gemm_layernorm: lda < K or ldy < N");
  if (b_layout == LUNARA_B_KN ? ldb < N : ldb < K)
    return fail(LUNARA_ERR_INVALID_ARG, "lunara_gemm_layernorm: ldb too small for the B layout");
  if (residual != nullptr && ldr < N) return fail(LUNARA_ERR_INVALID_ARG, "lunara_gemm_layernorm: ldr < N");
  if (M >= (int64_t{1} << 31) || K < 1)
    return fail(LUNARA_ERR_UNSUPPORTED, "lunara_gemm_layernorm: M must be below 2^31 and K positive");
  GemmArgs g{};
  g.A = A;
  g.B = B;
  g.C = Y;
  g.bias = bias;
  g.residual = residual;
  g.M = M;
  g.N = N;
  g.K = K;
  g.lda = lda;
  g.ldb = ldb;
  g.ldc = ldy;
  g.ldr = ldr;
  g.b_layout = b_layout;
  g.dtype = dtype;
  g.act = LUNARA_ACT_NONE;
  if (config != nullptr) {
    g.block_n = config->block_n;
    g.stages = config->stages;
    g.num_ctas = config->num_ctas;
  }
  if (!gemm_ln_supported(g, gamma, beta))
    return fail(LUNARA_ERR_UNSUPPORTED,
                "lunara_gemm_layernorm: needs f16/bf16, N = G x {128,192,256} with 2 <= G <= 8, and 16-byte "
                "aligned operands (got N=%lld); run lunara_gemm then lunara_layernorm",
                (long long)N);
  return from_cuda(launch_gemm_layernorm(g, gamma, beta, eps, static_cast<cudaStream_t>(stream)),
                   "lunara_gemm_layernorm");
}

int lunara_attention(const void* Q, const void* K, const void* V, void* O, int64_t B, int64_t H, int64_t Sq,
                     int64_t Skv, int64_t D, const int64_t* q_strides, const int64_t* k_strides,
                     const int64_t* v_strides, const int64_t* o_strides, float scale, int causal, int dtype,
                     void* stream) {
  if (!valid_dtype(dtype)) return fail(LUNARA_ERR_INVALID_ARG, "lunara_attention: bad dtype %d", dtype);
  if (B < 0 || H < 0 || Sq < 0 || Skv < 0 || D < 0)
    return fail(LUNARA_ERR_INVALID_ARG, "lunara_attention: negative shape");
  if (B == 0 || H == 0 || Sq == 0) return ok();
  if (Skv == 0 || D == 0) return fail(LUNARA_ERR_INVALID_ARG, "lunara_attention: Skv and D must be positive");
  if (D > 256) return fail(LUNARA_ERR_UNSUPPORTED, "lunara_attention: head dim %lld > 256", (long long)D);
  if (B > 65535 || H > 65535 || Sq >= (int64_t{1} << 31) / 4)
    return fail(LUNARA_ERR_UNSUPPORTED, "lunara_attention: grid too large");
  if (!Q || !K || !V || !O) return fail(LUNARA_ERR_INVALID_ARG, "lunara_attention: NULL tensor");
  if (!q_strides || !k_strides || !v_strides || !o_strides)
    return fail(LUNARA_ERR_INVALID_ARG, "lunara_attention: NULL strides");
  AttnArgs a{};
  a.Q = Q;
  a.K = K;
  a.V = V;
  a.O = O;
  a.B = B;
  a.H = H;
  a.Sq = Sq;
  a.Skv = Skv;
  a.D = D;
  for (int i = 0; i < 4; ++i) {
    a.qs[i] = q_strides[i];
    a.ks[i] = k_strides[i];
    a.vs[i] = v_strides[i];
    a.os[i] = o_strides[i];
  }
  a.scale = scale;
  a.causal = causal ? 1 : 0;
  a.dtype = dtype;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (attention_tc_supported(a)) {
    bool handled = false;
    const cudaError_t e = launch_attention_tcgen05(a, s, &handled);
    if (handled) return from_cuda(e, "lunara_attention(tcgen05)");
  }
  return from_cuda(launch_attention_simt(a, s), "lunara_attention(simt)");
}

int lunara_layernorm(const void* X, const void* gamma, const void* beta, void* Y, int64_t M, int64_t N, float eps,
                     int dtype, void* stream) {
  if (!valid_dtype(dtype)) return fail(LUNARA_ERR_INVALID_ARG, "lunara_layernorm: bad dtype %d", dtype);
  if (M < 0 || N <= 0) return fail(LUNARA_ERR_INVALID_ARG, "lunara_layernorm: bad shape M=%lld N=%lld",
                                   (long long)M, (long long)N);
  if (M >= (int64_t{1} << 31)) return fail(LUNARA_ERR_UNSUPPORTED, "lunara_layernorm: M >= 2^31");
  if (M == 0) return ok();
  if (!X || !gamma || !beta || !Y) return fail(LUNARA_ERR_INVALID_ARG, "lunara_layernorm: NULL tensor");
  if (!(eps >= 0.0f)) return fail(LUNARA_ERR_INVALID_ARG, "lunara_layernorm: eps must be >= 0");
  return from_cuda(launch_layernorm(X, gamma, beta, Y, M, N, eps, dtype, static_cast<cudaStream_t>(stream)),
                   "lunara_layernorm");
}

int lunara_softmax(const void* X, void* Y, int64_t M, int64_t N, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return fail(LUNARA_ERR_INVALID_ARG, "lunara_softmax: bad dtype %d", dtype);
  if (M < 0 || N <= 0) return fail(LUNARA_ERR_INVALID_ARG, "lunara_softmax: bad shape");
  if (M >= (int64_t{1} << 31)) return fail(LUNARA_ERR_UNSUPPORTED, "lunara_softmax: M >= 2^31");
  if (M == 0) return ok();
  if (!X || !Y) return fail(LUNARA_ERR_INVALID_ARG, "lunara_softmax: NULL tensor");
  return from_cuda(launch_softmax(X, Y, M, N, dtype, static_cast<cudaStream_t>(stream)), "lunara_softmax");
}

int lunara_eltwise_unary(int activation, const void* X, void* Y, int64_t n, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return fail(LUNARA_ERR_INVALID_ARG, "lunara_eltwise_unary: bad dtype %d", dtype);
  if (!valid_act(activation)) return fail(LUNARA_ERR_INVALID_ARG, "lunara_eltwise_unary: bad op %d", activation);
  if (n < 0) return fail(LUNARA_ERR_INVALID_ARG, "lunara_eltwise_unary: n < 0");
  if (n == 0) return ok();
  if (!X || !Y) return fail(LUNARA_ERR_INVALID_ARG, "lunara_eltwise_unary: NULL tensor");
  return from_cuda(launch_eltwise_unary(activation, X, Y, n, dtype, static_cast<cudaStream_t>(stream)),
                   "lunara_eltwise_unary");
}

int lunara_eltwise_binary(int op, const void* X, const void* Y, void* Out, int64_t n, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return fail(LUNARA_ERR_INVALID_ARG, "lunara_eltwise_binary: bad dtype %d", dtype);
  if (op != LUNARA_BIN_ADD && op != LUNARA_BIN_MUL)
    return fail(LUNARA_ERR_INVALID_ARG, "lunara_eltwise_binary: bad op %d", op);
  if (n < 0) return fail(LUNARA_ERR_INVALID_ARG, "lunara_eltwise_binary: n < 0");
  if (n == 0) return ok();
  if (!X || !Y || !Out) return fail(LUNARA_ERR_INVALID_ARG, "lunara_eltwise_binary: NULL tensor");
  return from_cuda(launch_eltwise_binary(op, X, Y, Out, n, dtype, static_cast<cudaStream_t>(stream)),
                   "lunara_eltwise_binary");
}

int lunara_bias_act(const void* X, const void* bias, void* Y, int64_t rows, int64_t cols, int activation, int dtype,
                    void* stream) {
  if (!valid_dtype(dtype)) return fail(LUNARA_ERR_INVALID_ARG, "lunara_bias_act: bad dtype %d", dtype);
  if (!valid_act(activation)) return fail(LUNARA_ERR_INVALID_ARG, "lunara_bias_act: bad activation %d", activation);
  if (rows < 0 || cols < 0) return fail(LUNARA_ERR_INVALID_ARG, "lunara_bias_act: negative shape");
  if (rows == 0 || cols == 0) return ok();
  if (!X || !bias || !Y) return fail(LUNARA_ERR_INVALID_ARG, "lunara_bias_act: NULL tensor");
  return from_cuda(launch_bias_act(X, bias, Y, rows, cols, activation, dtype, static_cast<cudaStream_t>(stream)),
                   "lunara_bias_act");
}

int lunara_gather(const void* src, const int64_t* index, void* dst, int64_t n_index, int64_t src_rows,
                  int64_t row_bytes, void* stream) {
  if (n_index < 0 || src_rows < 0 || row_bytes < 0) return fail(LUNARA_ERR_INVALID_ARG, "lunara_gather: negative size");
  if (n_index == 0 || row_bytes == 0) return ok();
  if (!index || !dst) return fail(LUNARA_ERR_INVALID_ARG, "lunara_gather: NULL pointer");
  if (!src && src_rows > 0) return fail(LUNARA_ERR_INVALID_ARG, "lunara_gather: NULL source");
  // One warp per row, 8 rows per 256-thread block: the grid's x dimension
  // (at most 2^31 - 1 blocks) bounds the row count.
  if (n_index > int64_t{8} * ((int64_t{1} << 31) - 1))
    return fail(LUNARA_ERR_UNSUPPORTED, "lunara_gather: too many indices");
  return from_cuda(launch_gather(src, index, dst, n_index, src_rows, row_bytes, static_cast<cudaStream_t>(stream)),
                   "lunara_gather");
}

int lunara_copy_strided(const void* src, void* dst, int ndim, const int64_t* sizes, const int64_t* src_strides,
                        int64_t elem_bytes, void* stream) {
  if (ndim < 0 || ndim > 8) return fail(LUNARA_ERR_UNSUPPORTED, "lunara_copy_strided: ndim %d not in [0, 8]", ndim);
  if (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4 && elem_bytes != 8)
    return fail(LUNARA_ERR_INVALID_ARG, "lunara_copy_strided: elem_bytes %lld", (long long)elem_bytes);
  if (ndim > 0 && (!sizes || !src_strides)) return fail(LUNARA_ERR_INVALID_ARG, "lunara_copy_strided: NULL sizes");
  for (int k = 0; k < ndim; ++k) {
    if (sizes[k] < 0) return fail(LUNARA_ERR_INVALID_ARG, "lunara_copy_strided: negative size");
    if (sizes[k] == 0) return ok();
  }
  if (!src || !dst) return fail(LUNARA_ERR_INVALID_ARG, "lunara_copy_strided: NULL pointer");
  const int64_t one = 1, zero = 0;
  const int64_t* sz = ndim > 0 ? sizes : &one;
  const int64_t* st = ndim > 0 ? src_strides : &zero;
  return from_cuda(launch_copy_strided(src, dst, ndim > 0 ? ndim : 1, sz, st, elem_bytes,
                                       static_cast<cudaStream_t>(stream)),
                   "lunara_copy_strided");
}

int lunara_slice(const void* src, void* dst, int ndim, const int64_t* src_sizes, const int64_t* starts,
                 const int64_t* steps, const int64_t* dst_sizes, int64_t elem_bytes, void* stream) {
  if (ndim < 1 || ndim > 8) return fail(LUNARA_ERR_UNSUPPORTED, "lunara_slice: ndim %d not in [1, 8]", ndim);
  if (!src_sizes || !starts || !steps || !dst_sizes) return fail(LUNARA_ERR_INVALID_ARG, "lunara_slice: NULL array");
  int64_t strides[8];
  int64_t acc = 1;
  for (int k = ndim - 1; k >= 0; --k) {
    strides[k] = acc;
    acc *= src_sizes[k];
  }
  int64_t offset = 0;
  int64_t step_strides[8];
  for (int k = 0; k < ndim; ++k) {
    if (src_sizes[k] < 0 || dst_sizes[k] < 0) return fail(LUNARA_ERR_INVALID_ARG, "lunara_slice: negative size");
    if (steps[k] < 1) return fail(LUNARA_ERR_INVALID_ARG, "lunara_slice: step must be >= 1");
    if (dst_sizes[k] == 0) return ok();
    const int64_t last = starts[k] + (dst_sizes[k] - 1) * steps[k];
    if (starts[k] < 0 || last >= src_sizes[k])
      return fail(LUNARA_ERR_INVALID_ARG, "lunara_slice: dim %d range [%lld, %lld] outside [0, %lld)", k,
                  (long long)starts[k], (long long)last, (long long)src_sizes[k]);
    offset += starts[k] * strides[k];
    step_strides[k] = strides[k] * steps[k];
  }
  if (!src || !dst) return fail(LUNARA_ERR_INVALID_ARG, "lunara_slice: NULL pointer");
  const char* base = static_cast<const char*>(src) + offset * elem_bytes;
  return lunara_copy_strided(base, dst, ndim, dst_sizes, step_strides, elem_bytes, stream);
}

int lunara_qkv_split(const void* qkv, void* q, void* k, void* v, int64_t B, int64_t S, int64_t H, int64_t D,
                     int64_t elem_bytes, void* stream) {
  if (B < 0 || S < 0 || H < 0 || D < 0) return fail(LUNARA_ERR_INVALID_ARG, "lunara_qkv_split: negative shape");
  if (B == 0 || S == 0 || H == 0 || D == 0) return ok();
  if (!qkv || !q || !k || !v) return fail(LUNARA_ERR_INVALID_ARG, "lunara_qkv_split: NULL pointer");
  if (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4 && elem_bytes != 8)
    return fail(LUNARA_ERR_INVALID_ARG, "lunara_qkv_split: elem_bytes %lld", (long long)elem_bytes);
  bool handled = false;
  const cudaError_t e = launch_qkv_split(qkv, q, k, v, B, S, H, D, elem_bytes, static_cast<cudaStream_t>(stream),
                                         &handled);
  if (handled) return from_cuda(e, "lunara_qkv_split");
  // Source viewed as [B, S, 3, H, D]; destination [B, H, S, D] for each of q, k, v.
  const int64_t sizes[4] = {B, H, S, D};
  const int64_t strides[4] = {S * 3 * H * D, D, 3 * H * D, 1};
  void* outs[3] = {q, k, v};
  for (int which = 0; which < 3; ++which) {
    const char* base = static_cast<const char*>(qkv) + which * H * D * elem_bytes;
    const int rc = lunara_copy_strided(base, outs[which], 4, sizes, strides, elem_bytes, stream);
    if (rc != LUNARA_OK) return rc;
  }
  return ok();
}

}  // extern "C"
