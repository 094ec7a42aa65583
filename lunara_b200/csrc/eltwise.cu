// Elementwise bandwidth kernels: unary activations, binary Add/Mul and the
// fused bias-add + activation over a [rows, cols] matrix.
//
// 128-bit vectorised and coalesced. Unary and binary ops: grid-stride loops
// sized to a whole number of waves over the SMs, two vectors in flight per
// thread per iteration. Bias + activation: one CTA per tile of consecutive
// vectors (two per thread). The activation is a template parameter so the
// inner loop has no branches.
// The unary bodies follow lunara/codegen/triton_emitter.py:452-458 (relu,
// erf-GELU, sigmoid, tanh, identity); the tanh-form GELU of the encoder block
// is added. Math is fp32; the result is rounded once to the output dtype.
#include "common.cuh"
#include "kernels.h"

namespace lunara {
namespace {

template <typename T>
constexpr int kEpv = 16 / sizeof(T);

template <typename T>
__device__ __forceinline__ void unpack16(const uint4& u, float* f) {
  if constexpr (sizeof(T) == 4) {
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
  } else {
    float2 a = Io<T>::unpack2(u.x), b = Io<T>::unpack2(u.y), c = Io<T>::unpack2(u.z), d = Io<T>::unpack2(u.w);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y; f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack16(const float* f) {
  uint4 u;
  if constexpr (sizeof(T) == 4) {
    u.x = __float_as_uint(f[0]); u.y = __float_as_uint(f[1]);
    u.z = __float_as_uint(f[2]); u.w = __float_as_uint(f[3]);
  } else {
    u.x = Io<T>::pack2(f[0], f[1]); u.y = Io<T>::pack2(f[2], f[3]);
    u.z = Io<T>::pack2(f[4], f[5]); u.w = Io<T>::pack2(f[6], f[7]);
  }
  return u;
}

__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
  uint4 u;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
               : "l"(p));
  return u;
}

constexpr int kThreads = 256;

template <typename T, int ACT>
__global__ void __launch_bounds__(kThreads) unary_kernel(const T* __restrict__ X, T* __restrict__ Y, int64_t n) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int EPV = kEpv<T>;
  const int64_t nvec = n / EPV;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const uint4* xv = reinterpret_cast<const uint4*>(X);
  uint4* yv = reinterpret_cast<uint4*>(Y);
  int64_t i = tid;
  for (; i + stride < nvec; i += 2 * stride) {
    uint4 u0 = ldg_stream(xv + i), u1 = ldg_stream(xv + i + stride);
    float f0[EPV], f1[EPV];
    unpack16<T>(u0, f0);
    unpack16<T>(u1, f1);
#pragma unroll
    for (int e = 0; e < EPV; ++e) { f0[e] = apply_act(f0[e], ACT); f1[e] = apply_act(f1[e], ACT); }
    yv[i] = pack16<T>(f0);
    yv[i + stride] = pack16<T>(f1);
  }
  if (i < nvec) {
    float f0[EPV];
    unpack16<T>(ldg_stream(xv + i), f0);
#pragma unroll
    for (int e = 0; e < EPV; ++e) f0[e] = apply_act(f0[e], ACT);
    yv[i] = pack16<T>(f0);
  }
  const int64_t tail = nvec * EPV + tid;
  if (tail < n) Y[tail] = Io<T>::from_f(apply_act(Io<T>::to_f(X[tail]), ACT));
}

template <typename T, int ACT>
__global__ void __launch_bounds__(kThreads) unary_scalar_kernel(const T* __restrict__ X, T* __restrict__ Y,
                                                                int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n; i += stride)
    Y[i] = Io<T>::from_f(apply_act(Io<T>::to_f(X[i]), ACT));
}

template <int OP>
__device__ __forceinline__ float bin(float a, float b) {
  return OP == LUNARA_BIN_ADD ? a + b : a * b;
}

template <typename T, int OP>
__global__ void __launch_bounds__(kThreads) binary_kernel(const T* __restrict__ X, const T* __restrict__ Yin,
                                                          T* __restrict__ Out, int64_t n, int vec) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int EPV = kEpv<T>;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  int64_t done = 0;
  if (vec) {
    const int64_t nvec = n / EPV;
    const uint4* xv = reinterpret_cast<const uint4*>(X);
    const uint4* yv = reinterpret_cast<const uint4*>(Yin);
    uint4* ov = reinterpret_cast<uint4*>(Out);
    for (int64_t i = tid; i < nvec; i += stride) {
      float a[EPV], b[EPV];
      unpack16<T>(ldg_stream(xv + i), a);
      unpack16<T>(ldg_stream(yv + i), b);
#pragma unroll
      for (int e = 0; e < EPV; ++e) a[e] = bin<OP>(a[e], b[e]);
      ov[i] = pack16<T>(a);
    }
    done = nvec * EPV;
  }
  for (int64_t i = done + tid; i < n; i += stride)
    Out[i] = Io<T>::from_f(bin<OP>(Io<T>::to_f(X[i]), Io<T>::to_f(Yin[i])));
}

// Y[r, c] = act(X[r, c] + bias[c]); vectors never straddle rows (cols % EPV == 0).
// Each iteration issues the loads of U vectors (a grid stride apart) before
// using any of them.
template <typename T, int ACT, typename IdxT, int U>
__global__ void __launch_bounds__(kThreads) bias_act_kernel(const T* __restrict__ X, const T* __restrict__ bias,
                                                            T* __restrict__ Y, IdxT nvec, IdxT vec_per_row) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int EPV = kEpv<T>;
  const IdxT stride = static_cast<IdxT>(gridDim.x) * kThreads;
  const uint4* xv = reinterpret_cast<const uint4*>(X);
  const uint4* bv = reinterpret_cast<const uint4*>(bias);
  uint4* yv = reinterpret_cast<uint4*>(Y);
  IdxT i = static_cast<IdxT>(blockIdx.x) * kThreads + threadIdx.x;
  for (; i + (U - 1) * stride < nvec; i += U * stride) {
    uint4 u[U], bb[U];
#pragma unroll
    for (int k = 0; k < U; ++k) u[k] = ldg_stream(xv + i + k * stride);
#pragma unroll
    for (int k = 0; k < U; ++k) bb[k] = __ldg(bv + ((i + k * stride) % vec_per_row));
#pragma unroll
    for (int k = 0; k < U; ++k) {
      float f[EPV], g[EPV];
      unpack16<T>(u[k], f);
      unpack16<T>(bb[k], g);
#pragma unroll
      for (int e = 0; e < EPV; ++e) f[e] = apply_act(f[e] + g[e], ACT);
      yv[i + k * stride] = pack16<T>(f);
    }
  }
  for (; i < nvec; i += stride) {
    float f0[EPV], g0[EPV];
    unpack16<T>(ldg_stream(xv + i), f0);
    unpack16<T>(__ldg(bv + (i % vec_per_row)), g0);
#pragma unroll
    for (int e = 0; e < EPV; ++e) f0[e] = apply_act(f0[e] + g0[e], ACT);
    yv[i] = pack16<T>(f0);
  }
}

// Vectors per thread of the tiled bias + activation kernel.
constexpr int kBiasActTile = 2;

// Tiled form (the main path): CTA b owns the U * kThreads consecutive vectors
// starting at b * U * kThreads; thread t handles vectors t, t + kThreads, ...
// of the tile, all loads issued before any is used. One CTA per tile, no
// grid-stride loop: on B200 this reached 6.4 TB/s at 16384 x 3072 fp16 (0.98
// of a device copy) where a grid-stride loop over 8 CTAs per SM reached 5.5
// TB/s, and more vectors per thread (4, 8) or per-thread loops were slower.
template <typename T, int ACT, typename IdxT, int U>
__global__ void __launch_bounds__(kThreads) bias_act_tile_kernel(const T* __restrict__ X, const T* __restrict__ bias,
                                                                 T* __restrict__ Y, IdxT nvec, IdxT vec_per_row) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int EPV = kEpv<T>;
  const uint4* xv = reinterpret_cast<const uint4*>(X);
  const uint4* bv = reinterpret_cast<const uint4*>(bias);
  uint4* yv = reinterpret_cast<uint4*>(Y);
  const IdxT i0 = static_cast<IdxT>(blockIdx.x) * (U * kThreads) + threadIdx.x;
  uint4 u[U], bb[U];
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const IdxT i = i0 + k * kThreads;
    if (i < nvec) u[k] = ldg_stream(xv + i);
  }
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const IdxT i = i0 + k * kThreads;
    if (i < nvec) bb[k] = __ldg(bv + (i % vec_per_row));
  }
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const IdxT i = i0 + k * kThreads;
    if (i < nvec) {
      float f[EPV], g[EPV];
      unpack16<T>(u[k], f);
      unpack16<T>(bb[k], g);
#pragma unroll
      for (int e = 0; e < EPV; ++e) f[e] = apply_act(f[e] + g[e], ACT);
      yv[i] = pack16<T>(f);
    }
  }
}

template <typename T, int ACT>
__global__ void __launch_bounds__(kThreads) bias_act_scalar_kernel(const T* __restrict__ X,
                                                                   const T* __restrict__ bias, T* __restrict__ Y,
                                                                   int64_t n, int64_t cols) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n; i += stride)
    Y[i] = Io<T>::from_f(apply_act(Io<T>::to_f(X[i]) + Io<T>::to_f(bias[i % cols]), ACT));
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Grid for the grid-stride loops: enough CTAs of 256 threads for `per_thread`
// items each, capped at 64 CTAs per SM (8 waves). On B200 more, shorter-lived
// CTAs streamed faster than one resident wave looping over the data (bias +
// GELU, 16384 x 3072 fp16: 8 CTAs per SM 5.5 TB/s, 16: 5.8, 32: 6.1, 64: 6.3).
unsigned grid_for(int64_t work_items, int per_thread) {
  const int64_t need = ceil_div64(work_items, int64_t{kThreads} * per_thread);
  const int64_t cap = int64_t{device_num_sms()} * 64;
  int64_t g = need < cap ? need : cap;
  return static_cast<unsigned>(g < 1 ? 1 : g);
}

template <typename T>
cudaError_t unary_t(int act, const void* X, void* Y, int64_t n, cudaStream_t s) {
  const T* x = static_cast<const T*>(X);
  T* y = static_cast<T*>(Y);
  const bool vec = al16(X) && al16(Y);
  const unsigned grid = grid_for(vec ? n / kEpv<T> + 1 : n, 2);
  cudaError_t e = cudaSuccess;
#define UN_CASE(A)                                                                           \
  case A:                                                                                    \
    if (vec) e = launch_pdl(unary_kernel<T, A>, dim3(grid), dim3(kThreads), 0, s, x, y, n);  \
    else unary_scalar_kernel<T, A><<<grid, kThreads, 0, s>>>(x, y, n);                       \
    break;
  switch (act) {
    UN_CASE(LUNARA_ACT_NONE) UN_CASE(LUNARA_ACT_RELU) UN_CASE(LUNARA_ACT_GELU_ERF)
    UN_CASE(LUNARA_ACT_GELU_TANH) UN_CASE(LUNARA_ACT_SIGMOID) UN_CASE(LUNARA_ACT_TANH)
    default: return cudaErrorInvalidValue;
  }
#undef UN_CASE
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <typename T>
cudaError_t binary_t(int op, const void* X, const void* Yin, void* Out, int64_t n, cudaStream_t s) {
  const int vec = al16(X) && al16(Yin) && al16(Out);
  const unsigned grid = grid_for(vec ? n / kEpv<T> + 1 : n, 1);
  const T* x = static_cast<const T*>(X);
  const T* yi = static_cast<const T*>(Yin);
  T* o = static_cast<T*>(Out);
  if (op == LUNARA_BIN_ADD)
    return launch_pdl(binary_kernel<T, LUNARA_BIN_ADD>, dim3(grid), dim3(kThreads), 0, s, x, yi, o, n, vec);
  return launch_pdl(binary_kernel<T, LUNARA_BIN_MUL>, dim3(grid), dim3(kThreads), 0, s, x, yi, o, n, vec);
}

template <typename T, int ACT>
cudaError_t bias_act_tt(const T* x, const T* b, T* y, int64_t rows, int64_t cols, cudaStream_t s) {
  constexpr int EPV = kEpv<T>;
  const int64_t n = rows * cols;
  if (cols % EPV == 0 && al16(x) && al16(b) && al16(y)) {
    const int64_t nvec = n / EPV, vpr = cols / EPV;
    constexpr int U = kBiasActTile;
    if (nvec + int64_t{U} * kThreads < (int64_t{1} << 31)) {
      const int64_t tiles = ceil_div64(nvec, int64_t{U} * kThreads);
      return launch_pdl(bias_act_tile_kernel<T, ACT, uint32_t, U>, dim3(static_cast<unsigned>(tiles)),
                        dim3(kThreads), 0, s, x, b, y, static_cast<uint32_t>(nvec), static_cast<uint32_t>(vpr));
    }
    // 2^31 vectors or more: a grid-stride loop with 64-bit indices.
    return launch_pdl(bias_act_kernel<T, ACT, uint64_t, 2>, dim3(grid_for(nvec, 2)), dim3(kThreads), 0, s, x, b,
                      y, static_cast<uint64_t>(nvec), static_cast<uint64_t>(vpr));
  } else {
    bias_act_scalar_kernel<T, ACT><<<grid_for(n, 1), kThreads, 0, s>>>(x, b, y, n, cols);
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t bias_act_t(int act, const void* X, const void* bias, void* Y, int64_t rows, int64_t cols,
                       cudaStream_t s) {
  const T* x = static_cast<const T*>(X);
  const T* b = static_cast<const T*>(bias);
  T* y = static_cast<T*>(Y);
  switch (act) {
    case LUNARA_ACT_NONE: return bias_act_tt<T, LUNARA_ACT_NONE>(x, b, y, rows, cols, s);
    case LUNARA_ACT_RELU: return bias_act_tt<T, LUNARA_ACT_RELU>(x, b, y, rows, cols, s);
    case LUNARA_ACT_GELU_ERF: return bias_act_tt<T, LUNARA_ACT_GELU_ERF>(x, b, y, rows, cols, s);
    case LUNARA_ACT_GELU_TANH: return bias_act_tt<T, LUNARA_ACT_GELU_TANH>(x, b, y, rows, cols, s);
    case LUNARA_ACT_SIGMOID: return bias_act_tt<T, LUNARA_ACT_SIGMOID>(x, b, y, rows, cols, s);
    case LUNARA_ACT_TANH: return bias_act_tt<T, LUNARA_ACT_TANH>(x, b, y, rows, cols, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_eltwise_unary(int act, const void* X, void* Y, int64_t n, int dtype, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  switch (dtype) {
    case LUNARA_F16: return unary_t<__half>(act, X, Y, n, stream);
    case LUNARA_BF16: return unary_t<__nv_bfloat16>(act, X, Y, n, stream);
    default: return unary_t<float>(act, X, Y, n, stream);
  }
}

cudaError_t launch_eltwise_binary(int op, const void* X, const void* Yin, void* Out, int64_t n, int dtype,
                                  cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  switch (dtype) {
    case LUNARA_F16: return binary_t<__half>(op, X, Yin, Out, n, stream);
    case LUNARA_BF16: return binary_t<__nv_bfloat16>(op, X, Yin, Out, n, stream);
    default: return binary_t<float>(op, X, Yin, Out, n, stream);
  }
}

cudaError_t launch_bias_act(const void* X, const void* bias, void* Y, int64_t rows, int64_t cols, int act, int dtype,
                            cudaStream_t stream) {
  if (rows == 0 || cols == 0) return cudaSuccess;
  switch (dtype) {
    case LUNARA_F16: return bias_act_t<__half>(act, X, bias, Y, rows, cols, stream);
    case LUNARA_BF16: return bias_act_t<__nv_bfloat16>(act, X, bias, Y, rows, cols, stream);
    default: return bias_act_t<float>(act, X, bias, Y, rows, cols, stream);
  }
}

}  // namespace lunara
