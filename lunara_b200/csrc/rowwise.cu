// Row-wise bandwidth kernels: LayerNorm and Softmax over the last dimension.
//
// Main path: one warp per row, 128-bit coalesced loads (8 x 16-bit or 4 x fp32
// per lane per vector), the whole row held in registers, warp-shuffle
// reductions, statistics in fp32. HBM traffic is one read and one write of the
// row (plus gamma/beta, which stay in L1/L2).
// Fallback path (rows that are not a whole number of 16-byte vectors, or
// longer than 16 vectors per lane): one CTA per row with block reductions.
//
// LayerNorm follows lunara/codegen/triton_emitter.py:382-398 (two-pass mean and
// variance in fp32, then (x - mean) / sqrt(var + eps) * w + b), with the
// variance taken over exactly N elements: the reference also sums (0 - mean)^2
// for the padding lanes of its power-of-two block, which is not kept.
// Softmax follows triton_emitter.py:341-353 (max, exp(x - max), / sum; the
// division taken as one reciprocal per row and a multiply per element).
#include "common.cuh"
#include "kernels.h"

namespace lunara {
namespace {

template <typename T>
struct VecTraits {
  static constexpr int kElems = 16 / sizeof(T);
};

template <typename T>
__device__ __forceinline__ void unpack_vec(const uint4& u, float* f) {
  if constexpr (sizeof(T) == 4) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  } else {
    float2 a = Io<T>::unpack2(u.x), b = Io<T>::unpack2(u.y), c = Io<T>::unpack2(u.z), d = Io<T>::unpack2(u.w);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
    f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack_vec(const float* f) {
  uint4 u;
  if constexpr (sizeof(T) == 4) {
    u.x = __float_as_uint(f[0]);
    u.y = __float_as_uint(f[1]);
    u.z = __float_as_uint(f[2]);
    u.w = __float_as_uint(f[3]);
  } else {
    u.x = Io<T>::pack2(f[0], f[1]);
    u.y = Io<T>::pack2(f[2], f[3]);
    u.z = Io<T>::pack2(f[4], f[5]);
    u.w = Io<T>::pack2(f[6], f[7]);
  }
  return u;
}

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 u;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
               : "l"(p));
  return u;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// CTA size of the one-CTA-per-row fallbacks.
constexpr int kRowThreads = 256;
// The warp-per-row paths use 4 rows per 128-thread CTA: on B200 these measured
// faster than 8-row CTAs (LayerNorm 16384 x 768 fp16: 10.44 vs 10.65 us, 16384
// x 1024 bf16: 13.5 vs 15.6 us; softmax 8192 x 4096 fp16: 49.2 vs 62.9 us,
// 16384 x 1024: 15.8 vs 16.4 us) and 16-row CTAs were slower still.
constexpr int kWarpRowThreads = 128;

// ------------------------------------------------------------ LayerNorm ----
template <typename T, int VPL>
__global__ void __launch_bounds__(kWarpRowThreads) layernorm_warp_kernel(const T* __restrict__ X,
                                                                     const T* __restrict__ gamma,
                                                                     const T* __restrict__ beta, T* __restrict__ Y,
                                                                     int64_t M, int N, float eps) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int EPV = VecTraits<T>::kElems;
  const int nv = N / EPV;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (kWarpRowThreads / 32) + (threadIdx.x >> 5);
  if (row >= M) return;
  const uint4* xr = reinterpret_cast<const uint4*>(X + row * N);
  float v[VPL][EPV];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int vi = lane + i * 32;
    if (vi < nv) {
      unpack_vec<T>(ld_stream(xr + vi), v[i]);
#pragma unroll
      for (int e = 0; e < EPV; ++e) sum += v[i][e];
    } else {
#pragma unroll
      for (int e = 0; e < EPV; ++e) v[i][e] = 0.f;
    }
  }
  const float inv_n = 1.0f / static_cast<float>(N);
  const float mean = warp_sum(sum) * inv_n;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    if (lane + i * 32 < nv) {
#pragma unroll
      for (int e = 0; e < EPV; ++e) {
        v[i][e] -= mean;
        sq = fmaf(v[i][e], v[i][e], sq);
      }
    }
  }
  const float rstd = rsqrtf(warp_sum(sq) * inv_n + eps);
  const uint4* gv = reinterpret_cast<const uint4*>(gamma);
  const uint4* bv = reinterpret_cast<const uint4*>(beta);
  uint4* yr = reinterpret_cast<uint4*>(Y + row * N);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int vi = lane + i * 32;
    if (vi < nv) {
      float g[EPV], b[EPV], o[EPV];
      unpack_vec<T>(__ldg(gv + vi), g);
      unpack_vec<T>(__ldg(bv + vi), b);
#pragma unroll
      for (int e = 0; e < EPV; ++e) o[e] = fmaf(v[i][e] * rstd, g[e], b[e]);
      yr[vi] = pack_vec<T>(o);
    }
  }
}

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = (lane < NT / 32) ? red[lane] : 0.f;
  return warp_sum(t);
}

template <int NT>
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = (lane < NT / 32) ? red[lane] : -INFINITY;
  return warp_max(t);
}

template <typename T>
__global__ void __launch_bounds__(kRowThreads) layernorm_block_kernel(const T* __restrict__ X,
                                                                      const T* __restrict__ gamma,
                                                                      const T* __restrict__ beta, T* __restrict__ Y,
                                                                      int64_t N, float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = X + row * N;
  float s = 0.f;
  for (int64_t c = threadIdx.x; c < N; c += kRowThreads) s += Io<T>::to_f(xr[c]);
  const float mean = block_sum<kRowThreads>(s, red) / static_cast<float>(N);
  float q = 0.f;
  for (int64_t c = threadIdx.x; c < N; c += kRowThreads) {
    const float d = Io<T>::to_f(xr[c]) - mean;
    q = fmaf(d, d, q);
  }
  const float rstd = rsqrtf(block_sum<kRowThreads>(q, red) / static_cast<float>(N) + eps);
  T* yr = Y + row * N;
  for (int64_t c = threadIdx.x; c < N; c += kRowThreads) {
    const float o = fmaf((Io<T>::to_f(xr[c]) - mean) * rstd, Io<T>::to_f(gamma[c]), Io<T>::to_f(beta[c]));
    yr[c] = Io<T>::from_f(o);
  }
}

// -------------------------------------------------------------- Softmax ----
constexpr float kLog2e = 1.4426950408889634f;

template <typename T, int VPL>
__global__ void __launch_bounds__(kWarpRowThreads) softmax_warp_kernel(const T* __restrict__ X, T* __restrict__ Y,
                                                                   int64_t M, int N) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int EPV = VecTraits<T>::kElems;
  const int nv = N / EPV;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (kWarpRowThreads / 32) + (threadIdx.x >> 5);
  if (row >= M) return;
  const uint4* xr = reinterpret_cast<const uint4*>(X + row * N);
  float v[VPL][EPV];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int vi = lane + i * 32;
    if (vi < nv) {
      unpack_vec<T>(ld_stream(xr + vi), v[i]);
#pragma unroll
      for (int e = 0; e < EPV; ++e) mx = fmaxf(mx, v[i][e]);
    }
  }
  mx = warp_max(mx);
  const float mxs = mx * kLog2e;
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    if (lane + i * 32 < nv) {
#pragma unroll
      for (int e = 0; e < EPV; ++e) {
        v[i][e] = ex2_approx(fmaf(v[i][e], kLog2e, -mxs));
        sum += v[i][e];
      }
    }
  }
  // One division per row, then a multiply per element: an IEEE division per
  // element made this kernel ALU-bound (49152 x 512 fp16: 21.5 us, against
  // 17.2 us with the reciprocal, which is what a plain copy of the rows takes).
  const float rsum = 1.0f / warp_sum(sum);
  uint4* yr = reinterpret_cast<uint4*>(Y + row * N);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int vi = lane + i * 32;
    if (vi < nv) {
      float o[EPV];
#pragma unroll
      for (int e = 0; e < EPV; ++e) o[e] = v[i][e] * rsum;
      yr[vi] = pack_vec<T>(o);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kRowThreads) softmax_block_kernel(const T* __restrict__ X, T* __restrict__ Y,
                                                                    int64_t N) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = X + row * N;
  float mx = -INFINITY;
  for (int64_t c = threadIdx.x; c < N; c += kRowThreads) mx = fmaxf(mx, Io<T>::to_f(xr[c]));
  mx = block_max<kRowThreads>(mx, red);
  const float mxs = mx * kLog2e;
  float s = 0.f;
  for (int64_t c = threadIdx.x; c < N; c += kRowThreads) s += ex2_approx(fmaf(Io<T>::to_f(xr[c]), kLog2e, -mxs));
  const float rs = 1.0f / block_sum<kRowThreads>(s, red);
  T* yr = Y + row * N;
  for (int64_t c = threadIdx.x; c < N; c += kRowThreads)
    yr[c] = Io<T>::from_f(ex2_approx(fmaf(Io<T>::to_f(xr[c]), kLog2e, -mxs)) * rs);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Smallest supported registers-per-lane count covering `need` vectors per lane.
int pick_vpl(int64_t need) {
  static const int kChoices[] = {1, 2, 3, 4, 6, 8, 12, 16};
  for (int c : kChoices)
    if (need <= c) return c;
  return 0;
}

template <typename T>
cudaError_t layernorm_t(const void* X, const void* g, const void* b, void* Y, int64_t M, int64_t N, float eps,
                        cudaStream_t s) {
  constexpr int EPV = VecTraits<T>::kElems;
  const T* x = static_cast<const T*>(X);
  const T* gg = static_cast<const T*>(g);
  const T* bb = static_cast<const T*>(b);
  T* y = static_cast<T*>(Y);
  const bool vec_ok = (N % EPV == 0) && aligned16(X) && aligned16(Y) && aligned16(g) && aligned16(b) &&
                      N <= (int64_t{1} << 30);
  const int vpl = vec_ok ? pick_vpl(ceil_div64(N / EPV, 32)) : 0;
  if (vpl > 0) {
    const dim3 grid(static_cast<unsigned>(ceil_div64(M, kWarpRowThreads / 32)));
    const int n = static_cast<int>(N);
    cudaError_t e = cudaSuccess;
    switch (vpl) {
#define LN_CASE(V)                                                                               \
  case V:                                                                                        \
    e = launch_pdl(layernorm_warp_kernel<T, V>, grid, dim3(kWarpRowThreads), 0, s, x, gg, bb, y, M, n, eps); \
    break;
      LN_CASE(1) LN_CASE(2) LN_CASE(3) LN_CASE(4) LN_CASE(6) LN_CASE(8) LN_CASE(12) LN_CASE(16)
#undef LN_CASE
    }
    return e;
  } else {
    layernorm_block_kernel<T><<<static_cast<unsigned>(M), kRowThreads, 0, s>>>(x, gg, bb, y, N, eps);
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t softmax_t(const void* X, void* Y, int64_t M, int64_t N, cudaStream_t s) {
  constexpr int EPV = VecTraits<T>::kElems;
  const T* x = static_cast<const T*>(X);
  T* y = static_cast<T*>(Y);
  const bool vec_ok = (N % EPV == 0) && aligned16(X) && aligned16(Y) && N <= (int64_t{1} << 30);
  const int vpl = vec_ok ? pick_vpl(ceil_div64(N / EPV, 32)) : 0;
  if (vpl > 0) {
    const dim3 grid(static_cast<unsigned>(ceil_div64(M, kWarpRowThreads / 32)));
    const int n = static_cast<int>(N);
    cudaError_t e = cudaSuccess;
    switch (vpl) {
#define SM_CASE(V)                                                                 \
  case V:                                                                          \
    e = launch_pdl(softmax_warp_kernel<T, V>, grid, dim3(kWarpRowThreads), 0, s, x, y, M, n); \
    break;
      SM_CASE(1) SM_CASE(2) SM_CASE(3) SM_CASE(4) SM_CASE(6) SM_CASE(8) SM_CASE(12) SM_CASE(16)
#undef SM_CASE
    }
    return e;
  } else {
    softmax_block_kernel<T><<<static_cast<unsigned>(M), kRowThreads, 0, s>>>(x, y, N);
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_layernorm(const void* X, const void* gamma, const void* beta, void* Y, int64_t M, int64_t N,
                             float eps, int dtype, cudaStream_t stream) {
  if (M == 0) return cudaSuccess;
  switch (dtype) {
    case LUNARA_F16: return layernorm_t<__half>(X, gamma, beta, Y, M, N, eps, stream);
    case LUNARA_BF16: return layernorm_t<__nv_bfloat16>(X, gamma, beta, Y, M, N, eps, stream);
    default: return layernorm_t<float>(X, gamma, beta, Y, M, N, eps, stream);
  }
}

cudaError_t launch_softmax(const void* X, void* Y, int64_t M, int64_t N, int dtype, cudaStream_t stream) {
  if (M == 0) return cudaSuccess;
  switch (dtype) {
    case LUNARA_F16: return softmax_t<__half>(X, Y, M, N, stream);
    case LUNARA_BF16: return softmax_t<__nv_bfloat16>(X, Y, M, N, stream);
    default: return softmax_t<float>(X, Y, M, N, stream);
  }
}

}  // namespace lunara
