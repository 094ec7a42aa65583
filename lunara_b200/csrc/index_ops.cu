// Index graph ops, bit-exact byte movement: Gather (rows by int64 index) and a
// strided copy into a contiguous destination, which serves Slice, Reshape of a
// non-contiguous view, Transpose/permute and the QKV split + head reshape.
// The graph ops are listed in lunara/frontend/graph_ir.h:15-30 (OpKind) and
// have no kernel in the reference; BASELINE-level requirement: bit-exact.
//
// Both kernels move 16-byte units when sizes, strides and pointers allow it,
// and fall back to element-sized units otherwise.
#include "common.cuh"
#include "kernels.h"

namespace lunara {

namespace {

constexpr int kThreads = 256;

// One warp per output row.
template <typename U>
__global__ void __launch_bounds__(kThreads) gather_kernel(const U* __restrict__ src, const int64_t* __restrict__ idx,
                                                          U* __restrict__ dst, int64_t n_index, int64_t src_rows,
                                                          int64_t units_per_row, unsigned int* err) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= n_index) return;
  const int64_t s = idx[row];
  U* d = dst + row * units_per_row;
  if (s < 0 || s >= src_rows) {
    if (lane == 0) atomicCAS(err, 0u, static_cast<unsigned>(kErrGatherIndex));
    for (int64_t c = lane; c < units_per_row; c += 32) d[c] = U{};
    return;
  }
  const U* sr = src + s * units_per_row;
  for (int64_t c = lane; c < units_per_row; c += 32) d[c] = sr[c];
}

constexpr int kMaxDims = 8;

struct StridedDesc {
  int ndim;
  int64_t sizes[kMaxDims];
  int64_t strides[kMaxDims];  // in units
};

template <typename U>
__global__ void __launch_bounds__(kThreads) copy_strided_kernel(const U* __restrict__ src, U* __restrict__ dst,
                                                                StridedDesc d, int64_t total) {
  const int64_t step = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total; i += step) {
    int64_t rem = i, off = 0;
#pragma unroll
    for (int k = kMaxDims - 1; k >= 0; --k) {
      if (k < d.ndim) {
        const int64_t q = rem / d.sizes[k];
        off += (rem - q * d.sizes[k]) * d.strides[k];
        rem = q;
      }
    }
    dst[i] = src[off];
  }
}

bool al(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

template <typename U>
cudaError_t gather_u(const void* src, const int64_t* index, void* dst, int64_t n_index, int64_t src_rows,
                     int64_t units, cudaStream_t s) {
  const unsigned grid = static_cast<unsigned>(ceil_div64(n_index, kThreads / 32));
  unsigned int* err = device_error_word();
  if (err == nullptr) return cudaErrorInvalidDevice;
  gather_kernel<U><<<grid, kThreads, 0, s>>>(static_cast<const U*>(src), index, static_cast<U*>(dst), n_index,
                                             src_rows, units, err);
  return cudaGetLastError();
}

template <typename U>
cudaError_t copy_u(const void* src, void* dst, const StridedDesc& d, int64_t total, cudaStream_t s) {
  const int64_t need = ceil_div64(total, kThreads);
  const int64_t cap = int64_t{device_num_sms()} * 16;
  const unsigned grid = static_cast<unsigned>(need < cap ? (need < 1 ? 1 : need) : cap);
  copy_strided_kernel<U><<<grid, kThreads, 0, s>>>(static_cast<const U*>(src), static_cast<U*>(dst), d, total);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gather(const void* src, const int64_t* index, void* dst, int64_t n_index, int64_t src_rows,
                          int64_t row_bytes, cudaStream_t stream) {
  if (n_index == 0 || row_bytes == 0) return cudaSuccess;
  if (row_bytes % 16 == 0 && al(src, 16) && al(dst, 16))
    return gather_u<uint4>(src, index, dst, n_index, src_rows, row_bytes / 16, stream);
  if (row_bytes % 4 == 0 && al(src, 4) && al(dst, 4))
    return gather_u<uint32_t>(src, index, dst, n_index, src_rows, row_bytes / 4, stream);
  return gather_u<uint8_t>(src, index, dst, n_index, src_rows, row_bytes, stream);
}

cudaError_t launch_copy_strided(const void* src, void* dst, int ndim, const int64_t* sizes,
                                const int64_t* src_strides, int64_t elem_bytes, cudaStream_t stream) {
  StridedDesc d{};
  int64_t total = 1;
  // Drop size-1 dimensions; they do not move the source offset.
  for (int k = 0; k < ndim; ++k) {
    if (sizes[k] == 0) return cudaSuccess;
    if (sizes[k] == 1) continue;
    d.sizes[d.ndim] = sizes[k];
    d.strides[d.ndim] = src_strides[k];
    ++d.ndim;
    total *= sizes[k];
  }
  if (d.ndim == 0) {
    d.ndim = 1;
    d.sizes[0] = 1;
    d.strides[0] = 0;
  }
  // Widen the unit to 16 bytes when the innermost dimension is contiguous and
  // every byte stride and both pointers are 16-byte aligned.
  const int in = d.ndim - 1;
  const int64_t inner_bytes = d.sizes[in] * elem_bytes;
  bool wide = d.strides[in] == 1 && inner_bytes % 16 == 0 && al(src, 16) && al(dst, 16);
  for (int k = 0; wide && k < in; ++k) wide = (d.strides[k] * elem_bytes) % 16 == 0;
  if (wide) {
    const int64_t f = 16 / elem_bytes;
    d.sizes[in] /= f;
    for (int k = 0; k < in; ++k) d.strides[k] /= f;
    return copy_u<uint4>(src, dst, d, total / f, stream);
  }
  switch (elem_bytes) {
    case 1: return copy_u<uint8_t>(src, dst, d, total, stream);
    case 2: return copy_u<uint16_t>(src, dst, d, total, stream);
    case 4: return copy_u<uint32_t>(src, dst, d, total, stream);
    case 8: return copy_u<uint64_t>(src, dst, d, total, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace lunara
