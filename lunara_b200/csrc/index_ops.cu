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

// IdxT is uint32_t when the element count fits (32-bit division is several
// times cheaper than 64-bit on the SM), else int64_t; source offsets stay
// 64-bit either way.
template <typename U, typename IdxT>
__global__ void __launch_bounds__(kThreads) copy_strided_kernel(const U* __restrict__ src, U* __restrict__ dst,
                                                                StridedDesc d, int64_t total) {
  const IdxT step = static_cast<IdxT>(gridDim.x) * kThreads;
  const IdxT n = static_cast<IdxT>(total);
  for (IdxT i = static_cast<IdxT>(blockIdx.x) * kThreads + threadIdx.x; i < n; i += step) {
    IdxT rem = i;
    int64_t off = 0;
#pragma unroll
    for (int k = kMaxDims - 1; k >= 0; --k) {
      if (k < d.ndim) {
        const IdxT sz = static_cast<IdxT>(d.sizes[k]);
        const IdxT q = rem / sz;
        off += static_cast<int64_t>(rem - q * sz) * d.strides[k];
        rem = q;
      }
    }
    dst[i] = src[off];
  }
}

bool al(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// QKV split + head reshape in one launch: source [B, S, 3, H, DU] in 16-byte
// units, destinations [B, H, S, DU] for q, k and v. grid = (ceil(S*DU /
// (kQkvUnits*256)), B*H, 3): each thread moves kQkvUnits units 256 apart
// (both loads before either store); a warp reads 128-byte head rows of
// consecutive positions and writes 512 contiguous bytes. The only division
// per unit is by DU (position and unit within the head row).
constexpr int kQkvUnits = 4;

__global__ void __launch_bounds__(kThreads) qkv_split_kernel(const uint4* __restrict__ src, uint4* __restrict__ q,
                                                             uint4* __restrict__ k, uint4* __restrict__ v,
                                                             int S, int H, int DU) {
  pdl_wait();
  pdl_launch_dependents();
  const int bh = static_cast<int>(blockIdx.y);
  const int b = bh / H;
  const int h = bh - b * H;
  const int which = static_cast<int>(blockIdx.z);
  uint4* dst = which == 0 ? q : (which == 1 ? k : v);
  const int t0 = static_cast<int>(blockIdx.x) * (kQkvUnits * kThreads) + static_cast<int>(threadIdx.x);
  uint4 val[kQkvUnits];
#pragma unroll
  for (int j = 0; j < kQkvUnits; ++j) {
    const int t = t0 + j * kThreads;
    if (t < S * DU) {
      const int s = t / DU;
      const int u = t - s * DU;
      val[j] = src[((static_cast<int64_t>(b) * S + s) * 3 + which) * H * DU + static_cast<int64_t>(h) * DU + u];
    }
  }
#pragma unroll
  for (int j = 0; j < kQkvUnits; ++j) {
    const int t = t0 + j * kThreads;
    if (t < S * DU) dst[static_cast<int64_t>(bh) * S * DU + t] = val[j];
  }
}

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
  if (total + int64_t{grid} * kThreads < (int64_t{1} << 32))
    copy_strided_kernel<U, uint32_t><<<grid, kThreads, 0, s>>>(static_cast<const U*>(src), static_cast<U*>(dst), d,
                                                                total);
  else
    copy_strided_kernel<U, int64_t><<<grid, kThreads, 0, s>>>(static_cast<const U*>(src), static_cast<U*>(dst), d,
                                                               total);
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

cudaError_t launch_qkv_split(const void* qkv, void* q, void* k, void* v, int64_t B, int64_t S, int64_t H,
                             int64_t D, int64_t elem_bytes, cudaStream_t stream, bool* handled) {
  *handled = false;
  const int64_t row_bytes = D * elem_bytes;
  if (row_bytes % 16 != 0 || !al(qkv, 16) || !al(q, 16) || !al(k, 16) || !al(v, 16)) return cudaSuccess;
  const int64_t du = row_bytes / 16;
  if (B * H > 65535 || S * du >= (int64_t{1} << 31) || H * du >= (int64_t{1} << 31)) return cudaSuccess;
  *handled = true;
  const dim3 grid(static_cast<unsigned>(ceil_div64(S * du, kQkvUnits * kThreads)), static_cast<unsigned>(B * H), 3);
  return launch_pdl(qkv_split_kernel, grid, dim3(kThreads), 0, stream, static_cast<const uint4*>(qkv),
                    static_cast<uint4*>(q), static_cast<uint4*>(k), static_cast<uint4*>(v), static_cast<int>(S),
                    static_cast<int>(H), static_cast<int>(du));
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
