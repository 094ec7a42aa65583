// Internal self-test entry points (include/lunara_b200_selftest.h): device
// code paths that tests must reach but that no product input reaches on
// purpose.
//   * the FMA-pipe exponential of the attention softmax, evaluated over a
//     buffer so that its error can be bounded against exp2;
//   * the bounded mbarrier wait every warp-specialised kernel uses, run
//     against a barrier that nothing arrives on, so that a test sees the wait
//     give up, record its site code and return.
#include "../../include/lunara_b200_selftest.h"
#include "common.cuh"
#include "kernels.h"

namespace lunara {
namespace {

// y[i] = 2^x[i]: the scalar ex2_poly (mode 0), the f32x2 ex2_poly2 on
// (x[2i], x[2i+1]) (mode 1), or the clamped f32x2 form the attention softmax
// runs, ex2_poly2_clamped (mode 2).
__global__ void ex2_poly_selftest_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n, int mode) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (mode) {
    if (2 * i + 1 >= n) return;
    const uint64_t in = f2_pack(x[2 * i], x[2 * i + 1]);
    const float2 r = f2_unpack(mode == 2 ? ex2_poly2_clamped(in) : ex2_poly2(in));
    y[2 * i] = r.x;
    y[2 * i + 1] = r.y;
  } else if (i < n) {
    y[i] = ex2_poly(x[i]);
  }
}

// One thread waits, with the product kernels' mbar_wait, for phase 0 of a
// freshly initialised barrier whose single expected arrival never comes. The
// wait runs out after budget_ns, sets the CTA's abort flag and records `site`.
__global__ void bounded_wait_selftest_kernel(unsigned long long budget_ns, unsigned int site, unsigned int* err) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool completed = mbar_wait(&bar, 0u, &abort_flag, err, site, budget_ns);
    (void)completed;   // false: the budget ran out and the site code is recorded
  }
  __syncthreads();
}

}  // namespace
}  // namespace lunara

extern "C" {

int lunara_selftest_ex2_poly(const float* x, float* y, int64_t n, int pair, void* stream) {
  if (pair < 0 || pair > 2) return 1;
  if (n < 0 || (n > 0 && (x == nullptr || y == nullptr)) || (pair && (n & 1)) || n > (int64_t{1} << 30)) return 1;
  if (n == 0) return 0;
  const int64_t threads = pair ? n / 2 : n;
  const unsigned grid = static_cast<unsigned>((threads + 255) / 256);
  lunara::ex2_poly_selftest_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n, pair);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int lunara_selftest_bounded_wait(uint64_t budget_ns, unsigned int site, void* stream) {
  if (budget_ns < 1000ull || budget_ns > 1000000000ull) return 1;
  if (site < 0x401u || site > 0x4ffu) return 1;
  unsigned int* err = lunara::device_error_word();
  if (err == nullptr) return 3;
  lunara::bounded_wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<unsigned long long>(budget_ns), site, err);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

}  // extern "C"
