// GEMM with fused epilogue: C = act(A * B + bias) + residual.
//
// tcgen05 path (f16 / bf16, TMA-compatible strides): persistent,
// warp-specialised kernels with one CTA per SM and 448 threads (14 warps):
//     warp 0      TMA producer: A [128 x 64] and B [BN x 64] tiles, 128-byte
//                 swizzle, into a STAGES-deep shared-memory ring
//     warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//                 (M=128, N=BN, K=16 per instruction, fp32 accumulate)
//     warps 2..13 epilogue, three warps per TMEM lane quarter (warp % 4): the
//                 tile's 32-column chunks are dealt to the three round-robin;
//                 each chunk is read from TMEM (thread = row), gets bias
//                 (staged per warp in shared memory) + activation + residual
//                 (loaded one chunk ahead) in fp32 with one rounding, is staged
//                 as a 32 x 32 tile in shared memory (64-byte swizzle) and
//                 written by one TMA store (direct 16-byte stores when C is
//                 unaligned)
//   Two TMEM accumulators (2 x BN fp32 columns) let the epilogue of tile i
//   overlap the main loop of tile i+1. gemm_tc2_kernel runs the same roles on
//   a CTA pair (cta_group::2, 256-row tiles). No TMA multicast is used
//   anywhere (the same kernels run in multi-GPU jobs).
// SIMT path: any shape / stride / dtype (incl. f32), 64x64 register tiles.
//
// Semantics follow the reference GEMM template,
// lunara/codegen/triton_emitter.py:107-152: fp32 accumulation over K, then
// bias and activation (145-147). The reference rounds to the output dtype
// before the bias/activation; here the epilogue stays in fp32 and rounds once.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace lunara {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
// Epilogue: three warps per TMEM lane quarter (a warp may only read the 32
// lanes of its quarter, warp % 4); the tile's 32-column chunks are dealt to the
// three column slices round-robin. 14 warps in all keep 128 registers per
// thread (at most 4 warps share an SM sub-partition's 64 KB register file).
constexpr int kEpiWarps = 12;
constexpr int kEpiSlices = kEpiWarps / 4;
constexpr int kMaxWarpChunks = (256 / 32 + kEpiSlices - 1) / kEpiSlices;  // chunks per warp at the widest tile
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kGemmThreads = 64 + kEpiThreads;
constexpr int kMaxDynSmem = 232448;  // 227 KB opt-in limit per block on sm_100
constexpr int kStageC = 2048;       // per epilogue warp: one 32 x 32 16-bit output chunk
constexpr int kBiasPerWarp = 32 * kMaxWarpChunks;   // fp32 bias values staged per epilogue warp
// Alignment slack, barriers and flags, bias staging, output staging.
constexpr int kSmemReserve = 1024 + 512 + kEpiWarps * kBiasPerWarp * 4 + kEpiWarps * kStageC;

struct EpiParams {
  void* C;
  const void* bias;
  const void* residual;
  int64_t ldc, ldr;
  int M, N;
  int act;
  int vec_ok;     // C / residual / bias allow 16-byte accesses
  int tma_store;  // C written through the tensor map (tiles staged in shared memory)
};

__host__ __device__ constexpr int gemm_stages(int bn) {
  return std::min(8, (kMaxDynSmem - kSmemReserve) / (BM * BK * 2 + bn * BK * 2));
}

__host__ __device__ constexpr uint32_t tmem_cols_for(int bn) {
  return (2 * bn <= 128) ? 128u : (2 * bn <= 256 ? 256u : 512u);
}

constexpr int gemm_smem_bytes(int bn, int stages) {
  return stages * (BM * BK * 2 + bn * BK * 2) + kSmemReserve;
}

// Epilogue modes (a template parameter, so the common cases carry no switch
// and the epilogue code stays small enough for the instruction cache).
enum EpiMode : int { kEpiPlain = 0, kEpiGeluTanh = 1, kEpiAnyAct = 2 };

inline int epi_mode_for(int act) {
  return act == LUNARA_ACT_NONE ? kEpiPlain : (act == LUNARA_ACT_GELU_TANH ? kEpiGeluTanh : kEpiAnyAct);
}

// Activation over a 32-value chunk; the switch is taken once per chunk.
__device__ __noinline__ void act_chunk_any(float (&f)[32], int act) {
  switch (act) {
    case LUNARA_ACT_NONE:
      break;
#define LUNARA_ACT_CASE(CODE)                                          \
  case CODE:                                                           \
    _Pragma("unroll") for (int i = 0; i < 32; ++i) f[i] = apply_act(f[i], CODE); \
    break;
      LUNARA_ACT_CASE(LUNARA_ACT_RELU)
      LUNARA_ACT_CASE(LUNARA_ACT_GELU_ERF)
      LUNARA_ACT_CASE(LUNARA_ACT_GELU_TANH)
      LUNARA_ACT_CASE(LUNARA_ACT_SIGMOID)
      LUNARA_ACT_CASE(LUNARA_ACT_TANH)
#undef LUNARA_ACT_CASE
    default:
      break;
  }
}

// Residual values of one chunk, loaded one chunk ahead of their use.
struct ResChunk {
  uint4 q[4];
};

template <typename T>
__device__ __forceinline__ void load_residual(ResChunk& rc, int row, int col0, const EpiParams& ep) {
  if (ep.residual == nullptr || row >= ep.M) return;
  const T* r = static_cast<const T*>(ep.residual) + static_cast<int64_t>(row) * ep.ldr + col0;
  if ((col0 + 32 <= ep.N) && ep.vec_ok) {
    const uint4* rv = reinterpret_cast<const uint4*>(r);
#pragma unroll
    for (int q = 0; q < 4; ++q) rc.q[q] = __ldg(rv + q);
  }
}

// Epilogue for 32 consecutive accumulator columns of one row: + bias (staged
// in shared memory as fp32), activation, + residual, one rounding, store.
template <typename T, int EPI>
__device__ __forceinline__ void epilogue_chunk(const uint32_t (&acc)[32], int row, int col0, const float* s_bias,
                                               const ResChunk& rc, const EpiParams& ep) {
  if (row >= ep.M) return;
  float f[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(acc[i]);
  const bool full = (col0 + 32 <= ep.N) && ep.vec_ok;
  if (ep.bias != nullptr) {
#pragma unroll
    for (int i = 0; i < 32; ++i) f[i] += s_bias[i];
  }
  if constexpr (EPI == kEpiGeluTanh) {
#pragma unroll
    for (int i = 0; i < 32; ++i) f[i] = apply_act(f[i], LUNARA_ACT_GELU_TANH);
  } else if constexpr (EPI == kEpiAnyAct) {
    act_chunk_any(f, ep.act);
  }
  if (ep.residual != nullptr) {
    if (full) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t w[4] = {rc.q[q].x, rc.q[q].y, rc.q[q].z, rc.q[q].w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float2 p = Io<T>::unpack2(w[h]);
          f[q * 8 + 2 * h] += p.x;
          f[q * 8 + 2 * h + 1] += p.y;
        }
      }
    } else {
      const T* r = static_cast<const T*>(ep.residual) + static_cast<int64_t>(row) * ep.ldr + col0;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col0 + i < ep.N) f[i] += Io<T>::to_f(r[i]);
    }
  }
  T* c = static_cast<T*>(ep.C) + static_cast<int64_t>(row) * ep.ldc + col0;
  if (full) {
    uint4* cv = reinterpret_cast<uint4*>(c);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 u;
      u.x = Io<T>::pack2(f[q * 8 + 0], f[q * 8 + 1]);
      u.y = Io<T>::pack2(f[q * 8 + 2], f[q * 8 + 3]);
      u.z = Io<T>::pack2(f[q * 8 + 4], f[q * 8 + 5]);
      u.w = Io<T>::pack2(f[q * 8 + 6], f[q * 8 + 7]);
      cv[q] = u;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (col0 + i < ep.N) c[i] = Io<T>::from_f(f[i]);
  }
}

// Bias + activation + residual of one 32-column chunk of one row, rounded and
// packed as 16 pairs of 16-bit values.
template <typename T, int EPI>
__device__ __forceinline__ void epilogue_pack(const uint32_t (&acc)[32], int row, int col0, const float* s_bias,
                                              const ResChunk& rc, const EpiParams& ep, uint32_t (&pk)[16]) {
  float f[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(acc[i]);
  if (ep.bias != nullptr) {
#pragma unroll
    for (int i = 0; i < 32; ++i) f[i] += s_bias[i];
  }
  if constexpr (EPI == kEpiGeluTanh) {
#pragma unroll
    for (int i = 0; i < 32; ++i) f[i] = apply_act(f[i], LUNARA_ACT_GELU_TANH);
  } else if constexpr (EPI == kEpiAnyAct) {
    act_chunk_any(f, ep.act);
  }
  if (ep.residual != nullptr && row < ep.M) {
    if (col0 + 32 <= ep.N) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t w[4] = {rc.q[q].x, rc.q[q].y, rc.q[q].z, rc.q[q].w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float2 p = Io<T>::unpack2(w[h]);
          f[q * 8 + 2 * h] += p.x;
          f[q * 8 + 2 * h + 1] += p.y;
        }
      }
    } else {
      const T* r = static_cast<const T*>(ep.residual) + static_cast<int64_t>(row) * ep.ldr + col0;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col0 + i < ep.N) f[i] += Io<T>::to_f(r[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) pk[i] = Io<T>::pack2(f[2 * i], f[2 * i + 1]);
}

// One 32-row x 32-column output chunk of a warp, already rounded and packed:
// staged in the warp's shared buffer with the 64-byte swizzle (16-byte chunk q
// of row r at slot q ^ ((r >> 1) & 3), conflict-free) and written by one TMA
// store that clips rows >= M and columns >= N.
__device__ __forceinline__ void store_chunk_tma(const uint32_t (&pk)[16], int col0, int row0_warp,
                                                const CUtensorMap* tma_c, uint8_t* s_stage, int lane) {
  if (lane == 0) bulk_wait_group_read<0>();   // the previous chunk's store has read the buffer
  __syncwarp();
  uint8_t* dst = s_stage + lane * 64;
#pragma unroll
  for (int q = 0; q < 4; ++q)
    *reinterpret_cast<uint4*>(dst + ((q ^ ((lane >> 1) & 3)) << 4)) =
        make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tma_c, s_stage, col0, row0_warp);
    bulk_commit_group();
  }
}

// The epilogue of one accumulator tile for one warp: its chunks
// c = slice + j * kEpiSlices of the 32 rows starting at row0_warp (this lane's
// row = row0_warp + lane). A chunk's TMEM load and residual load are issued as
// soon as the previous chunk has been packed, so they run under that chunk's
// store; `res` holds the first chunk's residual, loaded by the caller before
// the accumulator was ready.
template <typename T, int BN, int EPI>
__device__ __forceinline__ void epilogue_tile(uint32_t t_tile, int row0_warp, int n0, int slice, const float* sb,
                                              const EpiParams& ep, const CUtensorMap* tma_c, uint8_t* s_stage,
                                              int lane, ResChunk& res) {
  constexpr int kChunks = BN / 32;
  static_assert(kChunks <= kEpiSlices * kMaxWarpChunks, "epilogue chunk split");
  if (slice >= kChunks) return;
  const int row = row0_warp + lane;
  uint32_t v[32];
  tmem_ld_32x32b_x32(t_tile + slice * 32, v);
#pragma unroll
  for (int j = 0; j < kMaxWarpChunks; ++j) {
    const int c = slice + j * kEpiSlices;
    if (c >= kChunks) break;
    const bool more = c + kEpiSlices < kChunks;
    tmem_ld_wait_regs(v);
    if (ep.tma_store) {
      uint32_t pk[16];
      epilogue_pack<T, EPI>(v, row, n0 + c * 32, sb + j * 32, res, ep, pk);
      if (more) {
        tmem_ld_32x32b_x32(t_tile + (c + kEpiSlices) * 32, v);
        load_residual<T>(res, row, n0 + (c + kEpiSlices) * 32, ep);
      }
      store_chunk_tma(pk, n0 + c * 32, row0_warp, tma_c, s_stage, lane);
    } else {
      epilogue_chunk<T, EPI>(v, row, n0 + c * 32, sb + j * 32, res, ep);
      if (more) {
        tmem_ld_32x32b_x32(t_tile + (c + kEpiSlices) * 32, v);
        load_residual<T>(res, row, n0 + (c + kEpiSlices) * 32, ep);
      }
    }
  }
}

// Stage the bias (fp32) of this warp's chunks in its own shared-memory region;
// only this warp reads it, so __syncwarp orders writes and reads.
template <typename T, int BN>
__device__ __forceinline__ void stage_bias(float* sb, int n0, int slice, const EpiParams& ep, int lane) {
  if (ep.bias == nullptr) return;
#pragma unroll
  for (int j = 0; j < kMaxWarpChunks; ++j) {
    const int c = slice + j * kEpiSlices;
    if (c >= BN / 32) break;
    const int col = n0 + c * 32 + lane;
    sb[j * 32 + lane] = col < ep.N ? Io<T>::to_f(static_cast<const T*>(ep.bias)[col]) : 0.f;
  }
}

template <typename T, int BN, bool B_KMAJOR, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                   const __grid_constant__ CUtensorMap tma_c, const EpiParams ep, const int M, const int N, const int K, const int STAGES,
                   unsigned int* err) {
  // STAGES (ring depth) is chosen on the host, 2 <= STAGES <= gemm_stages(BN);
  // the dynamic shared-memory size is sized for it.
  constexpr uint32_t A_BYTES = BM * BK * 2;
  constexpr uint32_t B_BYTES = BN * BK * 2;
  constexpr uint32_t TMEM_COLS = tmem_cols_for(BN);
  constexpr uint32_t ACC_STRIDE = TMEM_COLS / 2;  // column offset of the second accumulator
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t IDESC = idesc_f16(BM, BN, kBF16, false, !B_KMAJOR);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t{1023});
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sC = sB + STAGES * B_BYTES;   // kEpiWarps x kStageC output staging (1024-aligned)
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sC + kEpiWarps * kStageC);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* s_bias = reinterpret_cast<float*>(drain_bar + 2);  // [kEpiWarps][kBiasPerWarp] fp32

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tiles = (M + BM - 1) / BM;
  const int n_tiles = (N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int kblocks = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], kEpiWarps);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (warp == 0 && lane == 0 && static_cast<int>(blockIdx.x) < num_tiles) {
    // Before the predecessor has finished: descriptors, and the first ring's
    // worth of B (typically weights, cold after other work) into L2.
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
    const int n0 = (static_cast<int>(blockIdx.x) / m_tiles) * BN;
    for (int kb = 0; kb < kblocks && kb < STAGES; ++kb) {
      if constexpr (B_KMAJOR) {
        tma_prefetch_l2_2d(&tma_b, kb * BK, n0);
      } else {
#pragma unroll
        for (int j = 0; j < BN / 64; ++j) tma_prefetch_l2_2d(&tma_b, n0 + j * 64, kb * BK);
      }
    }
  }
  pdl_wait();
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------ TMA producer --
      uint32_t stage = 0, phase = 0, issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        const int m0 = (tile % m_tiles) * BM;
        const int n0 = (tile / m_tiles) * BN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, err, kErrGemmProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], A_BYTES + B_BYTES);
          tma_load_2d(sA + stage * A_BYTES, &tma_a, &full_bar[stage], kb * BK, m0);
          if constexpr (B_KMAJOR) {
            tma_load_2d(sB + stage * B_BYTES, &tma_b, &full_bar[stage], kb * BK, n0);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sB + stage * B_BYTES + j * (BK * 128), &tma_b, &full_bar[stage], n0 + j * 64, kb * BK);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let every load already issued land before the CTA can exit.
        const uint32_t first = issued > STAGES ? issued - STAGES : 0u;
        for (uint32_t i = first; i < issued; ++i)
          mbar_drain_wait(&full_bar[i % STAGES], (i / STAGES) & 1u, 1000000000ull);
      }
    }
  } else if (warp == 1) {
    {
      // ------------------------------------------------------- MMA issuer --
      // The whole warp runs the loop (every lane waits, the outcomes combined),
      // so its counters and descriptors stay warp-uniform; one elected lane
      // issues the MMAs and commits.
      const bool elected = elect_one_sync();
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        if (!mbar_wait_warp(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, err, kErrGemmMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * ACC_STRIDE;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_warp(&full_bar[stage], phase, abort_flag, err, kErrGemmMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
          uint64_t ad[BK / 16], bd[BK / 16];
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            ad[k] = sw128_desc(a_addr + k * 32, 16, 1024);
            bd[k] = B_KMAJOR ? sw128_desc(b_addr + k * 32, 16, 1024) : sw128_desc(b_addr + k * 2048, BK * 128, 1024);
          }
          if (elected) {
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) umma_f16_ss(d_tmem, ad[k], bd[k], IDESC, (kb | k) != 0 ? 1u : 0u);
            umma_commit(&empty_bar[stage]);
          }
          __syncwarp();
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (elected) umma_commit(&tfull_bar[acc]);
        __syncwarp();
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok) {
        // Wait for the MMAs already issued before TMEM is released.
        if (elected) umma_commit(drain_bar);
        __syncwarp();
        mbar_drain_wait(drain_bar, 0, 1000000000ull);
      }
    }
  } else {
    // ----------------------------------------------------------- epilogue --
    // Warps 2..13: warp & 3 is the TMEM lane quarter it may read (rows
    // 32*q .. 32*q+31 of the tile); (warp - 2) / 4 is its column slice.
    const int quarter = warp & 3;
    const int slice = (warp - 2) >> 2;
    float* sb = s_bias + (warp - 2) * kBiasPerWarp;
    uint8_t* s_stage = sC + (warp - 2) * kStageC;
    uint32_t acc = 0, acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int m0 = (tile % m_tiles) * BM;
      const int n0 = (tile / m_tiles) * BN;
      ResChunk res;
      if (slice < BN / 32) load_residual<T>(res, m0 + quarter * 32 + lane, n0 + slice * 32, ep);
      stage_bias<T, BN>(sb, n0, slice, ep, lane);
      __syncwarp();
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, err, kErrGemmEpilogue)) break;
      tc_fence_after();
      const uint32_t t_tile = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * ACC_STRIDE;
      epilogue_tile<T, BN, EPI>(t_tile, m0 + quarter * 32, n0, slice, sb, ep, &tma_c, s_stage, lane, res);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_group_all();   // output stores done before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------ CTA-pair (2-SM) tcgen05 ----
// Same roles as gemm_tc_kernel, on a cluster of two CTAs that computes
// 256 x BN output tiles with cta_group::2 MMAs (M=256, N=BN, K=16):
//   * each CTA's TMA warp loads its own 128 rows of A and its own BN/2 rows
//     (K-major) or columns (MN-major) of B -- no multicast -- and completes the
//     bytes on the even CTA's full barrier, which the even CTA's producer armed
//     with the pair's total;
//   * the even CTA's MMA thread issues the pair's MMAs and commits (multicast
//     to both CTAs) the smem-stage "empty" and the accumulator "full" barriers;
//   * each CTA's epilogue reads its 128 accumulator rows from its own TMEM and
//     arrives on the even CTA's accumulator "empty" barrier.
// Per CTA and K block this moves 16 KB of A + BN/2 x 128 B of B for half of a
// 256 x BN x 64 MMA: BN=256 halves the B traffic of the 1-CTA 128x256 tile.
__host__ __device__ constexpr int pair_stages(int bn) {
  return std::min(8, (kMaxDynSmem - kSmemReserve) / (BM * BK * 2 + (bn / 2) * BK * 2));
}

template <typename T, int BN, bool B_KMAJOR, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                    const __grid_constant__ CUtensorMap tma_c, const EpiParams ep, const int M, const int N, const int K, const int STAGES,
                    unsigned int* err) {
  constexpr int BH = BN / 2;                     // B rows (K-major) / columns (MN-major) per CTA
  static_assert(B_KMAJOR || BH % 64 == 0, "MN-major B halves are loaded as whole 64-column boxes");
  constexpr uint32_t A_BYTES = BM * BK * 2;
  constexpr uint32_t B_BYTES = BH * BK * 2;
  constexpr uint32_t TMEM_COLS = tmem_cols_for(BN);
  constexpr uint32_t ACC_STRIDE = TMEM_COLS / 2;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t IDESC = idesc_f16(2 * BM, BN, kBF16, false, !B_KMAJOR);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t{1023});
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sC = sB + STAGES * B_BYTES;   // kEpiWarps x kStageC output staging (1024-aligned)
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sC + kEpiWarps * kStageC);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* s_bias = reinterpret_cast<float*>(drain_bar + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster_id = static_cast<int>(blockIdx.x >> 1);
  const int num_clusters = static_cast<int>(gridDim.x >> 1);
  const int m_tiles = (M + 2 * BM - 1) / (2 * BM);
  const int n_tiles = (N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int kblocks = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 2 * kEpiWarps);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();   // barriers of both CTAs initialised before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (warp == 0 && lane == 0 && cluster_id < num_tiles) {
    // Before the predecessor has finished: descriptors, and this CTA's half of
    // the first ring's worth of B into L2.
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
    const int nb0 = (cluster_id / m_tiles) * BN + static_cast<int>(rank) * BH;
    for (int kb = 0; kb < kblocks && kb < STAGES; ++kb) {
      if constexpr (B_KMAJOR) {
        tma_prefetch_l2_2d(&tma_b, kb * BK, nb0);
      } else {
#pragma unroll
        for (int j = 0; j < BH / 64; ++j) tma_prefetch_l2_2d(&tma_b, nb0 + j * 64, kb * BK);
      }
    }
  }
  pdl_wait();
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------ TMA producer --
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int tile = cluster_id; ok && tile < num_tiles; tile += num_clusters) {
        const int m0 = (tile % m_tiles) * 2 * BM + static_cast<int>(rank) * BM;
        const int nb0 = (tile / m_tiles) * BN + static_cast<int>(rank) * BH;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, err, kErrGemmProducer)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * (A_BYTES + B_BYTES));
          const uint32_t leader_full = smem_u32(&full_bar[stage]) & kPeerBitMask;
          tma_load_2d_pair(sA + stage * A_BYTES, &tma_a, leader_full, kb * BK, m0);
          if constexpr (B_KMAJOR) {
            tma_load_2d_pair(sB + stage * B_BYTES, &tma_b, leader_full, kb * BK, nb0);
          } else {
#pragma unroll
            for (int j = 0; j < BH / 64; ++j)
              tma_load_2d_pair(sB + stage * B_BYTES + j * (BK * 128), &tma_b, leader_full, nb0 + j * 64, kb * BK);
          }
          if (++stage == static_cast<uint32_t>(STAGES)) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (ok) {
        // Producer tail: wait until the even CTA's MMA has released every stage
        // of this CTA once more, so no multicast commit can still be headed
        // for this CTA's barriers when it exits.
        for (int i = 0; ok && i < STAGES; ++i) {
          ok = mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, err, kErrGemmProducer);
          if (++stage == static_cast<uint32_t>(STAGES)) {
            stage = 0;
            phase ^= 1u;
          }
        }
      } else {
        // The loads complete on the even CTA's barrier; give those in flight time to land.
        const unsigned long long t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 200000ull) {
        }
      }
    }
  } else if (warp == 1) {
    if (leader) {
      // ------------------------------------------------ MMA issuer (pair) --
      // Warp-uniform loop, elected lane issues (as in the single-CTA kernel).
      const bool elected = elect_one_sync();
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool ok = true;
      for (int tile = cluster_id; ok && tile < num_tiles; tile += num_clusters) {
        if (!mbar_wait_warp(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, err, kErrGemmMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * ACC_STRIDE;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_warp(&full_bar[stage], phase, abort_flag, err, kErrGemmMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
          uint64_t ad[BK / 16], bd[BK / 16];
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            ad[k] = sw128_desc(a_addr + k * 32, 16, 1024);
            bd[k] = B_KMAJOR ? sw128_desc(b_addr + k * 32, 16, 1024) : sw128_desc(b_addr + k * 2048, BK * 128, 1024);
          }
          if (elected) {
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) umma_f16_ss_pair(d_tmem, ad[k], bd[k], IDESC, (kb | k) != 0 ? 1u : 0u);
            umma_commit_pair(&empty_bar[stage], 0x3);
          }
          __syncwarp();
          if (++stage == static_cast<uint32_t>(STAGES)) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (elected) umma_commit_pair(&tfull_bar[acc], 0x3);
        __syncwarp();
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok) {
        if (elected) umma_commit_pair(drain_bar, 0x1);
        __syncwarp();
        mbar_drain_wait(drain_bar, 0, 1000000000ull);
      }
    }
  } else {
    // ----------------------------------------------------------- epilogue --
    const int quarter = warp & 3;
    const int slice = (warp - 2) >> 2;
    const uint32_t leader_tempty = smem_u32(tempty_bar) & kPeerBitMask;
    float* sb = s_bias + (warp - 2) * kBiasPerWarp;
    uint8_t* s_stage = sC + (warp - 2) * kStageC;
    uint32_t acc = 0, acc_phase = 0;
    for (int tile = cluster_id; tile < num_tiles; tile += num_clusters) {
      const int m0 = (tile % m_tiles) * 2 * BM + static_cast<int>(rank) * BM;
      const int n0 = (tile / m_tiles) * BN;
      ResChunk res;
      if (slice < BN / 32) load_residual<T>(res, m0 + quarter * 32 + lane, n0 + slice * 32, ep);
      stage_bias<T, BN>(sb, n0, slice, ep, lane);
      __syncwarp();
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, err, kErrGemmEpilogue)) break;
      tc_fence_after();
      const uint32_t t_tile = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * ACC_STRIDE;
      epilogue_tile<T, BN, EPI>(t_tile, m0 + quarter * 32, n0, slice, sb, ep, &tma_c, s_stage, lane, res);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(leader_tempty + acc * 8);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_group_all();   // output stores done before the CTA exits
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync();   // neither CTA leaves while the pair's MMAs, TMA bytes or arrivals may target it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------ SIMT path ----
constexpr int ST = 64;   // output tile
constexpr int SK = 16;   // K step

template <typename T>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const T* __restrict__ A, const T* __restrict__ B,
                                                        const EpiParams ep, int64_t K, int64_t lda, int64_t ldb,
                                                        int b_layout) {
  __shared__ float As[SK][ST + 1];
  __shared__ float Bs[SK][ST + 1];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * ST, n0 = static_cast<int64_t>(blockIdx.x) * ST;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += SK) {
    for (int i = threadIdx.x; i < SK * ST; i += 256) {
      const int kk = i % SK, mm = i / SK;
      const int64_t gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < ep.M && gk < K) ? Io<T>::to_f(A[gm * lda + gk]) : 0.f;
      const int nn = i % ST, kb = i / ST;
      const int64_t gn = n0 + nn, gk2 = k0 + kb;
      float bval = 0.f;
      if (gn < ep.N && gk2 < K)
        bval = Io<T>::to_f(b_layout == LUNARA_B_KN ? B[gk2 * ldb + gn] : B[gn * ldb + gk2]);
      Bs[kb][nn] = bval;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
  const T* bias = static_cast<const T*>(ep.bias);
  const T* res = static_cast<const T*>(ep.residual);
  T* C = static_cast<T*>(ep.C);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t gm = m0 + ty * 4 + i;
    if (gm >= ep.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t gn = n0 + tx * 4 + j;
      if (gn >= ep.N) continue;
      float v = acc[i][j];
      if (bias) v += Io<T>::to_f(bias[gn]);
      v = apply_act(v, ep.act);
      if (res) v += Io<T>::to_f(res[gm * ep.ldr + gn]);
      C[gm * ep.ldc + gn] = Io<T>::from_f(v);
    }
  }
}

// ------------------------------------------------------------ host side ----
bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

EpiParams make_epi(const GemmArgs& g) {
  EpiParams ep{};
  ep.C = g.C;
  ep.bias = g.bias;
  ep.residual = g.residual;
  ep.ldc = g.ldc;
  ep.ldr = g.ldr;
  ep.M = static_cast<int>(g.M);
  ep.N = static_cast<int>(g.N);
  ep.act = g.act;
  ep.vec_ok = al16(g.C) && (g.ldc % 8 == 0) && (g.bias == nullptr || al16(g.bias)) &&
              (g.residual == nullptr || (al16(g.residual) && g.ldr % 8 == 0));
  ep.tma_store = 0;
  return ep;
}

bool encode_2d(CUtensorMap* map, const void* base, int dtype, uint64_t inner, uint64_t outer, uint64_t stride_bytes,
               uint32_t box_inner, uint32_t box_outer,
               CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(tensor_map_encoder());
  if (encode == nullptr) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt =
      dtype == LUNARA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Cost model used to pick the kernel when the caller does not: per-CTA
// cycles of one 64-deep K block are bounded by the tensor pipe (2*BN for both
// the 128-row and the 256-row pair MMA) and by the operand bytes each CTA must
// pull from L2 (about 60 B/cycle/SM sustained when every SM streams); tiles
// are handed out in rounds over the persistent CTAs (pairs). A CTA pair pays a
// further ~3200 cycles per tile (cross-CTA barriers, cluster synchronisation,
// the pair's epilogue hand-off): fitted to a sweep of 12 shapes on B200
// (block, 12-layer-stack and square GEMMs), where, with the one-round rate
// below, it picks the fastest plan or one within 2% for every shape
// (single-CTA 128x192 tiles for N=768 outputs of 4096 rows at K=768, 256x192
// CTA pairs at K=3072, CTA pairs for wide N and for many rounds).
struct GemmPlan {
  int block_n;
  bool pair;
};

double gemm_cost(int64_t M, int64_t N, int64_t K, GemmPlan p, int sms) {
  const int tile_m = p.pair ? 2 * BM : BM;
  const int64_t tiles = ceil_div64(M, tile_m) * ceil_div64(N, p.block_n);
  const int64_t units = p.pair ? sms / 2 : sms;
  const int64_t rounds = ceil_div64(tiles, units);
  // Tiles that all fit in one round stream their operands at a higher rate
  // than the all-SMs-busy figure (measured: single-CTA 4096x768 at K=768 and
  // K=3072, 2048^3; CTA pairs with a 5-stage ring, 4096x768 at K=3072), so they
  // are costed at 80 B/cycle instead of 60.
  const double l2_bytes_per_cycle = (rounds == 1) ? 80.0 : 60.0;
  const double bytes = BM * BK * 2.0 + (p.pair ? p.block_n / 2 : p.block_n) * BK * 2.0;
  const double per_kb = std::max(2.0 * p.block_n, bytes / l2_bytes_per_cycle);
  return static_cast<double>(rounds) * (static_cast<double>(ceil_div64(K, BK)) * per_kb + (p.pair ? 3200.0 : 0.0));
}

GemmPlan choose_plan(int64_t M, int64_t N, int64_t K, int sms, int block_n, int cta_pair, bool b_kmajor) {
  static const GemmPlan kChoices[] = {{256, true}, {192, true}, {128, true}, {256, false}, {192, false},
                                      {128, false}, {64, false}};
  GemmPlan best{256, true};
  double best_cost = 1e300;
  for (const GemmPlan& c : kChoices) {
    if (block_n != 0 && c.block_n != block_n) continue;
    if (cta_pair == 1 && c.pair) continue;
    if (cta_pair == 2 && !c.pair) continue;
    if (c.pair && c.block_n == 192 && !b_kmajor) continue;   // MN-major halves must be whole 64-column boxes
    const double cost = gemm_cost(M, N, K, c, sms);
    if (cost < best_cost * 0.999) {
      best_cost = cost;
      best = c;
    }
  }
  return best;
}

template <typename T, int BN, bool B_KMAJOR, int EPI>
cudaError_t run_tc(const GemmArgs& g, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc,
                   const EpiParams& ep, cudaStream_t s) {
  auto kern = gemm_tc_kernel<T, BN, B_KMAJOR, EPI>;
  constexpr int kMaxStages = gemm_stages(BN);
  static_assert(gemm_smem_bytes(BN, kMaxStages) <= kMaxDynSmem, "shared memory budget");
  const int stages = (g.stages >= 2 && g.stages <= kMaxStages) ? g.stages : kMaxStages;
  const int smem = gemm_smem_bytes(BN, stages);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       gemm_smem_bytes(BN, kMaxStages));
  if (e != cudaSuccess) return e;
  const int sms = device_num_sms();
  const int64_t tiles = ceil_div64(g.M, BM) * ceil_div64(g.N, BN);
  int64_t grid = g.num_ctas > 0 ? g.num_ctas : sms;
  if (grid > tiles) grid = tiles;
  unsigned int* err = device_error_word();
  if (err == nullptr) return cudaErrorInvalidDevice;
  return launch_pdl(kern, dim3(static_cast<unsigned>(grid)), dim3(kGemmThreads), static_cast<size_t>(smem), s, ma, mb,
                    mc, ep, static_cast<int>(g.M), static_cast<int>(g.N), static_cast<int>(g.K), stages, err);
}

template <typename T, int BN, bool B_KMAJOR, int EPI>
cudaError_t run_tc2(const GemmArgs& g, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc,
                    const EpiParams& ep, cudaStream_t s) {
  auto kern = gemm_tc2_kernel<T, BN, B_KMAJOR, EPI>;
  constexpr int kMaxStages = pair_stages(BN);
  constexpr int kStageBytes = BM * BK * 2 + (BN / 2) * BK * 2;
  static_assert(kMaxStages * kStageBytes + kSmemReserve <= kMaxDynSmem, "shared memory budget");
  // Default ring depth: the deepest that fits, except for 192-wide tiles, where
  // 5 stages measured fastest on B200 of the 3 to 7 that fit (4096 x 768
  // outputs; K = 3072 inside the encoder block step: 98.1 / 95.2 / 95.3 / 95.3 us
  // with 4 / 5 / 6 / 7 stages; K = 768 alone with cold operands: 11.8 / 11.3 /
  // 12.0 us with 4 / 5 / 7).
  constexpr int kDefaultStages = (BN == 192 && kMaxStages > 5) ? 5 : kMaxStages;
  const int stages = (g.stages >= 2 && g.stages <= kMaxStages) ? g.stages : kDefaultStages;
  const int smem = stages * kStageBytes + kSmemReserve;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kMaxStages * kStageBytes + kSmemReserve);
  if (e != cudaSuccess) return e;
  // Persistent grid: as many CTA pairs as can be resident (clusters of two
  // need both SMs of a pair free), capped by the number of 256-row tiles. The
  // occupancy query depends on the shared-memory size, so its answer is cached
  // per device and ring depth, under a lock.
  static std::mutex cache_mu;
  static int cached_clusters[64][9] = {};   // [device][stages], for this kernel instantiation
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
  int max_clusters = device_num_sms() / 2;
  const bool cacheable = dev >= 0 && dev < 64 && stages >= 0 && stages < 9;
  int cached = 0;
  if (cacheable) {
    std::lock_guard<std::mutex> lk(cache_mu);
    cached = cached_clusters[dev][stages];
  }
  if (cached > 0) {
    max_clusters = cached;
  } else {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(2 * max_clusters));
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = s;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0 && n < max_clusters)
      max_clusters = n;
    cudaGetLastError();
    if (cacheable) {
      std::lock_guard<std::mutex> lk(cache_mu);
      cached_clusters[dev][stages] = max_clusters;
    }
  }
  const int64_t tiles = ceil_div64(g.M, 2 * BM) * ceil_div64(g.N, BN);
  int64_t clusters = g.num_ctas > 1 ? g.num_ctas / 2 : max_clusters;
  if (clusters > tiles) clusters = tiles;
  if (clusters < 1) clusters = 1;
  unsigned int* err = device_error_word();
  if (err == nullptr) return cudaErrorInvalidDevice;
  return launch_pdl(kern, dim3(static_cast<unsigned>(2 * clusters)), dim3(kGemmThreads), static_cast<size_t>(smem), s,
                    ma, mb, mc, ep, static_cast<int>(g.M), static_cast<int>(g.N), static_cast<int>(g.K), stages,
                    err);
}

template <typename T, bool B_KMAJOR, int EPI>
cudaError_t dispatch_epi(const GemmArgs& g, GemmPlan plan, const CUtensorMap& ma, const CUtensorMap& mb,
                         const CUtensorMap& mc, const EpiParams& ep, cudaStream_t s) {
  if (plan.pair) {
    if (plan.block_n == 128) return run_tc2<T, 128, B_KMAJOR, EPI>(g, ma, mb, mc, ep, s);
    if constexpr (B_KMAJOR) {
      if (plan.block_n == 192) return run_tc2<T, 192, B_KMAJOR, EPI>(g, ma, mb, mc, ep, s);
    }
    return run_tc2<T, 256, B_KMAJOR, EPI>(g, ma, mb, mc, ep, s);
  }
  switch (plan.block_n) {
    case 64: return run_tc<T, 64, B_KMAJOR, EPI>(g, ma, mb, mc, ep, s);
    case 128: return run_tc<T, 128, B_KMAJOR, EPI>(g, ma, mb, mc, ep, s);
    case 192: return run_tc<T, 192, B_KMAJOR, EPI>(g, ma, mb, mc, ep, s);
    default: return run_tc<T, 256, B_KMAJOR, EPI>(g, ma, mb, mc, ep, s);
  }
}

template <typename T, bool B_KMAJOR>
cudaError_t dispatch_plan(const GemmArgs& g, GemmPlan plan, cudaStream_t s) {
  CUtensorMap ma, mb;
  // B rows (K-major) or columns (MN-major) loaded by one CTA per K block.
  const int b_box = plan.pair ? plan.block_n / 2 : plan.block_n;
  if (!encode_2d(&ma, g.A, g.dtype, g.K, g.M, g.lda * 2, BK, BM)) return cudaErrorInvalidValue;
  const bool ok_b = B_KMAJOR ? encode_2d(&mb, g.B, g.dtype, g.K, g.N, g.ldb * 2, BK, b_box)
                             : encode_2d(&mb, g.B, g.dtype, g.N, g.K, g.ldb * 2, 64, BK);
  if (!ok_b) return cudaErrorInvalidValue;
  // Output through TMA stores of 32 x 32 chunks (64-byte swizzle) when C allows
  // 16-byte accesses; otherwise each thread stores its row directly.
  EpiParams ep = make_epi(g);
  CUtensorMap mc;
  std::memset(&mc, 0, sizeof(mc));
  if (ep.vec_ok && encode_2d(&mc, g.C, g.dtype, g.N, g.M, g.ldc * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
    ep.tma_store = 1;
  switch (epi_mode_for(g.act)) {
    case kEpiPlain: return dispatch_epi<T, B_KMAJOR, kEpiPlain>(g, plan, ma, mb, mc, ep, s);
    case kEpiGeluTanh: return dispatch_epi<T, B_KMAJOR, kEpiGeluTanh>(g, plan, ma, mb, mc, ep, s);
    default: return dispatch_epi<T, B_KMAJOR, kEpiAnyAct>(g, plan, ma, mb, mc, ep, s);
  }
}


// ------------------------------------------- GEMM + residual + LayerNorm ----
// Y = LayerNorm(A * B + bias + residual) * gamma + beta over rows of N = G * BN
// columns, each row split over a cluster of G CTAs (2 <= G <= 8): CTA r of a
// cluster computes columns [r * BN, (r + 1) * BN) of the same 128 rows with the
// single-CTA main loop above (TMA warp, MMA thread, two TMEM accumulators), and
// the cluster loops persistently over 128-row blocks. The epilogue warps
//   1. read their 32-column chunks from TMEM, add bias and residual in fp32
//      and round once to the output type -- the value the unfused GEMM would
//      store for the LayerNorm to read -- keeping the rounded row segment
//      packed in registers, then hand the accumulator back;
//   2. take the mean and M2 (sum of squared deviations) of their row segment
//      (exact two-pass over the registers), write that pair into the row's
//      slot of the CTA's statistics buffer, and send the warp's 32 pairs
//      (256 bytes) to the same slot of every other CTA of the cluster with one
//      bulk copy each, which completes its bytes on the receiving CTA's
//      statistics barrier (36 barrier updates per CTA for G = 4, where one
//      8-byte store per row and CTA took 1536 and cost as much as a
//      separate LayerNorm kernel);
//   3. once all 3 * G pairs of the block have arrived, combine them (Chan et
//      al.'s pairwise update with known counts) into the row's mean and
//      population variance over N, normalise, scale by gamma, add beta, round
//      once and write the output chunk with a TMA store.
// No intermediate [M, N] tensor is written or read back. Statistics buffers
// alternate with the block parity: a CTA can send block t+2's pairs only after
// every CTA of the cluster has sent its block t+1 pairs, which each warp does
// only after reading its block t pairs, so a buffer is never overwritten while
// it is read. Every CTA of a cluster passes a final cluster barrier before it
// exits, so no st.async can target the shared memory of a CTA that has left.
struct LnParams {
  const void* gamma;
  const void* beta;
  float eps;
};

__host__ __device__ constexpr int ln_reserve(int G) {
  return 1024 + kEpiWarps * kStageC + 2 * 3 * G * BM * 8 + 512 + kEpiWarps * 3 * kBiasPerWarp * 4;
}

constexpr int ln_stage_bytes(int bn) { return BM * BK * 2 + bn * BK * 2; }

constexpr int ln_max_stages(int bn, int G) {
  return std::min(8, (kMaxDynSmem - ln_reserve(G)) / ln_stage_bytes(bn));
}

template <typename T, int BN, bool B_KMAJOR>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_ln_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                   const __grid_constant__ CUtensorMap tma_c, const EpiParams ep, const LnParams ln, const int M,
                   const int K, const int STAGES, unsigned int* err) {
  constexpr uint32_t A_BYTES = BM * BK * 2;
  constexpr uint32_t B_BYTES = BN * BK * 2;
  constexpr uint32_t TMEM_COLS = tmem_cols_for(BN);
  constexpr uint32_t ACC_STRIDE = TMEM_COLS / 2;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t IDESC = idesc_f16(BM, BN, kBF16, false, !B_KMAJOR);
  constexpr int kChunks = BN / 32;
  constexpr int kWarpChunks = (kChunks + kEpiSlices - 1) / kEpiSlices;   // most chunks one warp owns
  static_assert(kChunks >= kEpiSlices && kWarpChunks <= kMaxWarpChunks, "every epilogue warp owns a chunk");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t{1023});
  const uint32_t G = cluster_nctarank();
  const uint32_t rank = cluster_ctarank();
  const int nslots = 3 * static_cast<int>(G);
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * A_BYTES;
  uint8_t* sC = sB + STAGES * B_BYTES;                                       // kEpiWarps x kStageC
  float2* s_stats = reinterpret_cast<float2*>(sC + kEpiWarps * kStageC);    // [2][nslots][BM] (mean, M2)
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(s_stats + 2 * nslots * BM);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint64_t* stats_bar = drain_bar + 1;                                      // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(stats_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* s_vec = reinterpret_cast<float*>(stats_bar + 4);   // [kEpiWarps][bias | gamma | beta][kBiasPerWarp]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cid = static_cast<int>(cluster_id_x());
  const int ncl = static_cast<int>(nclusters_x());
  const int m_tiles = (M + BM - 1) / BM;
  const int kblocks = (K + BK - 1) / BK;
  const int n0 = static_cast<int>(rank) * BN;
  const int N = static_cast<int>(G) * BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], kEpiWarps);
      mbar_init(&stats_bar[a], kEpiThreads);   // every epilogue thread, after writing its local pair
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  cluster_sync();   // every CTA's statistics barriers are initialised before any st.async targets them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (warp == 0 && lane == 0 && cid < m_tiles) {
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
    for (int kb = 0; kb < kblocks && kb < STAGES; ++kb) {
      if constexpr (B_KMAJOR) {
        tma_prefetch_l2_2d(&tma_b, kb * BK, n0);
      } else {
#pragma unroll
        for (int j = 0; j < BN / 64; ++j) tma_prefetch_l2_2d(&tma_b, n0 + j * 64, kb * BK);
      }
    }
  }
  pdl_wait();
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------ TMA producer --
      uint32_t stage = 0, phase = 0, issued = 0;
      bool ok = true;
      for (int tile = cid; ok && tile < m_tiles; tile += ncl) {
        const int m0 = tile * BM;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, err, kErrGemmProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], A_BYTES + B_BYTES);
          tma_load_2d(sA + stage * A_BYTES, &tma_a, &full_bar[stage], kb * BK, m0);
          if constexpr (B_KMAJOR) {
            tma_load_2d(sB + stage * B_BYTES, &tma_b, &full_bar[stage], kb * BK, n0);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sB + stage * B_BYTES + j * (BK * 128), &tma_b, &full_bar[stage], n0 + j * 64, kb * BK);
          }
          ++issued;
          if (++stage == static_cast<uint32_t>(STAGES)) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        const uint32_t first = issued > static_cast<uint32_t>(STAGES) ? issued - STAGES : 0u;
        for (uint32_t i = first; i < issued; ++i)
          mbar_drain_wait(&full_bar[i % STAGES], (i / STAGES) & 1u, 1000000000ull);
      }
    }
  } else if (warp == 1) {
    {
      // ------------------------------------------------------- MMA issuer --
      // The whole warp runs the loop (every lane waits, the outcomes combined),
      // so its counters and descriptors stay warp-uniform; one elected lane
      // issues the MMAs and commits.
      const bool elected = elect_one_sync();
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool ok = true;
      for (int tile = cid; ok && tile < m_tiles; tile += ncl) {
        if (!mbar_wait_warp(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, err, kErrGemmMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * ACC_STRIDE;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_warp(&full_bar[stage], phase, abort_flag, err, kErrGemmMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
          uint64_t ad[BK / 16], bd[BK / 16];
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            ad[k] = sw128_desc(a_addr + k * 32, 16, 1024);
            bd[k] = B_KMAJOR ? sw128_desc(b_addr + k * 32, 16, 1024) : sw128_desc(b_addr + k * 2048, BK * 128, 1024);
          }
          if (elected) {
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) umma_f16_ss(d_tmem, ad[k], bd[k], IDESC, (kb | k) != 0 ? 1u : 0u);
            umma_commit(&empty_bar[stage]);
          }
          __syncwarp();
          if (++stage == static_cast<uint32_t>(STAGES)) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (elected) umma_commit(&tfull_bar[acc]);
        __syncwarp();
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok) {
        if (elected) umma_commit(drain_bar);
        __syncwarp();
        mbar_drain_wait(drain_bar, 0, 1000000000ull);
      }
    }
  } else {
    // ----------------------------------------------------------- epilogue --
    // Warps 2..13: warp & 3 is the TMEM lane quarter (rows 32q .. 32q+31 of the
    // block), (warp - 2) / 4 the column slice: chunks slice, slice + 3, ...
    const int quarter = warp & 3;
    const int slice = (warp - 2) >> 2;
    const int row_t = quarter * 32 + lane;
    float* sv = s_vec + (warp - 2) * 3 * kBiasPerWarp;
    uint8_t* s_stage = sC + (warp - 2) * kStageC;
    // Bias, gamma and beta of this warp's columns: the same for every block.
#pragma unroll
    for (int j = 0; j < kWarpChunks; ++j) {
      const int c = slice + j * kEpiSlices;
      if (c >= kChunks) break;
      const int col = n0 + c * 32 + lane;
      sv[j * 32 + lane] = ep.bias != nullptr ? Io<T>::to_f(static_cast<const T*>(ep.bias)[col]) : 0.f;
      sv[kBiasPerWarp + j * 32 + lane] = Io<T>::to_f(static_cast<const T*>(ln.gamma)[col]);
      sv[2 * kBiasPerWarp + j * 32 + lane] = Io<T>::to_f(static_cast<const T*>(ln.beta)[col]);
    }
    __syncwarp();
    const int my_chunks = (kChunks - slice + kEpiSlices - 1) / kEpiSlices;
    const float inv_mine = 1.0f / static_cast<float>(my_chunks * 32);
    const float inv_n = 1.0f / static_cast<float>(N);
    uint32_t acc = 0, acc_phase = 0;
    int it = 0;
    for (int tile = cid; tile < m_tiles; tile += ncl, ++it) {
      const int m0 = tile * BM;
      const int row = m0 + row_t;
      ResChunk res;
      load_residual<T>(res, row, n0 + slice * 32, ep);
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, err, kErrGemmEpilogue)) break;
      tc_fence_after();
      const uint32_t t_tile = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * ACC_STRIDE;
      // 1. acc + bias + residual, rounded once, packed in registers.
      uint32_t pk[kWarpChunks][16];
      float sum0 = 0.f, sum1 = 0.f;
      uint32_t v[32];
      tmem_ld_32x32b_x32(t_tile + slice * 32, v);
#pragma unroll
      for (int j = 0; j < kWarpChunks; ++j) {
        const int c = slice + j * kEpiSlices;
        if (c >= kChunks) break;
        tmem_ld_wait_regs(v);
        epilogue_pack<T, kEpiPlain>(v, row, n0 + c * 32, sv + j * 32, res, ep, pk[j]);
        if (c + kEpiSlices < kChunks) {
          tmem_ld_32x32b_x32(t_tile + (c + kEpiSlices) * 32, v);
          load_residual<T>(res, row, n0 + (c + kEpiSlices) * 32, ep);
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 f = Io<T>::unpack2(pk[j][i]);
          sum0 += f.x;
          sum1 += f.y;
        }
      }
      // The accumulator is in registers: hand the TMEM buffer back to the MMA thread.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
      // 2. This segment's mean and M2, sent to slot (rank, slice) of every CTA.
      const float mean_l = (sum0 + sum1) * inv_mine;
      float m2v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < kWarpChunks; ++j) {
        if (slice + j * kEpiSlices >= kChunks) break;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 f = Io<T>::unpack2(pk[j][i]);
          const float da = f.x - mean_l, db = f.y - mean_l;
          m2v[(2 * i) & 3] = fmaf(da, da, m2v[(2 * i) & 3]);
          m2v[(2 * i + 1) & 3] = fmaf(db, db, m2v[(2 * i + 1) & 3]);
        }
      }
      const int b = it & 1;
      const uint32_t bphase = static_cast<uint32_t>(it >> 1) & 1u;
      float2* seg = &s_stats[(b * nslots + static_cast<int>(rank) * kEpiSlices + slice) * BM + quarter * 32];
      seg[lane] = make_float2(mean_l, (m2v[0] + m2v[1]) + (m2v[2] + m2v[3]));
      fence_proxy_async_smem();   // the pairs are visible to the bulk copies below
      __syncwarp();
      if (warp == 2 && lane == 0)
        mbar_expect_tx(&stats_bar[b], (G - 1u) * static_cast<uint32_t>(kEpiWarps * 32 * 8));
      mbar_arrive(&stats_bar[b]);
      if (lane == 0) {
        const uint32_t src = smem_u32(seg);
        const uint32_t bar_addr = smem_u32(&stats_bar[b]);
        for (uint32_t r = 0; r < G; ++r)
          if (r != rank) bulk_copy_to_cluster(mapa_shared(src, r), src, 32 * 8, mapa_shared(bar_addr, r));
      }
      if (!mbar_wait_cluster(&stats_bar[b], bphase, abort_flag, err, kErrGemmEpilogue)) break;
      // 3. Row statistics over all N columns, then normalise and store.
      const float2* st = s_stats + b * nslots * BM + row_t;
      float wsum = 0.f;
      for (int sl = 0; sl < nslots; ++sl) {
        const int cnt = 32 * ((kChunks - (sl % kEpiSlices) + kEpiSlices - 1) / kEpiSlices);
        wsum = fmaf(static_cast<float>(cnt), st[sl * BM].x, wsum);
      }
      const float mean = wsum * inv_n;
      float m2 = 0.f;
      for (int sl = 0; sl < nslots; ++sl) {
        const int cnt = 32 * ((kChunks - (sl % kEpiSlices) + kEpiSlices - 1) / kEpiSlices);
        const float2 pr = st[sl * BM];
        const float d = pr.x - mean;
        m2 += pr.y + static_cast<float>(cnt) * d * d;
      }
      const float rstd = rsqrtf(m2 * inv_n + ln.eps);
#pragma unroll
      for (int j = 0; j < kWarpChunks; ++j) {
        const int c = slice + j * kEpiSlices;
        if (c >= kChunks) break;
        const float* g = sv + kBiasPerWarp + j * 32;
        const float* be = sv + 2 * kBiasPerWarp + j * 32;
        uint32_t out[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 f = Io<T>::unpack2(pk[j][i]);
          out[i] = Io<T>::pack2(fmaf((f.x - mean) * rstd, g[2 * i], be[2 * i]),
                                fmaf((f.y - mean) * rstd, g[2 * i + 1], be[2 * i + 1]));
        }
        store_chunk_tma(out, n0 + c * 32, m0 + quarter * 32, &tma_c, s_stage, lane);
      }
    }
    if (lane == 0) bulk_wait_group_all();   // output stores done before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
  cluster_sync();   // no CTA leaves while a peer may still send statistics into its shared memory
}

template <typename T, int BN, bool B_KMAJOR>
cudaError_t run_ln(const GemmArgs& g, const LnParams& ln, int G, const CUtensorMap& ma, const CUtensorMap& mb,
                   const CUtensorMap& mc, const EpiParams& ep, cudaStream_t s) {
  auto kern = gemm_ln_kernel<T, BN, B_KMAJOR>;
  const int max_stages = ln_max_stages(BN, G);
  if (max_stages < 2) return cudaErrorInvalidConfiguration;
  const int stages = (g.stages >= 2 && g.stages <= max_stages) ? g.stages : std::min(4, max_stages);
  const int smem = stages * ln_stage_bytes(BN) + ln_reserve(G);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem);
  if (e != cudaSuccess) return e;
  // Persistent grid: as many clusters of G as can be resident, cached per
  // (device, G, stages) under a lock; never more clusters than row blocks.
  static std::mutex cache_mu;
  static int cached[64][9][9] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
  const bool cacheable = dev >= 0 && dev < 64;
  int max_clusters = 0;
  if (cacheable) {
    std::lock_guard<std::mutex> lk(cache_mu);
    max_clusters = cached[dev][G][stages];
  }
  if (max_clusters == 0) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(G);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(G * (device_num_sms() / G)));
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      return cudaErrorInvalidConfiguration;
    }
    max_clusters = n;
    if (cacheable) {
      std::lock_guard<std::mutex> lk(cache_mu);
      cached[dev][G][stages] = max_clusters;
    }
  }
  const int64_t m_tiles = ceil_div64(g.M, BM);
  int64_t clusters = g.num_ctas >= G ? g.num_ctas / G : max_clusters;
  if (clusters > max_clusters) clusters = max_clusters;
  if (clusters > m_tiles) clusters = m_tiles;
  if (clusters < 1) clusters = 1;
  unsigned int* err = device_error_word();
  if (err == nullptr) return cudaErrorInvalidDevice;
  return launch_pdl_cluster(kern, dim3(static_cast<unsigned>(clusters * G)), dim3(kGemmThreads),
                            static_cast<unsigned>(G), static_cast<size_t>(smem), s, ma, mb, mc, ep, ln,
                            static_cast<int>(g.M), static_cast<int>(g.K), stages, err);
}

template <typename T, bool B_KMAJOR>
cudaError_t dispatch_ln(const GemmArgs& g, const LnParams& ln, int bn, cudaStream_t s) {
  const int G = static_cast<int>(g.N / bn);
  CUtensorMap ma, mb, mc;
  if (!encode_2d(&ma, g.A, g.dtype, g.K, g.M, g.lda * 2, BK, BM)) return cudaErrorInvalidValue;
  const bool ok_b = B_KMAJOR ? encode_2d(&mb, g.B, g.dtype, g.K, g.N, g.ldb * 2, BK, bn)
                             : encode_2d(&mb, g.B, g.dtype, g.N, g.K, g.ldb * 2, 64, BK);
  if (!ok_b) return cudaErrorInvalidValue;
  EpiParams ep = make_epi(g);
  if (!encode_2d(&mc, g.C, g.dtype, g.N, g.M, g.ldc * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
    return cudaErrorInvalidValue;
  ep.tma_store = 1;
  switch (bn) {
    case 128: return run_ln<T, 128, B_KMAJOR>(g, ln, G, ma, mb, mc, ep, s);
    case 192: return run_ln<T, 192, B_KMAJOR>(g, ln, G, ma, mb, mc, ep, s);
    default: return run_ln<T, 256, B_KMAJOR>(g, ln, G, ma, mb, mc, ep, s);
  }
}

}  // namespace

bool gemm_tc_supported(const GemmArgs& g) {
  if (g.dtype != LUNARA_F16 && g.dtype != LUNARA_BF16) return false;
  if (g.M < 1 || g.N < 1 || g.K < 1) return false;
  if (g.M >= (int64_t{1} << 31) || g.N >= (int64_t{1} << 31) || g.K >= (int64_t{1} << 31)) return false;
  if (!al16(g.A) || !al16(g.B)) return false;
  if (g.lda % 8 != 0 || g.ldb % 8 != 0) return false;
  return true;
}

cudaError_t launch_gemm_tcgen05(const GemmArgs& g, cudaStream_t stream) {
  // Requested tile: block_n in {64,128,192,256} (pairs take 128 or 256), cta_pair 1 = single CTA, 2 = pair.
  int bn = g.block_n;
  if (bn != 64 && bn != 128 && bn != 192 && bn != 256) bn = 0;
  int pair = g.cta_pair;
  const bool kmajor = g.b_layout == LUNARA_B_NK;
  if (bn == 64 || (bn == 192 && !kmajor)) pair = 1;
  const GemmPlan plan = choose_plan(g.M, g.N, g.K, device_num_sms(), bn, pair, kmajor);
  if (g.dtype == LUNARA_BF16)
    return kmajor ? dispatch_plan<__nv_bfloat16, true>(g, plan, stream)
                  : dispatch_plan<__nv_bfloat16, false>(g, plan, stream);
  return kmajor ? dispatch_plan<__half, true>(g, plan, stream) : dispatch_plan<__half, false>(g, plan, stream);
}

cudaError_t launch_gemm_simt(const GemmArgs& g, cudaStream_t stream) {
  if (g.M == 0 || g.N == 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>(ceil_div64(g.N, ST)), static_cast<unsigned>(ceil_div64(g.M, ST)));
  const EpiParams ep = make_epi(g);
  switch (g.dtype) {
    case LUNARA_F16:
      gemm_simt_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<const __half*>(g.A),
                                                         static_cast<const __half*>(g.B), ep, g.K, g.lda, g.ldb,
                                                         g.b_layout);
      break;
    case LUNARA_BF16:
      gemm_simt_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(g.A),
                                                                static_cast<const __nv_bfloat16*>(g.B), ep, g.K,
                                                                g.lda, g.ldb, g.b_layout);
      break;
    default:
      gemm_simt_kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float*>(g.A),
                                                        static_cast<const float*>(g.B), ep, g.K, g.lda, g.ldb,
                                                        g.b_layout);
      break;
  }
  return cudaGetLastError();
}

}  // namespace lunara

namespace lunara {

int gemm_ln_block_n(int64_t N, int requested) {
  // Column slice per CTA: the requested one when it divides N into 2..8 slices,
  // else 192, 256, 128 in that order of preference (192 gives the 4-CTA
  // clusters that cover 768 columns with one 128 x 192 tile per CTA).
  const int pref[4] = {requested, 192, 256, 128};
  for (int bn : pref) {
    if (bn != 128 && bn != 192 && bn != 256) continue;
    if (N % bn == 0 && N / bn >= 2 && N / bn <= 8) return bn;
  }
  return 0;
}

bool gemm_ln_supported(const GemmArgs& g, const void* gamma, const void* beta) {
  if (g.dtype != LUNARA_F16 && g.dtype != LUNARA_BF16) return false;
  if (g.act != LUNARA_ACT_NONE) return false;
  if (!gemm_tc_supported(g)) return false;
  if (gemm_ln_block_n(g.N, g.block_n) == 0) return false;
  const EpiParams ep = make_epi(g);
  if (!ep.vec_ok) return false;
  return al16(gamma) && al16(beta);
}

cudaError_t launch_gemm_layernorm(const GemmArgs& g, const void* gamma, const void* beta, float eps,
                                  cudaStream_t stream) {
  LnParams ln{gamma, beta, eps};
  const int bn = gemm_ln_block_n(g.N, g.block_n);
  const bool kmajor = g.b_layout == LUNARA_B_NK;
  if (g.dtype == LUNARA_BF16)
    return kmajor ? dispatch_ln<__nv_bfloat16, true>(g, ln, bn, stream)
                  : dispatch_ln<__nv_bfloat16, false>(g, ln, bn, stream);
  return kmajor ? dispatch_ln<__half, true>(g, ln, bn, stream) : dispatch_ln<__half, false>(g, ln, bn, stream);
}

}  // namespace lunara
