// Scaled-dot-product attention forward, O = softmax(Q K^T * scale [+ causal]) V.
//
// tcgen05 path (f16 / bf16, D == 64): FlashAttention-style single pass with an
// online softmax. One CTA owns one 128-row Q tile of one (batch, head); its two
// halves split the key blocks (half 0 takes blocks 0, 2, 4, ..., half 1 takes
// 1, 3, 5, ...), each keeping its own running max, row sum and O, and merge
// them at the end. One tile per CTA gives twice as many CTAs as tile pairs
// would, which evens out the last wave on 148 SMs.
//   warps 0-3   softmax warpgroup 0 (thread = query row), half 0
//   warps 4-7   softmax warpgroup 1 (same rows), half 1
//   warp 8      TMA producer: the Q tile once, K and V [128 x 64] blocks into a
//               4-deep ring (128-byte swizzle, 4-D tensor maps over the
//               caller's strides, so a fused QKV buffer is read in place)
//   warps 9-10  tcgen05.mma issuers, one per half (warp 9 also allocates TMEM)
//                 S_w = Q K_j^T     (M=128, N=128, K=64; A, B from shared memory)
//                 O_w += P_w V_j    (M=128, N=64, K=128; A = P_w from TMEM)
// Everything the softmax exchanges with the tensor core stays in TMEM: it
// loads the whole S row once, hands the S buffer back at once (so the half's
// next scores are computed while it works on the current block), writes P as
// 16-bit pairs into TMEM for the PV MMA, and O accumulates in TMEM with a
// lazily applied rescale. Causal masking skips key blocks above the diagonal
// and masks the diagonal block; the heaviest tiles are scheduled first.
// SIMT path: any D <= 256, any dtype, one warp per query row.
//
// Semantics follow lunara/codegen/triton_emitter.py:212-293: scale applied to
// Q K^T (launcher passes 1/sqrt(D), 302), causal keep-mask row >= col
// (265-268), fp32 softmax and accumulation. Keys past the end of the sequence
// are excluded from the softmax (the reference loads them as zeros and lets
// them take part, which only matters when Skv is not a multiple of its block).
#include <cudaTypedefs.h>

#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace lunara {
namespace {

constexpr int kQTile = 128;     // query rows per softmax warpgroup
constexpr int kKvBlock = 128;   // keys per iteration
constexpr int kHeadDim = 64;
constexpr int kKvStages = 4;
constexpr int kAttnThreads = 384;  // warpgroups: 0-1 softmax, 2 = TMA warp, 2 MMA warps, 1 idle warp
// Register split with setmaxnreg: the kernel launches with 168 registers per
// thread (384 x 168 = 64512); warpgroup 2 drops to 56 and the two softmax
// warpgroups rise to 224: 128 x 56 + 256 x 224 = 64512, exactly the launch total.
constexpr int kLaunchRegs = 168;
constexpr int kProducerRegs = 56;
constexpr int kSoftmaxRegs = 224;
static_assert(128 * kProducerRegs + 256 * kSoftmaxRegs <= kAttnThreads * kLaunchRegs, "register split");
constexpr float kRescaleLog2 = 8.0f;
// Of the 16 exponential pairs in each 32-column chunk, kPolyPairs are computed
// by a cubic on the f32x2 FMA pipe and the rest by MUFU ex2 (16 results per
// clock per SM), so the two pipes share the softmax's exponentials.
#ifndef LUNARA_ATTN_POLY_PAIRS
#define LUNARA_ATTN_POLY_PAIRS 0
#endif
constexpr int kPolyPairs = LUNARA_ATTN_POLY_PAIRS;
static_assert(kPolyPairs >= 0 && kPolyPairs <= 16, "poly pairs per chunk");
constexpr uint32_t kTileBytes = 128 * 128;  // one [128 x 64] 16-bit tile
constexpr int kAttnSmem = kTileBytes + 2 * kKvStages * kTileBytes + 4 * kQTile * 4 + 256 + 1024;
// TMEM columns: S_w (128 fp32 columns per Q tile), O_w (64), P_w (128 16-bit
// values packed in 64 columns).
constexpr uint32_t kTmemS = 0;
constexpr uint32_t kTmemO = 256;
constexpr uint32_t kTmemP = 384;
constexpr uint32_t kAttnTmemCols = 512;

struct AttnParams {
  void* O;
  int64_t os_b, os_h, os_s;
  int H, Sq, Skv;
  int n_qtiles;
  float scale_log2;
  int causal;
};

template <typename T>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, const AttnParams p, unsigned int* err) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t IDESC_S = idesc_f16(128, kKvBlock, kBF16, false, false);
  constexpr uint32_t IDESC_PV = idesc_f16(128, kHeadDim, kBF16, false, true);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t{1023});
  uint8_t* sQ = smem;                                   // the Q tile
  uint8_t* sK = sQ + kTileBytes;                        // kKvStages tiles
  uint8_t* sV = sK + kKvStages * kTileBytes;            // kKvStages tiles
  float* s_stats = reinterpret_cast<float*>(sV + kKvStages * kTileBytes);   // [half][m | l][row]
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_stats + 2 * 2 * kQTile);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + kKvStages;
  uint64_t* v_full = k_empty + kKvStages;
  uint64_t* v_empty = v_full + kKvStages;
  uint64_t* s_full = v_empty + kKvStages;   // [2] S_w computed
  uint64_t* s_free = s_full + 2;            // [2] S_w read into registers (buffer reusable)
  uint64_t* p_ready = s_free + 2;           // [2] P_w written to TMEM
  uint64_t* o_full = p_ready + 2;           // [2] P_w V done (O_w updated, P_w consumed)
  uint64_t* stats_ready = o_full + 2;       // both halves' O, m, l final
  uint64_t* drain_bar = stats_ready + 1;    // [2] one per MMA issuer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qt = p.causal ? (p.n_qtiles - 1 - static_cast<int>(blockIdx.x)) : static_cast<int>(blockIdx.x);
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int q0 = qt * kQTile;
  // Key blocks of this Q tile: 0 .. nb-1 (causal: up to the diagonal block).
  // Half w of the CTA (softmax warpgroup w and MMA warp 9+w) takes blocks j = w, w+2, ...
  const int nb_total = (p.Skv + kKvBlock - 1) / kKvBlock;
  int nb = nb_total;
  if (p.causal) {
    const int lim = (q0 + kQTile - 1) / kKvBlock + 1;
    nb = lim < nb_total ? lim : nb_total;
  }
  const int nb_h0 = (nb + 1) / 2, nb_h1 = nb / 2;   // blocks of half 0 / half 1

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kKvStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int w = 0; w < 2; ++w) {
      mbar_init(&s_full[w], 1);
      mbar_init(&s_free[w], kQTile);
      mbar_init(&p_ready[w], kQTile);
      mbar_init(&o_full[w], 1);
      mbar_init(&drain_bar[w], 1);
    }
    mbar_init(stats_ready, 2 * kQTile);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, kAttnTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();
  pdl_launch_dependents();
  // Each role adjusts its register budget at the top of its own branch, so the
  // compiler allocates every branch with that branch's budget.
  if (warp == 8) {
    reg_dealloc<kProducerRegs>();
    if (lane == 0) {
      // -------------------------------------------------------- TMA producer --
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      mbar_arrive_expect_tx(q_full, kTileBytes);
      tma_load_4d(sQ, &tq, q_full, 0, q0, h, b);
      int issued_k = 0, issued_v = 0;
      bool ok = true;
      for (int j = 0; j < nb && ok; ++j) {
        const int st = j % kKvStages;
        const uint32_t ph = static_cast<uint32_t>(j / kKvStages) & 1u;
        if (!mbar_wait(&k_empty[st], ph ^ 1u, abort_flag, err, kErrAttnProducer)) { ok = false; break; }
        mbar_arrive_expect_tx(&k_full[st], kTileBytes);
        tma_load_4d(sK + st * kTileBytes, &tk, &k_full[st], 0, j * kKvBlock, h, b);
        ++issued_k;
        if (!mbar_wait(&v_empty[st], ph ^ 1u, abort_flag, err, kErrAttnProducer)) { ok = false; break; }
        mbar_arrive_expect_tx(&v_full[st], kTileBytes);
        tma_load_4d(sV + st * kTileBytes, &tv, &v_full[st], 0, j * kKvBlock, h, b);
        ++issued_v;
      }
      if (!ok) {
        mbar_drain_wait(q_full, 0, 1000000000ull);
        for (int i = (issued_k > kKvStages ? issued_k - kKvStages : 0); i < issued_k; ++i)
          mbar_drain_wait(&k_full[i % kKvStages], static_cast<uint32_t>(i / kKvStages) & 1u, 1000000000ull);
        for (int i = (issued_v > kKvStages ? issued_v - kKvStages : 0); i < issued_v; ++i)
          mbar_drain_wait(&v_full[i % kKvStages], static_cast<uint32_t>(i / kKvStages) & 1u, 1000000000ull);
      }
    }
  } else if (warp == 9 || warp == 10) {
    reg_dealloc<kProducerRegs>();
    if (lane == 0) {
      // ------------------------------------------------------ MMA issuers --
      // Warp 9 + w issues the MMAs of half w, for its key blocks j = w + 2i:
      // S_w(next) as soon as the softmax has pulled S_w(j) into registers (the
      // next scores are ready when it finishes block j), then P_w(j) V_j once
      // P_w(j) is in TMEM. Each ring stage holds one key block and is released
      // by the issuer of the half that uses it.
      const int w = warp - 9;
      const int nbw = w ? nb_h1 : nb_h0;
      bool ok = mbar_wait(q_full, 0, abort_flag, err, kErrAttnMma);
      if (ok && nbw > 0) {
        tc_fence_after();
        // Descriptors are built once; the start-address field (bits 0-13, in
        // 16-byte units) then moves by constants: +32 B per K step within a
        // K-major row (Q, K), +2048 B (16 rows of 128 B) per K step down V,
        // and one tile (16 KB) per ring stage.
        constexpr uint64_t kTileStep = kTileBytes >> 4;
        const uint64_t qd = sw128_desc(smem_u32(sQ), 16, 1024);
        const uint64_t kd0 = sw128_desc(smem_u32(sK), 16, 1024);
        const uint64_t vd0 = sw128_desc(smem_u32(sV), kTileBytes, 1024);
        const uint32_t d_s = tmem_base + kTmemS + w * 128;
        const uint32_t d_o = tmem_base + kTmemO + w * kHeadDim;
        const uint32_t a_p = tmem_base + kTmemP + w * (kKvBlock / 2);
        auto issue_s = [&](int st) {
          const uint64_t kd = kd0 + st * kTileStep;
#pragma unroll
          for (int k = 0; k < kHeadDim / 16; ++k)
            umma_f16_ss(d_s, qd + 2 * k, kd + 2 * k, IDESC_S, k > 0 ? 1u : 0u);
        };
        auto issue_pv = [&](int st, bool first) {
          const uint64_t vd = vd0 + st * kTileStep;
#pragma unroll
          for (int k = 0; k < kKvBlock / 16; ++k)
            umma_f16_ts(d_o, a_p + k * 8, vd + 128 * k, IDESC_PV, (!first || k > 0) ? 1u : 0u);
        };
        {
          const int j = w;
          ok = mbar_wait(&k_full[j % kKvStages], static_cast<uint32_t>(j / kKvStages) & 1u, abort_flag, err,
                         kErrAttnMma);
          if (ok) {
            tc_fence_after();
            issue_s(j % kKvStages);
            umma_commit(&s_full[w]);
            umma_commit(&k_empty[j % kKvStages]);
          }
        }
        for (int i = 0; i < nbw && ok; ++i) {
          const int j = w + 2 * i;
          const uint32_t ipar = static_cast<uint32_t>(i) & 1u;
          if (i + 1 < nbw) {
            const int jn = j + 2;
            const int stn = jn % kKvStages;
            if (!mbar_wait(&k_full[stn], static_cast<uint32_t>(jn / kKvStages) & 1u, abort_flag, err, kErrAttnMma)) {
              ok = false;
              break;
            }
            if (!mbar_wait(&s_free[w], ipar, abort_flag, err, kErrAttnMma)) { ok = false; break; }
            tc_fence_after();
            issue_s(stn);
            umma_commit(&s_full[w]);
            umma_commit(&k_empty[stn]);
          }
          const int st = j % kKvStages;
          if (!mbar_wait(&v_full[st], static_cast<uint32_t>(j / kKvStages) & 1u, abort_flag, err, kErrAttnMma)) {
            ok = false;
            break;
          }
          if (!mbar_wait(&p_ready[w], ipar, abort_flag, err, kErrAttnMma)) { ok = false; break; }
          tc_fence_after();
          issue_pv(st, i == 0);
          umma_commit(&o_full[w]);
          umma_commit(&v_empty[st]);
        }
      }
      if (!ok) {
        umma_commit(&drain_bar[w]);
        mbar_drain_wait(&drain_bar[w], 0, 1000000000ull);
      }
    }
  } else if (warp == 11) {
    reg_dealloc<kProducerRegs>();   // idle warp of warpgroup 2
  } else {
    reg_alloc<kSoftmaxRegs>();
    // ------------------------------------------------------------- softmax --
    // Thread = one query row of the tile; warpgroup w holds the online-softmax
    // state (running max m, sum l, O_w in TMEM) of that row over its half of
    // the key blocks. The two halves are merged at the end.
    const int w = warp >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int qrow = q0 + r;
    const int my_nb = w ? nb_h1 : nb_h0;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tS = tmem_base + lane_off + kTmemS + w * 128;
    const uint32_t tO = tmem_base + lane_off + kTmemO + w * kHeadDim;
    const uint32_t tP = tmem_base + lane_off + kTmemP + w * (kKvBlock / 2);
    const float sl2 = p.scale_log2;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;

    for (int i = 0; i < my_nb; ++i) {
      const int j = w + 2 * i;
      if (!mbar_wait(&s_full[w], static_cast<uint32_t>(i) & 1u, abort_flag, err, kErrAttnSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // The whole 128-column score row: four TMEM loads, one wait; then the S
      // buffer is handed back so the next block's scores can be computed.
      uint32_t sc[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(tS + c * 32, sc[c]);
      tmem_ld_wait_regs(sc[0]);
      reg_fence(sc[1]);
      reg_fence(sc[2]);
      reg_fence(sc[3]);
      tc_fence_before();
      mbar_arrive(&s_free[w]);
      const int kv0 = j * kKvBlock;
      if ((kv0 + kKvBlock > p.Skv) || (p.causal && kv0 + kKvBlock - 1 > q0)) {
        // Keep key columns < Skv and (causal) <= this query row.
        int lim = p.Skv - kv0;
        if (p.causal && qrow - kv0 + 1 < lim) lim = qrow - kv0 + 1;
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (c * 32 + e >= lim) sc[c][e] = __float_as_uint(-INFINITY);
      }
      // Row maximum: three-input max, eight independent partial maxima.
      float mxp[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) mxp[t] = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int e = 0; e < 32; e += 2)
          mxp[(e >> 1) & 7] = fmax3(mxp[(e >> 1) & 7], __uint_as_float(sc[c][e]), __uint_as_float(sc[c][e + 1]));
      const float mx = fmax3(fmax3(mxp[0], mxp[1], mxp[2]), fmax3(mxp[3], mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7]));
      const float m_cand = mx * sl2;
      // Running maximum: raised only when a row's maximum grows by more than
      // 2^kRescaleLog2 (decided warp-wide); O is rescaled below, once the
      // previous block's P V has landed.
      bool rescale = false;
      float alpha = 1.f;
      if (i == 0) {
        m_used = m_cand;
      } else if (__any_sync(0xffffffffu, m_cand > m_used + kRescaleLog2)) {
        const float m_next = fmaxf(m_used, m_cand);
        alpha = ex2_approx(m_used - m_next);
        l *= alpha;
        m_used = m_next;
        rescale = true;
      }
      const float m_off = (m_used == -INFINITY) ? 0.f : m_used;
      // P = exp2(S * scale * log2e - m) as 16-bit pairs held in registers, row
      // sum in fp32; two columns per f32x2 op.
      const uint64_t sl2x2 = f2_pack(sl2, sl2);
      const uint64_t negm2 = f2_pack(-m_off, -m_off);
      uint64_t sum2[4] = {0ull, 0ull, 0ull, 0ull};   // packed (+0.0f, +0.0f)
      uint32_t pk[4][16];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const int pair = i >> 1;
          const bool poly = ((pair * kPolyPairs) % 16) < kPolyPairs;   // spread evenly over the chunk
          const uint64_t x2 = f2_fma(f2_pack(__uint_as_float(sc[c][i]), __uint_as_float(sc[c][i + 1])), sl2x2, negm2);
          uint64_t e2;
          if (poly) {
            e2 = ex2_poly2(x2);
          } else {
            const float2 x = f2_unpack(x2);
            e2 = f2_pack(ex2_approx(x.x), ex2_approx(x.y));
          }
          sum2[pair & 3] = f2_add(sum2[pair & 3], e2);
          const float2 e = f2_unpack(e2);
          pk[c][pair] = Io<T>::pack2(e.x, e.y);
        }
      }
      const float2 ls = f2_unpack(f2_add(f2_add(sum2[0], sum2[1]), f2_add(sum2[2], sum2[3])));
      l += ls.x + ls.y;
      // The previous block's P V must be complete (P_w consumed, O_w updated)
      // before P_w is overwritten and O_w is rescaled; by now it normally is.
      if (i > 0) {
        if (!mbar_wait(&o_full[w], static_cast<uint32_t>(i - 1) & 1u, abort_flag, err, kErrAttnSoftmax)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      if (rescale) {
        const uint64_t a2 = f2_pack(alpha, alpha);
#pragma unroll
        for (int c = 0; c < kHeadDim / 32; ++c) {
          uint32_t ov[32];
          tmem_ld_32x32b_x32(tO + c * 32, ov);
          tmem_ld_wait_regs(ov);
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float2 v2 = f2_unpack(f2_mul(f2_pack(__uint_as_float(ov[i]), __uint_as_float(ov[i + 1])), a2));
            ov[i] = __float_as_uint(v2.x);
            ov[i + 1] = __float_as_uint(v2.y);
          }
          tmem_st_32x32b_x32(tO + c * 32, ov);
        }
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_st_32x32b_x16(tP + c * 16, pk[c]);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_ready[w]);
    }
    // ------------------------------------------------------------ merge --
    // Publish this half's (m, l) after its last P V has landed, wait for the
    // other half, then warpgroup w writes output columns [32w, 32w + 32) of
    // the row: O = (O_0 2^(m_0 - m) + O_1 2^(m_1 - m)) / (l_0 2^(m_0 - m) + l_1 2^(m_1 - m)).
    if (ok && my_nb > 0) {
      ok = mbar_wait(&o_full[w], static_cast<uint32_t>(my_nb - 1) & 1u, abort_flag, err, kErrAttnSoftmax);
    }
    if (ok) {
      s_stats[(w * 2 + 0) * kQTile + r] = m_used;
      s_stats[(w * 2 + 1) * kQTile + r] = l;
      tc_fence_before();
      mbar_arrive(stats_ready);
      ok = mbar_wait(stats_ready, 0, abort_flag, err, kErrAttnSoftmax);
    }
    if (ok) {
      tc_fence_after();
      const float m0 = s_stats[0 * kQTile + r], l0 = s_stats[1 * kQTile + r];
      const float m1 = s_stats[2 * kQTile + r], l1 = s_stats[3 * kQTile + r];
      const bool has0 = nb_h0 > 0, has1 = nb_h1 > 0;
      const float m = fmaxf(has0 ? m0 : -INFINITY, has1 ? m1 : -INFINITY);
      const float a0 = (has0 && m0 != -INFINITY) ? ex2_approx(m0 - m) : 0.f;
      const float a1 = (has1 && m1 != -INFINITY) ? ex2_approx(m1 - m) : 0.f;
      const float inv_l = 1.0f / (l0 * a0 + l1 * a1);
      const float c0 = a0 * inv_l, c1 = a1 * inv_l;
      const uint32_t col = static_cast<uint32_t>(w * 32);
      uint32_t o0[32], o1[32];
      if (has0) tmem_ld_32x32b_x32(tmem_base + lane_off + kTmemO + col, o0);
      if (has1) tmem_ld_32x32b_x32(tmem_base + lane_off + kTmemO + kHeadDim + col, o1);
      tmem_ld_wait_regs(o0);
      reg_fence(o1);
      if (qrow < p.Sq) {
        T* out = static_cast<T*>(p.O) + b * p.os_b + h * p.os_h + static_cast<int64_t>(qrow) * p.os_s + col;
        uint4* ov4 = reinterpret_cast<uint4*>(out);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float v0 = has0 ? __uint_as_float(o0[8 * q + e]) * c0 : 0.f;
            const float v1 = has1 ? __uint_as_float(o1[8 * q + e]) * c1 : 0.f;
            f[e] = v0 + v1;
          }
          uint4 u;
          u.x = Io<T>::pack2(f[0], f[1]);
          u.y = Io<T>::pack2(f[2], f[3]);
          u.z = Io<T>::pack2(f[4], f[5]);
          u.w = Io<T>::pack2(f[6], f[7]);
          ov4[q] = u;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kAttnTmemCols);
  }
}

// ------------------------------------------------------------ SIMT path ----
// One warp per query row; lane holds D/32 (<= 8) elements of q and o.
template <typename T>
__global__ void __launch_bounds__(128) attn_simt_kernel(const T* __restrict__ Q, const T* __restrict__ K,
                                                        const T* __restrict__ V, T* __restrict__ O, AttnArgs a) {
  const int64_t qi = static_cast<int64_t>(blockIdx.x) * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t h = blockIdx.y, b = blockIdx.z;
  if (qi >= a.Sq) return;
  constexpr int kMaxPer = 8;
  const int per = static_cast<int>((a.D + 31) / 32);
  const T* q = Q + b * a.qs[0] + h * a.qs[1] + qi * a.qs[2];
  float qv[kMaxPer], ov[kMaxPer];
#pragma unroll
  for (int e = 0; e < kMaxPer; ++e) {
    const int64_t d = lane + 32 * e;
    qv[e] = (e < per && d < a.D) ? Io<T>::to_f(q[d * a.qs[3]]) * a.scale : 0.f;
    ov[e] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const int64_t kend = a.causal ? (qi + 1 < a.Skv ? qi + 1 : a.Skv) : a.Skv;
  for (int64_t j = 0; j < kend; ++j) {
    const T* k = K + b * a.ks[0] + h * a.ks[1] + j * a.ks[2];
    const T* v = V + b * a.vs[0] + h * a.vs[1] + j * a.vs[2];
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < kMaxPer; ++e) {
      const int64_t d = lane + 32 * e;
      if (e < per && d < a.D) s = fmaf(qv[e], Io<T>::to_f(k[d * a.ks[3]]), s);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float m_new = fmaxf(m, s);
    const float corr = __expf(m - m_new);
    const float pj = __expf(s - m_new);
    l = l * corr + pj;
#pragma unroll
    for (int e = 0; e < kMaxPer; ++e) {
      const int64_t d = lane + 32 * e;
      if (e < per && d < a.D) ov[e] = fmaf(ov[e], corr, pj * Io<T>::to_f(v[d * a.vs[3]]));
    }
    m = m_new;
  }
  T* out = O + b * a.os[0] + h * a.os[1] + qi * a.os[2];
  const float inv = 1.0f / l;
#pragma unroll
  for (int e = 0; e < kMaxPer; ++e) {
    const int64_t d = lane + 32 * e;
    if (e < per && d < a.D) out[d * a.os[3]] = Io<T>::from_f(ov[e] * inv);
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool encode_4d(CUtensorMap* map, const void* base, int dtype, int64_t S, int64_t H, int64_t B, const int64_t* st) {
  auto encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(tensor_map_encoder());
  if (encode == nullptr) return false;
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(kHeadDim), static_cast<cuuint64_t>(S),
                              static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(B)};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(st[2] * 2), static_cast<cuuint64_t>(st[1] * 2),
                                 static_cast<cuuint64_t>(st[0] * 2)};
  const cuuint32_t box[4] = {kHeadDim, 128, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt =
      dtype == LUNARA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return encode(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool strides_ok(const int64_t* s) {
  // dim stride 1; batch/head/seq strides give 16-byte aligned rows and fit TMA's 40-bit stride field.
  if (s[3] != 1) return false;
  for (int i = 0; i < 3; ++i)
    if (s[i] < 0 || (s[i] * 2) % 16 != 0 || s[i] * 2 >= (int64_t{1} << 40)) return false;
  return true;
}

template <typename T>
cudaError_t run_tc(const AttnArgs& a, cudaStream_t s) {
  CUtensorMap mq, mk, mv;
  if (!encode_4d(&mq, a.Q, a.dtype, a.Sq, a.H, a.B, a.qs) || !encode_4d(&mk, a.K, a.dtype, a.Skv, a.H, a.B, a.ks) ||
      !encode_4d(&mv, a.V, a.dtype, a.Skv, a.H, a.B, a.vs))
    return cudaErrorInvalidValue;
  auto kern = attn_tc_kernel<T>;
  // The setmaxnreg split assumes the kernel launches with exactly kLaunchRegs
  // registers per thread; refuse to launch a build where that does not hold.
  cudaFuncAttributes fa{};
  cudaError_t e = cudaFuncGetAttributes(&fa, kern);
  if (e != cudaSuccess) return e;
  if (fa.numRegs != kLaunchRegs) return cudaErrorInvalidConfiguration;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
  if (e != cudaSuccess) return e;
  AttnParams p{};
  p.O = a.O;
  p.os_b = a.os[0];
  p.os_h = a.os[1];
  p.os_s = a.os[2];
  p.H = static_cast<int>(a.H);
  p.Sq = static_cast<int>(a.Sq);
  p.Skv = static_cast<int>(a.Skv);
  p.n_qtiles = static_cast<int>(ceil_div64(a.Sq, kQTile));
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.causal = a.causal;
  unsigned int* err = device_error_word();
  if (err == nullptr) return cudaErrorInvalidDevice;
  const dim3 grid(static_cast<unsigned>(p.n_qtiles), static_cast<unsigned>(a.H), static_cast<unsigned>(a.B));
  return launch_pdl(kern, grid, dim3(kAttnThreads), static_cast<size_t>(kAttnSmem), s, mq, mk, mv, p, err);
}

}  // namespace

bool attention_tc_supported(const AttnArgs& a) {
  if (a.dtype != LUNARA_F16 && a.dtype != LUNARA_BF16) return false;
  if (a.D != kHeadDim) return false;
  if (a.Sq < 1 || a.Skv < 1 || a.Sq >= (int64_t{1} << 30) || a.Skv >= (int64_t{1} << 30)) return false;
  if (a.H > 65535 || a.B > 65535) return false;
  if (!al16(a.Q) || !al16(a.K) || !al16(a.V) || !al16(a.O)) return false;
  if (!strides_ok(a.qs) || !strides_ok(a.ks) || !strides_ok(a.vs) || !strides_ok(a.os)) return false;
  return true;
}

cudaError_t launch_attention_tcgen05(const AttnArgs& a, cudaStream_t stream) {
  return a.dtype == LUNARA_BF16 ? run_tc<__nv_bfloat16>(a, stream) : run_tc<__half>(a, stream);
}

cudaError_t launch_attention_simt(const AttnArgs& a, cudaStream_t stream) {
  if (a.Sq == 0 || a.B == 0 || a.H == 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>(ceil_div64(a.Sq, 4)), static_cast<unsigned>(a.H),
                  static_cast<unsigned>(a.B));
  switch (a.dtype) {
    case LUNARA_F16:
      attn_simt_kernel<__half><<<grid, 128, 0, stream>>>(static_cast<const __half*>(a.Q),
                                                         static_cast<const __half*>(a.K),
                                                         static_cast<const __half*>(a.V), static_cast<__half*>(a.O),
                                                         a);
      break;
    case LUNARA_BF16:
      attn_simt_kernel<__nv_bfloat16><<<grid, 128, 0, stream>>>(
          static_cast<const __nv_bfloat16*>(a.Q), static_cast<const __nv_bfloat16*>(a.K),
          static_cast<const __nv_bfloat16*>(a.V), static_cast<__nv_bfloat16*>(a.O), a);
      break;
    default:
      attn_simt_kernel<float><<<grid, 128, 0, stream>>>(static_cast<const float*>(a.Q),
                                                        static_cast<const float*>(a.K),
                                                        static_cast<const float*>(a.V), static_cast<float*>(a.O), a);
      break;
  }
  return cudaGetLastError();
}

}  // namespace lunara
