// Scaled-dot-product attention forward, O = softmax(Q K^T * scale [+ causal]) V.
//
// tcgen05 path (f16 / bf16, D == 64): FlashAttention-style single pass with an
// online softmax. A persistent CTA (one per SM) works through 128-row Q tiles
// of (batch, head) pairs; for each tile its two halves split the key blocks
// (half 0 takes blocks 0, 2, 4, ..., half 1 takes 1, 3, 5, ...), each keeping
// its own running max, row sum and O, and merge them at the end. Tile-sized
// work items even out the last round on 148 SMs, and persistence pays the
// set-up (TMEM allocation, barriers, first loads) once per SM: the next
// tile's Q and key blocks load while the current tile finishes.
//   warps 0-3   softmax warpgroup 0 (thread = query row), half 0
//   warps 4-7   softmax warpgroup 1 (same rows), half 1
//   warp 8      TMA producers: lane 0 loads Q tiles into a 2-deep buffer and
//               K [128 x 64] blocks into a 4-deep ring, lane 1 loads V blocks
//               into their own 4-deep ring (128-byte swizzle, 4-D tensor maps
//               over the caller's strides, so a fused QKV buffer is read in
//               place); K never waits behind a V slot that a late PV holds
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
// 4 of 16 measured fastest on B200 with the persistent kernel (B2 H12 S2048:
// 47.9 us against 49.6 with none, 49.0 with 6 and 53.9 with 8; the block
// shape B8 H12 S512: 19.3 against 19.7 us).
#ifndef LUNARA_ATTN_POLY_PAIRS
#define LUNARA_ATTN_POLY_PAIRS 4
#endif
constexpr int kPolyPairs = LUNARA_ATTN_POLY_PAIRS;

static_assert(kPolyPairs >= 0 && kPolyPairs <= 16, "poly pairs per chunk");
constexpr uint32_t kTileBytes = 128 * 128;  // one [128 x 64] 16-bit tile
constexpr int kAttnSmem = 2 * kTileBytes + 2 * kKvStages * kTileBytes + 4 * kQTile * 4 + 512 + 1024;
// TMEM columns: S_w (128 fp32 columns per Q tile), O_w (64), P_w (128 16-bit
// values packed in 64 columns).
constexpr uint32_t kTmemS = 0;
constexpr uint32_t kTmemO = 256;
constexpr uint32_t kTmemP = 384;
constexpr uint32_t kAttnTmemCols = 512;

struct AttnParams {
  void* O;
  int64_t os_b, os_h, os_s;
  int B, H, Sq, Skv;
  int n_qtiles;
  float scale_log2;
  int causal;
};

// Work item of a persistent CTA: one 128-row Q tile of one (batch, head).
// Tiles are numbered with the query-tile index outermost (for causal
// attention, heaviest first); CTA c takes tiles c, 2G-1-c, 2G+c, 4G-1-c, ...
// (a snake over rounds of G = gridDim.x tiles), which pairs heavy and light
// causal tiles on the same CTA.
struct AttnTile {
  int q0, h, b, nb;
};

__device__ __forceinline__ int attn_tile_index(int k, int c, int G) {
  return k * G + ((k & 1) ? (G - 1 - c) : c);
}

__device__ __forceinline__ AttnTile attn_tile(int t, const AttnParams& p) {
  const int hb_count = p.H * p.B;
  const int qi = t / hb_count;
  const int hb = t - qi * hb_count;
  AttnTile x;
  const int qt = p.causal ? (p.n_qtiles - 1 - qi) : qi;
  x.q0 = qt * kQTile;
  x.h = hb % p.H;
  x.b = hb / p.H;
  const int nb_total = (p.Skv + kKvBlock - 1) / kKvBlock;
  x.nb = nb_total;
  if (p.causal) {
    const int lim = (x.q0 + kQTile - 1) / kKvBlock + 1;
    x.nb = lim < nb_total ? lim : nb_total;
  }
  return x;
}

template <typename T>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, const AttnParams p, unsigned int* err) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t IDESC_S = idesc_f16(128, kKvBlock, kBF16, false, false);
  constexpr uint32_t IDESC_PV = idesc_f16(128, kHeadDim, kBF16, false, true);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t{1023});
  uint8_t* sQ = smem;                                   // 2 Q tiles (double buffer over work items)
  uint8_t* sK = sQ + 2 * kTileBytes;                    // kKvStages tiles
  uint8_t* sV = sK + kKvStages * kTileBytes;            // kKvStages tiles
  float* s_stats = reinterpret_cast<float*>(sV + kKvStages * kTileBytes);   // [half][m | l][row]
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_stats + 2 * 2 * kQTile);
  uint64_t* q_full = bars;                  // [2]
  uint64_t* q_empty = q_full + 2;           // [2] both issuers done with the Q buffer
  uint64_t* k_full = q_empty + 2;
  uint64_t* k_empty = k_full + kKvStages;
  uint64_t* v_full = k_empty + kKvStages;
  uint64_t* v_empty = v_full + kKvStages;
  uint64_t* s_full = v_empty + kKvStages;   // [2] S_w computed
  uint64_t* s_free = s_full + 2;            // [2] S_w read into registers (buffer reusable)
  uint64_t* p_ready = s_free + 2;           // [2] P_w written to TMEM
  uint64_t* o_full = p_ready + 2;           // [2] P_w V done (O_w updated, P_w consumed)
  uint64_t* stats_ready = o_full + 2;       // both halves' O, m, l of the work item final
  uint64_t* o_free = stats_ready + 1;       // the merge has read both O buffers
  uint64_t* drain_bar = o_free + 1;         // [2] one per MMA issuer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = static_cast<int>(gridDim.x);
  const int cta = static_cast<int>(blockIdx.x);
  const int n_tiles = p.n_qtiles * p.H * p.B;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 2);
    }
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
    mbar_init(o_free, 2 * kQTile);
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
      // ------------------------------------------------- TMA producer: Q, K --
      // Per work item: its Q tile into the free Q buffer, then its key blocks'
      // K tiles into the K ring (ring slots and phases count blocks across
      // items). K runs ahead on its own: a K slot frees as soon as the S MMA
      // that read it completes, so the next S never waits behind a V slot.
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      int issued_q = 0, issued_k = 0;
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int t = attn_tile_index(k, cta, G);
        if (t >= n_tiles) break;
        const AttnTile x = attn_tile(t, p);
        const int buf = k & 1;
        if (!mbar_wait(&q_empty[buf], (static_cast<uint32_t>(k >> 1) & 1u) ^ 1u, abort_flag, err, kErrAttnProducer)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&q_full[buf], kTileBytes);
        tma_load_4d(sQ + buf * kTileBytes, &tq, &q_full[buf], 0, x.q0, x.h, x.b);
        ++issued_q;
        for (int j = 0; j < x.nb; ++j) {
          const int g = issued_k;
          const int st = g % kKvStages;
          const uint32_t ph = static_cast<uint32_t>(g / kKvStages) & 1u;
          if (!mbar_wait(&k_empty[st], ph ^ 1u, abort_flag, err, kErrAttnProducer)) { ok = false; break; }
          mbar_arrive_expect_tx(&k_full[st], kTileBytes);
          tma_load_4d(sK + st * kTileBytes, &tk, &k_full[st], 0, j * kKvBlock, x.h, x.b);
          ++issued_k;
        }
      }
      if (!ok) {
        for (int i = (issued_q > 2 ? issued_q - 2 : 0); i < issued_q; ++i)
          mbar_drain_wait(&q_full[i & 1], static_cast<uint32_t>(i >> 1) & 1u, 1000000000ull);
        for (int i = (issued_k > kKvStages ? issued_k - kKvStages : 0); i < issued_k; ++i)
          mbar_drain_wait(&k_full[i % kKvStages], static_cast<uint32_t>(i / kKvStages) & 1u, 1000000000ull);
      }
    } else if (lane == 1) {
      // ---------------------------------------------------- TMA producer: V --
      // The same walk over work items and key blocks, V tiles into the V ring.
      tma_prefetch_desc(&tv);
      int issued_v = 0;
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int t = attn_tile_index(k, cta, G);
        if (t >= n_tiles) break;
        const AttnTile x = attn_tile(t, p);
        for (int j = 0; j < x.nb; ++j) {
          const int g = issued_v;
          const int st = g % kKvStages;
          const uint32_t ph = static_cast<uint32_t>(g / kKvStages) & 1u;
          if (!mbar_wait(&v_empty[st], ph ^ 1u, abort_flag, err, kErrAttnProducer)) { ok = false; break; }
          mbar_arrive_expect_tx(&v_full[st], kTileBytes);
          tma_load_4d(sV + st * kTileBytes, &tv, &v_full[st], 0, j * kKvBlock, x.h, x.b);
          ++issued_v;
        }
      }
      if (!ok) {
        for (int i = (issued_v > kKvStages ? issued_v - kKvStages : 0); i < issued_v; ++i)
          mbar_drain_wait(&v_full[i % kKvStages], static_cast<uint32_t>(i / kKvStages) & 1u, 1000000000ull);
      }
    }
  } else if (warp == 9 || warp == 10) {
    reg_dealloc<kProducerRegs>();
    {
      // ------------------------------------------------------ MMA issuers --
      // Warp 9 + w issues the MMAs of half w, for its key blocks j = w + 2i of
      // each work item: S_w(next) as soon as the softmax has pulled the current
      // S_w into registers (the next scores are ready when it finishes the
      // current block), then P_w V_j once P_w is in TMEM. A ring stage holds
      // one key block and is released by the issuer of the half that uses it;
      // a Q buffer is released by both issuers after their last S of the item.
      // The whole warp runs the loop (every lane waits and the outcomes are
      // combined, so all values stay warp-uniform) and one elected lane issues
      // each MMA and commit.
      const int w = warp - 9;
      const bool leader = elect_one_sync();
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return mbar_wait_warp(bar, parity, abort_flag, err, kErrAttnMma);
      };
      constexpr uint64_t kTileStep = kTileBytes >> 4;
      // Descriptors are built once; the start-address field (bits 0-13, in
      // 16-byte units) then moves by constants: +32 B per K step within a
      // K-major row (Q, K), +2048 B (16 rows of 128 B) per K step down V, and
      // one tile (16 KB) per Q buffer or ring stage.
      const uint64_t qd0 = sw128_desc(smem_u32(sQ), 16, 1024);
      const uint64_t kd0 = sw128_desc(smem_u32(sK), 16, 1024);
      const uint64_t vd0 = sw128_desc(smem_u32(sV), kTileBytes, 1024);
      const uint32_t d_s = tmem_base + kTmemS + w * 128;
      const uint32_t d_o = tmem_base + kTmemO + w * kHeadDim;
      const uint32_t a_p = tmem_base + kTmemP + w * (kKvBlock / 2);
      auto issue_s = [&](uint64_t qd, int st) {
        const uint64_t kd = kd0 + st * kTileStep;
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk)
          umma_f16_ss(d_s, qd + 2 * kk, kd + 2 * kk, IDESC_S, kk > 0 ? 1u : 0u);
      };
      auto issue_pv = [&](int st, bool first) {
        const uint64_t vd = vd0 + st * kTileStep;
#pragma unroll
        for (int kk = 0; kk < kKvBlock / 16; ++kk)
          umma_f16_ts(d_o, a_p + kk * 8, vd + 128 * kk, IDESC_PV, (!first || kk > 0) ? 1u : 0u);
      };
      bool ok = true;
      int gi = 0;        // this half's blocks so far (phase of s_full / s_free / p_ready / o_full)
      int gb_base = 0;   // ring index of the current item's block 0
      for (int k = 0; ok; ++k) {
        const int t = attn_tile_index(k, cta, G);
        if (t >= n_tiles) break;
        const AttnTile x = attn_tile(t, p);
        const int nbw = w ? x.nb / 2 : (x.nb + 1) / 2;
        const int buf = k & 1;
        if (!wait(&q_full[buf], static_cast<uint32_t>(k >> 1) & 1u)) {
          ok = false;
          break;
        }
        if (nbw == 0) {
          if (leader) mbar_arrive(&q_empty[buf]);
          __syncwarp();
          gb_base += x.nb;
          continue;
        }
        tc_fence_after();
        const uint64_t qd = qd0 + buf * kTileStep;
        {
          const int g = gb_base + w;
          if (!wait(&k_full[g % kKvStages], static_cast<uint32_t>(g / kKvStages) & 1u)) {
            ok = false;
            break;
          }
          if (gi > 0 && !wait(&s_free[w], static_cast<uint32_t>(gi - 1) & 1u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (leader) {
            issue_s(qd, g % kKvStages);
            umma_commit(&s_full[w]);
            umma_commit(&k_empty[g % kKvStages]);
            if (nbw == 1) umma_commit(&q_empty[buf]);
          }
          __syncwarp();
        }
        for (int i = 0; i < nbw && ok; ++i) {
          const int g = gb_base + w + 2 * i;
          const uint32_t cpar = static_cast<uint32_t>(gi + i) & 1u;
          if (i + 1 < nbw) {
            const int gn = g + 2;
            if (!wait(&k_full[gn % kKvStages], static_cast<uint32_t>(gn / kKvStages) & 1u)) {
              ok = false;
              break;
            }
            if (!wait(&s_free[w], cpar)) { ok = false; break; }
            tc_fence_after();
            if (leader) {
              issue_s(qd, gn % kKvStages);
              umma_commit(&s_full[w]);
              umma_commit(&k_empty[gn % kKvStages]);
              if (i + 2 == nbw) umma_commit(&q_empty[buf]);
            }
            __syncwarp();
          }
          const int st = g % kKvStages;
          if (!wait(&v_full[st], static_cast<uint32_t>(g / kKvStages) & 1u)) {
            ok = false;
            break;
          }
          if (!wait(&p_ready[w], cpar)) { ok = false; break; }
          // The first P V of an item overwrites O_w: the previous item's merge
          // must have read it.
          if (i == 0 && k > 0 && !wait(o_free, static_cast<uint32_t>(k - 1) & 1u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (leader) {
            issue_pv(st, i == 0);
            umma_commit(&o_full[w]);
            umma_commit(&v_empty[st]);
          }
          __syncwarp();
        }
        gi += nbw;
        gb_base += x.nb;
      }
      if (!ok) {
        if (leader) umma_commit(&drain_bar[w]);
        __syncwarp();
        mbar_drain_wait(&drain_bar[w], 0, 1000000000ull);
      }
    }
  } else if (warp == 11) {
    reg_dealloc<kProducerRegs>();   // idle warp of warpgroup 2
  } else {
    reg_alloc<kSoftmaxRegs>();
    // ------------------------------------------------------------- softmax --
    // Thread = one query row of the work item; warpgroup w holds the online-
    // softmax state (running max m, sum l, O_w in TMEM) of that row over its
    // half of the key blocks. The two halves are merged at the end of the item.
    const int w = warp >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tS = tmem_base + lane_off + kTmemS + w * 128;
    const uint32_t tO = tmem_base + lane_off + kTmemO + w * kHeadDim;
    const uint32_t tP = tmem_base + lane_off + kTmemP + w * (kKvBlock / 2);
    const float sl2 = p.scale_log2;
    bool ok = true;
    int gi = 0;   // this half's blocks so far (barrier phases)
    for (int k = 0; ok; ++k) {
      const int t = attn_tile_index(k, cta, G);
      if (t >= n_tiles) break;
      const AttnTile x = attn_tile(t, p);
      const int q0 = x.q0;
      const int qrow = q0 + r;
      const int nb_h0 = (x.nb + 1) / 2, nb_h1 = x.nb / 2;
      const int my_nb = w ? nb_h1 : nb_h0;
      float m_used = -INFINITY, l = 0.f;

    for (int i = 0; i < my_nb; ++i) {
      const int j = w + 2 * i;
      const int cur = gi + i;
      if (!mbar_wait(&s_full[w], static_cast<uint32_t>(cur) & 1u, abort_flag, err, kErrAttnSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // The whole 128-column score row: four TMEM loads, one wait; then the S
      // buffer is handed back so the next block's scores can be computed.
      uint32_t sc[4][32];
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) tmem_ld_32x32b_x32(tS + cc * 32, sc[cc]);
      tmem_ld_wait_regs(sc[0]);
      reg_fence(sc[1]);
      reg_fence(sc[2]);
      reg_fence(sc[3]);
      tc_fence_before();
      mbar_arrive(&s_free[w]);
      const int kv0 = j * kKvBlock;
      const bool masked = (kv0 + kKvBlock > p.Skv) || (p.causal && kv0 + kKvBlock - 1 > q0);
      int lim = kKvBlock;
      if (masked) {
        // Keep key columns < Skv and (causal) <= this query row.
        lim = p.Skv - kv0;
        if (p.causal && qrow - kv0 + 1 < lim) lim = qrow - kv0 + 1;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (cc * 32 + e >= lim) sc[cc][e] = __float_as_uint(-INFINITY);
      }
      // Row maximum: three-input max, eight independent partial maxima. NaN
      // propagates (max.NaN): a NaN score makes the running maximum, and so
      // every exponent and the whole output row, NaN -- as the softmax of a
      // row holding a NaN is.
      float mxp[8];
#pragma unroll
      for (int tt = 0; tt < 8; ++tt) mxp[tt] = -INFINITY;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc)
#pragma unroll
        for (int e = 0; e < 32; e += 2)
          mxp[(e >> 1) & 7] = fmax3_nan(mxp[(e >> 1) & 7], __uint_as_float(sc[cc][e]), __uint_as_float(sc[cc][e + 1]));
      const float mx = fmax3_nan(fmax3_nan(mxp[0], mxp[1], mxp[2]), fmax3_nan(mxp[3], mxp[4], mxp[5]),
                                 fmax_nan(mxp[6], mxp[7]));
      const float m_cand = mx * sl2;
      // Running maximum: raised only when a row's maximum grows by more than
      // 2^kRescaleLog2 (decided warp-wide); O is rescaled below, once the
      // previous block's P V has landed.
      bool rescale = false;
      float alpha = 1.f;
      if (i == 0) {
        m_used = m_cand;
      } else if (__any_sync(0xffffffffu, !(m_cand <= m_used + kRescaleLog2))) {   // true for NaN too
        const float m_next = fmax_nan(m_used, m_cand);
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
      // Staged in groups of 8 pairs: all scale-and-subtract FMAs of the group,
      // then all its exponentials, then its sums and 16-bit packs, so that
      // many independent MUFU operations are in flight at once (measured
      // ~1% faster than one pair at a time).
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int g0 = 0; g0 < 16; g0 += 8) {
          uint64_t x2[8], e2[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int i = 2 * (g0 + q);
            x2[q] = f2_fma(f2_pack(__uint_as_float(sc[c][i]), __uint_as_float(sc[c][i + 1])), sl2x2, negm2);
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int pair = g0 + q;
            if (((pair * kPolyPairs) % 16) < kPolyPairs) {   // spread evenly over the chunk
              e2[q] = ex2_poly2_clamped(x2[q]);
            } else {
              const float2 x = f2_unpack(x2[q]);
              e2[q] = f2_pack(ex2_approx(x.x), ex2_approx(x.y));
            }
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int pair = g0 + q;
            sum2[pair & 3] = f2_add(sum2[pair & 3], e2[q]);
            const float2 e = f2_unpack(e2[q]);
            pk[c][pair] = Io<T>::pack2(e.x, e.y);
          }
        }
      }
      if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        // The FMA-pipe exponential gives ~2^-126 for a masked (-inf) score,
        // which bf16 can hold: masked columns get an exact zero P here (the
        // fp16 rounding already flushes it to zero).
        if (masked) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int pair = 0; pair < 16; ++pair) {
              const int col = c * 32 + 2 * pair;
              if (col >= lim) pk[c][pair] = 0u;
              else if (col + 1 >= lim) pk[c][pair] &= 0xFFFFu;
            }
        }
      }
      const float2 ls = f2_unpack(f2_add(f2_add(sum2[0], sum2[1]), f2_add(sum2[2], sum2[3])));
      l += ls.x + ls.y;
      // The previous block's P V must be complete (P_w consumed, O_w updated)
      // before P_w is overwritten and O_w is rescaled; by now it normally is.
      if (i > 0) {
        if (!mbar_wait(&o_full[w], static_cast<uint32_t>(cur - 1) & 1u, abort_flag, err, kErrAttnSoftmax)) {
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
      // ---------------------------------------------------------- merge --
      // Publish this half's (m, l) once its last P V has landed, wait for the
      // other half, then warpgroup w writes output columns [32w, 32w + 32) of
      // the row: O = (O_0 2^(m_0 - m) + O_1 2^(m_1 - m)) / (l_0 2^(m_0 - m) + l_1 2^(m_1 - m)).
      if (ok && my_nb > 0) {
        ok = mbar_wait(&o_full[w], static_cast<uint32_t>(gi + my_nb - 1) & 1u, abort_flag, err, kErrAttnSoftmax);
      }
      if (!ok) break;
      s_stats[(w * 2 + 0) * kQTile + r] = m_used;
      s_stats[(w * 2 + 1) * kQTile + r] = l;
      tc_fence_before();
      mbar_arrive(stats_ready);
      if (!mbar_wait(stats_ready, static_cast<uint32_t>(k) & 1u, abort_flag, err, kErrAttnSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float m0 = s_stats[0 * kQTile + r], l0 = s_stats[1 * kQTile + r];
      const float m1 = s_stats[2 * kQTile + r], l1 = s_stats[3 * kQTile + r];
      const bool has0 = nb_h0 > 0, has1 = nb_h1 > 0;
      const float m = fmax_nan(has0 ? m0 : -INFINITY, has1 ? m1 : -INFINITY);
      const float a0 = (has0 && m0 != -INFINITY) ? ex2_approx(m0 - m) : 0.f;
      const float a1 = (has1 && m1 != -INFINITY) ? ex2_approx(m1 - m) : 0.f;
      const float inv_l = 1.0f / (l0 * a0 + l1 * a1);
      const float c0 = a0 * inv_l, c1 = a1 * inv_l;
      const uint32_t col = static_cast<uint32_t>(w * 32);
      T* out = static_cast<T*>(p.O) + x.b * p.os_b + x.h * p.os_h + static_cast<int64_t>(qrow) * p.os_s + col;
      // All four TMEM loads (both halves' O, this warpgroup's 32 columns) are
      // issued together and waited for once.
      uint32_t o0[32], o1[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) o0[e] = o1[e] = 0u;
      if (has0) tmem_ld_32x32b_x32(tmem_base + lane_off + kTmemO + col, o0);
      if (has1) tmem_ld_32x32b_x32(tmem_base + lane_off + kTmemO + kHeadDim + col, o1);
      tmem_ld_wait_regs(o0);
      reg_fence(o1);
      // Both O buffers read: the next item's first P V may overwrite them.
      tc_fence_before();
      mbar_arrive(o_free);
      if (qrow < p.Sq) {
        uint4* ov4 = reinterpret_cast<uint4*>(out);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e)
            f[e] = __uint_as_float(o0[8 * q + e]) * c0 + __uint_as_float(o1[8 * q + e]) * c1;
          uint4 u;
          u.x = Io<T>::pack2(f[0], f[1]);
          u.y = Io<T>::pack2(f[2], f[3]);
          u.z = Io<T>::pack2(f[4], f[5]);
          u.w = Io<T>::pack2(f[6], f[7]);
          ov4[q] = u;
        }
      }
      gi += my_nb;
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

// Strides of a [B, H, S, D] view as the tensor map takes them: a dimension of
// extent 1 is never stepped, so whatever stride torch gives it (0 after an
// expand, anything after a slice) is replaced by a harmless 16-byte multiple.
void map_strides(const int64_t* st, int64_t B, int64_t H, int64_t S, int64_t (&out)[4]) {
  const int64_t ext[3] = {B, H, S};
  for (int i = 0; i < 3; ++i) out[i] = ext[i] == 1 ? kHeadDim : st[i];
  out[3] = st[3];
}

bool strides_ok(const int64_t* st, int64_t B, int64_t H, int64_t S) {
  // Dim stride 1; each stepped batch / head / seq stride positive (a zero
  // stride, e.g. K/V expanded over the batch, goes to the CUDA-core kernel),
  // a multiple of 16 bytes and within TMA's 40-bit stride field.
  int64_t s[4];
  map_strides(st, B, H, S, s);
  if (s[3] != 1) return false;
  for (int i = 0; i < 3; ++i)
    if (s[i] <= 0 || (s[i] * 2) % 16 != 0 || s[i] * 2 >= (int64_t{1} << 40)) return false;
  return true;
}

template <typename T>
cudaError_t run_tc(const AttnArgs& a, cudaStream_t s, bool* handled) {
  CUtensorMap mq, mk, mv;
  int64_t qs[4], ks[4], vs[4];
  map_strides(a.qs, a.B, a.H, a.Sq, qs);
  map_strides(a.ks, a.B, a.H, a.Skv, ks);
  map_strides(a.vs, a.B, a.H, a.Skv, vs);
  if (!encode_4d(&mq, a.Q, a.dtype, a.Sq, a.H, a.B, qs) || !encode_4d(&mk, a.K, a.dtype, a.Skv, a.H, a.B, ks) ||
      !encode_4d(&mv, a.V, a.dtype, a.Skv, a.H, a.B, vs)) {
    *handled = false;   // the driver refused a tensor map: the CUDA-core kernel takes the call
    return cudaSuccess;
  }
  *handled = true;
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
  p.B = static_cast<int>(a.B);
  p.H = static_cast<int>(a.H);
  p.Sq = static_cast<int>(a.Sq);
  p.Skv = static_cast<int>(a.Skv);
  p.n_qtiles = static_cast<int>(ceil_div64(a.Sq, kQTile));
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.causal = a.causal;
  unsigned int* err = device_error_word();
  if (err == nullptr) return cudaErrorInvalidDevice;
  // Persistent: one CTA per SM (the 512-column TMEM allocation allows one),
  // each looping over work items; never more CTAs than items.
  const int64_t n_items = static_cast<int64_t>(p.n_qtiles) * a.H * a.B;
  const int sms = device_num_sms();
  const dim3 grid(static_cast<unsigned>(n_items < sms ? n_items : sms));
  return launch_pdl(kern, grid, dim3(kAttnThreads), static_cast<size_t>(kAttnSmem), s, mq, mk, mv, p, err);
}

}  // namespace

bool attention_tc_supported(const AttnArgs& a) {
  if (a.dtype != LUNARA_F16 && a.dtype != LUNARA_BF16) return false;
  if (a.D != kHeadDim) return false;
  if (a.Sq < 1 || a.Skv < 1 || a.Sq >= (int64_t{1} << 30) || a.Skv >= (int64_t{1} << 30)) return false;
  if (a.H > 65535 || a.B > 65535) return false;
  if (!al16(a.Q) || !al16(a.K) || !al16(a.V) || !al16(a.O)) return false;
  if (!strides_ok(a.qs, a.B, a.H, a.Sq) || !strides_ok(a.ks, a.B, a.H, a.Skv) || !strides_ok(a.vs, a.B, a.H, a.Skv))
    return false;
  if (a.os[3] != 1) return false;   // O is written with plain 16-byte stores: unit dim stride, aligned rows
  for (int i = 0; i < 3; ++i)
    if ((a.os[i] * 2) % 16 != 0) return false;
  return true;
}

cudaError_t launch_attention_tcgen05(const AttnArgs& a, cudaStream_t stream, bool* handled) {
  return a.dtype == LUNARA_BF16 ? run_tc<__nv_bfloat16>(a, stream, handled) : run_tc<__half>(a, stream, handled);
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
