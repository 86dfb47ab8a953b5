// sm100_fwd.cu -- tcgen05 / TMA / TMEM flash-attention forward for B200.
//
// Replaces flash_attn_fwd_kernel (npu_flash_attention.py:17-166) for bf16/fp16
// inputs with head_dim 64 or 128 (head_dim 256 runs on sm100_fwd256.cu). Same math: S = QKᵀ·scale, optional soft-cap
// and ALiBi, causal / sliding-window masks, online softmax in base 2, O = PV/l
// and LSE = m + ln(l) in natural log.
//
// One CTA owns two 128-row query tiles of one (batch, q-head) and walks the key
// tiles (128 keys) that any of its rows can see. Warp roles:
//   warp 0      TMA producer: Q once, then K_j, V_j into a ring of smem slots
//   warp 1      MMA issuer: S_t = Q_t K_jᵀ into TMEM, O_t += P_t V_j into TMEM
//   warp 2      TMEM allocator (512 columns)
//   warps 4-7   softmax for query tile 0, warps 8-11 for tile 1: each thread
//               owns one query row (one TMEM lane), reads its S row with
//               tcgen05.ld, writes P (16-bit) over the first 64 columns of its
//               S in TMEM, the A operand of the PV MMA (TS form), rescales its
//               O row in TMEM when the running max grows, and finally writes O
//               via smem + TMA store and the LSE.
// The MMA order S_0(j), S_1(j), then per step PV_0(j), S_0(j+1), PV_1(j),
// S_1(j+1) lets one tile's softmax run while the tensor core works on the
// other tile; each PV_t(j) goes out in two halves of 64 keys, the first once
// the softmax has stored P for those keys. K/V are read with the GQA head map hkv = hq / G
// (npu_flash_attention.py:42); no K/V expansion happens anywhere.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>
#include <type_traits>

#include "bfa_internal.h"
#include "sm100_host.h"
#include "sm100_ptx.cuh"

namespace bfa {
namespace {

using namespace sm100;

constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kThreads = 384;
// Rescale O only when a row's running max grows by more than this (base-2
// units). Until then P is computed against the stale max, so P <= 2^8; the
// final O/l and LSE are exact either way.
constexpr float kRescaleThreshold = 8.0f;
// Every kPolyEvery-th exponential of a fully kept tile runs on the FMA pipe
// (ex2_poly) instead of the MUFU unit.
constexpr int kPolyEvery = 8;

template <int D>
struct FwdLayout {
  static constexpr int kSub = D / 64;
  static constexpr uint32_t kQBytes = kBM * D * 2;
  static constexpr uint32_t kKVBytes = kBN * D * 2;
  static constexpr int kStages = (D <= 64) ? 8 : 5;  // K/V ring slots
  static constexpr uint32_t kOffQ = 0;
  static constexpr uint32_t kOffKV = kOffQ + 2 * kQBytes;
  static constexpr uint32_t kOffBar = kOffKV + kStages * kKVBytes;
  static constexpr uint32_t kSmemBytes = kOffBar + 512 + 1024;
  // TMEM: S_t (fp32, 128 columns) at t * kBN; P_t (16-bit, packed two per
  // column) overwrites the first 64 columns of S_t; O_t at kTmemO + t * D.
  static constexpr uint32_t kTmemS = 0;
  static constexpr uint32_t kTmemO = 2 * kBN;
  static_assert(kTmemO + 2 * D <= 512, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "smem budget");
};

// True when every (row, key) pair of the tile is kept and inside Sk.
__device__ __forceinline__ bool tile_full(const Params& p, int r0, int r1, int c0, int c1) {
  if (c1 > p.Sk) return false;
  if (p.doc_lo && r1 > p.Sq) return false;  // document bounds exist only for rows < Sq
  const int64_t i_min = r0 + p.q_off, i_max = r1 - 1 + p.q_off;
  const int64_t j_min = c0 + p.k_off, j_max = c1 - 1 + p.k_off;
  if (p.causal && j_max > i_min) return false;
  if (p.window > 0 && i_max - j_min > p.window) return false;
  return same_document(p, i_min, i_max, j_min, j_max);
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  return BF16 ? pack_bf16(a, b) : pack_f16(a, b);
}

// BLK: a block-sparse mask is given (p.blk); without it the tile walk is the
// plain range [jlo, jend), resolved at compile time.
template <int D, bool BF16, bool CAP, bool ALIBI, bool BLK>
__global__ void __launch_bounds__(kThreads, 1)
    fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
               const Params p) {
  using L = FwdLayout<D>;
  constexpr int NS = L::kStages;
  enum {
    kQFull = 0,
    kKVFull = 1,
    kKVEmpty = 1 + NS,
    kSFull = 1 + 2 * NS,
    kPFull = kSFull + 2,   // all of P_t(j) (and a rescaled O_t) in TMEM
    kPHalf = kPFull + 2,   // P_t(j) of keys [0, 64) in TMEM (and a rescaled O_t)
    kODone = kPHalf + 2,
    kDrain = kODone + 2,
    kNever = kDrain + 1,
    kNumBars = kNever + 1
  };

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  auto bar = [&](int i) -> uint32_t { return sbase + L::kOffBar + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = (uint32_t*)(smem + L::kOffBar + 8 * kNumBars);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  int* warp_ok = (int*)(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_mblk = (p.Sq + 2 * kBM - 1) / (2 * kBM);
  const int bh = blockIdx.x % (p.B * p.Hq);
  const int mblk = n_mblk - 1 - (int)(blockIdx.x / (p.B * p.Hq));  // heaviest causal blocks first
  const int hq = bh % p.Hq, b = bh / p.Hq;
  const int hkv = hq / p.G;
  const int q0 = mblk * 2 * kBM;
  int klo, khi;
  key_range(p, q0, min(q0 + 2 * kBM, p.Sq), &klo, &khi);
  const int jlo = klo / kBN;
  const int jend = (khi > klo) ? (khi + kBN - 1) / kBN : jlo;
  // Block-sparse mask: key tile j (one 128-key block) is visited when either
  // query tile's block (q0 / 128 + t, j) is on; a tile off for one query tile
  // only is masked whole in that tile's softmax. Every role walks the visited
  // tiles in the same order with next_tile().
  const int qb0 = q0 / kMaskBlock;
  const bool two_tiles = q0 + kBM < p.Sq;
  auto tile_on = [&](int j) {
    return !BLK || block_on(p, b, hq, qb0, j) || (two_tiles && block_on(p, b, hq, qb0 + 1, j));
  };
  int n_iter = jend - jlo;
  if (BLK) {
    n_iter = 0;
    for (int j = jlo; j < jend; ++j) n_iter += tile_on(j) ? 1 : 0;
  }
  auto next_tile = [&](int j) {  // the first visited tile after j
    do { ++j; } while (BLK && j < jend && !tile_on(j));
    return j;
  };

  WaitCtl ctl{abort_flag, p.status, p.timeout_ns};

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i)
      mbar_init(bar(i), (i >= kPFull && i < kPHalf + 2) ? 4u : 1u);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      // A block that sees no key loads nothing: its epilogue stages zeros in
      // the Q tiles, which must not have a TMA write in flight.
      if (n_iter > 0) {
        mbar_arrive_expect_tx(bar(kQFull), 2 * L::kQBytes);
        for (int t = 0; t < 2; ++t)
          for (int s = 0; s < L::kSub; ++s)
            tma_load_4d(sbase + L::kOffQ + t * L::kQBytes + s * (kBM * 128), &tmQ, bar(kQFull),
                        s * 64, q0 + t * kBM, hq, b);
      }
      int n = 0;
      bool ok = true;
      int j = jlo - 1;
      for (int it = 0; it < n_iter && ok; ++it) {
        j = next_tile(j);
        for (int kv = 0; kv < 2; ++kv) {
          const int slot = n % NS;
          if (n >= NS) {
            ok = mbar_wait(bar(kKVEmpty + slot), ((n / NS) & 1) ^ 1, ctl, BFA_ERR_DEVICE_TIMEOUT);
            if (!ok) break;
          }
          mbar_arrive_expect_tx(bar(kKVFull + slot), L::kKVBytes);
          for (int s = 0; s < L::kSub; ++s)
            tma_load_4d(sbase + L::kOffKV + slot * L::kKVBytes + s * (kBN * 128), kv ? &tmV : &tmK,
                        bar(kKVFull + slot), s * 64, j * kBN, hkv, b);
          ++n;
        }
      }
      if (n_iter > 0) drain_wait(bar(kQFull), 0, p.timeout_ns);
      for (int i = (n > NS ? n - NS : 0); i < n; ++i)
        drain_wait(bar(kKVFull + i % NS), (i / NS) & 1, p.timeout_ns);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // Order: S_0(j), S_1(j), then per step PV_0(j), S_0(j+1), PV_1(j), S_1(j+1).
    // tcgen05 MMAs of one thread run in issue order, so S_t(j+1) (which
    // overwrites the TMEM holding P_t(j)) runs after PV_t(j) has read P_t(j).
    if (lane == 0) {
      constexpr uint32_t idS = idesc_f16(kBM, kBN, BF16, false);
      constexpr uint32_t idO = idesc_f16(kBM, D, BF16, true);
      auto kv_addr = [&](int idx) -> uint32_t {
        return sbase + L::kOffKV + (uint32_t)(idx % NS) * L::kKVBytes;
      };
      // Descriptors are built once per tile; a K step only moves the start
      // address (a compile-time offset added to the low field).
      auto issue_s = [&](int t, int idx) {
        const uint64_t dq = desc_kmajor(sbase + L::kOffQ + t * L::kQBytes);
        const uint64_t dk = desc_kmajor(kv_addr(idx));
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t offq = (kk >> 2) * (kBM * 128) + (kk & 3) * 32;
          const uint32_t offk = (kk >> 2) * (kBN * 128) + (kk & 3) * 32;
          mma_ss(tmem + L::kTmemS + t * kBN, dq + (offq >> 4), dk + (offk >> 4), idS,
                 kk > 0 ? 1u : 0u);
        }
        mma_commit(bar(kSFull + t));
      };
      // PV_t(j) in two halves of 64 keys: the first is issued once the
      // softmax has stored P for those keys, and runs while it forms the rest.
      auto issue_pv = [&](int t, int idx, bool acc, int half) {
        const uint64_t dv = desc_mnmajor(kv_addr(idx), kBN * 128);
#pragma unroll
        for (int k4 = 0; k4 < kBN / 32; ++k4) {
          const int kk = half * (kBN / 32) + k4;
          mma_ts(tmem + L::kTmemO + t * D, tmem + L::kTmemS + t * kBN + kk * 8,
                 dv + ((kk * 16 * 128) >> 4), idO, (acc || kk > 0) ? 1u : 0u);
        }
        if (half == 1) mma_commit(bar(kODone + t));
      };
      auto wait_pv = [&](int t, int it) {  // both halves of PV_t(it), each once its P is stored
        if (!mbar_wait(bar(kPHalf + t), it & 1, ctl, BFA_ERR_DEVICE_TIMEOUT)) return false;
        tc_fence_after();
        issue_pv(t, 2 * it + 1, it > 0, 0);
        if (!mbar_wait(bar(kPFull + t), it & 1, ctl, BFA_ERR_DEVICE_TIMEOUT)) return false;
        tc_fence_after();
        issue_pv(t, 2 * it + 1, it > 0, 1);
        return true;
      };
      auto wait_load = [&](int idx) {
        return mbar_wait(bar(kKVFull + idx % NS), (idx / NS) & 1, ctl, BFA_ERR_DEVICE_TIMEOUT);
      };
      bool ok = n_iter == 0 || mbar_wait(bar(kQFull), 0, ctl, BFA_ERR_DEVICE_TIMEOUT);
      if (ok && n_iter > 0) {
        ok = wait_load(0);
        if (ok) {
          tc_fence_after();
          issue_s(0, 0);
          issue_s(1, 0);
          mma_commit(bar(kKVEmpty + 0));
        }
        for (int it = 0; it < n_iter && ok; ++it) {
          const int iv = 2 * it + 1, ik = 2 * it + 2;
          const bool more = it + 1 < n_iter;
          if (!(ok = wait_load(iv))) break;
          if (!(ok = wait_pv(0, it))) break;
          if (more) {
            // K comes by TMA (ordered by the mbarrier); the softmax reads of
            // S_0 were ordered by the PFull wait and fence above.
            if (!(ok = wait_load(ik))) break;
            issue_s(0, ik);
          }
          if (!(ok = wait_pv(1, it))) break;
          mma_commit(bar(kKVEmpty + iv % NS));
          if (more) {
            issue_s(1, ik);
            mma_commit(bar(kKVEmpty + ik % NS));
          }
        }
      }
      mma_commit(bar(kDrain));
      drain_wait(bar(kDrain), 0, p.timeout_ns);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax
    const int t = (warp - 4) >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const int r_local = q0 + t * kBM + row;
    const int64_t gi = (int64_t)r_local + p.q_off;
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const uint32_t tS = tmem + lane_base + L::kTmemS + t * kBN;
    const uint32_t tO = tmem + lane_base + L::kTmemO + t * D;
    const float sl2 = p.scale * kLog2e;
    const float cap_in = CAP ? p.scale / p.soft_cap : 0.f;
    const float cap_out = CAP ? p.soft_cap * kLog2e : 0.f;
    const float slope = ALIBI ? p.alibi[hq] : 0.f;
    const float slope2 = slope * kLog2e;
    // ALiBi: bias slope·(g0 - j); slope·(i - g0) goes into the LSE only.
    const int64_t g0 = ALIBI ? alibi_ref(p, slope, gi, r_local < p.Sq) : gi;
    const int tr0 = q0 + t * kBM;
    float m = neg_inf(), l = 0.f;
    bool ok = true;
    // Without documents a key tile is fully kept exactly when its first key
    // lies in `kept` (no general tile test per step). Rows past Sq may share
    // a full tile: their results are not stored.
    const bool lin_full = p.doc_lo == nullptr;
    const KeptRange kept = kept_keys(p, tr0, kBM, kBN, false);

    int jt = jlo - 1;
    for (int it = 0; it < n_iter; ++it) {
      jt = next_tile(jt);
      const int c0 = jt * kBN;
      const bool blk_on = !BLK || ((t == 0 || two_tiles) && block_on(p, b, hq, qb0 + t, jt));  // this query tile's block
      // The whole 128-column S row comes into registers with four TMEM loads
      // and one wait: one TMEM round trip per step instead of one per
      // 32-column chunk and pass. Logits in base 2 (cap, ALiBi, mask) are
      // formed in place; a plain, fully kept tile only needs max(S) (the
      // scale is > 0) and folds the scale into the exponent with one FMA.
      // Four independent max accumulators (three-input max) and two packed
      // sum accumulators break the dependency chains. The step's mask
      // constants come first: they overlap the wait for S.
      const bool full = blk_on && (lin_full ? kept.has(c0) : tile_full(p, tr0, tr0 + kBM, c0, c0 + kBN));
      const bool store_x = CAP || ALIBI || !full || !(sl2 > 0.f);  // x != S * sl2
      const float abase = ALIBI ? slope2 * (float)(g0 - (int64_t)c0 - p.k_off) : 0.f;
      int clo = 0, chi = kBN;  // kept key columns [clo, chi) of this row (all of them on a full tile)
      if (!full) keys_for_query(p, gi, r_local < p.Sq && blk_on, c0, kBN, &clo, &chi);
      uint32_t wbar = bar(kSFull + t), wpar = (uint32_t)(it & 1);
      if ((p.debug_flags & BFA_DEBUG_INJECT_STALL) && t == 0 && it == 0) {
        wbar = bar(kNever);
        wpar = 0;
      }
      if (!(ok = warp_wait(wbar, wpar, ctl))) break;
      tc_fence_after();
      uint32_t r[kBN / 32][32];
#pragma unroll
      for (int ch = 0; ch < kBN / 32; ++ch) tmem_ld32(tS + 32 * ch, r[ch]);
      tmem_ld_wait();
      float mx;
      {
        float m4[4] = {neg_inf(), neg_inf(), neg_inf(), neg_inf()};
        if (!store_x) {
#pragma unroll
          for (int ch = 0; ch < kBN / 32; ++ch)
#pragma unroll
            for (int e = 0; e < 32; e += 2)
              m4[(e >> 1) & 3] = fmax3(m4[(e >> 1) & 3], __uint_as_float(r[ch][e]), __uint_as_float(r[ch][e + 1]));
        } else {
          // Logits in base 2, formed in place: cap, ALiBi, mask. The cap's
          // tanh (cap_tier, warp-uniform per step): the odd Taylor series on
          // the FMA pipe when every |s/cap| of the warp's step is <= 1/8 (to
          // u^7) or <= 1/2 (to u^11), else the closed form on MUFU; without
          // ALiBi two keys per packed instruction. The mask select runs only
          // on tiles that are not fully kept.
          auto form = [&](auto tier_tag, auto masked_tag) {
            constexpr int TIER = decltype(tier_tag)::value;
            constexpr bool MASKED = decltype(masked_tag)::value;
#pragma unroll
            for (int ch = 0; ch < kBN / 32; ++ch) {
#pragma unroll
              for (int e = 0; e < 32; e += 2) {
                const int c = 32 * ch + e;
                const float2 raw2 = make_float2(__uint_as_float(r[ch][e]), __uint_as_float(r[ch][e + 1]));
                float xv[2];
                if (CAP && !ALIBI) {
                  float2 th;
                  const float2 x2 = cap_logit2x2<TIER>(raw2, cap_in, cap_out, &th);
                  xv[0] = x2.x;
                  xv[1] = x2.y;
                } else if (ALIBI && !CAP) {
                  // ALiBi without cap, two keys per packed instruction:
                  // x = s·scale·log2(e) + (abase - slope·log2(e)·c).
                  const float2 bias = __ffma2_rn(make_float2(-slope2, -slope2), make_float2((float)c, (float)(c + 1)),
                                                 make_float2(abase, abase));
                  const float2 x2 = __ffma2_rn(raw2, make_float2(sl2, sl2), bias);
                  xv[0] = x2.x;
                  xv[1] = x2.y;
                } else {
#pragma unroll
                  for (int h = 0; h < 2; ++h) {
                    const float raw = h ? raw2.y : raw2.x;
                    float x = raw * sl2;
                    if (CAP) {
                      const float u = raw * cap_in;
                      x = cap_out * (TIER == 2 ? tanh_tiny(u) : TIER == 1 ? tanh_small(u) : tanh_any(u));
                    }
                    if (ALIBI) x = fmaf(-slope2, (float)(c + h), x + abase);
                    xv[h] = x;
                  }
                }
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  float x = xv[h];
                  if (MASKED) x = ((unsigned)(c + h - clo) < (unsigned)(chi - clo)) ? x : neg_inf();
                  r[ch][e + h] = __float_as_uint(x);
                  m4[(e + h) & 3] = fmaxf(m4[(e + h) & 3], x);
                }
              }
            }
          };
          const int tier = CAP ? cap_tier<kBN>(&r[0][0], cap_in) : 0;
          using I2 = std::integral_constant<int, 2>;
          using I1 = std::integral_constant<int, 1>;
          using I0 = std::integral_constant<int, 0>;
          // (Plain logits reach here on a full tile only with scale <= 0:
          // they keep the one masked form.)
          if ((CAP || ALIBI) && full) {
            if (tier == 2) form(I2{}, std::false_type{});
            else if (tier == 1) form(I1{}, std::false_type{});
            else form(I0{}, std::false_type{});
          } else {
            if (tier == 2) form(I2{}, std::true_type{});
            else if (tier == 1) form(I1{}, std::true_type{});
            else form(I0{}, std::true_type{});
          }
        }
        mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        if (!store_x) mx *= sl2;
      }
      // Raise the reference max only when it grows by more than the threshold
      // (or is still -inf); the decision is warp-uniform because the O rescale
      // uses warp-collective TMEM loads/stores.
      const bool grow = (mx > m + kRescaleThreshold) || (m == neg_inf() && mx != neg_inf());
      const bool rescale = __any_sync(0xffffffffu, grow) && it > 0;
      float m_new = m;
      if (__any_sync(0xffffffffu, grow)) m_new = fmaxf(m, mx);
      const float m_use = (m_new == neg_inf()) ? 0.f : m_new;
      const float alpha = ex2(m - m_use);
      // P = 2^(x - m) packed to 16 bits over the first 64 columns of the S
      // region (the row is already in registers). The softmax warps share
      // each sub-partition's issue slots with the single thread that issues
      // the MMAs, and a warp with a long run of ready FMA-pipe instructions
      // starves it (measured: MMA steps up to 3x slower). So x and the row
      // sums are formed in packed pairs (one fma.f32x2 / add.f32x2 per two
      // keys); on a fully kept tile every kPolyEvery-th exponential runs on
      // the FMA pipe (ex2_poly) to unload the MUFU unit.
      float2 s2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      const float2 xs2 = make_float2(store_x ? 1.f : sl2, store_x ? 1.f : sl2);
      const float2 nm2 = make_float2(-m_use, -m_use);
      auto exps = [&](auto split) {
        constexpr bool SPLIT = decltype(split)::value && kPolyEvery > 0;
#pragma unroll
        for (int ch = 0; ch < kBN / 32; ++ch) {
          if (ch == 2) {  // P of keys [0, 64) is stored: the first PV half may start
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kPHalf + t));
          }
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float2 x = __ffma2_rn(make_float2(__uint_as_float(r[ch][e]), __uint_as_float(r[ch][e + 1])), xs2, nm2);
            const float p0 = ex2(x.x);
            const float p1 = (SPLIT && e % kPolyEvery == kPolyEvery - 2) ? ex2_poly(x.y) : ex2(x.y);
            s2[(e >> 1) & 1] = __fadd2_rn(s2[(e >> 1) & 1], make_float2(p0, p1));
            pk[e / 2] = pack2<BF16>(p0, p1);
          }
          tmem_st16(tS + 16 * ch, pk);
        }
      };
      // O_t is rescaled (rarely) before the first PV half may read it.
      if (it > 0) {
        // PV_t(it-1) is complete (its commit precedes S_t(it)'s), so O_t is stable.
        if (!(ok = warp_wait(bar(kODone + t), (uint32_t)((it - 1) & 1), ctl))) break;
        tc_fence_after();
        if (rescale) {
          // 16 columns at a time: the S row is still live in registers.
#pragma unroll 1
          for (int c = 0; c < D / 16; ++c) {
            uint32_t o16[16];
            tmem_ld16(tO + 16 * c, o16);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) o16[i] = __float_as_uint(__uint_as_float(o16[i]) * alpha);
            tmem_st16(tO + 16 * c, o16);
          }
        }
      }
      if (full) exps(std::true_type{});
      else exps(std::false_type{});
      const float rs = (s2[0].x + s2[0].y) + (s2[1].x + s2[1].y);
      l = l * alpha + rs;
      m = m_new;
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kPFull + t));
    }

    // ------------------------------------------------------------ epilogue
    bool good = ok;
    if (good && n_iter > 0) good = warp_wait(bar(kODone + t), (uint32_t)((n_iter - 1) & 1), ctl);
    // Q_t's smem tile is free once the last S_t MMA has run; it stages O_t.
    uint8_t* Ot = smem + L::kOffQ + t * L::kQBytes;
    // This row's LSE (natural log); -inf when it sees no key.
    const float lse_row = (l > 0.f) ? fmaf(slope, (float)(gi - g0), (m + lg2(l)) * kLn2) : neg_inf();
    if (good && p.out_acc) {
      // Merge into the running fp32 output and LSE (bfa_fwd_args.accumulate):
      // each thread owns its row, so it reads and rewrites it directly, 16
      // bytes at a time. The TMEM loads are warp-collective: every lane takes
      // part, rows past Sq skip only the memory accesses.
      tc_fence_after();
      const bool live = r_local < p.Sq;
      float* lse_p = p.lse + ((int64_t)b * p.Hq + hq) * p.Sq + r_local;
      const MergeWeights w = merge_weights(live ? *lse_p : neg_inf(), lse_row);
      const float sp = (l > 0.f) ? w.wp / l : 0.f;
      float* orow = (float*)p.o + (int64_t)b * p.so_[0] + (int64_t)hq * p.so_[1] + (int64_t)r_local * p.so_[2];
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        if (n_iter > 0) {
          tmem_ld32(tO + 32 * c, r);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = 0u;
        }
        if (live) {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            float4* dst = reinterpret_cast<float4*>(orow + 32 * c + 4 * q);
            float4 a = w.wa != 0.f ? *dst : make_float4(0.f, 0.f, 0.f, 0.f);
            a.x = fmaf(__uint_as_float(r[4 * q + 0]), sp, a.x * w.wa);
            a.y = fmaf(__uint_as_float(r[4 * q + 1]), sp, a.y * w.wa);
            a.z = fmaf(__uint_as_float(r[4 * q + 2]), sp, a.z * w.wa);
            a.w = fmaf(__uint_as_float(r[4 * q + 3]), sp, a.w * w.wa);
            *dst = a;
          }
        }
      }
      if (live) *lse_p = w.ln;
    } else if (good) {
      tc_fence_after();
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        if (n_iter > 0) {
          tmem_ld32(tO + 32 * c, r);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = 0u;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 v;
          v.x = pack2<BF16>(__uint_as_float(r[8 * q + 0]) * inv, __uint_as_float(r[8 * q + 1]) * inv);
          v.y = pack2<BF16>(__uint_as_float(r[8 * q + 2]) * inv, __uint_as_float(r[8 * q + 3]) * inv);
          v.z = pack2<BF16>(__uint_as_float(r[8 * q + 4]) * inv, __uint_as_float(r[8 * q + 5]) * inv);
          v.w = pack2<BF16>(__uint_as_float(r[8 * q + 6]) * inv, __uint_as_float(r[8 * q + 7]) * inv);
          const int col = 32 * c + 8 * q;
          *reinterpret_cast<uint4*>(Ot + (col >> 6) * (kBM * 128) + sw128_offset(row, (col & 63) >> 3)) = v;
        }
      }
      fence_async_shared();
    }
    if (lane == 0) warp_ok[warp - 4] = good ? 1 : 0;
    named_sync(1 + t, 128);
    if (wq == 0 && lane == 0 && !p.out_acc) {
      const bool all = warp_ok[4 * t] && warp_ok[4 * t + 1] && warp_ok[4 * t + 2] && warp_ok[4 * t + 3];
      if (all) {
        for (int s = 0; s < L::kSub; ++s)
          tma_store_4d(&tmO, smem_u32(Ot) + s * (kBM * 128), s * 64, tr0, hq, b);
        tma_store_commit();
        tma_store_wait_all();
      }
    }
    if (good && r_local < p.Sq && !p.out_acc) p.lse[((int64_t)b * p.Hq + hq) * p.Sq + r_local] = lse_row;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D, bool BF16, bool CAP, bool ALIBI, bool BLK>
int launch_fwd(const Params& p, const Tmaps4& tm, cudaStream_t st) {
  using L = FwdLayout<D>;
  auto kern = fwd_kernel<D, BF16, CAP, ALIBI, BLK>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)L::kSmemBytes);
  });
  if (attr_err != cudaSuccess) return cuda_fail("fwd_kernel shared-memory attribute", attr_err);
  const int n_mblk = (p.Sq + 2 * kBM - 1) / (2 * kBM);
  const unsigned grid = (unsigned)n_mblk * (unsigned)p.B * (unsigned)p.Hq;
  kern<<<grid, kThreads, L::kSmemBytes, st>>>(tm.m[0], tm.m[1], tm.m[2], tm.m[3], p);
  note_launch();
  return launch_status("fwd_kernel launch");
}

template <int D, bool BF16, bool BLK>
int dispatch_cap(const Params& p, const Tmaps4& tm, cudaStream_t st) {
  const bool cap = p.soft_cap > 0.f, alibi = p.alibi != nullptr;
  if (cap && alibi) return launch_fwd<D, BF16, true, true, BLK>(p, tm, st);
  if (cap) return launch_fwd<D, BF16, true, false, BLK>(p, tm, st);
  if (alibi) return launch_fwd<D, BF16, false, true, BLK>(p, tm, st);
  return launch_fwd<D, BF16, false, false, BLK>(p, tm, st);
}

template <int D, bool BF16>
int dispatch_flags(const Params& p, const Tmaps4& tm, cudaStream_t st) {
  return p.blk ? dispatch_cap<D, BF16, true>(p, tm, st) : dispatch_cap<D, BF16, false>(p, tm, st);
}

}  // namespace

bool sm100_fwd_eligible(const Params& p, int dtype) {
  if (dtype != BFA_DTYPE_BF16 && dtype != BFA_DTYPE_F16) return false;
  if (p.D != 64 && p.D != 128 && p.D != 256) return false;
  if (p.Sq < 1 || p.Sk < 1 || p.B < 1 || p.Hq < 1) return false;
  if (!device_is_sm100()) return false;
  // A merging call's fp32 output is read and written 16 bytes at a time.
  return tma_layout_ok(p.q, p.sq_, 2) && tma_layout_ok(p.k, p.sk_, 2) &&
         tma_layout_ok(p.v, p.sv_, 2) && tma_layout_ok(p.o, p.so_, p.out_acc ? 4 : 2);
}

int sm100_fwd(const Params& p, int dtype, cudaStream_t st) {
  if (p.D == 256) return sm100_fwd256(p, dtype, st);
  Tmaps4 tm;
  if (!make_tmap_bhsd(&tm.m[0], p.q, dtype, p.D, p.Sq, p.Hq, p.B, p.sq_, kBM) ||
      !make_tmap_bhsd(&tm.m[1], p.k, dtype, p.D, p.Sk, p.Hkv, p.B, p.sk_, kBN) ||
      !make_tmap_bhsd(&tm.m[2], p.v, dtype, p.D, p.Sk, p.Hkv, p.B, p.sv_, kBN) ||
      !(p.out_acc ? (tm.m[3] = tm.m[0], true)  // no TMA store of O when merging
                  : make_tmap_bhsd(&tm.m[3], p.o, dtype, p.D, p.Sq, p.Hq, p.B, p.so_, kBM)))
    return simt_fwd(p, dtype, st);
  const bool bf16 = dtype == BFA_DTYPE_BF16;
  if (p.D == 64) return bf16 ? dispatch_flags<64, true>(p, tm, st) : dispatch_flags<64, false>(p, tm, st);
  return bf16 ? dispatch_flags<128, true>(p, tm, st) : dispatch_flags<128, false>(p, tm, st);
}

}  // namespace bfa
