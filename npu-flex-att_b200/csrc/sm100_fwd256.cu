// sm100_fwd256.cu -- tcgen05 / TMA / TMEM flash-attention forward for
// head_dim 256 (bf16 / fp16), e.g. Gemma2-style layers.
//
// Same math as flash_attn_fwd_kernel (npu_flash_attention.py:17-166) with
// HEAD_DIM = 256: S = QKᵀ·scale, optional soft-cap (:105-106) then ALiBi
// (:108-109), causal / window masks (:139, :141), online softmax in base 2,
// O = PV / l, LSE = m + ln(l) in natural log (:161).
//
// Why a separate kernel: at D = 256 one 128-row query tile needs O in 256
// TMEM columns and its two S buffers in the other 256, so a CTA owns ONE
// query tile (the D <= 128 kernel owns two), and a 128-key K or V tile is
// 64 KB, so K and V stream through a ring of 32 KB units in the order the
// MMAs consume them:
//   S(0): K0[dims 0-127], K0[dims 128-255]   S(1): K1 lo, K1 hi
//   PV(0): V0[keys 0-63], V0[keys 64-127]    S(2): K2 lo, K2 hi   PV(1) ...
// Warp roles (384 threads):
//   warp 0      TMA producer: Q once (64 KB), then the ring units
//   warp 1      MMA issuer: S(j) = Q K_jᵀ (M=128, N=128, 16 K-steps), and
//               O += P(j) V_j (M=128, N=256, TS form: P read from TMEM)
//   warp 2      TMEM allocator (512 columns: S0, S1, O)
//   warps 4-11  softmax, two warpgroups over the same 128 query rows (one
//               TMEM lane per thread): warpgroup h reads keys [64h, 64h + 64)
//               of the S row, the two exchange the row maximum, and each
//               writes its P (16-bit) into packed columns [32h, 32h + 32) of
//               that S buffer and rescales O columns [128h, 128h + 128) when
//               the running max grows by more than 2^8; then O and the LSE.
// MMA order S(0), S(1), PV(0), S(2), PV(1), S(3), ...: the softmax of step j
// overlaps PV(j-1) and S(j+1) on the tensor core.
//
// Soft-cap: the reference's logits are cap·tanh(s/cap). With N(0,1)-scale
// logits |s/cap| is small, and tanh there is evaluated on the FMA pipe by its
// odd Taylor series to u^11 (truncation error < 1e-6 relative for |u| <= 1/2),
// which leaves the MUFU unit to the exponentials. A step whose raw logits of
// some row in the warp reach |s/cap| > 1/2 uses tanh_any, the closed form
// 1 - 2/(1 + e^{2u}) (warp-uniform choice per step).
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

constexpr int kD = 256;
constexpr int kBM = 128;  // query rows per CTA (TMEM lanes)
constexpr int kBN = 128;  // keys per step
constexpr int kThreads = 384;
constexpr int kStages = 4;                        // ring units in flight
constexpr uint32_t kUnitBytes = 32768;            // one ring unit
constexpr uint32_t kQSub = kBM * 128;             // [128 rows][64 dims], 128-byte swizzle
constexpr uint32_t kQBytes = 4 * kQSub;           // 64 KB
constexpr uint32_t kKSub = kBN * 128;             // [128 keys][64 dims]
constexpr uint32_t kVSub = 64 * 128;              // [64 keys][64 dims]
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffRing = kQBytes;
constexpr uint32_t kOffX = kOffRing + kStages * kUnitBytes;  // row-maximum exchange, 2 KB
constexpr uint32_t kOffBar = kOffX + 2 * 2 * kBM * 4;
constexpr uint32_t kSmemBytes = kOffBar + 512 + 1024;
constexpr uint32_t kTmemS = 0;       // S(b) at 128·b, fp32; P(b) packed over its first 64 columns
constexpr uint32_t kTmemO = 2 * kBN; // O: 256 fp32 columns
constexpr float kRescaleThreshold = 8.0f;
constexpr int kPolyEvery = 8;
static_assert(kSmemBytes <= 232448, "smem budget");
static_assert(2 * kKSub == kUnitBytes && 4 * kVSub == kUnitBytes, "ring unit");

// Taylor coefficients of tanh(u)/u in z = u^2 (the series of tanh).
constexpr float kT1 = -1.0f / 3.0f;
constexpr float kT2 = 2.0f / 15.0f;
constexpr float kT3 = -17.0f / 315.0f;
constexpr float kT4 = 62.0f / 2835.0f;
constexpr float kT5 = -1382.0f / 155925.0f;

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

// Calls f(op, j) for the MMA operations in issue order: op 0 = S(j), op 1 = PV(j).
template <typename F>
__device__ __forceinline__ bool for_each_op(int n_iter, F&& f) {
  for (int j = 0; j < n_iter; ++j) {
    if (j == 0) {
      if (!f(0, 0)) return false;
      if (n_iter > 1 && !f(0, 1)) return false;
    }
    if (!f(1, j)) return false;
    if (j + 2 < n_iter && !f(0, j + 2)) return false;
  }
  return true;
}

template <bool BF16, bool CAP, bool ALIBI>
__global__ void __launch_bounds__(kThreads, 1)
    fwd256_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                  const Params p) {
  constexpr int NS = kStages;
  enum {
    kQFull = 0,
    kFull = 1,
    kEmpty = 1 + NS,
    kSFull = 1 + 2 * NS,
    kPFull = kSFull + 2,
    kODone = kPFull + 2,
    kXch = kODone + 1,  // row-maximum exchange of parity b (8 softmax warps)
    kXchL = kXch + 2,   // row-sum exchange in the epilogue (8 softmax warps)
    kDrain = kXchL + 1,
    kNever = kDrain + 1,
    kNumBars = kNever + 1
  };

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  auto bar = [&](int i) -> uint32_t { return sbase + kOffBar + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = (uint32_t*)(smem + kOffBar + 8 * kNumBars);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  int* warp_ok = (int*)(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (p.Sq + kBM - 1) / kBM;
  const int bh = blockIdx.x % (p.B * p.Hq);
  const int qt = n_qt - 1 - (int)(blockIdx.x / (p.B * p.Hq));  // heaviest causal tiles first
  const int hq = bh % p.Hq, b = bh / p.Hq;
  const int hkv = hq / p.G;
  const int q0 = qt * kBM;
  int klo, khi;
  key_range(p, q0, min(q0 + kBM, p.Sq), &klo, &khi);
  const int jlo = klo / kBN;
  const int jend = (khi > klo) ? (khi + kBN - 1) / kBN : jlo;
  // Block-sparse mask: key tile j (one 128-key block) is visited only when
  // block (q0 / 128, j) is on. Step j of the loops below is the j-th visited
  // tile; each consumer walks them with its own walker.
  int n_iter = jend - jlo;
  if (p.blk) {
    n_iter = 0;
    for (int j = jlo; j < jend; ++j) n_iter += block_on(p, b, hq, q0 / kMaskBlock, j) ? 1 : 0;
  }
  auto next_tile = [&](int j) {
    do { ++j; } while (p.blk && j < jend && !block_on(p, b, hq, q0 / kMaskBlock, j));
    return j;
  };

  WaitCtl ctl{abort_flag, p.status, p.timeout_ns};

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i)
      mbar_init(bar(i), ((i >= kPFull && i < kPFull + 2) || (i >= kXch && i <= kXchL)) ? 8u : 1u);
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
  auto unit_addr = [&](int n) -> uint32_t { return sbase + kOffRing + (uint32_t)(n % NS) * kUnitBytes; };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      // A tile that sees no key loads nothing: its epilogue stages zeros in
      // the Q tile, which must not have a TMA write in flight.
      if (n_iter > 0) {
        mbar_arrive_expect_tx(bar(kQFull), kQBytes);
        for (int s = 0; s < 4; ++s)
          tma_load_4d(sbase + kOffQ + s * kQSub, &tmQ, bar(kQFull), s * 64, q0, hq, b);
      }
      int n = 0;
      auto walk_s = make_walker(next_tile, jlo - 1), walk_pv = make_walker(next_tile, jlo - 1);
      for_each_op(n_iter, [&](int op, int j) -> bool {
        const int key0 = (op == 0 ? walk_s.step(j) : walk_pv.step(j)) * kBN;
        for (int h = 0; h < 2; ++h, ++n) {
          const int slot = n % NS;
          if (n >= NS && !mbar_wait(bar(kEmpty + slot), ((n / NS) & 1) ^ 1, ctl, BFA_ERR_DEVICE_TIMEOUT))
            return false;
          mbar_arrive_expect_tx(bar(kFull + slot), kUnitBytes);
          const uint32_t dst = unit_addr(n);
          if (op == 0) {  // K, dims [128h, 128h + 128)
            for (int s = 0; s < 2; ++s)
              tma_load_4d(dst + s * kKSub, &tmK, bar(kFull + slot), (2 * h + s) * 64, key0, hkv, b);
          } else {  // V, keys [64h, 64h + 64), all dims
            for (int s = 0; s < 4; ++s)
              tma_load_4d(dst + s * kVSub, &tmV, bar(kFull + slot), s * 64, key0 + 64 * h, hkv, b);
          }
        }
        return true;
      });
      if (n_iter > 0) drain_wait(bar(kQFull), 0, p.timeout_ns);
      for (int i = (n > NS ? n - NS : 0); i < n; ++i)
        drain_wait(bar(kFull + i % NS), (i / NS) & 1, p.timeout_ns);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_f16(kBM, kBN, BF16, false);
      constexpr uint32_t idO = idesc_f16(kBM, kD, BF16, true);
      const uint64_t dq0 = desc_kmajor(sbase + kOffQ);
      int n = 0;
      bool ok = n_iter == 0 || mbar_wait(bar(kQFull), 0, ctl, BFA_ERR_DEVICE_TIMEOUT);
      if (ok) {
        for_each_op(n_iter, [&](int op, int j) -> bool {
          const int bf = j & 1;
          if (op == 1) {
            // P(j) is in TMEM (and O rescaled) once the softmax arrives.
            if (!(ok = mbar_wait(bar(kPFull + bf), (j >> 1) & 1, ctl, BFA_ERR_DEVICE_TIMEOUT))) return false;
            tc_fence_after();
          }
          for (int h = 0; h < 2; ++h, ++n) {
            if (!(ok = mbar_wait(bar(kFull + n % NS), (n / NS) & 1, ctl, BFA_ERR_DEVICE_TIMEOUT))) return false;
            tc_fence_after();
            const uint32_t u = unit_addr(n);
            if (op == 0) {
              const uint64_t dk = desc_kmajor(u);
#pragma unroll
              for (int kk = 0; kk < 8; ++kk) {
                const int kq = 8 * h + kk;  // K-step over the 256 dims
                const uint32_t offq = ((kq >> 2) * kQSub + (kq & 3) * 32) >> 4;
                const uint32_t offk = ((kk >> 2) * kKSub + (kk & 3) * 32) >> 4;
                mma_ss(tmem + kTmemS + bf * kBN, dq0 + offq, dk + offk, idS, kq > 0 ? 1u : 0u);
              }
            } else {
              const uint64_t dv = desc_mnmajor(u, kVSub);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                const int kp = 4 * h + kk;  // K-step over the 128 keys
                mma_ts(tmem + kTmemO, tmem + kTmemS + bf * kBN + kp * 8, dv + ((kk * 2048) >> 4), idO,
                       (j > 0 || kp > 0) ? 1u : 0u);
              }
            }
            mma_commit(bar(kEmpty + n % NS));
          }
          mma_commit(bar(op == 0 ? kSFull + bf : kODone));
          return true;
        });
      }
      mma_commit(bar(kDrain));
      drain_wait(bar(kDrain), 0, p.timeout_ns);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax
    // Two warpgroups split every step's 128 keys: warpgroup h forms and
    // exponentiates keys [64h, 64h + 64) and rescales O columns
    // [128h, 128h + 128) of the same 128 rows (lane = row in both). They
    // exchange each row's partial maximum through shared memory, so both
    // derive the same running maximum; each keeps its partial row sum.
    const int eg = (warp - 4) >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const int r_local = q0 + row;
    const int64_t gi = (int64_t)r_local + p.q_off;
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const uint32_t tO = tmem + lane_base + kTmemO + 128 * eg;
    float* xchg = (float*)(smem + kOffX);  // [parity][warpgroup][row]
    const float sl2 = p.scale * kLog2e;
    const float cap_in = CAP ? p.scale / p.soft_cap : 0.f;
    const float cap_out = CAP ? p.soft_cap * kLog2e : 0.f;
    const float slope = ALIBI ? p.alibi[hq] : 0.f;
    const float slope2 = slope * kLog2e;
    // ALiBi: bias slope·(g0 - j); slope·(i - g0) goes into the LSE only.
    const int64_t g0 = ALIBI ? alibi_ref(p, slope, gi, r_local < p.Sq) : gi;
    // cap_out · tanh(u) = u · (c0 + z (c1 + z (c2 + ...))), z = u^2.
    const float c0 = cap_out, c1 = cap_out * kT1, c2 = cap_out * kT2, c3 = cap_out * kT3,
                c4 = cap_out * kT4, c5 = cap_out * kT5;
    float m = neg_inf(), l = 0.f;
    bool ok = true;
    // Without documents a key tile is fully kept exactly when its first key
    // lies in `kept` (no general tile test per step). Rows past Sq may share
    // a full tile: their results are not stored.
    const bool lin_full = p.doc_lo == nullptr;
    const KeptRange kept = kept_keys(p, q0, kBM, kBN, false);

    int jt = jlo - 1;
    for (int it = 0; it < n_iter; ++it) {
      const int bf = it & 1;
      jt = next_tile(jt);
      const int c0k = jt * kBN;
      const uint32_t tS = tmem + lane_base + kTmemS + bf * kBN;
      uint32_t wbar = bar(kSFull + bf), wpar = (uint32_t)((it >> 1) & 1);
      if ((p.debug_flags & BFA_DEBUG_INJECT_STALL) && it == 0) {
        wbar = bar(kNever);
        wpar = 0;
      }
      if (!(ok = warp_wait(wbar, wpar, ctl))) break;
      tc_fence_after();

      const bool full = lin_full ? kept.has(c0k) : tile_full(p, q0, q0 + kBM, c0k, c0k + kBN);
      const bool store_x = CAP || ALIBI || !full || !(sl2 > 0.f);  // x != S * sl2
      const float abase = ALIBI ? slope2 * (float)(g0 - (int64_t)c0k - p.k_off) : 0.f;
      int clo = 0, chi = kBN;  // kept key columns [clo, chi) of this row (all of them on a full tile)
      if (!full) keys_for_query(p, gi, r_local < p.Sq, c0k, kBN, &clo, &chi);
      uint32_t r[2][32];  // this warpgroup's keys [64h, 64h + 64)
      tmem_ld32(tS + 64 * eg, r[0]);
      tmem_ld32(tS + 64 * eg + 32, r[1]);
      tmem_ld_wait();

      float pm;  // partial maximum over this warpgroup's keys
      {
        float m4[4] = {neg_inf(), neg_inf(), neg_inf(), neg_inf()};
        if (!store_x) {
#pragma unroll
          for (int ch = 0; ch < 2; ++ch)
#pragma unroll
            for (int e = 0; e < 32; e += 2)
              m4[(e >> 1) & 3] = fmax3(m4[(e >> 1) & 3], __uint_as_float(r[ch][e]), __uint_as_float(r[ch][e + 1]));
        } else {
          // Logits in base 2, formed in place: cap, ALiBi, mask. The cap's
          // tanh: the odd Taylor series on the FMA pipe when every |s/cap| of
          // the warp's step is <= 1/2 (to u^11), or <= 1/8 (to u^7, below
          // 2e-9 relative there), else the closed form on MUFU; the mask
          // select only on tiles that are not fully kept.
          auto form = [&](auto poly_tag, auto tiny_tag, auto masked_tag) {
            constexpr bool POLY = decltype(poly_tag)::value;
            constexpr bool TINY = decltype(tiny_tag)::value;
            constexpr bool MASKED = decltype(masked_tag)::value;
#pragma unroll
            for (int ch = 0; ch < 2; ++ch) {
#pragma unroll
              for (int e = 0; e < 32; e += 2) {
                const int c = 64 * eg + 32 * ch + e;
                float2 x2;
                const float2 raw2 = make_float2(__uint_as_float(r[ch][e]), __uint_as_float(r[ch][e + 1]));
                if (CAP) {
                  const float2 u = __fmul2_rn(raw2, make_float2(cap_in, cap_in));
                  if (POLY && TINY) {
                    const float2 z = __fmul2_rn(u, u);
                    float2 q = __ffma2_rn(z, make_float2(c3, c3), make_float2(c2, c2));
                    q = __ffma2_rn(z, q, make_float2(c1, c1));
                    q = __ffma2_rn(z, q, make_float2(c0, c0));
                    x2 = __fmul2_rn(u, q);
                  } else if (POLY) {
                    const float2 z = __fmul2_rn(u, u);
                    float2 q = __ffma2_rn(z, make_float2(c5, c5), make_float2(c4, c4));
                    q = __ffma2_rn(z, q, make_float2(c3, c3));
                    q = __ffma2_rn(z, q, make_float2(c2, c2));
                    q = __ffma2_rn(z, q, make_float2(c1, c1));
                    q = __ffma2_rn(z, q, make_float2(c0, c0));
                    x2 = __fmul2_rn(u, q);
                  } else {
                    x2 = make_float2(cap_out * tanh_any(u.x), cap_out * tanh_any(u.y));
                  }
                } else {
                  x2 = __fmul2_rn(raw2, make_float2(sl2, sl2));
                }
                float xv[2] = {x2.x, x2.y};
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  float x = xv[h];
                  if (ALIBI) x = fmaf(-slope2, (float)(c + h), x + abase);
                  if (MASKED) x = ((unsigned)(c + h - clo) < (unsigned)(chi - clo)) ? x : neg_inf();
                  r[ch][e + h] = __float_as_uint(x);
                  m4[(e + h) & 3] = fmaxf(m4[(e + h) & 3], x);
                }
              }
            }
          };
          int tier = 0;  // 2: |s/cap| <= 1/8 for the whole warp, 1: <= 1/2, 0: larger
          if (CAP) {
            float am = 0.f;
#pragma unroll
            for (int ch = 0; ch < 2; ++ch)
#pragma unroll
              for (int e = 0; e < 32; e += 2)
                am = fmax3(am, fabsf(__uint_as_float(r[ch][e])), fabsf(__uint_as_float(r[ch][e + 1])));
            am *= cap_in;
            tier = __all_sync(0xffffffffu, am <= 0.125f) ? 2 : __all_sync(0xffffffffu, am <= 0.5f) ? 1 : 0;
          }
          using T_ = std::true_type;
          using F_ = std::false_type;
          if (full) {
            if (tier == 2) form(T_{}, T_{}, F_{});
            else if (tier == 1) form(T_{}, F_{}, F_{});
            else form(F_{}, F_{}, F_{});
          } else {
            if (tier == 2) form(T_{}, T_{}, T_{});
            else if (tier == 1) form(T_{}, F_{}, T_{});
            else form(F_{}, F_{}, T_{});
          }
        }
        pm = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        if (!store_x) pm *= sl2;
      }
      // The row maximum over both halves, through shared memory and an
      // mbarrier (a bounded wait: a warpgroup that gave up cannot strand the
      // other one). The other warpgroup has loaded its S columns once it has
      // arrived, so P may then be written over them. Two parity buffers: a
      // slot is rewritten two steps later, after the other warpgroup has
      // arrived in between, i.e. read it.
      xchg[(bf * 2 + eg) * kBM + row] = pm;
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kXch + bf));
      if (!(ok = warp_wait(bar(kXch + bf), (uint32_t)((it >> 1) & 1), ctl))) break;
      const float mx = fmaxf(pm, xchg[(bf * 2 + (eg ^ 1)) * kBM + row]);
      // Raise the reference max only when it grows by more than the
      // threshold (or is still -inf); warp-uniform, because the O rescale
      // uses warp-collective TMEM loads / stores. Both warpgroups see the
      // same maxima for the same 32 rows, so they decide alike.
      const bool grow = (mx > m + kRescaleThreshold) || (m == neg_inf() && mx != neg_inf());
      const bool any_grow = __any_sync(0xffffffffu, grow);
      const bool rescale = any_grow && it > 0;
      float m_new = m;
      if (any_grow) m_new = fmaxf(m, mx);
      const float m_use = (m_new == neg_inf()) ? 0.f : m_new;
      const float alpha = ex2(m - m_use);
      float2 s2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      const float2 xs2 = make_float2(store_x ? 1.f : sl2, store_x ? 1.f : sl2);
      const float2 nm2 = make_float2(-m_use, -m_use);
      auto exps = [&](auto split) {
        constexpr bool SPLIT = decltype(split)::value && kPolyEvery > 0;
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float2 x = __ffma2_rn(make_float2(__uint_as_float(r[ch][e]), __uint_as_float(r[ch][e + 1])), xs2, nm2);
            const float p0 = ex2(x.x);
            const float p1 = (SPLIT && e % kPolyEvery == kPolyEvery - 2) ? ex2_poly(x.y) : ex2(x.y);
            s2[(e >> 1) & 1] = __fadd2_rn(s2[(e >> 1) & 1], make_float2(p0, p1));
            pk[e / 2] = pack2<BF16>(p0, p1);
          }
          // Keys [64h + 32ch, +32) -> packed columns [32h + 16ch, +16).
          tmem_st16(tS + 32 * eg + 16 * ch, pk);
        }
      };
      if (full) exps(std::true_type{});
      else exps(std::false_type{});
      const float rs = (s2[0].x + s2[0].y) + (s2[1].x + s2[1].y);
      l = l * alpha + rs;
      m = m_new;
      if (it > 0) {
        // Wait for PV(it-1) every step, so the ODone phases and this parity
        // wait stay in lockstep (and O is stable for a rescale). It costs
        // nothing in the steady state: PV(it-1) runs right after S(it), and
        // PV(it) cannot start before S(it+1), issued after PV(it-1), is done.
        if (!(ok = warp_wait(bar(kODone), (uint32_t)((it - 1) & 1), ctl))) break;
        tc_fence_after();
      }
      if (rescale) {
#pragma unroll 1
        for (int c = 0; c < 128 / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + 32 * c, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tO + 32 * c, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kPFull + bf));
    }

    // ------------------------------------------------------------ epilogue
    // Row sum: the two partial sums, exchanged through the parity buffer the
    // last step did not use (the other warpgroup read it before arriving at
    // that step's exchange), with a bounded wait.
    bool good = ok;
    if (good && n_iter > 0) good = warp_wait(bar(kODone), (uint32_t)((n_iter - 1) & 1), ctl);
    const int lp = (n_iter & 1) * 2;
    xchg[(lp + eg) * kBM + row] = l;
    __syncwarp();
    if (lane == 0) mbar_arrive(bar(kXchL));
    good = warp_wait(bar(kXchL), 0, ctl) && good;
    const float l_tot = l + xchg[(lp + (eg ^ 1)) * kBM + row];
    // The Q tile is free once the last S MMA has run (MMAs complete in
    // order, and PV(n-1) came after it): it stages O, warpgroup h its
    // columns [128h, 128h + 128) (sub-tiles 2h, 2h + 1).
    uint8_t* Ot = smem + kOffQ;
    // This row's LSE (natural log); -inf when it sees no key.
    const float lse_row =
        (l_tot > 0.f) ? fmaf(slope, (float)(gi - g0), (m + lg2(l_tot)) * kLn2) : neg_inf();
    float* lse_p = p.lse + ((int64_t)b * p.Hq + hq) * p.Sq + r_local;
    const bool live = r_local < p.Sq;
    MergeWeights mw{0.f, 0.f, neg_inf()};
    if (good && p.out_acc) {
      // Merge into the running fp32 output and LSE (bfa_fwd_args.accumulate):
      // each thread reads and rewrites its row's 128 columns directly, 16
      // bytes at a time; both warpgroups read the running LSE before the
      // barrier below, after which warpgroup 0 rewrites it. The TMEM loads
      // are warp-collective: rows past Sq skip only the memory accesses.
      tc_fence_after();
      mw = merge_weights(live ? *lse_p : neg_inf(), lse_row);
      const float sp = (l_tot > 0.f) ? mw.wp / l_tot : 0.f;
      float* orow = (float*)p.o + (int64_t)b * p.so_[0] + (int64_t)hq * p.so_[1] +
                    (int64_t)r_local * p.so_[2] + 128 * eg;
#pragma unroll 1
      for (int c = 0; c < 128 / 32; ++c) {
        uint32_t o[32];
        if (n_iter > 0) {
          tmem_ld32(tO + 32 * c, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
        if (live) {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            float4* dst = reinterpret_cast<float4*>(orow + 32 * c + 4 * q);
            float4 a = mw.wa != 0.f ? *dst : make_float4(0.f, 0.f, 0.f, 0.f);
            a.x = fmaf(__uint_as_float(o[4 * q + 0]), sp, a.x * mw.wa);
            a.y = fmaf(__uint_as_float(o[4 * q + 1]), sp, a.y * mw.wa);
            a.z = fmaf(__uint_as_float(o[4 * q + 2]), sp, a.z * mw.wa);
            a.w = fmaf(__uint_as_float(o[4 * q + 3]), sp, a.w * mw.wa);
            *dst = a;
          }
        }
      }
    } else if (good) {
      tc_fence_after();
      const float inv = (l_tot > 0.f) ? 1.f / l_tot : 0.f;
#pragma unroll 1
      for (int c = 0; c < 128 / 32; ++c) {
        uint32_t o[32];
        if (n_iter > 0) {
          tmem_ld32(tO + 32 * c, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 v;
          v.x = pack2<BF16>(__uint_as_float(o[8 * q + 0]) * inv, __uint_as_float(o[8 * q + 1]) * inv);
          v.y = pack2<BF16>(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv);
          v.z = pack2<BF16>(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv);
          v.w = pack2<BF16>(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv);
          const int col = 128 * eg + 32 * c + 8 * q;
          *reinterpret_cast<uint4*>(Ot + (col >> 6) * kQSub + sw128_offset(row, (col & 63) >> 3)) = v;
        }
      }
      fence_async_shared();
    }
    if (lane == 0) warp_ok[warp - 4] = good ? 1 : 0;
    named_sync(3, 256);
    if (warp == 4 && lane == 0 && !p.out_acc) {
      bool all = true;
      for (int w = 0; w < 8; ++w) all = all && warp_ok[w];
      if (all) {
        for (int s = 0; s < 4; ++s) tma_store_4d(&tmO, smem_u32(Ot) + s * kQSub, s * 64, q0, hq, b);
        tma_store_commit();
        tma_store_wait_all();
      }
    }
    if (good && eg == 0 && live) *lse_p = p.out_acc ? mw.ln : lse_row;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <bool BF16, bool CAP, bool ALIBI>
int launch(const Params& p, const Tmaps4& tm, cudaStream_t st) {
  auto kern = fwd256_kernel<BF16, CAP, ALIBI>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
  });
  if (attr_err != cudaSuccess) return cuda_fail("fwd256_kernel shared-memory attribute", attr_err);
  const int n_qt = (p.Sq + kBM - 1) / kBM;
  const unsigned grid = (unsigned)n_qt * (unsigned)p.B * (unsigned)p.Hq;
  kern<<<grid, kThreads, kSmemBytes, st>>>(tm.m[0], tm.m[1], tm.m[2], tm.m[3], p);
  note_launch();
  return launch_status("fwd256_kernel launch");
}

template <bool BF16>
int dispatch(const Params& p, const Tmaps4& tm, cudaStream_t st) {
  const bool cap = p.soft_cap > 0.f, alibi = p.alibi != nullptr;
  if (cap && alibi) return launch<BF16, true, true>(p, tm, st);
  if (cap) return launch<BF16, true, false>(p, tm, st);
  if (alibi) return launch<BF16, false, true>(p, tm, st);
  return launch<BF16, false, false>(p, tm, st);
}

}  // namespace

// Tensor maps: Q / O boxes of 128 rows, K boxes of 128 keys, V boxes of 64
// keys (a ring unit holds half a V tile), all 64 dims wide.
int sm100_fwd256(const Params& p, int dtype, cudaStream_t st) {
  Tmaps4 tm;
  if (!make_tmap_bhsd(&tm.m[0], p.q, dtype, kD, p.Sq, p.Hq, p.B, p.sq_, kBM) ||
      !make_tmap_bhsd(&tm.m[1], p.k, dtype, kD, p.Sk, p.Hkv, p.B, p.sk_, kBN) ||
      !make_tmap_bhsd(&tm.m[2], p.v, dtype, kD, p.Sk, p.Hkv, p.B, p.sv_, 64) ||
      !(p.out_acc ? (tm.m[3] = tm.m[0], true)  // no TMA store of O when merging
                  : make_tmap_bhsd(&tm.m[3], p.o, dtype, kD, p.Sq, p.Hq, p.B, p.so_, kBM)))
    return simt_fwd(p, dtype, st);
  return dtype == BFA_DTYPE_BF16 ? dispatch<true>(p, tm, st) : dispatch<false>(p, tm, st);
}

}  // namespace bfa
