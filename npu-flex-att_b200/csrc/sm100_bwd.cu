// sm100_bwd.cu -- tcgen05 / TMA / TMEM attention backward for B200.
//
// Replaces flash_attn_bwd_dkdv_kernel (npu_flash_attention.py:407-560),
// flash_attn_bwd_dq_kernel (:298-402) and the host GQA sum (:735-737) for
// bf16/fp16 inputs with head_dim 64 or 128 (head_dim 256: sm100_bwd256.cu).
// Per pair (i, j):
//   P  = exp(u_ij − lse_i)        u = transformed logit (cap, ALiBi), masked
//   dP = dO_i · V_j
//   dS = P ∘ (dP − Δ_i) · scale · (1 − tanh²)   (tanh term only with soft-cap)
//   dV_j += P_ij dO_i,  dK_j += dS_ij Q_i,  dQ_i += dS_ij K_j
// ALiBi enters P exactly as in the forward, so these are the true gradients
// of the forward (the reference backward leaves the slopes out).
//
// dkdv_kernel: one CTA per (batch, kv-head, 128-key tile); loops over the
//   GQA group's q-heads and their 64-row query tiles, so dK/dV are summed over
//   the group in fp32 TMEM -- no per-q-head copies, no atomics, deterministic.
//   MMAs (M = 128 keys): Sᵀ = K Qᵢᵀ, dPᵀ = V dOᵢᵀ (N = 64), then
//   dV += Pᵀ dOᵢ and dK += dSᵀ Qᵢ (N = D, B operand MN-major).
// dq_kernel: one CTA per (batch, q-head, 128-row query tile); loops over
//   128-key tiles: S = Q Kⱼᵀ, dP = dO Vⱼᵀ (Q, dO held in TMEM), dQ += dS Kⱼ.
// Warp roles in both: warp 0 TMA producer (+ LSE/Δ staging), warps 1 and 3
// MMA issuers (warp 1 the S/dP products, warp 3 the accumulating dV/dK or dQ
// products), warp 2 TMEM allocator, warps 4-11 elementwise: two warpgroups,
// one row per thread, each taking half of every step's columns. The dQ
// kernel forms Δ in its prologue when the call has both the Δ and dQ
// phases. S/dP are double-buffered (dK/dV) or released early (dQ) in TMEM so
// the MMAs of step i+1 overlap the elementwise work of step i.
// Accumulate mode (Params::grad_acc): dq/dk/dv are fp32 and the epilogues
// TMA reduce-add their fp32 tiles into them instead of storing 16-bit tiles.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <mutex>
#include <type_traits>

#include "bfa_internal.h"
#include "sm100_host.h"
#include "sm100_bwd_common.cuh"
#include "sm100_ptx.cuh"

namespace bfa {
namespace {

using namespace sm100;
using namespace bwd;

// ============================================================== dK / dV
// TMEM: Sᵀ(b) at 64·b, dPᵀ(b) at 128 + 64·b (b = step parity, fp32, 64
// columns each); the elementwise warps overwrite columns [0, 16) and
// [32, 48) of each with Pᵀ / dSᵀ (16-bit, two per column; query columns 0-31
// and 32-63), the A operands of the dV / dK MMAs. dV at 256, dK at 256 + D.
template <int D>
struct DkdvLayout {
  static constexpr int kSub = D / 64;
  static constexpr int kStages = (D <= 64) ? 8 : 4;
  static constexpr uint32_t kKVBytes = kRows * D * 2;    // K or V tile (128 keys)
  static constexpr uint32_t kQBytes = kInner * D * 2;    // Q or dO tile (64 rows)
  static constexpr uint32_t kOffK = 0;
  static constexpr uint32_t kOffV = kOffK + kKVBytes;
  static constexpr uint32_t kOffStage = kOffV + kKVBytes;       // Q_s, dO_s per stage
  static constexpr uint32_t kStageBytes = 2 * kQBytes;
  static constexpr uint32_t kOffRow = kOffStage + kStages * kStageBytes;  // lse2_s[64], delta_s[64]
  static constexpr uint32_t kOffBar = kOffRow + kStages * 512;
  static constexpr uint32_t kSmemBytes = kOffBar + 512 + 1024;
  static constexpr uint32_t kTmemS = 0, kTmemDP = 128, kTmemDV = 256, kTmemDK = 256 + D;
  static_assert(kTmemDK + D <= 512, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "smem budget");
  static_assert((2 * kQBytes) % 1024 == 0, "stage alignment");
  static_assert(kStages * kStageBytes >= 2u * kRows * D * 4, "fp32 dK/dV staging");
};

// (batch, kv-head) units per group in the dK/dV block order (see below).
#ifndef BFA_DKDV_UNIT_GROUP
#define BFA_DKDV_UNIT_GROUP 8
#endif
constexpr int kUnitGroup = BFA_DKDV_UNIT_GROUP;

template <int D, bool BF16, bool CAP, bool ALIBI>
__global__ void __launch_bounds__(kThreads, 1)
    dkdv_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                const __grid_constant__ CUtensorMap tmDK, const __grid_constant__ CUtensorMap tmDV,
                const Params p) {
  using L = DkdvLayout<D>;
  constexpr int NS = L::kStages;
  enum {
    kKVFull = 0,
    kQFull = 1,
    kQEmpty = 1 + NS,
    kSPFull = 1 + 2 * NS,
    kDSFull = kSPFull + 2,
    kDDDone = kDSFull + 2,  // dV/dK(i) complete (parity i % 2): Pᵀ/dSᵀ(i) read
    kAccDone = kDDDone + 2,
    kDrain = kAccDone + 1,
    kDrainSP = kDrain + 1,
    kNever = kDrainSP + 1,
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
  // Block order: (batch, kv-head) units in groups of kUnitGroup; within a
  // group the key tile is the slow index, so the group's first key tiles --
  // the longest under a causal mask -- are dispatched first (longest-first),
  // and the CTAs in flight share one group's Q and dO in L2 instead of every
  // unit's (which would not fit).
  const int BHkv = p.B * p.Hkv;
  const int n_kt = (p.Sk + kRows - 1) / kRows;
  const int grp = (int)(blockIdx.x / ((unsigned)kUnitGroup * n_kt));
  const int gsize = min(kUnitGroup, BHkv - grp * kUnitGroup);
  const int rem = (int)(blockIdx.x - (unsigned)grp * kUnitGroup * n_kt);
  const int kt = rem / gsize;
  const int bh = grp * kUnitGroup + rem % gsize;
  const int hkv = bh % p.Hkv, b = bh / p.Hkv;
  const int c0 = kt * kRows;
  int qlo, qhi;
  query_range(p, c0, min(c0 + kRows, p.Sk), &qlo, &qhi);
  const int qt0 = qlo / kInner;
  const int n_qt = (qhi > qlo) ? (qhi + kInner - 1) / kInner - qt0 : 0;
  // Steps s in [0, n_qt * G): q-head hkv * G + s / n_qt, 64-row query tile
  // qt0 + s % n_qt. With a block-sparse mask a step is visited only when its
  // (query block, key block) is on; every role walks the visited steps in
  // the same order with next_step().
  auto step_hq = [&](int s) { return hkv * p.G + s / n_qt; };
  auto step_q0 = [&](int s) { return (qt0 + s % n_qt) * kInner; };
  auto step_on = [&](int s) { return block_on(p, b, step_hq(s), step_q0(s) / kMaskBlock, kt); };
  int n_iter = n_qt * p.G;
  if (p.blk) {
    n_iter = 0;
    for (int s = 0; s < n_qt * p.G; ++s) n_iter += step_on(s) ? 1 : 0;
  }
  auto next_step = [&](int s) {
    do { ++s; } while (p.blk && s < n_qt * p.G && !step_on(s));
    return s;
  };

  WaitCtl ctl{abort_flag, p.status, p.timeout_ns};

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i)
      mbar_init(bar(i), (i >= kDSFull && i < kDSFull + 2) ? 8u : 1u);
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
      // A key tile no query sees loads nothing: its epilogue stages zeros in
      // the K / V tiles, which must not have a TMA write in flight.
      if (n_iter > 0) {
        mbar_arrive_expect_tx(bar(kKVFull), 2 * L::kKVBytes);
        for (int s = 0; s < L::kSub; ++s) {
          tma_load_4d(sbase + L::kOffK + s * (kRows * 128), &tmK, bar(kKVFull), s * 64, c0, hkv, b);
          tma_load_4d(sbase + L::kOffV + s * (kRows * 128), &tmV, bar(kKVFull), s * 64, c0, hkv, b);
        }
      }
      int issued = 0;
      int sv = -1;
      for (int i = 0; i < n_iter; ++i) {
        const int st = i % NS;
        if (i >= NS && !mbar_wait(bar(kQEmpty + st), ((i / NS) & 1) ^ 1, ctl, BFA_ERR_DEVICE_TIMEOUT))
          break;
        sv = next_step(sv);
        const int hq = step_hq(sv);
        const int q0 = step_q0(sv);
        const uint32_t qs = sbase + L::kOffStage + st * L::kStageBytes;
        const int64_t rrow = ((int64_t)b * p.Hq + hq) * p.Sq_pad + q0;
        const uint32_t rs = sbase + L::kOffRow + st * 512;
        mbar_arrive_expect_tx(bar(kQFull + st), L::kStageBytes + 512);
        for (int s = 0; s < L::kSub; ++s) {
          tma_load_4d(qs + s * (kInner * 128), &tmQ, bar(kQFull + st), s * 64, q0, hq, b);
          tma_load_4d(qs + L::kQBytes + s * (kInner * 128), &tmDO, bar(kQFull + st), s * 64, q0, hq, b);
        }
        bulk_load(rs, p.lse2 + rrow, 256, bar(kQFull + st));
        bulk_load(rs + 256, p.delta + rrow, 256, bar(kQFull + st));
        issued = i + 1;
      }
      if (n_iter > 0) drain_wait(bar(kKVFull), 0, p.timeout_ns);
      for (int i = (issued > NS ? issued - NS : 0); i < issued; ++i)
        drain_wait(bar(kQFull + i % NS), (i / NS) & 1, p.timeout_ns);
    }
  } else if (warp == 1 || warp == 3) {
    // ------------------------------------------------------------ MMA issuers
    // Two threads issue the MMAs: warp 1 Sᵀ/dPᵀ(i), warp 3 dV/dK(i). A
    // thread whose MMA queue is full blocks at the next issue, so with one
    // issuer dV/dK(i) queued behind Sᵀ/dPᵀ(i+1) and reached the tensor pipe
    // several hundred cycles after dSᵀ(i) was ready. Split, dV/dK(i) is issued
    // as soon as the elementwise warps release it. Ordering between the two
    // comes from mbarriers: Sᵀ/dPᵀ(i+2) overwrite the TMEM of Pᵀ/dSᵀ(i), so
    // they wait for dV/dK(i) to complete (kDDDone), and dV/dK(i) follows the
    // elementwise step, which waited for Sᵀ/dPᵀ(i).
    if (lane == 0) {
      constexpr uint32_t idSP = idesc_f16(kRows, kInner, BF16, false);
      constexpr uint32_t idAcc = idesc_f16(kRows, D, BF16, true);
      auto stage = [&](int i) -> uint32_t { return sbase + L::kOffStage + (i % NS) * L::kStageBytes; };
      if (warp == 1) {
        // Descriptors are built once; a K step only moves the start address
        // (a compile-time offset added to the low field).
        const uint64_t dK0 = desc_kmajor(sbase + L::kOffK), dV0 = desc_kmajor(sbase + L::kOffV);
        bool ok = n_iter == 0 || mbar_wait(bar(kKVFull), 0, ctl, BFA_ERR_DEVICE_TIMEOUT);
        for (int i = 0; i < n_iter && ok; ++i) {
          const int bf = i & 1;
          if (!(ok = mbar_wait(bar(kQFull + i % NS), (i / NS) & 1, ctl, BFA_ERR_DEVICE_TIMEOUT))) break;
          if (i >= 2 && !(ok = mbar_wait(bar(kDDDone + bf), ((i - 2) >> 1) & 1, ctl, BFA_ERR_DEVICE_TIMEOUT)))
            break;
          tc_fence_after();
          const uint64_t dq = desc_kmajor(stage(i)), ddo = desc_kmajor(stage(i) + L::kQBytes);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t offkv = ((kk >> 2) * (kRows * 128) + (kk & 3) * 32) >> 4;
            const uint32_t offq = ((kk >> 2) * (kInner * 128) + (kk & 3) * 32) >> 4;
            mma_ss(tmem + L::kTmemS + 64 * bf, dK0 + offkv, dq + offq, idSP, kk > 0 ? 1u : 0u);
            mma_ss(tmem + L::kTmemDP + 64 * bf, dV0 + offkv, ddo + offq, idSP, kk > 0 ? 1u : 0u);
          }
          mma_commit(bar(kSPFull + bf));
        }
        mma_commit(bar(kDrainSP));
        drain_wait(bar(kDrainSP), 0, p.timeout_ns);
      } else {
        bool ok = true;
        for (int i = 0; i < n_iter && ok; ++i) {
          const int bf = i & 1, k = i >> 1;
          if (!(ok = mbar_wait(bar(kDSFull + bf), k & 1, ctl, BFA_ERR_DEVICE_TIMEOUT))) break;
          tc_fence_after();
          const uint64_t mq = desc_mnmajor(stage(i), kInner * 128);
          const uint64_t mdo = desc_mnmajor(stage(i) + L::kQBytes, kInner * 128);
#pragma unroll
          for (int kk = 0; kk < kInner / 16; ++kk) {
            const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
            mma_ts(tmem + L::kTmemDV, tmem + L::kTmemS + 64 * bf + 32 * (kk >> 1) + 8 * (kk & 1),
                   mdo + ((kk * 2048) >> 4), idAcc, acc);
            mma_ts(tmem + L::kTmemDK, tmem + L::kTmemDP + 64 * bf + 32 * (kk >> 1) + 8 * (kk & 1),
                   mq + ((kk * 2048) >> 4), idAcc, acc);
          }
          mma_commit(bar(kQEmpty + i % NS));
          mma_commit(bar(kDDDone + bf));
        }
        mma_commit(bar(kAccDone));
        mma_commit(bar(kDrain));
        drain_wait(bar(kDrain), 0, p.timeout_ns);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ elementwise
    // Both warpgroups work on every step: warpgroup h takes query columns
    // [32h, 32h + 32) of it, so a step's elementwise latency is that of 32
    // columns. Each thread owns one key row (TMEM lane).
    const int eg = (warp - 4) >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;  // key row within the tile
    const int kj = c0 + row;
    const int64_t gj = (int64_t)kj + p.k_off;
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const float sl2 = p.scale * kLog2e;
    const float cap_in = CAP ? p.scale / p.soft_cap : 0.f;
    const float cap_out = CAP ? p.soft_cap * kLog2e : 0.f;
    bool ok = true;
    // Per-step metadata without a division or the general tile test per step
    // (a step's setup is a serial chain on the elementwise warps' critical
    // path): the q-head offset hs and query-tile index ts advance
    // incrementally (a division only under a block-sparse mask, whose walk
    // skips steps), and without documents the step is fully kept exactly
    // when its first query lies in `kept`.
    int hs = 0, ts = -1;
    const bool lin_full = p.doc_lo == nullptr;
    const KeptRange kept = kept_queries(p, c0, kRows, kInner);
    int sv = -1;
    for (int i = 0; i < n_iter; ++i) {
      const int bf = i & 1, k = i >> 1, st = i % NS;
      sv = next_step(sv);
      if (p.blk) {
        hs = sv / n_qt;
        ts = sv - hs * n_qt;
      } else if (++ts == n_qt) {
        ts = 0;
        ++hs;
      }
      const int hq = hkv * p.G + hs;
      const int q0 = (qt0 + ts) * kInner;
      // The step's mask and bias constants first: they overlap the wait.
      const uint32_t tSb = tmem + lane_base + L::kTmemS + 64 * bf;
      const uint32_t tDb = tmem + lane_base + L::kTmemDP + 64 * bf;
      const float* rowv = (const float*)(smem + L::kOffRow + st * 512);
      const bool full = lin_full ? kept.has(q0) : tile_full(p, q0, q0 + kInner, c0, c0 + kRows);
      const float slope = ALIBI ? p.alibi[hq] : 0.f;
      const float slope2 = slope * kLog2e;
      // ALiBi bias slope·(g0_i - j) (alibi_ref): with slope > 0, g0_i =
      // max(0, i - W, document start) and the bias is the larger of the two
      // terms below (every query kept with key j shares j's document); with
      // slope <= 0, g0_i = i (the second term alone).
      const bool shifted = ALIBI && slope > 0.f;
      const int64_t dstart = (p.doc_lo && kj < p.Sk) ? (int64_t)p.doc_lo[gj] : 0;
      const float ba = shifted ? slope2 * (float)(dstart - gj) : neg_inf();
      const float bq = !ALIBI ? 0.f
                       : !shifted ? slope2 * (float)((int64_t)q0 + p.q_off - gj)
                       : p.window > 0 ? slope2 * (float)((int64_t)q0 + p.q_off - p.window - gj)
                                      : neg_inf();
      int clo = 0, chi = kInner;  // kept query columns [clo, chi) of this key row (masked steps)
      if (!full) queries_for_key(p, gj, kj < p.Sk, q0, kInner, &clo, &chi);
      uint32_t wbar = bar(kSPFull + bf), wpar = (uint32_t)(k & 1);
      if ((p.debug_flags & BFA_DEBUG_INJECT_STALL) && i == 0) {
        wbar = bar(kNever);
        wpar = 0;
      }
      if (!(ok = warp_wait(wbar, wpar, ctl))) break;
      // The stage's lse2 / Δ arrived with its Q / dO (same barrier phase).
      if (!(ok = warp_wait(bar(kQFull + st), (uint32_t)((i / NS) & 1), ctl))) break;
      tc_fence_after();
      // One body per case (mask or not), chosen once per step: no branches
      // inside the unrolled column loop.
      const int half = eg;
      // Sᵀ first; dPᵀ loads while P is formed (pass 1), dS follows (pass 2).
      uint32_t sr[32], dr[32];
      tmem_ld32(tSb + 32 * half, sr);
      tmem_ld_wait();
      tmem_ld32(tDb + 32 * half, dr);
      const int tier = CAP ? cap_tier<32>(sr, cap_in) : 0;
      auto step = [&](auto masked, auto small_tag) {
        constexpr bool MASKED = decltype(masked)::value;
        constexpr int TIER = decltype(small_tag)::value;
        float pr[32];
        float tt[CAP ? 32 : 1];
        uint32_t ppk[16];
#pragma unroll
        for (int c = 0; c < 32; c += 4) {
          const float4 l4 = *reinterpret_cast<const float4*>(rowv + 32 * half + c);
          const float lse_c[4] = {l4.x, l4.y, l4.z, l4.w};
          if (!CAP && !ALIBI) {
            // Plain logits: two keys per packed instruction, which leaves
            // issue slots to the MMA thread on the same sub-partition.
#pragma unroll
            for (int h = 0; h < 4; h += 2) {
              const float2 x = __ffma2_rn(make_float2(__uint_as_float(sr[c + h]), __uint_as_float(sr[c + h + 1])),
                                          make_float2(sl2, sl2), make_float2(-lse_c[h], -lse_c[h + 1]));
              float pr0 = ex2(x.x), pr1 = ex2(x.y);
              if (MASKED) {
                const int cc = 32 * half + c + h;
                pr0 = ((unsigned)(cc - clo) < (unsigned)(chi - clo)) ? pr0 : 0.f;
                pr1 = ((unsigned)(cc + 1 - clo) < (unsigned)(chi - clo)) ? pr1 : 0.f;
              }
              pr[c + h] = pr0;
              pr[c + h + 1] = pr1;
            }
          } else if (CAP && !ALIBI) {
            // Soft-cap without ALiBi: two keys per packed instruction.
#pragma unroll
            for (int h = 0; h < 4; h += 2) {
              float2 th;
              const float2 x = cap_logit2x2<TIER>(make_float2(__uint_as_float(sr[c + h]), __uint_as_float(sr[c + h + 1])),
                                                   cap_in, cap_out, &th);
              float pr0 = ex2(x.x - lse_c[h]), pr1 = ex2(x.y - lse_c[h + 1]);
              if (MASKED) {
                const int cc = 32 * half + c + h;
                pr0 = ((unsigned)(cc - clo) < (unsigned)(chi - clo)) ? pr0 : 0.f;
                pr1 = ((unsigned)(cc + 1 - clo) < (unsigned)(chi - clo)) ? pr1 : 0.f;
              }
              pr[c + h] = pr0;
              pr[c + h + 1] = pr1;
              if (CAP) {
                tt[c + h] = th.x;
                tt[c + h + 1] = th.y;
              }
            }
          } else if (ALIBI && !CAP) {
            // ALiBi without cap: the bias per key (its reference point
            // clamped as alibi_ref does), the rest two keys per packed
            // instruction.
#pragma unroll
            for (int h = 0; h < 4; h += 2) {
              const int cc = 32 * half + c + h;
              const float2 bias = __fadd2_rn(make_float2(fmaxf(ba, fmaf(slope2, (float)cc, bq)),
                                                         fmaxf(ba, fmaf(slope2, (float)(cc + 1), bq))),
                                             make_float2(-lse_c[h], -lse_c[h + 1]));
              const float2 x = __ffma2_rn(make_float2(__uint_as_float(sr[c + h]), __uint_as_float(sr[c + h + 1])),
                                          make_float2(sl2, sl2), bias);
              float pr0 = ex2(x.x), pr1 = ex2(x.y);
              if (MASKED) {
                pr0 = ((unsigned)(cc - clo) < (unsigned)(chi - clo)) ? pr0 : 0.f;
                pr1 = ((unsigned)(cc + 1 - clo) < (unsigned)(chi - clo)) ? pr1 : 0.f;
              }
              pr[c + h] = pr0;
              pr[c + h + 1] = pr1;
            }
          } else {
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              const int cc = 32 * half + c + h;
              const float raw = __uint_as_float(sr[c + h]);
              float pv, t = 0.f;
              if (CAP || ALIBI) {
                float x = logit2<CAP, TIER>(raw, sl2, cap_in, cap_out, &t);
                if (ALIBI) x += fmaxf(ba, fmaf(slope2, (float)cc, bq));
                pv = ex2(x - lse_c[h]);
              } else {
                pv = ex2(fmaf(raw, sl2, -lse_c[h]));
              }
              if (MASKED) pv = ((unsigned)(cc - clo) < (unsigned)(chi - clo)) ? pv : 0.f;
              pr[c + h] = pv;
              if (CAP) tt[c + h] = t;
            }
          }
          ppk[c / 2] = pack2<BF16>(pr[c], pr[c + 1]);
          ppk[c / 2 + 1] = pack2<BF16>(pr[c + 2], pr[c + 3]);
        }
        // Pᵀ of half h -> packed columns [32h, 32h + 16) of the S buffer:
        // inside this half's own fp32 columns, read above.
        tmem_st16(tSb + 32 * half, ppk);
        tmem_ld_wait();  // dPᵀ
        uint32_t dpk[16];
#pragma unroll
        for (int c = 0; c < 32; c += 4) {
          const float4 d4 = *reinterpret_cast<const float4*>(rowv + 64 + 32 * half + c);
          const float dl_c[4] = {d4.x, d4.y, d4.z, d4.w};
          float ds4[4];
          if (!CAP) {
#pragma unroll
            for (int h = 0; h < 4; h += 2) {
              const float2 dd = __fadd2_rn(make_float2(__uint_as_float(dr[c + h]), __uint_as_float(dr[c + h + 1])),
                                           make_float2(-dl_c[h], -dl_c[h + 1]));
              const float2 ds = __fmul2_rn(__fmul2_rn(make_float2(pr[c + h], pr[c + h + 1]), dd),
                                           make_float2(p.scale, p.scale));
              ds4[h] = ds.x;
              ds4[h + 1] = ds.y;
            }
          } else if (CAP && !ALIBI) {
#pragma unroll
            for (int h = 0; h < 4; h += 2) {
              const float2 dd = __fadd2_rn(make_float2(__uint_as_float(dr[c + h]), __uint_as_float(dr[c + h + 1])),
                                           make_float2(-dl_c[h], -dl_c[h + 1]));
              const float2 th = make_float2(tt[c + h], tt[c + h + 1]);
              float2 ds = __fmul2_rn(__fmul2_rn(make_float2(pr[c + h], pr[c + h + 1]), dd),
                                     make_float2(p.scale, p.scale));
              ds = __fmul2_rn(ds, __ffma2_rn(make_float2(-th.x, -th.y), th, make_float2(1.f, 1.f)));
              ds4[h] = ds.x;
              ds4[h + 1] = ds.y;
            }
          } else {
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              float ds = pr[c + h] * (__uint_as_float(dr[c + h]) - dl_c[h]) * p.scale;
              if (CAP) ds *= (1.f - tt[c + h] * tt[c + h]);
              ds4[h] = ds;
            }
          }
          dpk[c / 2] = pack2<BF16>(ds4[0], ds4[1]);
          dpk[c / 2 + 1] = pack2<BF16>(ds4[2], ds4[3]);
        }
        tmem_st16(tDb + 32 * half, dpk);
      };
      using I2 = std::integral_constant<int, 2>;
      using I1 = std::integral_constant<int, 1>;
      using I0 = std::integral_constant<int, 0>;
      if (tier == 2) {
        if (full) step(std::false_type{}, I2{});
        else step(std::true_type{}, I2{});
      } else if (tier == 1) {
        if (full) step(std::false_type{}, I1{});
        else step(std::true_type{}, I1{});
      } else {
        if (full) step(std::false_type{}, I0{});
        else step(std::true_type{}, I0{});
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kDSFull + bf));
    }
    // Warpgroup 0 runs the epilogue; warpgroup 1 goes straight to the exit.
    if (eg == 0) {
      bool good = ok;
      if (good && n_iter > 0) good = warp_wait(bar(kAccDone), 0, ctl);
      good = good && !*abort_flag;
      // K and V tiles are free once every MMA is done: they stage dK and dV.
      // In accumulate mode the fp32 tiles (2 x 128 x D x 4 bytes) go to the
      // Q/dO stages instead, which are free too; a key tile no query sees
      // adds nothing and skips the epilogue.
      const bool acc = p.grad_acc != 0;
      uint8_t* stage_dk = acc ? smem + L::kOffStage + kRows * D * 4 : smem + L::kOffK;
      uint8_t* stage_dv = acc ? smem + L::kOffStage : smem + L::kOffV;
      if (good && !(acc && n_iter == 0)) {
        tc_fence_after();
        if (acc) {
          stage_tmem_row_f32<D>(tmem + lane_base + L::kTmemDV, stage_dv, row);
          stage_tmem_row_f32<D>(tmem + lane_base + L::kTmemDK, stage_dk, row);
        } else {
          stage_tmem_row<D, BF16>(tmem + lane_base + L::kTmemDV, stage_dv, row, n_iter == 0);
          stage_tmem_row<D, BF16>(tmem + lane_base + L::kTmemDK, stage_dk, row, n_iter == 0);
        }
        fence_async_shared();
      }
      if (lane == 0) warp_ok[wq] = good ? 1 : 0;
      named_sync(1, 128);
      if (wq == 0 && lane == 0 && warp_ok[0] && warp_ok[1] && warp_ok[2] && warp_ok[3]) {
        if (!acc) {
          for (int s = 0; s < L::kSub; ++s) {
            tma_store_4d(&tmDV, smem_u32(stage_dv) + s * (kRows * 128), s * 64, c0, hkv, b);
            tma_store_4d(&tmDK, smem_u32(stage_dk) + s * (kRows * 128), s * 64, c0, hkv, b);
          }
        } else if (n_iter > 0) {
          for (int s = 0; s < D / 32; ++s) {
            tma_reduce_add_4d(&tmDV, smem_u32(stage_dv) + s * (kRows * 128), s * 32, c0, hkv, b);
            tma_reduce_add_4d(&tmDK, smem_u32(stage_dk) + s * (kRows * 128), s * 32, c0, hkv, b);
          }
        }
        tma_store_commit();
        tma_store_wait_all();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================== dQ
// One CTA per (batch, q-head, 128-row query tile) loops over 128-key tiles:
//   S = Q Kⱼᵀ, dP = dO Vⱼᵀ, dS (elementwise), dQ += dS Kⱼ.
// Every MMA has N = 128: on B200 a tcgen05.mma with N = 64 costs about 1.4x
// its nominal time (a fixed per-instruction cost), with N >= 128 it runs at
// the nominal rate.
// TMEM: S at 0 and dP at 128 (128 fp32 columns each), dQ at 256, Q and dO at
// 256 + D and 256 + 3D/2 (16-bit, two per column). Q and dO are the A
// operands of S and dP and constant for the CTA, so they are moved into TMEM
// once and those MMAs read only K / V from shared memory. dS (16-bit) goes to
// a 128-byte-swizzled shared tile [128 rows][128 keys], the A operand of
// dQ += dS·K.
// The elementwise warps release S(i) as soon as it is in registers and dP(i)
// as soon as its second half is, so the MMA warp issues S(i+1) and dP(i+1)
// while they compute dS(i); dQ(i) follows once dS(i) is in shared memory.
// Shared memory: Q, dO, then K/V stages, then the dS tile; once Q and dO are
// in TMEM their tile is the last K/V stage.
template <int D>
struct DqLayout {
  static constexpr int kKeys = 128;  // keys per step
  static constexpr int kSub = D / 64;
  static constexpr uint32_t kQBytes = kRows * D * 2;    // Q or dO tile (128 rows)
  static constexpr uint32_t kKVBytes = kKeys * D * 2;   // K or V tile (128 keys)
  static constexpr uint32_t kStageBytes = 2 * kKVBytes;
  static constexpr int kStages = (D <= 64) ? 5 : 3;     // the last one is the Q/dO tile
  static constexpr uint32_t kDSBytes = kRows * kKeys * 2;  // dS [128 rows][128 keys]
  static constexpr uint32_t kOffQ = 0;
  static constexpr uint32_t kOffDO = kOffQ + kQBytes;
  static constexpr uint32_t kOffStage = kOffDO + kQBytes;
  static constexpr uint32_t kOffDS = kOffStage + (kStages - 1) * kStageBytes;
  static constexpr uint32_t kOffBar = kOffDS + kDSBytes;
  static constexpr uint32_t kOffDlt = kOffBar + 512;  // Δ of the 128 rows (fused Δ)
  static constexpr uint32_t kSmemBytes = kOffDlt + kRows * 4 + 1024;
  static constexpr uint32_t kTmemS = 0, kTmemDP = 128, kTmemDQ = 256;
  static constexpr uint32_t kTmemQ = kTmemDQ + D, kTmemDO = kTmemQ + D / 2;
  static __host__ __device__ constexpr uint32_t stage_off(int st) {
    return st < kStages - 1 ? kOffStage + st * kStageBytes : kOffQ;
  }
  static_assert(kTmemDO + D / 2 <= 512, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "smem budget");
  static_assert(2 * kQBytes == kStageBytes, "the Q/dO tile doubles as a K/V stage");
  static_assert(kOffDO == kOffQ + kQBytes && 2 * kQBytes >= kRows * D * 4, "fp32 dQ staging");
};

#ifndef BFA_DQ_UNIT_GROUP
#define BFA_DQ_UNIT_GROUP 4
#endif
constexpr int kDqUnitGroup = BFA_DQ_UNIT_GROUP;

template <int D, bool BF16, bool CAP, bool ALIBI>
__global__ void __launch_bounds__(kThreads, 1)
    dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
              const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
              const __grid_constant__ CUtensorMap tmDQ, const __grid_constant__ CUtensorMap tmO,
              const Params p) {
  using L = DqLayout<D>;
  constexpr int NS = L::kStages;
  constexpr int NK = L::kKeys;
  enum {
    kQFull = 0,
    kKVFull = 1,
    kKVEmpty = 1 + NS,
    kSPFull = 1 + 2 * NS,  // MMA -> elementwise: S(i) and dP(i) are in TMEM
    kSRead = kSPFull + 1,  // elementwise -> MMA: S(i) is in registers (8 warps)
    kDPRead = kSRead + 1,  // elementwise -> MMA: dP(i) is in registers (8 warps)
    kDSFull = kDPRead + 1,  // elementwise -> MMA: dS(i) is in shared memory (8 warps)
    kOpsReady = kDSFull + 1,  // Q and dO are in TMEM (8 warps)
    kDSFree = kOpsReady + 1,  // MMA -> elementwise: dQ(i) has read the dS tile
    kAccDone = kDSFree + 1,
    kDrain = kAccDone + 1,
    kDrainSP = kDrain + 1,
    kNever = kDrainSP + 1,
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
  const int n_qt = (p.Sq + kRows - 1) / kRows;
  // Block order: (batch, kv-head) units in groups of kDqUnitGroup; within a
  // group the query tile is the slow index, heaviest causal tiles first, so
  // the CTAs in flight share a few units' K / V in L2.
  const int BHkv = p.B * p.Hkv;
  const int grp = (int)(blockIdx.x / ((unsigned)kDqUnitGroup * p.G * n_qt));
  const int gsize = min(kDqUnitGroup, BHkv - grp * kDqUnitGroup) * p.G;  // q-heads in the group
  const int rem = (int)(blockIdx.x - (unsigned)grp * kDqUnitGroup * p.G * n_qt);
  const int qt = n_qt - 1 - rem / gsize;
  const int bhq = grp * kDqUnitGroup * p.G + rem % gsize;  // (b, hq) with hq fastest
  const int hq = bhq % p.Hq, b = bhq / p.Hq;
  const int hkv = hq / p.G;
  const int q0 = qt * kRows;
  int klo, khi;
  key_range(p, q0, min(q0 + kRows, p.Sq), &klo, &khi);
  const int jt0 = klo / NK;
  const int jend = (khi > klo) ? (khi + NK - 1) / NK : jt0;
  // Block-sparse mask: key tile j (one 128-key block) is visited only when
  // block (q0 / 128, j) is on; producer and elementwise warps walk the
  // visited tiles with next_tile().
  int n_iter = jend - jt0;
  if (p.blk) {
    n_iter = 0;
    for (int j = jt0; j < jend; ++j) n_iter += block_on(p, b, hq, q0 / kMaskBlock, j) ? 1 : 0;
  }
  auto next_tile = [&](int j) {
    do { ++j; } while (p.blk && j < jend && !block_on(p, b, hq, q0 / kMaskBlock, j));
    return j;
  };

  WaitCtl ctl{abort_flag, p.status, p.timeout_ns};

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i)
      mbar_init(bar(i), (i >= kSRead && i <= kOpsReady) ? 8u : 1u);
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
    if (lane == 0) {
      // A query tile that sees no key loads nothing: its epilogue stages zeros
      // in the Q tile, which must not have a TMA write in flight.
      if (n_iter > 0) {
        const bool fuse = p.fuse_delta != 0;
        mbar_arrive_expect_tx(bar(kQFull), (fuse ? 3 : 2) * L::kQBytes);
        for (int s = 0; s < L::kSub; ++s) {
          tma_load_4d(sbase + L::kOffQ + s * (kRows * 128), &tmQ, bar(kQFull), s * 64, q0, hq, b);
          tma_load_4d(sbase + L::kOffDO + s * (kRows * 128), &tmDO, bar(kQFull), s * 64, q0, hq, b);
          // Fused Δ: the O tile goes to the dS tile, free until the first dS.
          if (fuse) tma_load_4d(sbase + L::kOffDS + s * (kRows * 128), &tmO, bar(kQFull), s * 64, q0, hq, b);
        }
      }
      int n = 0;
      bool ok = true;
      int jv = jt0 - 1;
      for (int i = 0; i < n_iter && ok; ++i) {
        const int st = i % NS;
        if (i >= NS) ok = mbar_wait(bar(kKVEmpty + st), ((i / NS) & 1) ^ 1, ctl, BFA_ERR_DEVICE_TIMEOUT);
        else if (st == NS - 1) ok = mbar_wait(bar(kOpsReady), 0, ctl, BFA_ERR_DEVICE_TIMEOUT);
        if (!ok) break;
        jv = next_tile(jv);
        const int j0 = jv * NK;
        const uint32_t ks = sbase + L::stage_off(st);
        mbar_arrive_expect_tx(bar(kKVFull + st), L::kStageBytes);
        for (int s = 0; s < L::kSub; ++s) {
          tma_load_4d(ks + s * (NK * 128), &tmK, bar(kKVFull + st), s * 64, j0, hkv, b);
          tma_load_4d(ks + L::kKVBytes + s * (NK * 128), &tmV, bar(kKVFull + st), s * 64, j0, hkv, b);
        }
        n = i + 1;
      }
      if (n_iter > 0) drain_wait(bar(kQFull), 0, p.timeout_ns);
      for (int i = (n > NS ? n - NS : 0); i < n; ++i)
        drain_wait(bar(kKVFull + i % NS), (i / NS) & 1, p.timeout_ns);
    }
  } else if (warp == 1 || warp == 3) {
    // Two threads issue the MMAs: warp 1 S(i+1) and dP(i+1), warp 3 dQ(i). A
    // thread whose MMA queue is full blocks at its next issue, so with one
    // issuer dQ(i) reached the tensor pipe several hundred cycles after dS(i)
    // was ready. The stage's K/V is released after dQ(i), which is issued
    // after the elementwise step that waited for S(i) and dP(i).
    if (lane == 0) {
      auto stage = [&](int i) -> uint32_t { return sbase + L::stage_off(i % NS); };
      if (warp == 1) {
        constexpr uint32_t idSP = idesc_f16(kRows, NK, BF16, false);
        auto issue_s = [&](int i) {
          const uint64_t dk = desc_kmajor(stage(i));
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t offk = ((kk >> 2) * (NK * 128) + (kk & 3) * 32) >> 4;
            mma_ts(tmem + L::kTmemS, tmem + L::kTmemQ + 8 * kk, dk + offk, idSP, kk > 0 ? 1u : 0u);
          }
        };
        auto issue_dp = [&](int i) {
          const uint64_t dv = desc_kmajor(stage(i) + L::kKVBytes);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t offk = ((kk >> 2) * (NK * 128) + (kk & 3) * 32) >> 4;
            mma_ts(tmem + L::kTmemDP, tmem + L::kTmemDO + 8 * kk, dv + offk, idSP, kk > 0 ? 1u : 0u);
          }
          mma_commit(bar(kSPFull));
        };
        bool ok = n_iter == 0 || mbar_wait(bar(kOpsReady), 0, ctl, BFA_ERR_DEVICE_TIMEOUT);
        for (int i = 0; i < n_iter && ok; ++i) {
          if (!(ok = mbar_wait(bar(kKVFull + i % NS), (i / NS) & 1, ctl, BFA_ERR_DEVICE_TIMEOUT))) break;
          // S(i) / dP(i) overwrite the TMEM the elementwise warps read for step i - 1.
          if (i > 0 && !(ok = mbar_wait(bar(kSRead), (i - 1) & 1, ctl, BFA_ERR_DEVICE_TIMEOUT))) break;
          tc_fence_after();
          issue_s(i);
          if (i > 0 && !(ok = mbar_wait(bar(kDPRead), (i - 1) & 1, ctl, BFA_ERR_DEVICE_TIMEOUT))) break;
          tc_fence_after();
          issue_dp(i);
        }
        mma_commit(bar(kDrainSP));
        drain_wait(bar(kDrainSP), 0, p.timeout_ns);
      } else {
        constexpr uint32_t idAcc = idesc_f16(kRows, D, BF16, true);
        const uint64_t dS0 = desc_kmajor(sbase + L::kOffDS);
        bool ok = true;
        for (int i = 0; i < n_iter && ok; ++i) {
          if (!(ok = mbar_wait(bar(kDSFull), i & 1, ctl, BFA_ERR_DEVICE_TIMEOUT))) break;
          tc_fence_after();
          const uint64_t mk = desc_mnmajor(stage(i), NK * 128);
#pragma unroll
          for (int kk = 0; kk < NK / 16; ++kk) {
            const uint32_t offs = ((kk >> 2) * (kRows * 128) + (kk & 3) * 32) >> 4;
            mma_ss(tmem + L::kTmemDQ, dS0 + offs, mk + ((kk * 2048) >> 4), idAcc, (i > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(bar(kKVEmpty + i % NS));
          mma_commit(bar(kDSFree));
        }
        mma_commit(bar(kAccDone));
        mma_commit(bar(kDrain));
        drain_wait(bar(kDrain), 0, p.timeout_ns);
      }
    }
  } else if (warp >= 4) {
    // Both warpgroups work on every step: warpgroup h takes key columns
    // [64h, 64h + 64) of it. Each thread owns one query row.
    const int eg = (warp - 4) >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const int qi = q0 + row;
    const int64_t gi = (int64_t)qi + p.q_off;
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const float sl2 = p.scale * kLog2e;
    const float cap_in = CAP ? p.scale / p.soft_cap : 0.f;
    const float cap_out = CAP ? p.soft_cap * kLog2e : 0.f;
    const float slope = ALIBI ? p.alibi[hq] : 0.f;
    const float slope2 = slope * kLog2e;
    const int64_t g0 = ALIBI ? alibi_ref(p, slope, gi, qi < p.Sq) : gi;  // ALiBi bias slope·(g0 - j)
    const int64_t ridx = ((int64_t)b * p.Hq + hq) * p.Sq_pad + qi;
    const bool fuse = p.fuse_delta != 0;
    float lse2, dlt = 0.f;
    if (!fuse) {
      lse2 = p.lse2[ridx];
      dlt = p.delta[ridx];
    } else {
      // lse2 as the Δ pass forms it: +inf past Sq and for rows that see no key.
      lse2 = __int_as_float(0x7f800000);
      if (qi < p.Sq) {
        const float lse = p.lse[((int64_t)b * p.Hq + hq) * p.Sq + qi];
        if (lse != neg_inf()) lse2 = row_lse2(p, lse, hq, qi);
      }
    }
    // Fused Δ: warpgroup 1 forms Δ = Σ O·dO of its row from the O tile (TMA-
    // loaded with Q and dO into the dS tile, which is free until the first
    // dS) and the dO row it copies into TMEM below. A tile that sees no key
    // has Δ = 0 (its P is 0). TMA fills rows past Sq with zeros.
    const bool form_delta = fuse && eg == 1 && n_iter > 0;
    bool ok = true;
    // Warpgroup 0 moves this thread's Q row, warpgroup 1 its dO row, from the
    // swizzled shared tile into TMEM (lane = row, two elements per column).
    if (n_iter > 0) {
      ok = warp_wait(bar(kQFull), 0, ctl);
      if (ok) {
        const uint8_t* tile = smem + (eg == 0 ? L::kOffQ : L::kOffDO);
        const uint32_t tcol = tmem + lane_base + (eg == 0 ? L::kTmemQ : L::kTmemDO);
        float2 acc2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int s = 0; s < L::kSub; ++s) {
          uint32_t r[32];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 w = *reinterpret_cast<const uint4*>(tile + s * (kRows * 128) + sw128_offset(row, c));
            r[4 * c] = w.x; r[4 * c + 1] = w.y; r[4 * c + 2] = w.z; r[4 * c + 3] = w.w;
          }
          tmem_st32(tcol + 32 * s, r);
          if (form_delta) {
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const uint4 o4 =
                  *reinterpret_cast<const uint4*>(smem + L::kOffDS + s * (kRows * 128) + sw128_offset(row, c));
              const uint32_t ow[4] = {o4.x, o4.y, o4.z, o4.w};
#pragma unroll
              for (int e = 0; e < 4; ++e)
                acc2 = __ffma2_rn(unpack2<BF16>(ow[e]), unpack2<BF16>(r[4 * c + e]), acc2);
            }
          }
        }
        if (form_delta) {
          dlt = acc2.x + acc2.y;
          reinterpret_cast<float*>(smem + L::kOffDlt)[row] = dlt;
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(kOpsReady));
        // Warpgroup 0 takes its row's Δ from warpgroup 1 (the arrivals on
        // kOpsReady release the shared stores).
        if (fuse && eg == 0 && (ok = warp_wait(bar(kOpsReady), 0, ctl)))
          dlt = reinterpret_cast<const float*>(smem + L::kOffDlt)[row];
      }
    }
    if (fuse && eg == 1 && qi < p.Sq_pad) {
      p.delta[ridx] = dlt;
      p.lse2[ridx] = lse2;
    }
    // Without documents a key tile is fully kept exactly when its first key
    // lies in `kept` (no general tile test on the critical path).
    const bool lin_full = p.doc_lo == nullptr;
    const KeptRange kept = kept_keys(p, q0, kRows, NK, true);
    int jv = jt0 - 1;
    for (int i = 0; i < n_iter && ok; ++i) {
      jv = next_tile(jv);
      const int j0 = jv * NK;
      const bool full = lin_full ? kept.has(j0) : tile_full(p, q0, q0 + kRows, j0, j0 + NK);
      const float abase = ALIBI ? slope2 * (float)(g0 - (int64_t)j0 - p.k_off) : 0.f;
      int clo = 0, chi = NK;  // kept key columns [clo, chi) of this query row (masked tiles)
      if (!full) keys_for_query(p, gi, qi < p.Sq, j0, NK, &clo, &chi);
      uint32_t wbar = bar(kSPFull), wpar = (uint32_t)(i & 1);
      if ((p.debug_flags & BFA_DEBUG_INJECT_STALL) && i == 0) {
        wbar = bar(kNever);
        wpar = 0;
      }
      if (!(ok = warp_wait(wbar, wpar, ctl))) break;
      tc_fence_after();
      const uint32_t tSb = tmem + lane_base + L::kTmemS + 64 * eg;
      const uint32_t tDb = tmem + lane_base + L::kTmemDP + 64 * eg;
      // This warpgroup's 64 S columns into registers; S(i+1) may then start.
      uint32_t sr[64];
      tmem_ld32(tSb, *reinterpret_cast<uint32_t(*)[32]>(sr));
      tmem_ld32(tSb + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kSRead));
      uint8_t* ds_row = smem + L::kOffDS + eg * (kRows * 128);  // this warpgroup's 64 keys
      const int tier = CAP ? cap_tier<64>(sr, cap_in) : 0;
      auto step = [&](auto masked, auto small_tag) {
        constexpr bool MASKED = decltype(masked)::value;
        constexpr int TIER = decltype(small_tag)::value;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t dr[32];
          tmem_ld32(tDb + 32 * half, dr);
          tmem_ld_wait();
          if (half == 1) {  // all of dP(i) is in registers: dP(i+1) may start
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kDPRead));
          }
          uint32_t dpk[16];
          if (!CAP && !ALIBI) {
            // Plain logits: two keys per packed instruction (fma / mul
            // .f32x2), which leaves issue slots to the MMA thread on the same
            // sub-partition; dS = P (dP·scale - Δ·scale).
            const float2 sl22 = make_float2(sl2, sl2), nl2 = make_float2(-lse2, -lse2);
            const float2 sc2 = make_float2(p.scale, p.scale), nds2 = make_float2(-dlt * p.scale, -dlt * p.scale);
#pragma unroll
            for (int c = 0; c < 32; c += 2) {
              const float2 x = __ffma2_rn(make_float2(__uint_as_float(sr[32 * half + c]),
                                                      __uint_as_float(sr[32 * half + c + 1])), sl22, nl2);
              float pr0 = ex2(x.x), pr1 = ex2(x.y);
              if (MASKED) {
                const int cc = 64 * eg + 32 * half + c;
                pr0 = ((unsigned)(cc - clo) < (unsigned)(chi - clo)) ? pr0 : 0.f;
                pr1 = ((unsigned)(cc + 1 - clo) < (unsigned)(chi - clo)) ? pr1 : 0.f;
              }
              const float2 ds = __fmul2_rn(make_float2(pr0, pr1),
                                           __ffma2_rn(make_float2(__uint_as_float(dr[c]), __uint_as_float(dr[c + 1])), sc2, nds2));
              dpk[c / 2] = pack2<BF16>(ds.x, ds.y);
            }
          } else if (CAP && !ALIBI) {
            // Soft-cap without ALiBi: two keys per packed instruction;
            // dS = P (dP - Δ)·scale·(1 - tanh²).
            const float2 sc2 = make_float2(p.scale, p.scale), ndl2 = make_float2(-dlt, -dlt);
#pragma unroll
            for (int c = 0; c < 32; c += 2) {
              float2 th;
              const float2 x = cap_logit2x2<TIER>(make_float2(__uint_as_float(sr[32 * half + c]),
                                                               __uint_as_float(sr[32 * half + c + 1])),
                                                   cap_in, cap_out, &th);
              float pr0 = ex2(x.x - lse2), pr1 = ex2(x.y - lse2);
              if (MASKED) {
                const int cc = 64 * eg + 32 * half + c;
                pr0 = ((unsigned)(cc - clo) < (unsigned)(chi - clo)) ? pr0 : 0.f;
                pr1 = ((unsigned)(cc + 1 - clo) < (unsigned)(chi - clo)) ? pr1 : 0.f;
              }
              const float2 dd = __fadd2_rn(make_float2(__uint_as_float(dr[c]), __uint_as_float(dr[c + 1])), ndl2);
              float2 ds = __fmul2_rn(__fmul2_rn(make_float2(pr0, pr1), dd), sc2);
              ds = __fmul2_rn(ds, __ffma2_rn(make_float2(-th.x, -th.y), th, make_float2(1.f, 1.f)));
              dpk[c / 2] = pack2<BF16>(ds.x, ds.y);
            }
          } else if (ALIBI && !CAP) {
            // ALiBi without cap: x = s·scale·log2(e) + (abase - lse2 -
            // slope·log2(e)·c), two keys per packed instruction.
            const float2 sc2 = make_float2(p.scale, p.scale), ndl2 = make_float2(-dlt, -dlt);
            const float2 base2 = make_float2(abase - lse2, abase - lse2), nsl2 = make_float2(-slope2, -slope2);
#pragma unroll
            for (int c = 0; c < 32; c += 2) {
              const int cc = 64 * eg + 32 * half + c;
              const float2 bias = __ffma2_rn(nsl2, make_float2((float)cc, (float)(cc + 1)), base2);
              const float2 x = __ffma2_rn(make_float2(__uint_as_float(sr[32 * half + c]), __uint_as_float(sr[32 * half + c + 1])),
                                          make_float2(sl2, sl2), bias);
              float pr0 = ex2(x.x), pr1 = ex2(x.y);
              if (MASKED) {
                pr0 = ((unsigned)(cc - clo) < (unsigned)(chi - clo)) ? pr0 : 0.f;
                pr1 = ((unsigned)(cc + 1 - clo) < (unsigned)(chi - clo)) ? pr1 : 0.f;
              }
              const float2 dd = __fadd2_rn(make_float2(__uint_as_float(dr[c]), __uint_as_float(dr[c + 1])), ndl2);
              const float2 ds = __fmul2_rn(__fmul2_rn(make_float2(pr0, pr1), dd), sc2);
              dpk[c / 2] = pack2<BF16>(ds.x, ds.y);
            }
          } else
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            float ds2[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int cc = 64 * eg + 32 * half + c + h;
              const float raw = __uint_as_float(sr[32 * half + c + h]);
              float pr, t = 0.f;
              float x;
              if (CAP || ALIBI) {
                x = logit2<CAP, TIER>(raw, sl2, cap_in, cap_out, &t);
                if (ALIBI) x = fmaf(-slope2, (float)cc, x + abase);
                x -= lse2;
              } else {
                x = fmaf(raw, sl2, -lse2);
              }
              pr = ex2(x);
              if (MASKED) pr = ((unsigned)(cc - clo) < (unsigned)(chi - clo)) ? pr : 0.f;
              float ds = pr * (__uint_as_float(dr[c + h]) - dlt) * p.scale;
              if (CAP) ds *= (1.f - t * t);
              ds2[h] = ds;
            }
            dpk[c / 2] = pack2<BF16>(ds2[0], ds2[1]);
          }
          // dS of this 32-key half -> 16-byte chunks [4·half, 4·half + 4) of
          // this row of the warpgroup's swizzled sub-tile; dQ(i-1) has read
          // the tile by then.
          if (half == 0 && i > 0 && !warp_wait(bar(kDSFree), (uint32_t)((i - 1) & 1), ctl)) return false;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            *reinterpret_cast<uint4*>(ds_row + sw128_offset(row, 4 * half + j)) =
                make_uint4(dpk[4 * j], dpk[4 * j + 1], dpk[4 * j + 2], dpk[4 * j + 3]);
        }
        return true;
      };
      using I2 = std::integral_constant<int, 2>;
      using I1 = std::integral_constant<int, 1>;
      using I0 = std::integral_constant<int, 0>;
      if (tier == 2) ok = full ? step(std::false_type{}, I2{}) : step(std::true_type{}, I2{});
      else if (tier == 1) ok = full ? step(std::false_type{}, I1{}) : step(std::true_type{}, I1{});
      else ok = full ? step(std::false_type{}, I0{}) : step(std::true_type{}, I0{});
      if (!ok) break;
      fence_async_shared();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kDSFull));
    }
    if (eg == 0) {
      bool good = ok;
      if (good && n_iter > 0) good = warp_wait(bar(kAccDone), 0, ctl);
      good = good && !*abort_flag;
      // Q's tile (and dO's after it, for the fp32 tile of accumulate mode)
      // is free once every MMA is done.
      uint8_t* stage_dq = smem + L::kOffQ;
      const bool acc = p.grad_acc != 0;
      if (good && !(acc && n_iter == 0)) {
        tc_fence_after();
        if (acc) stage_tmem_row_f32<D>(tmem + lane_base + L::kTmemDQ, stage_dq, row);
        else stage_tmem_row<D, BF16>(tmem + lane_base + L::kTmemDQ, stage_dq, row, n_iter == 0);
        fence_async_shared();
      }
      if (lane == 0) warp_ok[wq] = good ? 1 : 0;
      named_sync(1, 128);
      if (wq == 0 && lane == 0 && warp_ok[0] && warp_ok[1] && warp_ok[2] && warp_ok[3]) {
        if (!acc) {
          for (int s = 0; s < L::kSub; ++s)
            tma_store_4d(&tmDQ, smem_u32(stage_dq) + s * (kRows * 128), s * 64, q0, hq, b);
        } else if (n_iter > 0) {
          for (int s = 0; s < D / 32; ++s)
            tma_reduce_add_4d(&tmDQ, smem_u32(stage_dq) + s * (kRows * 128), s * 32, q0, hq, b);
        }
        tma_store_commit();
        tma_store_wait_all();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <typename K>
bool set_smem(K kern, uint32_t bytes) {
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) ==
         cudaSuccess;
}

template <int D, bool BF16, bool CAP, bool ALIBI>
int launch_bwd(const Params& p, int dtype, cudaStream_t st) {
  const int gdt = p.grad_acc ? BFA_DTYPE_F32 : dtype;  // dtype of dq/dk/dv
  auto run_dkdv = [&]() -> int {
    using L = DkdvLayout<D>;
    auto kern = dkdv_kernel<D, BF16, CAP, ALIBI>;
    static std::once_flag once;
    static bool attr_ok = false;
    std::call_once(once, [&] { attr_ok = set_smem(kern, L::kSmemBytes); });
    if (!attr_ok) return cuda_fail("dkdv_kernel shared-memory attribute", cudaSuccess);
    CUtensorMap m[6];
    if (!make_tmap_bhsd(&m[0], p.k, dtype, D, p.Sk, p.Hkv, p.B, p.sk_, kRows) ||
        !make_tmap_bhsd(&m[1], p.v, dtype, D, p.Sk, p.Hkv, p.B, p.sv_, kRows) ||
        !make_tmap_bhsd(&m[2], p.q, dtype, D, p.Sq, p.Hq, p.B, p.sq_, kInner) ||
        !make_tmap_bhsd(&m[3], p.dout, dtype, D, p.Sq, p.Hq, p.B, p.sdo_, kInner) ||
        !make_tmap_bhsd(&m[4], p.dk, gdt, D, p.Sk, p.Hkv, p.B, p.sdk_, kRows) ||
        !make_tmap_bhsd(&m[5], p.dv, gdt, D, p.Sk, p.Hkv, p.B, p.sdv_, kRows))
      return BFA_ERR_CUDA;  // make_tmap_bhsd recorded the detail
    const unsigned grid = (unsigned)((p.Sk + kRows - 1) / kRows) * p.Hkv * p.B;
    kern<<<grid, kThreads, L::kSmemBytes, st>>>(m[0], m[1], m[2], m[3], m[4], m[5], p);
    note_launch();
    return launch_status("dkdv_kernel launch");
  };
  auto run_dq = [&]() -> int {
    using L = DqLayout<D>;
    auto kern = dq_kernel<D, BF16, CAP, ALIBI>;
    static std::once_flag once;
    static bool attr_ok = false;
    std::call_once(once, [&] { attr_ok = set_smem(kern, L::kSmemBytes); });
    if (!attr_ok) return cuda_fail("dq_kernel shared-memory attribute", cudaSuccess);
    CUtensorMap m[6];
    if (!make_tmap_bhsd(&m[0], p.q, dtype, D, p.Sq, p.Hq, p.B, p.sq_, kRows) ||
        !make_tmap_bhsd(&m[1], p.dout, dtype, D, p.Sq, p.Hq, p.B, p.sdo_, kRows) ||
        !make_tmap_bhsd(&m[2], p.k, dtype, D, p.Sk, p.Hkv, p.B, p.sk_, L::kKeys) ||
        !make_tmap_bhsd(&m[3], p.v, dtype, D, p.Sk, p.Hkv, p.B, p.sv_, L::kKeys) ||
        !make_tmap_bhsd(&m[4], p.dq, gdt, D, p.Sq, p.Hq, p.B, p.sdq_, kRows))
      return BFA_ERR_CUDA;  // make_tmap_bhsd recorded the detail
    // O (fused Δ only; otherwise a copy of the Q map that is never read).
    if (p.fuse_delta) {
      if (!make_tmap_bhsd(&m[5], p.o, dtype, D, p.Sq, p.Hq, p.B, p.so_, kRows))
        return BFA_ERR_CUDA;  // make_tmap_bhsd recorded the detail
    } else {
      m[5] = m[0];
    }
    const unsigned grid = (unsigned)((p.Sq + kRows - 1) / kRows) * p.Hq * p.B;
    kern<<<grid, kThreads, L::kSmemBytes, st>>>(m[0], m[1], m[2], m[3], m[4], m[5], p);
    note_launch();
    return launch_status("dq_kernel launch");
  };
  // With a fused Δ the dQ kernel writes the row statistics dK/dV reads, so
  // it runs first.
  int rc = BFA_OK;
  if (p.fuse_delta) {
    rc = run_dq();
    if (rc == BFA_OK && (p.phases & BFA_BWD_PHASE_DKDV)) rc = run_dkdv();
    return rc;
  }
  if (p.phases & BFA_BWD_PHASE_DKDV) rc = run_dkdv();
  if (rc == BFA_OK && (p.phases & BFA_BWD_PHASE_DQ)) rc = run_dq();
  return rc;
}

template <int D, bool BF16>
int dispatch_flags(const Params& p, int dtype, cudaStream_t st) {
  const bool cap = p.soft_cap > 0.f, alibi = p.alibi != nullptr;
  if (cap && alibi) return launch_bwd<D, BF16, true, true>(p, dtype, st);
  if (cap) return launch_bwd<D, BF16, true, false>(p, dtype, st);
  if (alibi) return launch_bwd<D, BF16, false, true>(p, dtype, st);
  return launch_bwd<D, BF16, false, false>(p, dtype, st);
}

}  // namespace

bool sm100_bwd_eligible(const Params& p, int dtype) {
  if (dtype != BFA_DTYPE_BF16 && dtype != BFA_DTYPE_F16) return false;
  if (p.D != 64 && p.D != 128 && p.D != 256) return false;
  if (p.Sq < 1 || p.Sk < 1 || p.B < 1 || p.Hq < 1) return false;
  if (!device_is_sm100()) return false;
  const int ges = p.grad_acc ? 4 : 2;
  return tma_layout_ok(p.q, p.sq_, 2) && tma_layout_ok(p.k, p.sk_, 2) &&
         tma_layout_ok(p.v, p.sv_, 2) && tma_layout_ok(p.dout, p.sdo_, 2) &&
         tma_layout_ok(p.dq, p.sdq_, ges) && tma_layout_ok(p.dk, p.sdk_, ges) &&
         tma_layout_ok(p.dv, p.sdv_, ges);
}

bool sm100_bwd_fuses_delta(const Params& p, int dtype) {
  static const bool enabled = [] {
    const char* e = std::getenv("BFA_BWD_FUSE_DELTA");
    return !(e && e[0] == '0');
  }();
  if (!enabled || !p.lse || !p.lse2 || !sm100_bwd_eligible(p, dtype))
    return false;
  return tma_layout_ok(p.o, p.so_, 2);  // the dQ kernel TMA-loads the O tile
}

int sm100_bwd(const Params& p, int dtype, cudaStream_t st) {
  if (p.D == 256) return sm100_bwd256(p, dtype, st);
  const bool bf16 = dtype == BFA_DTYPE_BF16;
  if (p.D == 64) return bf16 ? dispatch_flags<64, true>(p, dtype, st) : dispatch_flags<64, false>(p, dtype, st);
  return bf16 ? dispatch_flags<128, true>(p, dtype, st) : dispatch_flags<128, false>(p, dtype, st);
}

}  // namespace bfa
