// sm100_bwd256.cu -- tcgen05 / TMA / TMEM attention backward for head_dim 256
// (bf16 / fp16), e.g. Gemma2-style layers.
//
// Same gradients as sm100_bwd.cu (which covers head_dim 64 / 128) and the
// reference kernels flash_attn_bwd_dq_kernel (npu_flash_attention.py:298-402)
// and flash_attn_bwd_dkdv_kernel (:407-560) with HEAD_DIM = 256, plus the
// host GQA sum (:735-737), which happens in TMEM here:
//   P  = exp(u_ij - lse_i)        u = transformed logit (cap, ALiBi), masked
//   dP = dO_i · V_j,  dS = P ∘ (dP - Δ_i) · scale · (1 - tanh²)
//   dV_j += P_ij dO_i,  dK_j += dS_ij Q_i,  dQ_i += dS_ij K_j
//
// At D = 256 the fp32 accumulators of a 128-row tile are 256 TMEM columns
// each, half of the 512 a CTA has, and a 128 x 256 bf16 operand tile is 64 KB
// of shared memory. So:
//  * dK and dV are two passes of one kernel template over the same key tile
//    (MODE_DV: Sᵀ, Pᵀ, dV += Pᵀ dO; MODE_DK: Sᵀ, dPᵀ, dSᵀ, dK += dSᵀ Q), each
//    with its accumulator and double-buffered 64-column Sᵀ / dPᵀ in TMEM.
//    The dV pass recomputes Sᵀ once more than a joint pass would (10·D
//    instead of 8·D FLOP per pair for dK/dV).
//  * dQ takes 64-key steps: S and dP (64 columns each), dQ (256) and Q
//    itself (the A operand of S, 16-bit, 128 columns) fill the 512 columns;
//    dO stays in shared memory.
//  * Operands stream through rings of 32 KB units (64 rows x 256 dims) in the
//    order the MMAs consume them; a unit that two MMAs read far apart (Q for
//    Sᵀ and for dK; K for S and for dQ) is loaded twice, once per use, so
//    every unit is released by one MMA and the rings stay FIFO.
// Warp roles (384 threads): warp 0 TMA producer, warp 1 MMA issuer, warp 2
// TMEM allocator, warps 4-11 two elementwise warpgroups that split each
// step's 64 columns; each thread owns one TMEM lane (a key row in the dK/dV
// kernel, a query row in the dQ kernel).
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>
#include <type_traits>

#include "bfa_internal.h"
#include "sm100_bwd_common.cuh"
#include "sm100_host.h"
#include "sm100_ptx.cuh"

namespace bfa {
namespace {

using namespace sm100;
using namespace bwd;

constexpr int kD = 256;
constexpr uint32_t kUnit = 32768;       // 64 rows x 256 dims x 2 bytes
constexpr uint32_t kSub64 = 64 * 128;   // [64 rows][64 dims] swizzled sub-tile
constexpr uint32_t kSub128 = 128 * 128; // [128 rows][64 dims]
constexpr int kModeDV = 0, kModeDK = 1;

// (batch, kv-head) units per group in the dK/dV block order (as sm100_bwd.cu).
constexpr int kUnitGroup = 8;

// Stage columns [c_begin, c_end) (multiples of 32) of a D = 256 fp32 TMEM row:
// 16-bit into 128-row swizzled sub-tiles of 64 columns, or (F32) fp32 into
// sub-tiles of 32 columns.
template <bool F32, bool BF16>
__device__ __forceinline__ void stage_cols(uint32_t taddr, uint8_t* stage, int row, int c_begin, int c_end,
                                           bool zero) {
#pragma unroll 1
  for (int c = c_begin; c < c_end; c += 32) {
    uint32_t r[32];
    if (!zero) {
      tmem_ld32(taddr + c, r);
      tmem_ld_wait();
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) r[i] = 0u;
    }
    if (F32) {
#pragma unroll
      for (int q = 0; q < 8; ++q)
        *reinterpret_cast<uint4*>(stage + (c / 32) * kSub128 + sw128_offset(row, q)) =
            make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w;
        w.x = pack2<BF16>(__uint_as_float(r[8 * q + 0]), __uint_as_float(r[8 * q + 1]));
        w.y = pack2<BF16>(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3]));
        w.z = pack2<BF16>(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5]));
        w.w = pack2<BF16>(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7]));
        const int col = c + 8 * q;
        *reinterpret_cast<uint4*>(stage + (col >> 6) * kSub128 + sw128_offset(row, (col & 63) >> 3)) = w;
      }
    }
  }
}

// ============================================================== dK / dV
// MODE_DV: K resident; ring units Q_i (Sᵀ) and dO_i (dV), consumed in the
//   order Sᵀ(0), Sᵀ(1), dV(0), Sᵀ(2), dV(1), ...
// MODE_DK: K and V resident; ring units Q_i (Sᵀ), dO_i (dPᵀ), Q'_i (dK),
//   consumed in the order Sᵀ(0), dPᵀ(0), Sᵀ(1), dPᵀ(1), dK(0), Sᵀ(2), ...
// Row statistics of step i (lse·log2 e and Δ of its 64 query rows) come in
// a separate two-entry ring that the elementwise warps release.
template <int MODE>
struct Kv256Layout {
  static constexpr int NS = MODE == kModeDV ? 5 : 3;  // ring units
  static constexpr int NR = MODE == kModeDV ? 4 : 2;  // row-statistics entries
  static constexpr uint32_t kRowBytes = MODE == kModeDV ? 256 : 512;
  static constexpr uint32_t kOffK = 0;
  static constexpr uint32_t kOffV = 65536;
  static constexpr uint32_t kOffRing = MODE == kModeDV ? 65536 : 131072;
  static constexpr uint32_t kOffRow = kOffRing + NS * kUnit;
  static constexpr uint32_t kOffBar = kOffRow + NR * kRowBytes;
  static constexpr uint32_t kSmemBytes = kOffBar + 512 + 1024;
  // TMEM: Sᵀ(b) at 64·b; dPᵀ(b) at 128 + 64·b (MODE_DK); the accumulator at 256.
  static constexpr uint32_t kTmemS = 0, kTmemDP = 128, kTmemAcc = 256;
  static_assert(kSmemBytes <= 232448, "smem budget");
};

// Calls f(op, i) in MMA issue order. MODE_DV: op 0 = Sᵀ(i), 1 = dV(i).
// MODE_DK: op 0 = Sᵀ(i), 2 = dPᵀ(i), 3 = dK(i).
template <int MODE, typename F>
__device__ __forceinline__ bool kv_ops(int n, F&& f) {
  if (MODE == kModeDV) {
    for (int i = 0; i < n; ++i) {
      if (i == 0) {
        if (!f(0, 0)) return false;
      }
      if (i + 1 < n && !f(0, i + 1)) return false;
      if (!f(1, i)) return false;
    }
  } else {
    for (int i = 0; i < n; ++i) {
      if (i == 0) {
        if (!f(0, 0) || !f(2, 0)) return false;
      }
      if (i + 1 < n && (!f(0, i + 1) || !f(2, i + 1))) return false;
      if (!f(3, i)) return false;
    }
  }
  return true;
}

template <int MODE, bool BF16, bool CAP, bool ALIBI>
__global__ void __launch_bounds__(kThreads, 1)
    dkdv256_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                   const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                   const __grid_constant__ CUtensorMap tmOut, const Params p) {
  using L = Kv256Layout<MODE>;
  constexpr int NS = L::NS, NR = L::NR;
  constexpr bool DK = MODE == kModeDK;
  enum {
    kKVFull = 0,
    kFull = 1,
    kEmpty = 1 + NS,
    kRFull = 1 + 2 * NS,
    kREmpty = kRFull + NR,
    kSFull = kREmpty + NR,  // Sᵀ (and dPᵀ) of buffer b are in TMEM
    kEWDone = kSFull + 2,   // Pᵀ / dSᵀ of buffer b are in TMEM (8 warps)
    kAccDone = kEWDone + 2,
    kDrain = kAccDone + 1,
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
  // (query block, key block) is on; step i of the loops below is the i-th
  // visited step, which each consumer finds with its own walker.
  auto step_head = [&](int s) { return hkv * p.G + s / n_qt; };
  auto step_q0 = [&](int s) { return (qt0 + s % n_qt) * kInner; };
  auto step_on = [&](int s) { return block_on(p, b, step_head(s), step_q0(s) / kMaskBlock, kt); };
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
    for (int i = 0; i < kNumBars; ++i) {
      const bool ew = (i >= kREmpty && i < kREmpty + NR) || (i >= kEWDone && i < kEWDone + 2);
      mbar_init(bar(i), ew ? 8u : 1u);
    }
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
  auto unit_addr = [&](int n) -> uint32_t { return sbase + L::kOffRing + (uint32_t)(n % NS) * kUnit; };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      if (n_iter > 0) {
        mbar_arrive_expect_tx(bar(kKVFull), DK ? 2 * 65536 : 65536);
        for (int s = 0; s < 4; ++s) {
          tma_load_4d(sbase + L::kOffK + s * kSub128, &tmK, bar(kKVFull), s * 64, c0, hkv, b);
          if (DK) tma_load_4d(sbase + L::kOffV + s * kSub128, &tmV, bar(kKVFull), s * 64, c0, hkv, b);
        }
      }
      int n = 0;
      int nr = 0;
      auto w0 = make_walker(next_step, -1), w1 = make_walker(next_step, -1), w2 = make_walker(next_step, -1);
      kv_ops<MODE>(n_iter, [&](int op, int i) -> bool {
        const int sv = op == 0 ? w0.step(i) : (op == 1 || op == 2) ? w1.step(i) : w2.step(i);
        if (op == 1 && !DK) {
          // dV(i) needs dO_i; nothing else to load here.
        }
        const int slot = n % NS;
        if (n >= NS && !mbar_wait(bar(kEmpty + slot), ((n / NS) & 1) ^ 1, ctl, BFA_ERR_DEVICE_TIMEOUT))
          return false;
        const int hq = step_head(sv), q0 = step_q0(sv);
        const bool is_do = DK ? op == 2 : op == 1;
        mbar_arrive_expect_tx(bar(kFull + slot), kUnit);
        for (int s = 0; s < 4; ++s)
          tma_load_4d(unit_addr(n) + s * kSub64, is_do ? &tmDO : &tmQ, bar(kFull + slot), s * 64, q0, hq, b);
        ++n;
        if (op == 0) {
          // Row statistics of step i, with its first unit.
          const int e = nr % NR;
          if (nr >= NR && !mbar_wait(bar(kREmpty + e), ((nr / NR) & 1) ^ 1, ctl, BFA_ERR_DEVICE_TIMEOUT))
            return false;
          const int64_t rrow = ((int64_t)b * p.Hq + hq) * p.Sq_pad + q0;
          const uint32_t ra = sbase + L::kOffRow + e * L::kRowBytes;
          mbar_arrive_expect_tx(bar(kRFull + e), L::kRowBytes);
          bulk_load(ra, p.lse2 + rrow, 256, bar(kRFull + e));
          if (DK) bulk_load(ra + 256, p.delta + rrow, 256, bar(kRFull + e));
          ++nr;
        }
        return true;
      });
      if (n_iter > 0) drain_wait(bar(kKVFull), 0, p.timeout_ns);
      for (int i = (n > NS ? n - NS : 0); i < n; ++i) drain_wait(bar(kFull + i % NS), (i / NS) & 1, p.timeout_ns);
      for (int i = (nr > NR ? nr - NR : 0); i < nr; ++i)
        drain_wait(bar(kRFull + i % NR), (i / NR) & 1, p.timeout_ns);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idT = idesc_f16(kRows, kInner, BF16, false);  // Sᵀ / dPᵀ: M=128, N=64
      constexpr uint32_t idAcc = idesc_f16(kRows, kD, BF16, true);     // dV / dK: M=128, N=256
      const uint64_t dK0 = desc_kmajor(sbase + L::kOffK), dV0 = desc_kmajor(sbase + L::kOffV);
      int n = 0;
      bool ok = n_iter == 0 || mbar_wait(bar(kKVFull), 0, ctl, BFA_ERR_DEVICE_TIMEOUT);
      if (ok) {
        kv_ops<MODE>(n_iter, [&](int op, int i) -> bool {
          const int bf = i & 1;
          if (op == 1 || op == 3) {
            // Pᵀ(i) / dSᵀ(i) are in TMEM.
            if (!(ok = mbar_wait(bar(kEWDone + bf), (i >> 1) & 1, ctl, BFA_ERR_DEVICE_TIMEOUT))) return false;
          }
          if (!(ok = mbar_wait(bar(kFull + n % NS), (n / NS) & 1, ctl, BFA_ERR_DEVICE_TIMEOUT))) return false;
          tc_fence_after();
          const uint32_t u = unit_addr(n);
          if (op == 0 || op == 2) {
            // Sᵀ = K Q_iᵀ or dPᵀ = V dO_iᵀ: M = 128 keys, N = 64 queries, 16 K-steps of dims.
            const uint64_t da = op == 0 ? dK0 : dV0;
            const uint64_t db = desc_kmajor(u);
            const uint32_t dst = tmem + (op == 0 ? L::kTmemS : L::kTmemDP) + 64 * bf;
#pragma unroll
            for (int kk = 0; kk < kD / 16; ++kk) {
              const uint32_t offa = ((kk >> 2) * kSub128 + (kk & 3) * 32) >> 4;
              const uint32_t offb = ((kk >> 2) * kSub64 + (kk & 3) * 32) >> 4;
              mma_ss(dst, da + offa, db + offb, idT, kk > 0 ? 1u : 0u);
            }
            mma_commit(bar(kEmpty + n % NS));
            if (op == (DK ? 2 : 0)) mma_commit(bar(kSFull + bf));
          } else {
            // dV += Pᵀ dO_i (MODE_DV) or dK += dSᵀ Q_i (MODE_DK): A from TMEM
            // (packed columns [32h, 32h + 16) of the buffer hold query
            // columns [32h, 32h + 32)), B = the unit, MN-major, N = 256 dims.
            const uint32_t a0 = tmem + (DK ? L::kTmemDP : L::kTmemS) + 64 * bf;
            const uint64_t db = desc_mnmajor(u, kSub64);
#pragma unroll
            for (int kk = 0; kk < kInner / 16; ++kk)
              mma_ts(tmem + L::kTmemAcc, a0 + 32 * (kk >> 1) + 8 * (kk & 1), db + ((kk * 2048) >> 4), idAcc,
                     (i > 0 || kk > 0) ? 1u : 0u);
            mma_commit(bar(kEmpty + n % NS));
          }
          ++n;
          return true;
        });
      }
      mma_commit(bar(kAccDone));
      mma_commit(bar(kDrain));
      drain_wait(bar(kDrain), 0, p.timeout_ns);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ elementwise
    // Warpgroup h takes query columns [32h, 32h + 32) of every step; each
    // thread owns one key row (TMEM lane).
    const int eg = (warp - 4) >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const int kj = c0 + row;
    const int64_t gj = (int64_t)kj + p.k_off;
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const float sl2 = p.scale * kLog2e;
    const float cap_in = CAP ? p.scale / p.soft_cap : 0.f;
    const float cap_out = CAP ? p.soft_cap * kLog2e : 0.f;
    bool ok = true;
    // Without documents a step is fully kept exactly when its first query
    // lies in `kept` (no general tile test per step).
    const bool lin_full = p.doc_lo == nullptr;
    const KeptRange kept = kept_queries(p, c0, kRows, kInner);
    int sv = -1;
    for (int i = 0; i < n_iter; ++i) {
      const int bf = i & 1, e = i % NR;
      sv = next_step(sv);
      const int hq = step_head(sv), q0 = step_q0(sv);
      uint32_t wbar = bar(kSFull + bf), wpar = (uint32_t)((i >> 1) & 1);
      if ((p.debug_flags & BFA_DEBUG_INJECT_STALL) && i == 0) {
        wbar = bar(kNever);
        wpar = 0;
      }
      if (!(ok = warp_wait(wbar, wpar, ctl))) break;
      if (!(ok = warp_wait(bar(kRFull + e), (uint32_t)((i / NR) & 1), ctl))) break;
      tc_fence_after();
      const uint32_t tSb = tmem + lane_base + L::kTmemS + 64 * bf + 32 * eg;
      const uint32_t tDb = tmem + lane_base + L::kTmemDP + 64 * bf + 32 * eg;
      const float* rowv = (const float*)(smem + L::kOffRow + e * L::kRowBytes);
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
      uint32_t sr[32], dr[32];
      tmem_ld32(tSb, sr);
      if (DK) tmem_ld32(tDb, dr);
      tmem_ld_wait();
      uint32_t pk[16];
      auto body = [&](auto masked, auto small_tag) {
        constexpr bool MASKED = decltype(masked)::value;
        constexpr int TIER = decltype(small_tag)::value;
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          float v2[2];
          if (CAP && !ALIBI) {
            // Soft-cap without ALiBi: both keys in packed instructions.
            const int cc = 32 * eg + c;
            float2 th;
            const float2 x = cap_logit2x2<TIER>(make_float2(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])),
                                                 cap_in, cap_out, &th);
            const float2 l2 = *reinterpret_cast<const float2*>(rowv + cc);
            float pr0 = ex2(x.x - l2.x), pr1 = ex2(x.y - l2.y);
            if (MASKED) {
              pr0 = ((unsigned)(cc - clo) < (unsigned)(chi - clo)) ? pr0 : 0.f;
              pr1 = ((unsigned)(cc + 1 - clo) < (unsigned)(chi - clo)) ? pr1 : 0.f;
            }
            if (DK) {
              const float2 d2 = *reinterpret_cast<const float2*>(rowv + 64 + cc);
              const float2 dd = __fadd2_rn(make_float2(__uint_as_float(dr[c]), __uint_as_float(dr[c + 1])),
                                           make_float2(-d2.x, -d2.y));
              float2 ds = __fmul2_rn(__fmul2_rn(make_float2(pr0, pr1), dd), make_float2(p.scale, p.scale));
              ds = __fmul2_rn(ds, __ffma2_rn(make_float2(-th.x, -th.y), th, make_float2(1.f, 1.f)));
              v2[0] = ds.x;
              v2[1] = ds.y;
            } else {
              v2[0] = pr0;
              v2[1] = pr1;
            }
          } else {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int cc = 32 * eg + c + h;
            const float raw = __uint_as_float(sr[c + h]);
            float t = 0.f;
            float x = (CAP || ALIBI) ? logit2<CAP, TIER>(raw, sl2, cap_in, cap_out, &t) : raw * sl2;
            if (ALIBI) x += fmaxf(ba, fmaf(slope2, (float)cc, bq));
            float pr = ex2(x - rowv[cc]);
            if (MASKED) pr = ((unsigned)(cc - clo) < (unsigned)(chi - clo)) ? pr : 0.f;
            if (DK) {
              float ds = pr * (__uint_as_float(dr[c + h]) - rowv[64 + cc]) * p.scale;
              if (CAP) ds *= (1.f - t * t);
              v2[h] = ds;
            } else {
              v2[h] = pr;
            }
          }
          }
          pk[c / 2] = pack2<BF16>(v2[0], v2[1]);
        }
      };
      const int tier = CAP ? cap_tier<32>(sr, cap_in) : 0;
      using I2 = std::integral_constant<int, 2>;
      using I1 = std::integral_constant<int, 1>;
      using I0 = std::integral_constant<int, 0>;
      if (tier == 2) {
        if (full) body(std::false_type{}, I2{});
        else body(std::true_type{}, I2{});
      } else if (tier == 1) {
        if (full) body(std::false_type{}, I1{});
        else body(std::true_type{}, I1{});
      } else {
        if (full) body(std::false_type{}, I0{});
        else body(std::true_type{}, I0{});
      }
      // The row statistics are in registers' use: release the entry.
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kREmpty + e));
      // Pᵀ (MODE_DV) over the Sᵀ columns, dSᵀ (MODE_DK) over the dPᵀ
      // columns: packed columns [32h, 32h + 16) of this warpgroup's own fp32
      // columns, read above.
      tmem_st16(DK ? tDb : tSb, pk);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kEWDone + bf));
    }
    // ------------------------------------------------------------ epilogue
    // Warpgroup h writes accumulator columns [128h, 128h + 128). The K (and
    // V) tiles are free once every MMA is done: they stage the 16-bit tile,
    // or (accumulate mode) the fp32 tile.
    bool good = ok;
    if (good && n_iter > 0) good = warp_wait(bar(kAccDone), 0, ctl);
    good = good && !*abort_flag;
    const bool acc = p.grad_acc != 0;
    uint8_t* stage = smem + (acc && !DK ? L::kOffRing : L::kOffK);
    if (good && !(acc && n_iter == 0)) {
      tc_fence_after();
      const uint32_t tacc = tmem + lane_base + L::kTmemAcc;
      if (acc) stage_cols<true, BF16>(tacc, stage, row, 128 * eg, 128 * eg + 128, false);
      else stage_cols<false, BF16>(tacc, stage, row, 128 * eg, 128 * eg + 128, n_iter == 0);
      fence_async_shared();
    }
    if (lane == 0) warp_ok[warp - 4] = good ? 1 : 0;
    named_sync(1, 256);
    if (warp == 4 && lane == 0) {
      bool all = true;
      for (int w = 0; w < 8; ++w) all = all && warp_ok[w];
      if (all) {
        if (!acc) {
          for (int s = 0; s < 4; ++s) tma_store_4d(&tmOut, smem_u32(stage) + s * kSub128, s * 64, c0, hkv, b);
        } else if (n_iter > 0) {
          for (int s = 0; s < 8; ++s)
            tma_reduce_add_4d(&tmOut, smem_u32(stage) + s * kSub128, s * 32, c0, hkv, b);
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
// One CTA per (batch, q-head, 128-row query tile), 64-key steps:
//   S = Q K_jᵀ (TS: Q from TMEM), dP = dO V_jᵀ (SS), dS (elementwise, into a
//   swizzled shared tile), dQ += dS K_j (SS, K_j MN-major).
// TMEM: S [0, 64), dP [64, 128), dQ [128, 384), Q [384, 512) (16-bit, two
// per column). S and dP are single-buffered: the elementwise warps release
// each as soon as it is in registers, so S(j+1), dP(j+1) run while dS(j) is
// computed. Ring units (64 keys x 256 dims), in MMA order:
//   K_0, V_0, K_1, V_1, K'_0, K_2, V_2, K'_1, ...
// (K'_j: K_j again, for dQ(j)). Q arrives in ring slots 2-3 and is copied
// into TMEM before those slots are used. With a fused Δ, the O tile arrives
// in slots 0-1 and the ring starts once Δ is formed.
struct Dq256Layout {
  static constexpr int kKeys = 64;
  static constexpr int NS = 4;
  static constexpr uint32_t kOffDO = 0;                      // [128 rows][256 dims]: 64 KB
  static constexpr uint32_t kOffDS = 65536;                  // [128 rows][64 keys]: 16 KB
  static constexpr uint32_t kOffRing = kOffDS + 16384;       // NS x 32 KB
  static constexpr uint32_t kOffQ = kOffRing + 2 * kUnit;    // Q staging = ring slots 2-3
  static constexpr uint32_t kOffBar = kOffRing + NS * kUnit;
  static constexpr uint32_t kOffDlt = kOffBar + 512;         // fused Δ: [2 warpgroups][128 rows] partials
  static constexpr uint32_t kSmemBytes = kOffDlt + 1024 + 1024;
  static constexpr uint32_t kTmemS = 0, kTmemDP = 64, kTmemDQ = 128, kTmemQ = 384;
  static_assert(kSmemBytes <= 232448, "smem budget");
};

// Calls f(op, j) in MMA issue order: op 0 = S(j), 1 = dP(j), 2 = dQ(j).
template <typename F>
__device__ __forceinline__ bool dq_ops(int n, F&& f) {
  for (int j = 0; j < n; ++j) {
    if (j == 0 && (!f(0, 0) || !f(1, 0))) return false;
    if (j + 1 < n && (!f(0, j + 1) || !f(1, j + 1))) return false;
    if (!f(2, j)) return false;
  }
  return true;
}

template <bool BF16, bool CAP, bool ALIBI>
__global__ void __launch_bounds__(kThreads, 1)
    dq256_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                 const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                 const __grid_constant__ CUtensorMap tmDQ, const __grid_constant__ CUtensorMap tmO,
                 const Params p) {
  using L = Dq256Layout;
  constexpr int NS = L::NS;
  constexpr int NK = L::kKeys;
  enum {
    kQFull = 0,
    kFull = 1,
    kEmpty = 1 + NS,
    kSPFull = 1 + 2 * NS,   // S(j), dP(j) in TMEM
    kSRead = kSPFull + 1,   // S(j) in registers (8 warps)
    kDPRead = kSRead + 1,   // dP(j) in registers (8 warps)
    kDSFull = kDPRead + 1,  // dS(j) in shared memory (8 warps)
    kOpsReady = kDSFull + 1,  // Q in TMEM (8 warps)
    kDSFree = kOpsReady + 1,  // dQ(j) has read dS(j)
    kAccDone = kDSFree + 1,
    kDrain = kAccDone + 1,
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
  const int n_qt = (p.Sq + kRows - 1) / kRows;
  const int bh = blockIdx.x % (p.B * p.Hq);
  const int qt = n_qt - 1 - (int)(blockIdx.x / (p.B * p.Hq));  // heaviest causal tiles first
  const int hq = bh % p.Hq, b = bh / p.Hq;
  const int hkv = hq / p.G;
  const int q0 = qt * kRows;
  int klo, khi;
  key_range(p, q0, min(q0 + kRows, p.Sq), &klo, &khi);
  const int jt0 = klo / NK;
  const int jend = (khi > klo) ? (khi + NK - 1) / NK : jt0;
  // Block-sparse mask: 64-key step j is visited only when block
  // (q0 / 128, 64 j / 128) is on; each consumer walks the visited steps.
  auto step_on = [&](int j) { return block_on(p, b, hq, q0 / kMaskBlock, j * NK / kMaskBlock); };
  int n_iter = jend - jt0;
  if (p.blk) {
    n_iter = 0;
    for (int j = jt0; j < jend; ++j) n_iter += step_on(j) ? 1 : 0;
  }
  auto next_tile = [&](int j) {
    do { ++j; } while (p.blk && j < jend && !step_on(j));
    return j;
  };

  WaitCtl ctl{abort_flag, p.status, p.timeout_ns};

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i) mbar_init(bar(i), (i >= kSRead && i <= kOpsReady) ? 8u : 1u);
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
  auto unit_addr = [&](int n) -> uint32_t { return sbase + L::kOffRing + (uint32_t)(n % NS) * kUnit; };

  if (warp == 0) {
    if (lane == 0) {
      // A query tile that sees no key loads nothing: its epilogue stages
      // zeros, which must not meet a TMA write in flight.
      const bool fuse = p.fuse_delta != 0;
      if (n_iter > 0) {
        mbar_arrive_expect_tx(bar(kQFull), (fuse ? 3 : 2) * 65536);
        for (int s = 0; s < 4; ++s) {
          tma_load_4d(sbase + L::kOffQ + s * kSub128, &tmQ, bar(kQFull), s * 64, q0, hq, b);
          tma_load_4d(sbase + L::kOffDO + s * kSub128, &tmDO, bar(kQFull), s * 64, q0, hq, b);
          // Fused Δ: the O tile into ring slots 0-1, free until Δ is formed.
          if (fuse) tma_load_4d(sbase + L::kOffRing + s * kSub128, &tmO, bar(kQFull), s * 64, q0, hq, b);
        }
      }
      int n = 0;
      auto w0 = make_walker(next_tile, jt0 - 1), w1 = make_walker(next_tile, jt0 - 1),
           w2 = make_walker(next_tile, jt0 - 1);
      dq_ops(n_iter, [&](int op, int j) -> bool {
        const int slot = n % NS;
        bool ok = true;
        if (n >= NS) ok = mbar_wait(bar(kEmpty + slot), ((n / NS) & 1) ^ 1, ctl, BFA_ERR_DEVICE_TIMEOUT);
        else if (slot >= 2 || fuse)  // Q staging (and, fused, the O tile) consumed
          ok = mbar_wait(bar(kOpsReady), 0, ctl, BFA_ERR_DEVICE_TIMEOUT);
        if (!ok) return false;
        mbar_arrive_expect_tx(bar(kFull + slot), kUnit);
        const int key0 = (op == 0 ? w0.step(j) : op == 1 ? w1.step(j) : w2.step(j)) * NK;
        for (int s = 0; s < 4; ++s)
          tma_load_4d(unit_addr(n) + s * kSub64, op == 1 ? &tmV : &tmK, bar(kFull + slot), s * 64, key0, hkv, b);
        ++n;
        return true;
      });
      if (n_iter > 0) drain_wait(bar(kQFull), 0, p.timeout_ns);
      for (int i = (n > NS ? n - NS : 0); i < n; ++i) drain_wait(bar(kFull + i % NS), (i / NS) & 1, p.timeout_ns);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idSP = idesc_f16(kRows, NK, BF16, false);  // M=128, N=64
      constexpr uint32_t idAcc = idesc_f16(kRows, kD, BF16, true);   // M=128, N=256
      const uint64_t dDO = desc_kmajor(sbase + L::kOffDO);
      const uint64_t dS0 = desc_kmajor(sbase + L::kOffDS);
      int n = 0;
      bool ok = n_iter == 0 || mbar_wait(bar(kOpsReady), 0, ctl, BFA_ERR_DEVICE_TIMEOUT);
      if (ok) {
        dq_ops(n_iter, [&](int op, int j) -> bool {
          if (op == 0 && j > 0) {
            if (!(ok = mbar_wait(bar(kSRead), (j - 1) & 1, ctl, BFA_ERR_DEVICE_TIMEOUT))) return false;
          } else if (op == 1 && j > 0) {
            if (!(ok = mbar_wait(bar(kDPRead), (j - 1) & 1, ctl, BFA_ERR_DEVICE_TIMEOUT))) return false;
          } else if (op == 2) {
            if (!(ok = mbar_wait(bar(kDSFull), j & 1, ctl, BFA_ERR_DEVICE_TIMEOUT))) return false;
          }
          if (!(ok = mbar_wait(bar(kFull + n % NS), (n / NS) & 1, ctl, BFA_ERR_DEVICE_TIMEOUT))) return false;
          tc_fence_after();
          const uint32_t u = unit_addr(n);
          if (op == 0) {
            const uint64_t dk = desc_kmajor(u);
#pragma unroll
            for (int kk = 0; kk < kD / 16; ++kk) {
              const uint32_t offk = ((kk >> 2) * kSub64 + (kk & 3) * 32) >> 4;
              mma_ts(tmem + L::kTmemS, tmem + L::kTmemQ + 8 * kk, dk + offk, idSP, kk > 0 ? 1u : 0u);
            }
          } else if (op == 1) {
            const uint64_t dv = desc_kmajor(u);
#pragma unroll
            for (int kk = 0; kk < kD / 16; ++kk) {
              const uint32_t offa = ((kk >> 2) * kSub128 + (kk & 3) * 32) >> 4;
              const uint32_t offv = ((kk >> 2) * kSub64 + (kk & 3) * 32) >> 4;
              mma_ss(tmem + L::kTmemDP, dDO + offa, dv + offv, idSP, kk > 0 ? 1u : 0u);
            }
          } else {
            const uint64_t mk = desc_mnmajor(u, kSub64);
#pragma unroll
            for (int kk = 0; kk < NK / 16; ++kk)
              mma_ss(tmem + L::kTmemDQ, dS0 + ((kk * 32) >> 4), mk + ((kk * 2048) >> 4), idAcc,
                     (j > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(bar(kEmpty + n % NS));
          if (op == 1) mma_commit(bar(kSPFull));
          if (op == 2) mma_commit(bar(kDSFree));
          ++n;
          return true;
        });
      }
      mma_commit(bar(kAccDone));
      mma_commit(bar(kDrain));
      drain_wait(bar(kDrain), 0, p.timeout_ns);
    }
  } else if (warp >= 4) {
    // Warpgroup h takes key columns [32h, 32h + 32) of every step; each
    // thread owns one query row.
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
    float* dpart = reinterpret_cast<float*>(smem + L::kOffDlt);  // [warpgroup][row]
    bool ok = true;
    // Q into TMEM: warpgroup h moves dims [128h, 128h + 128) of this thread's
    // row (two 64-dim sub-tiles) into columns [64h, 64h + 64) of the Q area.
    // Fused Δ: each warpgroup also sums O·dO over the same dims (O in ring
    // slots 0-1, dO resident); the halves meet through shared memory. A tile
    // that sees no key has Δ = 0 (its P is 0). TMA fills rows past Sq with 0.
    if (n_iter > 0) {
      ok = warp_wait(bar(kQFull), 0, ctl);
      if (ok) {
        float2 acc2 = make_float2(0.f, 0.f);
#pragma unroll 1
        for (int s = 2 * eg; s < 2 * eg + 2; ++s) {
          uint32_t r[32];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 w = *reinterpret_cast<const uint4*>(smem + L::kOffQ + s * kSub128 + sw128_offset(row, c));
            r[4 * c] = w.x; r[4 * c + 1] = w.y; r[4 * c + 2] = w.z; r[4 * c + 3] = w.w;
          }
          tmem_st32(tmem + lane_base + L::kTmemQ + 32 * s, r);
          if (fuse) {
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const uint4 o4 = *reinterpret_cast<const uint4*>(smem + L::kOffRing + s * kSub128 + sw128_offset(row, c));
              const uint4 d4 = *reinterpret_cast<const uint4*>(smem + L::kOffDO + s * kSub128 + sw128_offset(row, c));
              const uint32_t ow[4] = {o4.x, o4.y, o4.z, o4.w}, dw[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) acc2 = __ffma2_rn(unpack2<BF16>(ow[e]), unpack2<BF16>(dw[e]), acc2);
            }
          }
        }
        if (fuse) dpart[eg * kRows + row] = acc2.x + acc2.y;
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(kOpsReady));
        // Both warpgroups' halves (the arrivals release the shared stores),
        // added in the same order in both.
        if (fuse && (ok = warp_wait(bar(kOpsReady), 0, ctl))) dlt = dpart[row] + dpart[kRows + row];
      }
    }
    if (fuse && eg == 0 && qi < p.Sq_pad) {
      p.delta[ridx] = dlt;
      p.lse2[ridx] = lse2;
    }
    uint8_t* ds_base = smem + L::kOffDS;
    // Without documents a key step is fully kept exactly when its first key
    // lies in `kept` (no general tile test per step).
    const bool lin_full = p.doc_lo == nullptr;
    const KeptRange kept = kept_keys(p, q0, kRows, NK, true);
    int jv = jt0 - 1;
    for (int j = 0; j < n_iter && ok; ++j) {
      jv = next_tile(jv);
      const int j0 = jv * NK;
      uint32_t wbar = bar(kSPFull), wpar = (uint32_t)(j & 1);
      if ((p.debug_flags & BFA_DEBUG_INJECT_STALL) && j == 0) {
        wbar = bar(kNever);
        wpar = 0;
      }
      if (!(ok = warp_wait(wbar, wpar, ctl))) break;
      tc_fence_after();
      uint32_t sr[32], dr[32];
      tmem_ld32(tmem + lane_base + L::kTmemS + 32 * eg, sr);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kSRead));
      tmem_ld32(tmem + lane_base + L::kTmemDP + 32 * eg, dr);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kDPRead));
      const bool full = lin_full ? kept.has(j0) : tile_full(p, q0, q0 + kRows, j0, j0 + NK);
      const float abase = ALIBI ? slope2 * (float)(g0 - (int64_t)j0 - p.k_off) : 0.f;
      int clo = 0, chi = NK;  // kept key columns [clo, chi) of this query row (masked steps)
      if (!full) keys_for_query(p, gi, qi < p.Sq, j0, NK, &clo, &chi);
      uint32_t dpk[16];
      auto body = [&](auto masked, auto small_tag) {
        constexpr bool MASKED = decltype(masked)::value;
        constexpr int TIER = decltype(small_tag)::value;
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          float ds2[2];
#pragma unroll
          if (CAP && !ALIBI) {
            // Soft-cap without ALiBi: both keys in packed instructions.
            const int cc = 32 * eg + c;
            float2 th;
            const float2 x = cap_logit2x2<TIER>(make_float2(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])),
                                                 cap_in, cap_out, &th);
            float pr0 = ex2(x.x - lse2), pr1 = ex2(x.y - lse2);
            if (MASKED) {
              pr0 = ((unsigned)(cc - clo) < (unsigned)(chi - clo)) ? pr0 : 0.f;
              pr1 = ((unsigned)(cc + 1 - clo) < (unsigned)(chi - clo)) ? pr1 : 0.f;
            }
            const float2 dd = __fadd2_rn(make_float2(__uint_as_float(dr[c]), __uint_as_float(dr[c + 1])),
                                         make_float2(-dlt, -dlt));
            float2 ds = __fmul2_rn(__fmul2_rn(make_float2(pr0, pr1), dd), make_float2(p.scale, p.scale));
            ds = __fmul2_rn(ds, __ffma2_rn(make_float2(-th.x, -th.y), th, make_float2(1.f, 1.f)));
            ds2[0] = ds.x;
            ds2[1] = ds.y;
          } else {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int cc = 32 * eg + c + h;
            const float raw = __uint_as_float(sr[c + h]);
            float t = 0.f;
            float x = (CAP || ALIBI) ? logit2<CAP, TIER>(raw, sl2, cap_in, cap_out, &t) : raw * sl2;
            if (ALIBI) x = fmaf(-slope2, (float)cc, x + abase);
            float pr = ex2(x - lse2);
            if (MASKED) pr = ((unsigned)(cc - clo) < (unsigned)(chi - clo)) ? pr : 0.f;
            float ds = pr * (__uint_as_float(dr[c + h]) - dlt) * p.scale;
            if (CAP) ds *= (1.f - t * t);
            ds2[h] = ds;
          }
          }
          dpk[c / 2] = pack2<BF16>(ds2[0], ds2[1]);
        }
      };
      const int tier = CAP ? cap_tier<32>(sr, cap_in) : 0;
      using I2 = std::integral_constant<int, 2>;
      using I1 = std::integral_constant<int, 1>;
      using I0 = std::integral_constant<int, 0>;
      if (tier == 2) {
        if (full) body(std::false_type{}, I2{});
        else body(std::true_type{}, I2{});
      } else if (tier == 1) {
        if (full) body(std::false_type{}, I1{});
        else body(std::true_type{}, I1{});
      } else {
        if (full) body(std::false_type{}, I0{});
        else body(std::true_type{}, I0{});
      }
      // dS of this warpgroup's 32 keys -> 16-byte chunks [4h, 4h + 4) of this
      // row of the swizzled [128 rows][64 keys] tile, once dQ(j-1) has read it.
      if (j > 0 && !(ok = warp_wait(bar(kDSFree), (uint32_t)((j - 1) & 1), ctl))) break;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint4*>(ds_base + sw128_offset(row, 4 * eg + q)) =
            make_uint4(dpk[4 * q], dpk[4 * q + 1], dpk[4 * q + 2], dpk[4 * q + 3]);
      fence_async_shared();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kDSFull));
    }
    // ------------------------------------------------------------ epilogue
    // Warpgroup h writes dQ columns [128h, 128h + 128). dO's tile (16-bit) or
    // the ring (fp32, accumulate mode) stages the result; both are free once
    // every MMA is done.
    bool good = ok;
    if (good && n_iter > 0) good = warp_wait(bar(kAccDone), 0, ctl);
    good = good && !*abort_flag;
    const bool acc = p.grad_acc != 0;
    uint8_t* stage = smem + (acc ? L::kOffRing : L::kOffDO);
    if (good && !(acc && n_iter == 0)) {
      tc_fence_after();
      const uint32_t tacc = tmem + lane_base + L::kTmemDQ;
      if (acc) stage_cols<true, BF16>(tacc, stage, row, 128 * eg, 128 * eg + 128, false);
      else stage_cols<false, BF16>(tacc, stage, row, 128 * eg, 128 * eg + 128, n_iter == 0);
      fence_async_shared();
    }
    if (lane == 0) warp_ok[warp - 4] = good ? 1 : 0;
    named_sync(1, 256);
    if (warp == 4 && lane == 0) {
      bool all = true;
      for (int w = 0; w < 8; ++w) all = all && warp_ok[w];
      if (all) {
        if (!acc) {
          for (int s = 0; s < 4; ++s) tma_store_4d(&tmDQ, smem_u32(stage) + s * kSub128, s * 64, q0, hq, b);
        } else if (n_iter > 0) {
          for (int s = 0; s < 8; ++s) tma_reduce_add_4d(&tmDQ, smem_u32(stage) + s * kSub128, s * 32, q0, hq, b);
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
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) == cudaSuccess;
}

template <int MODE, bool BF16, bool CAP, bool ALIBI>
int launch_kv(const Params& p, int dtype, cudaStream_t st) {
  using L = Kv256Layout<MODE>;
  const int gdt = p.grad_acc ? BFA_DTYPE_F32 : dtype;
  auto kern = dkdv256_kernel<MODE, BF16, CAP, ALIBI>;
  static std::once_flag once;
  static bool attr_ok = false;
  std::call_once(once, [&] { attr_ok = set_smem(kern, L::kSmemBytes); });
  if (!attr_ok) return cuda_fail("dkdv256_kernel shared-memory attribute", cudaSuccess);
  CUtensorMap m[5];
  const bool dk = MODE == kModeDK;
  if (!make_tmap_bhsd(&m[0], p.k, dtype, kD, p.Sk, p.Hkv, p.B, p.sk_, kRows) ||
      !make_tmap_bhsd(&m[1], p.v, dtype, kD, p.Sk, p.Hkv, p.B, p.sv_, kRows) ||
      !make_tmap_bhsd(&m[2], p.q, dtype, kD, p.Sq, p.Hq, p.B, p.sq_, kInner) ||
      !make_tmap_bhsd(&m[3], p.dout, dtype, kD, p.Sq, p.Hq, p.B, p.sdo_, kInner) ||
      !make_tmap_bhsd(&m[4], dk ? p.dk : p.dv, gdt, kD, p.Sk, p.Hkv, p.B, dk ? p.sdk_ : p.sdv_, kRows))
    return BFA_ERR_CUDA;  // make_tmap_bhsd recorded the detail
  const unsigned grid = (unsigned)((p.Sk + kRows - 1) / kRows) * p.Hkv * p.B;
  kern<<<grid, kThreads, L::kSmemBytes, st>>>(m[0], m[1], m[2], m[3], m[4], p);
  note_launch();
  return launch_status("dkdv256_kernel launch");
}

template <bool BF16, bool CAP, bool ALIBI>
int launch_bwd(const Params& p, int dtype, cudaStream_t st) {
  const int gdt = p.grad_acc ? BFA_DTYPE_F32 : dtype;
  auto run_dkdv = [&]() -> int {
    const int rc = launch_kv<kModeDV, BF16, CAP, ALIBI>(p, dtype, st);
    return rc ? rc : launch_kv<kModeDK, BF16, CAP, ALIBI>(p, dtype, st);
  };
  auto run_dq = [&]() -> int {
    using L = Dq256Layout;
    auto kern = dq256_kernel<BF16, CAP, ALIBI>;
    static std::once_flag once;
    static bool attr_ok = false;
    std::call_once(once, [&] { attr_ok = set_smem(kern, L::kSmemBytes); });
    if (!attr_ok) return cuda_fail("dq256_kernel shared-memory attribute", cudaSuccess);
    CUtensorMap m[6];
    if (!make_tmap_bhsd(&m[0], p.q, dtype, kD, p.Sq, p.Hq, p.B, p.sq_, kRows) ||
        !make_tmap_bhsd(&m[1], p.dout, dtype, kD, p.Sq, p.Hq, p.B, p.sdo_, kRows) ||
        !make_tmap_bhsd(&m[2], p.k, dtype, kD, p.Sk, p.Hkv, p.B, p.sk_, L::kKeys) ||
        !make_tmap_bhsd(&m[3], p.v, dtype, kD, p.Sk, p.Hkv, p.B, p.sv_, L::kKeys) ||
        !make_tmap_bhsd(&m[4], p.dq, gdt, kD, p.Sq, p.Hq, p.B, p.sdq_, kRows))
      return BFA_ERR_CUDA;  // make_tmap_bhsd recorded the detail
    // O (fused Δ only; otherwise a copy of the Q map that is never read).
    if (p.fuse_delta) {
      if (!make_tmap_bhsd(&m[5], p.o, dtype, kD, p.Sq, p.Hq, p.B, p.so_, kRows))
        return BFA_ERR_CUDA;  // make_tmap_bhsd recorded the detail
    } else {
      m[5] = m[0];
    }
    const unsigned grid = (unsigned)((p.Sq + kRows - 1) / kRows) * p.Hq * p.B;
    kern<<<grid, kThreads, L::kSmemBytes, st>>>(m[0], m[1], m[2], m[3], m[4], m[5], p);
    note_launch();
    return launch_status("dq256_kernel launch");
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

template <bool BF16>
int dispatch(const Params& p, int dtype, cudaStream_t st) {
  const bool cap = p.soft_cap > 0.f, alibi = p.alibi != nullptr;
  if (cap && alibi) return launch_bwd<BF16, true, true>(p, dtype, st);
  if (cap) return launch_bwd<BF16, true, false>(p, dtype, st);
  if (alibi) return launch_bwd<BF16, false, true>(p, dtype, st);
  return launch_bwd<BF16, false, false>(p, dtype, st);
}

}  // namespace

int sm100_bwd256(const Params& p, int dtype, cudaStream_t st) {
  return dtype == BFA_DTYPE_BF16 ? dispatch<true>(p, dtype, st) : dispatch<false>(p, dtype, st);
}

}  // namespace bfa
