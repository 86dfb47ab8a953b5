// sm100_bwd_fused.cu -- one-kernel tcgen05 attention backward (head_dim 128).
//
// Replaces flash_attn_bwd_dkdv_kernel (npu_flash_attention.py:407-560),
// flash_attn_bwd_dq_kernel (:298-402) and the host GQA sum (:735-737) with a
// single pass over the (key tile, query tile) pairs: S and dP are computed
// once per pair instead of once in each of two kernels.
//
// One CTA per (batch, kv-head, 128-key tile) loops over its 64-row query
// tiles and, inside, the GQA group's q-heads (step i: tile i / G, head
// i % G). Per step, M = 128 keys:
//   Sᵀ  = K Qᵢᵀ, dPᵀ = V dOᵢᵀ          (N = 64, TMEM, double-buffered)
//   Pᵀ  -> TMEM (16-bit, A operand of dV);  dSᵀ -> shared memory
//   dQᵢᵀ = Kᵀ dSᵀ                       (M = D, N = 64: A = the K tile read
//                                        MN-major, B = dSᵀ read MN-major)
//   dV += Pᵀ dOᵢ,  dK += dSᵀ Qᵢ          (N = D, fp32 TMEM, summed over the group)
// dQᵢᵀ lands in the TMEM of dPᵀ (read by then). dV, dK and dQ of a step are
// issued in that order, so once dQᵢᵀ is complete the step's Q/dO stage is no
// longer read: the elementwise warps read dQᵢᵀ out (lane = d) and write it
// into that stage as a plain fp32 tile [64 rows][D] -- exactly the rows'
// contiguous 32 KB of the fp32 dQ buffer [B, Hq, Sq, D]. Warp 3 adds the tile
// there with one 1-D bulk reduce-add (cp.reduce.async.bulk .add.f32, done in
// L2) and hands the stage back to the producer once the tile has been read.
// dQ stays bitwise deterministic: the contributions to each query tile are
// added in a fixed order (descending key tile), enforced by a per-tile
// counter in global memory -- warp 3 waits for the counter to reach its turn
// before it adds, and bumps it once the add is complete (checked one step
// later). Key tiles are numbered so that a tile's predecessors have smaller
// block indices (they are dispatched first), and with the query tile as the
// outer loop a key tile reaches a query tile 2·G steps after its predecessor.
// The first contributor stores instead of adding, so the buffer needs no
// clearing; a conversion kernel then writes dQ in the input dtype (0 where no
// key contributed). In accumulate mode every contribution is added straight
// into the caller's fp32 dQ (rows of D contiguous floats) and nothing is
// converted.
//
// Warps: 0 TMA producer, 1 MMA issuer, 2 TMEM allocator, 3 dQ writer,
// 4-11 two elementwise warpgroups taking alternate steps.
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

constexpr int kD = 128;

struct FusedLayout {
  static constexpr int kSub = kD / 64;
  static constexpr int kStages = 4;
  static constexpr uint32_t kKVBytes = kRows * kD * 2;   // K or V tile (128 keys), 32 KB
  static constexpr uint32_t kQBytes = kInner * kD * 2;   // Q or dO tile (64 rows), 16 KB
  static constexpr uint32_t kDSBytes = kRows * kInner * 2;    // dSᵀ [128 keys][64 q], 16 KB
  static constexpr uint32_t kOffK = 0;
  static constexpr uint32_t kOffV = kOffK + kKVBytes;
  static constexpr uint32_t kOffStage = kOffV + kKVBytes;  // Q_s, dO_s per stage
  static constexpr uint32_t kStageBytes = 2 * kQBytes;
  static constexpr uint32_t kOffDS = kOffStage + kStages * kStageBytes;  // 2 buffers
  static constexpr uint32_t kOffRow = kOffDS + 2 * kDSBytes;  // lse2_s[64], delta_s[64] per stage
  static constexpr uint32_t kOffBar = kOffRow + kStages * 512;
  // No alignment slack: the kernel checks that dynamic shared memory starts
  // on a 1024-byte boundary (the 128-byte swizzle needs it) and reports an
  // error otherwise.
  static constexpr uint32_t kSmemBytes = kOffBar + 256;
  // TMEM: Sᵀ(b) at 64·b, dPᵀ(b) / dQᵀ(b) at 128 + 64·b, dV at 256, dK at 384.
  static constexpr uint32_t kTmemS = 0, kTmemDP = 128, kTmemDV = 256, kTmemDK = 384;
  static_assert(kSmemBytes <= 232448, "smem budget");
  static_assert(kOffDS % 1024 == 0, "operand alignment");
  static_assert(2 * kKVBytes >= kRows * kD * 4, "fp32 dK or dV staging in the K/V tiles");
};

// Bounded wait until a query tile's counter reaches `turn` (false: aborted
// or timed out, with the abort flag raised).
__device__ __forceinline__ bool wait_turn(const uint32_t* cnt, uint32_t turn, const WaitCtl& ctl) {
  if (ld_acquire_gpu(cnt) == turn) return true;
  const uint64_t t0 = globaltimer();
  while (ld_acquire_gpu(cnt) != turn) {
    if (*ctl.abort) return false;
    if (globaltimer() - t0 > ctl.timeout_ns) {
      *ctl.abort = 1;
      if (ctl.status) atomicExch(ctl.status, BFA_ERR_DEVICE_TIMEOUT);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// Query tiles [X·64, X·64 + 64) see the key tiles [kt_min, kt_max]; the
// contribution of key tile kt is number kt_max − kt in the fixed order.
__device__ __forceinline__ int last_key_tile(const Params& p, int q0) {
  int klo, khi;
  key_range(p, q0, min(q0 + kInner, p.Sq), &klo, &khi);
  return (khi - 1) / kRows;
}

template <bool BF16, bool CAP, bool ALIBI>
__global__ void __launch_bounds__(kThreads, 1)
    fused_bwd_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                     const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                     const __grid_constant__ CUtensorMap tmDK, const __grid_constant__ CUtensorMap tmDV,
                     float* __restrict__ dq_acc, uint32_t* __restrict__ order, const Params p) {
  using L = FusedLayout;
  constexpr int NS = L::kStages;
  constexpr int D = kD;
  enum {
    kKVFull = 0,
    kQFull = 1,
    kQEmpty = 1 + NS,
    kSPFull = 1 + 2 * NS,  // [2] MMA -> elementwise: Sᵀ, dPᵀ of the step are in TMEM
    kDSFull = kSPFull + 2,  // [2] elementwise -> MMA: Pᵀ in TMEM, dSᵀ in smem (4 warps)
    kDQFull = kDSFull + 2,  // [2] MMA -> elementwise: dQᵀ of the step is in TMEM
    kTmemFree = kDQFull + 2,  // [2] elementwise -> MMA: dQᵀ read out (4 warps)
    kStaged = kTmemFree + 2,  // [NS] per stage: the step's fp32 dQ tile is in it (4 warps)
    kAccDone = kStaged + NS,
    kDrain = kAccDone + 1,
    kNever = kDrain + 1,
    kNumBars = kNever + 1
  };

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023u) {  // uniform: every thread leaves before any work
    if (threadIdx.x == 0 && p.status) atomicExch(p.status, BFA_ERR_CUDA);
    return;
  }
  uint8_t* smem = smem_raw;
  const uint32_t sbase = smem_u32(smem);
  auto bar = [&](int i) -> uint32_t { return sbase + L::kOffBar + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = (uint32_t*)(smem + L::kOffBar + 8 * kNumBars);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  int* warp_ok = (int*)(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_kt = (p.Sk + kRows - 1) / kRows;
  // Descending key tiles within each (batch, kv-head): the predecessors of a
  // tile in the dQ order have smaller block indices.
  const int kt = n_kt - 1 - (int)(blockIdx.x % n_kt);
  const int bh = blockIdx.x / n_kt;
  const int hkv = bh % p.Hkv, b = bh / p.Hkv;
  const int c0 = kt * kRows;
  int qlo, qhi;
  query_range(p, c0, min(c0 + kRows, p.Sk), &qlo, &qhi);
  const int qt0 = qlo / kInner;
  const int n_qt = (qhi > qlo) ? (qhi + kInner - 1) / kInner - qt0 : 0;
  const int n_iter = n_qt * p.G;
  const int n_xt = p.Sq_pad / kInner;  // query tiles per head (order counters)

  WaitCtl ctl{abort_flag, p.status, p.timeout_ns};

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i) {
      const bool four = (i >= kDSFull && i < kDSFull + 2) ||
                        (i >= kTmemFree && i < kTmemFree + 2) || (i >= kStaged && i < kStaged + NS);
      mbar_init(bar(i), four ? 4u : 1u);
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      if (n_iter > 0) {
        mbar_arrive_expect_tx(bar(kKVFull), 2 * L::kKVBytes);
        for (int s = 0; s < L::kSub; ++s) {
          tma_load_4d(sbase + L::kOffK + s * (kRows * 128), &tmK, bar(kKVFull), s * 64, c0, hkv, b);
          tma_load_4d(sbase + L::kOffV + s * (kRows * 128), &tmV, bar(kKVFull), s * 64, c0, hkv, b);
        }
      }
      int issued = 0;
      for (int i = 0; i < n_iter; ++i) {
        const int st = i % NS;
        if (i >= NS && !mbar_wait(bar(kQEmpty + st), ((i / NS) & 1) ^ 1, ctl, BFA_ERR_DEVICE_TIMEOUT))
          break;
        const int hq = hkv * p.G + i % p.G;
        const int q0 = (qt0 + i / p.G) * kInner;
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
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // Order per step i: dV(i), dK(i), dQᵀ(i), then Sᵀ/dPᵀ(i+2) into the same
    // TMEM buffer once dQᵀ(i) has been read out. Pᵀ(i) in the Sᵀ buffer and
    // dSᵀ(i) in smem are read by MMAs issued before Sᵀ(i+2) and before the
    // elementwise warps of step i+2 are released (one thread's MMAs run in
    // order).
    if (lane == 0) {
      constexpr uint32_t idSP = idesc_f16(kRows, kInner, BF16, false);
      constexpr uint32_t idAcc = idesc_f16(kRows, D, BF16, true);
      constexpr uint32_t idDQ = idesc_f16(D, kInner, BF16, true, true);
      auto stage = [&](int i) -> uint32_t { return sbase + L::kOffStage + (i % NS) * L::kStageBytes; };
      const uint64_t dK0 = desc_kmajor(sbase + L::kOffK), dV0 = desc_kmajor(sbase + L::kOffV);
      const uint64_t dKt = desc_mnmajor(sbase + L::kOffK, kRows * 128);  // Kᵀ: M = D
      auto issue_sp = [&](int i) {
        const int bf = i & 1;
        const uint64_t dq = desc_kmajor(stage(i)), ddo = desc_kmajor(stage(i) + L::kQBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t offkv = ((kk >> 2) * (kRows * 128) + (kk & 3) * 32) >> 4;
          const uint32_t offq = ((kk >> 2) * (kInner * 128) + (kk & 3) * 32) >> 4;
          mma_ss(tmem + L::kTmemS + 64 * bf, dK0 + offkv, dq + offq, idSP, kk > 0 ? 1u : 0u);
          mma_ss(tmem + L::kTmemDP + 64 * bf, dV0 + offkv, ddo + offq, idSP, kk > 0 ? 1u : 0u);
        }
        mma_commit(bar(kSPFull + bf));
      };
      bool ok = n_iter == 0 || mbar_wait(bar(kKVFull), 0, ctl, BFA_ERR_DEVICE_TIMEOUT);
      for (int i = 0; i < 2 && i < n_iter && ok; ++i) {
        ok = mbar_wait(bar(kQFull + i), 0, ctl, BFA_ERR_DEVICE_TIMEOUT);
        if (ok) {
          tc_fence_after();
          issue_sp(i);
        }
      }
      for (int i = 0; i < n_iter && ok; ++i) {
        const int bf = i & 1, k = i >> 1;
        if (!(ok = mbar_wait(bar(kDSFull + bf), k & 1, ctl, BFA_ERR_DEVICE_TIMEOUT))) break;
        tc_fence_after();
        const uint32_t ds = sbase + L::kOffDS + bf * L::kDSBytes;
        const uint64_t dsB = desc_mnmajor(ds, 8192);  // dSᵀ as B (N = 64 queries)
        const uint64_t dsA = desc_kmajor(ds);         // dSᵀ as A (K = 64 queries)
        const uint64_t mq = desc_mnmajor(stage(i), kInner * 128);
        const uint64_t mdo = desc_mnmajor(stage(i) + L::kQBytes, kInner * 128);
#pragma unroll
        for (int kk = 0; kk < kInner / 16; ++kk) {
          const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
          mma_ts(tmem + L::kTmemDV, tmem + L::kTmemS + 64 * bf + kk * 8, mdo + ((kk * 2048) >> 4),
                 idAcc, acc);
          mma_ss(tmem + L::kTmemDK, dsA + ((kk * 32) >> 4), mq + ((kk * 2048) >> 4), idAcc, acc);
        }
#pragma unroll
        for (int kk = 0; kk < kRows / 16; ++kk)
          mma_ss(tmem + L::kTmemDP + 64 * bf, dKt + ((kk * 2048) >> 4), dsB + ((kk * 2048) >> 4),
                 idDQ, kk > 0 ? 1u : 0u);
        // Completes when every MMA of the step is done: dQᵀ is in TMEM and the
        // step's Q/dO stage and dSᵀ buffer are no longer read.
        mma_commit(bar(kDQFull + bf));
        if (i + 2 < n_iter) {
          const int n2 = i + 2;
          if (!(ok = mbar_wait(bar(kQFull + n2 % NS), (n2 / NS) & 1, ctl, BFA_ERR_DEVICE_TIMEOUT))) break;
          if (!(ok = mbar_wait(bar(kTmemFree + bf), k & 1, ctl, BFA_ERR_DEVICE_TIMEOUT))) break;
          tc_fence_after();
          issue_sp(n2);
        }
      }
      mma_commit(bar(kAccDone));
      mma_commit(bar(kDrain));
      drain_wait(bar(kDrain), 0, p.timeout_ns);
    }
  } else if (warp == 3) {
    // ------------------------------------------------------------ dQ writer
    // Steps in order: take the staged tile, wait for this step's turn, store
    // or add the tile, return the stage to the producer once it was read,
    // and publish the counter of the step two back once its add is complete
    // (up to three adds in flight; each takes about a microsecond).
    if (lane == 0) {
      const bool acc_mode = p.grad_acc != 0;
      uint32_t* pend1 = nullptr;  // counter of step i - 1
      uint32_t* pend2 = nullptr;  // counter of step i - 2
      auto release = [&](uint32_t* c) {
        fence_proxy_async();
        red_release_gpu_add(c, 1u);
      };
      bool ok = true;
      for (int i = 0; i < n_iter && ok; ++i) {
        const int st = i % NS;
        if (!(ok = mbar_wait(bar(kStaged + st), (i / NS) & 1, ctl, BFA_ERR_DEVICE_TIMEOUT))) break;
        const int hq = hkv * p.G + i % p.G;
        const int xt = qt0 + i / p.G;
        const int q0 = xt * kInner;
        uint32_t* cnt = order + ((int64_t)b * p.Hq + hq) * n_xt + xt;
        const uint32_t turn = (uint32_t)(last_key_tile(p, q0) - kt);
        if (!(ok = wait_turn(cnt, turn, ctl))) break;
        fence_proxy_async();
        float* dst = acc_mode ? (float*)p.dq + (int64_t)b * p.sdq_[0] + (int64_t)hq * p.sdq_[1] +
                                    (int64_t)q0 * p.sdq_[2]
                              : dq_acc + (((int64_t)b * p.Hq + hq) * p.Sq + q0) * D;
        const uint32_t bytes = (uint32_t)min(kInner, p.Sq - q0) * D * 4;
        const uint32_t src = sbase + L::kOffStage + st * L::kStageBytes;
        if (turn == 0 && !acc_mode) bulk_store(dst, src, bytes);
        else bulk_reduce_add_f32(dst, src, bytes);
        tma_store_commit();
        bulk_wait_read<0>();
        mbar_arrive(bar(kQEmpty + st));
        bulk_wait<2>();  // the add of step i - 2 is complete
        if (pend2) release(pend2);
        pend2 = pend1;
        pend1 = cnt;
      }
      bulk_wait<0>();
      if (ok) {
        if (pend2) release(pend2);
        if (pend1) release(pend1);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ elementwise
    const int eg = (warp - 4) >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;  // key row within the tile (and d for dQᵀ)
    const int kj = c0 + row;
    const int64_t gj = (int64_t)kj + p.k_off;
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const float sl2 = p.scale * kLog2e;
    const float cap_in = CAP ? p.scale / p.soft_cap : 0.f;
    const float cap_out = CAP ? p.soft_cap * kLog2e : 0.f;
    bool ok = true;
    for (int i = eg; i < n_iter; i += 2) {
      const int bf = i & 1, k = i >> 1, st = i % NS;
      const int hq = hkv * p.G + i % p.G;
      const int q0 = (qt0 + i / p.G) * kInner;
      uint32_t wbar = bar(kSPFull + bf), wpar = (uint32_t)(k & 1);
      if ((p.debug_flags & BFA_DEBUG_INJECT_STALL) && i == 0) {
        wbar = bar(kNever);
        wpar = 0;
      }
      if (!(ok = warp_wait(wbar, wpar, ctl))) break;
      if (!(ok = warp_wait(bar(kQFull + st), (uint32_t)((i / NS) & 1), ctl))) break;
      tc_fence_after();
      const uint32_t tSb = tmem + lane_base + L::kTmemS + 64 * bf;
      const uint32_t tDb = tmem + lane_base + L::kTmemDP + 64 * bf;
      uint8_t* dsrow = smem + L::kOffDS + bf * L::kDSBytes;
      const float* rowv = (const float*)(smem + L::kOffRow + st * 512);
      const bool full = tile_full(p, q0, q0 + kInner, c0, c0 + kRows);
      const float slope2 = ALIBI ? p.alibi[hq] * kLog2e : 0.f;
      const float abase = ALIBI ? slope2 * (float)((int64_t)q0 + p.q_off - gj) : 0.f;
      int clo, chi;
      queries_for_key(p, gj, kj < p.Sk, q0, kInner, &clo, &chi);
      auto step = [&](auto masked) {
        constexpr bool MASKED = decltype(masked)::value;
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          uint32_t sr[32], dr[32];
          tmem_ld32(tSb + 32 * half, sr);
          tmem_ld32(tDb + 32 * half, dr);
          tmem_ld_wait();
          uint32_t ppk[16], dpk[16];
#pragma unroll
          for (int c = 0; c < 32; c += 4) {
            const float4 l4 = *reinterpret_cast<const float4*>(rowv + 32 * half + c);
            const float4 d4 = *reinterpret_cast<const float4*>(rowv + 64 + 32 * half + c);
            const float lse_c[4] = {l4.x, l4.y, l4.z, l4.w};
            const float dl_c[4] = {d4.x, d4.y, d4.z, d4.w};
            float pr4[4], ds4[4];
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              const int cc = 32 * half + c + h;
              const float raw = __uint_as_float(sr[c + h]);
              float pr, t = 0.f;
              if (CAP || ALIBI) {
                float x = logit2<CAP>(raw, sl2, cap_in, cap_out, &t);
                if (ALIBI) x = fmaf(slope2, (float)cc, x + abase);
                pr = ex2(x - lse_c[h]);
              } else {
                pr = ex2(fmaf(raw, sl2, -lse_c[h]));
              }
              if (MASKED) pr = ((unsigned)(cc - clo) < (unsigned)(chi - clo)) ? pr : 0.f;
              float ds = pr * (__uint_as_float(dr[c + h]) - dl_c[h]) * p.scale;
              if (CAP) ds *= (1.f - t * t);
              pr4[h] = pr;
              ds4[h] = ds;
            }
            ppk[c / 2] = pack2<BF16>(pr4[0], pr4[1]);
            ppk[c / 2 + 1] = pack2<BF16>(pr4[2], pr4[3]);
            dpk[c / 2] = pack2<BF16>(ds4[0], ds4[1]);
            dpk[c / 2 + 1] = pack2<BF16>(ds4[2], ds4[3]);
          }
          // Pᵀ half -> packed TMEM columns [16·half, 16·half + 16) of the Sᵀ
          // buffer (its fp32 columns there were read above).
          tmem_st16(tSb + 16 * half, ppk);
          // dSᵀ half -> 16-byte chunks [4·half, 4·half + 4) of this key's
          // 128-byte row in the swizzled dSᵀ tile.
#pragma unroll
          for (int j = 0; j < 4; ++j)
            *reinterpret_cast<uint4*>(dsrow + sw128_offset(row, 4 * half + j)) =
                make_uint4(dpk[4 * j], dpk[4 * j + 1], dpk[4 * j + 2], dpk[4 * j + 3]);
        }
      };
      if (full) step(std::false_type{});
      else step(std::true_type{});
      tmem_st_wait();
      fence_async_shared();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kDSFull + bf));

      // dQᵀ(i): lane = d, 64 columns = the step's query rows.
      if (!(ok = warp_wait(bar(kDQFull + bf), (uint32_t)(k & 1), ctl))) break;
      tc_fence_after();
      uint32_t q_lo[32], q_hi[32];
      tmem_ld32(tDb, q_lo);
      tmem_ld32(tDb + 32, q_hi);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kTmemFree + bf));
      // fp32 tile [64 rows][D], row-major, into the step's Q/dO stage (free:
      // every MMA of the step is done). For each row a warp writes 32
      // consecutive floats.
      float* tile = (float*)(smem + L::kOffStage + st * L::kStageBytes) + row;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        tile[j * D] = __uint_as_float(q_lo[j]);
        tile[(32 + j) * D] = __uint_as_float(q_hi[j]);
      }
      fence_async_shared();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kStaged + st));
    }
    // Warpgroup 0 writes dK / dV.
    if (eg == 0) {
      bool good = ok;
      if (good && n_iter > 0) good = warp_wait(bar(kAccDone), 0, ctl);
      good = good && !*abort_flag;
      const bool acc = p.grad_acc != 0;
      uint8_t* stage_k = smem + L::kOffK;  // free once every MMA is done
      if (lane == 0) warp_ok[wq] = good ? 1 : 0;
      named_sync(1, 128);
      const bool all_ok = warp_ok[0] && warp_ok[1] && warp_ok[2] && warp_ok[3];
      if (!acc) {
        if (all_ok) {
          tc_fence_after();
          stage_tmem_row<D, BF16>(tmem + lane_base + L::kTmemDV, smem + L::kOffV, row, n_iter == 0);
          stage_tmem_row<D, BF16>(tmem + lane_base + L::kTmemDK, stage_k, row, n_iter == 0);
          fence_async_shared();
        }
        named_sync(1, 128);
        if (wq == 0 && lane == 0 && all_ok) {
          for (int s = 0; s < L::kSub; ++s) {
            tma_store_4d(&tmDV, sbase + L::kOffV + s * (kRows * 128), s * 64, c0, hkv, b);
            tma_store_4d(&tmDK, sbase + L::kOffK + s * (kRows * 128), s * 64, c0, hkv, b);
          }
          tma_store_commit();
          tma_store_wait_all();
        }
      } else if (all_ok && n_iter > 0) {
        // fp32 dV, then dK, through the 64 KB of the K/V tiles.
        for (int t = 0; t < 2; ++t) {
          tc_fence_after();
          stage_tmem_row_f32<D>(tmem + lane_base + (t == 0 ? L::kTmemDV : L::kTmemDK), stage_k, row);
          fence_async_shared();
          named_sync(1, 128);
          if (wq == 0 && lane == 0) {
            for (int s = 0; s < D / 32; ++s)
              tma_reduce_add_4d(t == 0 ? &tmDV : &tmDK, sbase + L::kOffK + s * (kRows * 128), s * 32,
                                c0, hkv, b);
            tma_store_commit();
            tma_store_wait_all();
          }
          named_sync(1, 128);
        }
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

// dQ (input dtype) from the fp32 buffer; query tiles no key tile reached
// (counter still 0) are written as zeros.
template <typename T>
__global__ void __launch_bounds__(256) dq_convert_kernel(const float* __restrict__ acc,
                                                         const uint32_t* __restrict__ order,
                                                         Params p) {
  const int64_t n8 = (int64_t)p.B * p.Hq * p.Sq * (p.D / 8);
  const int n_xt = p.Sq_pad / kInner;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n8;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int d0 = (int)(t % (p.D / 8)) * 8;
    const int64_t r = t / (p.D / 8);  // (b·Hq + hq)·Sq + i
    const int i = (int)(r % p.Sq);
    const int64_t bh = r / p.Sq;
    const int hq = (int)(bh % p.Hq), b = (int)(bh / p.Hq);
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (order[bh * n_xt + i / kInner] != 0u) {
      const float4 a = *reinterpret_cast<const float4*>(acc + r * p.D + d0);
      const float4 c = *reinterpret_cast<const float4*>(acc + r * p.D + d0 + 4);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
    }
    T* out = (T*)p.dq + (int64_t)b * p.sdq_[0] + (int64_t)hq * p.sdq_[1] + (int64_t)i * p.sdq_[2] +
             (int64_t)d0 * p.sdq_[3];
    if (p.sdq_[3] == 1 && ((uintptr_t)out & 15u) == 0) {
      uint4 w;
      w.x = pack2<std::is_same<T, __nv_bfloat16>::value>(v[0], v[1]);
      w.y = pack2<std::is_same<T, __nv_bfloat16>::value>(v[2], v[3]);
      w.z = pack2<std::is_same<T, __nv_bfloat16>::value>(v[4], v[5]);
      w.w = pack2<std::is_same<T, __nv_bfloat16>::value>(v[6], v[7]);
      *reinterpret_cast<uint4*>(out) = w;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) out[(int64_t)e * p.sdq_[3]] = from_f32<T>(v[e]);
    }
  }
}

template <typename K>
bool set_smem(K kern, uint32_t bytes) {
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) ==
         cudaSuccess;
}

template <bool BF16, bool CAP, bool ALIBI>
int launch_fused(const Params& p, int dtype, uint32_t* order, float* dq_acc, cudaStream_t st) {
  using L = FusedLayout;
  auto kern = fused_bwd_kernel<BF16, CAP, ALIBI>;
  static std::once_flag once;
  static bool attr_ok = false;
  std::call_once(once, [&] { attr_ok = set_smem(kern, L::kSmemBytes); });
  if (!attr_ok) return BFA_ERR_CUDA;
  const int gdt = p.grad_acc ? BFA_DTYPE_F32 : dtype;
  const int n_xt = p.Sq_pad / kInner;
  if (cudaMemsetAsync(order, 0, (size_t)p.B * p.Hq * n_xt * sizeof(uint32_t), st) != cudaSuccess)
    return BFA_ERR_CUDA;
  CUtensorMap m[6];
  if (!make_tmap_bhsd(&m[0], p.k, dtype, kD, p.Sk, p.Hkv, p.B, p.sk_, kRows) ||
      !make_tmap_bhsd(&m[1], p.v, dtype, kD, p.Sk, p.Hkv, p.B, p.sv_, kRows) ||
      !make_tmap_bhsd(&m[2], p.q, dtype, kD, p.Sq, p.Hq, p.B, p.sq_, kInner) ||
      !make_tmap_bhsd(&m[3], p.dout, dtype, kD, p.Sq, p.Hq, p.B, p.sdo_, kInner) ||
      !make_tmap_bhsd(&m[4], p.dk, gdt, kD, p.Sk, p.Hkv, p.B, p.sdk_, kRows) ||
      !make_tmap_bhsd(&m[5], p.dv, gdt, kD, p.Sk, p.Hkv, p.B, p.sdv_, kRows))
    return BFA_ERR_CUDA;
  const unsigned grid = (unsigned)((p.Sk + kRows - 1) / kRows) * p.Hkv * p.B;
  kern<<<grid, kThreads, L::kSmemBytes, st>>>(m[0], m[1], m[2], m[3], m[4], m[5], dq_acc, order, p);
  note_launch();
  if (cudaGetLastError() != cudaSuccess) return BFA_ERR_CUDA;
  if (!p.grad_acc) {
    const int64_t n8 = (int64_t)p.B * p.Hq * p.Sq * (kD / 8);
    const unsigned blocks = (unsigned)std::min<int64_t>((n8 + 255) / 256, 148 * 16);
    if (BF16) dq_convert_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(dq_acc, order, p);
    else dq_convert_kernel<__half><<<blocks, 256, 0, st>>>(dq_acc, order, p);
    note_launch();
    if (cudaGetLastError() != cudaSuccess) return BFA_ERR_CUDA;
  }
  return BFA_OK;
}

template <bool BF16>
int dispatch_fused(const Params& p, int dtype, uint32_t* order, float* dq_acc, cudaStream_t st) {
  const bool cap = p.soft_cap > 0.f, alibi = p.alibi != nullptr;
  if (cap && alibi) return launch_fused<BF16, true, true>(p, dtype, order, dq_acc, st);
  if (cap) return launch_fused<BF16, true, false>(p, dtype, order, dq_acc, st);
  if (alibi) return launch_fused<BF16, false, true>(p, dtype, order, dq_acc, st);
  return launch_fused<BF16, false, false>(p, dtype, order, dq_acc, st);
}

}  // namespace

bool sm100_bwd_fused_eligible(const Params& p, int dtype) {
  if (p.D != kD || !sm100_bwd_eligible(p, dtype)) return false;
  if (!p.grad_acc) return true;
  // Accumulate mode adds 64-row tiles straight into the caller's fp32 dQ
  // with 1-D bulk copies: rows of D contiguous floats, 16-byte aligned.
  return p.sdq_[3] == 1 && p.sdq_[2] == kD && ((uintptr_t)p.dq & 15u) == 0 &&
         (p.sdq_[1] & 3) == 0 && (p.sdq_[0] & 3) == 0;
}

int sm100_bwd_fused(const Params& p, int dtype, uint32_t* order, float* dq_acc, cudaStream_t st) {
  return dtype == BFA_DTYPE_BF16 ? dispatch_fused<true>(p, dtype, order, dq_acc, st)
                                 : dispatch_fused<false>(p, dtype, order, dq_acc, st);
}

}  // namespace bfa
