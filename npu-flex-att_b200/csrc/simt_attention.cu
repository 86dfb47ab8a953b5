// simt_attention.cu -- generic CUDA-core attention kernels (any dtype, any
// strides, head_dim <= 256).
//
// These are the library's fp32 path (the tcgen05 path computes in bf16/fp16
// operands and cannot meet the fp32 tolerance) and its path for layouts the
// TMA path does not take (odd head dims, unaligned strides). Every value is
// carried in fp32. Structure mirrors the reference kernels one-to-one:
//   simt_fwd_kernel    <- flash_attn_fwd_kernel      npu_flash_attention.py:17-166
//   simt_bwd_dq_kernel <- flash_attn_bwd_dq_kernel   npu_flash_attention.py:298-402
//   simt_bwd_dkdv_kernel <- flash_attn_bwd_dkdv_kernel npu_flash_attention.py:407-560,
//       except that one CTA owns a (b, kv-head, kv-tile) and loops over the
//       GQA group, so dK/dV come out already summed (the reference sums per-q-head
//       copies on the host at :735-737) and the sum is deterministic.
//
// Tiles are 32 query rows x 32 key rows, 128 threads: thread t owns tile row
// t/4 and, within it, every 4th key column and every 4th float4 of the head
// dim (starting at float4 t%4).
#include <algorithm>
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include "bfa_common.cuh"
#include "bfa_internal.h"

namespace bfa {
namespace {

constexpr int TM = 32;
constexpr int TN = 32;
constexpr int NT = 128;

template <typename T>
__device__ __forceinline__ const T* head_ptr(const void* base, const int64_t* st, int b, int h) {
  return (const T*)base + (int64_t)b * st[0] + (int64_t)h * st[1];
}

// Stage rows [row0, row0 + nvalid) x [0, D) of a strided [S, D] slice into
// shared memory as fp32 with row pitch DP+4; missing rows/cols become 0.
template <typename T, int DP>
__device__ __forceinline__ void stage_rows(float* dst, const T* src, int64_t srow, int64_t scol,
                                           int row0, int nvalid, int D, int nrows) {
  for (int idx = threadIdx.x; idx < nrows * DP; idx += NT) {
    const int r = idx / DP, c = idx - r * DP;
    float val = 0.f;
    if (r < nvalid && c < D) val = to_f32<T>(src[(int64_t)(row0 + r) * srow + (int64_t)c * scol]);
    dst[r * (DP + 4) + c] = val;
  }
}

// Rows of the staged tiles have pitch DP + 4 floats: 16-byte aligned, so dot
// products and accumulations read them with 16-byte shared loads, and rows
// r, r+1, ... start 4 banks apart, so the 8 rows a warp reads at once fill
// the 32 banks without conflicts.
// The 8 dot products of row `a` with rows b0 + 4u·pitch, u = 0..7 (a thread's
// 8 columns of a 32-wide tile): each float4 of `a` is read once for all 8.
template <int DP>
__device__ __forceinline__ void dots8(const float* a, const float* b0, float (&out)[8]) {
  const float4* a4 = reinterpret_cast<const float4*>(a);
#pragma unroll
  for (int u = 0; u < 8; ++u) out[u] = 0.f;
#pragma unroll 4
  for (int d = 0; d < DP / 4; ++d) {
    const float4 x = a4[d];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float4 y = reinterpret_cast<const float4*>(b0 + 4 * u * (DP + 4))[d];
      out[u] = fmaf(x.x, y.x, out[u]);
      out[u] = fmaf(x.y, y.y, out[u]);
      out[u] = fmaf(x.z, y.z, out[u]);
      out[u] = fmaf(x.w, y.w, out[u]);
    }
  }
}

// Column of accumulator e of the thread with column group c: the thread
// owns every 4th float4 of a row, starting at float4 c (the four threads of a
// row read four consecutive float4s: no bank conflicts).
__device__ __forceinline__ int acc_col(int e, int c) { return 16 * (e >> 2) + 4 * c + (e & 3); }

template <int DP>
__device__ __forceinline__ float dot_rows(const float* a, const float* b) {
  const float4* a4 = reinterpret_cast<const float4*>(a);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  float acc0 = 0.f, acc1 = 0.f;
#pragma unroll 8
  for (int d = 0; d < DP / 4; ++d) {
    const float4 x = a4[d], y = b4[d];
    acc0 = fmaf(x.x, y.x, acc0);
    acc1 = fmaf(x.y, y.y, acc1);
    acc0 = fmaf(x.z, y.z, acc0);
    acc1 = fmaf(x.w, y.w, acc1);
  }
  return acc0 + acc1;
}

template <typename T, int DP>
__global__ void __launch_bounds__(NT) simt_fwd_kernel(Params p) {
  extern __shared__ float smem[];
  float* sQ = smem;
  float* sK = sQ + TM * (DP + 4);
  float* sV = sK + TN * (DP + 4);
  float* sP = sV + TN * (DP + 4);  // [TM][TN+1]

  const int r0 = blockIdx.x * TM, hq = blockIdx.y, b = blockIdx.z;
  const int hkv = hq / p.G;
  const int rows = min(TM, p.Sq - r0);
  const T* Q = head_ptr<T>(p.q, p.sq_, b, hq);
  const T* K = head_ptr<T>(p.k, p.sk_, b, hkv);
  const T* V = head_ptr<T>(p.v, p.sv_, b, hkv);
  stage_rows<T, DP>(sQ, Q, p.sq_[2], p.sq_[3], r0, rows, p.D, TM);

  const int tid = threadIdx.x, r = tid >> 2, c = tid & 3;
  const int64_t gi = (int64_t)r0 + r + p.q_off;
  const float slope = p.alibi ? p.alibi[hq] : 0.f;
  float m = neg_inf(), l = 0.f;
  float acc[DP / 4];
#pragma unroll
  for (int e = 0; e < DP / 4; ++e) acc[e] = 0.f;

  int lo, hi;
  key_range(p, r0, r0 + rows, &lo, &hi);
  // Key tiles every row of the block keeps (inside Sk; no documents or
  // block mask) skip the per-element mask.
  const KeptRange kept = kept_keys(p, r0, rows, TN, false);
  const bool may_skip = p.doc_lo == nullptr && p.blk == nullptr;
  for (int k0 = (lo / TN) * TN; k0 < hi; k0 += TN) {
    const int kn = min(TN, p.Sk - k0);
    const bool full = may_skip && kept.has(k0);
    __syncthreads();
    stage_rows<T, DP>(sK, K, p.sk_[2], p.sk_[3], k0, kn, p.D, TN);
    stage_rows<T, DP>(sV, V, p.sv_[2], p.sv_[3], k0, kn, p.D, TN);
    __syncthreads();
    float s[TN / 4];
    float mx = neg_inf();
    float dot8[8];
    dots8<DP>(sQ + r * (DP + 4), sK + c * (DP + 4), dot8);
#pragma unroll
    for (int u = 0; u < TN / 4; ++u) {
      const int jj = c + 4 * u;
      const int64_t gj = (int64_t)k0 + jj + p.k_off;
      const float dot = dot8[u];
      const float val = transform_logit(dot, p.scale, p.soft_cap, slope, gi, gj, nullptr);
      const bool ok = (r < rows) && (full || ((jj < kn) && keep_elem(p, b, hq, gi, gj)));
      s[u] = ok ? val : neg_inf();
      mx = fmaxf(mx, s[u]);
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m, mx);
    const float alpha = (m_new == neg_inf()) ? 1.f : expf(m - m_new);
    float rs = 0.f;
#pragma unroll
    for (int u = 0; u < TN / 4; ++u) {
      const float pv = (s[u] == neg_inf()) ? 0.f : expf(s[u] - m_new);
      sP[r * (TN + 1) + c + 4 * u] = pv;
      rs += pv;
    }
    rs += __shfl_xor_sync(0xffffffffu, rs, 1);
    rs += __shfl_xor_sync(0xffffffffu, rs, 2);
    l = l * alpha + rs;
    m = m_new;
    __syncwarp();
#pragma unroll
    for (int e = 0; e < DP / 4; ++e) acc[e] *= alpha;
    for (int jj = 0; jj < TN; ++jj) {
      const float pv = sP[r * (TN + 1) + jj];
      const float4* vrow = reinterpret_cast<const float4*>(sV + jj * (DP + 4)) + c;
#pragma unroll
      for (int g = 0; g < DP / 16; ++g) {
        const float4 v4 = vrow[4 * g];
        acc[4 * g] = fmaf(pv, v4.x, acc[4 * g]);
        acc[4 * g + 1] = fmaf(pv, v4.y, acc[4 * g + 1]);
        acc[4 * g + 2] = fmaf(pv, v4.z, acc[4 * g + 2]);
        acc[4 * g + 3] = fmaf(pv, v4.w, acc[4 * g + 3]);
      }
    }
  }

  if (p.out_acc) {
    // Merge into the running fp32 output and LSE (bfa_fwd_args.accumulate).
    float* lse_p = p.lse + ((int64_t)b * p.Hq + hq) * p.Sq + r0 + r;
    const MergeWeights w = merge_weights((r < rows) ? *lse_p : neg_inf(), (l > 0.f) ? m + logf(l) : neg_inf());
    __syncwarp();  // the row's four threads have read the running LSE
    if (r < rows) {
      const float sp = (l > 0.f) ? w.wp / l : 0.f;
      float* O = (float*)p.o + (int64_t)b * p.so_[0] + (int64_t)hq * p.so_[1] + (int64_t)(r0 + r) * p.so_[2];
#pragma unroll
      for (int e = 0; e < DP / 4; ++e) {
        const int d = acc_col(e, c);
        if (d < p.D) {
          float* dst = O + (int64_t)d * p.so_[3];
          *dst = fmaf(acc[e], sp, w.wa != 0.f ? *dst * w.wa : 0.f);
        }
      }
      if (c == 0) *lse_p = w.ln;
    }
    return;
  }
  if (r < rows) {
    const float inv = (l > 0.f) ? 1.f / l : 0.f;
    T* O = (T*)p.o + (int64_t)b * p.so_[0] + (int64_t)hq * p.so_[1] + (int64_t)(r0 + r) * p.so_[2];
#pragma unroll
    for (int e = 0; e < DP / 4; ++e) {
      const int d = acc_col(e, c);
      if (d < p.D) O[(int64_t)d * p.so_[3]] = from_f32<T>(acc[e] * inv);
    }
    if (c == 0) {
      p.lse[((int64_t)b * p.Hq + hq) * p.Sq + r0 + r] = (l > 0.f) ? m + logf(l) : neg_inf();
    }
  }
}

template <typename T, int DP>
__global__ void __launch_bounds__(NT) simt_bwd_dq_kernel(Params p) {
  extern __shared__ float smem[];
  float* sQ = smem;
  float* sDO = sQ + TM * (DP + 4);
  float* sK = sDO + TM * (DP + 4);
  float* sV = sK + TN * (DP + 4);
  float* sDS = sV + TN * (DP + 4);  // [TM][TN+1]

  const int r0 = blockIdx.x * TM, hq = blockIdx.y, b = blockIdx.z;
  const int hkv = hq / p.G;
  const int rows = min(TM, p.Sq - r0);
  stage_rows<T, DP>(sQ, head_ptr<T>(p.q, p.sq_, b, hq), p.sq_[2], p.sq_[3], r0, rows, p.D, TM);
  stage_rows<T, DP>(sDO, head_ptr<T>(p.dout, p.sdo_, b, hq), p.sdo_[2], p.sdo_[3], r0, rows, p.D, TM);
  const T* K = head_ptr<T>(p.k, p.sk_, b, hkv);
  const T* V = head_ptr<T>(p.v, p.sv_, b, hkv);

  const int tid = threadIdx.x, r = tid >> 2, c = tid & 3;
  const int64_t gi = (int64_t)r0 + r + p.q_off;
  const float slope = p.alibi ? p.alibi[hq] : 0.f;
  const int64_t row_idx = ((int64_t)b * p.Hq + hq) * p.Sq + r0 + r;
  const float lse = (r < rows) ? p.lse[row_idx] : 0.f;
  const float dlt = (r < rows) ? p.delta[((int64_t)b * p.Hq + hq) * p.Sq_pad + r0 + r] : 0.f;
  const bool row_live = (r < rows) && (lse != neg_inf());
  float acc[DP / 4];
#pragma unroll
  for (int e = 0; e < DP / 4; ++e) acc[e] = 0.f;

  int lo, hi;
  key_range(p, r0, r0 + rows, &lo, &hi);
  // Key tiles every row of the block keeps (inside Sk; no documents or
  // block mask) skip the per-element mask.
  const KeptRange kept = kept_keys(p, r0, rows, TN, false);
  const bool may_skip = p.doc_lo == nullptr && p.blk == nullptr;
  for (int k0 = (lo / TN) * TN; k0 < hi; k0 += TN) {
    const int kn = min(TN, p.Sk - k0);
    const bool full = may_skip && kept.has(k0);
    __syncthreads();
    stage_rows<T, DP>(sK, K, p.sk_[2], p.sk_[3], k0, kn, p.D, TN);
    stage_rows<T, DP>(sV, V, p.sv_[2], p.sv_[3], k0, kn, p.D, TN);
    __syncthreads();
    float sdot[8], pdot[8];
    dots8<DP>(sQ + r * (DP + 4), sK + c * (DP + 4), sdot);
    dots8<DP>(sDO + r * (DP + 4), sV + c * (DP + 4), pdot);
#pragma unroll
    for (int u = 0; u < TN / 4; ++u) {
      const int jj = c + 4 * u;
      const int64_t gj = (int64_t)k0 + jj + p.k_off;
      float ds = 0.f;
      if (row_live && (full || (jj < kn && keep_elem(p, b, hq, gi, gj)))) {
        float t;
        const float dot = sdot[u];
        const float val = transform_logit(dot, p.scale, p.soft_cap, slope, gi, gj, &t);
        const float pr = expf(val - lse);
        const float dp = pdot[u];
        ds = pr * (dp - dlt);
        if (p.soft_cap > 0.f) ds *= (1.f - t * t);
        ds *= p.scale;
      }
      sDS[r * (TN + 1) + jj] = ds;
    }
    __syncwarp();
    for (int jj = 0; jj < TN; ++jj) {
      const float dsv = sDS[r * (TN + 1) + jj];
      const float4* krow = reinterpret_cast<const float4*>(sK + jj * (DP + 4)) + c;
#pragma unroll
      for (int g = 0; g < DP / 16; ++g) {
        const float4 k4 = krow[4 * g];
        acc[4 * g] = fmaf(dsv, k4.x, acc[4 * g]);
        acc[4 * g + 1] = fmaf(dsv, k4.y, acc[4 * g + 1]);
        acc[4 * g + 2] = fmaf(dsv, k4.z, acc[4 * g + 2]);
        acc[4 * g + 3] = fmaf(dsv, k4.w, acc[4 * g + 3]);
      }
    }
  }
  if (r < rows) {
    const int64_t base = (int64_t)b * p.sdq_[0] + (int64_t)hq * p.sdq_[1] + (int64_t)(r0 + r) * p.sdq_[2];
#pragma unroll
    for (int e = 0; e < DP / 4; ++e) {
      const int d = acc_col(e, c);
      if (d >= p.D) continue;
      const int64_t at = base + (int64_t)d * p.sdq_[3];
      if (p.grad_acc) ((float*)p.dq)[at] += acc[e];
      else ((T*)p.dq)[at] = from_f32<T>(acc[e]);
    }
  }
}

// One cluster of `nsplit` CTAs per (b, kv-head, kv tile): CTA `split` takes
// every nsplit-th (q-head, query tile) work item, and the cluster's partial
// dK / dV are added in rank order through distributed shared memory, so the
// result does not depend on timing (deterministic) while nsplit times more
// CTAs share the work.
template <typename T, int DP>
__global__ void __launch_bounds__(NT) simt_bwd_dkdv_kernel(Params p) {
  namespace cg = cooperative_groups;
  extern __shared__ float smem[];
  float* sK = smem;
  float* sV = sK + TN * (DP + 4);
  float* sQ = sV + TN * (DP + 4);
  float* sDO = sQ + TM * (DP + 4);
  float* sP = sDO + TM * (DP + 4);   // [TN][TM+1]
  float* sDS = sP + TN * (TM + 1);   // [TN][TM+1]
  float* sL = sDS + TN * (TM + 1);   // [TM]
  float* sDl = sL + TM;              // [TM]

  cg::cluster_group cluster = cg::this_cluster();
  const int nsplit = (int)cluster.dim_blocks().x, split = (int)cluster.block_rank();
  const int c0 = (blockIdx.x / nsplit) * TN, hkv = blockIdx.y, b = blockIdx.z;
  const int cols = min(TN, p.Sk - c0);
  stage_rows<T, DP>(sK, head_ptr<T>(p.k, p.sk_, b, hkv), p.sk_[2], p.sk_[3], c0, cols, p.D, TN);
  stage_rows<T, DP>(sV, head_ptr<T>(p.v, p.sv_, b, hkv), p.sv_[2], p.sv_[3], c0, cols, p.D, TN);

  const int tid = threadIdx.x, r = tid >> 2, c = tid & 3;  // r: kv row in tile
  const int64_t gj = (int64_t)c0 + r + p.k_off;
  float adk[DP / 4], adv[DP / 4];
#pragma unroll
  for (int e = 0; e < DP / 4; ++e) { adk[e] = 0.f; adv[e] = 0.f; }

  int qlo, qhi;
  query_range(p, c0, c0 + cols, &qlo, &qhi);
  // Head dims <= 64: query tiles that keep every key of this tile (inside Sq
  // and Sk; no documents or block mask) skip the per-element mask. (At 128
  // the extra state cost more than it saved.)
  const KeptRange kq = kept_queries(p, c0, TN, TM);
  const bool may_skip = DP <= 64 && p.doc_lo == nullptr && p.blk == nullptr;
  int work = 0;  // work item index over (q-head, query tile)
  for (int g = 0; g < p.G; ++g) {
    const int hq = hkv * p.G + g;
    const float slope = p.alibi ? p.alibi[hq] : 0.f;
    const T* Q = head_ptr<T>(p.q, p.sq_, b, hq);
    const T* DO = head_ptr<T>(p.dout, p.sdo_, b, hq);
    for (int q0 = (qlo / TM) * TM; q0 < qhi; q0 += TM) {
      if ((work++ % nsplit) != split) continue;  // another CTA of the cluster's
      const int qn = min(TM, p.Sq - q0);
      const bool full = may_skip && kq.has(q0);
      __syncthreads();
      stage_rows<T, DP>(sQ, Q, p.sq_[2], p.sq_[3], q0, qn, p.D, TM);
      stage_rows<T, DP>(sDO, DO, p.sdo_[2], p.sdo_[3], q0, qn, p.D, TM);
      if (tid < TM) {
        const int64_t row_idx = ((int64_t)b * p.Hq + hq) * p.Sq + q0 + tid;
        sL[tid] = (tid < qn) ? p.lse[row_idx] : neg_inf();
        sDl[tid] = (tid < qn) ? p.delta[((int64_t)b * p.Hq + hq) * p.Sq_pad + q0 + tid] : 0.f;
      }
      __syncthreads();
      float sdot[8], pdot[8];
      dots8<DP>(sK + r * (DP + 4), sQ + c * (DP + 4), sdot);
      dots8<DP>(sV + r * (DP + 4), sDO + c * (DP + 4), pdot);
#pragma unroll
      for (int u = 0; u < TM / 4; ++u) {
        const int ii = c + 4 * u;
        const int64_t gi = (int64_t)q0 + ii + p.q_off;
        float pr = 0.f, ds = 0.f;
        const float lse = sL[ii];
        if (lse != neg_inf() && (full || (r < cols && ii < qn && keep_elem(p, b, hq, gi, gj)))) {
          float t;
          const float dot = sdot[u];
          const float val = transform_logit(dot, p.scale, p.soft_cap, slope, gi, gj, &t);
          pr = expf(val - lse);
          const float dp = pdot[u];
          ds = pr * (dp - sDl[ii]);
          if (p.soft_cap > 0.f) ds *= (1.f - t * t);
          ds *= p.scale;
        }
        sP[r * (TM + 1) + ii] = pr;
        sDS[r * (TM + 1) + ii] = ds;
      }
      __syncwarp();
      for (int ii = 0; ii < TM; ++ii) {
        const float pv = sP[r * (TM + 1) + ii];
        const float dsv = sDS[r * (TM + 1) + ii];
        const float4* dorow = reinterpret_cast<const float4*>(sDO + ii * (DP + 4)) + c;
        const float4* qrow = reinterpret_cast<const float4*>(sQ + ii * (DP + 4)) + c;
#pragma unroll
        for (int g = 0; g < DP / 16; ++g) {
          const float4 o4 = dorow[4 * g], q4 = qrow[4 * g];
          adv[4 * g] = fmaf(pv, o4.x, adv[4 * g]);
          adv[4 * g + 1] = fmaf(pv, o4.y, adv[4 * g + 1]);
          adv[4 * g + 2] = fmaf(pv, o4.z, adv[4 * g + 2]);
          adv[4 * g + 3] = fmaf(pv, o4.w, adv[4 * g + 3]);
          adk[4 * g] = fmaf(dsv, q4.x, adk[4 * g]);
          adk[4 * g + 1] = fmaf(dsv, q4.y, adk[4 * g + 1]);
          adk[4 * g + 2] = fmaf(dsv, q4.z, adk[4 * g + 2]);
          adk[4 * g + 3] = fmaf(dsv, q4.w, adk[4 * g + 3]);
        }
      }
    }
  }
  if (nsplit > 1) {
    // Partials into this CTA's Q / dO tiles, then rank 0 adds the others'
    // in rank order and writes the result.
    float* pk = sQ;
    float* pv = sDO;
    __syncthreads();
#pragma unroll
    for (int e = 0; e < DP / 4; ++e) {
      pk[r * (DP + 4) + acc_col(e, c)] = adk[e];
      pv[r * (DP + 4) + acc_col(e, c)] = adv[e];
    }
    cluster.sync();
    if (split == 0) {
      for (int rk = 1; rk < nsplit; ++rk) {
        const float* rpk = cluster.map_shared_rank(pk, rk);
        const float* rpv = cluster.map_shared_rank(pv, rk);
#pragma unroll
        for (int e = 0; e < DP / 4; ++e) {
          adk[e] += rpk[r * (DP + 4) + acc_col(e, c)];
          adv[e] += rpv[r * (DP + 4) + acc_col(e, c)];
        }
      }
    }
    cluster.sync();  // the other ranks' shared memory stays alive until read
    if (split != 0) return;
  }
  if (r < cols) {
    const int64_t bk = (int64_t)b * p.sdk_[0] + (int64_t)hkv * p.sdk_[1] + (int64_t)(c0 + r) * p.sdk_[2];
    const int64_t bv = (int64_t)b * p.sdv_[0] + (int64_t)hkv * p.sdv_[1] + (int64_t)(c0 + r) * p.sdv_[2];
#pragma unroll
    for (int e = 0; e < DP / 4; ++e) {
      const int d = acc_col(e, c);
      if (d >= p.D) continue;
      const int64_t ak = bk + (int64_t)d * p.sdk_[3], av = bv + (int64_t)d * p.sdv_[3];
      if (p.grad_acc) {
        ((float*)p.dk)[ak] += adk[e];
        ((float*)p.dv)[av] += adv[e];
      } else {
        ((T*)p.dk)[ak] = from_f32<T>(adk[e]);
        ((T*)p.dv)[av] = from_f32<T>(adv[e]);
      }
    }
  }
}

// Δ = rowsum(O∘dO): one warp per (b, hq, i) row of pitch Sq_pad; rows past Sq
// get Δ = 0. When `lse2` is set the kernel also writes the tcgen05 backward's
// row statistic there: lse·log2(e), less the ALiBi row constant (row_lse2),
// and +inf for rows past Sq and rows whose LSE is −inf.
template <typename T>
__global__ void __launch_bounds__(256) delta_kernel(Params p) {
  const int64_t warp = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t nrows = (int64_t)p.B * p.Hq * p.Sq_pad;
  if (warp >= nrows) return;
  const int i = (int)(warp % p.Sq_pad);
  const int hq = (int)((warp / p.Sq_pad) % p.Hq);
  const int b = (int)(warp / ((int64_t)p.Sq_pad * p.Hq));
  float acc = 0.f;
  if (i < p.Sq) {
    const T* O = (const T*)p.o + (int64_t)b * p.so_[0] + (int64_t)hq * p.so_[1] + (int64_t)i * p.so_[2];
    const T* DO = (const T*)p.dout + (int64_t)b * p.sdo_[0] + (int64_t)hq * p.sdo_[1] + (int64_t)i * p.sdo_[2];
    for (int d = lane; d < p.D; d += 32)
      acc = fmaf(to_f32<T>(O[(int64_t)d * p.so_[3]]), to_f32<T>(DO[(int64_t)d * p.sdo_[3]]), acc);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  }
  if (lane == 0) {
    p.delta[warp] = acc;
    if (p.lse2) {
      float l2 = __int_as_float(0x7f800000);
      if (i < p.Sq) {
        const float lse = p.lse[((int64_t)b * p.Hq + hq) * p.Sq + i];
        if (lse != neg_inf()) l2 = row_lse2(p, lse, hq, i);
      }
      p.lse2[warp] = l2;
    }
  }
}

// Δ for 16-bit rows with unit inner stride and 16-byte aligned rows: G = D/8
// threads per row, each loading 8 elements of O and dO with one 16-byte load
// apiece (the kernel is HBM-bound: 4·D bytes read per row), reduced with
// shuffles inside the group. Same outputs as delta_kernel.
template <typename T, int G>
__global__ void __launch_bounds__(256) delta_vec_kernel(Params p) {
  const int64_t row = (int64_t)blockIdx.x * (256 / G) + (threadIdx.x / G);
  const int g = threadIdx.x % G;
  const int64_t nrows = (int64_t)p.B * p.Hq * p.Sq_pad;
  if (row >= nrows) return;  // whole groups leave together (256 is a multiple of G)
  const int i = (int)(row % p.Sq_pad);
  const int hq = (int)((row / p.Sq_pad) % p.Hq);
  const int b = (int)(row / ((int64_t)p.Sq_pad * p.Hq));
  float acc = 0.f;
  if (i < p.Sq) {
    const T* O = (const T*)p.o + (int64_t)b * p.so_[0] + (int64_t)hq * p.so_[1] + (int64_t)i * p.so_[2];
    const T* DO = (const T*)p.dout + (int64_t)b * p.sdo_[0] + (int64_t)hq * p.sdo_[1] + (int64_t)i * p.sdo_[2];
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(O) + g);
    const uint4 c = __ldg(reinterpret_cast<const uint4*>(DO) + g);
    const T* ae = reinterpret_cast<const T*>(&a);
    const T* ce = reinterpret_cast<const T*>(&c);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc = fmaf(to_f32<T>(ae[e]), to_f32<T>(ce[e]), acc);
  }
#pragma unroll
  for (int off = G / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (g == 0) {
    p.delta[row] = acc;
    if (p.lse2) {
      float l2 = __int_as_float(0x7f800000);
      if (i < p.Sq) {
        const float lse = p.lse[((int64_t)b * p.Hq + hq) * p.Sq + i];
        if (lse != neg_inf()) l2 = row_lse2(p, lse, hq, i);
      }
      p.lse2[row] = l2;
    }
  }
}

// Rows of a [B, H, S, D] 16-bit tensor start on 16-byte boundaries and are
// contiguous in D.
static bool rows_vec_ok(const void* ptr, const int64_t* st, int D) {
  if (((uintptr_t)ptr & 15u) != 0 || st[3] != 1 || (D % 8) != 0) return false;
  for (int k = 0; k < 3; ++k)
    if ((st[k] * 2) % 16 != 0) return false;
  return true;
}

template <typename T, int DP>
int launch_fwd_t(const Params& p, cudaStream_t st) {
  const size_t smem = (size_t)(TM + 2 * TN) * (DP + 4) * 4 + (size_t)TM * (TN + 1) * 4;
  auto kern = simt_fwd_kernel<T, DP>;
  if (cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem))
    return cuda_fail("simt_fwd_kernel shared-memory attribute", e);
  dim3 grid((p.Sq + TM - 1) / TM, p.Hq, p.B);
  if (grid.x == 0 || grid.y == 0 || grid.z == 0) return BFA_OK;
  kern<<<grid, NT, smem, st>>>(p);
  note_launch();
  return launch_status("simt_fwd_kernel launch");
}

template <typename T, int DP>
int launch_bwd_t(const Params& p, cudaStream_t st) {
  if (p.phases & BFA_BWD_PHASE_DQ) {
    const size_t smem = (size_t)(2 * TM + 2 * TN) * (DP + 4) * 4 + (size_t)TM * (TN + 1) * 4;
    auto kern = simt_bwd_dq_kernel<T, DP>;
    if (cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem))
      return cuda_fail("simt backward shared-memory attribute", e);
    dim3 grid((p.Sq + TM - 1) / TM, p.Hq, p.B);
    if (grid.x && grid.y && grid.z) {
      kern<<<grid, NT, smem, st>>>(p);
      note_launch();
      if (int rc = launch_status("simt backward kernel launch")) return rc;
    }
  }
  if (p.phases & BFA_BWD_PHASE_DKDV) {
    const size_t smem = (size_t)(2 * TM + 2 * TN) * (DP + 4) * 4 + (size_t)2 * TN * (TM + 1) * 4 + 2 * TM * 4;
    auto kern = simt_bwd_dkdv_kernel<T, DP>;
    if (cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem))
      return cuda_fail("simt backward shared-memory attribute", e);
    const int n_kt = (p.Sk + TN - 1) / TN;
    // Split each kv tile's work over a cluster of up to 8 CTAs until about
    // two waves of CTAs cover the SMs (bounded by the work items a tile has).
    const long long units = (long long)n_kt * p.Hkv * p.B;
    int nsplit = 1;
    if (units > 0) {
      const long long want = (2LL * sm_count() + units - 1) / units;
      const int items = p.G * ((p.Sq + TM - 1) / TM);
      nsplit = (int)std::min<long long>({8LL, want, (long long)std::max(items, 1)});
      nsplit = std::max(nsplit, 1);
    }
    if (units > 0) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)(n_kt * nsplit), p.Hkv, p.B);
      cfg.blockDim = dim3(NT);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = st;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = (unsigned)nsplit;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p)) return cuda_fail("simt dK/dV cluster launch", e);
      note_launch();
      if (int rc = launch_status("simt backward kernel launch")) return rc;
    }
  }
  return BFA_OK;
}

template <typename T>
int dispatch_dp_fwd(const Params& p, cudaStream_t st) {
  if (p.D <= 32) return launch_fwd_t<T, 32>(p, st);
  if (p.D <= 64) return launch_fwd_t<T, 64>(p, st);
  if (p.D <= 128) return launch_fwd_t<T, 128>(p, st);
  return launch_fwd_t<T, 256>(p, st);
}

template <typename T>
int dispatch_dp_bwd(const Params& p, cudaStream_t st) {
  if (p.D <= 32) return launch_bwd_t<T, 32>(p, st);
  if (p.D <= 64) return launch_bwd_t<T, 64>(p, st);
  if (p.D <= 128) return launch_bwd_t<T, 128>(p, st);
  return launch_bwd_t<T, 256>(p, st);
}

}  // namespace

int simt_fwd(const Params& p, int dtype, cudaStream_t st) {
  switch (dtype) {
    case BFA_DTYPE_F32: return dispatch_dp_fwd<float>(p, st);
    case BFA_DTYPE_F16: return dispatch_dp_fwd<__half>(p, st);
    case BFA_DTYPE_BF16: return dispatch_dp_fwd<__nv_bfloat16>(p, st);
  }
  return BFA_ERR_UNSUPPORTED;
}

int simt_bwd(const Params& p, int dtype, cudaStream_t st) {
  switch (dtype) {
    case BFA_DTYPE_F32: return dispatch_dp_bwd<float>(p, st);
    case BFA_DTYPE_F16: return dispatch_dp_bwd<__half>(p, st);
    case BFA_DTYPE_BF16: return dispatch_dp_bwd<__nv_bfloat16>(p, st);
  }
  return BFA_ERR_UNSUPPORTED;
}

int launch_delta(const Params& p, int dtype, cudaStream_t st) {
  const int64_t rows = (int64_t)p.B * p.Hq * p.Sq_pad;
  if (rows == 0) return BFA_OK;
  if ((dtype == BFA_DTYPE_BF16 || dtype == BFA_DTYPE_F16) && (p.D == 64 || p.D == 128 || p.D == 256) &&
      rows_vec_ok(p.o, p.so_, p.D) && rows_vec_ok(p.dout, p.sdo_, p.D)) {
    const int G = p.D / 8, per_block = 256 / G;
    const unsigned vblocks = (unsigned)((rows + per_block - 1) / per_block);
    const bool bf = dtype == BFA_DTYPE_BF16;
    if (G == 32) {
      if (bf) delta_vec_kernel<__nv_bfloat16, 32><<<vblocks, 256, 0, st>>>(p);
      else delta_vec_kernel<__half, 32><<<vblocks, 256, 0, st>>>(p);
    } else if (G == 16) {
      if (bf) delta_vec_kernel<__nv_bfloat16, 16><<<vblocks, 256, 0, st>>>(p);
      else delta_vec_kernel<__half, 16><<<vblocks, 256, 0, st>>>(p);
    } else {
      if (bf) delta_vec_kernel<__nv_bfloat16, 8><<<vblocks, 256, 0, st>>>(p);
      else delta_vec_kernel<__half, 8><<<vblocks, 256, 0, st>>>(p);
    }
    note_launch();
    return launch_status("delta_vec_kernel launch");
  }
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  switch (dtype) {
    case BFA_DTYPE_F32: delta_kernel<float><<<blocks, 256, 0, st>>>(p); break;
    case BFA_DTYPE_F16: delta_kernel<__half><<<blocks, 256, 0, st>>>(p); break;
    case BFA_DTYPE_BF16: delta_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(p); break;
    default: return BFA_ERR_UNSUPPORTED;
  }
  note_launch();
  return launch_status("delta_kernel launch");
}

}  // namespace bfa
