// bfa_common.cuh -- device helpers shared by every attention kernel.
//
// The logit transform and the keep-mask follow the reference kernel
// (npu_flash_attention.py:102-141):
//   s = (q·k) * scale
//   s = cap * tanh(s / cap)            if soft_cap > 0       (:105-106)
//   s = s + slope[hq] * (i - j)        if ALiBi              (:108-109)
//   keep iff (!causal || i >= j) && (W == 0 || i - j <= W) && j < Sk  (:139,141)
// with i, j absolute positions (local index + the problem's position offset).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "bfa.h"

namespace bfa {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ float neg_inf() { return __int_as_float(0xff800000); }

// Parameters of one launch, flattened for the device.
struct Params {
  const void* q; const void* k; const void* v; void* o;
  const void* dout; void* dq; void* dk; void* dv;
  float* lse; float* delta;
  // Backward row statistics, one row pitch `Sq_pad` per (b, hq): `delta` holds
  // Δ and `lse2` (may be null) holds lse·log2(e), +inf for rows past Sq or
  // rows that see no key, so that exp2(x − lse2) is 0 there.
  float* lse2;
  int32_t Sq_pad;
  int64_t sq_[4], sk_[4], sv_[4], so_[4], sdo_[4], sdq_[4], sdk_[4], sdv_[4];
  int32_t B, Hq, Hkv, G, Sq, Sk, D;
  int32_t causal, window;
  float scale, soft_cap;
  const float* alibi;
  int64_t q_off, k_off;
  // Document masking (null: off): for every absolute position x, the
  // document holding x spans positions [doc_lo[x], doc_hi[x]); pairs (i, j)
  // are kept only inside one document.
  const int32_t* doc_lo;
  const int32_t* doc_hi;
  // Block-sparse mask (null: off): byte [b, hq, r / 128, c / 128] at strides
  // blk_s (batch, q-head, query block; key block stride 1), r and c local.
  const uint8_t* blk;
  int64_t blk_s[3];
  int32_t* status;
  uint64_t timeout_ns;
  uint32_t debug_flags;
  uint32_t phases;  // backward: mask of BFA_BWD_PHASE_* (never 0 here)
  uint32_t grad_acc;  // backward: dq/dk/dv are fp32 accumulators (add, don't store)
  // backward: the dQ kernel forms Δ and lse2 of its rows itself and writes
  // them for the dK/dV kernel that runs after it (no separate Δ pass).
  uint32_t fuse_delta;
  // forward: `o` is an fp32 running output and `lse` its running LSE; the
  // epilogue merges the call's result into both (merge_weights).
  uint32_t out_acc;
};

// The LSE merge of a block's result (LSE lp) into a running one (LSE la):
// ln = logaddexp(la, lp), the running output's weight wa = e^(la − ln) and the
// block's wp = e^(lp − ln); both weights 0 and ln = −inf when neither has a key.
struct MergeWeights {
  float wa, wp, ln;
};

__device__ __forceinline__ MergeWeights merge_weights(float la, float lp) {
  MergeWeights w{0.f, 0.f, neg_inf()};
  const float mx = fmaxf(la, lp);
  if (mx != neg_inf()) {
    const float ea = expf(la - mx), ep = expf(lp - mx);
    w.ln = mx + logf(ea + ep);
    w.wa = expf(la - w.ln);
    w.wp = expf(lp - w.ln);
  }
  return w;
}

template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Keep-mask on absolute positions.
__device__ __forceinline__ bool keep_pair(const Params& p, int64_t i, int64_t j) {
  if (p.causal && j > i) return false;
  if (p.window > 0 && i - j > p.window) return false;
  if (p.doc_lo && (j < p.doc_lo[i] || j >= p.doc_hi[i])) return false;
  return true;
}

constexpr int kMaskBlock = 128;  // block-sparse mask granularity (rows and keys)

// Whether block (qb, kb) of (b, hq) is computed (always without a mask).
__device__ __forceinline__ bool block_on(const Params& p, int b, int hq, int qb, int kb) {
  return !p.blk || p.blk[(int64_t)b * p.blk_s[0] + (int64_t)hq * p.blk_s[1] + (int64_t)qb * p.blk_s[2] + kb] != 0;
}

// Visits the steps of a loop that a block-sparse mask leaves on: step(j)
// returns the j-th visited step for nondecreasing j, where next(s) gives the
// first visited step after s. A kernel whose roles consume steps out of order
// keeps one walker per kind of consumer.
template <typename Next>
struct StepWalker {
  Next next;
  int j, s;
  __device__ __forceinline__ StepWalker(Next n, int start) : next(n), j(-1), s(start) {}
  __device__ __forceinline__ int step(int want) {
    while (j < want) {
      s = next(s);
      ++j;
    }
    return s;
  }
};
template <typename Next>
__device__ __forceinline__ StepWalker<Next> make_walker(Next n, int start) {
  return StepWalker<Next>(n, start);
}

// Without documents, whether a tile is fully kept is linear in its moving
// coordinate: a kernel that walks key tiles for fixed query rows (or query
// tiles for fixed keys) finds the kept range once and tests each step with
// two compares instead of the general tile test.
struct KeptRange {
  int64_t lo, hi;
  __device__ __forceinline__ bool has(int64_t x) const { return x >= lo && x <= hi; }
};

// Key tiles [c, c + nk) against fixed query rows [r0, r0 + nr) (local
// indices): every pair is kept for c in the range (causal: the tile's last
// key is at or before the first row; window: the last row minus the first
// key is at most W; the tile lies inside Sk; with rows_in, the rows inside Sq).
__device__ __forceinline__ KeptRange kept_keys(const Params& p, int r0, int nr, int nk, bool rows_in) {
  KeptRange k;
  k.lo = p.window > 0 ? (int64_t)r0 + nr - 1 + p.q_off - p.k_off - p.window : 0;
  k.hi = (int64_t)p.Sk - nk;
  if (p.causal) k.hi = min(k.hi, (int64_t)r0 + p.q_off - p.k_off - (nk - 1));
  if (rows_in && r0 + nr > p.Sq) k.hi = k.lo - 1;
  return k;
}

// Query tiles [q, q + nq) against fixed keys [c0, c0 + nk): the same
// conditions, with the rows inside Sq and the keys inside Sk.
__device__ __forceinline__ KeptRange kept_queries(const Params& p, int c0, int nk, int nq) {
  KeptRange k;
  k.lo = p.causal ? (int64_t)c0 + nk - 1 + p.k_off - p.q_off : -((int64_t)1 << 40);
  k.hi = (int64_t)p.Sq - nq;
  if (p.window > 0) k.hi = min(k.hi, (int64_t)p.window + c0 + p.k_off - p.q_off - (nq - 1));
  if (c0 + nk > p.Sk) k.hi = k.lo - 1;
  return k;
}

// keep_pair plus the block-sparse mask of (b, hq); positions absolute.
__device__ __forceinline__ bool keep_elem(const Params& p, int b, int hq, int64_t gi, int64_t gj) {
  return keep_pair(p, gi, gj) &&
         block_on(p, b, hq, (int)((gi - p.q_off) / kMaskBlock), (int)((gj - p.k_off) / kMaskBlock));
}

// True when every query row of [i_min, i_max] and every key of [j_min,
// j_max] (absolute positions) lie in one document (always without documents).
__device__ __forceinline__ bool same_document(const Params& p, int64_t i_min, int64_t i_max, int64_t j_min,
                                              int64_t j_max) {
  if (!p.doc_lo) return true;
  const int32_t lo = p.doc_lo[i_min];
  return p.doc_lo[i_max] == lo && j_min >= lo && j_max < p.doc_hi[i_min];
}

// Logit transform (cap then ALiBi). `t_out` receives tanh(s/cap) for the
// backward chain (1 when no cap).
__device__ __forceinline__ float transform_logit(float dot, float scale, float cap,
                                                 float slope, int64_t i, int64_t j,
                                                 float* t_out) {
  float s = dot * scale;
  float t = 0.f;
  if (cap > 0.f) {
    t = tanhf(s / cap);
    s = cap * t;
  }
  if (t_out) *t_out = t;
  s += slope * (float)(i - j);
  return s;
}

// ALiBi reference key g0 of query row i (absolute positions). The tcgen05
// kernels form the bias of pair (i, j) as slope·(g0 - j) and fold the row
// constant slope·(i - g0), which the softmax does not see, into the LSE
// alone (the forward adds it to its LSE output; the backward's row statistic
// is lse - slope·(i - g0), formed in double). For slope > 0 (the reference's
// sign, npu_flash_attention.py:109) g0 is the first key the row can see at
// all, max(0, i - W) (0 without a window; no earlier than the start of the
// row's document): the logits that carry the softmax
// then stay O(1) instead of growing with i - j (an fp32 logit near 6e4,
// slope ~1 at 64k positions, has an ulp of 4e-3, which shifts each
// probability by up to 0.3%). g0 does not depend on the call's key offset, so
// the row statistic agrees across the calls of a blockwise (context-parallel)
// backward. For slope <= 0 the bias peaks at the diagonal and g0 = i (the
// bias is slope·(i - j) as written).
// `row_ok` false (a padding row past Sq) skips the document lookup, whose
// array covers only the problem's positions.
__device__ __forceinline__ int64_t alibi_ref(const Params& p, float slope, int64_t gi, bool row_ok = true) {
  if (!(slope > 0.f)) return gi;
  int64_t g0 = p.window > 0 ? max((int64_t)0, gi - (int64_t)p.window) : (int64_t)0;
  if (p.doc_lo && row_ok) g0 = max(g0, (int64_t)p.doc_lo[gi]);
  return g0;
}

// Backward row statistic from the forward LSE of query row i of head hq:
// lse·log2(e) minus the ALiBi row constant slope·(i - g0)·log2(e) that the
// tcgen05 kernels keep out of their logits (alibi_ref). Formed in double, so
// that the statistic carries exactly the fp32 LSE it was given.
__device__ __forceinline__ float row_lse2(const Params& p, float lse, int hq, int i) {
  if (!p.alibi) return lse * kLog2e;
  const float slope = p.alibi[hq];
  const int64_t gi = (int64_t)i + p.q_off;
  const double shift = (double)slope * (double)(gi - alibi_ref(p, slope, gi));
  return (float)(((double)lse - shift) * 1.4426950408889634);
}

// Kept key columns [lo, hi) for one query row: the columns are local keys
// j0 + c, c in [0, n). `row_ok` false (a padding row) gives an empty range.
__device__ __forceinline__ void keys_for_query(const Params& p, int64_t gi, bool row_ok, int j0,
                                               int n, int* lo, int* hi) {
  int64_t l = 0, h = n;
  h = min(h, (int64_t)p.Sk - j0);
  if (p.causal) h = min(h, gi - p.k_off - j0 + 1);
  if (p.window > 0) l = max(l, gi - p.window - p.k_off - j0);
  if (p.doc_lo && row_ok) {
    l = max(l, (int64_t)p.doc_lo[gi] - p.k_off - j0);
    h = min(h, (int64_t)p.doc_hi[gi] - p.k_off - j0);
  }
  if (!row_ok || h < l) h = l;
  l = max((int64_t)0, min(l, (int64_t)n));
  h = max(l, min(h, (int64_t)n));
  *lo = (int)l;
  *hi = (int)h;
}

// Kept query columns [lo, hi) for one key row: the columns are local queries
// q0 + c, c in [0, n).
__device__ __forceinline__ void queries_for_key(const Params& p, int64_t gj, bool row_ok, int q0,
                                                int n, int* lo, int* hi) {
  int64_t l = 0, h = n;
  h = min(h, (int64_t)p.Sq - q0);
  if (p.causal) l = max(l, gj - p.q_off - q0);
  if (p.window > 0) h = min(h, gj + p.window - p.q_off - q0 + 1);
  if (p.doc_lo && row_ok) {
    l = max(l, (int64_t)p.doc_lo[gj] - p.q_off - q0);
    h = min(h, (int64_t)p.doc_hi[gj] - p.q_off - q0);
  }
  if (!row_ok || h < l) h = l;
  l = max((int64_t)0, min(l, (int64_t)n));
  h = max(l, min(h, (int64_t)n));
  *lo = (int)l;
  *hi = (int)h;
}

// Range of key indices [lo, hi) (local) that can be kept for local query
// rows [r0, r1). Tiles outside it are fully masked and skipped.
__device__ __forceinline__ void key_range(const Params& p, int r0, int r1, int* lo, int* hi) {
  int64_t l = 0, h = p.Sk;
  int64_t i_first = r0 + p.q_off, i_last = (r1 - 1) + p.q_off;
  if (p.causal) {  // j <= i_last
    int64_t lim = i_last - p.k_off + 1;
    if (lim < h) h = lim;
  }
  if (p.window > 0) {  // j >= i_first - W
    int64_t lim = i_first - p.window - p.k_off;
    if (lim > l) l = lim;
  }
  if (p.doc_lo) {  // documents are contiguous: the first row's start, the last row's end
    l = max(l, (int64_t)p.doc_lo[i_first] - p.k_off);
    h = min(h, (int64_t)p.doc_hi[i_last] - p.k_off);
  }
  if (h < l) h = l;
  if (l < 0) l = 0;
  if (h < 0) h = 0;
  *lo = (int)l;
  *hi = (int)h;
}

// Range of query rows [lo, hi) (local) that can keep any of key rows [c0, c1).
__device__ __forceinline__ void query_range(const Params& p, int c0, int c1, int* lo, int* hi) {
  int64_t l = 0, h = p.Sq;
  int64_t j_first = c0 + p.k_off, j_last = (c1 - 1) + p.k_off;
  if (p.causal) {  // i >= j_first
    int64_t lim = j_first - p.q_off;
    if (lim > l) l = lim;
  }
  if (p.window > 0) {  // i <= j_last + W
    int64_t lim = j_last + p.window - p.q_off + 1;
    if (lim < h) h = lim;
  }
  if (p.doc_lo) {
    l = max(l, (int64_t)p.doc_lo[j_first] - p.q_off);
    h = min(h, (int64_t)p.doc_hi[j_last] - p.q_off);
  }
  if (h < l) h = l;
  if (l < 0) l = 0;
  if (h < 0) h = 0;
  *lo = (int)l;
  *hi = (int)h;
}

}  // namespace bfa
