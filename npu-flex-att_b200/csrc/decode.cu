// decode.cu -- split-KV flash-decoding forward: few query rows per KV head,
// long key sequence.
//
// The reference carries a split-KV forward and its reduce for short Q_LEN
// (npu_flash_attention.py:171-293: flash_attn_fwd_split_kv_kernel writes a
// normalised partial O and a partial LSE per key split, and
// flash_attn_fwd_reduce_kernel merges them with an LSE-weighted sum). There it
// is never launched (and fixes B = 1). This is the working B200 version of that
// path, chosen automatically by bfa_fwd when the G q-heads of a KV head
// together have at most kMaxRowsTotal (64) query rows.
//
// Decode is HBM-bound: every K/V byte is used by only G·Sq rows. So:
//   - one CTA per (batch, KV head, key split, group of up to 16 rows) serves
//     those rows of all G q-heads of that KV head, so K/V cross HBM once however
//     large G is (the row groups of one KV head, up to 4, run side by side and
//     share the K/V in L2);
//   - K/V stream through a cp.async double buffer in 64-key chunks (rows
//     padded by 16 bytes so the shared-memory reads are conflict-free);
//   - for bf16 / fp16 the two small GEMMs (S = q·kᵀ and P·V, all rows in one
//     M = 16 tile) run on the tensor cores with mma.sync m16n8k16, the online
//     softmax on the CUDA cores; fp32 inputs run S, softmax and P·V on the
//     CUDA cores;
//   - the keys are split so that the CTAs fill the GPU in about one wave, and
//     a merge kernel combines the splits' partial (O, LSE) per row. The
//     partials live in the caller's workspace (bfa_fwd_workspace_bytes); the
//     library allocates nothing.
// The math per row is the forward's: S·scale, cap, ALiBi, mask on absolute
// positions (q_off, k_off), base-2 online softmax, O = PV/l and
// LSE = m + ln(l) (natural log), -inf with O = 0 for a row that sees no key.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <type_traits>

#include "bfa_internal.h"
#include "sm100_ptx.cuh"

namespace bfa {
namespace {

constexpr int kDecThreads = 256;
constexpr int kChunk = 64;    // keys per pipeline stage
constexpr int kMaxRows = 16;       // query rows per CTA (one row group)
constexpr int kMaxRowsTotal = 64;  // G·Sq rows per KV head on this path (<= 4 row groups)
constexpr int kRowGroupsS = kDecThreads / kChunk;  // row groups in the S phase

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}
__device__ __forceinline__ float fast_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 16 bytes / two consecutive elements of T -> fp32 (the CUDA-core kernel runs
// only for fp32 inputs; 16-bit inputs take the tensor-core kernel below).
template <typename T>
__device__ __forceinline__ void unpack16(const uint4& u, float* f);
template <>
__device__ __forceinline__ void unpack16<float>(const uint4& u, float* f) {
  f[0] = __uint_as_float(u.x);
  f[1] = __uint_as_float(u.y);
  f[2] = __uint_as_float(u.z);
  f[3] = __uint_as_float(u.w);
}
template <typename T>
__device__ __forceinline__ float2 load2(const uint8_t* p);
template <>
__device__ __forceinline__ float2 load2<float>(const uint8_t* p) {
  return *reinterpret_cast<const float2*>(p);
}

template <typename T, int D, int RB = kMaxRows>
struct DecLayout {
  static constexpr int kRowBytes = D * (int)sizeof(T) + 16;  // padded K/V row
  static constexpr int kTileBytes = kChunk * kRowBytes;
  static constexpr int kOffK = 0;                            // [2 stages][kChunk rows]
  static constexpr int kOffV = 2 * kTileBytes;
  static constexpr int kOffQ = 4 * kTileBytes;               // fp32 [kMaxRows][D]
  static constexpr int kOffP = kOffQ + kMaxRows * D * 4;     // fp32 [kMaxRows][kChunk]
  static constexpr int kOffRow = kOffP + kMaxRows * kChunk * 4;  // m, l, alpha per row
  static constexpr int kSmemBytes = kOffRow + 3 * kMaxRows * 4;
  static constexpr int kPairs = D / 2;                       // P·V: one thread per 2 columns
  static constexpr int kRowGroupsO = kDecThreads / kPairs;
  static constexpr int kRowsPerThreadO = (RB + kRowGroupsO - 1) / kRowGroupsO;
  static_assert(kDecThreads % kPairs == 0, "P·V thread map");
  static_assert(kSmemBytes <= 232448, "smem budget");
};

// One CTA: KV head (b, hkv), keys [kvis_lo + split·split_len, + split_len) of
// the visible range, all rows r = g·Sq + s (q-head hkv·G + g, query s).
// RB (4, 8 or 16) is R = G·Sq rounded up: the loops run over RB rows with no
// per-row test; rows R..RB-1 carry q = 0 and are never stored.
// Writes the split's normalised O (fp32) and LSE per row:
//   part_o[(row·n_split + split)·D + d], part_lse[row·n_split + split],
// row = (b·Hq + hq)·Sq + s.
template <typename T, int D, int RB, bool PLAIN>
__global__ void __launch_bounds__(kDecThreads)
    decode_split_kernel(const Params p, int n_split, int kvis_lo, int split_len, float* __restrict__ part_o,
                        float* __restrict__ part_lse) {
  using L = DecLayout<T, D, RB>;
  static_assert(RB % kRowGroupsS == 0 && RB <= kMaxRows, "row bucket");
  extern __shared__ __align__(16) uint8_t smem[];
  float* qs = reinterpret_cast<float*>(smem + L::kOffQ);
  float* ps = reinterpret_cast<float*>(smem + L::kOffP);
  float* row_m = reinterpret_cast<float*>(smem + L::kOffRow);
  float* row_l = row_m + kMaxRows;
  float* row_a = row_l + kMaxRows;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // Block: (KV head, split, row group); the row group is the fastest index so
  // that the CTAs of one KV head's row groups read the same K/V at once (L2).
  const int n_rg = (p.G * p.Sq + kMaxRows - 1) / kMaxRows;
  const int rg = (int)(blockIdx.x % n_rg);
  const int row0 = rg * kMaxRows;  // this CTA's rows: row0 + [0, R)
  const int R = min(kMaxRows, p.G * p.Sq - row0);
  const int split = (int)((blockIdx.x / n_rg) % n_split);
  const int bkv = (int)(blockIdx.x / n_rg / n_split);
  const int hkv = bkv % p.Hkv, b = bkv / p.Hkv;
  int klo, khi;
  key_range(p, 0, p.Sq, &klo, &khi);
  const int kb = max(kvis_lo + split * split_len, klo);
  const int ke = min(kvis_lo + (split + 1) * split_len, khi);
  const int n_chunks = (ke > kb) ? (ke - kb + kChunk - 1) / kChunk : 0;
  const T* qg = static_cast<const T*>(p.q);
  const T* kg = static_cast<const T*>(p.k);
  const T* vg = static_cast<const T*>(p.v);
  // q pre-scaled into base-2 logits on the plain path (x = q·k directly).
  const float qmul = PLAIN ? p.scale * kLog2e : 1.f;

  auto load_chunk = [&](int c, int stage) {
    constexpr int kPieces = D * (int)sizeof(T) / 16;
    const int key0 = kb + c * kChunk;
    for (int idx = tid; idx < 2 * kChunk * kPieces; idx += kDecThreads) {
      const int which = idx / (kChunk * kPieces);  // 0: K, 1: V
      const int rem = idx - which * (kChunk * kPieces);
      const int n = rem / kPieces, pc = rem - n * kPieces;
      const int key = key0 + n;
      uint8_t* dst = smem + (which ? L::kOffV : L::kOffK) + stage * L::kTileBytes + n * L::kRowBytes + pc * 16;
      if (key < ke) {
        const T* src = which ? vg + (int64_t)b * p.sv_[0] + (int64_t)hkv * p.sv_[1] + (int64_t)key * p.sv_[2]
                             : kg + (int64_t)b * p.sk_[0] + (int64_t)hkv * p.sk_[1] + (int64_t)key * p.sk_[2];
        cp_async16(dst, src + pc * (16 / (int)sizeof(T)));
      } else {
        *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    cp_async_commit();
  };
  if (n_chunks > 0) load_chunk(0, 0);

  for (int idx = tid; idx < kMaxRows * D; idx += kDecThreads) {
    const int r = idx / D, d = idx - r * D;
    float x = 0.f;
    if (r < R) {
      const int g = (row0 + r) / p.Sq, s = (row0 + r) - g * p.Sq;
      const int hq = hkv * p.G + g;
      x = to_f32(qg[(int64_t)b * p.sq_[0] + (int64_t)hq * p.sq_[1] + (int64_t)s * p.sq_[2] + (int64_t)d * p.sq_[3]]) *
          qmul;
    }
    qs[idx] = x;
  }
  if (tid < kMaxRows) {
    row_m[tid] = neg_inf();
    row_l[tid] = 0.f;
    row_a[tid] = 1.f;
  }
  // Padding rows R..RB-1 keep P = 0 (the S phase writes only rows < R).
  for (int idx = tid; idx < kMaxRows * kChunk; idx += kDecThreads) ps[idx] = 0.f;

  constexpr int RO = L::kRowsPerThreadO;
  const int dp = tid % L::kPairs, rgo = tid / L::kPairs;
  float2 oacc[RO];
#pragma unroll
  for (int j = 0; j < RO; ++j) oacc[j] = make_float2(0.f, 0.f);

  for (int c = 0; c < n_chunks; ++c) {
    const int stage = c & 1;
    if (c + 1 < n_chunks) {
      load_chunk(c + 1, stage ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // chunk c (and, at c = 0, q and the row state) visible

    // S: thread -> key n of the chunk, rows rgs + 4j.
    {
      const int n = tid % kChunk, rgs = tid / kChunk;
      const int key = kb + c * kChunk + n;
      const uint8_t* krow = smem + L::kOffK + stage * L::kTileBytes + n * L::kRowBytes;
      float acc[RB / kRowGroupsS];
#pragma unroll
      for (int j = 0; j < RB / kRowGroupsS; ++j) acc[j] = 0.f;
      constexpr int kPer = 16 / (int)sizeof(T);
#pragma unroll 4
      for (int d0 = 0; d0 < D; d0 += kPer) {
        float kf[kPer];
        unpack16<T>(*reinterpret_cast<const uint4*>(krow + d0 * (int)sizeof(T)), kf);
#pragma unroll
        for (int j = 0; j < RB / kRowGroupsS; ++j) {
          const float* qr = qs + (rgs + kRowGroupsS * j) * D + d0;
#pragma unroll
          for (int e = 0; e < kPer; ++e) acc[j] = fmaf(qr[e], kf[e], acc[j]);
        }
      }
#pragma unroll
      for (int j = 0; j < RB / kRowGroupsS; ++j) {
        const int r = rgs + kRowGroupsS * j;
        if (r < R) {
          const int g = (row0 + r) / p.Sq, s = (row0 + r) - g * p.Sq;
          const int64_t gi = (int64_t)s + p.q_off, gj = (int64_t)key + p.k_off;
          const bool keep = key < ke && keep_elem(p, b, hkv * p.G + g, gi, gj);
          float x = acc[j];
          if (!PLAIN) {
            const float slope = p.alibi ? p.alibi[hkv * p.G + g] : 0.f;
            x = transform_logit(x, p.scale, p.soft_cap, slope, gi, gj, nullptr) * kLog2e;
          }
          ps[r * kChunk + n] = keep ? x : neg_inf();
        }
      }
    }
    __syncthreads();

    // Online softmax: one warp per row, two keys per lane.
    for (int r = warp; r < R; r += kDecThreads / 32) {
      const float x0 = ps[r * kChunk + lane], x1 = ps[r * kChunk + lane + 32];
      const float mx = warp_max(fmaxf(x0, x1));
      const float m_old = row_m[r];
      const float m_new = fmaxf(m_old, mx);
      const float m_use = (m_new == neg_inf()) ? 0.f : m_new;
      const float p0 = fast_ex2(x0 - m_use), p1 = fast_ex2(x1 - m_use);
      ps[r * kChunk + lane] = p0;
      ps[r * kChunk + lane + 32] = p1;
      const float sum = warp_sum(p0 + p1);
      if (lane == 0) {
        const float alpha = fast_ex2(m_old - m_use);
        row_a[r] = alpha;
        row_l[r] = row_l[r] * alpha + sum;
        row_m[r] = m_new;
      }
    }
    __syncthreads();

    // O = O·alpha + P·V: thread -> columns (2dp, 2dp + 1), rows rgo + groups·j.
    {
      const uint8_t* vbase = smem + L::kOffV + stage * L::kTileBytes + dp * 2 * (int)sizeof(T);
#pragma unroll
      for (int j = 0; j < RO; ++j) {
        const float a = row_a[rgo + L::kRowGroupsO * j];
        oacc[j].x *= a;
        oacc[j].y *= a;
      }
#pragma unroll 4
      for (int n = 0; n < kChunk; ++n) {
        const float2 v2 = load2<T>(vbase + n * L::kRowBytes);
#pragma unroll
        for (int j = 0; j < RO; ++j) {
          const float pr = ps[(rgo + L::kRowGroupsO * j) * kChunk + n];
          oacc[j].x = fmaf(pr, v2.x, oacc[j].x);
          oacc[j].y = fmaf(pr, v2.y, oacc[j].y);
        }
      }
    }
    __syncthreads();  // the stage and ps are rewritten by the next chunk
  }

  // The split's normalised O and LSE.
#pragma unroll
  for (int j = 0; j < RO; ++j) {
    const int r = rgo + L::kRowGroupsO * j;
    if (r < R) {
      const int g = (row0 + r) / p.Sq, s = (row0 + r) - g * p.Sq;
      const int64_t row = ((int64_t)b * p.Hq + hkv * p.G + g) * p.Sq + s;
      const float l = row_l[r];
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
      *reinterpret_cast<float2*>(part_o + (row * n_split + split) * D + 2 * dp) =
          make_float2(oacc[j].x * inv, oacc[j].y * inv);
      if (dp == 0)
        part_lse[row * n_split + split] = (l > 0.f) ? (row_m[r] + __log2f(l)) * kLn2 : neg_inf();
    }
  }
}

// ------------------------------------------------------------------ 16-bit
// The same split kernel for bf16 / fp16 with the two small GEMMs on the
// tensor cores (mma.sync m16n8k16, fp32 accumulate): all <= 16 rows are one
// M = 16 tile. Per 64-key chunk:
//   S:   warp w computes keys [8w, 8w + 8) for all rows: A = q (fragments held
//        in registers for the whole CTA), B = K rows from shared memory;
//   softmax as in the CUDA-core kernel, on an fp32 P tile in shared memory;
//   P·V: warp w owns O columns [w·D/8, (w+1)·D/8): A = P rounded to the input
//        type (as the tcgen05 forward and the reference, p.to(v.dtype)), B = V
//        via ldmatrix.trans.
// This takes about a quarter of the instructions of the CUDA-core version,
// whose issue rate bounds it, so the kernel can run at HBM speed.
constexpr int kPRow = kChunk + 8;  // logit row pitch (floats)
// P (16-bit pairs) row pitch in 32-bit words: rows g and g + 1 four banks
// apart, so the A-fragment reads of P·V are conflict-free.
constexpr int kP16Row = kChunk / 2 + 4;
// K/V chunks per CTA: a double buffer. Two stages (three CTAs per SM at
// D = 128) measured faster than three (two CTAs per SM) on every decode shape
// tried: more CTAs per SM keep more loads in flight than a deeper ring.
constexpr int kStagesM = 2;

template <typename T, int D>
struct DecLayoutM {
  static constexpr int kRowBytes = D * 2 + 16;
  static constexpr int kTileBytes = kChunk * kRowBytes;
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kStagesM * kTileBytes;
  static constexpr int kOffP = 2 * kStagesM * kTileBytes;      // fp32 [16][kPRow]
  static constexpr int kOffRow = kOffP + kMaxRows * kPRow * 4;   // m, l, alpha per row
  static constexpr int kOffP16 = kOffRow + 3 * kMaxRows * 4;     // P packed to 16 bits, [16][kP16Row] words
  static constexpr int kSmemBytes = kOffP16 + kMaxRows * kP16Row * 4;
  static constexpr int kNT = D / 64;                           // 8-column n-tiles per warp in P·V
  static_assert(sizeof(T) == 2 && D % 64 == 0, "16-bit, D multiple of 64");
  static_assert(kSmemBytes <= 232448, "smem budget");
};

template <bool BF16>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (BF16)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                              uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_trans(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}

template <typename T, int D, bool PLAIN>
__global__ void __launch_bounds__(kDecThreads, D <= 128 ? 3 : 1)
    decode_mma_kernel(const Params p, int n_split, int kvis_lo, int split_len, float* __restrict__ part_o,
                      float* __restrict__ part_lse) {
  using L = DecLayoutM<T, D>;
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int NT = L::kNT;
  extern __shared__ __align__(16) uint8_t smem[];
  float* ps = reinterpret_cast<float*>(smem + L::kOffP);
  float* row_m = reinterpret_cast<float*>(smem + L::kOffRow);
  float* row_l = row_m + kMaxRows;
  float* row_a = row_l + kMaxRows;
  uint32_t* p16 = reinterpret_cast<uint32_t*>(smem + L::kOffP16);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  // Block: (KV head, split, row group); the row group is the fastest index so
  // that the CTAs of one KV head's row groups read the same K/V at once (L2).
  const int n_rg = (p.G * p.Sq + kMaxRows - 1) / kMaxRows;
  const int rg = (int)(blockIdx.x % n_rg);
  const int row0 = rg * kMaxRows;  // this CTA's rows: row0 + [0, R)
  const int R = min(kMaxRows, p.G * p.Sq - row0);
  const int split = (int)((blockIdx.x / n_rg) % n_split);
  const int bkv = (int)(blockIdx.x / n_rg / n_split);
  const int hkv = bkv % p.Hkv, b = bkv / p.Hkv;
  int klo, khi;
  key_range(p, 0, p.Sq, &klo, &khi);
  const int kb = max(kvis_lo + split * split_len, klo);
  const int ke = min(kvis_lo + (split + 1) * split_len, khi);
  const int n_chunks = (ke > kb) ? (ke - kb + kChunk - 1) / kChunk : 0;
  const T* kg = static_cast<const T*>(p.k);
  const T* vg = static_cast<const T*>(p.v);
  const float sl2 = p.scale * kLog2e;

  // K/V chunk loads: thread tid copies 16-byte piece tid % kPieces of rows
  // tid / kPieces + kRowsPerPass·i (K and V alike). The addresses come from
  // the launch parameters at each call (few live registers: three CTAs per
  // SM at head dim <= 128). Keys past the split's end (only in its last
  // chunk) are zero-filled.
  constexpr int kPieces = D * 2 / 16;
  constexpr int kRowsPerPass = kDecThreads / kPieces;
  constexpr int kPasses = kChunk / kRowsPerPass;
  static_assert(kDecThreads % kPieces == 0 && kChunk % kRowsPerPass == 0, "piece mapping");
  auto load_chunk = [&](int c, int stage) {
    const int n0 = tid / kPieces, pc = tid % kPieces;
    const int key0 = kb + c * kChunk;
    const bool whole = key0 + kChunk <= ke;
    const int64_t kr = key0 + n0;
    const T* kp = kg + (int64_t)b * p.sk_[0] + (int64_t)hkv * p.sk_[1] + kr * p.sk_[2] + pc * 8;
    const T* vp = vg + (int64_t)b * p.sv_[0] + (int64_t)hkv * p.sv_[1] + kr * p.sv_[2] + pc * 8;
    uint8_t* kd = smem + L::kOffK + stage * L::kTileBytes + n0 * L::kRowBytes + pc * 16;
    uint8_t* vd = kd + (L::kOffV - L::kOffK);
#pragma unroll
    for (int i = 0; i < kPasses; ++i) {
      if (whole || key0 + n0 + i * kRowsPerPass < ke) {
        cp_async16(kd + i * kRowsPerPass * L::kRowBytes, kp + (int64_t)(i * kRowsPerPass) * p.sk_[2]);
        cp_async16(vd + i * kRowsPerPass * L::kRowBytes, vp + (int64_t)(i * kRowsPerPass) * p.sv_[2]);
      } else {
        *reinterpret_cast<uint4*>(kd + i * kRowsPerPass * L::kRowBytes) = make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(vd + i * kRowsPerPass * L::kRowBytes) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    cp_async_commit();
  };
  if (n_chunks > 0) load_chunk(0, 0);

  // q as A fragments: rows g and g + 8, columns 16ks + 2t (+1) and
  // 16ks + 8 + 2t (+1); raw 16-bit pairs, low half = lower column.
  uint32_t qa[D / 16][4];
  {
    const uint16_t* qg = static_cast<const uint16_t*>(p.q);
    auto qpair = [&](int r, int c) -> uint32_t {
      if (r >= R) return 0u;
      const int gg = (row0 + r) / p.Sq, s = (row0 + r) - gg * p.Sq;
      const uint16_t* base = qg + (int64_t)b * p.sq_[0] + (int64_t)(hkv * p.G + gg) * p.sq_[1] + (int64_t)s * p.sq_[2];
      return (uint32_t)base[(int64_t)c * p.sq_[3]] | ((uint32_t)base[(int64_t)(c + 1) * p.sq_[3]] << 16);
    };
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      qa[ks][0] = qpair(g, 16 * ks + 2 * t);
      qa[ks][1] = qpair(g + 8, 16 * ks + 2 * t);
      qa[ks][2] = qpair(g, 16 * ks + 8 + 2 * t);
      qa[ks][3] = qpair(g + 8, 16 * ks + 8 + 2 * t);
    }
  }
  if (tid < kMaxRows) {
    row_m[tid] = neg_inf();
    row_l[tid] = 0.f;
    row_a[tid] = 1.f;
  }
  // Rows R..15 keep P = 0 (the softmax writes only rows < R).
  for (int idx = tid; idx < kMaxRows * kP16Row; idx += kDecThreads) p16[idx] = 0u;

  // Chunks whose 64 keys every row of the KV head keeps (all but the edges
  // of the causal / window range, without documents or a block mask) skip
  // the per-element mask and position arithmetic in the S phase.
  const KeptRange kept = kept_keys(p, 0, p.Sq, kChunk, false);
  const bool may_skip = p.doc_lo == nullptr && p.blk == nullptr;

  const int col0 = warp * (D / 8);  // this warp's O columns in P·V
  float o[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;

  // Three barriers per chunk. The one at the top also means every warp has
  // finished the previous chunk (its P·V read the other K/V slot and the P
  // tile), so the next chunk's loads and this chunk's S may overwrite them.
  for (int c = 0; c < n_chunks; ++c) {
    const int stage = c & 1;
    cp_async_wait<0>();
    __syncthreads();  // chunk c (and, at c = 0, the row state and P tile) visible
    if (c + 1 < n_chunks) load_chunk(c + 1, stage ^ 1);

    // S for keys [8w, 8w + 8) of the chunk, in two independent MMA chains.
    {
      // B fragments of keys [8w, 8w + 8) for two k-steps with one
      // ldmatrix: lanes 8m..8m+7 address key 8w + (lane & 7) at columns
      // 16ks + 8m, so fragment m is b_m.
      const uint32_t krow = sm100::smem_u32(smem + L::kOffK + stage * L::kTileBytes +
                                            (8 * warp + (lane & 7)) * L::kRowBytes) + 16u * (lane >> 3);
      float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < D / 16; ks += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(krow + 32u * ks, b0, b1, b2, b3);
        mma16816<BF16>(acc, qa[ks], b0, b1);
        mma16816<BF16>(acc2, qa[ks + 1], b2, b3);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[e] += acc2[e];
      const int key0 = kb + c * kChunk;
      const bool full = may_skip && key0 + kChunk <= ke && kept.has(key0);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = g + 8 * (e >> 1);
        const int n = 8 * warp + 2 * t + (e & 1);
        if (PLAIN && full) {
          if (r < R) ps[r * kPRow + n] = acc[e] * sl2;
        } else if (r < R) {
          const int key = kb + c * kChunk + n;
          const int gg = (row0 + r) / p.Sq, s = (row0 + r) - gg * p.Sq;
          const int64_t gi = (int64_t)s + p.q_off, gj = (int64_t)key + p.k_off;
          const bool keep = key < ke && keep_elem(p, b, hkv * p.G + gg, gi, gj);
          float x;
          if (PLAIN) {
            x = acc[e] * sl2;
          } else {
            const float slope = p.alibi ? p.alibi[hkv * p.G + gg] : 0.f;
            x = transform_logit(acc[e], p.scale, p.soft_cap, slope, gi, gj, nullptr) * kLog2e;
          }
          ps[r * kPRow + n] = keep ? x : neg_inf();
        }
      }
    }
    __syncthreads();

    // Online softmax: one warp per row, two keys per lane.
    for (int r = warp; r < R; r += kDecThreads / 32) {
      const float2 x = *reinterpret_cast<const float2*>(ps + r * kPRow + 2 * lane);
      const float mx = warp_max(fmaxf(x.x, x.y));
      const float m_old = row_m[r];
      const float m_new = fmaxf(m_old, mx);
      const float m_use = (m_new == neg_inf()) ? 0.f : m_new;
      const float p0 = fast_ex2(x.x - m_use), p1 = fast_ex2(x.y - m_use);
      p16[r * kP16Row + lane] = BF16 ? sm100::pack_bf16(p0, p1) : sm100::pack_f16(p0, p1);
      const float sum = warp_sum(p0 + p1);
      if (lane == 0) {
        const float alpha = fast_ex2(m_old - m_use);
        row_a[r] = alpha;
        row_l[r] = row_l[r] * alpha + sum;
        row_m[r] = m_new;
      }
    }
    __syncthreads();

    // O = O·alpha + P·V for this warp's columns.
    {
      const float a_lo = row_a[g], a_hi = row_a[g + 8];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        o[nt][0] *= a_lo;
        o[nt][1] *= a_lo;
        o[nt][2] *= a_hi;
        o[nt][3] *= a_hi;
      }
      const uint32_t vtile = sm100::smem_u32(smem + L::kOffV + stage * L::kTileBytes);
#pragma unroll
      for (int kk = 0; kk < kChunk / 16; ++kk) {
        // A fragments: P of rows g, g + 8 at keys 16kk + 2t (+1) and
        // 16kk + 8 + 2t (+1), packed by the softmax.
        uint32_t pa[4];
        pa[0] = p16[g * kP16Row + 8 * kk + t];
        pa[1] = p16[(g + 8) * kP16Row + 8 * kk + t];
        pa[2] = p16[g * kP16Row + 8 * kk + 4 + t];
        pa[3] = p16[(g + 8) * kP16Row + 8 * kk + 4 + t];
        // B fragments: keys 16kk + (lane & 15), columns col0 + 8nt (+8 for
        // the upper lanes), transposed on the way in.
        const uint32_t rowaddr = vtile + (uint32_t)((16 * kk + (lane & 15)) * L::kRowBytes);
        if constexpr (NT == 1) {
          uint32_t b0, b1;
          ldsm_x2_trans(rowaddr + (uint32_t)(col0 * 2), b0, b1);
          mma16816<BF16>(o[0], pa, b0, b1);
        } else {
#pragma unroll
          for (int nt = 0; nt < NT; nt += 2) {
            uint32_t b0, b1, b2, b3;
            ldsm_x4_trans(rowaddr + (uint32_t)((col0 + 8 * nt + 8 * (lane >> 4)) * 2), b0, b1, b2, b3);
            mma16816<BF16>(o[nt], pa, b0, b1);
            mma16816<BF16>(o[nt + 1], pa, b2, b3);
          }
        }
      }
    }
  }

  // The split's normalised O and LSE.
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = g + 8 * h;
    if (r < R) {
      const int gg = (row0 + r) / p.Sq, s = (row0 + r) - gg * p.Sq;
      const int64_t row = ((int64_t)b * p.Hq + hkv * p.G + gg) * p.Sq + s;
      const float l = row_l[r];
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
      float* dst = part_o + (row * n_split + split) * D + col0 + 2 * t;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        *reinterpret_cast<float2*>(dst + 8 * nt) = make_float2(o[nt][2 * h] * inv, o[nt][2 * h + 1] * inv);
    }
  }
  if (tid < R) {
    const int gg = (row0 + tid) / p.Sq, s = (row0 + tid) - gg * p.Sq;
    const int64_t row = ((int64_t)b * p.Hq + hkv * p.G + gg) * p.Sq + s;
    const float l = row_l[tid];
    part_lse[row * n_split + split] = (l > 0.f) ? (row_m[tid] + __log2f(l)) * kLn2 : neg_inf();
  }
}

// One block per row: lse = log Σ_s exp(lse_s), O = Σ_s exp(lse_s - lse) O_s
// (the reduce of npu_flash_attention.py:255-293, over the splits that exist).
// The split weights are formed once in shared memory; each thread then sums
// its columns over the splits (coalesced reads of the partial rows).
constexpr int kMergeThreads = 128;
constexpr int kMaxSplits = 256;

template <typename T>
__global__ void __launch_bounds__(kMergeThreads)
    decode_merge_kernel(const Params p, int n_split, const float* __restrict__ part_o,
                        const float* __restrict__ part_lse) {
  __shared__ float w[kMaxSplits];
  __shared__ float red[kMergeThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row = blockIdx.x;
  const int s = (int)(row % p.Sq);
  const int hq = (int)((row / p.Sq) % p.Hq);
  const int b = (int)(row / ((int64_t)p.Sq * p.Hq));
  const float* lr = part_lse + row * n_split;
  float m = neg_inf();
  for (int i = tid; i < n_split; i += kMergeThreads) m = fmaxf(m, lr[i]);
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int i = 1; i < kMergeThreads / 32; ++i) m = fmaxf(m, red[i]);
  __syncthreads();
  const float m_use = (m == neg_inf()) ? 0.f : m;
  float wsum = 0.f;
  for (int i = tid; i < n_split; i += kMergeThreads) {
    const float wi = fast_ex2((lr[i] - m_use) * kLog2e);
    w[i] = wi;
    wsum += wi;
  }
  wsum = warp_sum(wsum);
  if (lane == 0) red[warp] = wsum;
  __syncthreads();
  wsum = 0.f;
#pragma unroll
  for (int i = 0; i < kMergeThreads / 32; ++i) wsum += red[i];
  const float inv = (wsum > 0.f) ? 1.f / wsum : 0.f;
  T* og = static_cast<T*>(p.o);
  const int64_t obase = (int64_t)b * p.so_[0] + (int64_t)hq * p.so_[1] + (int64_t)s * p.so_[2];
  const float* po = part_o + row * n_split * p.D;
  for (int d = tid; d < p.D; d += kMergeThreads) {
    float acc = 0.f;
    for (int i = 0; i < n_split; ++i) acc = fmaf(w[i], po[(int64_t)i * p.D + d], acc);
    og[obase + (int64_t)d * p.so_[3]] = from_f32<T>(acc * inv);
  }
  if (tid == 0) p.lse[row] = (wsum > 0.f) ? m + logf(wsum) : neg_inf();
}

// BFA_FWD_DECODE=0 turns the path off (the regular forward runs instead).
bool decode_enabled() {
  const char* e = std::getenv("BFA_FWD_DECODE");
  return !(e && std::strcmp(e, "0") == 0);
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

// Launch plan of one decoding call: kernel, split count and the size of the
// partial results, computed the same way by bfa_fwd_workspace_bytes (to size
// the caller's workspace) and by the launch.
struct DecodePlan {
  void (*kern)(const Params, int, int, int, float*, float*);
  int smem_bytes;
  int klo, n_split, split_len, kv_heads;
  size_t o_bytes, l_bytes;
};

template <typename T, int D>
bool plan_decode(const Params& p, DecodePlan* pl) {
  using L = DecLayout<T, D>;
  {
    // key_range on the host: same arithmetic as the device helper.
    int64_t l = 0, h = p.Sk;
    const int64_t i_first = p.q_off, i_last = (int64_t)(p.Sq - 1) + p.q_off;
    if (p.causal) h = std::min<int64_t>(h, i_last - p.k_off + 1);
    if (p.window > 0) l = std::max<int64_t>(l, i_first - p.window - p.k_off);
    if (h < l) h = l;
    l = std::max<int64_t>(l, 0);
    h = std::max<int64_t>(h, 0);
    pl->klo = (int)l;
    pl->n_split = (int)(h - l);  // visible keys, replaced below
  }
  const bool plain = !(p.soft_cap > 0.f) && p.alibi == nullptr;
  const int n_rg = (p.G * p.Sq + kMaxRows - 1) / kMaxRows;  // row groups of <= 16 rows
  const int R = std::min(p.G * p.Sq, kMaxRows);             // rows of the largest group
  using Kern = void (*)(const Params, int, int, int, float*, float*);
  Kern kern;
  int smem_bytes;
  if constexpr (sizeof(T) == 2) {
    kern = plain ? decode_mma_kernel<T, D, true> : decode_mma_kernel<T, D, false>;
    smem_bytes = DecLayoutM<T, D>::kSmemBytes;
  } else {
    auto pick = [&](auto rb) -> Kern {
      constexpr int RB = decltype(rb)::value;
      return plain ? decode_split_kernel<T, D, RB, true> : decode_split_kernel<T, D, RB, false>;
    };
    kern = R <= 4 ? pick(std::integral_constant<int, 4>{})
                  : R <= 8 ? pick(std::integral_constant<int, 8>{}) : pick(std::integral_constant<int, 16>{});
    smem_bytes = L::kSmemBytes;
  }
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kDecThreads, smem_bytes) != cudaSuccess ||
      per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }

  const int kv_heads = p.B * p.Hkv * n_rg;  // (KV head, row group) pairs
  const int vis = pl->n_split;
  // One wave: as many splits as fill the resident CTA slots, each split a
  // long run of keys (the per-CTA start-up, pipeline fill and merge input grow
  // with the split count); two waves when one fills under 3/4 of the slots.
  // At least four 64-key chunks per split. (Same-box sweep on four decode
  // shapes: this beats two, four and eight waves by 0-30%.)
  const int slots = per_sm * sm_count();
  int n_split = std::max(1, slots / kv_heads);
  if (4 * kv_heads * n_split < 3 * slots) n_split = std::max(1, 2 * slots / kv_heads);
  n_split = std::max(1, std::min(n_split, std::min(kMaxSplits, (vis + 4 * kChunk - 1) / (4 * kChunk))));
  const int split_len = std::max(kChunk, (vis + n_split - 1) / n_split);
  n_split = std::max(1, (vis + split_len - 1) / split_len);

  const int64_t rows = (int64_t)p.B * p.Hq * p.Sq;
  pl->kern = kern;
  pl->smem_bytes = smem_bytes;
  pl->n_split = n_split;
  pl->split_len = split_len;
  pl->kv_heads = kv_heads;
  pl->o_bytes = (size_t)rows * n_split * D * sizeof(float);
  pl->l_bytes = (size_t)rows * n_split * sizeof(float);
  return true;
}

// The partial O (fp32 [rows][splits][D]) and LSE (fp32 [rows][splits]) live
// in the caller's workspace; -1 (the caller runs the regular forward) when it
// is missing or too small.
template <typename T, int D>
int launch_decode(const Params& p, void* ws, size_t ws_bytes, cudaStream_t st) {
  DecodePlan pl;
  if (!plan_decode<T, D>(p, &pl)) return cuda_fail("decode plan (device query)", cudaSuccess);
  if (!ws || ((uintptr_t)ws & 255u) != 0 || ws_bytes < pl.o_bytes + pl.l_bytes) return -1;
  float* part_o = static_cast<float*>(ws);
  float* part_lse = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + pl.o_bytes);
  const int64_t rows = (int64_t)p.B * p.Hq * p.Sq;
  pl.kern<<<(unsigned)(pl.kv_heads * pl.n_split), kDecThreads, pl.smem_bytes, st>>>(p, pl.n_split, pl.klo,
                                                                                    pl.split_len, part_o,
                                                                                    part_lse);
  note_launch();
  cudaError_t err = cudaGetLastError();
  if (err == cudaSuccess) {
    decode_merge_kernel<T><<<(unsigned)rows, kMergeThreads, 0, st>>>(p, pl.n_split, part_o, part_lse);
    note_launch();
    err = cudaGetLastError();
  }
  return err == cudaSuccess ? BFA_OK : cuda_fail("decode kernels launch", err);
}

template <typename T, int D>
size_t decode_bytes(const Params& p) {
  DecodePlan pl;
  if (!plan_decode<T, D>(p, &pl)) return 0;
  return pl.o_bytes + pl.l_bytes;
}

template <typename T>
int dispatch_d(const Params& p, void* ws, size_t ws_bytes, cudaStream_t st) {
  switch (p.D) {
    case 64: return launch_decode<T, 64>(p, ws, ws_bytes, st);
    case 128: return launch_decode<T, 128>(p, ws, ws_bytes, st);
    case 256:
      // fp32 rows of 256 do not fit two double-buffered 64-key K/V tiles.
      if constexpr (sizeof(T) == 2) return launch_decode<T, 256>(p, ws, ws_bytes, st);
      return -1;
    default: return -1;
  }
}

template <typename T>
size_t bytes_d(const Params& p) {
  switch (p.D) {
    case 64: return decode_bytes<T, 64>(p);
    case 128: return decode_bytes<T, 128>(p);
    case 256:
      if constexpr (sizeof(T) == 2) return decode_bytes<T, 256>(p);
      return 0;
    default: return 0;
  }
}

// The shape part of decode_eligible (no pointers or strides involved).
bool decode_shape_ok(const Params& p, int dtype) {
  if (!decode_enabled()) return false;
  if (dtype != BFA_DTYPE_BF16 && dtype != BFA_DTYPE_F16 && dtype != BFA_DTYPE_F32) return false;
  if (p.D != 64 && p.D != 128 && !(p.D == 256 && dtype != BFA_DTYPE_F32)) return false;
  return !(p.G * p.Sq > kMaxRowsTotal || p.Sq < 1 || p.Sk < 1 || p.B < 1 || p.Hkv < 1);
}

}  // namespace

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

bool decode_eligible(const Params& p, int dtype) {
  if (!decode_shape_ok(p, dtype)) return false;
  // K/V rows are copied in 16-byte pieces: unit stride along D, 16-byte
  // aligned bases and row / head / batch strides.
  const int64_t es = dtype == BFA_DTYPE_F32 ? 4 : 2;
  if (p.sk_[3] != 1 || p.sv_[3] != 1 || !aligned16(p.k) || !aligned16(p.v)) return false;
  for (int i = 0; i < 3; ++i)
    if ((p.sk_[i] * es) % 16 != 0 || (p.sv_[i] * es) % 16 != 0) return false;
  return true;
}

size_t decode_workspace_bytes(const Params& p, int dtype) {
  if (!decode_shape_ok(p, dtype)) return 0;
  size_t n = 0;
  switch (dtype) {
    case BFA_DTYPE_BF16: n = bytes_d<__nv_bfloat16>(p); break;
    case BFA_DTYPE_F16: n = bytes_d<__half>(p); break;
    case BFA_DTYPE_F32: n = bytes_d<float>(p); break;
    default: return 0;
  }
  return n ? (n + 255) / 256 * 256 : 0;
}

int decode_fwd(const Params& p, int dtype, void* ws, size_t ws_bytes, cudaStream_t st) {
  switch (dtype) {
    case BFA_DTYPE_BF16: return dispatch_d<__nv_bfloat16>(p, ws, ws_bytes, st);
    case BFA_DTYPE_F16: return dispatch_d<__half>(p, ws, ws_bytes, st);
    case BFA_DTYPE_F32: return dispatch_d<float>(p, ws, ws_bytes, st);
    default: return -1;
  }
}

}  // namespace bfa
