// decode.cu -- split-KV flash-decoding forward: few query rows per KV head,
// long key sequence.
//
// The reference carries a split-KV forward and its reduce for short Q_LEN
// (npu_flash_attention.py:171-293: flash_attn_fwd_split_kv_kernel writes a
// normalised partial O and a partial LSE per key split, and
// flash_attn_fwd_reduce_kernel merges them with an LSE-weighted sum). There it
// is never launched (and fixes B = 1). This is the working B200 version of that
// path, chosen automatically by bfa_fwd when the G q-heads of a KV head
// together have at most kMaxRows query rows.
//
// Decode is HBM-bound: every K/V byte is used by only G·Sq rows. So:
//   - one CTA per (batch, KV head, key split) serves all G·Sq rows of that KV
//     head, so K/V cross HBM once however large G is;
//   - K/V stream through a cp.async double buffer in 64-key chunks (rows
//     padded by 16 bytes so the 16-byte shared-memory reads are conflict-free);
//   - S = q·k, the online softmax and P·V run on the CUDA cores in fp32: at
//     <= 16 rows they take less time per chunk than the chunk's HBM transfer;
//   - the keys are split into about eight CTAs per resident CTA slot (two
//     per SM), so the GPU stays full to the last wave, and a merge kernel
//     combines the splits' partial (O, LSE) per row.
// The math per row is the forward's: S·scale, cap, ALiBi, mask on absolute
// positions (q_off, k_off), base-2 online softmax, O = PV/l and
// LSE = m + ln(l) (natural log), -inf with O = 0 for a row that sees no key.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <cstring>
#include <type_traits>

#include "bfa_internal.h"

namespace bfa {
namespace {

constexpr int kDecThreads = 256;
constexpr int kChunk = 64;    // keys per pipeline stage
constexpr int kMaxRows = 16;  // G·Sq rows per CTA
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

// 16 bytes of T -> fp32 values.
template <typename T>
__device__ __forceinline__ void unpack16(const uint4& u, float* f);
template <>
__device__ __forceinline__ void unpack16<__nv_bfloat16>(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
template <>
__device__ __forceinline__ void unpack16<__half>(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
template <>
__device__ __forceinline__ void unpack16<float>(const uint4& u, float* f) {
  f[0] = __uint_as_float(u.x);
  f[1] = __uint_as_float(u.y);
  f[2] = __uint_as_float(u.z);
  f[3] = __uint_as_float(u.w);
}

// Two consecutive T at p -> fp32.
template <typename T>
__device__ __forceinline__ float2 load2(const uint8_t* p);
template <>
__device__ __forceinline__ float2 load2<__nv_bfloat16>(const uint8_t* p) {
  const uint32_t w = *reinterpret_cast<const uint32_t*>(p);
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <>
__device__ __forceinline__ float2 load2<__half>(const uint8_t* p) {
  return __half22float2(*reinterpret_cast<const __half2*>(p));
}
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
  const int R = p.G * p.Sq;
  const int split = (int)(blockIdx.x % n_split);
  const int bkv = (int)(blockIdx.x / n_split);
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
      const int g = r / p.Sq, s = r - g * p.Sq;
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
          const int g = r / p.Sq, s = r - g * p.Sq;
          const int64_t gi = (int64_t)s + p.q_off, gj = (int64_t)key + p.k_off;
          const bool keep = key < ke && keep_pair(gi, gj, p.causal, p.window);
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
      const int g = r / p.Sq, s = r - g * p.Sq;
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

// Library-private stream-ordered memory pool per device for the partials:
// it keeps up to kPoolKeep bytes between calls, so a steady stream of decode
// calls allocates without mapping new memory, and no process-wide pool
// setting is touched.
constexpr uint64_t kPoolKeep = 256ull << 20;

cudaMemPool_t decode_pool() {
  static std::mutex mu;
  static cudaMemPool_t pools[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!pools[dev]) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t pool = nullptr;
    if (cudaMemPoolCreate(&pool, &props) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    uint64_t keep = kPoolKeep;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    pools[dev] = pool;
  }
  return pools[dev];
}

// BFA_FWD_DECODE=0 turns the path off (the regular forward runs instead).
bool decode_enabled() {
  const char* e = std::getenv("BFA_FWD_DECODE");
  return !(e && std::strcmp(e, "0") == 0);
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

template <typename T, int D>
int launch_decode(const Params& p, cudaStream_t st) {
  using L = DecLayout<T, D>;
  int klo, khi;
  {
    // key_range on the host: same arithmetic as the device helper.
    int64_t l = 0, h = p.Sk;
    const int64_t i_first = p.q_off, i_last = (int64_t)(p.Sq - 1) + p.q_off;
    if (p.causal) h = std::min<int64_t>(h, i_last - p.k_off + 1);
    if (p.window > 0) l = std::max<int64_t>(l, i_first - p.window - p.k_off);
    if (h < l) h = l;
    l = std::max<int64_t>(l, 0);
    h = std::max<int64_t>(h, 0);
    klo = (int)l;
    khi = (int)h;
  }
  const int kv_heads = p.B * p.Hkv;
  const int vis = khi - klo;
  // About eight CTAs per resident slot (two per SM), so that the last wave
  // is a small part of the run, and at least four 64-key chunks per split.
  int n_split = (16 * sm_count() + kv_heads - 1) / kv_heads;
  n_split = std::max(1, std::min(n_split, std::min(kMaxSplits, (vis + 4 * kChunk - 1) / (4 * kChunk))));
  const int split_len = std::max(kChunk, (vis + n_split - 1) / n_split);
  n_split = std::max(1, (vis + split_len - 1) / split_len);

  const int64_t rows = (int64_t)p.B * p.Hq * p.Sq;
  const size_t o_bytes = (size_t)rows * n_split * D * sizeof(float);
  const size_t l_bytes = (size_t)rows * n_split * sizeof(float);
  void* buf = nullptr;
  cudaMemPool_t pool = decode_pool();
  if (!pool || cudaMallocFromPoolAsync(&buf, o_bytes + l_bytes, pool, st) != cudaSuccess) {
    cudaGetLastError();
    return -1;  // caller falls back to the regular forward
  }
  float* part_o = static_cast<float*>(buf);
  float* part_lse = reinterpret_cast<float*>(static_cast<uint8_t*>(buf) + o_bytes);

  const bool plain = !(p.soft_cap > 0.f) && p.alibi == nullptr;
  const int R = p.G * p.Sq;
  auto pick = [&](auto rb) {
    constexpr int RB = decltype(rb)::value;
    return plain ? decode_split_kernel<T, D, RB, true> : decode_split_kernel<T, D, RB, false>;
  };
  auto kern = R <= 4 ? pick(std::integral_constant<int, 4>{})
                     : R <= 8 ? pick(std::integral_constant<int, 8>{}) : pick(std::integral_constant<int, 16>{});
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes);
  if (err == cudaSuccess) {
    kern<<<(unsigned)(kv_heads * n_split), kDecThreads, L::kSmemBytes, st>>>(p, n_split, klo, split_len, part_o,
                                                                             part_lse);
    note_launch();
    err = cudaGetLastError();
  }
  if (err == cudaSuccess) {
    decode_merge_kernel<T><<<(unsigned)rows, kMergeThreads, 0, st>>>(p, n_split, part_o, part_lse);
    note_launch();
    err = cudaGetLastError();
  }
  cudaFreeAsync(buf, st);
  return err == cudaSuccess ? BFA_OK : BFA_ERR_CUDA;
}

template <typename T>
int dispatch_d(const Params& p, cudaStream_t st) {
  switch (p.D) {
    case 64: return launch_decode<T, 64>(p, st);
    case 128: return launch_decode<T, 128>(p, st);
    case 256:
      // fp32 rows of 256 do not fit two double-buffered 64-key K/V tiles.
      if constexpr (sizeof(T) == 2) return launch_decode<T, 256>(p, st);
      return -1;
    default: return -1;
  }
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
  if (!decode_enabled()) return false;
  if (dtype != BFA_DTYPE_BF16 && dtype != BFA_DTYPE_F16 && dtype != BFA_DTYPE_F32) return false;
  if (p.D != 64 && p.D != 128 && !(p.D == 256 && dtype != BFA_DTYPE_F32)) return false;
  if (p.G * p.Sq > kMaxRows || p.Sq < 1 || p.Sk < 1 || p.B < 1 || p.Hkv < 1) return false;
  // K/V rows are copied in 16-byte pieces: unit stride along D, 16-byte
  // aligned bases and row / head / batch strides.
  const int64_t es = dtype == BFA_DTYPE_F32 ? 4 : 2;
  if (p.sk_[3] != 1 || p.sv_[3] != 1 || !aligned16(p.k) || !aligned16(p.v)) return false;
  for (int i = 0; i < 3; ++i)
    if ((p.sk_[i] * es) % 16 != 0 || (p.sv_[i] * es) % 16 != 0) return false;
  return true;
}

int decode_fwd(const Params& p, int dtype, cudaStream_t st) {
  switch (dtype) {
    case BFA_DTYPE_BF16: return dispatch_d<__nv_bfloat16>(p, st);
    case BFA_DTYPE_F16: return dispatch_d<__half>(p, st);
    case BFA_DTYPE_F32: return dispatch_d<float>(p, st);
    default: return -1;
  }
}

}  // namespace bfa
