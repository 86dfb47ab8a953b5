// sm100_bwd_common.cuh -- device helpers shared by the tcgen05 backward kernels
// (sm100_bwd.cu: head_dim 64 / 128; sm100_bwd256.cu: head_dim 256).
#pragma once

#include <stdint.h>

#include "bfa_common.cuh"
#include "sm100_ptx.cuh"

namespace bfa {
namespace bwd {

using namespace sm100;

constexpr int kThreads = 384;  // warps 0-3: TMA / MMA / TMEM alloc / MMA (D <= 128; idle at D = 256); 4-11: elementwise
constexpr int kRows = 128;  // TMEM lanes / rows owned by the elementwise warps
constexpr int kInner = 64;  // columns of one S/dP step

__device__ __forceinline__ bool tile_full(const Params& p, int r0, int r1, int c0, int c1) {
  if (r1 > p.Sq || c1 > p.Sk) return false;
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

// The two 16-bit values of a packed word (low half first) as floats.
template <bool BF16>
__device__ __forceinline__ float2 unpack2(uint32_t w) {
  if (BF16) return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

// Logit in the base-2 domain: (cap·tanh(s·scale/cap) or s·scale)·log2(e).
// `t` receives tanh(s·scale/cap) for the soft-cap chain. TIER (cap_tier)
// selects tanh_tiny (every |s·scale/cap| of the warp's step is <= 1/8, 2),
// tanh_small (<= 1/2, 1) or tanh_any (0).
template <bool CAP, int TIER = 0>
__device__ __forceinline__ float logit2(float raw, float sl2, float cap_in, float cap_out, float* t) {
  if (CAP) {
    const float u = raw * cap_in;
    const float th = TIER == 2 ? tanh_tiny(u) : TIER == 1 ? tanh_small(u) : tanh_any(u);
    *t = th;
    return cap_out * th;
  }
  *t = 0.f;
  return raw * sl2;
}

// Read a TMEM row of D fp32 columns, convert, and write it into a staging
// area of D/64 swizzled sub-tiles of 128 rows (for a TMA store).
template <int D, bool BF16>
__device__ __forceinline__ void stage_tmem_row(uint32_t taddr, uint8_t* stage, int row, bool zero) {
#pragma unroll 1
  for (int c = 0; c < D / 32; ++c) {
    uint32_t r[32];
    if (!zero) {
      tmem_ld32(taddr + 32 * c, r);
      tmem_ld_wait();
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) r[i] = 0u;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 w;
      w.x = pack2<BF16>(__uint_as_float(r[8 * q + 0]), __uint_as_float(r[8 * q + 1]));
      w.y = pack2<BF16>(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3]));
      w.z = pack2<BF16>(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5]));
      w.w = pack2<BF16>(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7]));
      const int col = 32 * c + 8 * q;
      *reinterpret_cast<uint4*>(stage + (col >> 6) * (kRows * 128) + sw128_offset(row, (col & 63) >> 3)) = w;
    }
  }
}

// Accumulate mode: the same row in fp32, D/32 swizzled sub-tiles of 128 rows
// x 32 floats, for a TMA reduce-add into the caller's fp32 gradient.
template <int D>
__device__ __forceinline__ void stage_tmem_row_f32(uint32_t taddr, uint8_t* stage, int row) {
#pragma unroll 1
  for (int c = 0; c < D / 32; ++c) {
    uint32_t r[32];
    tmem_ld32(taddr + 32 * c, r);
    tmem_ld_wait();
#pragma unroll
    for (int q = 0; q < 8; ++q)
      *reinterpret_cast<uint4*>(stage + c * (kRows * 128) + sw128_offset(row, q)) =
          make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
  }
}

}  // namespace bwd
}  // namespace bfa
