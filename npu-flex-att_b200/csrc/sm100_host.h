// sm100_host.h -- host helpers for the TMA / tcgen05 kernels.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace bfa {

struct Tmaps4 {
  CUtensorMap m[4];
};

// True when the current device is a B200-class part (compute capability 10.0).
bool device_is_sm100();

// True when a [B, H, S, D] tensor with these element strides can be read by
// TMA: unit innermost stride, 16-byte aligned base and outer strides.
bool tma_layout_ok(const void* ptr, const int64_t* stride, int elem_bytes);

// 4-D tensor map over a [B, H, S, D] tensor (fp16/bf16, or fp32 for the
// backward's accumulate mode): box = 128 bytes of D (64 16-bit or 32 fp32
// elements, 128-byte swizzle) x `box_rows` rows of S x 1 x 1. Rows past S
// read as zero and are not written. Returns false if the driver rejects it.
bool make_tmap_bhsd(CUtensorMap* map, const void* ptr, int dtype, int D, int S, int H, int B,
                    const int64_t* stride, int box_rows);

}  // namespace bfa
