// sm100_host.cu -- tensor-map encoding and device checks for the tcgen05 path.
//
// cuTensorMapEncodeTiled is fetched through cudaGetDriverEntryPoint, so the
// library does not link against libcuda directly.
#include <cstdio>
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "bfa.h"
#include "bfa_internal.h"
#include "sm100_host.h"

namespace bfa {
namespace {

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                              const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                              const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
  static std::once_flag once;
  static EncodeFn fn = nullptr;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(ptr);
  });
  return fn;
}

}  // namespace

bool device_is_sm100() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  static std::mutex mu;
  static int cached[64];
  static bool init = false;
  std::lock_guard<std::mutex> lock(mu);
  if (!init) {
    for (int i = 0; i < 64; ++i) cached[i] = -1;
    init = true;
  }
  if (dev < 0 || dev >= 64) return false;
  if (cached[dev] < 0) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cached[dev] = (major == 10 && minor == 0) ? 1 : 0;
  }
  return cached[dev] == 1;
}

bool tma_layout_ok(const void* ptr, const int64_t* stride, int elem_bytes) {
  if (((uintptr_t)ptr & 15u) != 0) return false;
  if (stride[3] != 1) return false;
  for (int i = 0; i < 3; ++i) {
    const int64_t bytes = stride[i] * elem_bytes;
    if (bytes <= 0 || (bytes & 15) != 0 || bytes >= ((int64_t)1 << 40)) return false;
  }
  return true;
}

// The tensor-map encoder is a driver call and needs the device's context
// current on the calling thread. The runtime makes it current lazily, on a
// thread's first runtime call that needs it, and a thread whose first CUDA
// work is this library's (PyTorch's autograd device threads, for instance,
// when every tensor they touch comes from the caching allocator) may not have
// made one yet: the encoder then fails with CUDA_ERROR_INVALID_CONTEXT.
// cudaSetDevice on the current device makes its primary context current;
// done once per thread and device.
static bool ensure_context() {
  thread_local unsigned long long done = 0;  // bit d: device d's context is current here
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  if (dev < 64 && (done >> dev) & 1ull) return true;
  if (cudaSetDevice(dev) != cudaSuccess) return false;
  if (dev < 64) done |= 1ull << dev;
  return true;
}

bool make_tmap_bhsd(CUtensorMap* map, const void* ptr, int dtype, int D, int S, int H, int B,
                    const int64_t* stride, int box_rows) {
  if (!ensure_context()) {
    cuda_fail("cudaSetDevice (making the device context current)", cudaGetLastError());
    return false;
  }
  EncodeFn fn = encode_fn();
  if (!fn) {
    cuda_fail("cuTensorMapEncodeTiled entry point", cudaSuccess);
    return false;
  }
  const int es = dtype == BFA_DTYPE_F32 ? 4 : 2;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t gstr[3] = {(cuuint64_t)(stride[2] * es), (cuuint64_t)(stride[1] * es),
                        (cuuint64_t)(stride[0] * es)};
  cuuint32_t box[4] = {(cuuint32_t)(128 / es), (cuuint32_t)box_rows, 1u, 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  const CUtensorMapDataType dt = dtype == BFA_DTYPE_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == BFA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                           : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  auto encode = [&] {
    return fn(map, dt, 4, const_cast<void*>(ptr), dims, gstr, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  };
  CUresult r = encode();
  if (r == CUDA_ERROR_INVALID_CONTEXT) {  // e.g. the context was reset since this thread's last call
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess) r = encode();
  }
  if (r != CUDA_SUCCESS) {
    char what[160];
    std::snprintf(what, sizeof(what),
                  "cuTensorMapEncodeTiled error %d (ptr %p, dims %d/%d/%d/%d, byte strides %lld/%lld/%lld, box rows %d)",
                  (int)r, ptr, D, S, H, B, (long long)gstr[0], (long long)gstr[1], (long long)gstr[2], box_rows);
    cuda_fail(what, cudaSuccess);
  }
  return r == CUDA_SUCCESS;
}

}  // namespace bfa
