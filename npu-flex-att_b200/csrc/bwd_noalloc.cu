// bwd_noalloc.cu -- bfa_bwd_noalloc: the attention backward for callers that
// cannot allocate device memory.
//
// bfa_bwd needs a caller-provided workspace for Δ = rowsum(O∘dO) (fp32, one
// value per query row). Some callers cannot provide one: a plugin inside a
// host framework that owns every device allocation and hands the plugin only
// its input and output buffers, or a caller whose hot path must not call
// cudaMalloc (it can synchronise the device). For them this entry point keeps
// Δ in a file-scope device array of fixed size instead.
//
// Limits and sharing:
//  * The array holds the backward's row statistics (Δ and lse·log2 e, fp32)
//    for kMaxRows = 2^21 query rows, counting each head's rows rounded up to
//    a multiple of 64 (batch * heads_q * ceil(seqlen_q / 64) * 64): 16 MiB
//    (+512 bytes of alignment slack). Larger problems are rejected with
//    BFA_ERR_SCRATCH_LIMIT.
//  * Every GPU that loads this library holds the array until process exit.
//  * All calls share the one array per device and it keeps the last call's
//    contents. Calls whose work overlaps on the GPU (different streams, or
//    different host threads on the same device) race on it; serialise them.
//    Each call computes Δ itself before reading it (a `phases` mask without
//    BFA_BWD_PHASE_DELTA is rejected: the array could hold another call's Δ),
//    so nothing needs clearing.
//  * The first call on a device looks up the array's device address
//    (cudaGetSymbolAddress, with that device current) and caches it; make that
//    first call before any stream capture. The cached address is kept for the
//    life of the process: do not use the library across a cudaDeviceReset.
//  * Nothing here calls cudaMalloc, cudaFree or an allocating library routine.
#include <cuda_runtime.h>

#include <mutex>

#include "bfa.h"
#include "bfa_internal.h"

namespace {

constexpr int64_t kMaxRows = int64_t(1) << 21;
constexpr size_t kScratchFloats = 2 * (size_t)kMaxRows + 128;  // + 512 B: bfa_bwd's workspace slack
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_delta_scratch[kScratchFloats];

std::mutex g_mu;
float* g_addr[kMaxDevices] = {};

// Device address of g_delta_scratch on the current device (looked up once).
int scratch_address(float** out) {
  int dev = 0;
  if (cudaError_t e = cudaGetDevice(&dev)) return bfa::cuda_fail("cudaGetDevice", e);
  if (dev < 0 || dev >= kMaxDevices) return bfa::cuda_fail("bfa_bwd_noalloc: device index out of range", cudaSuccess);
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_addr[dev]) {
    void* ptr = nullptr;
    if (cudaError_t e = cudaGetSymbolAddress(&ptr, g_delta_scratch)) return bfa::cuda_fail("cudaGetSymbolAddress", e);
    if (!ptr) return bfa::cuda_fail("cudaGetSymbolAddress", cudaSuccess);
    g_addr[dev] = static_cast<float*>(ptr);
  }
  *out = g_addr[dev];
  return BFA_OK;
}

}  // namespace

extern "C" int bfa_bwd_noalloc(const bfa_problem* problem, const bfa_bwd_args* args,
                               void* stream) {
  if (!problem) return BFA_ERR_INVALID_ARGUMENT;
  if (problem->batch >= 0 && problem->heads_q >= 0 && problem->seqlen_q >= 0) {
    const int64_t rows =
        (int64_t)problem->batch * problem->heads_q * (((int64_t)problem->seqlen_q + 63) / 64 * 64);
    if (rows > kMaxRows) return BFA_ERR_SCRATCH_LIMIT;
  }
  if (!args) return BFA_ERR_INVALID_ARGUMENT;
  if (args->phases != 0 && !(args->phases & BFA_BWD_PHASE_DELTA)) return BFA_ERR_INVALID_ARGUMENT;
  float* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != BFA_OK) return rc;
  return bfa_bwd(problem, args, scratch, kScratchFloats * sizeof(float), stream);
}
