// bfa_internal.h -- host-side declarations shared by the library's .cu files.
#pragma once

#include <cuda_runtime.h>

#include "bfa_common.cuh"

namespace bfa {

// Generic CUDA-core path (simt_attention.cu).
int simt_fwd(const Params& p, int dtype, cudaStream_t st);
int simt_bwd(const Params& p, int dtype, cudaStream_t st);  // needs p.delta filled
int launch_delta(const Params& p, int dtype, cudaStream_t st);

// tcgen05 / TMA path (sm100_fwd.cu, sm100_bwd.cu). `*_eligible` say whether
// the fast path takes this problem; the launchers return a bfa_status.
bool sm100_fwd_eligible(const Params& p, int dtype);
int sm100_fwd(const Params& p, int dtype, cudaStream_t st);
int sm100_fwd256(const Params& p, int dtype, cudaStream_t st);  // head_dim 256 (sm100_fwd256.cu)
bool sm100_bwd_eligible(const Params& p, int dtype);
int sm100_bwd(const Params& p, int dtype, cudaStream_t st);
int sm100_bwd256(const Params& p, int dtype, cudaStream_t st);  // head_dim 256 (sm100_bwd256.cu)
// Whether sm100_bwd's dQ kernel can form Δ itself (Params::fuse_delta): the
// tcgen05 path (head dims 64, 128, 256) with a TMA-compatible O.
// BFA_BWD_FUSE_DELTA=0 turns it off.
bool sm100_bwd_fuses_delta(const Params& p, int dtype);
// Split-KV decoding forward (decode.cu): the G q-heads of a KV head have at
// most 64 query rows. Its partial results live in a caller workspace of
// decode_workspace_bytes() bytes (0: the problem never takes this path).
// decode_fwd returns a bfa_status, or -1 when it could not run (no or too
// small a workspace; the caller falls back to the regular forward).
bool decode_eligible(const Params& p, int dtype);
size_t decode_workspace_bytes(const Params& p, int dtype);
int decode_fwd(const Params& p, int dtype, void* ws, size_t ws_bytes, cudaStream_t st);

// Multiprocessors of the current device (cached per device).
int sm_count();

// Partial-result merge (merge.cu).
int launch_merge(int B, int H, int S, int D, const bfa_tensor& oa, int adt, float* lse_a,
                 const bfa_tensor& op, int pdt, const float* lse_p, cudaStream_t st);

// Count one kernel launch (bfa_launch_count).
void note_launch();

// Record `what` and the CUDA error for bfa_last_error() and return
// BFA_ERR_CUDA. launch_status() does so for the last launch's error, if any.
int cuda_fail(const char* what, cudaError_t e);
int launch_status(const char* what);

// Bytes of one element of a bfa_dtype (0 when invalid).
inline int dtype_bytes(int dt) {
  return dt == BFA_DTYPE_F32 ? 4 : (dt == BFA_DTYPE_F16 || dt == BFA_DTYPE_BF16) ? 2 : 0;
}

}  // namespace bfa
