// merge.cu -- LSE merge of a partial attention result into a running one.
//
// lse' = logaddexp(lse_a, lse_p);  o' = o_a·e^(lse_a−lse') + o_p·e^(lse_p−lse').
// The forward merges its own result this way when called with
// bfa_fwd_args.accumulate (the context-parallel ring's path); this entry
// point merges two results already in memory. The reference has the same
// idea in its unused split-KV reduce kernel (npu_flash_attention.py:255-293).
#include <cuda_runtime.h>

#include "bfa_internal.h"

namespace bfa {
namespace {

template <typename TA, typename TP>
__global__ void __launch_bounds__(256) merge_kernel(int B, int H, int S, int D, bfa_tensor oa,
                                                     float* lse_a, bfa_tensor op,
                                                     const float* lse_p) {
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= (int64_t)B * H * S) return;
  const int i = (int)(row % S), h = (int)((row / S) % H), b = (int)(row / ((int64_t)S * H));
  const MergeWeights w = merge_weights(lse_a[row], lse_p[row]);
  const float wa = w.wa, wp = w.wp, ln = w.ln;
  TA* A = (TA*)oa.data + b * oa.stride[0] + h * oa.stride[1] + i * oa.stride[2];
  const TP* P = (const TP*)op.data + b * op.stride[0] + h * op.stride[1] + i * op.stride[2];
  for (int d = lane; d < D; d += 32) {
    const float va = (wa != 0.f) ? to_f32<TA>(A[d * oa.stride[3]]) * wa : 0.f;
    const float vp = (wp != 0.f) ? to_f32<TP>(P[d * op.stride[3]]) * wp : 0.f;
    A[d * oa.stride[3]] = from_f32<TA>(va + vp);
  }
  __syncwarp();
  if (lane == 0) lse_a[row] = ln;
}

template <typename TA>
int launch_a(int B, int H, int S, int D, const bfa_tensor& oa, float* la, const bfa_tensor& op,
             int pdt, const float* lp, cudaStream_t st) {
  const int64_t rows = (int64_t)B * H * S;
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  switch (pdt) {
    case BFA_DTYPE_F32: merge_kernel<TA, float><<<blocks, 256, 0, st>>>(B, H, S, D, oa, la, op, lp); break;
    case BFA_DTYPE_F16: merge_kernel<TA, __half><<<blocks, 256, 0, st>>>(B, H, S, D, oa, la, op, lp); break;
    case BFA_DTYPE_BF16: merge_kernel<TA, __nv_bfloat16><<<blocks, 256, 0, st>>>(B, H, S, D, oa, la, op, lp); break;
    default: return BFA_ERR_UNSUPPORTED;
  }
  note_launch();
  return launch_status("merge kernel launch");
}

}  // namespace

int launch_merge(int B, int H, int S, int D, const bfa_tensor& oa, int adt, float* lse_a,
                 const bfa_tensor& op, int pdt, const float* lse_p, cudaStream_t st) {
  if ((int64_t)B * H * S == 0) return BFA_OK;
  switch (adt) {
    case BFA_DTYPE_F32: return launch_a<float>(B, H, S, D, oa, lse_a, op, pdt, lse_p, st);
    case BFA_DTYPE_F16: return launch_a<__half>(B, H, S, D, oa, lse_a, op, pdt, lse_p, st);
    case BFA_DTYPE_BF16: return launch_a<__nv_bfloat16>(B, H, S, D, oa, lse_a, op, pdt, lse_p, st);
  }
  return BFA_ERR_UNSUPPORTED;
}

}  // namespace bfa
