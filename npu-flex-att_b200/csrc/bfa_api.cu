// bfa_api.cu -- the C ABI declared in include/bfa.h.
//
// Validation mirrors the reference host API (npu_flash_attention.py:617-626,
// :669-673): head dims must agree and Hq must be a multiple of Hkv. The fast
// tcgen05/TMA kernels take bf16/fp16 problems whose layout TMA can read; every
// other problem runs on the generic CUDA-core kernels. There is no CPU path.
#include <cstdio>
#include <cuda_runtime.h>

#include <atomic>
#include <climits>

#include "bfa.h"
#include "bfa_internal.h"

namespace bfa {
namespace {
std::atomic<uint64_t> g_launches{0};
}
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

namespace {
thread_local char g_last_error[192];
}

int cuda_fail(const char* what, cudaError_t e) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s: %s", what,
                e == cudaSuccess ? "failed" : cudaGetErrorName(e));
  return BFA_ERR_CUDA;
}

int launch_status(const char* what) {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? BFA_OK : cuda_fail(what, e);
}
}  // namespace bfa

namespace {

using bfa::Params;

int check_problem(const bfa_problem* pr) {
  if (!pr) return BFA_ERR_INVALID_ARGUMENT;
  if (pr->batch < 0 || pr->heads_q < 0 || pr->heads_kv <= 0 || pr->seqlen_q < 0 ||
      pr->seqlen_k < 0 || pr->sliding_window < 0 || pr->soft_cap < 0.f)
    return BFA_ERR_INVALID_ARGUMENT;
  // Query rows are padded to a multiple of 64 in int32 row pitches.
  if (pr->seqlen_q > INT32_MAX - 63) return BFA_ERR_INVALID_ARGUMENT;
  if ((pr->doc_start == nullptr) != (pr->doc_end == nullptr)) return BFA_ERR_INVALID_ARGUMENT;
  if (pr->heads_q % pr->heads_kv != 0) return BFA_ERR_SHAPE;
  if (pr->head_dim < 1 || pr->head_dim > 256) return BFA_ERR_UNSUPPORTED;
  if (bfa::dtype_bytes(pr->dtype) == 0) return BFA_ERR_UNSUPPORTED;
  return BFA_OK;
}

void copy_strides(int64_t* dst, const bfa_tensor& t) {
  for (int i = 0; i < 4; ++i) dst[i] = t.stride[i];
}

Params make_params(const bfa_problem* pr) {
  Params p{};
  p.B = pr->batch;
  p.Hq = pr->heads_q;
  p.Hkv = pr->heads_kv;
  p.G = pr->heads_q / pr->heads_kv;
  p.Sq = pr->seqlen_q;
  p.Sk = pr->seqlen_k;
  p.D = pr->head_dim;
  p.causal = pr->causal ? 1 : 0;
  p.window = pr->sliding_window;
  p.scale = pr->scale;
  p.soft_cap = pr->soft_cap;
  p.alibi = pr->alibi_slopes;
  p.q_off = pr->q_pos_offset;
  p.k_off = pr->k_pos_offset;
  p.doc_lo = pr->doc_start;
  p.doc_hi = pr->doc_end;
  p.blk = pr->block_mask;
  for (int i = 0; i < 3; ++i) p.blk_s[i] = pr->block_mask_stride[i];
  return p;
}

bool empty_q(const bfa_problem* pr) {
  return (int64_t)pr->batch * pr->heads_q * pr->seqlen_q == 0;
}

}  // namespace

extern "C" {

int bfa_abi_version(void) { return BFA_ABI_VERSION; }

uint64_t bfa_launch_count(void) { return bfa::g_launches.load(std::memory_order_relaxed); }

const char* bfa_last_error(void) { return bfa::g_last_error; }

const char* bfa_strerror(int status) {
  switch (status) {
    case BFA_OK: return "success";
    case BFA_ERR_INVALID_ARGUMENT: return "bfa: invalid argument (null pointer, negative size or flag)";
    case BFA_ERR_SHAPE: return "bfa: shape mismatch (head dims differ or Hq is not a multiple of Hkv)";
    case BFA_ERR_UNSUPPORTED: return "bfa: unsupported dtype or head_dim (need fp32/fp16/bf16, 1 <= D <= 256)";
    case BFA_ERR_WORKSPACE: return "bfa: workspace missing or smaller than bfa_bwd_workspace_bytes()";
    case BFA_ERR_CUDA: return "bfa: a CUDA runtime call or kernel launch failed";
    case BFA_ERR_DEVICE_TIMEOUT: return "bfa: a device-side wait timed out (pipeline stalled)";
    case BFA_ERR_SCRATCH_LIMIT:
      return "bfa: problem exceeds bfa_bwd_noalloc's static scratch "
             "(batch*heads_q*ceil(seqlen_q/64)*64 > 2097152)";
  }
  return "bfa: unknown status";
}

int bfa_fwd(const bfa_problem* pr, const bfa_fwd_args* a, void* stream) {
  int rc = check_problem(pr);
  if (rc) return rc;
  if (!a) return BFA_ERR_INVALID_ARGUMENT;
  if (empty_q(pr)) return BFA_OK;
  if (!a->q.data || !a->o.data || !a->lse || (pr->seqlen_k > 0 && (!a->k.data || !a->v.data)))
    return BFA_ERR_INVALID_ARGUMENT;
  Params p = make_params(pr);
  p.q = a->q.data; p.k = a->k.data; p.v = a->v.data; p.o = a->o.data;
  copy_strides(p.sq_, a->q); copy_strides(p.sk_, a->k);
  copy_strides(p.sv_, a->v); copy_strides(p.so_, a->o);
  p.lse = a->lse;
  p.status = a->status;
  p.timeout_ns = a->wait_timeout_ns > 0 ? (uint64_t)a->wait_timeout_ns : 1000000000ull;
  p.debug_flags = a->debug_flags;
  if (a->accumulate > 1) return BFA_ERR_INVALID_ARGUMENT;
  p.out_acc = a->accumulate;
  cudaStream_t st = (cudaStream_t)stream;
  // Few query rows per KV head (decoding): the split-KV path streams K/V once
  // per KV head across the whole GPU. The fault-injection flags exercise the
  // tcgen05 kernels' bounded waits, so they keep the regular path, and so
  // does a merging call (the decoding path writes its own output).
  if (p.debug_flags == 0 && !p.out_acc && a->workspace && bfa::decode_eligible(p, pr->dtype)) {
    const int rc = bfa::decode_fwd(p, pr->dtype, a->workspace, a->workspace_bytes, st);
    if (rc != -1) return rc;
  }
  if (bfa::sm100_fwd_eligible(p, pr->dtype)) return bfa::sm100_fwd(p, pr->dtype, st);
  return bfa::simt_fwd(p, pr->dtype, st);
}

size_t bfa_fwd_workspace_bytes(const bfa_problem* pr) {
  if (check_problem(pr) || empty_q(pr)) return 0;
  return bfa::decode_workspace_bytes(make_params(pr), pr->dtype);
}

// Backward workspace: Δ and the row statistic lse2 (row_lse2), each
// [B, Hq, Sq_pad] fp32 with the row pitch padded to a multiple of 64 (one
// bulk copy per 64-row tile), plus 256 bytes of slack that covers the
// padded rows of a last 128-row query tile.
static int64_t padded_rows(int32_t sq) { return ((int64_t)sq + 63) / 64 * 64; }

static size_t round256(size_t n) { return (n + 255) / 256 * 256; }

static size_t rowstat_bytes(const bfa_problem* pr) {
  return round256((size_t)pr->batch * pr->heads_q * padded_rows(pr->seqlen_q) * sizeof(float));
}

static size_t min_workspace_bytes(const bfa_problem* pr) { return 2 * rowstat_bytes(pr) + 256; }

size_t bfa_bwd_workspace_bytes(const bfa_problem* pr) {
  if (check_problem(pr)) return 0;
  return min_workspace_bytes(pr);
}

static int fill_bwd(const bfa_problem* pr, const bfa_bwd_args* a, Params* p) {
  if (!a) return BFA_ERR_INVALID_ARGUMENT;
  if (!a->q.data || !a->o.data || !a->dout.data || !a->lse || !a->dq.data)
    return BFA_ERR_INVALID_ARGUMENT;
  if (pr->seqlen_k > 0 && (!a->k.data || !a->v.data || !a->dk.data || !a->dv.data))
    return BFA_ERR_INVALID_ARGUMENT;
  *p = make_params(pr);
  p->q = a->q.data; p->k = a->k.data; p->v = a->v.data; p->o = a->o.data;
  p->dout = a->dout.data; p->dq = a->dq.data; p->dk = a->dk.data; p->dv = a->dv.data;
  copy_strides(p->sq_, a->q); copy_strides(p->sk_, a->k); copy_strides(p->sv_, a->v);
  copy_strides(p->so_, a->o); copy_strides(p->sdo_, a->dout); copy_strides(p->sdq_, a->dq);
  copy_strides(p->sdk_, a->dk); copy_strides(p->sdv_, a->dv);
  p->lse = const_cast<float*>(a->lse);
  p->status = a->status;
  p->timeout_ns = a->wait_timeout_ns > 0 ? (uint64_t)a->wait_timeout_ns : 1000000000ull;
  p->debug_flags = a->debug_flags;
  p->phases = a->phases ? a->phases
                        : (BFA_BWD_PHASE_DELTA | BFA_BWD_PHASE_DKDV | BFA_BWD_PHASE_DQ);
  if (a->accumulate > 1) return BFA_ERR_INVALID_ARGUMENT;
  p->grad_acc = a->accumulate;
  return BFA_OK;
}

int bfa_bwd_delta(const bfa_problem* pr, const bfa_bwd_args* a, float* delta, void* stream) {
  int rc = check_problem(pr);
  if (rc) return rc;
  if (empty_q(pr)) return BFA_OK;
  Params p;
  rc = fill_bwd(pr, a, &p);
  if (rc) return rc;
  if (!delta) return BFA_ERR_INVALID_ARGUMENT;
  p.delta = delta;
  p.lse2 = nullptr;
  p.Sq_pad = pr->seqlen_q;  // the caller's buffer is [B, Hq, Sq] contiguous
  return bfa::launch_delta(p, pr->dtype, (cudaStream_t)stream);
}

int bfa_bwd(const bfa_problem* pr, const bfa_bwd_args* a, void* workspace, size_t ws_bytes,
            void* stream) {
  int rc = check_problem(pr);
  if (rc) return rc;
  Params p;
  rc = fill_bwd(pr, a, &p);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  if (!workspace || ws_bytes < min_workspace_bytes(pr)) return BFA_ERR_WORKSPACE;
  if (((uintptr_t)workspace & 255u) != 0) return BFA_ERR_WORKSPACE;
  char* ws = (char*)workspace;
  p.delta = (float*)ws;
  p.lse2 = (float*)(ws + rowstat_bytes(pr));
  p.Sq_pad = (int32_t)padded_rows(pr->seqlen_q);
  // With Δ and dQ in one call the tcgen05 dQ kernel forms Δ in its prologue
  // and runs before dK/dV, which reads it.
  p.fuse_delta = (p.phases & BFA_BWD_PHASE_DELTA) && (p.phases & BFA_BWD_PHASE_DQ) &&
                 !empty_q(pr) && bfa::sm100_bwd_fuses_delta(p, pr->dtype);
  if (!empty_q(pr) && (p.phases & BFA_BWD_PHASE_DELTA) && !p.fuse_delta) {
    rc = bfa::launch_delta(p, pr->dtype, st);
    if (rc) return rc;
  }
  if (!(p.phases & (BFA_BWD_PHASE_DKDV | BFA_BWD_PHASE_DQ))) return BFA_OK;
  if (bfa::sm100_bwd_eligible(p, pr->dtype)) return bfa::sm100_bwd(p, pr->dtype, st);
  return bfa::simt_bwd(p, pr->dtype, st);
}

int bfa_merge_partial(int32_t batch, int32_t heads, int32_t seqlen, int32_t head_dim,
                      bfa_tensor o_acc, int32_t acc_dtype, float* lse_acc, bfa_tensor o_part,
                      int32_t part_dtype, const float* lse_part, void* stream) {
  if (batch < 0 || heads < 0 || seqlen < 0 || head_dim < 1 || head_dim > 256)
    return BFA_ERR_INVALID_ARGUMENT;
  if (bfa::dtype_bytes(acc_dtype) == 0 || bfa::dtype_bytes(part_dtype) == 0)
    return BFA_ERR_UNSUPPORTED;
  if ((int64_t)batch * heads * seqlen == 0) return BFA_OK;
  if (!o_acc.data || !o_part.data || !lse_acc || !lse_part) return BFA_ERR_INVALID_ARGUMENT;
  return bfa::launch_merge(batch, heads, seqlen, head_dim, o_acc, acc_dtype, lse_acc, o_part,
                           part_dtype, lse_part, (cudaStream_t)stream);
}

}  // extern "C"
