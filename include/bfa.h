/*
 * bfa.h -- C ABI of libbfa.so, the B200 (sm_100a) flash-attention library.
 *
 * This is the drop-in boundary for the attention hot path of
 * dropletzhu/npu-flex-att. The reference's Python host API launches three
 * Triton kernels and two host-side torch reductions; each entry point below
 * replaces one or more of those launch sites:
 *
 *   bfa_fwd        <- flash_attn_fwd_kernel launch, npu_flash_attention.py:631-652
 *   bfa_bwd_delta  <- host Δ = rowsum(O∘dO),        npu_flash_attention.py:685
 *   bfa_bwd        <- Δ (:685) + flash_attn_bwd_dq_kernel launch (:695-712)
 *                     + flash_attn_bwd_dkdv_kernel launch (:714-732)
 *                     + host GQA sum of dK/dV (:735-737)
 *   bfa_merge_partial  (no reference counterpart: LSE merge of two partial
 *                     attention results in memory; the context-parallel ring
 *                     has bfa_fwd merge its own result instead, with
 *                     bfa_fwd_args.accumulate. The idea follows the
 *                     reference's unused split-KV reduce kernel,
 *                     npu_flash_attention.py:255-293)
 *
 * Conventions
 *  - Plain C: pointers, sizes, int64 element strides. No torch or CUDA types;
 *    a stream is passed as `void*` holding a cudaStream_t (NULL = legacy default).
 *  - Tensors are [B, H, S, D] with arbitrary element strides per dimension, as
 *    the reference accepts (its kernels take four strides per tensor,
 *    npu_flash_attention.py:20-24). The fast tcgen05 path needs a unit innermost
 *    stride and 16-byte aligned outer strides; other layouts run on the
 *    generic CUDA path, never on the CPU.
 *  - The LSE is fp32, natural log, contiguous [B, Hq, Sq] (npu_flash_attention.py:632,161).
 *  - The library allocates no device memory. Scratch lives in caller-provided
 *    workspaces: the backward's row statistics (Δ) in one of
 *    bfa_bwd_workspace_bytes() bytes, the split-KV decoding forward's partial
 *    results in one of bfa_fwd_workspace_bytes() bytes.
 *  - Calls are asynchronous on the given stream; they are thread-safe and
 *    re-entrant. The device is the caller's current CUDA device.
 *  - Return value: BFA_OK (0) or a negative bfa_status. Nothing is thrown
 *    across the ABI. bfa_strerror() gives a message for any status.
 *  - Kernels that wait on mbarriers bound every wait. When a wait runs out the
 *    kernel writes BFA_ERR_DEVICE_TIMEOUT into the optional `status` word
 *    (device int32, caller-owned, may be NULL) and returns cleanly.
 */
#ifndef BFA_H
#define BFA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BFA_ABI_VERSION 5

typedef enum bfa_dtype {
  BFA_DTYPE_F32 = 0,
  BFA_DTYPE_F16 = 1,
  BFA_DTYPE_BF16 = 2
} bfa_dtype;

typedef enum bfa_status {
  BFA_OK = 0,
  BFA_ERR_INVALID_ARGUMENT = -1,  /* null pointer, negative size, bad flag value */
  BFA_ERR_SHAPE = -2,             /* D mismatch or Hq % Hkv != 0 */
  BFA_ERR_UNSUPPORTED = -3,       /* dtype or head_dim outside what is built */
  BFA_ERR_WORKSPACE = -4,         /* workspace missing or too small */
  BFA_ERR_CUDA = -5,              /* a CUDA runtime/driver call failed */
  BFA_ERR_DEVICE_TIMEOUT = -6,    /* a device-side wait ran out (status word) */
  BFA_ERR_SCRATCH_LIMIT = -7      /* bfa_bwd_noalloc: problem larger than its static scratch */
} bfa_status;

/* Problem description: the reference host API's arguments
 * (npu_flash_attention_forward, npu_flash_attention.py:606-616). */
typedef struct bfa_problem {
  int32_t batch;
  int32_t heads_q;
  int32_t heads_kv;        /* heads_q % heads_kv == 0; K/V head = hq / (Hq/Hkv) */
  int32_t seqlen_q;
  int32_t seqlen_k;
  int32_t head_dim;        /* 1..256 */
  int32_t dtype;           /* bfa_dtype of q, k, v, o, dout, dq, dk, dv */
  int32_t causal;          /* keep i >= j (top-left aligned) */
  int32_t sliding_window;  /* 0 = off; else keep i - j <= sliding_window */
  float scale;             /* logits scale (the reference default is 1/sqrt(D)) */
  float soft_cap;          /* 0 = off; else logits = cap * tanh(logits / cap) */
  const float* alibi_slopes; /* NULL or device fp32 [heads_q]: logits += slope * (i - j) */
  int64_t q_pos_offset;    /* absolute position of query row 0 (0 unless context-parallel) */
  int64_t k_pos_offset;    /* absolute position of key row 0 */
  /* Document masking (no reference counterpart; both NULL = off): device
   * int32 arrays indexed by absolute position x, covering every query and
   * key position of the problem. The document holding x spans
   * [doc_start[x], doc_end[x]); a pair (i, j) is kept only when j lies in
   * i's document (on top of causal / window). Tiles outside every row's
   * document are skipped like causal ones. */
  const int32_t* doc_start;
  const int32_t* doc_end;
  /* Block-sparse mask (no reference counterpart; NULL = off): device uint8
   * [B, Hq, ceil(Sq/128), ceil(Sk/128)] at element strides block_mask_stride
   * (batch, q-head, query block; the key-block stride is 1; a stride of 0
   * broadcasts). Query row r and key row c of the call (local indices) fall in
   * block (r / 128, c / 128); a zero byte drops the whole block, on top of the
   * other masks. Dropped blocks are skipped, not computed. */
  const uint8_t* block_mask;
  int64_t block_mask_stride[3];
} bfa_problem;

/* A strided 4-D device tensor [B, H, S, D]; strides are in elements. */
typedef struct bfa_tensor {
  void* data;
  int64_t stride[4];
} bfa_tensor;

/* Test-only switch for bfa_*_args.debug_flags: one device-side wait in the
 * tcgen05 kernels waits on a barrier that nothing completes, so the bounded
 * wait runs out and the kernel reports BFA_ERR_DEVICE_TIMEOUT in `status`. */
#define BFA_DEBUG_INJECT_STALL 1u

typedef struct bfa_fwd_args {
  bfa_tensor q;            /* [B, Hq, Sq, D] */
  bfa_tensor k;            /* [B, Hkv, Sk, D] */
  bfa_tensor v;            /* [B, Hkv, Sk, D] */
  bfa_tensor o;            /* [B, Hq, Sq, D], written */
  float* lse;              /* [B, Hq, Sq] fp32 contiguous, written */
  int32_t* status;         /* optional device status word */
  int64_t wait_timeout_ns; /* bound on any device-side wait; 0 = 1 second */
  uint32_t debug_flags;    /* 0 in production; BFA_DEBUG_* for tests */
  void* workspace;         /* optional device scratch, 256-byte aligned: lets problems
                              with few query rows per KV head take the split-KV
                              decoding path (NULL: the regular forward runs) */
  size_t workspace_bytes;  /* size of `workspace`; the decoding path needs
                              bfa_fwd_workspace_bytes(problem) */
  uint32_t accumulate;     /* 0: `o` has the input dtype and is overwritten, `lse` is
                              written. 1: `o` is an fp32 running output and `lse` its
                              running LSE (-inf: no key yet); the call merges its own
                              result into both in its epilogue,
                                lse' = logaddexp(lse, lse_call),
                                o'   = o·e^(lse - lse') + o_call·e^(lse_call - lse'),
                              as bfa_merge_partial does, with no partial result in
                              memory (one block of a context-parallel ring). */
} bfa_fwd_args;

typedef struct bfa_bwd_args {
  bfa_tensor q, k, v;      /* as in the forward */
  bfa_tensor o;            /* forward output */
  bfa_tensor dout;         /* [B, Hq, Sq, D] upstream gradient */
  const float* lse;        /* forward LSE [B, Hq, Sq] */
  bfa_tensor dq;           /* [B, Hq, Sq, D], written */
  bfa_tensor dk;           /* [B, Hkv, Sk, D], written (sum over the GQA group) */
  bfa_tensor dv;           /* [B, Hkv, Sk, D], written (sum over the GQA group) */
  int32_t* status;         /* optional device status word */
  int64_t wait_timeout_ns; /* bound on any device-side wait; 0 = 1 second */
  uint32_t debug_flags;    /* 0 in production; BFA_DEBUG_* for tests */
  uint32_t phases;         /* 0 = all; else a mask of BFA_BWD_PHASE_* (same workspace
                              across the calls, Δ first) -- lets a caller time each kernel.
                              A call with both DELTA and DQ on the tcgen05 path forms Δ
                              inside the dQ kernel and runs dQ before dK/dV */
  uint32_t accumulate;     /* 0: dq/dk/dv have the input dtype and are overwritten.
                              1: dq/dk/dv are fp32 accumulators and the gradients are
                              added to them (blockwise / context-parallel backward: no
                              16-bit rounding of partial gradients) */
} bfa_bwd_args;

#define BFA_BWD_PHASE_DELTA 1u  /* Δ = rowsum(O∘dO) into the workspace */
#define BFA_BWD_PHASE_DKDV 2u   /* dK, dV */
#define BFA_BWD_PHASE_DQ 4u     /* dQ */

/* ABI version of the loaded library (BFA_ABI_VERSION at build time). */
int bfa_abi_version(void);

/* Number of CUDA kernels this library has launched in this process (all
 * devices, all threads); a monotonically increasing counter. */
uint64_t bfa_launch_count(void);

/* Static message for a bfa_status value. */
const char* bfa_strerror(int status);

/* Detail of the last BFA_ERR_CUDA this thread got from the library: the
 * failing call (kernel launch, shared-memory attribute, tensor-map encode,
 * ...) and the CUDA error name, e.g. "dq_kernel launch: cudaErrorInvalidValue".
 * "" when none; valid until the thread's next library call fails. */
const char* bfa_last_error(void);

/* Forward: O and LSE. Replaces the launch at npu_flash_attention.py:631-652. */
int bfa_fwd(const bfa_problem* problem, const bfa_fwd_args* args, void* stream);

/* Bytes of workspace that let bfa_fwd take the split-KV decoding path for
 * this problem on the current device (the partial O / LSE of each key split;
 * the reference's unused split-KV forward, npu_flash_attention.py:171-293,
 * wrote them to torch tensors it allocated at :255-262). 0 when the problem
 * never takes that path (more than 64 query rows per KV head, or a dtype /
 * head_dim it does not cover). */
size_t bfa_fwd_workspace_bytes(const bfa_problem* problem);

/* Bytes of workspace bfa_bwd needs for this problem (Δ and alignment). */
size_t bfa_bwd_workspace_bytes(const bfa_problem* problem);

/* Δ = rowsum(O∘dO) in fp32 into `delta` [B, Hq, Sq] contiguous.
 * Replaces the host reduction at npu_flash_attention.py:685. */
int bfa_bwd_delta(const bfa_problem* problem, const bfa_bwd_args* args,
                  float* delta, void* stream);

/* Backward: dQ, dK, dV (dK/dV already summed over each GQA group).
 * Replaces npu_flash_attention.py:675-739 (Δ, the dQ and dK/dV launches and
 * the host GQA sum). `workspace` is device memory of at least
 * bfa_bwd_workspace_bytes(problem) bytes, 256-byte aligned. */
int bfa_bwd(const bfa_problem* problem, const bfa_bwd_args* args,
            void* workspace, size_t workspace_bytes, void* stream);

/* Backward that allocates nothing (no reference counterpart).
 * Same inputs, outputs and results as bfa_bwd, for callers that cannot
 * allocate device memory: a plugin whose host framework owns all device
 * allocations and passes only the input/output buffers, or a hot path that
 * must not call cudaMalloc because it can synchronise the device. The row
 * statistics (Δ, scaled LSE) go to a static device array sized for 2^21 query
 * rows, each head's rows rounded up to 64 (batch*heads_q*ceil(seqlen_q/64)*64;
 * 16 MiB per GPU that loads the library, held until exit); larger problems
 * return BFA_ERR_SCRATCH_LIMIT. All calls share that array: calls that overlap on the
 * GPU race, so serialise them. Each call computes Δ itself: a `phases` mask
 * without BFA_BWD_PHASE_DELTA is rejected (BFA_ERR_INVALID_ARGUMENT), since
 * the array may hold another call's Δ. The first call on each device looks up
 * the array's address and should come before any stream capture; the address
 * is cached for the life of the process, so the library must not be used
 * across a cudaDeviceReset. */
int bfa_bwd_noalloc(const bfa_problem* problem, const bfa_bwd_args* args, void* stream);

/* Merge a partial attention result into a running one, in place:
 *   lse' = logaddexp(lse_acc, lse_part)
 *   o'   = o_acc * exp(lse_acc - lse') + o_part * exp(lse_part - lse')
 * o_acc / o_part are [B, H, S, D] with the given strides and dtype `dtype`
 * (o_acc may be fp32 for accumulation: `acc_dtype`), lse_* contiguous fp32
 * [B, H, S]. No reference counterpart (see the header comment). */
int bfa_merge_partial(int32_t batch, int32_t heads, int32_t seqlen, int32_t head_dim,
                      bfa_tensor o_acc, int32_t acc_dtype, float* lse_acc,
                      bfa_tensor o_part, int32_t part_dtype, const float* lse_part,
                      void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BFA_H */
