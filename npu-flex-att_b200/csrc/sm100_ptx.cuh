// sm100_ptx.cuh -- thin inline-PTX layer for Blackwell (sm_100a): mbarriers
// with bounded waits, TMA tensor copies, and tcgen05 (TMEM alloc, MMA,
// commit, TMEM load/store) plus the shared-memory / instruction descriptors.
//
// Descriptor encodings (PTX ISA "tcgen05 matrix descriptors"):
//  shared-memory descriptor (64 bit)
//    [0,14)  start address >> 4        [16,30) leading byte offset >> 4
//    [32,46) stride byte offset >> 4   [46,48) version = 1 (Blackwell)
//    [49,52) base offset (0: atoms are 1024-byte aligned)
//    [52]    LBO mode = 0              [61,64) swizzle: 2 = 128-byte swizzle
//  instruction descriptor for kind::f16 (32 bit)
//    [4,6) D format (1 = f32)  [7,10) A format  [10,13) B format (0 f16, 1 bf16)
//    [15] A major (0 = K)  [16] B major (0 = K, 1 = MN)
//    [17,23) N >> 3        [24,29) M >> 4
//
// Canonical 128-byte-swizzled tiles as TMA writes them (box inner extent
// 64 16-bit elements = 128 bytes): row r of a sub-tile sits at r*128 bytes and
// its 16-byte chunk c at ((c ^ (r % 8)) * 16). Eight rows form a 1024-byte atom.
//  * K-major operand [rows][64 K]: SBO = 1024 (next 8 rows); one MMA (K = 16)
//    reads 32 bytes of every row, so K steps advance the start address by 32
//    bytes inside a sub-tile and jump to the next sub-tile every 64 elements.
//  * MN-major operand [K rows][64 MN]: SBO = 1024 (next 8 K rows), LBO = the
//    byte distance to the sub-tile holding the next 64 MN elements. K steps of
//    16 advance the start address by 16 rows = 2048 bytes.
#pragma once

#include <stdint.h>

#include "bfa.h"

namespace bfa {
namespace sm100 {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps in hardware until the
// phase completes (or the hint, in ns, runs out) instead of spinning.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity,
                                                    uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Shared abort state of one CTA: once any role gives up on a wait, every
// other bounded wait in the CTA returns false at once.
struct WaitCtl {
  volatile int* abort;      // shared-memory flag
  int32_t* status;          // global status word or nullptr
  uint64_t timeout_ns;
};

// Bounded wait for phase `parity` of an mbarrier. Returns false when the CTA
// is aborting or the wait exceeded the timeout (then it raises the abort flag
// and records `code` in the status word).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const WaitCtl& ctl,
                                          int code) {
  if (mbar_try_wait(bar, parity)) return true;
  // Slow path: sleep in try_wait (woken when the phase completes, at most
  // kSleepNs per call) so a waiting thread takes no issue slots from the
  // warps doing the work; check the abort flag and the clock between calls.
  constexpr uint32_t kSleepNs = 1000000;  // 1 ms
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, kSleepNs)) return true;
    if (*ctl.abort) return false;
    if (globaltimer() - t0 > ctl.timeout_ns) {
      *ctl.abort = 1;
      if (ctl.status) atomicExch(ctl.status, code);
      return false;
    }
  }
}

// Bounded wait for a whole warp. Fast path: every lane polls once and the
// warp stays converged. Otherwise lane 0 runs the bounded wait and shares the
// result, so warp-collective tcgen05 instructions that follow stay converged.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, const WaitCtl& ctl) {
  if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, ctl, BFA_ERR_DEVICE_TIMEOUT) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}

// Drain wait (ignores the abort flag, still bounded): used before exit so
// that no async copy or MMA is in flight when the CTA retires.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, uint64_t timeout_ns) {
  if (mbar_try_wait(bar, parity)) return;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait_sleep(bar, parity, 1000000)) {
    if (globaltimer() - t0 > timeout_ns) return;
  }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* tmap, uint32_t bar, int c0,
                                            int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(tmap), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// 1-D bulk copy global -> shared, completing `bytes` on an mbarrier. Both
// addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_store_4d(const void* tmap, uint32_t src, int c0, int c1, int c2,
                                             int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          tmap),
      "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// Element-wise add of a shared-memory tile into global memory (fp32 here):
// the reduction happens in L2, so CTAs adding into the same tile need no
// other synchronisation. Completes with the store bulk-group.
__device__ __forceinline__ void tma_reduce_add_4d(const void* tmap, uint32_t src, int c0, int c1,
                                                  int c2, int c3) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.4d.global.shared::cta.add.bulk_group [%0, {%2, %3, %4, %5}], "
      "[%1];" ::"l"(tmap),
      "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// 1-D bulk copy / element-wise fp32 add of `bytes` from shared to global
// memory (both addresses 16-byte aligned, size a multiple of 16). Complete
// with the store bulk-group.
__device__ __forceinline__ void bulk_store(void* dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_reduce_add_f32(void* dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(dst),
               "r"(src), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void tma_store_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__device__ __forceinline__ void tma_store_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Wait until at most N of this thread's bulk groups are pending: `_read` once
// their shared-memory sources have been read, plain once they are complete.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Ordering between generic-proxy accesses (flags) and async-proxy ones (TMA).
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async;" ::: "memory");
}

__device__ __forceinline__ void fence_acq_rel_gpu() {
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_gpu_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Make generic-proxy writes to shared memory visible to the async proxy
// (tensor cores, TMA).
__device__ __forceinline__ void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- named barriers
__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16, one CTA.
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16. A is K-major in TMEM: row m of
// A in lane m, 16-bit elements packed two per 32-bit column (K = 16 per
// instruction spans 8 columns).
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once every tcgen05 op this thread issued so far is done.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives
// lane (base lane + t), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- descriptors
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                               uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// K-major operand in 128-byte-swizzled sub-tiles: LBO unused (1), SBO 1024.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t saddr) {
  return desc_sw128(saddr, 16, 1024);
}

// MN-major operand: the next 64 MN elements live `mn_block_bytes` further.
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t saddr, uint32_t mn_block_bytes) {
  return desc_sw128(saddr, mn_block_bytes, 1024);
}

// kind::f16 instruction descriptor, f32 accumulate. `bf16` selects bf16 inputs.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool bf16, bool b_mn_major,
                                                 bool a_mn_major = false) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Byte offset of the 16-byte chunk `c16` (0..7) of row `r` inside a
// 128-byte-swizzled sub-tile.
__device__ __forceinline__ uint32_t sw128_offset(int r, int c16) {
  return (uint32_t)(r * 128 + ((c16 ^ (r & 7)) << 4));
}

// ---------------------------------------------------------------- math
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one instruction (three-input max.f32, sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x on the FMA pipe instead of the MUFU unit, to split the exponentials of
// a softmax between the two (the MUFU unit alone is a bottleneck on B200).
// Cody-Waite style reduction x = j + f, j = rint(x) taken from the low
// mantissa bits of x + 1.5·2^23, f in [-0.5, 0.5]; 2^f by a cubic fitted for
// this code by relative least squares on Chebyshev nodes (max relative error
// 7.8e-5, ample for 16-bit P); 2^j is added to the exponent bits. x is
// clamped to >= -126, so the result is never exactly 0: callers use it only
// where no element is masked to -inf (or zero masked elements themselves).
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -126.f);
  const float t = x + 12582912.f;
  const float f = x - (t - 12582912.f);
  const float p = fmaf(fmaf(fmaf(0.05508868f, f, 0.24260405f), f, 0.69327623f), f, 0.99992895f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The soft-cap logit is cap·tanh(s/cap). Two forms of tanh, both without
// data-dependent branches, so a warp never splits over them; a kernel picks
// one per warp and step (tanh_small when every |x| of the warp is <= 1/2):
//  * tanh_small: the odd Taylor series of tanh to x^11, on the FMA pipe;
//    truncation error below 1e-6 relative for |x| <= 1/2.
//  * tanh_any: sign(x)·(1 - 2/(1 + e^{2|x|})) with ex2 / rcp on the MUFU
//    unit; absolute error a few fp32 ulps of 1, so where tanh x is tiny its
//    relative error grows, but cap·tanh x is then tiny as well.
constexpr float kTanhT1 = -1.0f / 3.0f;
constexpr float kTanhT2 = 2.0f / 15.0f;
constexpr float kTanhT3 = -17.0f / 315.0f;
constexpr float kTanhT4 = 62.0f / 2835.0f;
constexpr float kTanhT5 = -1382.0f / 155925.0f;

__device__ __forceinline__ float tanh_small(float x) {
  const float z = x * x;
  float q = fmaf(z, kTanhT5, kTanhT4);
  q = fmaf(z, q, kTanhT3);
  q = fmaf(z, q, kTanhT2);
  q = fmaf(z, q, kTanhT1);
  q = fmaf(z, q, 1.0f);
  return x * q;
}

// The same series to x^7: truncation below 2e-9 relative for |x| <= 1/8.
__device__ __forceinline__ float tanh_tiny(float x) {
  const float z = x * x;
  float q = fmaf(z, kTanhT3, kTanhT2);
  q = fmaf(z, q, kTanhT1);
  q = fmaf(z, q, 1.0f);
  return x * q;
}

__device__ __forceinline__ float tanh_any(float x) {
  const float e = ex2(fminf(2.0f * 1.4426950408889634f * fabsf(x), 126.0f));
  return copysignf(1.0f - 2.0f * rcp(1.0f + e), x);
}

// Which tanh serves a warp's step (warp-uniform): 2 (tanh_tiny) when every
// |raw·cap_in| of the warp's n raw logits is <= 1/8, 1 (tanh_small) when <=
// 1/2, else 0 (tanh_any).
template <int N>
__device__ __forceinline__ int cap_tier(const uint32_t* raw, float cap_in) {
  float am = 0.f;
#pragma unroll
  for (int e = 0; e < N; e += 2)
    am = fmax3(am, fabsf(__uint_as_float(raw[e])), fabsf(__uint_as_float(raw[e + 1])));
  am *= cap_in;
  return __all_sync(0xffffffffu, am <= 0.125f) ? 2 : __all_sync(0xffffffffu, am <= 0.5f) ? 1 : 0;
}

// logit2 for a pair of raw logits with a soft-cap and no ALiBi, in packed
// f32x2 instructions (half the issue slots of two scalar calls): returns
// cap·tanh(raw·cap_in)·log2(e) and the two tanh values in *th.
template <int TIER>
__device__ __forceinline__ float2 cap_logit2x2(float2 raw, float cap_in, float cap_out, float2* th) {
  const float2 u = __fmul2_rn(raw, make_float2(cap_in, cap_in));
  float2 t;
  if (TIER == 2) {
    const float2 z = __fmul2_rn(u, u);
    float2 q = __ffma2_rn(z, make_float2(kTanhT3, kTanhT3), make_float2(kTanhT2, kTanhT2));
    q = __ffma2_rn(z, q, make_float2(kTanhT1, kTanhT1));
    q = __ffma2_rn(z, q, make_float2(1.f, 1.f));
    t = __fmul2_rn(u, q);
  } else if (TIER == 1) {
    const float2 z = __fmul2_rn(u, u);
    float2 q = __ffma2_rn(z, make_float2(kTanhT5, kTanhT5), make_float2(kTanhT4, kTanhT4));
    q = __ffma2_rn(z, q, make_float2(kTanhT3, kTanhT3));
    q = __ffma2_rn(z, q, make_float2(kTanhT2, kTanhT2));
    q = __ffma2_rn(z, q, make_float2(kTanhT1, kTanhT1));
    q = __ffma2_rn(z, q, make_float2(1.f, 1.f));
    t = __fmul2_rn(u, q);
  } else {
    t = make_float2(tanh_any(u.x), tanh_any(u.y));
  }
  *th = t;
  return __fmul2_rn(t, make_float2(cap_out, cap_out));
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %2, %1;" : "=r"(r) : "f"(a), "f"(b));
  return r;
}

__device__ __forceinline__ uint32_t pack_f16(float a, float b) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %2, %1;" : "=r"(r) : "f"(a), "f"(b));
  return r;
}

}  // namespace sm100
}  // namespace bfa
