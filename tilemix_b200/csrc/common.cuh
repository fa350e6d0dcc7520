// Shared device helpers for the TileMix B200 kernels (sm_100a only).
//
// Thin inline-PTX wrappers around mbarriers, TMA bulk tensor copies and the
// tcgen05 (5th-generation tensor core / tensor memory) instructions, plus the
// bounded-wait machinery every spin loop in this library goes through: a wait
// gives up after kWaitTimeoutNs of %globaltimer, records an error code in a
// device flag and returns false, so a broken pipeline ends the kernel with a
// status instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "tilemix_b200 kernels target sm_100a only"
#endif

namespace tilemix {

// Error codes written to the device error word (first writer wins).
enum : int {
  kErrNone = 0,
  kErrTimeoutFull = 1,      // consumer waited too long for a TMA stage
  kErrTimeoutEmpty = 2,     // producer waited too long for a free stage
  kErrTimeoutScores = 3,    // softmax waited too long for S
  kErrTimeoutP = 4,         // MMA warp waited too long for P
  kErrTimeoutPV = 5,        // waited too long for a PV completion
  kErrTimeoutQ = 6,         // MMA warp waited too long for Q in TMEM
  kErrTimeoutDrain = 7,     // final drain of in-flight work timed out
  kErrTimeoutQFree = 9,     // Q producer waited too long for the previous work item's last S
  kErrTimeoutOFree = 10,    // MMA warp waited too long for the previous work item's O to be read
};

constexpr unsigned long long kWaitTimeoutNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

// ----------------------------------------------------------------------------
// mbarrier
// ----------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking test of phase completion.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that lets the hardware keep the thread suspended for up to
// `suspend_ns` while the phase is incomplete (it resumes as soon as the phase
// completes), so a waiting warp takes no issue slots from the others.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t suspend_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(suspend_ns)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, 1000000u)) return true;
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
      record_error(err, code);
      return false;
    }
  }
}

// Wait for waits on the critical path: a loop of try_wait without a suspend
// hint. The hardware parks the warp inside try_wait until the phase completes
// (or a short system time limit passes), so the waiting warp takes no issue
// slots from the softmax warps and still resumes within about as many cycles
// as a test_wait poll; a long suspend hint (mbar_wait) resumes far later.
// Bounded like mbar_wait.
__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t n = 1;; ++n) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((n & 1023u) == 0 && globaltimer_ns() - t0 > kWaitTimeoutNs) {
      record_error(err, code);
      return false;
    }
  }
}

// ----------------------------------------------------------------------------
// TMA: plain tiled loads from this GPU's own memory
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_l2_4d(const CUtensorMap* map, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

// Warm L2 with a tile of a tensor (no shared-memory destination, no barrier).
__device__ __forceinline__ void tma_prefetch_l2_3d(const CUtensorMap* map, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ----------------------------------------------------------------------------
// tcgen05: tensor memory allocation, MMA, loads/stores, fences
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]   kind::f16 (fp16 inputs)
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]   kind::f16 (fp16 inputs)
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]   kind::i8 (signed int8 inputs, int32 accumulate)
__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// ----------------------------------------------------------------------------
// Elected-lane forms: called by a whole warp with warp-uniform arguments; one
// elected lane issues the instruction. Keeping the issuing warp converged lets
// descriptors and addresses stay warp-uniform, which is far cheaper per issued
// tcgen05 / bulk-tensor instruction than issuing from a branch taken by one
// lane.
// ----------------------------------------------------------------------------
__device__ __forceinline__ void mma_f16_ss_e(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_i8_ss_e(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_f16_ts_e(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tc_commit_e(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx_e(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_e(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                              int c2) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];\n\t}" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d_e(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                              int c2, int c3) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];\n\t}" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// Make this thread's generic-proxy shared-memory writes visible to the async
// proxy (TMA, tensor core) before signalling another thread.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]   kind::i8 (signed int8 inputs, int32 accumulate)
__device__ __forceinline__ void mma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns; thread i of the warp gets lane (base lane + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 64 columns whose values are 16-bit (the low half of each 32-bit column, as an
// fp16 MMA accumulator leaves them), packed in pairs during the load: r[i] holds
// column 2i in bits 0-15 and column 2i+1 in bits 16-31 (.x32 counts the 32-bit
// destination registers, each of two columns).
__device__ __forceinline__ void tmem_ld64_pack16(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.pack::16b.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// ----------------------------------------------------------------------------
// Descriptors
// ----------------------------------------------------------------------------
// Instruction descriptor (kind::f16 / kind::i8): D format, A/B formats, majors, N, M.
//   c_fmt: 0 = F16, 1 = F32, 2 = S32;  ab_fmt: kind::f16 -> 0 (F16); kind::i8 -> 1 (signed)
//   major: 0 = K-major, 1 = MN-major
__host__ __device__ constexpr uint32_t make_idesc(uint32_t c_fmt, uint32_t ab_fmt, uint32_t a_major,
                                                  uint32_t b_major, uint32_t M, uint32_t N) {
  return (c_fmt << 4) | (ab_fmt << 7) | (ab_fmt << 10) | (a_major << 15) | (b_major << 16) | ((N >> 3) << 17) |
         ((M >> 4) << 24);
}

// Shared-memory matrix descriptor (sm_100 format, version 1).
//   layout: 2 = 128-byte swizzle, 4 = 64-byte swizzle
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                               uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(layout & 0x7u) << 61;
  return d;
}

// ----------------------------------------------------------------------------
// Small numeric helpers
// ----------------------------------------------------------------------------
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_half2_rn(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ----------------------------------------------------------------------------
// Numerics of the reference's divisions and score accumulation
// ----------------------------------------------------------------------------
// The reference's kernels are Triton code. On the GPU, Triton compiles an fp32
// `a / b` to PTX div.full.f32 (a full-range approximate division, <= 2 ulp)
// and tl.dot(fp16, fp16, out_dtype=fp16) to tcgen05 MMAs with an fp16
// accumulator; its interpreter (and the reference algorithm read as exact
// arithmetic) divides with IEEE rounding and accumulates in fp32 before one
// rounding. The kernels here take the mode as a template argument:
//   kNumericsGpu   = the reference as it runs on the GPU (the default)
//   kNumericsExact = the reference's algorithm with IEEE division and fp32
//                    score accumulation (bit-exact with its interpreter run)
enum : int { kNumericsGpu = 0, kNumericsExact = 1 };

// PTX div.full.f32: the division the reference's Triton kernels execute.
__device__ __forceinline__ float div_full(float a, float b) {
  float r;
  asm("div.full.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// scale = absmax / 127 of a quantisation block in the given numerics.
template <int kNumerics>
__device__ __forceinline__ float quant_scale(float absmax) {
  return kNumerics == kNumericsGpu ? div_full(absmax, 127.f) : __fdiv_rn(absmax, 127.f);
}

// Symmetric per-block INT8 code of x for a given block scale, as the reference
// quantiser computes it: y = x / scale, y += (y >= 0 ? 0.5 : -0.5), truncate
// toward zero (NaN -> 0).
template <int kNumerics>
__device__ __forceinline__ int quant_code(float x, float scale) {
  float y = kNumerics == kNumericsGpu ? div_full(x, scale) : __fdiv_rn(x, scale);
  y = __fadd_rn(y, y >= 0.f ? 0.5f : -0.5f);
  return __float2int_rz(y);
}

// Round half away from zero of a pair of quotients y, on the FMA pipe (a
// cvt.rzi would share the conversion pipe with the softmax's ex2): trunc(|y| +
// 0.5) with the sign of y restored. |y| + 0.5 equals the reference's |y + (y >=
// 0 ? 0.5 : -0.5)| (round to nearest is symmetric); an add rounded toward zero
// against 1.5 * 2^23 truncates it (it is >= 0 and < 2^22), and adding 1.5 *
// 2^23 to the signed code leaves the code's two's complement byte in the low
// mantissa bits. Returns the low bytes of the two codes in bits 0-7 of *c0 /
// *c1 (upper bits unspecified). |y| < 2^22 required (quotients of a block's
// values by its scale are at most 127 in magnitude).
__device__ __forceinline__ void round_codes_pair_fma(uint64_t y, uint32_t* c0, uint32_t* c1) {
  constexpr uint64_t kMagic2 = 0x4B4000004B400000ull;  // (1.5 * 2^23, 1.5 * 2^23)
  const float y0 = __uint_as_float(static_cast<uint32_t>(y)), y1 = __uint_as_float(static_cast<uint32_t>(y >> 32));
  const float b0 = __fadd_rn(fabsf(y0), 0.5f), b1 = __fadd_rn(fabsf(y1), 0.5f);
  const uint64_t b2 = (static_cast<uint64_t>(__float_as_uint(b1)) << 32) | __float_as_uint(b0);
  uint64_t t, k;
  asm("add.rz.f32x2 %0, %1, %2;" : "=l"(t) : "l"(b2), "l"(kMagic2));
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(k) : "l"(t), "l"(kMagic2));
  const float k0 = copysignf(__uint_as_float(static_cast<uint32_t>(k)), y0);
  const float k1 = copysignf(__uint_as_float(static_cast<uint32_t>(k >> 32)), y1);
  const uint64_t ks = (static_cast<uint64_t>(__float_as_uint(k1)) << 32) | __float_as_uint(k0);
  uint64_t u;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(u) : "l"(ks), "l"(kMagic2));
  *c0 = static_cast<uint32_t>(u);
  *c1 = static_cast<uint32_t>(u >> 32);
}

// Per-block division constants of the quantiser for one block scale.
struct QuantDiv {
  float scale;
  uint64_t r2;   // (1/scale, 1/scale), correctly rounded (exact numerics)
  uint64_t ns2;  // (-scale, -scale)
  __device__ __forceinline__ void init(float s) {
    scale = s;
    const float r = __frcp_rn(s);
    r2 = (static_cast<uint64_t>(__float_as_uint(r)) << 32) | __float_as_uint(r);
    ns2 = (static_cast<uint64_t>(__float_as_uint(-s)) << 32) | __float_as_uint(-s);
  }
};

// Codes of a pair of x for a block scale: the quotient of the numerics, then
// the FMA-pipe rounding above. Exact numerics form the IEEE quotient from the
// correctly rounded reciprocal with one FMA residual correction (Markstein:
// q0 = x*r, q = q0 + (x - q0*scale)*r); for every finite fp16 x and every
// scale = fp16 magnitude / 127 it equals x / scale (checked exhaustively on a
// B200), except that x = -0 gives +0, which yields the same code. GPU
// numerics divide with div.full.f32. Requires a finite scale > 0 (callers
// treat other scales separately) and finite x (a NaN x yields an unspecified
// code instead of the reference's 0).
template <int kNumerics>
__device__ __forceinline__ void quant_code_pair(float x0, float x1, const QuantDiv& d, uint32_t* c0, uint32_t* c1) {
  uint64_t y;
  if (kNumerics == kNumericsGpu) {
    y = (static_cast<uint64_t>(__float_as_uint(div_full(x1, d.scale))) << 32) | __float_as_uint(div_full(x0, d.scale));
  } else {
    const uint64_t x2 = (static_cast<uint64_t>(__float_as_uint(x1)) << 32) | __float_as_uint(x0);
    uint64_t q0, e;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(q0) : "l"(x2), "l"(d.r2));
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(e) : "l"(q0), "l"(d.ns2), "l"(x2));
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(y) : "l"(e), "l"(d.r2), "l"(q0));
  }
  round_codes_pair_fma(y, c0, c1);
}

// fp16(acc / l) of a pair of fp32 accumulator values in the given numerics:
// div.full.f32 as the reference's kernel divides on the GPU, or the correctly
// rounded quotient (reciprocal rl = 1/l once per row, then per element one
// residual correction: q0 = a*rl, e = a - q0*l, q = q0 + e*rl).
template <int kNumerics>
__device__ __forceinline__ uint32_t normalize_pair(float a0, float a1, float l, float rl) {
  if (kNumerics == kNumericsGpu) return pack_half2_rn(div_full(a0, l), div_full(a1, l));
  const float q0 = a0 * rl, q1 = a1 * rl;
  return pack_half2_rn(fmaf(fmaf(-q0, l, a0), rl, q0), fmaf(fmaf(-q1, l, a1), rl, q1));
}

}  // namespace tilemix
