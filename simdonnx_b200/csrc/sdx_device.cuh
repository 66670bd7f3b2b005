// Device-side building blocks for the sm_100a kernels: bounded mbarrier waits, TMA tile loads,
// tcgen05 (UMMA + TMEM) wrappers and the fused-epilogue activations.
//
// Every spin-wait here is bounded: after SDX_WAIT_NS of wall time (the %globaltimer clock) the
// waiting thread records an error code in the caller's device error word, raises the CTA's shared
// abort flag and returns false, so the kernel winds down (no trap, no hang).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "sdx_status.h"

#ifndef SDX_WAIT_NS
#define SDX_WAIT_NS 2000000000ull  // 2 s
#endif

namespace sdx {

// ------------------------------------------------------------------ activations
// ActivationKind of the reference plan (src/Engine/ExecPlan.cs:42).
enum Act : int { ACT_NONE = 0, ACT_RELU = 1, ACT_SIGMOID = 2, ACT_GELU = 3, ACT_HARDSWISH = 4, ACT_SWISH = 5 };

// Compile-time activation: each kernel is instantiated per activation, so its inner loops carry
// only the one they apply (a runtime switch inlined per element bloats the loop past the
// instruction cache and stalls on branch resolution).
template <int ACT>
__device__ __forceinline__ float act_t(float v) {
  if constexpr (ACT == ACT_RELU) return fmaxf(v, 0.0f);
  else if constexpr (ACT == ACT_SIGMOID) return 1.0f / (1.0f + expf(-v));
  else if constexpr (ACT == ACT_GELU) return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
  else if constexpr (ACT == ACT_HARDSWISH) return v * __saturatef(fmaf(v, 1.0f / 6.0f, 0.5f));  // clamp to [0, 1]
  else if constexpr (ACT == ACT_SWISH) return v / (1.0f + expf(-v));
  else return v;
}

// Runtime dispatch of a kernel template over the activation kind.
#define SDX_ACT_DISPATCH(act, ACTC, ...)                   \
  switch (act) {                                          \
    case ACT_RELU: { constexpr int ACTC = ACT_RELU; __VA_ARGS__; } break;           \
    case ACT_SIGMOID: { constexpr int ACTC = ACT_SIGMOID; __VA_ARGS__; } break;     \
    case ACT_GELU: { constexpr int ACTC = ACT_GELU; __VA_ARGS__; } break;           \
    case ACT_HARDSWISH: { constexpr int ACTC = ACT_HARDSWISH; __VA_ARGS__; } break; \
    case ACT_SWISH: { constexpr int ACTC = ACT_SWISH; __VA_ARGS__; } break;         \
    default: { constexpr int ACTC = ACT_NONE; __VA_ARGS__; } break;                 \
  }

__device__ __forceinline__ float act_apply(float v, int act) {
  switch (act) {
    case ACT_RELU: return fmaxf(v, 0.0f);
    case ACT_SIGMOID: return 1.0f / (1.0f + expf(-v));
    case ACT_GELU: return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
    case ACT_HARDSWISH: return v * __saturatef(fmaf(v, 1.0f / 6.0f, 0.5f));
    case ACT_SWISH: return v / (1.0f + expf(-v));
    default: return v;
  }
}

// ------------------------------------------------------------------ misc
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_error(unsigned int* err, unsigned int code) {
  if (err) atomicCAS(err, 0u, code);
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// ---- issue from one lane of a converged warp without a divergent branch: the calling code stays
// warp-uniform (its values live in uniform registers) and the instruction is predicated on `p`
// (nonzero in exactly one lane, from elect_leader()). Keeping the issuing code warp-uniform cuts
// the per-issue cost of tcgen05.mma / TMA several-fold against an `if (lane == 0)` region.
__device__ __forceinline__ uint32_t elect_leader() {
  uint32_t e;
  asm volatile("{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\tselp.u32 %0, 1, 0, e;\n\t}" : "=r"(e));
  return e;
}
__device__ __forceinline__ void mbar_arrive_expect_tx_p(uint32_t p, uint32_t bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t"
               "@q mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n\t}" ::"r"(bar), "r"(bytes), "r"(p)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// try_wait with a suspend-time hint: the waiting thread is suspended (not spinning, so it takes no
// issue slots from the warps that share its scheduler) until the phase completes or about
// `hint_ns` passes.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return done != 0;
}

// Waits until the phase of `bar` with parity `parity` has completed. Bounded: returns false (after
// recording `code` and raising *abort_flag) when SDX_WAIT_NS passes, or at once when another role
// of the CTA has already raised *abort_flag. After the first probe the thread sleeps in the barrier
// (suspend hint) between checks of the abort flag and the clock.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned int* err, unsigned int code,
                                          volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if ((it & 15u) == 0) {
      if (*abort_flag) return false;
      if (global_timer_ns() - t0 > SDX_WAIT_NS) {
        record_error(err, code);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// Bounded wait used on the wind-down path: ignores the abort flag, only the time limit applies.
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity, unsigned int* err, unsigned int code) {
  uint64_t t0 = global_timer_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 255u && global_timer_ns() - t0 > SDX_WAIT_NS) {
      record_error(err, code);
      return false;
    }
  }
}

// ------------------------------------------------------------------ TMA (no multicast anywhere)
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d_p(uint32_t p, uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0,
                                              int c1) {
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %5, 0;\n\t"
      "@q cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      "\n\t}" ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(p)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d_p(uint32_t p, uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0,
                                              int c1, int c2, int c3) {
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %7, 0;\n\t"
      "@q cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];\n\t}" ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "r"(p)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// ------------------------------------------------------------------ tcgen05 / TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Makes this thread's generic-proxy shared-memory writes visible to later async-proxy readers (TMA
// stores, tcgen05 MMAs) once a barrier orders them.
__device__ __forceinline__ void fence_async_smem_cta() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrives once on `bar` when every tcgen05 op issued so far by this thread has completed.
__device__ __forceinline__ void tc_commit_p(uint32_t p, uint32_t bar) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %1, 0;\n\t"
               "@q tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(bar),
               "r"(p)
               : "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, f16 inputs, f32 accumulation. No memory clobber: the
// operands are ordered by the mbarrier waits (which carry one) and volatile asm keeps program order.
__device__ __forceinline__ void umma_f16_p(uint32_t p, uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred q, r;\n\t"
      "setp.ne.b32 q, %5, 0;\n\t"
      "setp.ne.b32 r, %4, 0;\n\t"
      "@q tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, r;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(p));
}
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Shared-memory matrix descriptor (tcgen05 format): K-major operand in the 128-byte swizzled
// canonical layout that a TMA SWIZZLE_128B load writes (rows of 64 halves, 8-row atoms 1024 B apart).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);  // start address, bits [0,14)
  d |= (uint64_t)1u << 16;                      // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;            // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1u << 46;                      // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;                      // SWIZZLE_128B
  return d;
}

// K-major operand whose rows are `row_bytes` (32, 64 or 128) long and stored under the TMA swizzle of
// the same span (SWIZZLE_32B / 64B / 128B): 8-row core-matrix groups 8 * row_bytes apart.
__device__ __forceinline__ uint64_t umma_desc_kmajor(uint32_t smem_addr, uint32_t row_bytes) {
  const uint64_t layout = row_bytes == 128u ? 2u : row_bytes == 64u ? 4u : 6u;
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);   // start address, bits [0,14)
  d |= (uint64_t)1u << 16;                       // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)((8u * row_bytes) >> 4) << 32;  // stride byte offset: 8 rows
  d |= (uint64_t)1u << 46;                       // descriptor version (sm_100)
  d |= layout << 61;                             // swizzle mode
  return d;
}

// Instruction descriptor: kind::f16, A = B = f16, D = f32, both K-major, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int m, int n) {
  return (1u << 4)                          // D format f32
         | (0u << 7) | (0u << 10)           // A, B format f16
         | ((uint32_t)(n >> 3) << 17)       // N >> 3
         | ((uint32_t)(m >> 4) << 24);      // M >> 4
}

// 32 lanes x 16 columns of 32-bit TMEM words into 16 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// Issue-only form: 16 columns into v[0..15] without waiting; call tmem_ld_wait16 on every loaded
// group after one tcgen05.wait::ld, which ties the registers to the wait (no use can move above it).
__device__ __forceinline__ void tmem_ld16_issue(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld_wait16(float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}

}  // namespace sdx
