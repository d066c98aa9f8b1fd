// sm100.cuh -- inline-PTX primitives for Blackwell (sm_100a): mbarriers, TMA,
// tcgen05 (TMEM allocation, UMMA issue/commit, TMEM loads) and descriptors.
//
// Written from the PTX ISA (tcgen05, cp.async.bulk.tensor, mbarrier sections)
// and the descriptor bit layouts of CUTLASS's cute/arch/mma_sm100_desc.hpp.
// Replaces the reference's blackwell.h, whose smem descriptor lacks the
// version field and whose tcgen05 forms do not assemble for sm_100a.
//
// Every wait is bounded: a spin that exceeds time limit (clock64 cycles for pipeline waits) sets a bit
// in a device error word and raises a CTA-wide abort flag instead of hanging.
#pragma once
#include <cstdint>
#include <cuda.h>

#ifndef GEMMS_WAIT_TIMEOUT_NS
#define GEMMS_WAIT_TIMEOUT_NS 4000000000ull  // 4 s (drain waits, %globaltimer)
#endif
#ifndef GEMMS_WAIT_TIMEOUT_CYCLES
#define GEMMS_WAIT_TIMEOUT_CYCLES 8000000000ll  // ~4 s at 2 GHz (pipeline waits, clock64)
#endif

namespace gemms {
namespace sm100 {

constexpr uint32_t kSuspendHintNs = 1000000;  // 1 ms; waiters resume on phase completion

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// try_wait with a suspend-time hint: a waiting thread sleeps until the phase
// completes (or the hint expires) instead of spinning, leaving issue slots to
// the warps that share its SM sub-partition.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

// Waits for the phase with `parity` to complete.  Returns false (after
// setting *abort and OR-ing `code` into *err) when the wait exceeds
// `limit_cycles`, or as soon as another role has raised *abort.  The timeout
// runs on the SM cycle counter (cheap to read); the abort flag is read every
// 256 polls and the clock every `clock_every` polls (a multiple of 256);
// reading %globaltimer on every miss added ~1 us to each pipeline hand-off.
// A suspended poll can last up to the suspend hint, so a lone waiting thread's
// first clock check can come long after `limit_cycles`, while a warp of
// polling lanes checks far sooner: a role that waits on another role's wait
// passes a larger limit (and `clock_every`), so that the role nearest a lost
// stage is the one that reports it.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int* err, int code, long long limit_cycles = GEMMS_WAIT_TIMEOUT_CYCLES,
                                          uint32_t clock_every = 256u) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  uint32_t n = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++n & 255u) == 0) {
      if (*abort_flag) return false;
      if (n % clock_every == 0 && clock64() - t0 > limit_cycles) {
        *abort_flag = 1;
        atomicOr(err, code);
        return false;
      }
    }
  }
  return true;
}

// Named barrier over `nthreads` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// -------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// L2 eviction policies for cache hints.
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 2-D tiled TMA load into this CTA's shared memory, completing on `bar`.
// x (innermost, bytes for 8-bit data) must be a multiple of 16.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Prefetch a 2-D tile into L2 (no shared memory, no completion tracking).
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int x, int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.prefetch.tensor.2d.L2.global.tile.L2::cache_hint [%0, {%1, %2}], %3;" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// ---------------------------------------------------------------- tcgen05
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

// D[tmem] (+)= A[smem] * B[smem]^T, e4m3 x e4m3 -> fp32, issued by one thread.
__device__ __forceinline__ void umma_f8f6f4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on `bar` when all previously issued tcgen05 ops of this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Each thread of the warp reads 32 consecutive 32-bit columns of its TMEM lane.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Hardware reciprocal approximation (MUFU, flush-to-zero); 1/inf = 0.
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// (a0, a1) += f * (v0, v1) as one packed fp32x2 FMA (sm_100 f32x2 pipe).
__device__ __forceinline__ void ffma2(float& a0, float& a1, float f, float v0, float v1) {
  asm("{\n\t.reg .b64 acc, fv, vv;\n\t"
      "mov.b64 acc, {%0, %1};\n\t"
      "mov.b64 fv, {%2, %2};\n\t"
      "mov.b64 vv, {%3, %4};\n\t"
      "fma.rn.f32x2 acc, fv, vv, acc;\n\t"
      "mov.b64 {%0, %1}, acc;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(f), "f"(v0), "f"(v1));
}

// ------------------------------------------------------------ descriptors
// Shared-memory matrix descriptor for a K-major operand in the 128-byte
// swizzle canonical layout: rows of 128 bytes, 8-row atoms of 1024 bytes
// stacked at a 1024-byte stride (SBO).  Bits: [0,14) start>>4, [16,30) LBO>>4
// (unused for swizzled K-major, set to 1), [32,46) SBO>>4, [46,48) version=1,
// [49,52) base offset=0 (atoms 1024-aligned), [61,64) layout=2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor, kind::f8f6f4: D fp32, A and B e4m3, both K-major.
// Bits: [4,6) D format (1 = f32), [7,10) A format (0 = e4m3), [10,13) B format,
// [15] A major (0 = K), [16] B major, [17,23) N>>3, [24,29) M>>4.
__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int M, int N) {
  return (1u << 4) | (0u << 7) | (0u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

}  // namespace sm100
}  // namespace gemms
