// Thin inline-PTX wrappers for the sm_100a features the MaxSim kernels use:
// mbarriers, TMA tensor loads, tcgen05 (MMA, TMEM alloc/ld, commit, fences)
// and bounded waits that report a status word instead of trapping.
//
// Written from the PTX ISA descriptions of these instructions; the shared
// memory / instruction descriptor bit layouts follow the tcgen05 "matrix
// descriptor" and "instruction descriptor" tables of the PTX ISA.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

#include "../../include/flash_maxsim_sm100.h"

namespace fm {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
// try_wait suspends the waiting thread until the phase completes or this many
// nanoseconds pass (the bounded-wait loop re-checks its limit after each try):
// waiting warps sleep instead of spinning, which measurably helps long runs
// under the power cap. -DFM_NO_TRYWAIT_HINT builds the plain form.
#if !defined(FM_TRYWAIT_HINT) && !defined(FM_NO_TRYWAIT_HINT)
#define FM_TRYWAIT_HINT 1000000
#endif
#ifdef FM_TRYWAIT_HINT
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "n"(FM_TRYWAIT_HINT)
      : "memory");
#else
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
#endif
  return ok != 0;
}

// Non-blocking probe of an mbarrier phase.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Shared control block of one CTA: an abort flag in shared memory that every
// role polls while it waits, the caller's global status word and the wait
// limit.  The first wait that runs out of time records its code, raises the
// abort flag, and every other role leaves its loop at its next wait.
struct WaitCtl {
  volatile int* abort_flag;  // shared memory
  int* status;               // global, may not be null
  uint64_t timeout_ns;
};

__device__ __forceinline__ void record_status(int* status, int code) {
  atomicCAS(status, 0, code);
}

#ifdef FM_TUNING
// Tuning builds only (never shipped): the launch plan's `dbg` bits switch off
// parts of the work (MMAs, epilogue reads, waits) to measure what is left.
#define FM_DBG(a, bits) (((a).dbg & (bits)) != 0)
#else
#define FM_DBG(a, bits) false
#endif

#ifdef FM_PROFILE
// Profiling builds only (never shipped): cycles spent in each kind of wait
// (indexed by its timeout code) and in a few named sections, summed over the
// lane-0 threads of every CTA.
__device__ unsigned long long g_fm_prof[32];
#define FM_PROF_T0(v) const long long v = clock64()
#define FM_PROF_ADD(code, t0)                                                                  \
  do {                                                                                         \
    if ((threadIdx.x & 31) == 0)                                                               \
      atomicAdd(&g_fm_prof[code], static_cast<unsigned long long>(clock64() - (t0)));          \
  } while (0)
#else
#define FM_PROF_T0(v)
#define FM_PROF_ADD(code, t0) \
  do {                        \
  } while (0)
#endif

#ifdef FM_TRACE
// Tracing builds only (never shipped): timestamped events of the lane-0
// threads of CTA 0, one channel of 4096 entries per role, (clock64 << 8) | code.
__device__ unsigned long long g_fm_trace[8 * 4096];
#define FM_TR_DECL int tr_n_ = 0
#define FM_TR(ch, code)                                                                          \
  do {                                                                                           \
    if (blockIdx.x == 0 && (threadIdx.x & 31) == 0 && tr_n_ < 4096)                              \
      g_fm_trace[(ch) * 4096 + tr_n_++] = (static_cast<unsigned long long>(clock64()) << 8) | (code); \
  } while (0)
#else
#define FM_TR_DECL
#define FM_TR(ch, code) \
  do {                  \
  } while (0)
#endif

// Bounded wait on an mbarrier phase. Returns false when the CTA is aborting
// (this wait ran out of time, or another role's did).
__device__ __forceinline__ bool mbar_wait_impl(uint32_t bar, uint32_t parity, const WaitCtl& ctl,
                                               int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#ifdef FM_WAIT_SLEEP
    __nanosleep(FM_WAIT_SLEEP);
#endif
    if (mbar_try_wait(bar, parity)) return true;
    if (*ctl.abort_flag) return false;
    if (globaltimer_ns() - t0 > ctl.timeout_ns) {
      *ctl.abort_flag = 1;
      record_status(ctl.status, code);
      return false;
    }
  }
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const WaitCtl& ctl,
                                          int code) {
#ifdef FM_PROFILE
  FM_PROF_T0(c0);
  const bool r = mbar_wait_impl(bar, parity, ctl, code);
  FM_PROF_ADD(code & 31, c0);
  return r;
#else
  return mbar_wait_impl(bar, parity, ctl, code);
#endif
}

// ---------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor), no multicast anywhere in this library
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// Programmatic dependent launch: block until the grids this launch depends
// on have completed (a no-op when launched without the attribute), and let
// the next launch in the stream start its prologue early.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, int x, int y, int z,
                                            uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(bar), "l"(policy)
      : "memory");
}

// Untiled bulk copy global -> shared (16-byte aligned addresses, size % 16 == 0).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05
// ---------------------------------------------------------------------------
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
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16, fp32 accumulate, one CTA.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::i8 (8-bit integers, s32 accumulate).
__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor, kind::i8: D s32 [4,6)=2, A signed 8-bit [7,10)=1,
// B unsigned 8-bit [10,13)=0, both K-major, N>>3 at [17,23), M>>4 at [24,29).
__host__ __device__ __forceinline__ uint32_t idesc_s8u8_s32(int M, int N) {
  return (2u << 4) | (1u << 7) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// Shared-memory matrix descriptor for a K-major operand stored in the
// 128-byte-swizzled canonical layout: rows of 64 fp16 (128 B), 8-row groups
// 1024 B apart.  Fields: start>>4 [0,14), leading byte offset>>4 [16,30)
// (unused for swizzled K-major; 1), stride byte offset>>4 [32,46) = 1024>>4,
// descriptor version 1 at [46,48), swizzle mode 2 (128 B) at [61,64).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor, kind::f16: D fp32 [4,6)=1, A/B fp16 (0), both
// K-major, N>>3 at [17,23), M>>4 at [24,29).
__host__ __device__ __forceinline__ uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// 32 lanes x 32 consecutive fp32 columns from TMEM into registers.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// One fp32 column of 32 lanes to / from TMEM (per-row scratch values).
__device__ __forceinline__ void tmem_st1(uint32_t taddr, float v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(__float_as_uint(v))
               : "memory");
}
__device__ __forceinline__ float tmem_ld1(uint32_t taddr) {
  uint32_t r;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr) : "memory");
  return __uint_as_float(r);
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// three-input maximum (sm_100 adds a 3-operand max.f32)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Two fp32 fused multiply-adds in one instruction (sm_100 fma.rn.f32x2):
// (d0, d1) = (a0 * b0 + c0, a1 * b1 + c1), each rounded once.
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1,
                                      float c0, float c1) {
  uint64_t a, b, c, d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(b) : "f"(b0), "f"(b1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(c) : "f"(c0), "f"(c1));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d0), "=f"(d1) : "l"(d));
}

// Maximum over the 32 lanes of one float, returned to every lane
// (sm_100a: redux.sync on f32).
__device__ __forceinline__ float warp_max_f32(float x) {
  float r;
  asm("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(x));
  return r;
}

// Column maxima of a 32 x 32 tile held one row per lane (v[j] = column j):
// one warp reduction per column, then lane j picks column j's maximum by a
// five-level select tree (fewer and shorter dependent steps than a
// 31-shuffle transpose-and-max butterfly).
__device__ __forceinline__ float colmax32(float (&v)[32], int lane) {
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = warp_max_f32(v[j]);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
#pragma unroll
    for (int i = 0; i < o; ++i) v[i] = (lane & o) ? v[i + o] : v[i];
  }
  return v[0];
}

}  // namespace fm
