// sm100.cuh -- thin inline-PTX layer for Blackwell (sm_100a): mbarriers with bounded waits,
// TMA bulk-tensor loads, tcgen05 (TMEM alloc / MMA / commit / ld / st), thread-block-cluster
// barriers and distributed shared memory.  Every kernel of this library is written on top of
// these helpers; nothing here is specific to one kernel.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>

#include "specq.h"

namespace specq {

// ------------------------------------------------------------------------------------------
// generic helpers
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Programmatic dependent launch (see LaunchAttrs): let the next kernel on the stream begin
// launching, and wait until the previous one has completed and its writes are visible.  Every
// kernel waits before its first global-memory load (only L2 prefetches, which cannot observe
// stale data, and tensor-map prefetches come before it) and triggers its dependents at its
// start (short kernels) or when its main loop is done (the GEMMs and attention); without the
// launch attribute both return at once.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint32_t warp_id() { return threadIdx.x >> 5; }
__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31; }

// One lane of the (converged) warp returns true.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---- optional pipeline tracing (compiled in only with -DSPECQ_TRACE) -------------------------
// One selected CTA records SM-clock timestamps of its pipeline events into a device buffer
// [slot][iteration] (64 x 64 uint64) configured through specq_trace_configure().
#ifdef SPECQ_TRACE
__device__ unsigned long long* g_specq_trace_buf = nullptr;
__device__ int g_specq_trace_cta = 0;
// Resolve once per kernel (at entry) whether this CTA records, so that each trace point is
// only a clock read and a store.
#define SPECQ_TRACE_INIT()                                                                    \
  const int specq_cta_ = static_cast<int>(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z)); \
  unsigned long long* specq_trace_ =                                                         \
      (specq_cta_ == ::specq::g_specq_trace_cta) ? ::specq::g_specq_trace_buf : nullptr;    \
  if (::specq::g_specq_trace_cta < 0 && ::specq::g_specq_trace_buf != nullptr && threadIdx.x == 0 && \
      specq_cta_ < 2048)                                                                      \
  ::specq::g_specq_trace_buf[2 * specq_cta_] = ::specq::globaltimer_ns()
#define SPECQ_TRACE_POINT(slot, iter)                                                         \
  do {                                                                                        \
    if (specq_trace_ != nullptr) specq_trace_[(slot) * 64 + min(static_cast<int>(iter), 63)] = clock64(); \
  } while (0)
// All-CTA mode (trace CTA < 0): every CTA records its start and end in %globaltimer ns.
#define SPECQ_TRACE_CTA_END()                                                                 \
  do {                                                                                        \
    if (::specq::g_specq_trace_cta < 0 && ::specq::g_specq_trace_buf != nullptr && threadIdx.x == 0 && \
        specq_cta_ < 2048)                                                                    \
      ::specq::g_specq_trace_buf[2 * specq_cta_ + 1] = ::specq::globaltimer_ns();            \
  } while (0)
#else
#define SPECQ_TRACE_INIT() \
  do {                     \
  } while (0)
#define SPECQ_TRACE_POINT(slot, iter) \
  do {                                \
  } while (0)
#define SPECQ_TRACE_CTA_END() \
  do {                        \
  } while (0)
#endif

// Maximum of v over the 32 lanes of the warp in one instruction (sm_100a redux.sync on f32).
// A maximum is exact, so the result does not depend on the reduction order.
__device__ __forceinline__ float warp_max_f32(float v) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}

// Record the first error code of a launch; later codes do not overwrite it.
__device__ __forceinline__ void report_status(int* status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

// Every wait of this library gives up after this long, reports kTimeout and lets the
// kernel wind down instead of spinning forever.
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s

// ------------------------------------------------------------------------------------------
// mbarrier
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Make mbarrier initialisation visible to the async proxy (TMA, tcgen05) and the cluster.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps (instead of spinning and taking issue
// slots from the working warps) until the phase completes or ~0.5 ms pass.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(500000u)
      : "memory");
  return ok != 0;
}

// Bounded wait for phase `parity` of `bar`.  Returns false (and records `code` in the status
// word) when the limit runs out; the caller then abandons its loop.
// The timer is read once every 16 suspended tries: a waiting warp wakes often, and a timer read
// on every wake costs the working warps issue slots.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if ((it & 15u) == 0u) {
      const uint64_t now = globaltimer_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > kWaitLimitNs) {
        report_status(status, code);
        return false;
      }
    }
  }
}

// System-scope release reduction / acquire load on a word another GPU writes or reads over
// NVLink (the tensor-parallel exchanges' counters).
__device__ __forceinline__ void red_release_sys_add_u32(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait (one thread) until every other rank's count in `flags` (this rank's flag array of
// an exchange, one slot per rank) has reached this rank's own count in slot `rank`: the peers'
// producers have landed as many blocks here as this rank's producer did.
__device__ __forceinline__ bool wait_peer_counts(const uint32_t* flags, int rank, int world, int* status) {
  const uint32_t target = ld_acquire_sys_u32(flags + rank);
  const uint64_t t0 = globaltimer_ns();
  for (int q = 0; q < world; ++q) {
    if (q == rank) continue;
    while (static_cast<int32_t>(ld_acquire_sys_u32(flags + q) - target) < 0) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        report_status(status, SPECQ_STATUS_TIMEOUT_PEER);
        return false;
      }
    }
  }
  return true;
}

// Bounded wait that sleeps between polls, for waiters whose wake-up latency a pipeline hides
// (a producer waiting for a free stage, a converter or the MMA issuer waiting for its inputs):
// a polling warp takes an issue slot on every try, a sleeping one leaves them to the warps
// doing the arithmetic.  Returns false (and records `code`) when the wait limit runs out.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t sleep_ns, int* status,
                                                int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    __nanosleep(sleep_ns);
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      report_status(status, code);
      return false;
    }
  }
}

// 16-byte read-only global load issued where it stands: volatile, so the compiler keeps it in
// program order with the other volatile operations (ahead of a barrier, say) and its latency
// overlaps what follows instead of being paid where the value is first used.
__device__ __forceinline__ uint4 ldg_nc_v4_now(const void* ptr) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(ptr));
  return v;
}

// 4-byte cp.async global -> shared (4- and 8-byte copies take the L1-allocating .ca form).
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// wait until at most N of this thread's committed cp.async groups are still in flight
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Arrive on an mbarrier when all of this thread's earlier cp.async copies have landed.
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// ------------------------------------------------------------------------------------------
// proxy fences
// ------------------------------------------------------------------------------------------
// Generic-proxy writes to shared memory become visible to the async proxy (tcgen05.mma
// operand reads, TMA) after this fence.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor), no multicast anywhere in this library
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// L2 prefetch of one box of a tensor map (no shared memory, no barrier, no completion).  The
// kernels issue it before griddepcontrol.wait for operands whose addresses do not depend on the
// previous kernel's results, so the first HBM round trip overlaps that kernel's tail.  It only
// warms L2, through which every SM write passes, so it is correct even for data the previous
// grid is still writing: the later TMA load reads the current contents.
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void tma_prefetch_l2_4d(const CUtensorMap* map, int x, int y, int z, int w) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            uint64_t cache_hint) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(cache_hint)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            int z, uint64_t cache_hint) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "l"(cache_hint)
      : "memory");
}

// L2 cache policies (createpolicy): streamed-once weights vs re-read activations.
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

// ------------------------------------------------------------------------------------------
// tcgen05: tensor memory and the 5th-generation tensor core
// ------------------------------------------------------------------------------------------
// Allocate `ncols` (power of two, >= 32) TMEM columns; the base address is written to smem.
// Executed by one full warp.
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

// D[tmem] (+)= A[smem] * B[smem]^T, INT8 x INT8 -> INT32.
__device__ __forceinline__ void umma_i8_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, FP16 x FP16 -> FP32.
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, FP16 -> FP32 (A read from tensor memory).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on `bar` when every tcgen05 operation issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Instruction descriptor (kind::f16 / kind::i8), dense, no negate, no saturation.
//   bits 4-5 D format (1 = f32, 2 = s32), 7-9 A format, 10-12 B format (f16: 0 = f16;
//   i8: 1 = signed), 15 A major, 16 B major (0 = K-major, 1 = MN-major), 17-22 N >> 3,
//   24-28 M >> 4.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t d_fmt, uint32_t a_fmt, uint32_t b_fmt,
                                                  uint32_t a_mn_major, uint32_t b_mn_major, uint32_t m,
                                                  uint32_t n) {
  return (d_fmt << 4) | (a_fmt << 7) | (b_fmt << 10) | (a_mn_major << 15) | (b_mn_major << 16) |
         ((n >> 3) << 17) | ((m >> 4) << 24);
}
__device__ __forceinline__ uint32_t idesc_i8(uint32_t m, uint32_t n) { return make_idesc(2, 1, 1, 0, 0, m, n); }
__device__ __forceinline__ uint32_t idesc_f16(uint32_t m, uint32_t n, uint32_t a_mn = 0, uint32_t b_mn = 0) {
  return make_idesc(1, 0, 0, a_mn, b_mn, m, n);
}

// Shared-memory matrix descriptor for the 128-byte-swizzle canonical layouts.
//   K-major:  8-row x 128-byte atoms, rows 128 B apart, atom groups `sbo` bytes apart along
//             M/N (lbo unused).  Advancing K inside the atom = adding bytes to the address.
//   MN-major: 8 K-rows x 128 contiguous MN bytes per atom; `lbo` = byte distance between
//             atoms along MN, `sbo` = byte distance between 8-row groups along K.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
  d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
  return d;
}

// Shared-memory matrix descriptor, no swizzle (8-row x 16-byte core matrices; `lbo` / `sbo`
// the byte distances between core matrices along K / along M-N).
__device__ __forceinline__ uint64_t sdesc_plain(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100; layout 0 = no swizzle
  return d;
}


// Byte offset of the 16-byte chunk `chunk` (0..7) of row `row` inside a 128-byte-swizzled
// tile whose 8-row atoms are stored contiguously (1024 B per atom).
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

// TMEM -> registers: 32 lanes x 32 bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
      "%13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
      "%13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------------------------------------
// thread-block clusters and distributed shared memory
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
// Full cluster barrier (all threads of all CTAs), release/acquire.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Cluster barrier in two halves: arrive early, wait only where the peers' state is needed.
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Bulk asynchronous reduction (u32 add) of `bytes` bytes of this CTA's shared memory into a
// peer CTA's shared memory, counted on the peer's mbarrier (complete_tx).  dst_cluster and
// bar_cluster are shared::cluster addresses (dsmem_map); 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_reduce_add_u32_cluster(uint32_t dst_cluster, uint32_t src_cta, uint32_t bytes,
                                                            uint32_t bar_cluster) {
  asm volatile(
      "cp.reduce.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes.add.u32 [%0], [%1], %2, [%3];" ::"r"(
          dst_cluster),
      "r"(src_cta), "r"(bytes), "r"(bar_cluster)
      : "memory");
}

// Map a local shared-memory address to the same offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t dsmem_map(uint32_t local_saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_saddr), "r"(rank));
  return r;
}
// Generic address of the same shared-memory object in CTA `rank` of the cluster; ordinary
// loads through it can be scheduled (batched) by the compiler.
template <typename T>
__device__ __forceinline__ const T* dsmem_ptr(const T* local, uint32_t rank) {
  uint64_t r;
  asm("mapa.u64 %0, %1, %2;" : "=l"(r) : "l"(reinterpret_cast<uint64_t>(local)), "r"(rank));
  return reinterpret_cast<const T*>(r);
}

__device__ __forceinline__ uint4 dsmem_ld_v4(uint32_t cluster_saddr) {
  uint4 v;
  asm volatile("ld.shared::cluster.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(cluster_saddr)
               : "memory");
  return v;
}
__device__ __forceinline__ float dsmem_ld_f32(uint32_t cluster_saddr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_saddr) : "memory");
  return v;
}

__device__ __forceinline__ void dsmem_st_f32(uint32_t cluster_saddr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(cluster_saddr), "f"(v) : "memory");
}
__device__ __forceinline__ void dsmem_st_v4(uint32_t cluster_saddr, uint4 v) {
  asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(cluster_saddr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void dsmem_st_v2f32(uint32_t cluster_saddr, float a, float b) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(cluster_saddr), "f"(a), "f"(b) : "memory");
}

// Named barrier for a subset of warps (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace specq
