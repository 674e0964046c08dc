// mma_peak.cuh -- tensor-pipe throughput microbenchmark (no reference counterpart).
//
// The roofline of the GEMMs at large M needs the dense INT8 tensor peak of this GPU; the pool
// measures only copy bandwidth and a cuBLAS bf16 GEMM.  This kernel measures the tcgen05 pipe
// directly: one CTA per SM keeps a [128 x 128 B] A tile and a [256 x 128 B] B tile resident in
// shared memory (128B-swizzled) and one elected thread issues back-to-back M=128 MMAs
// (kind::i8: K=32 per instruction; kind::f16: K=16) of N columns into two alternating TMEM
// accumulators.  Nothing is loaded from global memory in the loop, so the time of a launch is
// the tensor pipe's.  The kind::f16 variant cross-checks the method against the measured
// cuBLAS bf16 figure.
//
// The same kernel also prices the small MMAs of the attention kernel: N below 256, operands
// K-major or MN-major, the A operand from tensor memory, and `busy_warps` extra warps that
// stream 16-byte shared-memory loads and stores (the traffic of softmax / conversion warps)
// while the MMAs run.  The only global write is one word per CTA (a checksum of its
// accumulator lane 0) so the work cannot be elided.
#pragma once

#include "sm100.cuh"

namespace specq {

constexpr int kPeakThreads = 128;
constexpr uint32_t kPeakATile = 128 * 128;   // bytes
constexpr uint32_t kPeakBTile = 256 * 128;
constexpr uint32_t kPeakBusyBytes = 32 * 1024;   // the busy warps' shared-memory region

struct MmaPeakParams {
  int iters;
  uint32_t n;           // MMA N (multiple of 16, <= 256)
  uint32_t a_mn, b_mn;  // operand majorness (1 = MN-major)
  int a_tmem;           // kind::f16 only: A operand from tensor memory
  int busy_warps;       // extra warps streaming shared memory during the MMAs
  int busy_iters;       // 16-byte loads + stores per busy thread
  int* status;
  uint32_t* sink;
};

template <int KIND>   // 0 = kind::i8 (s8 x s8 -> s32), 1 = kind::f16 (fp16 x fp16 -> fp32)
__global__ void __launch_bounds__(1024, 1) mma_peak_kernel(const __grid_constant__ MmaPeakParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_tile = smem;
  uint8_t* b_tile = a_tile + kPeakATile;
  uint8_t* busy = b_tile + kPeakBTile;
  uint64_t* done = reinterpret_cast<uint64_t*>(busy + kPeakBusyBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* mma_done_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const uint32_t warp = warp_id();

  // operand bytes: a per-CTA xorshift stream (int8 values, or fp16 values in [-2, 2])
  uint32_t x = 0x9E3779B9u ^ (blockIdx.x * 2654435761u) ^ (threadIdx.x * 40503u);
  for (uint32_t i = threadIdx.x; i < (kPeakATile + kPeakBTile + kPeakBusyBytes) / 4; i += blockDim.x) {
    x ^= x << 13;
    x ^= x >> 17;
    x ^= x << 5;
    uint32_t v = x;
    if (KIND == 1) v = (v & 0x83FF83FFu) | 0x3C003C00u;   // sign, mantissa; exponent of 1.0
    reinterpret_cast<uint32_t*>(smem)[i] = v;
  }
  if (threadIdx.x == 0) {
    mbar_init(done, 1u);
    *mma_done_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512u);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (KIND == 1 && p.a_tmem && warp < 4) {   // A operand in TMEM columns [384, 392): fp16 1.0
    uint32_t ones[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) ones[i] = 0x3C003C00u;
    tmem_st8(tmem + ((warp * 32u) << 16) + 384u, ones);
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp == 0) {
    if (elect_one()) {
      // K-major: 8-row x 128 B atoms, 1024 B apart along M/N.  MN-major: 128 MN-bytes x 8 K-rows
      // per atom; atoms along MN `lbo` apart, 8-row K groups 1024 B apart (inside the tiles).
      const uint64_t ad = p.a_mn ? sdesc_sw128(smem_u32(a_tile), 8192u, 1024u) : sdesc_sw128(smem_u32(a_tile), 16u, 1024u);
      const uint64_t bd = p.b_mn ? sdesc_sw128(smem_u32(b_tile), 8192u, 1024u) : sdesc_sw128(smem_u32(b_tile), 16u, 1024u);
      const uint32_t idesc = KIND == 0 ? make_idesc(2, 1, 1, p.a_mn, p.b_mn, 128, p.n)
                                       : make_idesc(1, 0, 0, p.a_mn, p.b_mn, 128, p.n);
      for (int it = 0; it < p.iters; ++it) {
        const uint32_t acc = tmem + (p.n <= 128u ? 128u : 256u) * static_cast<uint32_t>(it & 1);
#pragma unroll
        for (int k = 0; k < 4; ++k) {   // 32 bytes of K per instruction, 128 bytes per pass
          const uint32_t on = (it > 1 || k > 0) ? 1u : 0u;
          if (KIND == 0)
            umma_i8_ss(acc, ad + 2u * k, bd + 2u * k, idesc, on);
          else if (p.a_tmem)
            umma_f16_ts(acc, tmem + 384u, bd + 2u * k, idesc, on);
          else
            umma_f16_ss(acc, ad + 2u * k, bd + 2u * k, idesc, on);
        }
      }
      umma_commit(&done[0]);
    }
    __syncwarp();
    // the MMAs have completed (bounded wait): the busy warps stop
    if (lane_id() == 0) {
      (void)mbar_wait(done, 0u, p.status, SPECQ_STATUS_TIMEOUT_MMA);
      *mma_done_flag = 1;
    }
  } else if (warp >= 4 && static_cast<int>(warp) < 4 + p.busy_warps) {
    // busy warps: 16-byte shared loads and stores over their own region
    const uint32_t t = threadIdx.x - 128u;
    uint4* reg = reinterpret_cast<uint4*>(busy);
    uint4 acc = make_uint4(0u, 0u, 0u, 0u);
    // until the MMAs have completed (checked every 8 iterations), at most busy_iters
    for (int i = 0; i < p.busy_iters && ((i & 7) != 0 || *mma_done_flag == 0); ++i) {
      const uint32_t idx = (t + 32u * static_cast<uint32_t>(i)) & (kPeakBusyBytes / 16u - 1u);
      const uint4 v = reg[idx];
      acc.x ^= v.x; acc.y += v.y; acc.z ^= v.z; acc.w += v.w;
      reg[idx ^ 1u] = acc;
    }
    if (acc.x == 0x12345678u && p.sink != nullptr) p.sink[0] = acc.y;   // keeps the loop
  }
  __syncwarp();
  // every thread waits for the MMAs (bounded), then warp 0 reads lane 0..31 of column 0
  const bool ok = mbar_wait(done, 0u, p.status, SPECQ_STATUS_TIMEOUT_MMA);
  tc_fence_after();
  if (warp == 0) {
    uint32_t r[8];
    tmem_ld8(tmem, r);
    tmem_wait_ld();
    uint32_t h = r[0] ^ r[1] ^ r[2] ^ r[3] ^ r[4] ^ r[5] ^ r[6] ^ r[7];
    for (int o = 16; o > 0; o >>= 1) h ^= __shfl_xor_sync(0xffffffffu, h, o);
    if (lane_id() == 0 && ok) p.sink[blockIdx.x] = h;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512u);
  }
}

constexpr int kPeakSmem = 1024 + static_cast<int>(kPeakATile + kPeakBTile + kPeakBusyBytes) + 64;

}  // namespace specq
