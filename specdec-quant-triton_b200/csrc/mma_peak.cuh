// mma_peak.cuh -- tensor-pipe throughput microbenchmark (no reference counterpart).
//
// The roofline of the GEMMs at large M needs the dense INT8 tensor peak of this GPU; the pool
// measures only copy bandwidth and a cuBLAS bf16 GEMM.  This kernel measures the tcgen05 pipe
// directly: one CTA per SM keeps a [128 x 128 B] A tile and a [256 x 128 B] B tile resident in
// shared memory (128B-swizzled, K-major) and one elected thread issues back-to-back
// M=128 x N=256 MMAs (kind::i8: K=32 per instruction; kind::f16: K=16) into two alternating
// TMEM accumulators.  Nothing is loaded from global memory in the loop, so the time of a launch
// is the tensor pipe's.  The kind::f16 variant cross-checks the method against the measured
// cuBLAS bf16 figure.  The only global write is one word per CTA (a checksum of its accumulator
// lane 0) so the work cannot be elided.
#pragma once

#include "sm100.cuh"

namespace specq {

constexpr int kPeakThreads = 128;
constexpr uint32_t kPeakATile = 128 * 128;   // bytes
constexpr uint32_t kPeakBTile = 256 * 128;

template <int KIND>   // 0 = kind::i8 (s8 x s8 -> s32), 1 = kind::f16 (fp16 x fp16 -> fp32)
__global__ void __launch_bounds__(kPeakThreads, 1) mma_peak_kernel(int iters, int* status, uint32_t* sink) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_tile = smem;
  uint8_t* b_tile = a_tile + kPeakATile;
  uint64_t* done = reinterpret_cast<uint64_t*>(b_tile + kPeakBTile);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  const uint32_t warp = warp_id();

  // operand bytes: a per-CTA xorshift stream (int8 values, or fp16 values in [-2, 2])
  uint32_t x = 0x9E3779B9u ^ (blockIdx.x * 2654435761u) ^ (threadIdx.x * 40503u);
  for (uint32_t i = threadIdx.x; i < (kPeakATile + kPeakBTile) / 4; i += kPeakThreads) {
    x ^= x << 13;
    x ^= x >> 17;
    x ^= x << 5;
    uint32_t v = x;
    if (KIND == 1) v = (v & 0x83FF83FFu) | 0x3C003C00u;   // sign, mantissa; exponent of 1.0
    reinterpret_cast<uint32_t*>(smem)[i] = v;
  }
  if (threadIdx.x == 0) {
    mbar_init(done, 1u);
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

  if (warp == 0 && elect_one()) {
    const uint64_t ad = sdesc_sw128(smem_u32(a_tile), 16u, 1024u);
    const uint64_t bd = sdesc_sw128(smem_u32(b_tile), 16u, 1024u);
    const uint32_t idesc = KIND == 0 ? idesc_i8(128, 256) : idesc_f16(128, 256);
    for (int it = 0; it < iters; ++it) {
      const uint32_t acc = tmem + 256u * static_cast<uint32_t>(it & 1);
#pragma unroll
      for (int k = 0; k < 4; ++k) {   // 32 bytes of K per instruction, 128 bytes per pass
        if (KIND == 0)
          umma_i8_ss(acc, ad + 2u * k, bd + 2u * k, idesc, (it > 1 || k > 0) ? 1u : 0u);
        else
          umma_f16_ss(acc, ad + 2u * k, bd + 2u * k, idesc, (it > 1 || k > 0) ? 1u : 0u);
      }
    }
    umma_commit(done);
  }
  __syncwarp();
  // every thread waits for the MMAs (bounded), then warp 0 reads lane 0..31 of column 0
  const bool ok = mbar_wait(done, 0u, status, SPECQ_STATUS_TIMEOUT_MMA);
  tc_fence_after();
  if (warp == 0) {
    uint32_t r[8];
    tmem_ld8(tmem, r);
    tmem_wait_ld();
    uint32_t h = r[0] ^ r[1] ^ r[2] ^ r[3] ^ r[4] ^ r[5] ^ r[6] ^ r[7];
    for (int o = 16; o > 0; o >>= 1) h ^= __shfl_xor_sync(0xffffffffu, h, o);
    if (lane_id() == 0 && ok) sink[blockIdx.x] = h;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512u);
  }
}

constexpr int kPeakSmem = 1024 + static_cast<int>(kPeakATile + kPeakBTile) + 64;

}  // namespace specq
