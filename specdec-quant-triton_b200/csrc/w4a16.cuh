// w4a16.cuh -- W4A16 GEMM (fp16 activations x packed INT4 weights) on sm_100a.
//
// out[m, n] = fp16( sum_k a[m,k] * fp16(q[n,k] * sc[n, k/group]) ), q in [-8, 7], packed split-half:
// byte j of row n holds q[n,j]+8 (low nibble) and q[n,j+K/2]+8 (high nibble)
// (reference kernel: kernels.py:95-135, packing kernels.py:90-92 / 143-145).
//
// Design:
//   * Swap-AB as in the W8A8 kernel: tensor-core M=128 over weight channels, N over the
//     CTA's tokens (up to 256), FP32 accumulators in TMEM.
//   * Per packed K-block (64 bytes = 64 "low" + 64 "high" K-elements) TMA brings the packed
//     [128 x 64 B] weight tile and the two matching [tokens x 64] fp16 activation tiles
//     (128-byte swizzle).  Eight dequant warps turn the packed tile into two fp16 operand
//     tiles ONCE per K-block for all tokens of the CTA -- the reference redoes this for
//     every BLOCK_M rows (kernels.py:112-133), which is the cost the rebuild removes.
//   * Dequant = byte-permute + LOP3 into the fp16 exponent 2^10 ("1024 + nibble"), an exact
//     subtract / fma to q, then one fp16 multiply by the group scale: the same single
//     rounding as `lo.to(fp16) * sc` in the reference (kernels.py:126-127).
//   * Split-K over a cluster, reduced through DSMEM in a fixed rank order, so the result
//     depends only on (N, K) -- plan mode and non-plan mode give identical bits.
#pragma once

#include "gemm_common.cuh"

namespace specq {

struct W4A16Params {
  const __half* a;     // [m_rows, K], row stride lda elements
  const uint8_t* wp;   // [N, K/2], row stride ldwp bytes
  const __half* sc;    // [N, K/group], row stride ldsc elements
  __half* out;         // strides (ldo, ldo_n)
  const int32_t* plan;
  int* status;
  int64_t lda, ldwp, ldsc, ldo, ldo_n;
  int m_rows, N, K, group;
  int group_shift;     // log2(group) when group is a power of two, else -1
  int chunk;           // tokens per CTA (multiple of 16, <= 256)
  int kb_total;        // packed 64-byte blocks per row = K / 128
  int kb_per_split;
  int splits;
  int stages;          // TMA ring depth
  int dstages;         // dequantised-operand ring depth
  uint32_t stage_bytes;
  uint32_t sc_cache_cols;  // groups per row of the TMA-loaded scale tile (0: prefetch per K-block)
  uint32_t tmem_cols;
};

constexpr int kW4A16DequantWarps = 16;
constexpr int kW4A16DequantThreads = 32 * kW4A16DequantWarps;
// The dequant warps form two groups that take alternate K-blocks, so two blocks are being
// dequantised at any time (a single block's chain of smem load -> convert -> store -> fence
// is latency-bound).
constexpr int kW4A16Groups = 2;
constexpr int kW4A16GroupWarps = kW4A16DequantWarps / kW4A16Groups;
constexpr int kW4A16GroupThreads = 32 * kW4A16GroupWarps;
constexpr int kW4A16Threads = 64 + kW4A16DequantThreads;   // warp 0 TMA, warp 1 MMA, then dequant (2..5 epilogue)
constexpr uint32_t kW4A16PackTile = 128 * 64;   // packed bytes per stage
constexpr uint32_t kW4A16OpTile = 128 * 128;    // one fp16 [128 x 64] operand tile
constexpr uint32_t kW4A16DSlot = 2 * kW4A16OpTile;

// 16 packed bytes (packed columns j..j+15 of one row) -> 16 low-half weights (k = j..j+15)
// and 16 high-half weights (k = j+K/2 ..), each already multiplied by its fp16 group scale.
__device__ __forceinline__ void dequant_chunk(uint4 pk, __half2 slo, __half2 shi, uint4 (&lo)[2], uint4 (&hi)[2]) {
  const uint32_t w[4] = {pk.x, pk.y, pk.z, pk.w};
  const __half2 k1032 = __half2half2(__ushort_as_half(0x6408));       // 1032.0
  const __half2 k1_16 = __half2half2(__ushort_as_half(0x2C00));       // 0.0625
  const __half2 km72 = __half2half2(__ushort_as_half(0xD480));        // -72.0
  uint32_t ol[8], oh[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t p01 = __byte_perm(w[i], 0u, 0x4140);   // [b0, 0, b1, 0]
    const uint32_t p23 = __byte_perm(w[i], 0u, 0x4342);   // [b2, 0, b3, 0]
    const uint32_t l01 = (p01 & 0x000F000Fu) | 0x64006400u;  // fp16 1024 + low nibble
    const uint32_t l23 = (p23 & 0x000F000Fu) | 0x64006400u;
    const uint32_t h01 = (p01 & 0x00F000F0u) | 0x64006400u;  // fp16 1024 + 16 * high nibble
    const uint32_t h23 = (p23 & 0x00F000F0u) | 0x64006400u;
    __half2 ql01 = __hsub2(*reinterpret_cast<const __half2*>(&l01), k1032);
    __half2 ql23 = __hsub2(*reinterpret_cast<const __half2*>(&l23), k1032);
    __half2 qh01 = __hfma2(*reinterpret_cast<const __half2*>(&h01), k1_16, km72);
    __half2 qh23 = __hfma2(*reinterpret_cast<const __half2*>(&h23), k1_16, km72);
    ql01 = __hmul2(ql01, slo);
    ql23 = __hmul2(ql23, slo);
    qh01 = __hmul2(qh01, shi);
    qh23 = __hmul2(qh23, shi);
    ol[2 * i] = *reinterpret_cast<uint32_t*>(&ql01);
    ol[2 * i + 1] = *reinterpret_cast<uint32_t*>(&ql23);
    oh[2 * i] = *reinterpret_cast<uint32_t*>(&qh01);
    oh[2 * i + 1] = *reinterpret_cast<uint32_t*>(&qh23);
  }
  lo[0] = make_uint4(ol[0], ol[1], ol[2], ol[3]);
  lo[1] = make_uint4(ol[4], ol[5], ol[6], ol[7]);
  hi[0] = make_uint4(oh[0], oh[1], oh[2], oh[3]);
  hi[1] = make_uint4(oh[4], oh[5], oh[6], oh[7]);
}

__global__ void __launch_bounds__(kW4A16Threads, 1)
    w4a16_kernel(const __grid_constant__ W4A16Params p, const __grid_constant__ CUtensorMap tmap_wp,
                 const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_sc) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  SPECQ_TRACE_INIT();
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;                                              // TMA stages
  uint8_t* dring = ring + p.stages * p.stage_bytes;                  // dequantised operand slots
  __half* sc_cache = reinterpret_cast<__half*>(dring + p.dstages * kW4A16DSlot);
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      reinterpret_cast<uint8_t*>(sc_cache) + ((128u * p.sc_cache_cols * 2u + 15u) & ~15u));
  uint64_t* full = bars;
  uint64_t* empty = full + p.stages;
  uint64_t* dfull = empty + p.stages;
  uint64_t* dempty = dfull + p.dstages;
  uint64_t* acc_full = dempty + p.dstages;
  uint64_t* sc_full = acc_full + 1;                                  // scale tile landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const int split = blockIdx.x;
  const int n0 = blockIdx.y * 128;
  const int m0 = blockIdx.z * p.chunk;
  const int half_k = p.K / 2;

  int M = p.m_rows;
  if (p.plan != nullptr) {
    int pm = __ldg(p.plan);
    if (pm < 0 || pm > p.m_rows) {
      if (threadIdx.x == 0 && split == 0 && blockIdx.y == 0 && blockIdx.z == 0)
        report_status(p.status, SPECQ_STATUS_PLAN_CLAMPED);
      pm = pm < 0 ? 0 : p.m_rows;
    }
    M = pm;
  }
  const int m_cnt = min(p.chunk, M - m0);
  if (m_cnt <= 0) return;                       // whole cluster shares (y, z)
  const uint32_t n_pad = static_cast<uint32_t>((m_cnt + 15) & ~15);
  const int a_rows = (m_cnt + 15) & ~15;                       // TMA boxes of 16 rows
  const uint32_t a_bytes = static_cast<uint32_t>(a_rows) * 128u;

  const int kb0 = split * p.kb_per_split;
  const int kb1 = min(kb0 + p.kb_per_split, p.kb_total);
  const int nkb = kb1 - kb0;
  if (threadIdx.x == 0) SPECQ_TRACE_POINT(0, 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1u);
      mbar_init(&empty[s], kW4A16GroupWarps + 1u);   // the block's dequant group + 1 MMA commit
    }
    for (int d = 0; d < p.dstages; ++d) {
      mbar_init(&dfull[d], kW4A16GroupWarps);
      mbar_init(&dempty[d], 1u);
    }
    mbar_init(acc_full, 1u);
    mbar_init(sc_full, 1u);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_wp);
    tma_prefetch_desc(&tmap_a);
    if (p.sc_cache_cols > 0) tma_prefetch_desc(&tmap_sc);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_acc = *tmem_slot;
  if (threadIdx.x == 0) SPECQ_TRACE_POINT(1, 0);

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (elect_one()) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_a = policy_evict_last();
      if (p.sc_cache_cols > 0) {   // the CTA's [128 x K/group] fp16 scale tile, once
        mbar_arrive_expect_tx(sc_full, 128u * p.sc_cache_cols * 2u);
        tma_load_2d(sc_cache, &tmap_sc, sc_full, 0, n0, pol_a);
      }
      int issued = 0;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % p.stages;
        const uint32_t ph = static_cast<uint32_t>(i / p.stages) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, p.status, SPECQ_STATUS_TIMEOUT_PIPELINE)) { *abort_flag = 1; break; }
        SPECQ_TRACE_POINT(2, i);
        uint8_t* st = ring + s * p.stage_bytes;
        mbar_arrive_expect_tx(&full[s], kW4A16PackTile + 2u * a_bytes);
        const int kb = kb0 + i;
        tma_load_2d(st, &tmap_wp, &full[s], kb * 64, n0, pol_w);
        uint8_t* alo = st + kW4A16PackTile;
        uint8_t* ahi = alo + a_bytes;
        for (int r = 0; r < a_rows; r += 16) {
          tma_load_2d(alo + r * 128, &tmap_a, &full[s], kb * 64, m0 + r, pol_a);
          tma_load_2d(ahi + r * 128, &tmap_a, &full[s], half_k + kb * 64, m0 + r, pol_a);
        }
        ++issued;
      }
      if (*abort_flag) {   // let copies in flight land before the CTA can exit
        for (int i = max(0, issued - p.stages); i < issued; ++i)
          mbar_wait(&full[i % p.stages], static_cast<uint32_t>(i / p.stages) & 1u, p.status,
                    SPECQ_STATUS_TIMEOUT_PIPELINE);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (elect_one()) {
      const uint32_t idesc = idesc_f16(128, n_pad);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % p.stages;
        const int d = i % p.dstages;
        if (!mbar_wait(&full[s], static_cast<uint32_t>(i / p.stages) & 1u, p.status, SPECQ_STATUS_TIMEOUT_PIPELINE) ||
            !mbar_wait(&dfull[d], static_cast<uint32_t>(i / p.dstages) & 1u, p.status, SPECQ_STATUS_TIMEOUT_PIPELINE)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        SPECQ_TRACE_POINT(3, i);
        const uint32_t alo = smem_u32(ring + s * p.stage_bytes) + kW4A16PackTile;
        const uint32_t ahi = alo + a_bytes;
        const uint32_t wlo = smem_u32(dring + d * kW4A16DSlot);
        const uint32_t whi = wlo + kW4A16OpTile;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16_ss(tmem_acc, sdesc_sw128(wlo + 32u * k, 16u, 1024u), sdesc_sw128(alo + 32u * k, 16u, 1024u), idesc,
                      (i > 0 || k > 0) ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16_ss(tmem_acc, sdesc_sw128(whi + 32u * k, 16u, 1024u), sdesc_sw128(ahi + 32u * k, 16u, 1024u), idesc,
                      1u);
        umma_commit(&empty[s]);
        umma_commit(&dempty[d]);
        SPECQ_TRACE_POINT(4, i);
      }
      umma_commit(acc_full);
    }
  } else {
    // ---------------- dequant warps ----------------
    const int td = static_cast<int>(threadIdx.x) - 64;   // 0..511
    const int grp = td / kW4A16GroupThreads;               // K-blocks i with i % 2 == grp
    const int tg = td % kW4A16GroupThreads;                // 0..255 within the group
    // this thread dequantises 16-byte chunk (tg & 3) of rows r0 = tg / 4 and r0 + 64
    const int r0 = tg >> 2;
    const int c = tg & 3;
    const int scc = static_cast<int>(p.sc_cache_cols);
    const int64_t row0 = static_cast<int64_t>(min(n0 + r0, p.N - 1)) * p.ldsc;
    const int64_t row1 = static_cast<int64_t>(min(n0 + r0 + 64, p.N - 1)) * p.ldsc;
    auto group_of = [&](int k) { return p.group_shift >= 0 ? (k >> p.group_shift) : (k / p.group); };
    auto fetch = [&](int kb, __half (&s4)[4]) {
      const int glo = group_of(kb * 64);
      const int ghi = group_of(half_k + kb * 64);
      if (scc > 0) {
        s4[0] = sc_cache[r0 * scc + glo];
        s4[1] = sc_cache[r0 * scc + ghi];
        s4[2] = sc_cache[(r0 + 64) * scc + glo];
        s4[3] = sc_cache[(r0 + 64) * scc + ghi];
      } else {
        s4[0] = p.sc[row0 + glo];
        s4[1] = p.sc[row0 + ghi];
        s4[2] = p.sc[row1 + glo];
        s4[3] = p.sc[row1 + ghi];
      }
    };
    if (scc > 0 && !mbar_wait(sc_full, 0u, p.status, SPECQ_STATUS_TIMEOUT_PIPELINE)) *abort_flag = 1;
    for (int i = grp; i < nkb; i += kW4A16Groups) {
      const int s = i % p.stages;
      const int d = i % p.dstages;
      if (!mbar_wait(&full[s], static_cast<uint32_t>(i / p.stages) & 1u, p.status, SPECQ_STATUS_TIMEOUT_PIPELINE) ||
          !mbar_wait(&dempty[d], (static_cast<uint32_t>(i / p.dstages) & 1u) ^ 1u, p.status,
                     SPECQ_STATUS_TIMEOUT_PIPELINE)) {
        *abort_flag = 1;
        break;
      }
      if (td == 0) SPECQ_TRACE_POINT(10, i);
      const uint8_t* pk = ring + s * p.stage_bytes;
      uint8_t* wlo = dring + d * kW4A16DSlot;
      uint8_t* whi = wlo + kW4A16OpTile;
      __half sc4[4];
      fetch(kb0 + i, sc4);
      const uint4 raw0 = *reinterpret_cast<const uint4*>(pk + tg * 16);           // row r0
      const uint4 raw1 = *reinterpret_cast<const uint4*>(pk + (tg + 256) * 16);   // row r0 + 64
      if (td == 0) SPECQ_TRACE_POINT(12, raw0.x == 0x12345678u ? 63 : i);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);    // packed tile consumed (activations: MMA commit)
      uint4 lo[2], hi[2];
      dequant_chunk(raw0, __half2half2(sc4[0]), __half2half2(sc4[1]), lo, hi);
      *reinterpret_cast<uint4*>(wlo + sw128_offset(r0, 2 * c)) = lo[0];
      *reinterpret_cast<uint4*>(wlo + sw128_offset(r0, 2 * c + 1)) = lo[1];
      *reinterpret_cast<uint4*>(whi + sw128_offset(r0, 2 * c)) = hi[0];
      *reinterpret_cast<uint4*>(whi + sw128_offset(r0, 2 * c + 1)) = hi[1];
      dequant_chunk(raw1, __half2half2(sc4[2]), __half2half2(sc4[3]), lo, hi);
      *reinterpret_cast<uint4*>(wlo + sw128_offset(r0 + 64, 2 * c)) = lo[0];
      *reinterpret_cast<uint4*>(wlo + sw128_offset(r0 + 64, 2 * c + 1)) = lo[1];
      *reinterpret_cast<uint4*>(whi + sw128_offset(r0 + 64, 2 * c)) = hi[0];
      *reinterpret_cast<uint4*>(whi + sw128_offset(r0 + 64, 2 * c + 1)) = hi[1];
      if (td == 0) SPECQ_TRACE_POINT(13, i);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dfull[d]);
      if (td == 0) SPECQ_TRACE_POINT(11, i);
    }
  }
  __syncwarp();

  // ---------------- epilogue (warps 2..5) ----------------
  const bool epi = (warp >= 2 && warp < 6);
  const uint32_t quad = warp & 3u;
  const int row = static_cast<int>(quad * 32 + lane);
  bool ok = true;
  if (epi) {
    ok = mbar_wait(acc_full, 0u, p.status, SPECQ_STATUS_TIMEOUT_MMA) && (*abort_flag == 0);
    tc_fence_after();
    if (warp == 2 && lane == 0) SPECQ_TRACE_POINT(5, 0);
  }
  if (p.splits == 1) {
    if (epi && ok) {
      const int n = n0 + row;
      for (uint32_t c0 = 0; c0 < n_pad; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(tmem_acc + ((quad * 32u) << 16) + c0, r);
        tmem_wait_ld();
        if (n < p.N) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + static_cast<int>(c0) + j;
            if (m < M)
              p.out[static_cast<int64_t>(m) * p.ldo + static_cast<int64_t>(n) * p.ldo_n] =
                  __float2half_rn(__uint_as_float(r[j]));
          }
        }
      }
    }
  } else {
    const uint32_t pitch = n_pad * 4u + 16u;
    // The operand ring is idle now and large enough for the [128 x n_pad] fp32 partial.
    if (epi && ok) {
      uint8_t* red = ring;
      for (uint32_t c0 = 0; c0 < n_pad; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(tmem_acc + ((quad * 32u) << 16) + c0, r);
        tmem_wait_ld();
        uint4* dst = reinterpret_cast<uint4*>(red + row * pitch + c0 * 4u);
        dst[0] = make_uint4(r[0], r[1], r[2], r[3]);
        dst[1] = make_uint4(r[4], r[5], r[6], r[7]);
        dst[2] = make_uint4(r[8], r[9], r[10], r[11]);
        dst[3] = make_uint4(r[12], r[13], r[14], r[15]);
      }
    }
    cluster_sync();
    if (epi) {
      const int S = p.splits;
      const int lgR = 7 - (31 - __clz(S));
      const int R = 1 << lgR;
      const int nq = static_cast<int>(n_pad >> 2);
      const int te = static_cast<int>(threadIdx.x) - 64;
      for (int item = te; item < R * nq; item += 128) {
        const int cq = item >> lgR;
        const int trow = split * R + (item & (R - 1));
        const int n = n0 + trow;
        const float4* src = reinterpret_cast<const float4*>(ring + trow * pitch + cq * 16);
        float4 v[8];
#pragma unroll
        for (int pr = 0; pr < 8; ++pr)      // all peers' loads in flight together
          if (pr < S) v[pr] = *dsmem_ptr(src, static_cast<uint32_t>(pr));
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
        for (int pr = 0; pr < 8; ++pr) {    // fixed order: the same bits for any schedule
          if (pr < S) {
            s0 += v[pr].x;
            s1 += v[pr].y;
            s2 += v[pr].z;
            s3 += v[pr].w;
          }
        }
        if (ok && n < p.N) {
          const float sv[4] = {s0, s1, s2, s3};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int m = m0 + cq * 4 + j;
            if (m < M)
              p.out[static_cast<int64_t>(m) * p.ldo + static_cast<int64_t>(n) * p.ldo_n] = __float2half_rn(sv[j]);
          }
        }
      }
    }
    cluster_sync();
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) SPECQ_TRACE_POINT(9, 0);
  SPECQ_TRACE_CTA_END();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_acc, p.tmem_cols);
  }
}

}  // namespace specq
