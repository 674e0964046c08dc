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
//     [128 x 64 B] weight tile (64-byte swizzle) into a deep weight ring and the two matching
//     [tokens x 64] fp16 activation tiles (128-byte swizzle) into an activation ring.  Each
//     dequant thread owns one weight row = one TMEM lane: it dequantises the row ONCE per
//     K-block for all tokens of the CTA (the reference redoes this for every BLOCK_M rows,
//     kernels.py:112-133) and writes the fp16 weights straight into tensor memory, where the
//     MMA reads them as its A operand (tcgen05.mma with A in TMEM): the dequantised tile never
//     passes through shared memory, whose bandwidth would otherwise bound the kernel.
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
  int stages;          // packed-weight ring depth (kW4A16PackTile per stage)
  int xstages;         // activation ring depth (stage_bytes per stage)
  int aslots;          // A slots in tensor memory (64 columns each, after the accumulator)
  uint32_t a_col;      // first TMEM column of the A slots
  uint32_t stage_bytes;
  uint32_t sc_cache_cols;  // groups per row of the TMA-loaded scale tile (0: prefetch per K-block)
  uint32_t tmem_cols;
};

// Dequant warps form kW4A16Groups groups of four (one warp per TMEM lane quadrant); group g
// takes the K-blocks i with i % kW4A16Groups == g and writes them into A slots in tensor
// memory, so several blocks are being dequantised at any time.
constexpr int kW4A16Groups = 4;
constexpr int kW4A16GroupWarps = 4;
constexpr int kW4A16GroupThreads = 32 * kW4A16GroupWarps;
constexpr int kW4A16DequantWarps = kW4A16Groups * kW4A16GroupWarps;
constexpr int kW4A16DequantThreads = 32 * kW4A16DequantWarps;
// warp 0 weight TMA, warp 1 MMA, warps 2.. dequant (2..5 also the epilogue), last warp activation TMA
constexpr int kW4A16Threads = 64 + kW4A16DequantThreads + 32;
constexpr int kW4A16ActWarp = kW4A16Threads / 32 - 1;
constexpr uint32_t kW4A16PackTile = 128 * 64;   // packed bytes per stage
constexpr int kW4A16MaxSlots = 8;               // A slots of 64 TMEM columns (one K-block each)

// 16 packed bytes (packed columns j..j+15 of one row) -> 16 fp16 weights of the low half
// (k = j..j+15, low nibbles) or of the high half (k = K/2 + j.., high nibbles), multiplied by
// the fp16 group scale, as 8 words of consecutive fp16 pairs.
__device__ __forceinline__ void dequant_lo16(uint4 pk, __half2 sc, uint32_t (&o)[8]) {
  const uint32_t w[4] = {pk.x, pk.y, pk.z, pk.w};
  const __half2 k1032 = __half2half2(__ushort_as_half(0x6408));       // 1032.0
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t l01 = (__byte_perm(w[i], 0u, 0x4140) & 0x000F000Fu) | 0x64006400u;  // 1024 + nibble
    const uint32_t l23 = (__byte_perm(w[i], 0u, 0x4342) & 0x000F000Fu) | 0x64006400u;
    const __half2 q01 = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&l01), k1032), sc);
    const __half2 q23 = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&l23), k1032), sc);
    o[2 * i] = *reinterpret_cast<const uint32_t*>(&q01);
    o[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&q23);
  }
}
__device__ __forceinline__ void dequant_hi16(uint4 pk, __half2 sc, uint32_t (&o)[8]) {
  const uint32_t w[4] = {pk.x, pk.y, pk.z, pk.w};
  const __half2 k1_16 = __half2half2(__ushort_as_half(0x2C00));       // 0.0625
  const __half2 km72 = __half2half2(__ushort_as_half(0xD480));        // -72.0
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t h01 = (__byte_perm(w[i], 0u, 0x4140) & 0x00F000F0u) | 0x64006400u;  // 1024 + 16 nibble
    const uint32_t h23 = (__byte_perm(w[i], 0u, 0x4342) & 0x00F000F0u) | 0x64006400u;
    const __half2 q01 = __hmul2(__hfma2(*reinterpret_cast<const __half2*>(&h01), k1_16, km72), sc);
    const __half2 q23 = __hmul2(__hfma2(*reinterpret_cast<const __half2*>(&h23), k1_16, km72), sc);
    o[2 * i] = *reinterpret_cast<const uint32_t*>(&q01);
    o[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&q23);
  }
}

__global__ void __launch_bounds__(kW4A16Threads, 1)
    w4a16_kernel(const __grid_constant__ W4A16Params p, const __grid_constant__ CUtensorMap tmap_wp,
                 const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_sc,
                 const __grid_constant__ CUtensorMap tmap_a_chunk) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  SPECQ_TRACE_INIT();
  if (threadIdx.x == 0) SPECQ_TRACE_POINT(12, 0);
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;                                              // packed weights [stages][128 x 64 B]
  uint8_t* xring = ring + p.stages * kW4A16PackTile;                 // activations [xstages][lo | hi]
  __half* sc_cache = reinterpret_cast<__half*>(xring + p.xstages * p.stage_bytes);   // [128][G] as loaded
  __half* sc_t = sc_cache + 128u * p.sc_cache_cols;                  // [G][128] transposed
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      reinterpret_cast<uint8_t*>(sc_t) + ((128u * p.sc_cache_cols * 2u + 15u) & ~15u));
  uint64_t* full = bars;                                             // packed tile landed
  uint64_t* empty = full + p.stages;                                 // packed tile read by its dequant group
  uint64_t* xfull = empty + p.stages;                                // activation tile landed
  uint64_t* xempty = xfull + p.xstages;                              // activation tile read by the MMA
  uint64_t* afull = xempty + p.xstages;                              // [aslots] A slot written
  uint64_t* aempty = afull + kW4A16MaxSlots;                         // [aslots] A slot read
  uint64_t* acc_full = aempty + kW4A16MaxSlots;
  uint64_t* sc_full = acc_full + 1;                                  // scale tile landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const int split = blockIdx.x;
  const int n0 = blockIdx.y * 128;
  const int m0 = blockIdx.z * p.chunk;
  const int half_k = p.K / 2;
  const int kb0 = split * p.kb_per_split;
  const int kb1 = min(kb0 + p.kb_per_split, p.kb_total);
  const int nkb = kb1 - kb0;
  // Each N tile walks its K range from a different starting block, so the CTAs do not all
  // read the same activation lines (one set of L2 slices) at the same time.  The order depends
  // only on the tile, never on M: plan and non-plan launches add the same partial products in
  // the same order.
  const int rot = nkb > 0 ? static_cast<int>((static_cast<int64_t>(blockIdx.y) * 5) % nkb) : 0;
  auto kblock = [&](int i) { return kb0 + (i + rot < nkb ? i + rot : i + rot - nkb); };

  // While the previous kernel on the stream finishes, warm L2 with this CTA's scale tile and
  // first packed weight tiles (the first token chunk only: later chunks find them there).
  if (threadIdx.x == 0 && blockIdx.z == 0) {
    tma_prefetch_desc(&tmap_wp);
    if (p.sc_cache_cols > 0) {
      tma_prefetch_desc(&tmap_sc);
      tma_prefetch_l2_2d(&tmap_sc, 0, n0);
    }
    for (int i = 0; i < min(nkb, p.stages); ++i) tma_prefetch_l2_2d(&tmap_wp, kblock(i) * 64, n0);
  }
  pdl_wait();                // the previous kernel's writes are visible from here on

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

  if (threadIdx.x == 0) SPECQ_TRACE_POINT(0, 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1u);
      mbar_init(&empty[s], kW4A16GroupWarps);        // the block's dequant group
    }
    for (int s = 0; s < p.xstages; ++s) {
      mbar_init(&xfull[s], 1u);
      mbar_init(&xempty[s], 1u);                     // the MMA commit
    }
    for (int d = 0; d < p.aslots; ++d) {
      mbar_init(&afull[d], kW4A16GroupWarps);        // the dequant group that filled it
      mbar_init(&aempty[d], 1u);                     // the MMA commit
    }
    mbar_init(acc_full, 1u);
    mbar_init(sc_full, 1u);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_wp);
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_a_chunk);
    if (p.sc_cache_cols > 0) tma_prefetch_desc(&tmap_sc);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_acc = *tmem_slot;             // fp32 accumulator: columns [0, n_pad)
  const uint32_t tmem_a = tmem_acc + p.a_col;       // A slots: aslots x 64 columns
  if (threadIdx.x == 0) SPECQ_TRACE_POINT(1, 0);

  if (warp == 0) {
    // ---------------- weight TMA producer (runs up to `stages` K-blocks ahead) ----------------
    if (elect_one()) {
      const uint64_t pol_w = policy_evict_first();
      if (p.sc_cache_cols > 0) {   // the CTA's [128 x K/group] fp16 scale tile, once
        mbar_arrive_expect_tx(sc_full, 128u * p.sc_cache_cols * 2u);
        tma_load_2d(sc_cache, &tmap_sc, sc_full, 0, n0, policy_evict_last());
        SPECQ_TRACE_POINT(16, 0);
      }
      int issued = 0;
      int s = 0;
      uint32_t ph = 0;
      for (int i = 0; i < nkb; ++i) {
        // (a sleeping wait: the 16-stage ring hides its wake-up, the dequant warps need the slots)
        if (!mbar_wait_sleep(&empty[s], ph ^ 1u, 128u, p.status, SPECQ_STATUS_TIMEOUT_PIPELINE)) { *abort_flag = 1; break; }
        SPECQ_TRACE_POINT(2, i);
        mbar_arrive_expect_tx(&full[s], kW4A16PackTile);
        tma_load_2d(ring + s * kW4A16PackTile, &tmap_wp, &full[s], kblock(i) * 64, n0, pol_w);   // 64B-swizzled rows
        ++issued;
        if (++s == p.stages) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (*abort_flag) {   // let copies in flight land before the CTA can exit
        for (int i = max(0, issued - p.stages); i < issued; ++i)
          mbar_wait(&full[i % p.stages], static_cast<uint32_t>(i / p.stages) & 1u, p.status,
                    SPECQ_STATUS_TIMEOUT_PIPELINE);
      }
    }
  } else if (warp == kW4A16ActWarp) {
    // ---------------- activation TMA producer ----------------
    if (elect_one()) {
      const uint64_t pol_a = policy_evict_last();
      int issued = 0;
      int s = 0;
      uint32_t ph = 0;
      for (int i = 0; i < nkb; ++i) {
        if (!mbar_wait_sleep(&xempty[s], ph ^ 1u, 128u, p.status, SPECQ_STATUS_TIMEOUT_PIPELINE)) { *abort_flag = 1; break; }
        uint8_t* alo = xring + s * p.stage_bytes;
        uint8_t* ahi = alo + a_bytes;
        const int kb = kblock(i);
        mbar_arrive_expect_tx(&xfull[s], 2u * a_bytes);
        if (a_rows == p.chunk) {   // a full token chunk: one box per K half (TMA issue is serial)
          tma_load_2d(alo, &tmap_a_chunk, &xfull[s], kb * 64, m0, pol_a);
          tma_load_2d(ahi, &tmap_a_chunk, &xfull[s], half_k + kb * 64, m0, pol_a);
        } else {
          for (int r = 0; r < a_rows; r += 16) {
            tma_load_2d(alo + r * 128, &tmap_a, &xfull[s], kb * 64, m0 + r, pol_a);
            tma_load_2d(ahi + r * 128, &tmap_a, &xfull[s], half_k + kb * 64, m0 + r, pol_a);
          }
        }
        ++issued;
        SPECQ_TRACE_POINT(15, i);
        if (++s == p.xstages) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (*abort_flag) {
        for (int i = max(0, issued - p.xstages); i < issued; ++i)
          mbar_wait(&xfull[i % p.xstages], static_cast<uint32_t>(i / p.xstages) & 1u, p.status,
                    SPECQ_STATUS_TIMEOUT_PIPELINE);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // A (the dequantised weights) from tensor memory, B (the activations) from shared memory.
    if (elect_one()) {
      // This thread shares its scheduler with four busy dequant warps, so its loop is kept
      // short: ring indices and phases by counters (no divisions), operand descriptors by
      // adding address offsets (in 16-byte units) to one precomputed descriptor.
      // Two waits per K-block, both in block order: the dequantised A slot (afull) and the
      // activation tile (xfull).  This thread is the only consumer that waits on xfull, and it
      // consumed the stage's previous tile before the producer could reissue it, so the parity
      // wait can neither alias a phase behind nor two ahead.
      const uint32_t idesc = idesc_f16(128, n_pad);
      const uint64_t xdesc0 = sdesc_sw128(smem_u32(xring), 16u, 1024u);
      int s = 0, d = 0;
      uint32_t xph = 0, aph = 0;
      for (int i = 0; i < nkb; ++i) {
        if (!mbar_wait_sleep(&afull[d], aph, 32u, p.status, SPECQ_STATUS_TIMEOUT_PIPELINE) ||
            !mbar_wait(&xfull[s], xph, p.status, SPECQ_STATUS_TIMEOUT_PIPELINE)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        SPECQ_TRACE_POINT(3, i);
        const uint64_t dlo = xdesc0 + ((static_cast<uint32_t>(s) * p.stage_bytes) >> 4);
        const uint64_t dhi = dlo + (a_bytes >> 4);
        const uint32_t wa = tmem_a + 64u * static_cast<uint32_t>(d);
#pragma unroll
        for (int k = 0; k < 4; ++k)   // 16 low-half K values per step (32 bytes)
          umma_f16_ts(tmem_acc, wa + 8u * k, dlo + 2u * k, idesc, (i > 0 || k > 0) ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < 4; ++k)   // 16 high-half K values per step
          umma_f16_ts(tmem_acc, wa + 32u + 8u * k, dhi + 2u * k, idesc, 1u);
        umma_commit(&xempty[s]);
        umma_commit(&aempty[d]);
        SPECQ_TRACE_POINT(4, i);
        if (++s == p.xstages) {
          s = 0;
          xph ^= 1u;
        }
        if (++d == p.aslots) {
          d = 0;
          aph ^= 1u;
        }
      }
      umma_commit(acc_full);
    }
  } else {
    // ---------------- dequant warps ----------------
    // Group g (warps 2+4g .. 5+4g, one per TMEM lane quadrant) takes K-blocks i with
    // i % kW4A16Groups == g; thread = weight row r (its TMEM lane).  It reads the row's 64
    // packed bytes (64B swizzle: eight consecutive rows hit eight distinct bank groups),
    // applies the row's two group scales and writes the 128 fp16 weights into A slot
    // i % aslots.
    const int td = static_cast<int>(threadIdx.x) - 64;
    const int grp = td / kW4A16GroupThreads;
    const uint32_t quad = warp & 3u;
    const int r = static_cast<int>(quad * 32u + lane);
    const uint32_t lane_base = (quad * 32u) << 16;
    const int scc = static_cast<int>(p.sc_cache_cols);
    const int64_t rowg = static_cast<int64_t>(min(n0 + r, p.N - 1)) * p.ldsc;
    auto group_of = [&](int k) { return p.group_shift >= 0 ? (k >> p.group_shift) : (k / p.group); };
    if (scc > 0) {
      if (!mbar_wait(sc_full, 0u, p.status, SPECQ_STATUS_TIMEOUT_PIPELINE)) *abort_flag = 1;
      if (td == 0) SPECQ_TRACE_POINT(13, 0);
      // transpose the scale tile once: [g][row] reads are conflict-free in the loop below.
      // Item = (8 consecutive groups, row): one 16-byte read of the row's groups, eight 2-byte
      // writes; the 32 lanes of a warp take 32 consecutive rows, so each write is one
      // contiguous 64-byte row segment (reading element-wise instead, 64 bytes apart per lane,
      // cost ~1.3 us of 16-way bank conflicts at config 1).
      for (int e = td; e < (scc >> 3) * 128; e += kW4A16DequantThreads) {
        const int g8 = e >> 7, rr = e & 127;
        const uint4 v = *reinterpret_cast<const uint4*>(sc_cache + rr * scc + 8 * g8);
        const __half* h = reinterpret_cast<const __half*>(&v);
#pragma unroll
        for (int k = 0; k < 8; ++k) sc_t[(8 * g8 + k) * 128 + rr] = h[k];
      }
      named_barrier_sync(1, kW4A16DequantThreads);
      if (td == 0) SPECQ_TRACE_POINT(14, 0);
    }
    // K-block i = grp + 4 it: weight stage i % stages and its phase by a counter; A slot
    // i % aslots = grp (the host sizes aslots == kW4A16Groups), its phase flips every turn.
    int s = grp % p.stages;
    uint32_t wph = static_cast<uint32_t>(grp / p.stages) & 1u;
    const int d = grp;
    uint32_t aph = 0;
    // The A slot first: once the MMA has consumed block i - 4 (this group's previous block),
    // every block <= i - 4 has landed, so with >= 4 weight stages (host-enforced) the previous
    // tile of stage s has completed its phase and the parity wait on full[s] cannot alias it.
    for (int i = grp; i < nkb; i += kW4A16Groups) {
      if (!mbar_wait(&aempty[d], aph ^ 1u, p.status, SPECQ_STATUS_TIMEOUT_PIPELINE) ||
          !mbar_wait(&full[s], wph, p.status, SPECQ_STATUS_TIMEOUT_PIPELINE)) {
        *abort_flag = 1;
        break;
      }
      if (td == 0) SPECQ_TRACE_POINT(10, i);
      const uint8_t* pk = ring + s * kW4A16PackTile + r * 64;
      const uint32_t sw = (static_cast<uint32_t>(r) >> 1) & 3u;
      uint4 raw[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) raw[c] = *reinterpret_cast<const uint4*>(pk + ((static_cast<uint32_t>(c) ^ sw) << 4));
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);   // the packed tile can be refilled
      const int kb = kblock(i);
      const int glo = group_of(kb * 64), ghi = group_of(half_k + kb * 64);
      const __half slo = scc > 0 ? sc_t[glo * 128 + r] : p.sc[rowg + glo];
      const __half shi = scc > 0 ? sc_t[ghi * 128 + r] : p.sc[rowg + ghi];
      const uint32_t wa = tmem_a + lane_base + 64u * static_cast<uint32_t>(d);
#pragma unroll
      for (int half = 0; half < 2; ++half) {   // the low K half, then the high K half
        uint32_t w[32];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t o[8];
          if (half == 0)
            dequant_lo16(raw[c], __half2half2(slo), o);
          else
            dequant_hi16(raw[c], __half2half2(shi), o);
#pragma unroll
          for (int k = 0; k < 8; ++k) w[8 * c + k] = o[k];
        }
        tmem_st16(wa + 32u * half, *reinterpret_cast<const uint32_t(*)[16]>(w));
        tmem_st16(wa + 32u * half + 16u, *reinterpret_cast<const uint32_t(*)[16]>(w + 16));
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[d]);
      if (td == 0) SPECQ_TRACE_POINT(11, i);
      aph ^= 1u;
      for (s += kW4A16Groups; s >= p.stages; s -= p.stages) wph ^= 1u;
    }
  }
  __syncwarp();

  // The next kernel on the stream may begin launching once every CTA is here (its CTAs wait in
  // griddepcontrol.wait until this grid has completed): launching it at the start instead
  // measured slower, its early CTAs holding SMs this kernel's clusters could use.
  pdl_launch_dependents();
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
