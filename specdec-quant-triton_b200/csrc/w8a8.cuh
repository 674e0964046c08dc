// w8a8.cuh -- W8A8 INT8 GEMM for verification shapes on sm_100a.
//
// Computes out[m, n] = fp16((fp32(acc[m, n]) * sa[m]) * sw[n]), acc = sum_k a[m,k] * w[n,k]
// (reference kernel: kernels.py:27-55; the epilogue order acc*sa*sw follows kernels.py:53).
//
// Design (B200-first, not the reference's tiling):
//   * Swap-AB.  The tensor-core M=128 axis runs over 128 weight channels (A operand = the
//     weight tile); the N axis runs over the CTA's tokens (B operand = activations).  One CTA
//     holds the INT32 accumulators of up to 288 tokens (the largest verification batch,
//     32 x 9) for its 128 channels in TMEM -- two MMAs per K step past 256 tokens, the
//     instruction's N limit -- so the weights are streamed from HBM once whatever
//     M = B*(k+1) is: there is no M-tile staircase (the reference re-streams the weights for
//     every BLOCK_M rows).  A plan-buffer graph sized for M = 288 then has the same grid and
//     split-K as an eager call at any smaller M; eager calls of narrow shapes (fewer channel
//     tiles than SMs) keep chunks of at most 256 tokens, whose split-K partials are smaller.
//   * TMA loads 128-byte-swizzled [128 x 128 B] weight tiles and the token chunk's activations
//     (one box of the whole chunk, or 16-row boxes for a ragged last chunk) into a multi-stage
//     mbarrier ring; one elected thread issues tcgen05.mma kind::i8 (M=128, N=tokens rounded
//     up to 16, K=32 per instruction).
//   * Grid (split, chunk, tile): the CTAs of one weight tile are adjacent in launch order, so
//     a tile's second token chunk reads the weights from L2 while the first streams them.
//     Each tile walks its K range from its own starting block, so the CTAs do not all read
//     the same activation lines (one set of L2 slices) at once.
//   * Split-K across a thread-block cluster along grid.x fills the 148 SMs at small N; the
//     INT32 partials are reduced through distributed shared memory, no HBM partials.
//     Integer addition is exact, so any split gives the same bits.
//   * Plan mode: M is read from plan[0] on the device; CTAs whose token chunk is empty exit,
//     the MMA N extent is set from the active M, rows >= M are never written.
//   * When a row stride / base address is not 16-byte aligned (e.g. K = 520), TMA cannot be
//     used: the epilogue warps, idle during the main loop, load the tiles with vector loads
//     of the widest aligned width and write the same swizzled layout.
#pragma once

#include <type_traits>

#include "gemm_common.cuh"

namespace specq {

constexpr int kW8A8MaxPeers = 8;

struct W8A8Params {
  const int8_t* a;     // [m_rows, K], row stride lda bytes
  const int8_t* w;     // [N, K], row stride ldw bytes
  const float* sa;     // [m_rows]
  const float* sw;     // [N]
  __half* out;         // fp16 output, strides (ldo, ldo_n) elements   (null in acc mode)
  int32_t* acc_out;    // raw INT32 accumulator, row stride ldacc    (null in fp16 mode)
  const int32_t* plan; // optional: plan[0] = active M
  int* status;
  int64_t lda, ldw, ldo, ldo_n, ldacc;
  int m_rows;          // rows the kernel may touch (grid extent)
  int N, K;
  int chunk;           // tokens per CTA along grid.y (multiple of 16, <= kW8A8MaxChunk)
  int chunk_box;       // rows of one activation TMA box of a whole chunk (chunk, or chunk / 2)
  int kb_total;        // ceil(K / 128)
  int kb_per_split;    // 128-byte K blocks per split-K CTA
  int splits;          // cluster size along grid.x
  int stages;          // pipeline depth
  uint32_t stage_bytes;   // of the launch's largest token chunk
  uint32_t ring_bytes;    // stages * stage_bytes: the ring, re-cut at run time for the active chunk
  uint32_t tmem_cols;
};

// Tensor-parallel output (the W8A8PeerOut instantiation): every fp16 store goes to out[q] for
// each rank q (this rank's own full buffer included, each base at this rank's column block), and
// each CTA, once its stores are done, adds 1 to slot `rank` of every rank's flag array (its own
// included: the consumer on this rank reads its own count as the target).  The plain kernel is
// instantiated with W8A8NoPeer and carries none of it.
struct W8A8NoPeer {};
struct W8A8PeerOut {
  __half* out[kW8A8MaxPeers];
  uint32_t* flags[kW8A8MaxPeers];
  int world, rank;
};

constexpr int kW8A8Threads = 192;  // warp 0 TMA, warp 1 MMA, warps 2..5 epilogue (+ LDG producer)
constexpr uint32_t kW8A8WTile = 128 * 128;  // bytes of one weight tile
constexpr int kW8A8MaxStages = 8;
constexpr int kW8A8MaxChunk = 288;          // tokens per CTA: 256 + 32 in a second MMA

// Activation tensor maps: boxes of 16, 32, 64 and 128 rows (a token chunk of any multiple of 16
// rows arrives in at most four copies -- TMA copies issue one after another), and one box of a
// whole chunk (or half of one past 256 rows).
struct W8A8ActMaps {
  CUtensorMap rows[4];   // 16, 32, 64, 128 rows x 128 bytes
  CUtensorMap chunk;     // chunk_box rows x 128 bytes
};

// VEC = 0: TMA producer; VEC in {16, 8, 4, 2, 1}: register-staged loads of that width.
template <int VEC, typename PeerT>
__global__ void __launch_bounds__(kW8A8Threads, 1)
    w8a8_kernel(const __grid_constant__ W8A8Params p, const __grid_constant__ CUtensorMap tmap_w,
                const __grid_constant__ W8A8ActMaps tmap_a, const __grid_constant__ PeerT peer) {
  constexpr bool kPeer = std::is_same<PeerT, W8A8PeerOut>::value;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  SPECQ_TRACE_INIT();
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.ring_bytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + kW8A8MaxStages;
  uint64_t* acc_full = bars + 2 * kW8A8MaxStages;
  uint64_t* red_full = acc_full + 1;                          // split-K: the peers' rows landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kW8A8MaxStages + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* sa_s = reinterpret_cast<float*>(tmem_slot + 4);      // [kW8A8MaxChunk] token scales of this chunk
  float* sw_s = sa_s + kW8A8MaxChunk;                         // [128] channel scales of this tile

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const int split = blockIdx.x;             // == cluster rank (cluster spans grid.x)
  const int n0 = blockIdx.z * 128;
  const int m0 = blockIdx.y * p.chunk;
  const int kb0 = split * p.kb_per_split;
  const int kb1 = min(kb0 + p.kb_per_split, p.kb_total);
  const int nkb = kb1 - kb0;                                          // >= 1 (host guarantees)
  // K blocks in a per-tile rotated order (INT32 sums do not depend on the order)
  const int rot = static_cast<int>((static_cast<int64_t>(blockIdx.z) * 5) % nkb);
  auto kblock = [&](int i) { return kb0 + (i + rot < nkb ? i + rot : i + rot - nkb); };

  // While the previous kernel on the stream finishes, warm L2 with this CTA's first weight
  // tiles (the first token chunk only: later chunks of the tile find them there).
  // (an epilogue warp issues them: thread 0 initialises the barriers meanwhile)
  if (VEC == 0 && threadIdx.x == 64 && blockIdx.y == 0) {
    tma_prefetch_desc(&tmap_w);
    for (int i = 0; i < min(nkb, kW8A8MaxStages); ++i) tma_prefetch_l2_2d(&tmap_w, kblock(i) * 128, n0);
  }
  pdl_wait();                // the previous kernel's writes are visible from here on

  // ---- active extent (plan mode reads M on the device) --------------------------------
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
  // tensor-parallel output: this CTA's stores are done -> one release reduction per rank
  // (system scope, cumulative over the CTA's stores after the barrier that precedes it)
  auto signal_peers = [&]() {
    if constexpr (kPeer) {
      if (threadIdx.x == 0)
        for (int q = 0; q < peer.world; ++q) red_release_sys_add_u32(peer.flags[q] + peer.rank, 1u);
    }
  };
  // Every CTA of a cluster shares (blockIdx.y, blockIdx.z), so the whole cluster leaves
  // together and no cluster barrier is left waiting.  (It still counts itself in, so every
  // launch of a shape adds the same total.)
  if (m_cnt <= 0) {
    signal_peers();
    return;
  }
  const uint32_t n_pad = static_cast<uint32_t>((m_cnt + 15) & ~15);   // MMA N
  const int a_rows = (m_cnt + 15) & ~15;                               // activation rows staged
  const uint32_t a_bytes = static_cast<uint32_t>(a_rows) * 128u;
  // The ring is cut for the ACTIVE chunk: under a plan-buffer graph the launch is sized for
  // the largest M, and a smaller active M then gets more, smaller stages (more weight bytes
  // in flight) from the same shared memory.
  const uint32_t stage_bytes = kW8A8WTile + a_bytes;   // a multiple of 2048: TMA-aligned stages
  const int stages = min(kW8A8MaxStages, static_cast<int>(p.ring_bytes / stage_bytes));
  if (threadIdx.x == 0) SPECQ_TRACE_POINT(0, 0);

  // ---- setup ---------------------------------------------------------------------------
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], VEC == 0 ? 1u : 128u);
      mbar_init(&empty[s], 1u);
    }
    mbar_init(acc_full, 1u);
    mbar_init(red_full, 1u);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && VEC == 0 && lane == 0) {   // only the maps this CTA's copies use
    tma_prefetch_desc(&tmap_w);
    if (a_rows == p.chunk) {
      tma_prefetch_desc(&tmap_a.chunk);
    } else {
      if (a_rows >= 128) tma_prefetch_desc(&tmap_a.rows[3]);
      for (int b = 0; b < 3; ++b)
        if (a_rows & (16 << b)) tma_prefetch_desc(&tmap_a.rows[b]);
    }
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

  // ---- main loop -------------------------------------------------------------------------
  if (warp == 0) {
    if (VEC == 0 && elect_one()) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_a = policy_evict_last();
      int issued = 0;
      int s = 0;
      uint32_t ph = 0;
      for (int i = 0; i < nkb; ++i) {
        if (!mbar_wait(&empty[s], ph ^ 1u, p.status, SPECQ_STATUS_TIMEOUT_PIPELINE)) { *abort_flag = 1; break; }
        SPECQ_TRACE_POINT(2, i);
        uint8_t* wt = ring + s * stage_bytes;
        uint8_t* at = wt + kW8A8WTile;
        mbar_arrive_expect_tx(&full[s], kW8A8WTile + a_bytes);
        const int kx = kblock(i) * 128;
        tma_load_2d(wt, &tmap_w, &full[s], kx, n0, pol_w);
        if (a_rows == p.chunk) {   // a whole chunk: one box, or two past 256 rows (TMA issue is serial)
          for (int r = 0; r < a_rows; r += p.chunk_box) tma_load_2d(at + r * 128, &tmap_a.chunk, &full[s], kx, m0 + r, pol_a);
        } else {   // a ragged chunk (the last one, or the active rows of a plan-graph launch)
          int r = 0;
          for (int b = 3; b >= 0; --b)
            for (const int box = 16 << b; a_rows - r >= box; r += box)
              tma_load_2d(at + r * 128, &tmap_a.rows[b], &full[s], kx, m0 + r, pol_a);
        }
        ++issued;
        if (++s == stages) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (*abort_flag) {   // let copies in flight land before the CTA can exit
        for (int i = max(0, issued - stages); i < issued; ++i)
          mbar_wait(&full[i % stages], static_cast<uint32_t>(i / stages) & 1u, p.status,
                    SPECQ_STATUS_TIMEOUT_PIPELINE);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      // tokens [0, 256) in one MMA, the rest (at most 32, at TMEM column 256) in a second
      const uint32_t n_lo = n_pad < 256u ? n_pad : 256u;
      const uint32_t n_hi = n_pad - n_lo;
      const uint32_t idesc = idesc_i8(128, n_lo);
      const uint32_t idesc_hi = idesc_i8(128, n_hi > 0u ? n_hi : 16u);
      // descriptors advanced by address offsets in 16-byte units; ring index by a counter
      const uint64_t wdesc0 = sdesc_sw128(smem_u32(ring), 16u, 1024u);
      int s = 0;
      uint32_t ph = 0;
      for (int i = 0; i < nkb; ++i) {
        if (!mbar_wait(&full[s], ph, p.status, SPECQ_STATUS_TIMEOUT_PIPELINE)) { *abort_flag = 1; break; }
        tc_fence_after();
        SPECQ_TRACE_POINT(3, i);
        const uint64_t wd = wdesc0 + ((static_cast<uint32_t>(s) * stage_bytes) >> 4);
        const uint64_t ad = wd + (kW8A8WTile >> 4);
        if (n_hi == 0u) {   // (two loops: a branch per instruction measured slower)
#pragma unroll
          for (int k = 0; k < 4; ++k)   // 32 K bytes per step
            umma_i8_ss(tmem_acc, wd + 2u * k, ad + 2u * k, idesc, (i > 0 || k > 0) ? 1u : 0u);
        } else {   // token rows 256.. start 256 * 128 bytes into the activation tile
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            umma_i8_ss(tmem_acc, wd + 2u * k, ad + 2u * k, idesc, (i > 0 || k > 0) ? 1u : 0u);
            umma_i8_ss(tmem_acc + 256u, wd + 2u * k, ad + 2048u + 2u * k, idesc_hi, (i > 0 || k > 0) ? 1u : 0u);
          }
        }
        umma_commit(&empty[s]);   // stage is free once these MMAs have read it
        SPECQ_TRACE_POINT(4, i);
        if (++s == stages) {
          s = 0;
          ph ^= 1u;
        }
      }
      umma_commit(acc_full);      // accumulator complete
    }
  } else {
    // epilogue warps; in the LDG variant they first produce every stage.  They stage the
    // epilogue's scales in shared memory while the main loop runs (not before it starts).
    const int te = static_cast<int>(threadIdx.x) - 64;   // 0..127
    auto stage_scales = [&]() {
      if (p.acc_out != nullptr) return;
      for (int i = te; i < m_cnt; i += 128) sa_s[i] = __ldg(p.sa + m0 + i);
      sw_s[te] = (n0 + te < p.N) ? __ldg(p.sw + n0 + te) : 0.f;
    };
    if constexpr (VEC == 0) stage_scales();
    if constexpr (VEC != 0) {
      const uint8_t* wbase = reinterpret_cast<const uint8_t*>(p.w);
      const uint8_t* abase = reinterpret_cast<const uint8_t*>(p.a);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % stages;
        const uint32_t ph = static_cast<uint32_t>(i / stages) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, p.status, SPECQ_STATUS_TIMEOUT_PIPELINE)) { *abort_flag = 1; break; }
        uint8_t* wt = ring + s * stage_bytes;
        uint8_t* at = wt + kW8A8WTile;
        const int kx = kblock(i) * 128;
        ldg_tile_sw128<VEC>(wt, wbase, p.ldw, n0, 128, p.N, kx, p.K, te, 128);
        ldg_tile_sw128<VEC>(at, abase, p.lda, m0, a_rows, M, kx, p.K, te, 128);
        fence_proxy_async_smem();
        mbar_arrive(&full[s]);
      }
      stage_scales();
    }
  }
  __syncwarp();

  // The next kernel on the stream may begin launching once every CTA is here (its CTAs wait in
  // griddepcontrol.wait until this grid has completed): launching it at the start instead
  // measured slower, its early CTAs holding SMs this kernel's clusters could use.
  pdl_launch_dependents();
  // ---- epilogue --------------------------------------------------------------------------
  // fp16 output stores: to p.out, or (tensor-parallel output) to every rank's full buffer at
  // the same offset -- peer stores over NVLink
  auto store_h = [&](int64_t off, __half v) {
    if constexpr (kPeer) {
      for (int q = 0; q < peer.world; ++q) peer.out[q][off] = v;
    } else {
      p.out[off] = v;
    }
  };
  auto store_h8 = [&](int64_t off, uint4 v) {
    if constexpr (kPeer) {
      for (int q = 0; q < peer.world; ++q) *reinterpret_cast<uint4*>(peer.out[q] + off) = v;
    } else {
      *reinterpret_cast<uint4*>(p.out + off) = v;
    }
  };
  const bool epi = warp >= 2;
  const uint32_t quad = warp & 3u;                      // TMEM lane quadrant of this warp
  const int row = static_cast<int>(quad * 32 + lane);   // channel within the tile
  bool ok = true;
  if (epi) {
    ok = mbar_wait(acc_full, 0u, p.status, SPECQ_STATUS_TIMEOUT_MMA) && (*abort_flag == 0);
    tc_fence_after();
    named_barrier_sync(1, 128);   // every epilogue thread's staged scales are visible
    if (warp == 2 && lane == 0) SPECQ_TRACE_POINT(5, 0);
  }

  if (p.splits == 1) {
    if (epi && ok) {
      const int n = n0 + row;
      const float swn = sw_s[row];
      for (uint32_t c0 = 0; c0 < n_pad; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(tmem_acc + ((quad * 32u) << 16) + c0, r);
        tmem_wait_ld();
        if (n < p.N) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + static_cast<int>(c0) + j;
            if (m < M) {
              const int32_t acc = static_cast<int32_t>(r[j]);
              if (p.acc_out != nullptr) {
                p.acc_out[static_cast<int64_t>(m) * p.ldacc + n] = acc;
              } else {
                const float v = __fmul_rn(__fmul_rn(static_cast<float>(acc), sa_s[m - m0]), swn);
                store_h(static_cast<int64_t>(m) * p.ldo + static_cast<int64_t>(n) * p.ldo_n, __float2half_rn(v));
              }
            }
          }
        }
      }
    }
  } else {
    // Split-K: CTA r owns tile rows (channels) [r*R, (r+1)*R).  Every CTA parks its whole INT32
    // partial in its idle ring ([128 rows][pitch]); after one cluster barrier each CTA adds the
    // rows a peer owns into that peer's copy with one bulk asynchronous reduction per peer
    // (cp.reduce.async.bulk .add, completing on the owner's mbarrier), so the owner's rows hold
    // the full sums without a summation pass.  INT32 addition is exact: the bits do not depend
    // on the order.  A second cluster barrier (arrive once the own rows are complete, wait after
    // the output stores) keeps every CTA, and the ring its reductions read, alive until all of
    // them have landed.
    const int S = p.splits;
    const int lgR = 7 - (31 - __clz(S));       // rows owned by one CTA: R = 128 / S
    const int R = 1 << lgR;
    const uint32_t pitch = n_pad * 4u + 16u;   // padded row pitch: conflict-free v4 access
    if (epi && ok) {
      uint8_t* dst = ring + static_cast<uint32_t>(row) * pitch;
      for (uint32_t c0 = 0; c0 < n_pad; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(tmem_acc + ((quad * 32u) << 16) + c0, r);
        tmem_wait_ld();
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4)
          *reinterpret_cast<uint4*>(dst + c0 * 4u + 16u * q4) =
              make_uint4(r[4 * q4], r[4 * q4 + 1], r[4 * q4 + 2], r[4 * q4 + 3]);
      }
      fence_proxy_async_smem();   // the bulk reductions read the ring through the async proxy
    }
    cluster_sync();   // every CTA's partial is parked; every ring is idle
    if (warp == 2 && lane == 0) SPECQ_TRACE_POINT(6, 0);
    const uint32_t blk = static_cast<uint32_t>(R) * pitch;   // bytes of one owner's rows
    if (threadIdx.x == 64) {   // one epilogue thread issues this CTA's reductions
      mbar_arrive_expect_tx(red_full, static_cast<uint32_t>(S - 1) * blk);
      for (int q = 0; q < S; ++q) {
        if (q == split) continue;
        const uint32_t off = static_cast<uint32_t>(q) * blk;
        bulk_reduce_add_u32_cluster(dsmem_map(smem_u32(ring) + off, static_cast<uint32_t>(q)), smem_u32(ring) + off, blk,
                                    dsmem_map(smem_u32(red_full), static_cast<uint32_t>(q)));
      }
    }
    bool red_ok = true;
    if (epi) red_ok = mbar_wait(red_full, 0u, p.status, SPECQ_STATUS_TIMEOUT_PIPELINE);
    if (warp == 2 && lane == 0) SPECQ_TRACE_POINT(7, 0);
    // this CTA's incoming reductions have landed: arrive now, wait (for the peers' to have
    // landed too, so every ring may be released) after the output stores
    cluster_arrive();
    if (epi && ok && red_ok) {
      const int te = static_cast<int>(threadIdx.x) - 64;
      const uint8_t* own = ring + static_cast<uint32_t>(split * R) * pitch;
      const bool vec = p.acc_out == nullptr && p.ldo_n == 1 && (p.ldo % 8) == 0 &&
                       (reinterpret_cast<uintptr_t>(p.out) & 15u) == 0 && (n0 + split * R) % 8 == 0;
      if (vec) {
        // item = (token m, 8 consecutive owned channels): eight row reads, one 16-byte store
        const int ng = R >> 3;
        for (int item = te; item < ng * static_cast<int>(n_pad); item += 128) {
          const int m = item % static_cast<int>(n_pad);
          const int g = item / static_cast<int>(n_pad);
          if (m0 + m >= M) continue;
          const int nl = split * R + 8 * g;          // first channel of the group in the tile
          const float sam = sa_s[m];
          uint32_t hw[4];
#pragma unroll
          for (int k = 0; k < 8; k += 2) {
            const int32_t v0 = *reinterpret_cast<const int32_t*>(own + (8 * g + k) * pitch + m * 4);
            const int32_t v1 = *reinterpret_cast<const int32_t*>(own + (8 * g + k + 1) * pitch + m * 4);
            const __half2 h = __floats2half2_rn(__fmul_rn(__fmul_rn(static_cast<float>(v0), sam), sw_s[nl + k]),
                                                __fmul_rn(__fmul_rn(static_cast<float>(v1), sam), sw_s[nl + k + 1]));
            hw[k >> 1] = *reinterpret_cast<const uint32_t*>(&h);
          }
          const int n = n0 + nl;
          if (n + 8 <= p.N) {
            store_h8(static_cast<int64_t>(m0 + m) * p.ldo + n, make_uint4(hw[0], hw[1], hw[2], hw[3]));
          } else {
            const __half* hv = reinterpret_cast<const __half*>(hw);
            for (int k = 0; k < 8 && n + k < p.N; ++k) store_h(static_cast<int64_t>(m0 + m) * p.ldo + n + k, hv[k]);
          }
        }
      } else {
        const int nq = static_cast<int>(n_pad >> 2);
        for (int item = te; item < R * nq; item += 128) {
          const int rl = item % R;          // consecutive threads: consecutive rows (pitch-padded)
          const int cq = item / R;
          const int4 acc = *reinterpret_cast<const int4*>(own + rl * pitch + cq * 16);
          const int n = n0 + split * R + rl;
          if (n < p.N) {
            const int32_t sv[4] = {acc.x, acc.y, acc.z, acc.w};
            const float swn = sw_s[n - n0];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int m = m0 + cq * 4 + j;
              if (m < M) {
                if (p.acc_out != nullptr) {
                  p.acc_out[static_cast<int64_t>(m) * p.ldacc + n] = sv[j];
                } else {
                  const float val = __fmul_rn(__fmul_rn(static_cast<float>(sv[j]), sa_s[m - m0]), swn);
                  store_h(static_cast<int64_t>(m) * p.ldo + static_cast<int64_t>(n) * p.ldo_n, __float2half_rn(val));
                }
              }
            }
          }
        }
      }
    }
    cluster_wait();   // every reduction into every CTA has landed: rings may be released
    if (warp == 2 && lane == 0) SPECQ_TRACE_POINT(8, 0);
  }

  // ---- teardown ----------------------------------------------------------------------------
  tc_fence_before();
  __syncthreads();
  signal_peers();   // every output store of this CTA precedes the barrier above
  if (threadIdx.x == 0) SPECQ_TRACE_POINT(9, 0);
  SPECQ_TRACE_CTA_END();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_acc, p.tmem_cols);
  }
}

}  // namespace specq
