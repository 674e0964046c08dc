// paged_attn.cuh -- INT8 paged verification attention on sm_100a.
//
// For sequence b, query token qi < q_len and head h (kv head h / G):
//   out[b, qi, h, :] = softmax_t( (q . k_t) * ks_t / sqrt(D) ) . (v_t * vs_t),
//   over tokens t <= ctx_len[b] - q_len + qi reached through the block table
// (reference kernel: kernels.py:179-236; wrapper kernels.py:239-262).
//
// Design (B200-first):
//   * One CTA = (sequence, kv head, chunk of QPP query tokens, context split).  Its QPP*G query
//     rows (all heads of the GQA group) share every K/V byte it reads.
//   * Transposed products put the 128 tokens of a KV block on the tcgen05 M=128 axis and the
//     query rows (padded to a multiple of 16) on N:  S^T = K . Q^T  and  O^T = V^T . P^T.  No
//     tensor-core lane is wasted on padding query rows; the V tile is read MN-major straight
//     from the layout the K tile uses.
//   * K/V pages are gathered through the block table by TMA (one box per page run of one
//     head), into a multi-stage int8 ring; eight converter warps dequantise to fp16 operand
//     tiles (K exact, V with its per-token scale folded in).
//   * Softmax runs one thread per token row of S^T (TMEM lane = token): the per-token K scale
//     is a per-thread scalar.  The running max is "lazy": a block is exponentiated against the
//     current max and only when some score exceeds it by more than 2^8 does the CTA reduce
//     the block max, rescale O^T and the normaliser, and recompute.  The normaliser
//     l = sum_t p is produced by the tensor core itself (a ones operand in TMEM times P^T).
//   * Long contexts are split across a thread-block cluster; the partial (m, l, O) of every
//     split are combined through distributed shared memory in fixed rank order.  The split
//     count depends only on the block-table width, so plan mode and eager mode give the same
//     bits.
//   * Plan mode reads (n_seqs, q_len) on the device; CTAs outside them return, nothing outside
//     them is written.
#pragma once

#include "sm100.cuh"
#include "specq_host.cuh"

namespace specq {

struct AttnParams {
  const __half* q;
  int64_t q_sb, q_st, q_sh;
  const void* ks;
  const void* vs;
  int64_t s_sp, s_so, s_sh;
  int scale_f32;
  const int32_t* bt;
  int64_t bt_sb;
  int bt_cols;
  const int32_t* ctx_len;
  __half* out;
  int64_t o_sb, o_st, o_sh;
  const int32_t* plan;
  int* status;
  int n_pages;
  int b_grid, n_seqs, q_len, ql_max;
  int h_kv, g, page, qpp, nq, n_qc;
  int box_rows;
  int splits, stages;
  float sm_scale_log2;     // log2(e) / sqrt(D)
  uint32_t tmem_cols, col_stride;
};

constexpr int kAttnConvWarps = 6;
constexpr int kAttnConvThreads = 32 * kAttnConvWarps;
constexpr int kAttnThreads = 320 + kAttnConvThreads;   // warps 0-7 softmax, 8 TMA, 9 MMA, 10-15 convert
constexpr uint32_t kAttnKV8 = 128 * 128;       // int8 K (or V) block: 128 tokens x 128 B
constexpr uint32_t kAttnStage = 2 * kAttnKV8;  // K + V
constexpr uint32_t kAttnOp = 128 * 256;        // fp16 operand tile: 128 tokens x 128 d
constexpr float kLazyMaxLog2 = 8.0f;           // rescale once a score exceeds the max by 2^8

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                            int w, uint64_t cache_hint) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w), "l"(cache_hint)
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

__device__ __forceinline__ bool named_barrier_or(uint32_t id, uint32_t nthreads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.or.pred p, %2, %3, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 16 int8 -> 16 fp16 (exact): bias the byte by 128 into the mantissa of 1024.0, subtract 1152.
__device__ __forceinline__ void i8x16_to_f16(uint4 v, uint32_t (&h)[8]) {
  const uint32_t w[4] = {v.x ^ 0x80808080u, v.y ^ 0x80808080u, v.z ^ 0x80808080u, v.w ^ 0x80808080u};
  const __half2 bias = __half2half2(__ushort_as_half(0x6480));   // 1152.0
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t lo = __byte_perm(w[i], 0x64646464u, 0x4140);
    uint32_t hi = __byte_perm(w[i], 0x64646464u, 0x4342);
    __half2 a = __hsub2(*reinterpret_cast<__half2*>(&lo), bias);
    __half2 b = __hsub2(*reinterpret_cast<__half2*>(&hi), bias);
    h[2 * i] = *reinterpret_cast<uint32_t*>(&a);
    h[2 * i + 1] = *reinterpret_cast<uint32_t*>(&b);
  }
}

// Write the 16 fp16 values converted from int8 chunk `ch` (d = 16ch .. 16ch+15) of token `row`
// into a [2 atom columns][128 rows][128 B] 128B-swizzled operand tile.  Threads with ch < 4 and
// ch >= 4 of the same row land in the two atom columns (16 KB apart, same banks); the upper
// half stores its two chunks in the opposite order so each 8-thread phase hits 8 distinct
// bank groups.
__device__ __forceinline__ void store_f16_chunk_pair(uint8_t* tile, int row, int ch, const uint32_t (&h)[8]) {
  uint8_t* dst = tile + (ch >> 2) * 16384;
  const uint4 a = make_uint4(h[0], h[1], h[2], h[3]);
  const uint4 c = make_uint4(h[4], h[5], h[6], h[7]);
  const uint32_t k0 = 2u * static_cast<uint32_t>(ch & 3);
  if (ch < 4) {
    *reinterpret_cast<uint4*>(dst + sw128_offset(row, k0)) = a;
    *reinterpret_cast<uint4*>(dst + sw128_offset(row, k0 + 1)) = c;
  } else {
    *reinterpret_cast<uint4*>(dst + sw128_offset(row, k0 + 1)) = c;
    *reinterpret_cast<uint4*>(dst + sw128_offset(row, k0)) = a;
  }
}

__device__ __forceinline__ float load_scale(const void* base, int scale_f32, int64_t idx) {
  return scale_f32 ? __ldg(static_cast<const float*>(base) + idx)
                   : __half2float(__ldg(static_cast<const __half*>(base) + idx));
}

__global__ void __launch_bounds__(kAttnThreads, 1)
    paged_attn_kernel(const __grid_constant__ AttnParams p, const __grid_constant__ CUtensorMap tmap_k,
                      const __grid_constant__ CUtensorMap tmap_v) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  SPECQ_TRACE_INIT();
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int NQ = p.nq;
  uint8_t* ring = smem;                                           // stages x (K int8 | V int8)
  uint8_t* kop = ring + p.stages * kAttnStage;                    // fp16 K tile      [2][128][128 B]
  uint8_t* vop = kop + kAttnOp;                                   // fp16 V tiles  x2 [2][128][128 B]
  uint8_t* qop = vop + 2 * kAttnOp;                               // fp16 Q           [2][NQ][128 B]
  uint8_t* pop = qop + NQ * 256;                                  // fp16 P^T      x2 [2][NQ][128 B]
  float* scl_c = reinterpret_cast<float*>(pop + 2 * NQ * 256);    // [2][128] ks * log2e / sqrt(D)
  __half* scl_vh = reinterpret_cast<__half*>(scl_c + 256);       // [2][128] vs (fp16)
  float* m_s = scl_c + 512;                                       // [64] running max (log2 units)
  float* alpha_s = m_s + 64;                                      // [64]
  float* l_s = alpha_s + 64;                                      // [64]
  float* wmax = l_s + 64;                                         // [4][64]
  int* pgs = reinterpret_cast<int*>(wmax + 256);                  // [stages][128] page of each box
  uint64_t* bars = reinterpret_cast<uint64_t*>(pgs + p.stages * 128);
  uint64_t* stage_full = bars;
  uint64_t* stage_empty = stage_full + p.stages;
  uint64_t* k_full = stage_empty + p.stages;
  uint64_t* v_full = k_full + 1;         // [2]
  uint64_t* scl_full = v_full + 2;       // [2]
  uint64_t* scl_empty = scl_full + 2;    // [2]
  uint64_t* s_full = scl_empty + 2;      // [2]
  uint64_t* s_empty = s_full + 2;        // [2]
  uint64_t* p_full = s_empty + 2;        // [2]
  uint64_t* pv_done = p_full + 2;        // [2]  PV(j) done: frees P and V buffer j % 2
  uint64_t* q_full = pv_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_full + 1);

  const uint32_t warp = warp_id();
  const uint32_t lane = lane_id();
  const int split = blockIdx.x;
  const int kvh = blockIdx.y;
  const int b = blockIdx.z / p.n_qc;
  const int qc = blockIdx.z % p.n_qc;

  // ---- active extent -------------------------------------------------------------------
  int n_seqs = p.n_seqs, q_len = p.q_len;
  if (p.plan != nullptr) {
    n_seqs = __ldg(p.plan);
    q_len = __ldg(p.plan + 1);
    if (n_seqs < 0 || n_seqs > p.b_grid || q_len < 0 || q_len > p.ql_max) {
      if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
        report_status(p.status, SPECQ_STATUS_PLAN_CLAMPED);
      n_seqs = min(max(n_seqs, 0), p.b_grid);
      q_len = min(max(q_len, 0), p.ql_max);
    }
  }
  // the whole cluster (same blockIdx.y/z) leaves together
  if (b >= n_seqs || qc * p.qpp >= q_len) return;
  int L = __ldg(p.ctx_len + b);
  if (L < 0 || L > p.bt_cols * p.page) {
    if (threadIdx.x == 0 && split == 0) report_status(p.status, SPECQ_STATUS_PLAN_CLAMPED);
    L = min(max(L, 0), p.bt_cols * p.page);
  }
  const int q_lo = qc * p.qpp;
  const int q_hi = min(q_lo + p.qpp, q_len);
  const int rows_valid = (q_hi - q_lo) * p.g;
  const int qpos0 = L - q_len + q_lo;                 // last visible token of query-row group 0
  const int kv_end = max(0, L - q_len + q_hi);
  const int tchunk = ((kv_end + p.splits - 1) / p.splits + 127) & ~127;
  const int t_begin = split * tchunk;
  const int t_end = min(kv_end, t_begin + tchunk);
  const int nblk = (t_end > t_begin) ? (t_end - t_begin + 127) / 128 : 0;

  const uint32_t cs = p.col_stride;
  const uint32_t O_col = 2 * cs, L_col = 3 * cs, ONES_col = 4 * cs;

  // ---- setup ---------------------------------------------------------------------------------
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&stage_full[s], 1u);
      mbar_init(&stage_empty[s], kAttnConvWarps);
    }
    mbar_init(k_full, kAttnConvWarps);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&v_full[i], kAttnConvWarps);
      mbar_init(&scl_full[i], kAttnConvWarps);
      mbar_init(&scl_empty[i], 8u);
      mbar_init(&s_full[i], 1u);
      mbar_init(&s_empty[i], 8u);
      mbar_init(&p_full[i], 8u);
      mbar_init(&pv_done[i], 1u);
    }
    mbar_init(q_full, 8u);
    fence_barrier_init();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_v);
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  int* status = p.status;
  bool ok = true;
  if (threadIdx.x == 0) SPECQ_TRACE_POINT(1, 0);

  if (warp < 8) {
    // =================================== softmax warps ===================================
    // Warps w and w+4 share TMEM lane quadrant w: the same 32 tokens of S^T (the same 32 head
    // dims of O^T).  Warps 0-3 take the first half of the query columns, warps 4-7 the second.
    const int t = static_cast<int>(threadIdx.x);             // 0..255
    const int tl = t & 127;                                  // token lane of S^T, d lane of O^T
    const int grp = t >> 7;
    const int nqh = NQ >> 1;                                 // columns per group (multiple of 8)
    const int col0 = grp * nqh;
    const uint32_t quad = warp & 3u;
    const uint32_t lane_base = tmem + ((quad * 32u) << 16);
    // Q rows -> fp16 operand [2 atom columns][NQ rows][128 B], 128B-swizzled; padding rows = 0
    for (int c = t; c < NQ * 16; c += 256) {
      const int row = c >> 4;
      const int piece = c & 15;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (row < rows_valid) {
        const int qi = q_lo + row / p.g;
        const int head = kvh * p.g + row % p.g;
        const __half* src = p.q + b * p.q_sb + static_cast<int64_t>(qi) * p.q_st + static_cast<int64_t>(head) * p.q_sh;
        v = __ldg(reinterpret_cast<const uint4*>(src) + piece);
      }
      *reinterpret_cast<uint4*>(qop + (piece >> 3) * (NQ * 128) + sw128_offset(row, piece & 7)) = v;
    }
    if (t < 64) { m_s[t] = -INFINITY; alpha_s[t] = 1.f; l_s[t] = 0.f; }
    {   // ones operand for the normaliser MMA (fp16 1.0 pairs; 128 columns cover 8 K-steps)
      uint32_t ones[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) ones[i] = 0x3C003C00u;
#pragma unroll
      for (int c = 0; c < 64; c += 16) tmem_st16(lane_base + ONES_col + grp * 64 + c, ones);
      tmem_wait_st();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    named_barrier_sync(3, 256);
    __syncwarp();
    if (lane == 0) mbar_arrive(q_full);

    // Multi-thread roles never leave a loop early: after a wait runs out (ok = false) they skip
    // the remaining waits but still reach every named barrier, so no warp is stranded.
    for (int j = 0; j < nblk; ++j) {
      const int t_abs = t_begin + j * 128 + tl;
      const uint32_t sb = static_cast<uint32_t>(j & 1);
      const uint32_t par2 = static_cast<uint32_t>(j >> 1) & 1u;
      // query rows q >= q_first may see this token (causal window), rows >= q_stop never do
      const int q_first = max(0, (t_abs - qpos0) * p.g);
      const int q_stop = (t_abs < t_end) ? rows_valid : 0;
      ok = ok && mbar_wait(&scl_full[sb], par2, status, SPECQ_STATUS_TIMEOUT_PIPELINE);
      if (t == 0) SPECQ_TRACE_POINT(20, j);
      const float c_t = scl_c[sb * 128 + tl];
      __syncwarp();
      if (lane == 0) mbar_arrive(&scl_empty[sb]);
      ok = ok && mbar_wait(&s_full[sb], par2, status, SPECQ_STATUS_TIMEOUT_MMA);
      // P buffer sb is free once PV(j-2) has read it
      if (j >= 2) ok = ok && mbar_wait(&pv_done[sb], par2 ^ 1u, status, SPECQ_STATUS_TIMEOUT_MMA);
      tc_fence_after();
      if (t == 0) SPECQ_TRACE_POINT(21, j);
      const uint32_t s_addr = lane_base + sb * cs + col0;
      uint8_t* prow = pop + sb * (NQ * 256) + (tl >> 6) * (NQ * 128) + (tl & 7) * 2;
      const uint32_t tch = static_cast<uint32_t>((tl & 63) >> 3);

      // one optimistic pass: P against the current max, noting whether any score exceeds it
      // by more than 2^8 (then the block is redone below with a raised max)
      auto write_p = [&](float& xmax) {
        // every TMEM load of the pass is issued before a single wait (one round trip)
        uint32_t r[32];
#pragma unroll
        for (int c0 = 0; c0 < 32; c0 += 8)
          if (c0 < nqh) tmem_ld8(s_addr + c0, *reinterpret_cast<uint32_t(*)[8]>(r + c0));
        tmem_wait_ld();
#pragma unroll
        for (int c0 = 0; c0 < 32; c0 += 8) {
          if (c0 < nqh) {
            const float4* mv = reinterpret_cast<const float4*>(m_s + col0 + c0);
            const float4 m0 = mv[0], m1 = mv[1];
            const float mq[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int q = col0 + c0 + i;
              const bool valid = q >= q_first && q < q_stop;
              const float x = __uint_as_float(r[c0 + i]) * c_t - mq[i];
              xmax = valid ? fmaxf(xmax, x) : xmax;
              const float pr = valid ? fast_exp2(x) : 0.f;
              *reinterpret_cast<__half*>(prow + q * 128 + ((tch ^ (static_cast<uint32_t>(q) & 7u)) << 4)) =
                  __float2half_rn(pr);
            }
          }
        }
      };
      float xmax = -INFINITY;
      write_p(xmax);
      const bool need = named_barrier_or(2, 256, xmax > kLazyMaxLog2);
      if (t == 0) SPECQ_TRACE_POINT(22, j);
      if (need) {
        if (t == 0) SPECQ_TRACE_POINT(26, j);
        // the running O^T / normaliser must be final before they are rescaled
        if (j >= 1)
          ok = ok && mbar_wait(&pv_done[sb ^ 1u], static_cast<uint32_t>((j - 1) >> 1) & 1u, status,
                               SPECQ_STATUS_TIMEOUT_MMA);
        tc_fence_after();
        // block max per query column: warp shuffles, then across the four lane quadrants
        for (int c0 = 0; c0 < nqh; c0 += 8) {
          uint32_t r[8];
          tmem_ld8(s_addr + c0, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int q = col0 + c0 + i;
            float y = (q >= q_first && q < q_stop) ? __uint_as_float(r[i]) * c_t : -INFINITY;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) y = fmaxf(y, __shfl_xor_sync(0xffffffffu, y, o));
            if (lane == 0) wmax[quad * 64 + q] = y;
          }
        }
        named_barrier_sync(3, 256);
        if (t < NQ) {
          const float mb = fmaxf(fmaxf(wmax[t], wmax[64 + t]), fmaxf(wmax[128 + t], wmax[192 + t]));
          const float mo = m_s[t];
          const float mn = fmaxf(mo, mb);
          alpha_s[t] = (mn == -INFINITY) ? 1.f : fast_exp2(mo - mn);   // exp2(-inf) = 0
          m_s[t] = mn;
        }
        named_barrier_sync(3, 256);
        if (j > 0) {   // rescale this group's columns of O^T (all lanes) and of the normaliser row
          for (int c0 = 0; c0 < nqh; c0 += 8) {
            uint32_t r[8];
            tmem_ld8(lane_base + O_col + col0 + c0, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 8; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha_s[col0 + c0 + i]);
            tmem_st8(lane_base + O_col + col0 + c0, r);
            if (quad == 0) {
              tmem_ld8(lane_base + L_col + col0 + c0, r);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 8; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha_s[col0 + c0 + i]);
              tmem_st8(lane_base + L_col + col0 + c0, r);
            }
          }
          tmem_wait_st();
        }
        float unused = -INFINITY;
        write_p(unused);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s_empty[sb]);
        mbar_arrive(&p_full[sb]);
      }
      if (t == 0) SPECQ_TRACE_POINT(24, j);
    }
    // ---- final normaliser and accumulator ----
    if (nblk > 0) {
      // bounded even after a failure: the tensor core must be idle before TMEM is freed
      const int jl = nblk - 1;
      ok = mbar_wait(&pv_done[jl & 1], static_cast<uint32_t>(jl >> 1) & 1u, status, SPECQ_STATUS_TIMEOUT_MMA) && ok;
      tc_fence_after();
      if (quad == 0) {
        for (int c0 = 0; c0 < nqh; c0 += 8) {
          uint32_t r[8];
          tmem_ld8(lane_base + L_col + col0 + c0, r);
          tmem_wait_ld();
          if (lane == 0) {
#pragma unroll
            for (int i = 0; i < 8; ++i) l_s[col0 + c0 + i] = __uint_as_float(r[i]);
          }
        }
      }
    }
    named_barrier_sync(3, 256);
  } else if (warp == 8) {
    // =================================== TMA producer ===================================
    if (elect_one()) {
      const uint64_t pol = policy_evict_first();
      const int nbox = 128 / p.box_rows;
      // page ids of the next block are loaded into registers one block ahead (independent
      // loads, all in flight together), so the block-table latency overlaps the ring wait
      int pgv[16];
      auto load_pages = [&](int j) {
        const int tok0 = t_begin + j * 128;
        const int nb = (min(tok0 + 128, t_end) - tok0 + p.box_rows - 1) / p.box_rows;
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pgv[i] = (i < nb) ? __ldg(p.bt + b * p.bt_sb + (tok0 + i * p.box_rows) / p.page) : -1;
      };
      int issued = 0;
      if (nblk > 0) load_pages(0);
      for (int j = 0; j < nblk; ++j) {
        const int s = j % p.stages;
        if (!mbar_wait(&stage_empty[s], (static_cast<uint32_t>(j / p.stages) & 1u) ^ 1u, status,
                       SPECQ_STATUS_TIMEOUT_PIPELINE)) {
          ok = false;
          break;
        }
        const int tok0 = t_begin + j * 128;
        const int nb = (min(tok0 + 128, t_end) - tok0 + p.box_rows - 1) / p.box_rows;
        int* pg = pgs + s * 128;
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (i < nbox) pg[i] = pgv[i];
        for (int i = 16; i < nbox; ++i)      // page sizes below 8 tokens: more than 16 boxes
          pg[i] = (i < nb) ? __ldg(p.bt + b * p.bt_sb + (tok0 + i * p.box_rows) / p.page) : -1;
        SPECQ_TRACE_POINT(50, j);
        mbar_arrive_expect_tx(&stage_full[s], static_cast<uint32_t>(nb * p.box_rows * 128 * 2));
        uint8_t* kdst = ring + s * kAttnStage;
        uint8_t* vdst = kdst + kAttnKV8;
        for (int i = 0; i < nb; ++i) {
          const int tok = tok0 + i * p.box_rows;
          const int off = tok % p.page;
          tma_load_4d(kdst + i * p.box_rows * 128, &tmap_k, &stage_full[s], 0, kvh, off, pg[i], pol);
          tma_load_4d(vdst + i * p.box_rows * 128, &tmap_v, &stage_full[s], 0, kvh, off, pg[i], pol);
        }
        SPECQ_TRACE_POINT(51, j);
        ++issued;
        if (j + 1 < nblk) load_pages(j + 1);
      }
      if (!ok) {
        for (int j = max(0, issued - p.stages); j < issued; ++j)
          mbar_wait(&stage_full[j % p.stages], static_cast<uint32_t>(j / p.stages) & 1u, status,
                    SPECQ_STATUS_TIMEOUT_PIPELINE);
      }
    }
  } else if (warp == 9) {
    // =================================== MMA issuer ===================================
    if (elect_one()) {
      const uint32_t id_qk = idesc_f16(128, static_cast<uint32_t>(NQ));
      const uint32_t id_pv = idesc_f16(128, static_cast<uint32_t>(NQ), 1u, 0u);   // A (V^T) MN-major
      const uint32_t kop_a = smem_u32(kop), vop_a = smem_u32(vop), qop_a = smem_u32(qop), pop_a = smem_u32(pop);
      const uint32_t half_q = static_cast<uint32_t>(NQ) * 128u;
      auto issue_pv = [&](int i) {
        const uint32_t bi = static_cast<uint32_t>(i & 1);
        tc_fence_after();
        SPECQ_TRACE_POINT(32, i);
        const uint32_t vb = vop_a + bi * kAttnOp;
        const uint32_t pb = pop_a + bi * (2u * half_q);
#pragma unroll
        for (int k = 0; k < 8; ++k) {   // 16 tokens per step
          const uint64_t av = sdesc_sw128(vb + k * 2048u, 16384u, 1024u);
          const uint64_t bp = sdesc_sw128(pb + (k >> 2) * half_q + (k & 3) * 32u, 16u, 1024u);
          const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
          umma_f16_ss(tmem + O_col, av, bp, id_pv, acc);
          umma_f16_ts(tmem + L_col, tmem + ONES_col + 8u * k, bp, id_qk, acc);
        }
        umma_commit(&pv_done[bi]);
        SPECQ_TRACE_POINT(33, i);
      };
      auto issue_qk = [&](int j) {
        const uint32_t sb = static_cast<uint32_t>(j & 1);
        tc_fence_after();
        SPECQ_TRACE_POINT(30, j);
#pragma unroll
        for (int k = 0; k < 8; ++k) {   // 16 of the 128 head dims per step
          const uint64_t ak = sdesc_sw128(kop_a + (k >> 2) * 16384u + (k & 3) * 32u, 16u, 1024u);
          const uint64_t bq = sdesc_sw128(qop_a + (k >> 2) * half_q + (k & 3) * 32u, 16u, 1024u);
          umma_f16_ss(tmem + sb * cs, ak, bq, id_qk, k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[sb]);
        SPECQ_TRACE_POINT(31, j);
      };
      if (nblk > 0) ok = mbar_wait(q_full, 0u, status, SPECQ_STATUS_TIMEOUT_PIPELINE);
      // Event loop: QK(j) and PV(j) use disjoint TMEM, so each is issued as soon as its own
      // inputs are ready (PV(j) never waits behind the conversion of the next K tile).
      int nqk = 0, npv = 0;
      uint64_t idle_since = 0;
      while (ok && npv < nblk) {
        bool progressed = false;
        if (nqk < nblk && mbar_test_wait(k_full, static_cast<uint32_t>(nqk) & 1u) &&
            mbar_test_wait(&s_empty[nqk & 1], (static_cast<uint32_t>(nqk >> 1) & 1u) ^ 1u)) {
          issue_qk(nqk++);
          progressed = true;
        }
        if (npv < nqk) {
          const uint32_t bi = static_cast<uint32_t>(npv & 1);
          const uint32_t par = static_cast<uint32_t>(npv >> 1) & 1u;
          if (mbar_test_wait(&p_full[bi], par) && mbar_test_wait(&v_full[bi], par)) {
            issue_pv(npv++);
            progressed = true;
          }
        }
        if (progressed) {
          idle_since = 0;
        } else if (idle_since == 0) {
          idle_since = globaltimer_ns();
        } else if (globaltimer_ns() - idle_since > kWaitLimitNs) {
          report_status(status, SPECQ_STATUS_TIMEOUT_PIPELINE);
          ok = false;
        }
      }
    }
  } else {
    // =================================== converters ===================================
    const int c = static_cast<int>(threadIdx.x) - 320;   // 0..kAttnConvThreads-1
    float ks_cur = 0.f, vs_cur = 0.f;
    auto fetch_scales = [&](int j, float& ksv, float& vsv) -> bool {
      ksv = 0.f;
      vsv = 0.f;
      const int s = j % p.stages;
      if (!mbar_wait(&stage_full[s], static_cast<uint32_t>(j / p.stages) & 1u, status, SPECQ_STATUS_TIMEOUT_PIPELINE))
        return false;
      if (c < 128) {
        const int tok = t_begin + j * 128 + c;
        const int page = pgs[s * 128 + c / p.box_rows];
        if (tok < t_end && page >= 0 && page < p.n_pages) {
          const int64_t idx = static_cast<int64_t>(page) * p.s_sp + static_cast<int64_t>(tok % p.page) * p.s_so +
                              static_cast<int64_t>(kvh) * p.s_sh;
          ksv = load_scale(p.ks, p.scale_f32, idx);
          vsv = load_scale(p.vs, p.scale_f32, idx);
        }
      }
      return true;
    };
    if (nblk > 0) ok = fetch_scales(0, ks_cur, vs_cur);
    for (int j = 0; j < nblk; ++j) {
      const int s = j % p.stages;
      const uint32_t sb = static_cast<uint32_t>(j & 1);
      const uint32_t par2 = static_cast<uint32_t>(j >> 1) & 1u;
      if (c == 0) SPECQ_TRACE_POINT(40, j);
      const uint8_t* k8 = ring + s * kAttnStage;
      const uint8_t* v8 = k8 + kAttnKV8;
      // ---- K: the single fp16 K tile is free once QK(j-1) has completed
      if (j > 0)
        ok = ok && mbar_wait(&s_full[sb ^ 1u], static_cast<uint32_t>((j - 1) >> 1) & 1u, status,
                             SPECQ_STATUS_TIMEOUT_MMA);
      // 1024 16-byte chunks per tile: (token row = idx / 8, chunk = idx % 8)
      for (int idx = c; idx < 1024; idx += kAttnConvThreads) {
        const int row = idx >> 3;
        const int ch = idx & 7;
        const uint4 v = *reinterpret_cast<const uint4*>(k8 + row * 128 + ch * 16);
        uint32_t h[8];
        i8x16_to_f16(v, h);
        store_f16_chunk_pair(kop, row, ch, h);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(k_full);
      if (c == 0) SPECQ_TRACE_POINT(42, j);
      // ---- per-token scales of this block
      ok = ok && mbar_wait(&scl_empty[sb], par2 ^ 1u, status, SPECQ_STATUS_TIMEOUT_PIPELINE);
      if (c < 128) {
        scl_c[sb * 128 + c] = ks_cur * p.sm_scale_log2;
        scl_vh[sb * 128 + c] = __float2half_rn(vs_cur);
      }
      named_barrier_sync(1, kAttnConvThreads);
      __syncwarp();
      if (lane == 0) mbar_arrive(&scl_full[sb]);
      if (c == 0) SPECQ_TRACE_POINT(43, j);
      // ---- V (scale folded in) into buffer sb, free once PV(j-2) has completed
      if (j >= 2) ok = ok && mbar_wait(&pv_done[sb], par2 ^ 1u, status, SPECQ_STATUS_TIMEOUT_MMA);
      uint8_t* vdst = vop + sb * kAttnOp;
      for (int idx = c; idx < 1024; idx += kAttnConvThreads) {
        const int row = idx >> 3;
        const int ch = idx & 7;
        const uint4 v = *reinterpret_cast<const uint4*>(v8 + row * 128 + ch * 16);
        uint32_t h[8];
        i8x16_to_f16(v, h);
        // the token's V scale in fp16 (exact for fp16 scales; one rounding for fp32 scales), so
        // the per-element multiply stays on the fp16 pipe
        const __half2 s2 = __half2half2(scl_vh[sb * 128 + row]);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          __half2 o = __hmul2(*reinterpret_cast<__half2*>(&h[i]), s2);
          h[i] = *reinterpret_cast<uint32_t*>(&o);
        }
        store_f16_chunk_pair(vdst, row, ch, h);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&v_full[sb]);
        mbar_arrive(&stage_empty[s]);
      }
      if (c == 0) SPECQ_TRACE_POINT(45, j);
      if (j + 1 < nblk) ok = (ok && fetch_scales(j + 1, ks_cur, vs_cur)) && ok;
    }
  }
  __syncwarp();

  // ======================= epilogue: normalise, combine splits, store =======================
  // softmax warps: thread tl owns head dim d = tl (TMEM lane) for its group's query columns
  const bool soft = warp < 8;
  const int t = static_cast<int>(threadIdx.x);
  const int tl = t & 127;
  const int col0 = (t >> 7) * (NQ >> 1);
  const uint32_t o_lane = tmem + (((warp & 3u) * 32u) << 16) + O_col + static_cast<uint32_t>(col0);
  if (p.splits == 1) {
    if (soft && ok) {
      for (int c0 = 0; c0 < (NQ >> 1); c0 += 8) {
        uint32_t r[8];
        if (nblk > 0) {
          tmem_ld8(o_lane + c0, r);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) r[i] = 0u;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int q = col0 + c0 + i;
          if (q < rows_valid) {
            const int qi = q_lo + q / p.g;
            const int head = kvh * p.g + q % p.g;
            const float l = l_s[q];
            const float o = __uint_as_float(r[i]) / (l == 0.f ? 1.f : l);
            p.out[b * p.o_sb + static_cast<int64_t>(qi) * p.o_st + static_cast<int64_t>(head) * p.o_sh + tl] =
                __float2half_rn(o);
          }
        }
      }
    }
  } else {
    float* comb = reinterpret_cast<float*>(ring);   // [NQ][128] partial O (ring is idle now)
    if (soft) {
      for (int c0 = 0; c0 < (NQ >> 1); c0 += 8) {
        uint32_t r[8];
        if (nblk > 0 && ok) {
          tmem_ld8(o_lane + c0, r);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) r[i] = 0u;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) comb[(col0 + c0 + i) * 128 + tl] = __uint_as_float(r[i]);
      }
      if (nblk == 0 && t < 64) { m_s[t] = -INFINITY; l_s[t] = 0.f; }
    }
    cluster_sync();
    if (soft) {
      const int S = p.splits;
      const int lgdr = 7 - (31 - __clz(S));   // d columns per rank: 128 / S
      const int dr = 1 << lgdr;
      const int d0 = split * dr;
      for (int item = t; item < rows_valid * dr; item += 256) {
        const int q = item >> lgdr;
        const int d = d0 + (item & (dr - 1));
        float mp[8], lp[8], op[8];
#pragma unroll
        for (int pr = 0; pr < 8; ++pr) {     // every peer's loads in flight together
          if (pr < S) {
            mp[pr] = *dsmem_ptr(m_s + q, static_cast<uint32_t>(pr));
            lp[pr] = *dsmem_ptr(l_s + q, static_cast<uint32_t>(pr));
            op[pr] = *dsmem_ptr(comb + q * 128 + d, static_cast<uint32_t>(pr));
          }
        }
        float mmax = -INFINITY;
#pragma unroll
        for (int pr = 0; pr < 8; ++pr)
          if (pr < S) mmax = fmaxf(mmax, mp[pr]);
        float lsum = 0.f, osum = 0.f;
#pragma unroll
        for (int pr = 0; pr < 8; ++pr) {     // fixed order: identical bits for any schedule
          if (pr < S) {
            const float w = (mp[pr] == -INFINITY) ? 0.f : fast_exp2(mp[pr] - mmax);
            lsum += w * lp[pr];
            osum += w * op[pr];
          }
        }
        if (ok) {
          const int qi = q_lo + q / p.g;
          const int head = kvh * p.g + q % p.g;
          p.out[b * p.o_sb + static_cast<int64_t>(qi) * p.o_st + static_cast<int64_t>(head) * p.o_sh + d] =
              __float2half_rn(osum / (lsum == 0.f ? 1.f : lsum));
        }
      }
    }
    cluster_sync();
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) SPECQ_TRACE_POINT(9, 0);
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, p.tmem_cols);
  }
}

// ------------------------------------------------------------------------------------------
// host launcher
// ------------------------------------------------------------------------------------------
inline int run_paged_attention(const void* q, int64_t q_sb, int64_t q_st, int64_t q_sh, const int8_t* kc,
                               const int8_t* vc, int64_t kv_sp, int64_t kv_so, int64_t kv_sh, int n_pages,
                               const void* ks, const void* vs, int64_t s_sp, int64_t s_so, int64_t s_sh,
                               int scale_dtype, const int32_t* block_tbl, int64_t bt_sb, int bt_cols,
                               const int32_t* ctx_len, void* out, int64_t o_sb, int64_t o_st, int64_t o_sh,
                               const int32_t* plan, int B, int n_seqs, int q_len, int ql_max, int H, int H_KV, int D,
                               int page, int qpp, void* stream) {
  if (q == nullptr || kc == nullptr || vc == nullptr || ks == nullptr || vs == nullptr || block_tbl == nullptr ||
      ctx_len == nullptr || out == nullptr)
    return fail(SPECQ_ERR_INVALID_ARG, "paged_attention: null pointer");
  if (B < 0 || n_seqs < 0 || q_len < 0 || ql_max < 0 || H <= 0 || H_KV <= 0 || page <= 0 || n_pages < 0 ||
      bt_cols < 0)
    return fail(SPECQ_ERR_INVALID_ARG, "paged_attention: negative size");
  if (H % H_KV != 0) return fail(SPECQ_ERR_INVALID_ARG, "paged_attention: H=%d not a multiple of H_KV=%d", H, H_KV);
  if (D != 128) return fail(SPECQ_ERR_UNSUPPORTED, "paged_attention: head_dim %d (this build supports 128)", D);
  if (scale_dtype != SPECQ_DTYPE_F16 && scale_dtype != SPECQ_DTYPE_F32)
    return fail(SPECQ_ERR_INVALID_ARG, "paged_attention: scale dtype %d", scale_dtype);
  const int G = H / H_KV;
  if (G > 64) return fail(SPECQ_ERR_UNSUPPORTED, "paged_attention: GQA group %d > 64", G);
  if (qpp <= 0) return fail(SPECQ_ERR_INVALID_ARG, "paged_attention: QPP=%d", qpp);
  if (plan == nullptr && (n_seqs > B || q_len > ql_max))
    return fail(SPECQ_ERR_INVALID_ARG, "paged_attention: n_seqs/q_len exceed the q tensor");
  if (!aligned(kc, 16) || !aligned(vc, 16) || kv_sh % 16 || kv_so % 16 || kv_sp % 16)
    return fail(SPECQ_ERR_UNSUPPORTED, "paged_attention: KV cache strides must be multiples of 16 bytes");
  if (!aligned(q, 16) || (q_sb * 2) % 16 || (q_st * 2) % 16 || (q_sh * 2) % 16)
    return fail(SPECQ_ERR_UNSUPPORTED, "paged_attention: q rows must be 16-byte aligned");
  const int b_grid = plan ? B : n_seqs;
  const int ql_grid = plan ? ql_max : q_len;
  if (b_grid == 0 || ql_grid == 0 || n_pages == 0) return SPECQ_OK;
  DeviceState* dev = nullptr;
  if (int rc = get_device_state(&dev)) return rc;

  AttnParams p = {};
  p.q = static_cast<const __half*>(q);
  p.q_sb = q_sb; p.q_st = q_st; p.q_sh = q_sh;
  p.ks = ks; p.vs = vs;
  p.s_sp = s_sp; p.s_so = s_so; p.s_sh = s_sh;
  p.scale_f32 = scale_dtype == SPECQ_DTYPE_F32;
  p.bt = block_tbl; p.bt_sb = bt_sb; p.bt_cols = bt_cols;
  p.ctx_len = ctx_len;
  p.out = static_cast<__half*>(out);
  p.o_sb = o_sb; p.o_st = o_st; p.o_sh = o_sh;
  p.plan = plan;
  p.status = dev->status;
  p.n_pages = n_pages;
  p.b_grid = b_grid; p.n_seqs = n_seqs; p.q_len = q_len; p.ql_max = ql_max;
  p.h_kv = H_KV; p.g = G; p.page = page;
  p.qpp = std::min(qpp, 64 / G);                 // QPP only changes the schedule
  p.nq = round_up(p.qpp * G, 16);
  p.n_qc = ceil_div(ql_grid, p.qpp);
  int br = 1;
  while (br < 16 && page % (br * 2) == 0) br *= 2;
  p.box_rows = br;
  // Split count from the block-table width only (never from B or the plan), so eager and
  // plan-mode launches reduce identical partials.
  const int max_ctx = bt_cols * page;
  p.splits = std::min(8, std::max(1, ceil_div(max_ctx, 2048)));
  p.stages = 2;
  p.sm_scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(D));
  p.col_stride = static_cast<uint32_t>(round_up(p.nq, 32));
  p.tmem_cols = static_cast<uint32_t>(next_pow2(static_cast<int>(4 * p.col_stride + 128)));
  if (p.tmem_cols > 512) return fail(SPECQ_ERR_UNSUPPORTED, "paged_attention: too many query rows per CTA");
  if (static_cast<int64_t>(b_grid) * p.n_qc > 65535)
    return fail(SPECQ_ERR_UNSUPPORTED, "paged_attention: grid too large");

  // ring + fp16 K tile + two fp16 V tiles + Q + two P^T tiles + scales + softmax state + pages
  const int smem = 1024 + p.stages * static_cast<int>(kAttnStage) + 3 * static_cast<int>(kAttnOp) + 3 * p.nq * 256 +
                   512 * 4 + 448 * 4 + p.stages * 128 * 4 + (2 * p.stages + 16) * 8 + 64;
  if (smem > 232448) return fail(SPECQ_ERR_UNSUPPORTED, "paged_attention: shared memory %d too large", smem);
  if (p.nq * 128 * 4 > p.stages * static_cast<int>(kAttnStage))
    return fail(SPECQ_ERR_UNSUPPORTED, "paged_attention: combine buffer does not fit");

  CUtensorMap tk, tv;
  const uint64_t dims[4] = {128u, static_cast<uint64_t>(H_KV), static_cast<uint64_t>(page), static_cast<uint64_t>(n_pages)};
  const uint64_t strides[3] = {static_cast<uint64_t>(kv_sh), static_cast<uint64_t>(kv_so), static_cast<uint64_t>(kv_sp)};
  const uint32_t box[4] = {128u, 1u, static_cast<uint32_t>(br), 1u};
  if (int rc = encode_tiled(&tk, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, kc, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE)) return rc;
  if (int rc = encode_tiled(&tv, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, vc, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE)) return rc;

  const dim3 grid(static_cast<unsigned>(p.splits), static_cast<unsigned>(H_KV),
                  static_cast<unsigned>(b_grid * p.n_qc));
  SPECQ_CUDA_TRY(cudaFuncSetAttribute(paged_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kAttnThreads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(p.splits);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = p.splits > 1 ? 1 : 0;
  SPECQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, paged_attn_kernel, p, tk, tv));
  LaunchRecord& r = last_launch_ref();
  r.variant = 0;
  r.grid[0] = static_cast<int>(grid.x); r.grid[1] = static_cast<int>(grid.y); r.grid[2] = static_cast<int>(grid.z);
  r.cluster_x = p.splits;
  r.threads = kAttnThreads;
  r.dyn_smem = smem;
  return SPECQ_OK;
}

inline const void* paged_attn_kernel_by_variant(int variant) {
  return variant == 0 ? reinterpret_cast<const void*>(paged_attn_kernel) : nullptr;
}

}  // namespace specq
