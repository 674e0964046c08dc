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
//     tensor-core lane is wasted on padding query rows.
//   * The CTA's slice of the block table is read once into shared memory.  K and V arrive by
//     TMA (boxes of up to 16 slots of one page and one KV head, 128B-swizzled; K and V issued
//     by two warps in parallel) into a 3-stage ring: bytes in flight cost no registers or
//     load/store slots.  K feeds an INT8 MMA as it lands: the query rows are quantised once
//     per CTA to int16 with one scale (amax/32639) and split hi*256 + lo into two int8 operand
//     rows, so one kind::i8 MMA with N = 2*NQ gives both integer partial products exactly in
//     int32.  Four warps (one thread per token row) dequantise V to fp16 with the token's
//     scale folded in; the V tile is read MN-major by the PV product.  Per-token scales are
//     fetched two blocks ahead by cp.async into shared memory by the threads that use them.
//   * Softmax runs one thread per token row of S^T (TMEM lane = token): the per-token K scale
//     and the query scale fold into one per-thread scalar, the running max of each query column
//     lives in registers; the arithmetic runs on packed fp32 pairs.  The running max is "lazy": a block is exponentiated against the
//     current max and only when some score exceeds it by more than 2^8 does the CTA reduce
//     the block max, rescale O^T and the normaliser, and recompute.  Blocks that lie wholly
//     inside every query row's causal window take a mask-free path.  P is written MN-major
//     (one 16-byte store per 8 query rows).  The normaliser l = sum_t p is produced by the
//     tensor core itself (a ones operand in TMEM times P).  The score buffers are reset to
//     their bias by the MMA issuer with one fp16 MMA (see kScoreBias), in order with the QK
//     MMAs, so the softmax threads never write tensor memory in the steady state.
//   * Long contexts are split across a thread-block cluster (a power of two, from the
//     block-table width only, so plan mode and eager mode give the same bits).  Each CTA
//     pushes its partial (m, l, O) for the head dims a peer owns into that peer's shared
//     memory; every CTA then combines its own head dims in fixed split order.
//   * Plan mode reads (n_seqs, q_len) on the device; CTAs outside them return, nothing outside
//     them is written.
#pragma once

#include <type_traits>

#include "sm100.cuh"
#include "specq_host.cuh"

namespace specq {

struct AttnParams {
  const __half* q;
  int64_t q_sb, q_st, q_sh;
  const int8_t* kc;
  const int8_t* vc;
  int64_t kv_sp, kv_so, kv_sh;
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
  int g_shift, page_shift;  // log2 of g / page when they are powers of two, else -1
  int splits, stages;
  int box_rows, box_shift; // K tiles arrive by TMA in boxes of box_rows slots of one page
  float sm_scale_log2;     // log2(e) / sqrt(D)
  uint32_t tmem_cols;
  uint32_t col_stride;     // TMEM columns of one score buffer (2 * nq int32, rounded to 32)
  uint32_t o_cols;         // TMEM columns of O^T and of the normaliser (nq, rounded to 32)
  int out_vec;             // out rows are 16-byte aligned: 8 head dims per store
};

// warps [0, 8) softmax, 8 K gather + 9 V gather (TMA), 10 MMA issue + TMEM owner,
// [11, 15) V conversion
constexpr int kAttnLoadWarps = 2;
constexpr int kAttnMmaWarp = 8 + kAttnLoadWarps;
constexpr int kAttnConvWarps = 4;              // one thread per token row of a block
constexpr int kAttnThreads = 32 * (kAttnMmaWarp + 1) + 32 * kAttnConvWarps;
constexpr uint32_t kAttnKV8 = 128 * 128;       // int8 K (or V) block: 128 tokens x 128 B
constexpr uint32_t kAttnStage = 2 * kAttnKV8;  // K + V, both 128B-swizzled
constexpr uint32_t kAttnOp = 128 * 256;        // fp16 V tile: 128 tokens x 128 d
constexpr int kAttnStages = 3;
constexpr int kAttnMaxPages = 2048;            // block-table entries of one CTA's context range
constexpr uint32_t kAttnPTile = 128 * 128;     // fp16 P tile: 128 tokens x 64 query rows
constexpr float kLazyMaxLog2 = 8.0f;           // rescale once a score exceeds the max by 2^8
// 32-bit words of the bias MMA's constant B operand in shared memory (256 bytes used)
__host__ __device__ constexpr int attn_bias_words(int) { return 64; }



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
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
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

// Packed fp32 pairs (sm_100 f32x2 arithmetic: two lanes of work per instruction).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// The score accumulators start every block at the bit pattern of 1.5 * 2^23 (kScoreBias), so
// the int8 MMA leaves 1.5 * 2^23 + S in each column: read as a float that is S plus a constant
// (|S| < 2^22), with no integer-to-float conversion.  256 * hi + lo then comes out of one
// fused multiply-add and one exact subtraction of 257 * 1.5 * 2^23 (the sum rounds to a
// multiple of 256 near 2^31.6: an error of at most 128 units of the int16-scaled query,
// below the query's own quantisation error).
constexpr uint32_t kScoreBias = 0x4B400000u;
constexpr float kScoreBias257 = 3233808384.f;   // 257 * 1.5 * 2^23, exact in fp32
// The bias is written by one kind::f16 MMA with accumulate off: sixteen products
// 1024.0 x 768.0 (fp16 operands, exact) sum to 12582912.0 = 1.5 * 2^23 exactly, whose fp32 bit
// pattern is kScoreBias; the INT8 MMAs of the QK product then accumulate onto those bits as
// int32 (tensor memory is untyped).
constexpr uint32_t kBias1024x2 = 0x64006400u;   // fp16 1024.0, twice
constexpr uint32_t kBias768x2 = 0x62006200u;    // fp16 768.0, twice

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                            int w, uint64_t cache_hint) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w), "l"(cache_hint)
      : "memory");
}

template <int NQ>
__global__ void __launch_bounds__(kAttnThreads, 1)
    paged_attn_kernel(const __grid_constant__ AttnParams p, const __grid_constant__ CUtensorMap tmap_k,
                      const __grid_constant__ CUtensorMap tmap_v) {
  static_assert(NQ % 16 == 0 && NQ >= 16 && NQ <= 64, "query rows per CTA");
  constexpr int NQH = NQ / 2;   // query columns per softmax thread
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  SPECQ_TRACE_INIT();
  if (threadIdx.x == 0) {
    SPECQ_TRACE_POINT(0, 0);
    tma_prefetch_desc(&tmap_k);   // kernel parameters: fetched while the previous kernel finishes
    tma_prefetch_desc(&tmap_v);
  }
  pdl_wait();                // the previous kernel's writes are visible from here on
  if (threadIdx.x == 0) SPECQ_TRACE_POINT(3, 0);
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // ring stage: [K int8, 128 tokens x 128 B, 128B-swizzled (a tcgen05 operand as it lands)]
  //             [V int8, 128 tokens x 128 B, 128B-swizzled (read row-wise by the V warps)]
  uint8_t* ring = smem;
  uint8_t* vop = ring + kAttnStages * kAttnStage;                  // fp16 V tiles x2 [2][128][128 B]
  uint8_t* qop = vop + 2 * kAttnOp;                                // int8 Q: hi rows [0,NQ), lo rows [NQ,2NQ)
  uint8_t* pop = qop + NQ * 256;                                   // fp16 P x2 [2][128 tokens][128 B]
  float* m_s = reinterpret_cast<float*>(pop + 2 * kAttnPTile);     // [64] running max (log2 units)
  float* nm_s = m_s + 64;                                          // [64] -m_s
  float* alpha_s = nm_s + 64;                                      // [64]
  float* l_s = alpha_s + 64;                                       // [64]
  float* qamax = l_s + 64;                                         // [64] |q| max per query row
  float* wmax = qamax + 64;                                        // [4][64]
  float* ks_ring = wmax + 256;                                     // [3][256] softmax threads' K scales
  float* vs_ring = ks_ring + 3 * 256;                              // [3][128] V threads' V scales
  uint32_t* bias_s = reinterpret_cast<uint32_t*>(vs_ring + 3 * 128); // the score bias, copied into TMEM
  int* pages_s = reinterpret_cast<int*>(bias_s + attn_bias_words(NQ)); // [kAttnMaxPages] this CTA's page ids
  uint64_t* bars = reinterpret_cast<uint64_t*>(pages_s + kAttnMaxPages);
  uint64_t* stage_full = bars;
  uint64_t* stage_empty = stage_full + kAttnStages;
  uint64_t* v_full = stage_empty + kAttnStages;   // [2]
  uint64_t* s_full = v_full + 2;                  // [2]
  uint64_t* p_full = s_full + 2;                  // [2]  P(j) written, score buffer j % 2 read
  uint64_t* pv_done = p_full + 2;                 // [2]  PV of the last two blocks done (see wait_pv)
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
  // A zero sequence stride means packed token rows (sequence b's token t at row
  // b * q_len + t): the stride follows the active q_len, e.g. a projection's output under a
  // plan-buffer graph.
  const int64_t q_sb = p.q_sb != 0 ? p.q_sb : static_cast<int64_t>(q_len) * p.q_st;
  const int64_t o_sb = p.o_sb != 0 ? p.o_sb : static_cast<int64_t>(q_len) * p.o_st;
  const int q_lo = qc * p.qpp;
  const int q_hi = min(q_lo + p.qpp, q_len);
  const int rows_valid = (q_hi - q_lo) * p.g;

  // The sequence length, the block-table row (when it fits in shared memory) and the query
  // rows do not depend on one another: they are all requested here, so the prologue waits for
  // one memory round trip instead of three dependent ones.
  int L = __ldg(p.ctx_len + b);
  // softmax warps: the raw fp16 query pieces (row, 16 head dims) this thread quantises below
  constexpr int kItems = (NQ * 8 + 255) / 256;
  uint4 qraw[kItems][2];
  if (warp < 8) {
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      const int it = static_cast<int>(threadIdx.x) + 256 * k;
      const int row = it >> 3;
      const int piece = it & 7;
      qraw[k][0] = qraw[k][1] = make_uint4(0u, 0u, 0u, 0u);
      if (it < NQ * 8 && row < rows_valid) {
        const int qi = q_lo + (p.g_shift >= 0 ? (row >> p.g_shift) : (row / p.g));
        const int head = kvh * p.g + (p.g_shift >= 0 ? (row & (p.g - 1)) : (row % p.g));
        const uint4* src = reinterpret_cast<const uint4*>(p.q + b * q_sb + static_cast<int64_t>(qi) * p.q_st +
                                                          static_cast<int64_t>(head) * p.q_sh) + 2 * piece;
        qraw[k][0] = ldg_nc_v4_now(src);
        qraw[k][1] = ldg_nc_v4_now(src + 1);
      }
    }
  }
  const bool whole_row = p.bt_cols <= kAttnMaxPages;
  if (whole_row)
    for (int i = static_cast<int>(threadIdx.x); i < p.bt_cols; i += kAttnThreads)
      pages_s[i] = __ldg(p.bt + b * p.bt_sb + i);
  if (L < 0 || L > p.bt_cols * p.page) {
    if (threadIdx.x == 0 && split == 0) report_status(p.status, SPECQ_STATUS_PLAN_CLAMPED);
    L = min(max(L, 0), p.bt_cols * p.page);
  }
  const int qpos0 = L - q_len + q_lo;                 // last visible token of query-row group 0
  const int kv_end = max(0, L - q_len + q_hi);
  const int tchunk = ((kv_end + p.splits - 1) / p.splits + 127) & ~127;
  const int t_begin = split * tchunk;
  const int t_end = min(kv_end, t_begin + tchunk);
  const int nblk = (t_end > t_begin) ? (t_end - t_begin + 127) / 128 : 0;

  constexpr uint32_t cs2 = static_cast<uint32_t>((2 * NQ + 31) & ~31);   // S buffer: hi columns, lo columns
  constexpr uint32_t kOCols = static_cast<uint32_t>((NQ + 31) & ~31);
  constexpr uint32_t O_col = 2 * cs2;
  constexpr uint32_t L_col = O_col + kOCols;
  constexpr uint32_t ONES_col = L_col + kOCols;
  auto page_of = [&](int tok) { return p.page_shift >= 0 ? (tok >> p.page_shift) : (tok / p.page); };
  auto slot_of = [&](int tok) { return p.page_shift >= 0 ? (tok & (p.page - 1)) : (tok % p.page); };
  // The block-table entries of this CTA's token range live in shared memory (the whole row
  // read above, or else this range's entries, read here): a page lookup is then a
  // shared-memory read instead of a dependent global load (which takes longer than a whole
  // block under full HBM load).
  const int pg_first = whole_row ? 0 : page_of(t_begin);
  if (!whole_row) {
    const int pg_count = nblk > 0 ? page_of(t_end - 1) - pg_first + 1 : 0;
    for (int i = static_cast<int>(threadIdx.x); i < pg_count; i += kAttnThreads)
      pages_s[i] = __ldg(p.bt + b * p.bt_sb + pg_first + i);
  }
  // page id of token row `row` of block j (-1 past the split end)
  auto token_page = [&](int j, int row) -> int {
    const int tok = t_begin + j * 128 + row;
    return (j < nblk && tok < t_end) ? pages_s[page_of(tok) - pg_first] : -1;
  };
  // element offset of that token's (page, slot, kv head) in the KV cache and in the scales
  auto kv_offset = [&](int j, int row, int page) -> int64_t {
    const int tok = t_begin + j * 128 + row;
    return static_cast<int64_t>(page) * p.kv_sp + static_cast<int64_t>(slot_of(tok)) * p.kv_so +
           static_cast<int64_t>(kvh) * p.kv_sh;
  };
  auto scale_offset = [&](int j, int row, int page) -> int64_t {
    const int tok = t_begin + j * 128 + row;
    return static_cast<int64_t>(page) * p.s_sp + static_cast<int64_t>(slot_of(tok)) * p.s_so +
           static_cast<int64_t>(kvh) * p.s_sh;
  };
  auto page_ok = [&](int page) { return page >= 0 && page < p.n_pages; };
  // The per-token scale of token row `row` of block j, fetched by cp.async into *dst two
  // blocks before it is used (0 past the split end or on a bad page): the consumer reads it
  // from shared memory, so no register waits on a global load.  fp16 scales: the aligned
  // 4-byte word holding the value is copied (it never crosses a page, so it is mapped memory)
  // and bit `slot` of `sel` records which half the value is.
  // With a power-of-two page of at most one block, token row `row` keeps its slot in every
  // block and its place in the CTA's page list advances by 128 / page per block: the scale
  // address of block j is then one shared-memory read and one multiply-add (this runs on the
  // softmax warps' per-block critical path).
  const bool steady_pages = p.page_shift >= 0 && p.page <= 128;
  struct ScaleRow {
    int row, tok0, pidx0, pstep;
    int64_t soff;
  };
  auto scale_row = [&](int row) {
    ScaleRow r;
    r.row = row;
    r.tok0 = t_begin + row;
    r.pidx0 = steady_pages ? (r.tok0 >> p.page_shift) - pg_first : 0;
    r.pstep = steady_pages ? (128 >> p.page_shift) : 0;
    r.soff = steady_pages ? static_cast<int64_t>(r.tok0 & (p.page - 1)) * p.s_so + static_cast<int64_t>(kvh) * p.s_sh : 0;
    return r;
  };
  // The page of token row r.row in block j (-1 past the split end).  Split from fetch_scale so
  // the shared-memory read can be issued early and consumed later in the block.
  auto scale_page = [&](int j, const ScaleRow& r) -> int {
    if (steady_pages) return (j < nblk && r.tok0 + j * 128 < t_end) ? pages_s[r.pidx0 + j * r.pstep] : -1;
    return token_page(j, r.row);
  };
  auto fetch_scale = [&](const void* base, int j, const ScaleRow& r, int pg, float* dst, uint32_t& sel, int slot) {
    int64_t off = 0;
    if (steady_pages) {
      off = static_cast<int64_t>(pg) * p.s_sp + r.soff;
    } else if (pg >= 0) {
      off = scale_offset(j, r.row, pg);
    }
    if (page_ok(pg)) {
      if (p.scale_f32) {
        cp_async4(dst, static_cast<const float*>(base) + off);
      } else {
        const uintptr_t a = reinterpret_cast<uintptr_t>(static_cast<const __half*>(base) + off);
        cp_async4(dst, reinterpret_cast<const void*>(a & ~uintptr_t(3)));
        sel = (sel & ~(1u << slot)) | (static_cast<uint32_t>((a >> 1) & 1u) << slot);
      }
    } else {
      *dst = 0.f;
    }
    cp_async_commit();
  };
  auto read_scale = [&](const float* src, uint32_t sel, int slot) -> float {
    if (p.scale_f32) return *src;
    const uint32_t w = *reinterpret_cast<const uint32_t*>(src);
    return __half2float(__ushort_as_half(static_cast<unsigned short>(((sel >> slot) & 1u) ? (w >> 16) : w)));
  };

  // PV(i) has completed once this returns.  PV(i) and QK(i+2) are issued together and QK(i+2)'s
  // commit (s_full) comes after PV(i) from the same thread, so it also covers PV(i); only the
  // last two blocks, which have no QK(i+2), commit to pv_done (each buffer once: phase 0).
  // A parity wait is only meaningful when the barrier can be neither behind nor two phases
  // ahead of the awaited phase: the softmax has seen every earlier S complete, and the V warps
  // see QK(0) / QK(1) complete before they release V(0) / V(1).
  auto wait_pv = [&](int i, int code) -> bool {
    if (i + 2 < nblk) return mbar_wait(&s_full[i & 1], static_cast<uint32_t>((i + 2) >> 1) & 1u, p.status, code);
    return mbar_wait(&pv_done[i & 1], 0u, p.status, code);
  };

  // ---- setup ---------------------------------------------------------------------------------
  if (threadIdx.x == 0) {
    for (int s = 0; s < kAttnStages; ++s) {
      mbar_init(&stage_full[s], 2u);                     // the K and the V gather lanes' expect_tx
      mbar_init(&stage_empty[s], 1u + kAttnConvWarps);  // the QK commit + the V warps
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&v_full[i], kAttnConvWarps);
      mbar_init(&s_full[i], 1u);
      mbar_init(&p_full[i], 8u);
      mbar_init(&pv_done[i], 1u);
    }
    mbar_init(q_full, 8u);
    fence_barrier_init();
  }
  if (warp == kAttnMmaWarp) {
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
    const int col0 = grp * NQH;
    const uint32_t quad = warp & 3u;
    const uint32_t lane_base = tmem + ((quad * 32u) << 16);
    // Q rows -> int16 with one scale for the CTA (gmax / 32639), split as hi * 256 + lo with
    // hi, lo int8: two int8 operand rows each, so QK^T runs on the INT8 tensor core against
    // the raw K bytes.  One scale makes the score scale a per-token scalar (no per-column
    // constant); the rounding error of every row is relative to the CTA's largest |q|.
    float qv[kItems][16];   // (row, 16 head dims) pieces of this thread, loaded in the prologue
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      const int it = t + 256 * k;
      const int row = it >> 3;
      const int piece = it & 7;
      float amax = 0.f;
      if (it < NQ * 8 && row < rows_valid) {
        const uint4 u0 = qraw[k][0], u1 = qraw[k][1];
        const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
          qv[k][2 * i] = f.x;
          qv[k][2 * i + 1] = f.y;
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(qv[k][i]));
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) qv[k][i] = 0.f;
      }
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
      if (it < NQ * 8 && piece == 0) qamax[row] = amax;
    }
    named_barrier_sync(3, 256);
    if (t == 0) SPECQ_TRACE_POINT(11, 0);
    // the CTA's largest |q|: two rows per lane, one warp reduction (|q| >= 0, so 0 is neutral)
    const float gmax = warp_max_f32(fmaxf(static_cast<int>(lane) < NQ ? qamax[lane] : 0.f,
                                          static_cast<int>(lane) + 32 < NQ ? qamax[lane + 32] : 0.f));
    const float q_inv = gmax > 0.f ? 32639.f / gmax : 0.f;
    const float q_scale = gmax / 32639.f;
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      const int it = t + 256 * k;
      if (it >= NQ * 8) break;
      const int row = it >> 3;
      const int piece = it & 7;
      uint32_t hw[4] = {0u, 0u, 0u, 0u}, lw[4] = {0u, 0u, 0u, 0u};
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int v16 = __float2int_rn(qv[k][i] * q_inv);    // |v16| <= 32639
        const int hi = (v16 + 128) >> 8;                     // in [-127, 127]
        const int lo = v16 - (hi << 8);                      // in [-128, 127]
        hw[i >> 2] |= (static_cast<uint32_t>(hi) & 0xFFu) << (8 * (i & 3));
        lw[i >> 2] |= (static_cast<uint32_t>(lo) & 0xFFu) << (8 * (i & 3));
      }
      *reinterpret_cast<uint4*>(qop + sw128_offset(row, piece)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4*>(qop + sw128_offset(NQ + row, piece)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
    // padding rows (all-zero queries, never stored) start at max 0: their scores are exactly 0,
    // so they never trigger a rescale and the interior blocks need no column mask
    if (t < 64) {
      m_s[t] = t < rows_valid ? -INFINITY : 0.f;
      nm_s[t] = t < rows_valid ? INFINITY : 0.f;
      alpha_s[t] = 1.f;
      l_s[t] = 0.f;
    }
    // the constant the MMA issuer copies into a score buffer before each QK (tcgen05.cp)
    // B operand of the bias MMA: fp16 768.0 pairs (see kScoreBias)
    for (int w = t; w < attn_bias_words(NQ); w += 256) bias_s[w] = kBias768x2;
    if (grp == 0) {   // A operands in TMEM: 8 columns of fp16 1.0 (normaliser), 8 of 1024.0 (bias)
      uint32_t ones[16];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        ones[i] = 0x3C003C00u;
        ones[8 + i] = kBias1024x2;
      }
      tmem_st16(lane_base + ONES_col, ones);
    }
    tmem_wait_st();
    fence_proxy_async_smem();
    tc_fence_before();
    named_barrier_sync(3, 256);
    __syncwarp();
    if (lane == 0) mbar_arrive(q_full);
    if (t == 0) SPECQ_TRACE_POINT(13, 0);

    // -max of this thread's query columns, kept in registers (changes only on a rescale)
    float nmr[NQH];
#pragma unroll
    for (int i = 0; i < NQH; ++i) nmr[i] = nm_s[col0 + i];

    // Multi-thread roles never leave a loop early: after a wait runs out (ok = false) they skip
    // the remaining waits but still reach every named barrier, so no warp is stranded.
    // One copy of the block body (a plain loop, not unrolled): the softmax, V and MMA roles
    // share each scheduler's instruction cache, so the hot code is kept small.
    float* ksd = ks_ring + t;     // this thread's K-scale slots (stride 256)
    uint32_t ksel = 0u;
    const ScaleRow krow = scale_row(tl);
    fetch_scale(p.ks, 0, krow, scale_page(0, krow), ksd, ksel, 0);
    fetch_scale(p.ks, 1, krow, scale_page(1, krow), ksd + 256, ksel, 1);
    int slot = 0;                 // j % 3
#pragma unroll 1
    for (int j = 0; j < nblk; ++j) {
      const int slot2 = slot == 0 ? 2 : slot - 1;   // (j + 2) % 3
      const int pg2 = scale_page(j + 2, krow);   // page of this token in block j + 2
      const int t_abs = t_begin + j * 128 + tl;
      const uint32_t sb = static_cast<uint32_t>(j & 1);
      const uint32_t par2 = static_cast<uint32_t>(j >> 1) & 1u;
      // query rows q >= q_first may see this token (causal window), rows >= q_stop never do
      const int q_stop = (t_abs < t_end) ? rows_valid : 0;
      const int q_first = min(max(0, (t_abs - qpos0) * p.g), q_stop);
      if (t == 0) SPECQ_TRACE_POINT(20, j);
      cp_async_wait<1>();   // block j's scale (fetched two blocks ago) has landed
      // this token's score scale: K scale x log2(e) / sqrt(D) x the query scale
      const float a_t = read_scale(ksd + 256 * slot, ksel, slot) * p.sm_scale_log2 * q_scale;
      // block j + 2's scale into the slot block j - 1 used (issued here, at the top of the
      // block, it measured faster than after the P pass)
      fetch_scale(p.ks, j + 2, krow, pg2, ksd + 256 * slot2, ksel, slot2);
      // S(j) is ready; its commit also covers PV(j-2), so P buffer sb is free as well
      ok = ok && mbar_wait(&s_full[sb], par2, status, SPECQ_STATUS_TIMEOUT_MMA);
      tc_fence_after();
      if (t == 0) SPECQ_TRACE_POINT(21, j);
      const uint32_t s_addr = lane_base + sb * cs2 + col0;
      uint8_t* prow = pop + sb * kAttnPTile;   // P[token][query], MN-major, 128B-swizzled rows
      // every token of the block is visible to every query row: no column mask
      const int t_last = t_begin + j * 128 + 127;
      const bool interior = t_last < t_end && t_last <= qpos0;
      const float2 a2 = make_float2(a_t, a_t);

      // scaled score (log2 units) of query column q from its biased hi / lo accumulators
      auto score = [&](uint32_t hb, uint32_t lb) {
        return (fmaf(__uint_as_float(hb), 256.f, __uint_as_float(lb)) - kScoreBias257) * a_t;
      };
      // One pass: P against the current max, noting the largest exponent.
      auto write_p = [&](float& xmax) {
#pragma unroll
        for (int c0 = 0; c0 < NQH; c0 += 16) {   // 16 columns per TMEM round trip (hi and lo)
          constexpr int kW = 16;
          uint32_t rh[kW], rl[kW];
          const bool two = c0 + 8 < NQH;
          tmem_ld8(s_addr + c0, *reinterpret_cast<uint32_t(*)[8]>(rh));
          tmem_ld8(s_addr + NQ + c0, *reinterpret_cast<uint32_t(*)[8]>(rl));
          if (two) {
            tmem_ld8(s_addr + c0 + 8, *reinterpret_cast<uint32_t(*)[8]>(rh + 8));
            tmem_ld8(s_addr + NQ + c0 + 8, *reinterpret_cast<uint32_t(*)[8]>(rl + 8));
          }
          tmem_wait_ld();
          if (t == 0 && c0 == 0) SPECQ_TRACE_POINT(28, j);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (h == 1 && !two) break;
            const int qb = col0 + c0 + 8 * h;
            uint32_t pk[4];
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
              const int r0 = 8 * h + i;
              const float2 hb = make_float2(__uint_as_float(rh[r0]), __uint_as_float(rh[r0 + 1]));
              const float2 lb = make_float2(__uint_as_float(rl[r0]), __uint_as_float(rl[r0 + 1]));
              const float2 sv = fadd2(ffma2(hb, make_float2(256.f, 256.f), lb),
                                      make_float2(-kScoreBias257, -kScoreBias257));
              float2 x = ffma2(sv, a2, make_float2(nmr[c0 + r0], nmr[c0 + r0 + 1]));
              if (!interior) {   // causal window and split end; padding rows
                const uint32_t span = static_cast<uint32_t>(q_stop - q_first);
                x.x = static_cast<uint32_t>(qb + i - q_first) < span ? x.x : -INFINITY;
                x.y = static_cast<uint32_t>(qb + i + 1 - q_first) < span ? x.y : -INFINITY;
              }
              xmax = fmax3(xmax, x.x, x.y);
              const __half2 ph = __floats2half2_rn(fast_exp2(x.x), fast_exp2(x.y));
              pk[i >> 1] = *reinterpret_cast<const uint32_t*>(&ph);
            }
            *reinterpret_cast<uint4*>(prow + sw128_offset(static_cast<uint32_t>(tl), static_cast<uint32_t>(qb >> 3))) =
                make_uint4(pk[0], pk[1], pk[2], pk[3]);
          }
        }
      };
#pragma unroll
      for (int pass = 0; pass < 2; ++pass) {   // two straight-line copies: faster than a loop
        // Block 0 always rescales (the running max starts at -inf and the split's first token is
        // visible to its last query row), so its first pass, whose P would be overwritten, is
        // skipped.
        if (pass == 1 || j > 0) {
          float xmax = -INFINITY;
          write_p(xmax);
          if (pass == 1) break;
          const bool need = named_barrier_or(2, 256, xmax > kLazyMaxLog2);
          if (t == 0) SPECQ_TRACE_POINT(22, j);
          if (!need) break;
        }
        // ---- rescale: some score exceeds the running max by more than 2^8 ----
        if (t == 0) SPECQ_TRACE_POINT(26, j);
        // the running O^T / normaliser must be final before they are rescaled
        if (j >= 1) ok = ok && wait_pv(j - 1, SPECQ_STATUS_TIMEOUT_MMA);
        tc_fence_after();
        // block max per query column: warp shuffles, then across the four lane quadrants
#pragma unroll
        for (int c0 = 0; c0 < NQH; c0 += 8) {
          uint32_t rh[8], rl[8];
          tmem_ld8(s_addr + c0, rh);
          tmem_ld8(s_addr + NQ + c0, rl);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int q = col0 + c0 + i;
            const float y = warp_max_f32((q >= q_first && q < q_stop) ? score(rh[i], rl[i]) : -INFINITY);
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
          nm_s[t] = -mn;
        }
        named_barrier_sync(3, 256);
#pragma unroll
        for (int i = 0; i < NQH; ++i) nmr[i] = nm_s[col0 + i];
        if (j > 0) {   // rescale this group's columns of O^T (all lanes) and of the normaliser row
#pragma unroll
          for (int c0 = 0; c0 < NQH; c0 += 8) {
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
      }
      // P(j) is complete and score buffer sb has been read for the last time
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sb]);
      if (t == 0) SPECQ_TRACE_POINT(24, j);
      if (t == 0) SPECQ_TRACE_POINT(27, j);
      slot = slot == 2 ? 0 : slot + 1;
    }
    cp_async_wait<0>();
    // ---- final normaliser and accumulator ----
    if (nblk > 0) {
      // bounded even after a failure: the tensor core must be idle before TMEM is freed
      const int jl = nblk - 1;
      ok = wait_pv(jl, SPECQ_STATUS_TIMEOUT_MMA) && ok;
      tc_fence_after();
      if (t == 0) SPECQ_TRACE_POINT(60, 0);
      if (quad == 0) {
#pragma unroll
        for (int c0 = 0; c0 < NQH; c0 += 8) {
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
  } else if (warp < kAttnMmaWarp) {
    // =================================== K / V gather ===================================
    // K (warp 8) and V (warp 9) arrive by TMA in boxes of box_rows slots of one page and one
    // KV head, both 128B-swizzled (K in the layout the tensor core reads, V so the V warps' row
    // reads are free of bank conflicts); lane b issues box b of a block, the two warps in
    // parallel.  Invalid pages map past the tensor, which the TMA fills with zeros.  Bytes in
    // flight cost no registers here: the ring depth alone sets how much of the HBM latency is
    // covered.
    const bool is_v = warp == 9;
    const CUtensorMap* tmap = is_v ? &tmap_v : &tmap_k;
    const uint32_t half_off = is_v ? kAttnKV8 : 0u;
    const int l = static_cast<int>(lane);
    const int br = p.box_rows;
    const int nbox = 128 >> p.box_shift;
    const uint64_t hint = policy_evict_first();
    int s = 0;
    uint32_t phase = 0;
    int issued = 0;
    for (int j = 0; j < nblk; ++j) {
      if (!mbar_wait(&stage_empty[s], phase ^ 1u, status, SPECQ_STATUS_TIMEOUT_PIPELINE)) {
        ok = false;
        break;
      }
      if (!is_v) SPECQ_TRACE_POINT(50, j);
      uint8_t* dst = ring + s * kAttnStage + half_off;
      if (l == 0) mbar_arrive_expect_tx(&stage_full[s], kAttnKV8);
      __syncwarp();
      for (int bx = l; bx < nbox; bx += 32) {   // box bx starts at token row bx * br
        const int row = bx * br;
        const int pg = token_page(j, row);
        tma_load_4d(dst + row * 128, tmap, &stage_full[s], 0, kvh, slot_of(t_begin + j * 128 + row),
                    page_ok(pg) ? pg : p.n_pages, hint);
      }
      ++issued;
      if (!is_v) SPECQ_TRACE_POINT(51, j);
      if (++s == kAttnStages) {
        s = 0;
        phase ^= 1u;
      }
    }
    // the TMA copies of an abandoned loop land before the CTA exits: wait (bounded) for the
    // stages this warp armed
    if (!ok) {
      for (int jj = max(0, issued - kAttnStages); jj < issued; ++jj)
        (void)mbar_wait(&stage_full[jj % kAttnStages], static_cast<uint32_t>(jj / kAttnStages) & 1u, status,
                        SPECQ_STATUS_TIMEOUT_PIPELINE);
    }
  } else if (warp == kAttnMmaWarp) {
    // =================================== MMA issuer ===================================
    if (elect_one()) {
      const uint32_t id_qk = idesc_i8(128, static_cast<uint32_t>(2 * NQ));       // hi and lo columns
      // V^T (A) and P (B) both MN-major
      const uint32_t id_pv = idesc_f16(128, static_cast<uint32_t>(NQ), 1u, 1u);
      const uint32_t id_l = idesc_f16(128, static_cast<uint32_t>(NQ), 0u, 1u);
      const uint32_t ring_a = smem_u32(ring), vop_a = smem_u32(vop), qop_a = smem_u32(qop), pop_a = smem_u32(pop);
      // B of the bias MMA: K-major, no swizzle, both K core matrices (128 B apart) in bias_s and
      // every 8-row group at the same address (stride 0): 256 bytes serve any N
      const uint64_t bias_desc = sdesc_plain(smem_u32(bias_s), 128u, 0u);
      const uint32_t id_bias = idesc_f16(128, static_cast<uint32_t>(2 * NQ));
      // Operand descriptors: one precomputed descriptor per tile, advanced by adding address
      // offsets in 16-byte units (this thread shares a scheduler with busy softmax and V warps,
      // so its per-block instruction count is kept small).
      const uint64_t kdesc0 = sdesc_sw128(ring_a, 16u, 1024u);
      const uint64_t qdesc0 = sdesc_sw128(qop_a, 16u, 1024u);
      const uint64_t vdesc0 = sdesc_sw128(vop_a, 16384u, 1024u);
      const uint64_t pdesc0 = sdesc_sw128(pop_a, 16384u, 1024u);
      // score buffer sb <- the bias in all 2*NQ hi / lo columns (one MMA, accumulate off); the
      // QK MMAs issued after it by this thread accumulate onto it
      auto reset_scores = [&](uint32_t sb) {
        umma_f16_ts(tmem + sb * cs2, tmem + ONES_col + 8u, bias_desc, id_bias, 0u);
      };
      int qk_stage = 0;
      uint32_t qk_phase = 0;
      auto next_stage = [&]() {
        if (++qk_stage == kAttnStages) {
          qk_stage = 0;
          qk_phase ^= 1u;
        }
      };
      // QK(0) and QK(1) alone; then, per block i, once the softmax has finished block i (P(i)
      // written and score buffer i read for the last time, both signalled by p_full(i)) and V(i)
      // is converted: PV(i) interleaved with QK(i+2).  Three independent accumulation chains
      // (O, the normaliser, the next scores) are then in flight in the tensor pipe instead of
      // one at a time.  The blocking waits keep this thread off the issue slots the softmax
      // warps need.
      if (nblk > 0) ok = mbar_wait(q_full, 0u, status, SPECQ_STATUS_TIMEOUT_PIPELINE);
      for (int j = 0; ok && j < min(2, nblk); ++j) {
        ok = mbar_wait(&stage_full[qk_stage], qk_phase, status, SPECQ_STATUS_TIMEOUT_PIPELINE);
        if (!ok) break;
        tc_fence_after();
        SPECQ_TRACE_POINT(30, j);
        const uint32_t sb = static_cast<uint32_t>(j);
        const uint64_t kd = kdesc0 + ((static_cast<uint32_t>(qk_stage) * kAttnStage) >> 4);
        reset_scores(sb);
#pragma unroll
        for (int k = 0; k < 4; ++k)   // 32 of the 128 head dims (32 bytes) per step
          umma_i8_ss(tmem + sb * cs2, kd + 2u * k, qdesc0 + 2u * k, id_qk, 1u);
        umma_commit(&s_full[sb]);
        umma_commit(&stage_empty[qk_stage]);   // the K tile is consumed
        next_stage();
      }
      for (int i = 0; ok && i < nblk; ++i) {
        const uint32_t bi = static_cast<uint32_t>(i & 1);   // P / V buffer of block i = score buffer of i + 2
        const uint32_t par = static_cast<uint32_t>(i >> 1) & 1u;
        const bool more = i + 2 < nblk;
        ok = mbar_wait(&p_full[bi], par, status, SPECQ_STATUS_TIMEOUT_MMA) &&
             mbar_wait(&v_full[bi], par, status, SPECQ_STATUS_TIMEOUT_PIPELINE) &&
             (!more || mbar_wait(&stage_full[qk_stage], qk_phase, status, SPECQ_STATUS_TIMEOUT_PIPELINE));
        if (!ok) break;
        tc_fence_after();
        SPECQ_TRACE_POINT(32, i);
        const uint64_t vd = vdesc0 + ((bi * kAttnOp) >> 4);
        const uint64_t pd = pdesc0 + ((bi * kAttnPTile) >> 4);
        const uint64_t kd = kdesc0 + ((static_cast<uint32_t>(qk_stage) * kAttnStage) >> 4);
        if (more) reset_scores(bi);
#pragma unroll
        for (int k = 0; k < 8; ++k) {   // 16 tokens (two 1024-byte atoms) per PV step
          const uint64_t bp = pd + 128u * k;
          const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
          umma_f16_ss(tmem + O_col, vd + 128u * k, bp, id_pv, acc);
          if (more && k < 4) umma_i8_ss(tmem + bi * cs2, kd + 2u * k, qdesc0 + 2u * k, id_qk, 1u);
          umma_f16_ts(tmem + L_col, tmem + ONES_col, bp, id_l, acc);
        }
        if (more) {
          umma_commit(&s_full[bi]);   // QK(i+2) and, before it, PV(i)
          umma_commit(&stage_empty[qk_stage]);
          next_stage();
        } else {
          umma_commit(&pv_done[bi]);
        }
        SPECQ_TRACE_POINT(33, i);
      }
    }
  } else {
    // =================================== V warps ===================================
    // Thread c owns token row c of every block: it reads the row's 128 V bytes from the ring
    // (128B-swizzled, so eight consecutive rows hit eight distinct bank groups), converts them
    // to fp16 with the token's V scale folded in and stores the row into the V operand tile.
    const int c = static_cast<int>(threadIdx.x) - 32 * (kAttnMmaWarp + 1);   // 0..127
    float* vsd = vs_ring + c;     // this thread's V-scale slots (stride 128)
    uint32_t vsel = 0u;
    const ScaleRow vrow_s = scale_row(c);
    fetch_scale(p.vs, 0, vrow_s, scale_page(0, vrow_s), vsd, vsel, 0);
    fetch_scale(p.vs, 1, vrow_s, scale_page(1, vrow_s), vsd + 128, vsel, 1);
    int slot = 0;                 // j % 3
#pragma unroll 1
    for (int j = 0; j < nblk; ++j) {
      const int slot2 = slot == 0 ? 2 : slot - 1;   // (j + 2) % 3
      const int pg2 = scale_page(j + 2, vrow_s);      // fetched after this block's conversion
      const int s = j % kAttnStages;
      const uint32_t sb = static_cast<uint32_t>(j & 1);
      ok = ok && mbar_wait(&stage_full[s], static_cast<uint32_t>(j / kAttnStages) & 1u, status,
                           SPECQ_STATUS_TIMEOUT_PIPELINE);
      if (c == 0) SPECQ_TRACE_POINT(40, j);
      const uint8_t* vrow = ring + s * kAttnStage + kAttnKV8 + c * 128;
      uint4 raw[8];
#pragma unroll
      for (int ch = 0; ch < 8; ++ch)
        raw[ch] = *reinterpret_cast<const uint4*>(vrow + ((static_cast<uint32_t>(ch) ^ (static_cast<uint32_t>(c) & 7u)) << 4));
      cp_async_wait<1>();   // block j's scale (fetched two blocks ago) has landed
      // the token's V scale in fp16 (exact for fp16 scales; one rounding for fp32 scales), so
      // the per-element multiply stays on the fp16 pipe
      const __half2 s2 = __half2half2(__float2half_rn(read_scale(vsd + 128 * slot, vsel, slot)));
      // V buffer sb is free once PV(j-2) has completed
      if (j >= 2) ok = ok && wait_pv(j - 2, SPECQ_STATUS_TIMEOUT_MMA);
      uint8_t* vdst = vop + sb * kAttnOp;
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        uint32_t h[8];
        i8x16_to_f16(raw[ch], h);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          __half2 o = __hmul2(*reinterpret_cast<__half2*>(&h[i]), s2);
          h[i] = *reinterpret_cast<uint32_t*>(&o);
        }
        store_f16_chunk_pair(vdst, c, ch, h);
      }
      fence_proxy_async_smem();
      // Blocks 0 and 1: see QK(j) complete before releasing V(j).  QK(j + 2) cannot complete
      // before V(j) is released, so the parity waits in wait_pv(j) two blocks later find
      // s_full[j & 1] one phase ahead at most (costs nothing: PV(j) follows QK(j) anyway).
      if (j < 2) ok = ok && mbar_wait(&s_full[j], 0u, status, SPECQ_STATUS_TIMEOUT_MMA);
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&v_full[sb]);
        mbar_arrive(&stage_empty[s]);   // the V half of the stage is consumed
      }
      if (c == 0) SPECQ_TRACE_POINT(45, j);
      fetch_scale(p.vs, j + 2, vrow_s, pg2, vsd + 128 * slot2, vsel, slot2);
      slot = slot == 2 ? 0 : slot + 1;
    }
    cp_async_wait<0>();
  }
  __syncwarp();

  // The next kernel on the stream may begin launching once every CTA is here (its CTAs wait in
  // griddepcontrol.wait until this grid has completed): launching it at the start instead
  // measured slower, its early CTAs holding SMs this kernel's clusters could use.
  pdl_launch_dependents();
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
            const int qi = q_lo + (p.g_shift >= 0 ? (q >> p.g_shift) : (q / p.g));
            const int head = kvh * p.g + (p.g_shift >= 0 ? (q & (p.g - 1)) : (q % p.g));
            const float l = l_s[q];
            const float o = __uint_as_float(r[i]) / (l == 0.f ? 1.f : l);
            p.out[b * o_sb + static_cast<int64_t>(qi) * p.o_st + static_cast<int64_t>(head) * p.o_sh + tl] =
                __float2half_rn(o);
          }
        }
      }
    }
  } else {
    // Split combine, push model.  CTA r of the cluster owns head dims [r*dr, (r+1)*dr); every
    // CTA stores its partial O^T for those dims, and its (m, l), straight into CTA r's shared
    // memory (fire-and-forget st.shared::cluster), then each CTA combines its own dims
    // locally.  The first cluster barrier makes sure every ring is idle before it is written.
    const int S = p.splits;
    const int lgdr = 7 - (31 - __clz(S));   // head dims per rank: 128 / S
    const int dr = 1 << lgdr;
    float* comb = reinterpret_cast<float*>(ring);   // [S][NQ][dr] partial O of every split
    float* mlb = comb + NQ * 128;                   // [S][NQ] (m, l) of every split
    float* wts = mlb + S * NQ * 2;                  // [S][NQ] combine weights
    if (threadIdx.x == 0) SPECQ_TRACE_POINT(61, 0);
    cluster_sync();
    if (threadIdx.x == 0) SPECQ_TRACE_POINT(62, 0);
    if (soft) {
      const uint32_t dst = dsmem_map(smem_u32(comb), static_cast<uint32_t>(tl >> lgdr)) +
                           4u * static_cast<uint32_t>(split * NQ * dr + (tl & (dr - 1)));
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
        for (int i = 0; i < 8; ++i) dsmem_st_f32(dst + 4u * static_cast<uint32_t>((col0 + c0 + i) * dr), __uint_as_float(r[i]));
      }
      if (t < NQ) {
        const float mv = nblk > 0 ? m_s[t] : -INFINITY;
        const float lv = nblk > 0 ? l_s[t] : 0.f;
        const uint32_t ml = smem_u32(mlb + 2 * (split * NQ + t));
        for (int pr = 0; pr < S; ++pr) dsmem_st_v2f32(dsmem_map(ml, static_cast<uint32_t>(pr)), mv, lv);
      }
    }
    if (threadIdx.x == 0) SPECQ_TRACE_POINT(63, 0);
    cluster_sync();   // every partial has landed; nothing remote is touched after this
    if (threadIdx.x == 0) SPECQ_TRACE_POINT(63, 1);
    // The combine with the split count as a compile-time constant: every loop over the splits
    // unrolls, so each thread's loads are all in flight at once.
    auto combine = [&](auto s_const) {
      constexpr int kS = decltype(s_const)::value;
      if (t < rows_valid) {   // weights of the kS partials of query row t, in fixed split order
        float mp[kS], w[kS];
        float mmax = -INFINITY;
#pragma unroll
        for (int pr = 0; pr < kS; ++pr) {
          mp[pr] = mlb[2 * (pr * NQ + t)];
          mmax = fmaxf(mmax, mp[pr]);
        }
        float lsum = 0.f;
#pragma unroll
        for (int pr = 0; pr < kS; ++pr) {
          w[pr] = (mp[pr] == -INFINITY) ? 0.f : fast_exp2(mp[pr] - mmax);
          lsum = fmaf(w[pr], mlb[2 * (pr * NQ + t) + 1], lsum);
        }
        const float inv = lsum == 0.f ? 1.f : __frcp_rn(lsum);
#pragma unroll
        for (int pr = 0; pr < kS; ++pr) wts[pr * NQ + t] = w[pr] * inv;
      }
      named_barrier_sync(3, 256);
      if (t == 0) SPECQ_TRACE_POINT(63, 2);
      if (!ok) return;
      // one item = 8 consecutive head dims of one query row
      constexpr int kG8 = 128 / kS / 8;
      for (int item = t; item < rows_valid * kG8; item += 256) {
        const int q = item / kG8;
        const int d8 = item % kG8;
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
        for (int pr = 0; pr < kS; ++pr) {
          const float wq = wts[pr * NQ + q];
          const float4* src = reinterpret_cast<const float4*>(comb + (pr * NQ + q) * (128 / kS) + 8 * d8);
          const float4 u = src[0], v = src[1];
          acc[0] = fmaf(wq, u.x, acc[0]); acc[1] = fmaf(wq, u.y, acc[1]);
          acc[2] = fmaf(wq, u.z, acc[2]); acc[3] = fmaf(wq, u.w, acc[3]);
          acc[4] = fmaf(wq, v.x, acc[4]); acc[5] = fmaf(wq, v.y, acc[5]);
          acc[6] = fmaf(wq, v.z, acc[6]); acc[7] = fmaf(wq, v.w, acc[7]);
        }
        const int qi = q_lo + (p.g_shift >= 0 ? (q >> p.g_shift) : (q / p.g));
        const int head = kvh * p.g + (p.g_shift >= 0 ? (q & (p.g - 1)) : (q % p.g));
        __half* dst = p.out + b * o_sb + static_cast<int64_t>(qi) * p.o_st + static_cast<int64_t>(head) * p.o_sh +
                      split * (128 / kS) + 8 * d8;
        __half2 h[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(acc[2 * i], acc[2 * i + 1]);
        if (p.out_vec) {
          *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(h);
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            dst[2 * i] = __low2half(h[i]);
            dst[2 * i + 1] = __high2half(h[i]);
          }
        }
      }
    };
    if (soft) {
      if (S == 2) combine(std::integral_constant<int, 2>{});
      else if (S == 4) combine(std::integral_constant<int, 4>{});
      else combine(std::integral_constant<int, 8>{});
      if (t == 0) SPECQ_TRACE_POINT(63, 3);
    }
  }
  if (threadIdx.x == 256) SPECQ_TRACE_POINT(63, 4);

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) SPECQ_TRACE_POINT(9, 0);
  SPECQ_TRACE_CTA_END();
  if (warp == kAttnMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, p.tmem_cols);
  }
}

inline const void* paged_attn_kernel_by_variant(int variant) {
  switch (variant) {   // query rows per CTA = 16 * (variant + 1)
    case 0: return reinterpret_cast<const void*>(paged_attn_kernel<16>);
    case 1: return reinterpret_cast<const void*>(paged_attn_kernel<32>);
    case 2: return reinterpret_cast<const void*>(paged_attn_kernel<48>);
    case 3: return reinterpret_cast<const void*>(paged_attn_kernel<64>);
    default: return nullptr;
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
  p.kc = kc; p.vc = vc;
  int br = 1;
  while (br < 16 && page % (br * 2) == 0) br *= 2;
  // 128B-swizzled TMA boxes land on 1024-byte boundaries only for boxes of >= 8 slots
  if (br < 8) return fail(SPECQ_ERR_UNSUPPORTED, "paged_attention: page size %d is not a multiple of 8", page);
  p.box_rows = br;
  p.box_shift = __builtin_ctz(static_cast<unsigned>(br));
  p.out_vec = aligned(out, 16) && o_sb % 8 == 0 && o_st % 8 == 0 && o_sh % 8 == 0;   // o_sb 0: packed rows
  p.kv_sp = kv_sp; p.kv_so = kv_so; p.kv_sh = kv_sh;
  p.qpp = std::min(qpp, 64 / G);                 // QPP only changes the schedule
  p.nq = round_up(p.qpp * G, 16);
  p.n_qc = ceil_div(ql_grid, p.qpp);
  p.page_shift = ((page & (page - 1)) == 0) ? __builtin_ctz(static_cast<unsigned>(page)) : -1;
  p.g_shift = ((G & (G - 1)) == 0) ? __builtin_ctz(static_cast<unsigned>(G)) : -1;
  // Split count from the block-table width only (never from B or the plan), so eager and
  // plan-mode launches reduce identical partials.
  const int max_ctx = bt_cols * page;
  // A power of two (each split owns 128 / splits head dims in the combine): at least one split
  // per 2048 tokens, and more when a shard holds few KV heads (tensor-parallel shards keep the
  // SMs busy), but clusters of 8 only with one KV head: 16 such clusters do not fit the GPU in
  // one wave.  Splits of fewer than 512 tokens are not made.
  const int by_heads = H_KV >= 8 ? 2 : (H_KV >= 2 ? 4 : 8);
  p.splits = std::min(8, next_pow2(std::max({1, ceil_div(max_ctx, 2048), std::min(by_heads, ceil_div(max_ctx, 512))})));
  p.stages = kAttnStages;
  p.sm_scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(D));
  // TMEM: two score buffers (hi and lo int32 columns), O^T, normaliser, 16 columns of constant
  // A operands (fp16 ones for the normaliser, fp16 1024.0 for the bias MMA)
  p.col_stride = static_cast<uint32_t>(round_up(2 * p.nq, 32));
  p.o_cols = static_cast<uint32_t>(round_up(p.nq, 32));
  p.tmem_cols = static_cast<uint32_t>(next_pow2(static_cast<int>(2 * p.col_stride + 2 * p.o_cols + 16)));
  if (p.tmem_cols > 512) return fail(SPECQ_ERR_UNSUPPORTED, "paged_attention: too many query rows per CTA");
  if (static_cast<int64_t>(b_grid) * p.n_qc > 65535)
    return fail(SPECQ_ERR_UNSUPPORTED, "paged_attention: grid too large");
  {   // one CTA's block-table slice must fit its shared-memory copy
    const int tchunk_max = round_up(ceil_div(max_ctx, p.splits), 128);
    if (tchunk_max / page + 2 > kAttnMaxPages)
      return fail(SPECQ_ERR_UNSUPPORTED, "paged_attention: block table of %d pages per context split", tchunk_max / page);
  }

  // K ring + two fp16 V tiles + int8 Q (hi, lo) + two P tiles + softmax state + barriers
  const int smem = 1024 + p.stages * static_cast<int>(kAttnStage) + 2 * static_cast<int>(kAttnOp) +
                   p.nq * 256 + 2 * static_cast<int>(kAttnPTile) + 4096 + (3 * 256 + 3 * 128 + attn_bias_words(p.nq)) * 4 +
                   kAttnMaxPages * 4 +
                   (2 * p.stages + 17) * 8 + 16;
  if (smem > 232448) return fail(SPECQ_ERR_UNSUPPORTED, "paged_attention: shared memory %d too large", smem);
  if ((p.nq * 128 + 3 * p.splits * p.nq) * 4 > p.stages * static_cast<int>(kAttnStage))
    return fail(SPECQ_ERR_UNSUPPORTED, "paged_attention: combine buffer does not fit");

  CUtensorMap tk, tv;
  {
    const uint64_t dims[4] = {128u, static_cast<uint64_t>(H_KV), static_cast<uint64_t>(page), static_cast<uint64_t>(n_pages)};
    const uint64_t strides[3] = {static_cast<uint64_t>(kv_sh), static_cast<uint64_t>(kv_so), static_cast<uint64_t>(kv_sp)};
    const uint32_t box[4] = {128u, 1u, static_cast<uint32_t>(br), 1u};
    if (int rc = encode_tiled(&tk, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, kc, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
    if (int rc = encode_tiled(&tv, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, vc, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  }
  const int variant = p.nq / 16 - 1;
  const void* fn = paged_attn_kernel_by_variant(variant);
  const dim3 grid(static_cast<unsigned>(p.splits), static_cast<unsigned>(H_KV),
                  static_cast<unsigned>(b_grid * p.n_qc));
  SPECQ_CUDA_TRY(ensure_dyn_smem(fn, smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kAttnThreads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = static_cast<cudaStream_t>(stream);
  LaunchAttrs attrs(p.splits);
  attrs.apply(cfg);
  void* args[] = {&p, &tk, &tv};
  SPECQ_CUDA_TRY(cudaLaunchKernelExC(&cfg, fn, args));
  LaunchRecord& r = last_launch_ref();
  r.variant = variant;
  r.grid[0] = static_cast<int>(grid.x); r.grid[1] = static_cast<int>(grid.y); r.grid[2] = static_cast<int>(grid.z);
  r.cluster_x = p.splits;
  r.threads = kAttnThreads;
  r.dyn_smem = smem;
  return SPECQ_OK;
}



}  // namespace specq
