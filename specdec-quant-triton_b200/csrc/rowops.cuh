// rowops.cuh -- the per-token INT8 quantiser and the paged-KV append of a verification layer.
//
// quant_rows: dynamic per-token symmetric INT8 of an fp16 row, with the reference's formula
// (kernels.py:58-62):  s = max(amax|y|, 1e-8) / 127,  q = clamp(rint(y / s), -127, 127),
// evaluated the way torch evaluates it on a CUDA tensor -- the division by the Python scalar
// 127 is a multiplication by the fp32 reciprocal 1/127, the division by the scale tensor an
// IEEE division, round half to even -- so the int8 rows and the fp32 scales equal the
// reference's bit for bit.  y is one of
//   mode 0: y = x
//   mode 1: y = x + r, and the fp16 sum is written back to r (the residual stream)
//   mode 2: y = silu(g) * u with g = x[:, :N], u = x[:, N:2N]  (the MLP's gate / up halves)
// One CTA per row; rows >= the plan's M are skipped (plan-buffer graphs).
//
// kv_append: the K and V of the q_len newest tokens of each sequence (columns [k_col,
// k_col + H_KV*D) and [v_col, ..) of a packed [tokens x cols] fp16 projection output, token
// row b*q_len + t) are quantised per (token, KV head) with the formula the reference's cache
// fixture uses (kernels.py:280-283: fp32 scale amax/127 -- evaluated as above --, int8
// values, fp16 stored scale) and
// written to slot (ctx_len[b] - q_len + t) of the sequence's pages.  One warp per
// (token, KV head, K or V).
//
// pack_int4: the reference's group-wise INT4 weight quantiser (kernels.py:138-147) on the
// device: per group of `group` weights s = max(amax|w|, 1e-8) / 7 (fp32, torch's `/ 7.0` on a
// CUDA tensor: a multiplication by fp32(1/7)), q = clamp(rint(w / s), -8, 7), byte j of row n
// = (q[n, j] + 8) | (q[n, j + K/2] + 8) << 4, fp16 scales, and optionally the dequantised
// fp16 copy fp16(q * s).  One warp per (row, low group g, its high partner g + K/(2 group)):
// lane l takes elements l, l + 32, ... of both groups, so every load and store of the warp is
// a run of consecutive addresses.
#pragma once

#include <cuda_bf16.h>

#include <type_traits>

#include "sm100.cuh"
#include "specq_host.cuh"

namespace specq {

constexpr int kRowThreads = 256;
constexpr float kInv127 = 1.0f / 127.0f;   // fp32 reciprocal, as torch forms it for `/ 127.0`
constexpr int kRowMaxPerThread = 64;   // N up to 256 * 64 = 16384 per row

struct QuantRowsParams {
  const __half* x;     // [M, N] (mode 2: [M, 2N])
  __half* r;           // mode 1: residual [M, N], updated in place
  int8_t* q;           // [M, N]
  float* s;            // [M]
  const int32_t* plan; // plan[0] = active M
  const float* amax_in;  // optional: the row's amax over a wider row (tensor-parallel shards)
  float* amax_out;       // optional: write the row amax of y and stop (no quantisation)
  int* status;
  int64_t ldx, ldr, ldq;
  int M, N, mode;
  // optional tensor-parallel input: x is a full buffer that every rank's producer writes over
  // NVLink; wait until every rank's count in this flag array has reached this rank's own
  const uint32_t* wait_flags;
  int wait_rank, wait_world;
};

// silu(g) = g * sigmoid(g) with the fast exponential and division intrinsics: the fused
// SiLU-mul mode has no bit-exact counterpart (the reference has no such kernel); its int8
// output matches torch's silu * mul followed by the quantiser to within one unit.
__device__ __forceinline__ float silu_f32(float g) { return __fdividef(g, 1.f + __expf(-g)); }

template <int PER>
__global__ void __launch_bounds__(kRowThreads) quant_rows_kernel(const __grid_constant__ QuantRowsParams p) {
  pdl_launch_dependents();   // the next kernel on the stream may begin launching
  pdl_wait();                // the previous kernel's writes are visible from here on
  __shared__ float red[kRowThreads / 32];
  const int row = blockIdx.x;
  int M = p.M;
  if (p.plan != nullptr) {
    const int pm = __ldg(p.plan);
    if (pm < 0 || pm > p.M) {
      if (threadIdx.x == 0 && row == 0) report_status(p.status, SPECQ_STATUS_PLAN_CLAMPED);
    }
    M = min(max(pm, 0), p.M);
  }
  if (row >= M) return;
  if (p.wait_flags != nullptr) {
    if (threadIdx.x == 0) (void)wait_peer_counts(p.wait_flags, p.wait_rank, p.wait_world, p.status);
    __syncthreads();
  }
  const __half* x = p.x + static_cast<int64_t>(row) * p.ldx;
  float y[PER];
  float amax = 0.f;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int c = static_cast<int>(threadIdx.x) + k * kRowThreads;
    float v = 0.f;
    if (c < p.N) {
      if (p.mode == 0) {
        v = __half2float(x[c]);
      } else if (p.mode == 1) {
        __half* r = p.r + static_cast<int64_t>(row) * p.ldr;
        const __half h = __hadd(x[c], r[c]);   // the fp16 residual stream
        r[c] = h;
        v = __half2float(h);
      } else {
        v = silu_f32(__half2float(x[c])) * __half2float(x[c + p.N]);
      }
    }
    y[k] = v;
    amax = fmaxf(amax, fabsf(v));
  }
  amax = warp_max_f32(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  float m = 0.f;
#pragma unroll
  for (int w = 0; w < kRowThreads / 32; ++w) m = fmaxf(m, red[w]);
  if (p.amax_out != nullptr) {   // first pass of a sharded row: its amax only
    if (threadIdx.x == 0) p.amax_out[row] = m;
    return;
  }
  if (p.amax_in != nullptr) m = __ldg(p.amax_in + row);   // the whole row's amax
  const float s = __fmul_rn(fmaxf(m, 1e-8f), kInv127);
  int8_t* q = p.q + static_cast<int64_t>(row) * p.ldq;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int c = static_cast<int>(threadIdx.x) + k * kRowThreads;
    if (c < p.N) {
      const float v = fminf(fmaxf(rintf(__fdiv_rn(y[k], s)), -127.f), 127.f);
      q[c] = static_cast<int8_t>(v);
    }
  }
  if (threadIdx.x == 0) p.s[row] = s;
}

// The same with 16-byte accesses: thread t takes the 8-element chunks t, t + 256, ...
// (CH of them) -- rows 16-byte aligned, N a multiple of 8.
template <int CH>
__global__ void __launch_bounds__(kRowThreads) quant_rows_vec_kernel(const __grid_constant__ QuantRowsParams p) {
  pdl_launch_dependents();   // the next kernel on the stream may begin launching
  pdl_wait();                // the previous kernel's writes are visible from here on
  __shared__ float red[kRowThreads / 32];
  const int row = blockIdx.x;
  int M = p.M;
  if (p.plan != nullptr) {
    const int pm = __ldg(p.plan);
    if ((pm < 0 || pm > p.M) && threadIdx.x == 0 && row == 0) report_status(p.status, SPECQ_STATUS_PLAN_CLAMPED);
    M = min(max(pm, 0), p.M);
  }
  if (row >= M) return;
  if (p.wait_flags != nullptr) {
    if (threadIdx.x == 0) (void)wait_peer_counts(p.wait_flags, p.wait_rank, p.wait_world, p.status);
    __syncthreads();
  }
  const __half* x = p.x + static_cast<int64_t>(row) * p.ldx;
  float y[CH][8];
  float amax = 0.f;
#pragma unroll
  for (int k = 0; k < CH; ++k) {
    const int c = (static_cast<int>(threadIdx.x) + k * kRowThreads) * 8;
    if (c < p.N) {
      const uint4 a = *reinterpret_cast<const uint4*>(x + c);
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
      if (p.mode == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&aw[i]));
          y[k][2 * i] = f.x;
          y[k][2 * i + 1] = f.y;
        }
      } else if (p.mode == 1) {
        __half* r = p.r + static_cast<int64_t>(row) * p.ldr + c;
        const uint4 b = *reinterpret_cast<const uint4*>(r);
        const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
        uint32_t hw[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const __half2 h = __hadd2(*reinterpret_cast<const __half2*>(&aw[i]), *reinterpret_cast<const __half2*>(&bw[i]));
          hw[i] = *reinterpret_cast<const uint32_t*>(&h);
          const float2 f = __half22float2(h);
          y[k][2 * i] = f.x;
          y[k][2 * i + 1] = f.y;
        }
        *reinterpret_cast<uint4*>(r) = make_uint4(hw[0], hw[1], hw[2], hw[3]);   // the residual stream
      } else {
        const uint4 b = *reinterpret_cast<const uint4*>(x + c + p.N);
        const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 g = __half22float2(*reinterpret_cast<const __half2*>(&aw[i]));
          const float2 u = __half22float2(*reinterpret_cast<const __half2*>(&bw[i]));
          y[k][2 * i] = silu_f32(g.x) * u.x;
          y[k][2 * i + 1] = silu_f32(g.y) * u.y;
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(y[k][i]));
    }
  }
  amax = warp_max_f32(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  float m = 0.f;
#pragma unroll
  for (int w = 0; w < kRowThreads / 32; ++w) m = fmaxf(m, red[w]);
  if (p.amax_out != nullptr) {   // first pass of a sharded row: its amax only
    if (threadIdx.x == 0) p.amax_out[row] = m;
    return;
  }
  if (p.amax_in != nullptr) m = __ldg(p.amax_in + row);   // the whole row's amax
  const float s = __fmul_rn(fmaxf(m, 1e-8f), kInv127);
  int8_t* q = p.q + static_cast<int64_t>(row) * p.ldq;
#pragma unroll
  for (int k = 0; k < CH; ++k) {
    const int c = (static_cast<int>(threadIdx.x) + k * kRowThreads) * 8;
    if (c < p.N) {
      uint32_t w[2] = {0u, 0u};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int v = static_cast<int>(fminf(fmaxf(rintf(__fdiv_rn(y[k][i], s)), -127.f), 127.f));
        w[i >> 2] |= (static_cast<uint32_t>(v) & 0xFFu) << (8 * (i & 3));
      }
      *reinterpret_cast<uint2*>(q + c) = make_uint2(w[0], w[1]);
    }
  }
  if (threadIdx.x == 0) p.s[row] = s;
}

constexpr float kInv7 = 1.0f / 7.0f;   // fp32 reciprocal, as torch forms it for `/ 7.0`

struct PackInt4Params {
  const void* w;       // [N, K] fp16 / fp32 / bf16 (w_dtype 0 / 1 / 2), row stride ldw elements
  uint8_t* wp;         // [N, K/2], row stride ldwp bytes
  __half* sc;          // [N, K/group], row stride ldsc elements
  __half* deq;         // optional [N, K], row stride lddeq elements
  int64_t ldw, ldwp, ldsc, lddeq;
  int N, K, group, w_dtype;
};

template <typename T>
__device__ __forceinline__ float weight_to_f32(T v);
template <>
__device__ __forceinline__ float weight_to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float weight_to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float weight_to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// E consecutive elements from src into v: one vector load when VEC (E * sizeof(T) bytes,
// aligned by the host's check), else E scalar loads.
template <typename T, int E, bool VEC>
__device__ __forceinline__ void load_run(const T* src, float (&v)[E]) {
  if constexpr (VEC && E * sizeof(T) == 16) {
    const uint4 u = *reinterpret_cast<const uint4*>(src);
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < E; ++i) v[i] = weight_to_f32<T>(e[i]);
  } else if constexpr (VEC && E * sizeof(T) == 8) {
    const uint2 u = *reinterpret_cast<const uint2*>(src);
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < E; ++i) v[i] = weight_to_f32<T>(e[i]);
  } else if constexpr (VEC && E * sizeof(T) == 4) {
    const uint32_t u = *reinterpret_cast<const uint32_t*>(src);
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < E; ++i) v[i] = weight_to_f32<T>(e[i]);
  } else {
#pragma unroll
    for (int i = 0; i < E; ++i) v[i] = weight_to_f32<T>(src[i]);
  }
}

// Lane l takes the E consecutive elements l*E .. l*E + E-1 of the low group and of the high
// group, so each warp-wide load / store is one contiguous run.  A warp takes kPackUnits
// consecutive (row, group pair) units and issues all their loads before any arithmetic:
// enough bytes in flight per SM to cover the HBM latency.
constexpr int kPackUnits = 4;

template <typename T, int E, bool VEC>   // E = group / 32
__global__ void __launch_bounds__(256) pack_int4_kernel(const __grid_constant__ PackInt4Params p) {
  pdl_launch_dependents();   // the next kernel on the stream may begin launching
  pdl_wait();                // the previous kernel's writes are visible from here on
  const int pairs = p.K / (2 * p.group);
  const int64_t total = static_cast<int64_t>(p.N) * pairs;
  const int64_t unit0 = (static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5)) * kPackUnits;
  if (unit0 >= total) return;
  const int lane = static_cast<int>(threadIdx.x & 31);
  const int half = p.K / 2;
  float lo[kPackUnits][E], hi[kPackUnits][E];
#pragma unroll
  for (int u = 0; u < kPackUnits; ++u) {
    const int64_t unit = unit0 + u;
    if (unit < total) {
      const int n = static_cast<int>(unit / pairs);
      const int g = static_cast<int>(unit % pairs);
      const T* row = static_cast<const T*>(p.w) + static_cast<int64_t>(n) * p.ldw + g * p.group + lane * E;
      load_run<T, E, VEC>(row, lo[u]);
      load_run<T, E, VEC>(row + half, hi[u]);
    }
  }
#pragma unroll
  for (int u = 0; u < kPackUnits; ++u) {
    const int64_t unit = unit0 + u;
    if (unit >= total) break;
    const int n = static_cast<int>(unit / pairs);
    const int g = static_cast<int>(unit % pairs);
    const int k0 = g * p.group + lane * E;
    float alo = 0.f, ahi = 0.f;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      alo = fmaxf(alo, fabsf(lo[u][i]));
      ahi = fmaxf(ahi, fabsf(hi[u][i]));
    }
    alo = warp_max_f32(alo);
    ahi = warp_max_f32(ahi);
    const float slo = __fmul_rn(fmaxf(alo, 1e-8f), kInv7);
    const float shi = __fmul_rn(fmaxf(ahi, 1e-8f), kInv7);
    uint8_t bytes[E];
    __half dlo[E], dhi[E];
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const float ql = fminf(fmaxf(rintf(__fdiv_rn(lo[u][i], slo)), -8.f), 7.f);
      const float qh = fminf(fmaxf(rintf(__fdiv_rn(hi[u][i], shi)), -8.f), 7.f);
      bytes[i] = static_cast<uint8_t>((static_cast<int>(ql) + 8) | ((static_cast<int>(qh) + 8) << 4));
      dlo[i] = __float2half_rn(__fmul_rn(ql, slo));
      dhi[i] = __float2half_rn(__fmul_rn(qh, shi));
    }
    uint8_t* wp = p.wp + static_cast<int64_t>(n) * p.ldwp + k0;
    if constexpr (VEC && E == 4) {
      *reinterpret_cast<uint32_t*>(wp) = *reinterpret_cast<const uint32_t*>(bytes);
    } else if constexpr (VEC && E == 8) {
      *reinterpret_cast<uint2*>(wp) = *reinterpret_cast<const uint2*>(bytes);
    } else {
#pragma unroll
      for (int i = 0; i < E; ++i) wp[i] = bytes[i];
    }
    if (p.deq != nullptr) {
      __half* d = p.deq + static_cast<int64_t>(n) * p.lddeq + k0;
      if constexpr (VEC && E == 4) {
        *reinterpret_cast<uint2*>(d) = *reinterpret_cast<const uint2*>(dlo);
        *reinterpret_cast<uint2*>(d + half) = *reinterpret_cast<const uint2*>(dhi);
      } else if constexpr (VEC && E == 8) {
        *reinterpret_cast<uint4*>(d) = *reinterpret_cast<const uint4*>(dlo);
        *reinterpret_cast<uint4*>(d + half) = *reinterpret_cast<const uint4*>(dhi);
      } else {
#pragma unroll
        for (int i = 0; i < E; ++i) {
          d[i] = dlo[i];
          d[half + i] = dhi[i];
        }
      }
    }
    if (lane == 0) {
      p.sc[static_cast<int64_t>(n) * p.ldsc + g] = __float2half_rn(slo);
      p.sc[static_cast<int64_t>(n) * p.ldsc + g + pairs] = __float2half_rn(shi);
    }
  }
}

struct KvAppendParams {
  const __half* x;       // [M, ld] packed token rows b*q_len + t
  int8_t* kc;
  int8_t* vc;
  __half* ks;
  __half* vs;
  const int32_t* bt;
  const int32_t* ctx_len;
  const int32_t* plan;   // plan[0] = n_seqs, plan[1] = q_len
  int* status;
  int64_t ldx, kv_sp, kv_so, kv_sh, s_sp, s_so, s_sh, bt_sb;
  int k_col, v_col, n_seqs, q_len, b_grid, ql_max, h_kv, page, n_pages, bt_cols;
};

__global__ void __launch_bounds__(128) kv_append_kernel(const __grid_constant__ KvAppendParams p) {
  pdl_launch_dependents();   // the next kernel on the stream may begin launching
  pdl_wait();                // the previous kernel's writes are visible from here on
  // blockIdx.x = token slot (b * ql_max + t), warp = (KV head, K|V) pair index
  const int warp = static_cast<int>(threadIdx.x >> 5);
  const int lane = static_cast<int>(threadIdx.x & 31);
  const int item = blockIdx.y * 4 + warp;            // (head, which) pairs, 2 * h_kv of them
  if (item >= 2 * p.h_kv) return;
  int n_seqs = p.n_seqs, q_len = p.q_len;
  if (p.plan != nullptr) {
    n_seqs = min(max(__ldg(p.plan), 0), p.b_grid);
    q_len = min(max(__ldg(p.plan + 1), 0), p.ql_max);
  }
  const int b = blockIdx.x / p.ql_max;
  const int t = blockIdx.x % p.ql_max;
  if (b >= n_seqs || t >= q_len) return;
  const int head = item >> 1;
  const bool is_v = item & 1;
  const int pos = __ldg(p.ctx_len + b) - q_len + t;
  if (pos < 0 || pos >= p.bt_cols * p.page) {
    if (lane == 0) report_status(p.status, SPECQ_STATUS_PLAN_CLAMPED);
    return;
  }
  const int pg = __ldg(p.bt + b * p.bt_sb + pos / p.page);
  if (pg < 0 || pg >= p.n_pages) {
    if (lane == 0) report_status(p.status, SPECQ_STATUS_PLAN_CLAMPED);
    return;
  }
  const int slot = pos % p.page;
  // this lane's 4 of the head's 128 values
  const __half* src = p.x + static_cast<int64_t>(b * q_len + t) * p.ldx + (is_v ? p.v_col : p.k_col) + head * 128 + 4 * lane;
  const uint2 raw = *reinterpret_cast<const uint2*>(src);
  const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
  const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
  const float v[4] = {f01.x, f01.y, f23.x, f23.y};
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  amax = warp_max_f32(amax);
  const float s = __fmul_rn(fmaxf(amax, 1e-8f), kInv127);
  uint32_t packed = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int qv = static_cast<int>(fminf(fmaxf(rintf(__fdiv_rn(v[i], s)), -127.f), 127.f));
    packed |= (static_cast<uint32_t>(qv) & 0xFFu) << (8 * i);
  }
  const int64_t off = static_cast<int64_t>(pg) * p.kv_sp + static_cast<int64_t>(slot) * p.kv_so +
                      static_cast<int64_t>(head) * p.kv_sh;
  *reinterpret_cast<uint32_t*>((is_v ? p.vc : p.kc) + off + 4 * lane) = packed;
  if (lane == 0) {
    const int64_t so = static_cast<int64_t>(pg) * p.s_sp + static_cast<int64_t>(slot) * p.s_so +
                       static_cast<int64_t>(head) * p.s_sh;
    (is_v ? p.vs : p.ks)[so] = __float2half_rn(s);
  }
}

inline int run_quant_rows(const void* x, int64_t ldx, void* r, int64_t ldr, int8_t* q, int64_t ldq, float* s,
                          const int32_t* plan, const float* amax_in, float* amax_out, int M, int N, int mode,
                          void* stream, const uint32_t* wait_flags = nullptr, int wait_rank = 0, int wait_world = 0) {
  if (wait_flags != nullptr && (wait_world < 1 || wait_world > 8 || wait_rank < 0 || wait_rank >= wait_world))
    return fail(SPECQ_ERR_INVALID_ARG, "quant_rows: wait rank %d of world %d", wait_rank, wait_world);
  if (M < 0 || N <= 0) return fail(SPECQ_ERR_INVALID_ARG, "quant_rows: bad shape M=%d N=%d", M, N);
  if (mode < 0 || mode > 2) return fail(SPECQ_ERR_INVALID_ARG, "quant_rows: mode %d", mode);
  if (M == 0) return SPECQ_OK;
  if (amax_out != nullptr && (mode == 1 || amax_in != nullptr))
    return fail(SPECQ_ERR_INVALID_ARG, "quant_rows: amax_out is for modes 0 and 2 without amax_in");
  if (x == nullptr || (amax_out == nullptr && (q == nullptr || s == nullptr)) || (mode == 1 && r == nullptr))
    return fail(SPECQ_ERR_INVALID_ARG, "quant_rows: null pointer");
  if (ldx < (mode == 2 ? 2 * static_cast<int64_t>(N) : N) || (amax_out == nullptr && ldq < N) || (mode == 1 && ldr < N))
    return fail(SPECQ_ERR_INVALID_ARG, "quant_rows: row strides too small");
  if (N > kRowThreads * kRowMaxPerThread)
    return fail(SPECQ_ERR_UNSUPPORTED, "quant_rows: N=%d > %d", N, kRowThreads * kRowMaxPerThread);
  DeviceState* dev = nullptr;
  if (int rc = get_device_state(&dev)) return rc;
  QuantRowsParams p = {};
  p.x = static_cast<const __half*>(x);
  p.r = static_cast<__half*>(r);
  p.q = q;
  p.s = s;
  p.plan = plan;
  p.amax_in = amax_in;
  p.amax_out = amax_out;
  p.status = dev->status;
  p.ldx = ldx; p.ldr = ldr; p.ldq = ldq;
  p.M = M; p.N = N; p.mode = mode;
  p.wait_flags = wait_flags;
  p.wait_rank = wait_rank;
  p.wait_world = wait_world;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool vec = N % 8 == 0 && aligned(x, 16) && ldx % 8 == 0 && aligned(q, 8) && ldq % 8 == 0 &&
                   (mode != 1 || (aligned(r, 16) && ldr % 8 == 0));
  if (vec) {
    const int ch = ceil_div(N, 8 * kRowThreads);
    if (ch <= 1) SPECQ_CUDA_TRY(launch_plain(quant_rows_vec_kernel<1>, dim3(M), dim3(kRowThreads), st, p));
    else if (ch <= 2) SPECQ_CUDA_TRY(launch_plain(quant_rows_vec_kernel<2>, dim3(M), dim3(kRowThreads), st, p));
    else if (ch <= 4) SPECQ_CUDA_TRY(launch_plain(quant_rows_vec_kernel<4>, dim3(M), dim3(kRowThreads), st, p));
    else SPECQ_CUDA_TRY(launch_plain(quant_rows_vec_kernel<8>, dim3(M), dim3(kRowThreads), st, p));
    SPECQ_CUDA_TRY(cudaGetLastError());
    return SPECQ_OK;
  }
  const int per = ceil_div(N, kRowThreads);
  if (per <= 8) SPECQ_CUDA_TRY(launch_plain(quant_rows_kernel<8>, dim3(M), dim3(kRowThreads), st, p));
  else if (per <= 16) SPECQ_CUDA_TRY(launch_plain(quant_rows_kernel<16>, dim3(M), dim3(kRowThreads), st, p));
  else if (per <= 32) SPECQ_CUDA_TRY(launch_plain(quant_rows_kernel<32>, dim3(M), dim3(kRowThreads), st, p));
  else SPECQ_CUDA_TRY(launch_plain(quant_rows_kernel<64>, dim3(M), dim3(kRowThreads), st, p));
  SPECQ_CUDA_TRY(cudaGetLastError());
  return SPECQ_OK;
}

inline int run_kv_append(const void* x, int64_t ldx, int k_col, int v_col, int8_t* kc, int8_t* vc, int64_t kv_sp,
                         int64_t kv_so, int64_t kv_sh, int n_pages, void* ks, void* vs, int64_t s_sp, int64_t s_so,
                         int64_t s_sh, const int32_t* bt, int64_t bt_sb, int bt_cols, const int32_t* ctx_len,
                         const int32_t* plan, int B, int n_seqs, int q_len, int ql_max, int H_KV, int D, int page,
                         void* stream) {
  if (B < 0 || n_seqs < 0 || q_len < 0 || ql_max < 0 || H_KV <= 0 || page <= 0 || n_pages < 0 || bt_cols < 0)
    return fail(SPECQ_ERR_INVALID_ARG, "kv_append: negative size");
  if (D != 128) return fail(SPECQ_ERR_UNSUPPORTED, "kv_append: head_dim %d (this build supports 128)", D);
  if (x == nullptr || kc == nullptr || vc == nullptr || ks == nullptr || vs == nullptr || bt == nullptr ||
      ctx_len == nullptr)
    return fail(SPECQ_ERR_INVALID_ARG, "kv_append: null pointer");
  if (!aligned(x, 8) || ldx % 4 || k_col % 4 || v_col % 4 || !aligned(kc, 4) || !aligned(vc, 4) || kv_sh % 4 ||
      kv_so % 4 || kv_sp % 4)
    return fail(SPECQ_ERR_UNSUPPORTED, "kv_append: rows must be 8-byte (x) / 4-byte (cache) aligned");
  if (plan == nullptr && (n_seqs > B || q_len > ql_max))
    return fail(SPECQ_ERR_INVALID_ARG, "kv_append: n_seqs/q_len exceed the grid");
  const int b_grid = plan ? B : n_seqs;
  const int ql_grid = plan ? ql_max : q_len;
  if (b_grid == 0 || ql_grid == 0) return SPECQ_OK;
  DeviceState* dev = nullptr;
  if (int rc = get_device_state(&dev)) return rc;
  KvAppendParams p = {};
  p.x = static_cast<const __half*>(x);
  p.kc = kc; p.vc = vc;
  p.ks = static_cast<__half*>(ks); p.vs = static_cast<__half*>(vs);
  p.bt = bt; p.ctx_len = ctx_len; p.plan = plan; p.status = dev->status;
  p.ldx = ldx; p.kv_sp = kv_sp; p.kv_so = kv_so; p.kv_sh = kv_sh;
  p.s_sp = s_sp; p.s_so = s_so; p.s_sh = s_sh; p.bt_sb = bt_sb;
  p.k_col = k_col; p.v_col = v_col; p.n_seqs = n_seqs; p.q_len = q_len; p.b_grid = b_grid;
  p.ql_max = ql_grid; p.h_kv = H_KV; p.page = page; p.n_pages = n_pages; p.bt_cols = bt_cols;
  const dim3 grid(static_cast<unsigned>(b_grid * ql_grid), static_cast<unsigned>(ceil_div(2 * H_KV, 4)));
  SPECQ_CUDA_TRY(launch_plain(kv_append_kernel, grid, dim3(128), static_cast<cudaStream_t>(stream), p));
  SPECQ_CUDA_TRY(cudaGetLastError());
  return SPECQ_OK;
}

inline int run_pack_int4(const void* w, int w_dtype, int64_t ldw, int N, int K, int group, uint8_t* wp, int64_t ldwp,
                         void* sc, int64_t ldsc, void* deq, int64_t lddeq, void* stream) {
  if (N < 0 || K < 0 || group <= 0) return fail(SPECQ_ERR_INVALID_ARG, "pack_int4: negative size");
  if (K % 2 || (K / 2) % group)
    return fail(SPECQ_ERR_INVALID_ARG, "pack_int4: K=%d needs K %% 2 == 0 and (K/2) %% group == 0 (group %d)", K, group);
  if (group != 32 && group != 64 && group != 128 && group != 256)
    return fail(SPECQ_ERR_UNSUPPORTED, "pack_int4: group %d (this build supports 32, 64, 128, 256)", group);
  if (w_dtype < 0 || w_dtype > 2) return fail(SPECQ_ERR_INVALID_ARG, "pack_int4: weight dtype code %d", w_dtype);
  if (N == 0 || K == 0) return SPECQ_OK;
  if (w == nullptr || wp == nullptr || sc == nullptr) return fail(SPECQ_ERR_INVALID_ARG, "pack_int4: null pointer");
  if (ldw < K || ldwp < K / 2 || ldsc < K / group || (deq != nullptr && lddeq < K))
    return fail(SPECQ_ERR_INVALID_ARG, "pack_int4: a row stride is shorter than the row");
  PackInt4Params p = {};
  p.w = w; p.wp = wp; p.sc = static_cast<__half*>(sc); p.deq = static_cast<__half*>(deq);
  p.ldw = ldw; p.ldwp = ldwp; p.ldsc = ldsc; p.lddeq = lddeq;
  p.N = N; p.K = K; p.group = group; p.w_dtype = w_dtype;
  const int64_t units = static_cast<int64_t>(N) * (K / (2 * group));
  const int64_t blocks = (units + 8 * kPackUnits - 1) / (8 * kPackUnits);
  if (blocks > 0x7FFFFFFF) return fail(SPECQ_ERR_INVALID_ARG, "pack_int4: too many groups");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned gx = static_cast<unsigned>(blocks);
  const int E = group / 32;
  const int esz = w_dtype == 1 ? 4 : 2;
  // vector accesses: every run of E elements (weights), E bytes (packed) and E fp16 (deq) aligned
  const bool vec = E >= 4 && aligned(w, E * esz) && (ldw * esz) % (E * esz) == 0 && aligned(wp, E) && ldwp % E == 0 &&
                   (deq == nullptr || (aligned(deq, 2 * E) && lddeq % E == 0 && (K / 2) % E == 0));
  auto launch = [&](auto tag, auto e_tag, auto vec_tag) {
    using T = decltype(tag);
    return launch_plain(pack_int4_kernel<T, decltype(e_tag)::value, decltype(vec_tag)::value>, dim3(gx), dim3(256), st, p);
  };
  auto by_e = [&](auto tag) {
    using I1 = std::integral_constant<int, 1>;
    using I2 = std::integral_constant<int, 2>;
    using I4 = std::integral_constant<int, 4>;
    using I8 = std::integral_constant<int, 8>;
    using VT = std::integral_constant<bool, true>;
    using VF = std::integral_constant<bool, false>;
    if (E == 1) launch(tag, I1{}, VF{});
    else if (E == 2) launch(tag, I2{}, VF{});
    else if (E == 4) vec ? launch(tag, I4{}, VT{}) : launch(tag, I4{}, VF{});
    else vec ? launch(tag, I8{}, VT{}) : launch(tag, I8{}, VF{});
  };
  if (w_dtype == 0) by_e(__half{});
  else if (w_dtype == 1) by_e(float{});
  else by_e(__nv_bfloat16{});
  SPECQ_CUDA_TRY(cudaGetLastError());
  return SPECQ_OK;
}

}  // namespace specq
