// gemm_common.cuh -- the register-staged global->shared tile loader of the GEMMs: it writes
// the 128-byte-swizzled K-major layout the tensor core reads, for operands whose row stride or
// base address is not 16-byte aligned (so TMA cannot be used).  The split-K reductions live in
// the kernels themselves (w8a8.cuh: bulk asynchronous DSMEM adds; w4a16.cuh: fixed-order DSMEM
// loads).
#pragma once

#include "sm100.cuh"

namespace specq {

// Copy `nbytes` (<= 16, a multiple of VEC) starting at `src` into a 16-byte register chunk.
// Bytes at or beyond `valid` are zero.  VEC is the widest aligned access the caller proved.
template <int VEC>
__device__ __forceinline__ uint4 load_chunk16(const uint8_t* src, int valid) {
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  if (valid <= 0) return v;
  if constexpr (VEC == 16) {
    if (valid >= 16) return __ldg(reinterpret_cast<const uint4*>(src));
  }
  uint8_t tmp[16];
#pragma unroll
  for (int i = 0; i < 16; i += (VEC < 16 ? VEC : 8)) {
    constexpr int W = (VEC < 16 ? VEC : 8);
    if (i + W <= valid) {
      if constexpr (W == 8) {
        *reinterpret_cast<uint2*>(tmp + i) = __ldg(reinterpret_cast<const uint2*>(src + i));
      } else if constexpr (W == 4) {
        *reinterpret_cast<uint32_t*>(tmp + i) = __ldg(reinterpret_cast<const uint32_t*>(src + i));
      } else if constexpr (W == 2) {
        *reinterpret_cast<uint16_t*>(tmp + i) = __ldg(reinterpret_cast<const uint16_t*>(src + i));
      } else {
        tmp[i] = __ldg(src + i);
      }
    } else {
#pragma unroll
      for (int j = 0; j < W; ++j) tmp[i + j] = 0;
    }
  }
  v = *reinterpret_cast<uint4*>(tmp);
  return v;
}

// Load a [rows x 128 B] K-major tile (row r of the tile = global row row0 + r, bytes
// [kbyte0, kbyte0 + 128) of it) into a 128B-swizzled shared tile.  Rows >= row_limit and bytes
// >= kbytes read as zero.  `nthreads` threads cooperate; thread `t` of them calls this.
template <int VEC>
__device__ __forceinline__ void ldg_tile_sw128(uint8_t* smem_tile, const uint8_t* base, int64_t ld_bytes,
                                               int row0, int rows, int row_limit, int kbyte0, int kbytes,
                                               int t, int nthreads) {
  const int nchunks = rows * 8;
  for (int c = t; c < nchunks; c += nthreads) {
    const int r = c >> 3;
    const int ch = c & 7;
    const int grow = row0 + r;
    const int kb = kbyte0 + ch * 16;
    int valid = (grow < row_limit) ? (kbytes - kb) : 0;
    uint4 v = load_chunk16<VEC>(base + static_cast<int64_t>(grow) * ld_bytes + kb, valid);
    *reinterpret_cast<uint4*>(smem_tile + sw128_offset(static_cast<uint32_t>(r), static_cast<uint32_t>(ch))) = v;
  }
}

}  // namespace specq
