// peer_gather.cuh -- all-gather of row slices over NVLink by plain peer stores (no reference
// counterpart: the reference runs on one GPU; this is the exchange step of the tensor-parallel
// verification stack).
//
// Every rank holds a [rows, world * slice] "full" buffer in symmetric memory (mapped into every
// rank's address space).  Rank r's kernel writes its [rows, slice] block straight into column
// range [r * slice, (r + 1) * slice) of EVERY rank's full buffer -- its own included -- so the
// gathered rows need no re-layout pass; then it tells each peer, through a flag in the peer's
// memory, that its block has landed, and waits until every peer has told it the same.  When the
// kernel completes, this rank's full buffer holds all blocks and the next kernel on the stream
// can read it.
//
// Protocol (per exchange buffer; every rank launches the same sequence with the same grid):
//   1. the CTAs copy the block with 16-byte (or 4-byte) loads and peer stores;
//   2. once its threads are done (CTA barrier), each CTA adds 1 to flag[rank] of every peer's
//      flag array with a release reduction at system scope (cumulative: it publishes the whole
//      CTA's stores), so the flags count the CTAs that have landed, launch after launch;
//   3. CTA 0 advances this rank's running total by the grid size and polls its own flag array
//      (acquire, system scope) until every peer's count has reached that total -- a bounded
//      wait (1 s) that records SPECQ_STATUS_TIMEOUT_PEER and returns instead of hanging; the
//      kernel is complete once CTA 0 returns;
//   4. in max mode (the per-token amax of row-split activations) CTA 0 then reduces the
//      gathered [rows, world] floats to their per-row maximum (the grid is one CTA then).
// A rank cannot overwrite a peer's full buffer while the peer still reads the previous contents:
// the stack cycles through four exchange buffers per layer, and a rank reaches the next use of a
// buffer only after later exchanges whose epochs show every peer has moved past its reads.
#pragma once

#include "sm100.cuh"
#include "specq_host.cuh"

namespace specq {

constexpr int kPeerThreads = 256;
constexpr int kPeerMaxWorld = 8;

struct PeerGatherParams {
  const uint8_t* src;   // this rank's block: rows of row_bytes, row stride ld_src bytes
  int64_t ld_src;
  int row_bytes;        // multiple of 4
  int vec16;            // 1: 16-byte units (row_bytes, strides, bases and offset 16-byte aligned)
  const int32_t* plan;  // optional: plan[0] = active rows
  int rows;             // maximum rows (the launch's extent)
  uint8_t* dst[kPeerMaxWorld];     // every rank's full buffer (this rank's own included)
  int64_t ld_dst;                  // row stride of the full buffers, bytes
  int64_t dst_off;                 // byte offset of this rank's block in a full row
  uint32_t* flags[kPeerMaxWorld];  // every rank's flag array [world] for this exchange
  uint32_t* state;                 // this rank's [2]: running CTA total, unused (zero-initialised)
  float* max_out;                  // max mode: [rows] per-row maximum of the gathered floats
  int rank, world;
  int* status;
};

__global__ void __launch_bounds__(kPeerThreads) peer_gather_kernel(const __grid_constant__ PeerGatherParams p) {
  pdl_launch_dependents();   // the next kernel may begin launching (it waits for this grid)
  pdl_wait();                // the block was written by the previous kernel on the stream
  int rows = p.rows;
  if (p.plan != nullptr) {
    const int pm = __ldg(p.plan);
    rows = pm < 0 ? 0 : (pm > p.rows ? p.rows : pm);
  }
  // 1. copy the block into every rank's full buffer
  const int unit = p.vec16 ? 16 : 4;
  const int units = p.row_bytes / unit;
  const int64_t total = static_cast<int64_t>(rows) * units;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * kPeerThreads + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * kPeerThreads) {
    const int64_t r = e / units;
    const int64_t c = (e - r * units) * unit;
    const uint8_t* s = p.src + r * p.ld_src + c;
    const int64_t o = r * p.ld_dst + p.dst_off + c;
    if (p.vec16) {
      const uint4 v = *reinterpret_cast<const uint4*>(s);
      for (int q = 0; q < p.world; ++q) *reinterpret_cast<uint4*>(p.dst[q] + o) = v;
    } else {
      const uint32_t v = *reinterpret_cast<const uint32_t*>(s);
      for (int q = 0; q < p.world; ++q) *reinterpret_cast<uint32_t*>(p.dst[q] + o) = v;
    }
  }
  // 2. the CTA's stores are done (barrier); one release reduction per peer publishes them
  __syncthreads();
  if (threadIdx.x == 0)
    for (int q = 0; q < p.world; ++q)
      if (q != p.rank) red_release_sys_add_u32(p.flags[q] + p.rank, 1u);
  if (blockIdx.x != 0) return;
  // 3. CTA 0: wait until every peer's CTAs of this launch have landed here
  if (threadIdx.x == 0) {
    const uint32_t landed = p.state[0] + gridDim.x;   // peer CTAs landed here, all launches
    p.state[0] = landed;
    const uint64_t t0 = globaltimer_ns();
    bool timed_out = false;
    for (int q = 0; q < p.world && !timed_out; ++q) {
      if (q == p.rank) continue;
      while (static_cast<int32_t>(ld_acquire_sys_u32(p.flags[p.rank] + q) - landed) < 0) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          report_status(p.status, SPECQ_STATUS_TIMEOUT_PEER);
          timed_out = true;
          break;
        }
      }
    }
  }
  __syncthreads();
  // 4. max mode: per-row maximum of the gathered [rows, world] floats
  if (p.max_out != nullptr) {
    const float* full = reinterpret_cast<const float*>(p.dst[p.rank]);
    const int64_t ld = p.ld_dst / 4;
    for (int r = threadIdx.x; r < rows; r += kPeerThreads) {
      float m = full[r * ld];
      for (int q = 1; q < p.world; ++q) m = fmaxf(m, full[r * ld + q]);
      p.max_out[r] = m;
    }
  }
}

inline int run_peer_gather(const void* src, int64_t ld_src, int row_bytes, const int32_t* plan, int rows,
                           void* const* dst, int64_t ld_dst, int64_t dst_off, uint32_t* const* flags,
                           uint32_t* state, float* max_out, int rank, int world, void* stream) {
  if (world < 1 || world > kPeerMaxWorld || rank < 0 || rank >= world)
    return fail(SPECQ_ERR_INVALID_ARG, "peer_gather: rank %d of world %d (1..%d ranks)", rank, world, kPeerMaxWorld);
  if (rows < 0 || row_bytes <= 0 || row_bytes % 4 != 0)
    return fail(SPECQ_ERR_INVALID_ARG, "peer_gather: rows=%d row_bytes=%d (a positive multiple of 4)", rows, row_bytes);
  if (src == nullptr || dst == nullptr || flags == nullptr || state == nullptr)
    return fail(SPECQ_ERR_INVALID_ARG, "peer_gather: null pointer");
  for (int q = 0; q < world; ++q)
    if (dst[q] == nullptr || flags[q] == nullptr) return fail(SPECQ_ERR_INVALID_ARG, "peer_gather: null pointer of rank %d", q);
  if (ld_src < row_bytes || dst_off < 0 || dst_off + row_bytes > ld_dst || ld_src % 4 != 0 || ld_dst % 4 != 0 ||
      dst_off % 4 != 0 || !aligned(src, 4))
    return fail(SPECQ_ERR_INVALID_ARG, "peer_gather: strides / offset (ld_src %lld, ld_dst %lld, off %lld)",
                (long long)ld_src, (long long)ld_dst, (long long)dst_off);
  if (max_out != nullptr && (row_bytes != 4 || ld_dst != 4LL * world || dst_off != 4LL * rank))
    return fail(SPECQ_ERR_INVALID_ARG, "peer_gather: max mode takes one float per rank and row");
  DeviceState* dev = nullptr;
  if (int rc = get_device_state(&dev)) return rc;
  PeerGatherParams p = {};
  p.src = static_cast<const uint8_t*>(src);
  p.ld_src = ld_src;
  p.row_bytes = row_bytes;
  bool v16 = row_bytes % 16 == 0 && ld_src % 16 == 0 && ld_dst % 16 == 0 && dst_off % 16 == 0 && aligned(src, 16);
  for (int q = 0; q < world; ++q) {
    p.dst[q] = static_cast<uint8_t*>(dst[q]);
    p.flags[q] = flags[q];
    v16 = v16 && aligned(dst[q], 16);
    if (!aligned(dst[q], 4) || !aligned(flags[q], 4)) return fail(SPECQ_ERR_INVALID_ARG, "peer_gather: misaligned buffer");
  }
  p.vec16 = v16 ? 1 : 0;
  p.plan = plan;
  p.rows = rows;
  p.ld_dst = ld_dst;
  p.dst_off = dst_off;
  p.state = state;
  p.max_out = max_out;
  p.rank = rank;
  p.world = world;
  p.status = dev->status;
  const int64_t units = static_cast<int64_t>(rows) * (row_bytes / (v16 ? 16 : 4));
  // about four units per thread, at most one CTA per SM; one CTA in max mode (CTA 0 reduces
  // the rows, its own column included, after the wait).  The grid depends on the call's
  // arguments only, so every rank launches the same grid.
  const int ctas = max_out != nullptr ? 1 : static_cast<int>(std::max<int64_t>(
      1, std::min<int64_t>(dev->sm_count, (units + 4 * kPeerThreads - 1) / (4 * kPeerThreads))));
  SPECQ_CUDA_TRY(launch_plain(peer_gather_kernel, dim3(ctas), dim3(kPeerThreads), static_cast<cudaStream_t>(stream), p));
  SPECQ_CUDA_TRY(cudaGetLastError());
  return SPECQ_OK;
}

}  // namespace specq
