// specq_api.cu -- the extern "C" entry points of libspecq.so (declared in include/specq.h).
//
// Each entry point validates its arguments on the host, chooses the kernel variant and launch
// geometry (split-K, token chunks, pipeline depth), encodes the TMA tensor maps and launches
// on the caller's stream.  No allocation, no synchronisation: calls are graph-capturable.
#include <algorithm>

#include "specq_host.cuh"
#include "w8a8.cuh"
#include "w4a16.cuh"
#include "paged_attn.cuh"
#include "rowops.cuh"
#include "mma_peak.cuh"
#include "peer_gather.cuh"

namespace specq {

// Per-device status word: kernels record timeouts and clamped plan values here.
__device__ int g_specq_status = 0;

int* device_status_symbol_address() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_specq_status) != cudaSuccess) return nullptr;
  return static_cast<int*>(p);
}

// The running CTA totals of specq_peer_gather_noalloc: SPECQ_PEER_NOALLOC_SLOTS exchanges x
// {running total, unused}, in the same layout as specq_peer_gather's caller-owned `state`.
// Module-scope device storage: every GPU that loads the library holds these 512 bytes until
// the process exits.  Host code must not pass `g_peer_noalloc_state` itself to a kernel (on the
// host the name is a stand-in, not a device address); peer_noalloc_table() gives the address.
static __device__ __align__(256) uint32_t g_peer_noalloc_state[2 * SPECQ_PEER_NOALLOC_SLOTS];

// Device address of the table on the current device, looked up once per device (with that
// device current, as cudaGetSymbolAddress requires) and cached.
int peer_noalloc_table(uint32_t** out) {
  static std::mutex mu;
  static uint32_t* table[kMaxDevices] = {};
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(SPECQ_ERR_NO_DEVICE, "no current CUDA device");
  std::lock_guard<std::mutex> lock(mu);
  if (table[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_peer_noalloc_state);
    if (e != cudaSuccess || p == nullptr)
      return fail(SPECQ_ERR_CUDA, "peer_gather_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                  cudaGetErrorString(e));
    table[dev] = static_cast<uint32_t*>(p);
  }
  *out = table[dev];
  return SPECQ_OK;
}

// ---------------------------------------------------------------------------------------------
// W8A8
// ---------------------------------------------------------------------------------------------
namespace {

constexpr int kSmemLimit = 232448;  // 227 KB opt-in per block on sm_100

template <int VEC, typename PeerT>
int launch_w8a8_variant(const W8A8Params& p, const CUtensorMap& tw, const W8A8ActMaps& ta, const PeerT& peer,
                        dim3 grid, int smem, cudaStream_t stream) {
  auto kern = w8a8_kernel<VEC, PeerT>;
  SPECQ_CUDA_TRY(ensure_dyn_smem(reinterpret_cast<const void*>(kern), smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kW8A8Threads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream;
  LaunchAttrs attrs(p.splits);
  attrs.apply(cfg);
  SPECQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p, tw, ta, peer));
  return SPECQ_OK;
}

int w8a8_variant_id(int vec) {
  switch (vec) {
    case 0: return 0;
    case 16: return 1;
    case 8: return 2;
    case 4: return 3;
    case 2: return 4;
    default: return 5;
  }
}

// Tensor-parallel output of the W8A8 epilogue (null: the plain output): every rank's output
// block base (host array of `world` device pointers) and every rank's flag array.
struct W8A8PeerArgs {
  void* const* out;
  uint32_t* const* flags;
  int rank, world;
};

int run_w8a8(const int8_t* a, int64_t lda, const float* sa, const int8_t* w, int64_t ldw, const float* sw,
             void* out, int64_t ldo, int64_t ldo_n, int32_t* acc, int64_t ldacc, const int32_t* plan, int M, int N,
             int K, void* stream, const W8A8PeerArgs* peer = nullptr) {
  if (M < 0 || N <= 0 || K <= 0) return fail(SPECQ_ERR_INVALID_ARG, "w8a8: bad shape M=%d N=%d K=%d", M, N, K);
  if (M == 0) return SPECQ_OK;   // nothing to compute (empty tensors may carry null pointers)
  if (a == nullptr || w == nullptr) return fail(SPECQ_ERR_INVALID_ARG, "w8a8: null input pointer");
  if (acc == nullptr && (out == nullptr || sa == nullptr || sw == nullptr))
    return fail(SPECQ_ERR_INVALID_ARG, "w8a8: null output or scale pointer");
  if (lda < K || ldw < K) return fail(SPECQ_ERR_INVALID_ARG, "w8a8: row strides (%lld, %lld) < K=%d",
                                      (long long)lda, (long long)ldw, K);
  if (K > (1 << 30) / 127) return fail(SPECQ_ERR_UNSUPPORTED, "w8a8: K=%d could overflow the INT32 accumulator", K);
  if (acc != nullptr && ldacc < N)
    return fail(SPECQ_ERR_INVALID_ARG, "w8a8: accumulator row stride %lld < N=%d", (long long)ldacc, N);
  if (acc == nullptr && (ldo < 1 || ldo_n < 1))
    return fail(SPECQ_ERR_INVALID_ARG, "w8a8: output strides (%lld, %lld) must be positive", (long long)ldo,
                (long long)ldo_n);
  DeviceState* dev = nullptr;
  if (int rc = get_device_state(&dev)) return rc;

  W8A8Params p = {};
  p.a = a; p.w = w; p.sa = sa; p.sw = sw;
  p.out = static_cast<__half*>(out);
  p.acc_out = acc;
  p.plan = plan;
  p.status = dev->status;
  p.lda = lda; p.ldw = ldw; p.ldo = ldo; p.ldo_n = ldo_n; p.ldacc = ldacc;
  p.m_rows = M; p.N = N; p.K = K;
  W8A8PeerOut po = {};
  if (peer != nullptr) {
    if (peer->world < 1 || peer->world > kW8A8MaxPeers || peer->rank < 0 || peer->rank >= peer->world ||
        peer->out == nullptr || peer->flags == nullptr || acc != nullptr || ldo_n != 1)
      return fail(SPECQ_ERR_INVALID_ARG, "w8a8_peer: rank %d of world %d, fp16 rows of unit column stride",
                  peer->rank, peer->world);
    for (int q = 0; q < peer->world; ++q) {
      if (peer->out[q] == nullptr || peer->flags[q] == nullptr || !aligned(peer->out[q], 2) || !aligned(peer->flags[q], 4))
        return fail(SPECQ_ERR_INVALID_ARG, "w8a8_peer: null or misaligned buffer of rank %d", q);
      // the 16-byte epilogue stores need every rank's base aligned like this rank's own
      if ((reinterpret_cast<uintptr_t>(peer->out[q]) & 15u) != (reinterpret_cast<uintptr_t>(out) & 15u))
        return fail(SPECQ_ERR_INVALID_ARG, "w8a8_peer: rank %d's output base is aligned unlike this rank's", q);
      po.out[q] = static_cast<__half*>(peer->out[q]);
      po.flags[q] = peer->flags[q];
    }
    po.world = peer->world;
    po.rank = peer->rank;
  }

  // One token chunk per CTA up to kW8A8MaxChunk tokens (past 256 rows: a multiple of 32, so a
  // whole chunk arrives in two TMA boxes of chunk / 2 rows) for plan-buffer grids -- the same
  // grid and split-K as eager calls at the small active M a graph mostly serves -- and for
  // shapes with at least one channel tile per SM.  Eager calls of narrower shapes keep chunks
  // of at most 256 tokens: two chunks of 144 at M = 288 halve the split-K partials that the
  // cluster reduces (measured: o_proj 4096 x 4096 at M = 288 runs 11.5 us vs 17.7 us).
  // Int32 accumulation is exact, so the chunking never changes the bits.
  const int max_chunk = (plan != nullptr || ceil_div(N, 128) >= dev->sm_count) ? kW8A8MaxChunk : 256;
  const int n_chunks = ceil_div(M, max_chunk);
  p.chunk = round_up(ceil_div(M, n_chunks), 16);
  if (p.chunk > 256) p.chunk = round_up(p.chunk, 32);
  p.chunk_box = p.chunk > 256 ? p.chunk / 2 : p.chunk;
  p.kb_total = ceil_div(K, 128);
  const int n_tiles = ceil_div(N, 128);
  const int base = n_tiles * n_chunks;
  int S = 1;
  // Clusters of 8 only for grids of at most 64 CTAs: more of them do not fit the GPCs in one
  // wave (measured: 16 tiles x 8 splits ran 1.6x slower than 16 x 4).
  for (int cand : {8, 4, 2}) {
    const int kbps = ceil_div(p.kb_total, cand);
    if ((cand - 1) * kbps < p.kb_total && base * cand <= dev->sm_count && (cand < 8 || base * cand <= 64)) {
      S = cand;
      break;
    }
  }
  p.splits = S;
  p.kb_per_split = ceil_div(p.kb_total, S);

  p.stage_bytes = kW8A8WTile + static_cast<uint32_t>(round_up(p.chunk, 16)) * 128u;
  // split-K partial tile [128][chunk] int32 (padded rows), parked in the idle ring
  const uint32_t red_bytes = (S > 1) ? 128u * (static_cast<uint32_t>(round_up(p.chunk, 16)) * 4u + 16u) : 0u;
  const int overhead = 1024 + 256 + (kW8A8MaxChunk + 128) * 4;   // alignment slack, barriers, staged scales
  int stages = std::min(8, (kSmemLimit - overhead) / static_cast<int>(p.stage_bytes));
  if (stages < 2) return fail(SPECQ_ERR_UNSUPPORTED, "w8a8: token chunk %d does not fit shared memory", p.chunk);
  while (static_cast<uint32_t>(stages) * p.stage_bytes < red_bytes && stages < 8) ++stages;
  p.stages = stages;
  p.ring_bytes = static_cast<uint32_t>(stages) * p.stage_bytes;
  const int smem = overhead + stages * static_cast<int>(p.stage_bytes);
  if (smem > kSmemLimit) return fail(SPECQ_ERR_UNSUPPORTED, "w8a8: shared memory %d > limit", smem);
  p.tmem_cols = static_cast<uint32_t>(std::max(32, next_pow2(p.chunk)));

  // TMA needs 16-byte aligned bases and row strides; otherwise use the register-staged loader.
  const bool tma_ok = aligned(a, 16) && aligned(w, 16) && (lda % 16 == 0) && (ldw % 16 == 0);
  CUtensorMap tw;
  W8A8ActMaps ta;
  memset(&tw, 0, sizeof(tw));
  memset(&ta, 0, sizeof(ta));
  int vec = 0;
  if (tma_ok) {
    const uint64_t dw[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
    const uint64_t sw_[1] = {static_cast<uint64_t>(ldw)};
    const uint32_t bw[2] = {128, 128};
    if (int rc = encode_tiled(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w, dw, sw_, bw, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
    const uint64_t da[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    const uint64_t sa_[1] = {static_cast<uint64_t>(lda)};
    for (int b = 0; b < 4; ++b) {
      const uint32_t ba[2] = {128, 16u << b};
      if (int rc = encode_tiled(&ta.rows[b], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a, da, sa_, ba, CU_TENSOR_MAP_SWIZZLE_128B))
        return rc;
    }
    const uint32_t bac[2] = {128, static_cast<uint32_t>(p.chunk_box)};   // a whole token chunk (or half of it)
    if (int rc = encode_tiled(&ta.chunk, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a, da, sa_, bac, CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  } else {
    vec = common_vec_width({reinterpret_cast<uintptr_t>(a), reinterpret_cast<uintptr_t>(w),
                            static_cast<uint64_t>(lda), static_cast<uint64_t>(ldw), static_cast<uint64_t>(K)});
  }

  // (split, chunk, tile): a tile's chunks launch back to back and share its weights through L2
  if (n_tiles > 65535) return fail(SPECQ_ERR_UNSUPPORTED, "w8a8: N=%d exceeds the grid", N);
  const dim3 grid(static_cast<unsigned>(S), static_cast<unsigned>(n_chunks), static_cast<unsigned>(n_tiles));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc;
  if (peer != nullptr) {   // tensor-parallel output: the TMA variant (16-byte aligned operands)
    if (vec != 0) return fail(SPECQ_ERR_UNSUPPORTED, "w8a8_peer: operands must be 16-byte aligned (TMA)");
    rc = launch_w8a8_variant<0>(p, tw, ta, po, grid, smem, st);
  } else {
    const W8A8NoPeer np = {};
    switch (vec) {
      case 0: rc = launch_w8a8_variant<0>(p, tw, ta, np, grid, smem, st); break;
      case 16: rc = launch_w8a8_variant<16>(p, tw, ta, np, grid, smem, st); break;
      case 8: rc = launch_w8a8_variant<8>(p, tw, ta, np, grid, smem, st); break;
      case 4: rc = launch_w8a8_variant<4>(p, tw, ta, np, grid, smem, st); break;
      case 2: rc = launch_w8a8_variant<2>(p, tw, ta, np, grid, smem, st); break;
      default: rc = launch_w8a8_variant<1>(p, tw, ta, np, grid, smem, st); break;
    }
  }
  if (rc == SPECQ_OK) {
    LaunchRecord& r = last_launch_ref();
    r.variant = w8a8_variant_id(vec);
    r.grid[0] = static_cast<int>(grid.x); r.grid[1] = static_cast<int>(grid.y); r.grid[2] = static_cast<int>(grid.z);
    r.cluster_x = S;
    r.threads = kW8A8Threads;
    r.dyn_smem = smem;
  }
  return rc;
}

const void* w8a8_kernel_by_variant(int variant) {
  switch (variant) {
    case 0: return reinterpret_cast<const void*>(w8a8_kernel<0, W8A8NoPeer>);
    case 1: return reinterpret_cast<const void*>(w8a8_kernel<16, W8A8NoPeer>);
    case 2: return reinterpret_cast<const void*>(w8a8_kernel<8, W8A8NoPeer>);
    case 3: return reinterpret_cast<const void*>(w8a8_kernel<4, W8A8NoPeer>);
    case 4: return reinterpret_cast<const void*>(w8a8_kernel<2, W8A8NoPeer>);
    case 5: return reinterpret_cast<const void*>(w8a8_kernel<1, W8A8NoPeer>);
    default: return nullptr;
  }
}


// ---------------------------------------------------------------------------------------------
// W4A16
// ---------------------------------------------------------------------------------------------
int run_w4a16(const void* a, int64_t lda, const uint8_t* wp, int64_t ldwp, const void* sc, int64_t ldsc, int group,
              void* out, int64_t ldo, int64_t ldo_n, const int32_t* plan, int M, int N, int K, void* stream) {
  if (M < 0 || N <= 0 || K <= 0) return fail(SPECQ_ERR_INVALID_ARG, "w4a16: bad shape M=%d N=%d K=%d", M, N, K);
  if (M == 0) return SPECQ_OK;   // nothing to compute (empty tensors may carry null pointers)
  if (a == nullptr || wp == nullptr || sc == nullptr || out == nullptr)
    return fail(SPECQ_ERR_INVALID_ARG, "w4a16: null pointer");
  if (group <= 0) return fail(SPECQ_ERR_INVALID_ARG, "w4a16: group=%d", group);
  if (K % 2 != 0) return fail(SPECQ_ERR_INVALID_ARG, "w4a16: K=%d must be even (split-half packing)", K);
  if ((K / 2) % 64 != 0 || group % 64 != 0)
    return fail(SPECQ_ERR_UNSUPPORTED, "w4a16: needs (K/2) %% 64 == 0 and group %% 64 == 0 (K=%d, group=%d)", K, group);
  if (lda < K || ldwp < K / 2 || ldsc < (K + group - 1) / group)
    return fail(SPECQ_ERR_INVALID_ARG, "w4a16: row strides too small");
  if (ldo < 1 || ldo_n < 1)
    return fail(SPECQ_ERR_INVALID_ARG, "w4a16: output strides (%lld, %lld) must be positive", (long long)ldo,
                (long long)ldo_n);
  if (!aligned(a, 16) || (lda * 2) % 16 != 0 || !aligned(wp, 16) || ldwp % 16 != 0)
    return fail(SPECQ_ERR_UNSUPPORTED, "w4a16: activations/packed weights need 16-byte aligned rows");
  if (M == 0) return SPECQ_OK;
  DeviceState* dev = nullptr;
  if (int rc = get_device_state(&dev)) return rc;

  W4A16Params p = {};
  p.a = static_cast<const __half*>(a);
  p.wp = wp;
  p.sc = static_cast<const __half*>(sc);
  p.out = static_cast<__half*>(out);
  p.plan = plan;
  p.status = dev->status;
  p.lda = lda; p.ldwp = ldwp; p.ldsc = ldsc; p.ldo = ldo; p.ldo_n = ldo_n;
  p.m_rows = M; p.N = N; p.K = K; p.group = group;
  p.group_shift = ((group & (group - 1)) == 0) ? __builtin_ctz(static_cast<unsigned>(group)) : -1;
  p.kb_total = K / 128;
  const int n_tiles = ceil_div(N, 128);
  // The split depends on (N, K) only, never on M: plan and non-plan calls reduce the same
  // partial sums in the same order.
  int S = 1;
  for (int cand : {8, 4, 2}) {
    const int kbps = ceil_div(p.kb_total, cand);
    if ((cand - 1) * kbps < p.kb_total && n_tiles * cand <= dev->sm_count) { S = cand; break; }
  }
  p.splits = S;
  p.kb_per_split = ceil_div(p.kb_total, S);
  // Scale tile by TMA when its rows allow it (16-byte aligned, <= 32 KB); otherwise each
  // K-block's two scales per row are prefetched into registers one block ahead.  A row holds
  // ceil(K / group) groups: with K % group != 0 the last group is partial, and the high-half
  // K-blocks near the end read it (column (k + K/2) / group, as kernels.py:119-120 does).
  const int G = (K + group - 1) / group;
  const bool sc_tma = (G % 8 == 0) && G <= 128 && aligned(sc, 16) && (ldsc * 2) % 16 == 0;
  p.sc_cache_cols = sc_tma ? static_cast<uint32_t>(G) : 0u;
  const int sc_bytes = sc_tma ? 128 * G * 2 : 0;

  int n_chunks = ceil_div(M, 256);
  int smem = 0;
  while (true) {
    p.chunk = round_up(ceil_div(M, n_chunks), 16);
    p.stage_bytes = 2u * static_cast<uint32_t>(round_up(p.chunk, 16)) * 128u;   // activations, lo + hi
    const int fixed = 1024 + 2 * sc_bytes + 1024;   // + the scale tile and its transpose, barriers
    const uint32_t red_bytes = (S > 1) ? 128u * (static_cast<uint32_t>(p.chunk) * 4u + 16u) : 0u;
    // activation ring 2..6 deep (L2-resident, held until the MMA has read it); the
    // packed-weight ring (HBM, released as soon as dequant has read it) takes the rest, up
    // to 16 stages
    int xs = 6;
    while (xs > 2 && fixed + xs * static_cast<int>(p.stage_bytes) + 8 * static_cast<int>(kW4A16PackTile) > kSmemLimit) --xs;
    const int room = kSmemLimit - fixed - xs * static_cast<int>(p.stage_bytes);
    int ws = std::min(16, room / static_cast<int>(kW4A16PackTile));
    // the split-K partial tile is parked in the (then idle) rings
    while (ws < 16 && static_cast<uint32_t>(ws * kW4A16PackTile + xs * p.stage_bytes) < red_bytes &&
           fixed + (ws + 1) * static_cast<int>(kW4A16PackTile) + xs * static_cast<int>(p.stage_bytes) <= kSmemLimit)
      ++ws;
    // >= 4 weight stages: the dequant groups' parity waits on a stage rely on it (w4a16.cuh)
    if (ws >= 4 && static_cast<uint32_t>(ws * kW4A16PackTile + xs * p.stage_bytes) >= red_bytes) {
      p.stages = ws;
      p.xstages = xs;
      smem = fixed + ws * static_cast<int>(kW4A16PackTile) + xs * static_cast<int>(p.stage_bytes);
      break;
    }
    if (p.chunk <= 16) return fail(SPECQ_ERR_UNSUPPORTED, "w4a16: shapes do not fit shared memory");
    ++n_chunks;
  }
  // accumulator columns [0, round_up(chunk, 32)), then as many 64-column A slots as fit
  p.tmem_cols = 512;
  // one A slot per dequant group measured fastest (more slots let the groups run ahead and
  // compete with each other for issue slots without feeding the MMA any sooner)
  p.aslots = std::min(kW4A16Groups, (512 - round_up(p.chunk, 32)) / 64);
  if (p.aslots != kW4A16Groups)   // the dequant group g always fills A slot g
    return fail(SPECQ_ERR_UNSUPPORTED, "w4a16: token chunk %d leaves %d TMEM A slots", p.chunk, p.aslots);
  p.a_col = static_cast<uint32_t>(512 - 64 * p.aslots);

  CUtensorMap tw, ta, tac, tsc;
  memset(&tw, 0, sizeof(tw));
  memset(&ta, 0, sizeof(ta));
  memset(&tac, 0, sizeof(tac));
  memset(&tsc, 0, sizeof(tsc));
  if (sc_tma) {
    const uint64_t d[2] = {static_cast<uint64_t>(G), static_cast<uint64_t>(N)};
    const uint64_t s_[1] = {static_cast<uint64_t>(ldsc) * 2u};
    const uint32_t b[2] = {static_cast<uint32_t>(G), 128};
    if (int rc = encode_tiled(&tsc, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, sc, d, s_, b, CU_TENSOR_MAP_SWIZZLE_NONE)) return rc;
  }
  {
    const uint64_t d[2] = {static_cast<uint64_t>(K / 2), static_cast<uint64_t>(N)};
    const uint64_t s_[1] = {static_cast<uint64_t>(ldwp)};
    const uint32_t b[2] = {64, 128};
    if (int rc = encode_tiled(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, wp, d, s_, b, CU_TENSOR_MAP_SWIZZLE_64B)) return rc;
  }
  {
    const uint64_t d[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    const uint64_t s_[1] = {static_cast<uint64_t>(lda) * 2u};
    const uint32_t b[2] = {64, 16};
    if (int rc = encode_tiled(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a, d, s_, b, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
    const uint32_t bc[2] = {64, static_cast<uint32_t>(p.chunk)};   // a whole token chunk
    if (int rc = encode_tiled(&tac, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a, d, s_, bc, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
  }
  const dim3 grid(static_cast<unsigned>(S), static_cast<unsigned>(n_tiles), static_cast<unsigned>(n_chunks));
  SPECQ_CUDA_TRY(ensure_dyn_smem(reinterpret_cast<const void*>(w4a16_kernel), smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kW4A16Threads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = static_cast<cudaStream_t>(stream);
  LaunchAttrs attrs(S);
  attrs.apply(cfg);
  SPECQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, w4a16_kernel, p, tw, ta, tsc, tac));
  LaunchRecord& r = last_launch_ref();
  r.variant = 0;
  r.grid[0] = static_cast<int>(grid.x); r.grid[1] = static_cast<int>(grid.y); r.grid[2] = static_cast<int>(grid.z);
  r.cluster_x = S;
  r.threads = kW4A16Threads;
  r.dyn_smem = smem;
  return SPECQ_OK;
}

const void* w4a16_kernel_by_variant(int variant) {
  return variant == 0 ? reinterpret_cast<const void*>(w4a16_kernel) : nullptr;
}

// ---------------------------------------------------------------------------------------------
// failure-detection self test: a wait that nothing completes
// ---------------------------------------------------------------------------------------------
__global__ void selftest_wait_kernel(int* status, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1u);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(&bar, 0u)) {
      if (globaltimer_ns() - t0 > limit_ns) {
        report_status(status, SPECQ_STATUS_TIMEOUT_TEST);
        break;
      }
    }
  }
  __syncthreads();
}

}  // namespace
}  // namespace specq

using namespace specq;

extern "C" {

int specq_version(void) { return 100; }

const char* specq_last_error(void) { return last_error_ref().c_str(); }

int specq_w8a8(const int8_t* a, int64_t lda, const float* sa, const int8_t* w, int64_t ldw, const float* sw,
               void* out, int64_t ldo, int64_t ldo_n, const int32_t* plan, int M, int N, int K, void* stream) {
  last_launch_ref() = LaunchRecord();
  return run_w8a8(a, lda, sa, w, ldw, sw, out, ldo, ldo_n, nullptr, 0, plan, M, N, K, stream);
}

int specq_w8a8_peer(const int8_t* a, int64_t lda, const float* sa, const int8_t* w, int64_t ldw, const float* sw,
                    void* const* out, int64_t ldo, const int32_t* plan, int M, int N, int K, uint32_t* const* flags,
                    int rank, int world, void* stream) {
  last_launch_ref() = LaunchRecord();
  if (out == nullptr || world < 1 || rank < 0 || rank >= world || world > kW8A8MaxPeers)
    return fail(SPECQ_ERR_INVALID_ARG, "w8a8_peer: rank %d of world %d", rank, world);
  const W8A8PeerArgs peer = {out, flags, rank, world};
  return run_w8a8(a, lda, sa, w, ldw, sw, out[rank], ldo, 1, nullptr, 0, plan, M, N, K, stream, &peer);
}

int specq_w8a8_acc(const int8_t* a, int64_t lda, const int8_t* w, int64_t ldw, int32_t* acc, int64_t ldacc,
                   const int32_t* plan, int M, int N, int K, void* stream) {
  last_launch_ref() = LaunchRecord();
  if (acc == nullptr) return fail(SPECQ_ERR_INVALID_ARG, "w8a8_acc: null accumulator pointer");
  return run_w8a8(a, lda, nullptr, w, ldw, nullptr, nullptr, 0, 1, acc, ldacc, plan, M, N, K, stream);
}

int specq_w4a16(const void* a, int64_t lda, const uint8_t* wp, int64_t ldwp, const void* sc, int64_t ldsc, int group,
                void* out, int64_t ldo, int64_t ldo_n, const int32_t* plan, int M, int N, int K, void* stream) {
  last_launch_ref() = LaunchRecord();
  return run_w4a16(a, lda, wp, ldwp, sc, ldsc, group, out, ldo, ldo_n, plan, M, N, K, stream);
}

int specq_paged_attention(const void* q, int64_t q_sb, int64_t q_st, int64_t q_sh, const int8_t* kc, const int8_t* vc,
                          int64_t kv_sp, int64_t kv_so, int64_t kv_sh, int n_pages, const void* ks, const void* vs,
                          int64_t s_sp, int64_t s_so, int64_t s_sh, int scale_dtype, const int32_t* block_tbl,
                          int64_t bt_sb, int bt_cols, const int32_t* ctx_len, void* out, int64_t o_sb, int64_t o_st,
                          int64_t o_sh, const int32_t* plan, int B, int n_seqs, int q_len, int ql_max, int H,
                          int H_KV, int D, int page, int qpp, void* stream) {
  last_launch_ref() = LaunchRecord();
  return run_paged_attention(q, q_sb, q_st, q_sh, kc, vc, kv_sp, kv_so, kv_sh, n_pages, ks, vs, s_sp, s_so, s_sh,
                             scale_dtype, block_tbl, bt_sb, bt_cols, ctx_len, out, o_sb, o_st, o_sh, plan, B, n_seqs,
                             q_len, ql_max, H, H_KV, D, page, qpp, stream);
}

int specq_quant_rows(const void* x, int64_t ldx, void* r, int64_t ldr, int8_t* q, int64_t ldq, float* s,
                     const int32_t* plan, const float* amax_in, float* amax_out, int M, int N, int mode,
                     void* stream) {
  last_launch_ref() = LaunchRecord();
  return run_quant_rows(x, ldx, r, ldr, q, ldq, s, plan, amax_in, amax_out, M, N, mode, stream);
}

int specq_quant_rows_peer(const void* x, int64_t ldx, void* r, int64_t ldr, int8_t* q, int64_t ldq, float* s,
                          const int32_t* plan, const float* amax_in, float* amax_out, int M, int N, int mode,
                          const uint32_t* wait_flags, int rank, int world, void* stream) {
  last_launch_ref() = LaunchRecord();
  if (wait_flags == nullptr) return fail(SPECQ_ERR_INVALID_ARG, "quant_rows_peer: null flag array");
  return run_quant_rows(x, ldx, r, ldr, q, ldq, s, plan, amax_in, amax_out, M, N, mode, stream, wait_flags, rank,
                        world);
}

int specq_kv_append(const void* x, int64_t ldx, int k_col, int v_col, int8_t* kc, int8_t* vc, int64_t kv_sp,
                    int64_t kv_so, int64_t kv_sh, int n_pages, void* ks, void* vs, int64_t s_sp, int64_t s_so,
                    int64_t s_sh, const int32_t* block_tbl, int64_t bt_sb, int bt_cols, const int32_t* ctx_len,
                    const int32_t* plan, int B, int n_seqs, int q_len, int ql_max, int H_KV, int D, int page,
                    void* stream) {
  last_launch_ref() = LaunchRecord();
  return run_kv_append(x, ldx, k_col, v_col, kc, vc, kv_sp, kv_so, kv_sh, n_pages, ks, vs, s_sp, s_so, s_sh,
                       block_tbl, bt_sb, bt_cols, ctx_len, plan, B, n_seqs, q_len, ql_max, H_KV, D, page, stream);
}

int specq_pack_int4(const void* w, int w_dtype, int64_t ldw, int N, int K, int group, uint8_t* wp, int64_t ldwp,
                    void* sc, int64_t ldsc, void* deq, int64_t lddeq, void* stream) {
  last_launch_ref() = LaunchRecord();
  return run_pack_int4(w, w_dtype, ldw, N, K, group, wp, ldwp, sc, ldsc, deq, lddeq, stream);
}

int specq_kernel_info(int which, int variant, int* num_regs, int* local_bytes, int* static_smem, int* dynamic_smem,
                      int* max_threads) {
  const void* fn = nullptr;
  if (which == 0) fn = w8a8_kernel_by_variant(variant);
  else if (which == 1) fn = w4a16_kernel_by_variant(variant);
  else if (which == 2) fn = paged_attn_kernel_by_variant(variant);
  if (fn == nullptr) return fail(SPECQ_ERR_INVALID_ARG, "kernel_info: unknown kernel %d variant %d", which, variant);
  cudaFuncAttributes at;
  SPECQ_CUDA_TRY(cudaFuncGetAttributes(&at, fn));
  if (num_regs) *num_regs = at.numRegs;
  if (local_bytes) *local_bytes = static_cast<int>(at.localSizeBytes);
  if (static_smem) *static_smem = static_cast<int>(at.sharedSizeBytes);
  if (dynamic_smem) *dynamic_smem = at.maxDynamicSharedSizeBytes;
  if (max_threads) *max_threads = at.maxThreadsPerBlock;
  return SPECQ_OK;
}

int specq_last_launch(int* variant, int* grid_x, int* grid_y, int* grid_z, int* cluster_x, int* threads,
                      int* dynamic_smem) {
  const LaunchRecord& r = last_launch_ref();
  if (variant) *variant = r.variant;
  if (grid_x) *grid_x = r.grid[0];
  if (grid_y) *grid_y = r.grid[1];
  if (grid_z) *grid_z = r.grid[2];
  if (cluster_x) *cluster_x = r.cluster_x;
  if (threads) *threads = r.threads;
  if (dynamic_smem) *dynamic_smem = r.dyn_smem;
  return SPECQ_OK;
}

int specq_last_launch_packed(int* record) {
  if (record == nullptr) return fail(SPECQ_ERR_INVALID_ARG, "last_launch_packed: null record");
  const LaunchRecord& r = last_launch_ref();
  record[0] = r.variant;
  record[1] = r.grid[0];
  record[2] = r.grid[1];
  record[3] = r.grid[2];
  record[4] = r.cluster_x;
  record[5] = r.threads;
  record[6] = r.dyn_smem;
  return SPECQ_OK;
}

int specq_get_status(int* status, int clear) {
  DeviceState* dev = nullptr;
  if (int rc = get_device_state(&dev)) return rc;
  int v = 0;
  SPECQ_CUDA_TRY(cudaMemcpy(&v, dev->status, sizeof(int), cudaMemcpyDeviceToHost));
  if (clear) {
    const int zero = 0;
    SPECQ_CUDA_TRY(cudaMemcpy(dev->status, &zero, sizeof(int), cudaMemcpyHostToDevice));
  }
  if (status) *status = v;
  return SPECQ_OK;
}

int specq_trace_configure(void* buffer, int cta) {
#ifdef SPECQ_TRACE
  unsigned long long* b = static_cast<unsigned long long*>(buffer);
  SPECQ_CUDA_TRY(cudaMemcpyToSymbol(g_specq_trace_buf, &b, sizeof(b)));
  SPECQ_CUDA_TRY(cudaMemcpyToSymbol(g_specq_trace_cta, &cta, sizeof(cta)));
  return SPECQ_OK;
#else
  (void)buffer;
  (void)cta;
  return fail(SPECQ_ERR_UNSUPPORTED, "trace points are compiled in only with -DSPECQ_TRACE");
#endif
}

int specq_mma_peak(int kind, int n, int a_mn_major, int b_mn_major, int a_tmem, int busy_warps, int busy_iters,
                   int iters, int ctas, uint32_t* sink, void* stream) {
  last_launch_ref() = LaunchRecord();
  if (kind != 0 && kind != 1) return fail(SPECQ_ERR_INVALID_ARG, "mma_peak: kind %d (0 = i8, 1 = f16)", kind);
  if (n < 16 || n > 256 || n % 16 != 0) return fail(SPECQ_ERR_INVALID_ARG, "mma_peak: N=%d", n);
  if (a_tmem && (kind != 1 || n > 128 || a_mn_major))
    return fail(SPECQ_ERR_INVALID_ARG, "mma_peak: A from tensor memory needs kind f16, K-major, N <= 128");
  if (iters < 2 || ctas < 1 || sink == nullptr || busy_warps < 0 || busy_warps > 28 || busy_iters < 0)
    return fail(SPECQ_ERR_INVALID_ARG, "mma_peak: iters=%d ctas=%d busy_warps=%d", iters, ctas, busy_warps);
  DeviceState* dev = nullptr;
  if (int rc = get_device_state(&dev)) return rc;
  MmaPeakParams mp = {};
  mp.iters = iters;
  mp.n = static_cast<uint32_t>(n);
  mp.a_mn = a_mn_major ? 1u : 0u;
  mp.b_mn = b_mn_major ? 1u : 0u;
  mp.a_tmem = a_tmem;
  mp.busy_warps = busy_warps;
  mp.busy_iters = busy_iters;
  mp.status = dev->status;
  mp.sink = sink;
  auto kern = kind == 0 ? mma_peak_kernel<0> : mma_peak_kernel<1>;
  SPECQ_CUDA_TRY(ensure_dyn_smem(reinterpret_cast<const void*>(kern), kPeakSmem));
  const int threads = kPeakThreads + 32 * busy_warps;
  kern<<<ctas, threads, kPeakSmem, static_cast<cudaStream_t>(stream)>>>(mp);
  SPECQ_CUDA_TRY(cudaGetLastError());
  LaunchRecord& r = last_launch_ref();
  r.variant = kind;
  r.grid[0] = ctas; r.grid[1] = 1; r.grid[2] = 1;
  r.cluster_x = 1;
  r.threads = threads;
  r.dyn_smem = kPeakSmem;
  return SPECQ_OK;
}

int specq_peer_gather(const void* src, int64_t ld_src, int row_bytes, const int32_t* plan, int rows,
                      void* const* dst, int64_t ld_dst, int64_t dst_off, uint32_t* const* flags, uint32_t* state,
                      float* max_out, int rank, int world, void* stream) {
  last_launch_ref() = LaunchRecord();
  return run_peer_gather(src, ld_src, row_bytes, plan, rows, dst, ld_dst, dst_off, flags, state, max_out, rank,
                         world, stream);
}

int specq_peer_gather_noalloc(const void* src, int64_t ld_src, int row_bytes, const int32_t* plan, int rows,
                              void* const* dst, int64_t ld_dst, int64_t dst_off, uint32_t* const* flags, int slot,
                              int restart, float* max_out, int rank, int world, void* stream) {
  last_launch_ref() = LaunchRecord();
  if (slot < 0 || slot >= SPECQ_PEER_NOALLOC_SLOTS)
    return fail(SPECQ_ERR_INVALID_ARG, "peer_gather_noalloc: slot %d outside 0..%d (the library's table holds %d exchanges)",
                slot, SPECQ_PEER_NOALLOC_SLOTS - 1, SPECQ_PEER_NOALLOC_SLOTS);
  uint32_t* table = nullptr;
  if (int rc = peer_noalloc_table(&table)) return rc;
  uint32_t* state = table + 2 * slot;
  if (restart) SPECQ_CUDA_TRY(cudaMemsetAsync(state, 0, 2 * sizeof(uint32_t), static_cast<cudaStream_t>(stream)));
  return run_peer_gather(src, ld_src, row_bytes, plan, rows, dst, ld_dst, dst_off, flags, state, max_out, rank,
                         world, stream);
}

int specq_selftest_wait_timeout(uint64_t limit_ns, void* stream) {
  DeviceState* dev = nullptr;
  if (int rc = get_device_state(&dev)) return rc;
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(dev->status, limit_ns);
  SPECQ_CUDA_TRY(cudaGetLastError());
  return SPECQ_OK;
}

}  // extern "C"
