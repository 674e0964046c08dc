/*
 * specq.h -- C ABI of the B200 (sm_100a) verification-shape kernels.
 *
 * Drop-in boundary for the three kernels of Vaibhav1067/specdec-quant-triton:
 *   specq_w8a8            replaces kernels.py:71-86   (w8a8_matmul   -> _w8a8_kernel,  kernels.py:27-55)
 *   specq_w4a16           replaces kernels.py:150-166 (w4a16_matmul  -> _w4a16_kernel, kernels.py:95-135)
 *   specq_paged_attention replaces kernels.py:239-262 (paged_attention -> _paged_attn_kernel, kernels.py:179-236)
 *   specq_kernel_info     replaces the compiled-kernel handle the wrappers return
 *                         (`ck.n_regs`, `ck.n_spills`, `ck.metadata.shared`, read by regs.py:29-32)
 *
 * Conventions
 *   - Plain pointers to device memory, sizes and strides in ELEMENTS of the pointed-to type.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Every call is asynchronous,
 *     does no host synchronisation and no device allocation, so it may be captured in a CUDA
 *     graph.
 *   - `plan` (optional, device int32): when non-NULL the active extent is read on the device
 *     (GEMMs: plan[0] = M; attention: plan[0] = n_seqs, plan[1] = q_len), CTAs outside it exit
 *     early and outputs outside it are never written.  The grid is sized by the maximum
 *     extent passed on the host (`grid_m_max`, `B`, `ql_max`).
 *   - Return value: SPECQ_OK or an error code; specq_last_error() gives the message
 *     (thread-local).  Invalid arguments are rejected on the host; nothing traps on the device.
 *   - Device-side conditions (a bounded wait that ran out, a plan value that had to be
 *     clamped) are recorded in a per-device status word read by specq_get_status().
 */
#ifndef SPECQ_H_
#define SPECQ_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- return codes ---------------------------------------------------------------------- */
#define SPECQ_OK 0
#define SPECQ_ERR_INVALID_ARG 1  /* shape, stride, dtype or alignment the kernel cannot take   */
#define SPECQ_ERR_UNSUPPORTED 2  /* valid for the reference, not (yet) for this build          */
#define SPECQ_ERR_CUDA 3         /* a CUDA runtime / driver call failed                        */
#define SPECQ_ERR_NO_DEVICE 4    /* no sm_100 device is current                                */

/* ---- device status word bits (specq_get_status) ---------------------------------------- */
#define SPECQ_STATUS_TIMEOUT_PIPELINE 0x01 /* a producer/consumer mbarrier wait ran out            */
#define SPECQ_STATUS_TIMEOUT_MMA 0x02      /* waiting for tensor-core completion ran out           */
#define SPECQ_STATUS_TIMEOUT_TEST 0x04     /* specq_selftest_wait_timeout's deliberate wait         */
#define SPECQ_STATUS_TIMEOUT_PEER 0x08     /* a peer GPU's exchange signal did not arrive in time   */
#define SPECQ_STATUS_PLAN_CLAMPED 0x100    /* a plan value was outside [0, max] and was clamped     */

/* ---- dtypes for scale tensors ----------------------------------------------------------- */
#define SPECQ_DTYPE_F16 0
#define SPECQ_DTYPE_F32 1

/*
 * W8A8 GEMM.  out[m, n] = fp16( (fp32(sum_k a[m,k] * w[n,k]) * sa[m]) * sw[n] )
 *   a   int8  [M, K]  row stride lda     (per-token quantised activations)
 *   w   int8  [N, K]  row stride ldw     (per-channel quantised weights, "NT" layout)
 *   sa  fp32  [M]     sw fp32 [N]
 *   out fp16  [M, N]  strides (ldo, ldo_n)
 *   M   rows of a/sa/out the kernel may touch (the grid extent: grid_m_max in plan mode)
 * Reference: kernels.py:71-86 (wrapper), kernels.py:27-55 (kernel).
 */
int specq_w8a8(const int8_t* a, int64_t lda, const float* sa, const int8_t* w, int64_t ldw, const float* sw,
               void* out, int64_t ldo, int64_t ldo_n, const int32_t* plan, int M, int N, int K, void* stream);

/*
 * Same GEMM, but writes the raw INT32 accumulator acc[m, n] = sum_k a[m,k] * w[n,k] to
 * `acc` (row stride ldacc) instead of the scaled fp16 output.  Used to check the tensor-core
 * accumulator bit for bit against an exact integer reference (the `acc` of kernels.py:44-50).
 */
int specq_w8a8_acc(const int8_t* a, int64_t lda, const int8_t* w, int64_t ldw, int32_t* acc, int64_t ldacc,
                   const int32_t* plan, int M, int N, int K, void* stream);

/*
 * W4A16 GEMM.  out[m, n] = fp16( sum_k a[m,k] * fp16(q[n,k] * sc[n, k / group]) )
 *   a   fp16  [M, K]        row stride lda
 *   wp  uint8 [N, K/2]      row stride ldwp; byte j holds q[n,j]+8 (low nibble) and
 *                           q[n,j+K/2]+8 (high nibble)  (kernels.py:90-92, 143-145)
 *   sc  fp16  [N, K/group]  row stride ldsc
 *   out fp16  [M, N]        strides (ldo, ldo_n)
 * Reference: kernels.py:150-166 (wrapper), kernels.py:95-135 (kernel).
 */
int specq_w4a16(const void* a, int64_t lda, const uint8_t* wp, int64_t ldwp, const void* sc, int64_t ldsc,
                int group, void* out, int64_t ldo, int64_t ldo_n, const int32_t* plan, int M, int N, int K,
                void* stream);

/*
 * INT8 paged verification attention (kernels.py:239-262 wrapper, kernels.py:179-236 kernel).
 *   q        fp16 [B, QL_MAX, H, D]         strides (q_sb, q_st, q_sh), unit stride along D
 *   kc, vc   int8 [P, PAGE, H_KV, D]        strides (kv_sp, kv_so, kv_sh), unit stride along D;
 *                                           n_pages = P
 *   ks, vs   fp16 or fp32 [P, PAGE, H_KV]   strides (s_sp, s_so, s_sh); scale_dtype SPECQ_DTYPE_*
 *   block_tbl int32 [B, max_pages]          row stride bt_sb, bt_cols = max_pages
 *   ctx_len  int32 [B]                      context length including the q_len query tokens
 *   out      fp16 like q                    strides (o_sb, o_st, o_sh)
 * Rows (b, qi, head) with b < n_seqs and qi < q_len are written; nothing else is touched.
 * Row qi attends to tokens t <= ctx_len[b] - q_len + qi (causal verification window).
 * `qpp` (queries per program) only changes the schedule: 1 = one query token per CTA,
 * q_len = all k+1 tokens of a GQA group in one CTA (the fused verification kernel).
 * In plan mode, plan[0] = n_seqs and plan[1] = q_len; the grid is (B, ..., ceil(ql_max/qpp)).
 * q_sb = 0 (o_sb = 0) means packed token rows: sequence b's token t at row b * q_len + t of
 * a [tokens x ...] tensor, with q_len the active one (a projection's output under a plan graph).
 */
int specq_paged_attention(const void* q, int64_t q_sb, int64_t q_st, int64_t q_sh, const int8_t* kc,
                          const int8_t* vc, int64_t kv_sp, int64_t kv_so, int64_t kv_sh, int n_pages,
                          const void* ks, const void* vs, int64_t s_sp, int64_t s_so, int64_t s_sh,
                          int scale_dtype, const int32_t* block_tbl, int64_t bt_sb, int bt_cols,
                          const int32_t* ctx_len, void* out, int64_t o_sb, int64_t o_st, int64_t o_sh,
                          const int32_t* plan, int B, int n_seqs, int q_len, int ql_max, int H, int H_KV,
                          int D, int page, int qpp, void* stream);

/* Per-token symmetric INT8 quantisation of a verification layer's activations.
 * No reference counterpart as a kernel: it is the reference's quantize_act_int8
 * (kernels.py:58-62, a torch function) run on the device, bit-exact:
 *   s[m] = max(amax_n |y[m, n]|, 1e-8) * fp32(1/127)   (torch's `/ 127.0` on a CUDA tensor)
 *   q[m, n] = clamp(rint(y[m, n] / s[m]), -127, 127)
 * with, by `mode`,
 *   0  y = x                             x fp16 [M, N], row stride ldx
 *   1  y = x + r, and r <- fp16(x + r)    r fp16 [M, N] (the residual stream), row stride ldr
 *   2  y = silu(x[:, :N]) * x[:, N:2N]    x fp16 [M, 2N] (an MLP's gate and up halves)
 * q int8 [M, N] (row stride ldq), s fp32 [M].  plan (optional) = device int32, plan[0] = the
 * active M; rows past it are not touched.
 * Rows split across GPUs (tensor parallelism): amax_out (modes 0 and 2) makes this call only
 * write each row's amax |y| to amax_out[m] (q and s untouched); amax_in (any mode) makes it
 * quantise with amax_in[m] -- the maximum over all shards -- in place of the local amax, so
 * every shard gets the scale and the int8 values of the unsplit row.  Both may be null.
 */
int specq_quant_rows(const void* x, int64_t ldx, void* r, int64_t ldr, int8_t* q, int64_t ldq, float* s,
                     const int32_t* plan, const float* amax_in, float* amax_out, int M, int N, int mode,
                     void* stream);

/* Append the K and V of the q_len newest tokens of each sequence to an INT8 paged KV cache.
 * No reference counterpart as a kernel: the reference builds its cache with the fixture
 * make_paged_kv (kernels.py:265-286); this writes the same format for new tokens.
 *   x        fp16 [tokens, ...] packed token rows (sequence b's token t at row b*q_len + t),
 *            row stride ldx; K of KV head h at columns k_col + h*D .., V at v_col + h*D ..
 *   kc, vc   int8 [P, PAGE, H_KV, D], ks, vs fp16 [P, PAGE, H_KV] (strides as for attention)
 * Token t of sequence b goes to position ctx_len[b] - q_len + t through the block table, with
 * per (token, head) scale s = max(amax|k|, 1e-8) / 127 (fp32; stored fp16) and values
 * clamp(rint(k / s), -127, 127).  In plan mode plan[0] = n_seqs, plan[1] = q_len.
 */
int specq_kv_append(const void* x, int64_t ldx, int k_col, int v_col, int8_t* kc, int8_t* vc, int64_t kv_sp,
                    int64_t kv_so, int64_t kv_sh, int n_pages, void* ks, void* vs, int64_t s_sp, int64_t s_so,
                    int64_t s_sh, const int32_t* block_tbl, int64_t bt_sb, int bt_cols, const int32_t* ctx_len,
                    const int32_t* plan, int B, int n_seqs, int q_len, int ql_max, int H_KV, int D, int page,
                    void* stream);

/* Group-wise INT4 weight quantisation and packing on the device.
 * Replaces the reference's quantize_weight_int4 (kernels.py:138-147, a torch function), bit-exact
 * with it on a CUDA tensor:
 *   s[n, g] = max(amax |w[n, g*group ..]|, 1e-8) * fp32(1/7)   (torch's `/ 7.0` on a CUDA tensor)
 *   q[n, k] = clamp(rint(w[n, k] / s[n, k/group]), -8, 7)
 *   wp[n, j] = (q[n, j] + 8) | (q[n, j + K/2] + 8) << 4      uint8 [N, K/2], row stride ldwp
 *   sc[n, g] = fp16(s[n, g])                                 fp16 [N, K/group], row stride ldsc
 *   deq[n, k] = fp16(q[n, k] * s[n, k/group])                fp16 [N, K] (optional: null skips it)
 * w: [N, K] with row stride ldw elements, w_dtype 0 = fp16, 1 = fp32, 2 = bf16.
 * Requires K % 2 == 0 and (K/2) % group == 0 (kernels.py:140); group in {32, 64, 128, 256}.
 */
int specq_pack_int4(const void* w, int w_dtype, int64_t ldw, int N, int K, int group, uint8_t* wp, int64_t ldwp,
                    void* sc, int64_t ldsc, void* deq, int64_t lddeq, void* stream);

/*
 * Compiled-kernel metadata for the kernel variant a call with these arguments would launch
 * (the reference returns Triton's compiled kernel `ck`; regs.py:29-32 reads n_regs,
 * n_spills and metadata.shared from it).
 *   which: 0 = W8A8, 1 = W4A16, 2 = paged attention;  variant: as reported by the launch.
 */
int specq_kernel_info(int which, int variant, int* num_regs, int* local_bytes, int* static_smem,
                      int* dynamic_smem, int* max_threads);

/* Variant id and launch geometry of the most recent successful launch on this host thread:
 * kernel variant, grid (x, y, z), cluster size along x, threads per CTA, dynamic smem. */
int specq_last_launch(int* variant, int* grid_x, int* grid_y, int* grid_z, int* cluster_x, int* threads,
                      int* dynamic_smem);

/* The same record as one array: record[0..6] = variant, grid x, y, z, cluster x, threads,
 * dynamic smem (one pointer argument: the Python wrappers read it after every call). */
int specq_last_launch_packed(int* record);

/* Read (and with clear != 0, reset) the status word of the current device. Synchronous. */
int specq_get_status(int* status, int clear);

/*
 * Failure-detection self test: launches one CTA that waits on an mbarrier nothing will ever
 * complete, with a wait limit of `limit_ns` nanoseconds; the wait gives up, records
 * SPECQ_STATUS_TIMEOUT_TEST in the status word and the kernel returns normally.
 */
int specq_selftest_wait_timeout(uint64_t limit_ns, void* stream);

/*
 * Tensor-pipe throughput microbenchmark.  No reference counterpart: it measures the dense peak
 * that the GEMMs' large-M roofline is scored against (the pool measures only HBM copy bandwidth
 * and a cuBLAS bf16 GEMM), and prices the small MMAs the attention and GEMM kernels issue.
 * Launches `ctas` CTAs (one per SM: pass the SM count), each issuing `iters` x 4 back-to-back
 * tcgen05 MMAs of M=128 and N=`n` (16..256, multiple of 16) from shared-memory tiles into
 * tensor memory: kind 0 = kind::i8 (K=32, 2*128*n*32 ops each), kind 1 = kind::f16 (K=16).
 * a_mn_major / b_mn_major select MN-major operand layouts; a_tmem = 1 (kind 1, n <= 128) reads
 * A from tensor memory; `busy_warps` (0..28) extra warps each run `busy_iters` 16-byte
 * shared-memory loads and stores per thread meanwhile.  `sink` (device uint32 [ctas])
 * receives one checksum word per CTA.  Time it with events on `stream`.
 */
int specq_mma_peak(int kind, int n, int a_mn_major, int b_mn_major, int a_tmem, int busy_warps, int busy_iters,
                   int iters, int ctas, uint32_t* sink, void* stream);

/*
 * All-gather of row blocks over NVLink for tensor parallelism.  No reference counterpart (the
 * reference runs on one GPU): it is the exchange step of the tensor-parallel verification stack.
 * Rank `rank` of `world` (1..8) copies its block src [rows x row_bytes] (row stride ld_src
 * bytes) into byte columns [dst_off, dst_off + row_bytes) of EVERY rank's full buffer dst[q]
 * (row stride ld_dst bytes; memory that every rank can write, e.g. symmetric memory), signals
 * each peer q through flags[q][rank], and waits until flags[rank][q] shows that every peer's
 * block has landed (bounded: after 1 s it records SPECQ_STATUS_TIMEOUT_PEER and returns).
 * dst and flags are HOST arrays of `world` device pointers; flags[q] is rank q's uint32 [world]
 * flag array of this exchange and `state` this rank's device uint32 [2], both zero before the
 * first call.  Every rank must issue the same sequence of calls on each exchange.
 * max_out (optional): one float per rank and row (row_bytes = 4, ld_dst = 4 * world,
 * dst_off = 4 * rank); after the wait max_out[m] = the maximum over the ranks of row m.
 * plan (optional): plan[0] = the active rows (rows is the maximum).
 */
int specq_peer_gather(const void* src, int64_t ld_src, int row_bytes, const int32_t* plan, int rows,
                      void* const* dst, int64_t ld_dst, int64_t dst_off, uint32_t* const* flags, uint32_t* state,
                      float* max_out, int rank, int world, void* stream);

/*
 * specq_peer_gather for callers that cannot allocate device memory.  No counterpart in the
 * reference (which has no multi-GPU exchange at all).  Some hosts own every byte of device
 * memory themselves: a serving engine that reserves all free HBM for its KV cache at start-up
 * and forbids later cudaMalloc calls, or a plugin that may only use the buffers it is handed.
 * Such a caller still has its full buffers and flag arrays (they must be peer-visible, so they
 * come from the host's own symmetric pool), but it has nowhere to put the `state` words.  This
 * entry point keeps them in a table inside the library instead: a fixed device array of
 * SPECQ_PEER_NOALLOC_SLOTS exchanges x 2 words (512 bytes), which every GPU that loads the
 * library holds until the process exits.
 *   - slot (0 .. SPECQ_PEER_NOALLOC_SLOTS-1) picks the exchange's entry; any other value is
 *     rejected with SPECQ_ERR_INVALID_ARG.  One slot per flag-array set, like one `state`.
 *   - restart != 0 zeroes the slot on `stream` before the launch (a stream-ordered memset of the
 *     library's own table, no allocation).  Pass it on the first call that uses a freshly
 *     zeroed flag-array set: the table keeps whatever the last call on that slot left there.
 *   - Every other argument, and the result, is exactly as for specq_peer_gather.
 *   - The first call on a device looks up the table's device address (once per device, with
 *     that device current); make that first call before any stream capture.
 *   - All calls share the one table: calls that may overlap on the GPU (different streams with
 *     no ordering between them) and name the same slot race on its running total.
 * Nothing here calls cudaMalloc, cudaFree or any allocating library routine.
 */
#define SPECQ_PEER_NOALLOC_SLOTS 64
int specq_peer_gather_noalloc(const void* src, int64_t ld_src, int row_bytes, const int32_t* plan, int rows,
                              void* const* dst, int64_t ld_dst, int64_t dst_off, uint32_t* const* flags, int slot,
                              int restart, float* max_out, int rank, int world, void* stream);

/*
 * W8A8 GEMM with tensor-parallel output (no reference counterpart: the GEMM fused with the
 * tensor-parallel stack's all-gather).  The same product as specq_w8a8; its fp16 output rows
 * (unit column stride, row stride ldo) are stored into EVERY rank's full buffer over NVLink:
 * `out` is a HOST array of `world` (1..8) device pointers, out[q] = rank q's full buffer at this
 * rank's column block (out[rank] is this rank's own).  Once a CTA's stores are done it adds 1 to
 * slot `rank` of every rank's flag array flags[q] (host array of device pointers to uint32
 * [world], zero before the first call), its own included; the consumer waits with
 * specq_quant_rows_peer.  Every rank launches the same grid (same shapes and plan).
 */
int specq_w8a8_peer(const int8_t* a, int64_t lda, const float* sa, const int8_t* w, int64_t ldw, const float* sw,
                    void* const* out, int64_t ldo, const int32_t* plan, int M, int N, int K, uint32_t* const* flags,
                    int rank, int world, void* stream);

/*
 * specq_quant_rows on a full buffer written by every rank's specq_w8a8_peer: each CTA first
 * waits (bounded: 1 s, then SPECQ_STATUS_TIMEOUT_PEER and it goes on) until every rank's count
 * in wait_flags (this rank's flag array of that exchange) has reached this rank's own count.
 */
int specq_quant_rows_peer(const void* x, int64_t ldx, void* r, int64_t ldr, int8_t* q, int64_t ldq, float* s,
                          const int32_t* plan, const float* amax_in, float* amax_out, int M, int N, int mode,
                          const uint32_t* wait_flags, int rank, int world, void* stream);

/*
 * Pipeline tracing (builds compiled with -DSPECQ_TRACE only; other builds return
 * SPECQ_ERR_UNSUPPORTED): the CTA with linear index `cta` records SM-clock timestamps of its
 * pipeline events into `buffer` (device, 64 x 64 uint64: [event slot][iteration]).
 * buffer = NULL switches tracing off.
 */
int specq_trace_configure(void* buffer, int cta);

/* Message of the last error on this host thread ("" if none). */
const char* specq_last_error(void);

/* ABI version (major * 100 + minor). */
int specq_version(void);

#ifdef __cplusplus
}
#endif

#endif /* SPECQ_H_ */
