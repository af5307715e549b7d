/*
 * flagattn_b200.h -- C ABI of the B200 (sm_100a) paged / MLA decode engine.
 *
 * Every entry point takes plain device pointers, element strides, sizes and a
 * cudaStream_t (passed as void*), returns an int status (FA_OK == 0, negative
 * on error) and never allocates device memory: callers pass outputs and the
 * split scratch, sized with the *_workspace_* queries below.  Launches are
 * asynchronous on the given stream; argument errors are detected on the host
 * before anything is launched.
 *
 * Reference interfaces replaced (FlagAttention, src/flag_attn/...):
 *   fa_paged_attention        paged.py:20-177   (paged.attention, the Triton
 *                             _paged_attn_kernel :208-363 and the split reduce
 *                             _paged_attn_v2_reduce_kernel :366-449)
 *   fa_paged_num_splits       paged.py:54-67    (partition-count rule)
 *   fa_split_kv_attention     split_kv.py:279-344 and flash.py:72-143 (the
 *                             split-KV flash-decoding path that returns LSE)
 *   fa_split_kv_num_splits    split_kv.py:247-276 (num_splits_herustic)
 *   fa_lse_combine            split_kv.py:176-241 (_fwd_combine_kv_splits);
 *                             fa_lse_combine_strided is the same merge over
 *                             partials gathered from several GPUs
 *   fa_mla_get_metadata       no reference function: the FlashMLA-style
 *                             metadata call (get_mla_metadata) that the MLA
 *                             decode path needs; format defined in this file
 *   fa_mla_decode             paged.py:208-363 generalised to the MLA shape
 *                             (576-dim latent+rope keys, values = first 512
 *                             dims of the same rows, 128 query heads sharing
 *                             one latent head), dense or top-k sparse
 *   fa_mla_combine            paged.py:366-449 / split_kv.py:198-228, over the
 *                             per-sequence variable split counts of the
 *                             metadata
 *   fa_mla_append_rows        no reference function: writes new tokens'
 *                             latent rows into the paged pool read by the
 *                             decode (the cache layout of paged.py:22-23)
 *   fa_mla_combine_push,      paged.py:366-449 / split_kv.py:198-228 merges
 *   fa_lse_merge_wait         carried across GPUs (the reference has no
 *                             multi-GPU code); fa_ipc_* map peer memory
 */
#ifndef FLAGATTN_B200_H_
#define FLAGATTN_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define FA_OK 0
#define FA_ERR_INVALID_ARGUMENT (-1) /* shape / stride / alignment rejected  */
#define FA_ERR_UNSUPPORTED (-2)      /* valid but not handled by this build   */
#define FA_ERR_CUDA (-3)             /* a CUDA runtime/driver call failed     */
#define FA_ERR_NO_DEVICE (-4)        /* no usable sm_100 device               */

/* element types of q / caches / outputs */
#define FA_DTYPE_BF16 0
#define FA_DTYPE_F16 1
#define FA_DTYPE_F32 2

/* ---- MLA tile-scheduler metadata format ---------------------------------
 * tile_meta is int32 [num_sm_parts][FA_MLA_META_INTS].  Part p covers the
 * consecutive sequences begin_seq .. begin_seq + n_pieces - 1; the first piece
 * starts at 64-token block begin_blk, the last one (sequence end_seq) stops
 * before block end_blk, pieces in between are whole sequences.
 *   [0] begin_seq  [1] begin_blk  [2] end_seq  [3] end_blk
 *   [4] split index of the first piece inside its sequence
 *   [5] n_pieces (0: the part has no work)   [6],[7] zero
 * num_splits is int32 [batch + 1], the exclusive prefix sum of the number of
 * pieces per sequence: the partial results of sequence b occupy split slots
 * num_splits[b] .. num_splits[b+1]-1 of the workspace.  A sequence with one
 * piece is written straight to the output and skips the combine.          */
#define FA_MLA_META_INTS 8
#define FA_MLA_BLOCK_N 64      /* tokens per scheduled block (= page size) */
#define FA_MLA_FIXED_COST 5    /* per-piece overhead, in blocks            */

/* ---- library / device queries ------------------------------------------ */
int fa_version(void);                   /* (major << 16) | (minor << 8) | patch */
const char *fa_status_string(int status);
/* Last CUDA error text recorded by this thread's failing call (or ""). */
const char *fa_last_error(void);
/* Streaming multiprocessors of `device` (148 on B200). */
int fa_device_sm_count(int device, int *sm_count);

/* ---- reference split heuristics (pure host functions) ------------------- */
/* paged.py:54-67.  Inputs as in paged.attention; writes the partition count
 * and partition size (tokens; 0 when *num_splits == 1). */
int fa_paged_num_splits(int num_seqs, int num_kv_heads, int max_context_len,
                        int kv_block_size, int num_sms, int requested_splits,
                        int *num_splits, int *partition_size);
/* split_kv.py:247-276 (num_splits_herustic). */
int fa_split_kv_num_splits(int batch, int heads, int m, int n, int block_m,
                           int block_n, int num_sms, int max_splits,
                           int *num_splits);

/* ---- generic paged / contiguous decode ----------------------------------
 * Covers paged.attention (block_table != NULL) and the split-KV flash
 * decoding of split_kv.attention (block_table == NULL: sequence b's keys are
 * k + b*k_stride_seq + n*k_stride_tok + h*k_stride_head).  Any head size
 * d_qk <= 576 and d_v <= 512 (multiples of 8), grouped-query heads, optional
 * bottom-right causal masking for m_q > 1, f16/bf16/f32.
 * Query row (b, h, m) lives at q + b*q_stride_b + h*q_stride_h + m*q_stride_m;
 * the output uses the same scheme with o_* strides; lse (nullable) is f32
 * [batch][num_q_heads][m_q] contiguous.
 *
 * Two kernels serve it:
 *  - the tensor-core kernel (tcgen05 + TMA), used whenever
 *    fa_decode_uses_tensor_cores() says so: bf16/f16, d_qk == d_v in
 *    {16, 32, 64, 128, 256}, at most 128 query rows per kv head (group * m_q),
 *    scale > 0, 16-byte aligned rows, and (paged) num_pages > 0 with a page
 *    size of at least 16 tokens that divides the tile (128 tokens, 64 for
 *    head size 256) or is a multiple of it.  num_splits == 0 selects its
 *    balanced schedule (pieces cut by the device scheduler so that every SM
 *    gets the same work; needs `sched`); num_splits >= 1 keeps the
 *    reference's fixed partitions of partition_size tokens.  Paged head-128
 *    / 256 caches with 16- or 32-token pages, an even kv-head count and at
 *    most 32 query rows per kv head are served two adjacent kv heads per
 *    work entry (one TMA box over both heads' rows of a page).
 *  - the CUDA-core kernel for every other shape (num_splits >= 1).
 * With splits, partials go to part_o / part_lse and are merged in place
 * (part_lse f32; part_o f32 for the CUDA-core kernel, rows in the input type
 * for the tensor-core kernel).
 * fa_decode_workspace_size gives the bytes of part_o, part_lse and sched for
 * the kernel the arguments select (zero when nothing is split). */
typedef struct fa_decode_args {
  const void *q;
  int64_t q_stride_b, q_stride_h, q_stride_m;
  const void *k;
  const void *v;
  int64_t k_stride_seq, k_stride_tok, k_stride_head; /* same for v */
  const int32_t *block_table; /* [batch][bt_stride]; NULL = contiguous   */
  int64_t bt_stride;
  int32_t page_size; /* tokens per page (paged mode)                 */
  const int32_t *seq_lens; /* [batch] context lengths; NULL = all n_ctx */
  int32_t n_ctx;           /* contiguous length when seq_lens == NULL    */
  int32_t batch, num_q_heads, num_kv_heads, m_q, d_qk, d_v;
  int32_t causal;
  int32_t dtype;
  float scale;
  int32_t num_splits;     /* >= 1, or 0 = balanced (tensor-core kernel)   */
  int32_t partition_size; /* tokens per split; 0 = ceil-divide evenly    */
  void *o;
  int64_t o_stride_b, o_stride_h, o_stride_m;
  float *lse;
  float *part_o;
  float *part_lse;
  int32_t num_pages; /* paged: pages in k / v (the TMA bound); 0 = unknown,
                        which keeps the CUDA-core kernel                 */
  int32_t *sched;    /* int32 scheduler scratch (balanced schedule)      */
  int *status;       /* nullable device status word (kernel time-outs)   */
} fa_decode_args;

/* 1 when `args` run on the tensor-core kernel, 0 when on the CUDA-core one. */
int fa_decode_uses_tensor_cores(const fa_decode_args *args);
int fa_decode_workspace_size(const fa_decode_args *args, size_t *part_o_bytes,
                             size_t *part_lse_bytes, size_t *sched_bytes);
int fa_paged_attention(const fa_decode_args *args, void *stream);
int fa_split_kv_attention(const fa_decode_args *args, void *stream);

/* Merge `num_parts` partial results by log-sum-exp:
 *   lse = log(sum_s exp(lse_s)),  o = sum_s exp(lse_s - lse) * o_s
 * part_o: f32 [num_parts][rows][d_v] (row stride d_v), part_lse: f32
 * [num_parts][rows]; o: dtype [rows][d_v]; lse (nullable): f32 [rows].
 * d_v must be a multiple of 4 and at most 512. */
int fa_lse_combine(const float *part_o, const float *part_lse, int num_parts,
                   int64_t rows, int d_v, void *o, int dtype, float *lse,
                   void *stream);
/* fa_lse_combine with the partials at any distance from one another (in
 * f32 elements): partial p of row r has its O at part_o + p*o_part_stride +
 * r*d_v and its LSE at part_lse + p*lse_part_stride + r.  One buffer per
 * part holding [O rows | LSE rows] (o_part_stride == lse_part_stride ==
 * rows*(d_v+1), part_lse = part_o + rows*d_v) is what an all-gather of each
 * GPU's packed partial delivers (split_kv.py:198-228 merged across GPUs).
 * o_part_stride must be a multiple of 4 and at least rows*d_v. */
int fa_lse_combine_strided(const float *part_o, int64_t o_part_stride,
                           const float *part_lse, int64_t lse_part_stride,
                           int num_parts, int64_t rows, int d_v, void *o,
                           int dtype, float *lse, void *stream);

/* ---- MLA decode (tensor-core path) --------------------------------------
 * q      [batch][s_q][h_q][d_qk]   (q_stride_* in elements, last dim dense)
 * kcache paged:  [num_pages][page_size][1][d_qk], V = first d_v dims of the
 *        same rows;  contiguous (block_table == NULL): [batch][n_ctx][d_qk]
 *        with kv_stride_page == stride between sequences.
 * out    [batch][s_q][h_q][d_v] (dtype of q), lse f32 [batch][h_q][s_q].
 * Sparse mode (indices != NULL): indices int32 [batch][s_q][topk]; entry =
 * physical row page*page_size + offset of the cache viewed as
 * [num_pages*page_size][d_qk]; -1 (or any out-of-range entry) is masked.
 * Causal (dense only): query token i of s_q sees keys [0, len - s_q + i]. */
typedef struct fa_mla_args {
  const void *q;
  int64_t q_stride_b, q_stride_s, q_stride_h;
  const void *kcache;
  int64_t kv_stride_page, kv_stride_tok;
  int32_t num_pages, page_size;
  const int32_t *block_table;
  int64_t bt_stride;
  const int32_t *seq_lens;
  int32_t n_ctx;
  const int32_t *indices;
  int64_t idx_stride_b, idx_stride_s;
  int32_t topk;
  const int32_t *tile_meta;
  const int32_t *num_splits;
  int32_t num_sm_parts;
  void *out;
  int64_t o_stride_b, o_stride_s, o_stride_h;
  float *lse;
  float *part_o;   /* [batch + num_sm_parts][s_q*h_q][d_v] in the output
                      type (bf16 / f16 / f32); sized for f32 by
                      fa_mla_workspace_size                       */
  float *part_lse; /* f32 [batch + num_sm_parts][s_q*h_q]      */
  int32_t batch, s_q, h_q, d_qk, d_v;
  int32_t causal;
  int32_t dtype;     /* of q and kcache: FA_DTYPE_BF16 or FA_DTYPE_F16     */
  int32_t out_dtype; /* of out: dtype, or FA_DTYPE_F32 (partials that are
                        merged again, e.g. across GPUs)                    */
  float scale;
  int32_t *status; /* device int32 (nullable): nonzero after a bounded wait
                      inside the kernel gave up                             */
} fa_mla_args;

/* Number of 2-SM parts the scheduler should use on `device`: SMs / 2 / the
 * number of 128-row query blocks (dense: ceil(s_q*h_q/128); sparse: s_q, as
 * every query token has its own index list). */
int fa_mla_num_sm_parts(int device, int s_q, int h_q, int sparse, int *num_sm_parts);
int fa_mla_workspace_size(int batch, int s_q, int h_q, int d_v,
                          int num_sm_parts, size_t *part_o_bytes,
                          size_t *part_lse_bytes);
/* Device kernel: metadata for per-sequence lengths seq_lens[batch] (dense) or
 * the constant topk (sparse, when topk > 0 seq_lens may be NULL). */
int fa_mla_get_metadata(const int32_t *seq_lens, int batch, int topk,
                        int num_sm_parts, int32_t *tile_meta,
                        int32_t *num_splits, void *stream);
/* Decode kernel, then the combine kernel (queued as a programmatic
 * dependent of the decode: its launch overlaps the decode, and its blocks for
 * sequences that were not split exit before the decode ends). */
int fa_mla_decode(const fa_mla_args *args, void *stream);
/* Decode kernel only: sequences handled by one part are final in out / lse,
 * split sequences leave their partials in the workspace for fa_mla_combine. */
int fa_mla_decode_partial(const fa_mla_args *args, void *stream);
/* Combine only (the decode kernel's split partials -> out / lse). */
int fa_mla_combine(const fa_mla_args *args, void *stream);

/* ---- KV-page-sharded decode across GPUs (one process per GPU) -----------
 * The reference is single-GPU; these entry points carry its split merge
 * (split_kv.py:198-228) across GPUs with peer stores instead of a collective.
 * Each rank keeps a gather buffer, f32 [world][rows * (d_v + 1)] (part r:
 * O rows [rows][d_v] in (batch, token, head) order, then their LSEs), and
 * uint64 counters [world] (zero when allocated; counter r = rows delivered by
 * rank r, growing by `rows` per exchange, never reset).  dst_parts /
 * dst_counters are HOST arrays of `world` device addresses: this rank's
 * mappings of every rank's gather buffer / counters (its own included), e.g.
 * opened with fa_ipc_open.  Alternate two gather buffers between
 * consecutive exchanges: a rank may push exchange k + 1 while a slower peer
 * still merges exchange k (never k + 2, as its merge of k + 1 waits for that
 * peer's push of k + 1, issued after the peer's merge of k). */
#define FA_EXCHANGE_MAX_RANKS 8
#define FA_IPC_HANDLE_BYTES 64
/* CUDA IPC export of the allocation holding `ptr` (a cudaMalloc block):
 * writes the 64-byte handle and ptr's offset inside the block. */
int fa_ipc_export(const void *ptr, void *handle, uint64_t *offset);
/* Map a peer process's exported allocation into this process (peer access
 * enabled); *base is the block's start.  fa_ipc_close unmaps it. */
int fa_ipc_open(const void *handle, void **base);
int fa_ipc_close(void *base);
/* After fa_mla_decode_partial with out_dtype f32 (this rank's page range):
 * merge each sequence's split pieces and write every query row (O, LSE) into
 * slot `rank` of every rank's gather buffer, then add the rows delivered to
 * counter `rank` of every rank.  Launched as a programmatic dependent of the
 * decode.  paged.py:366-449 merge, fused with the exchange. */
int fa_mla_combine_push(const fa_mla_args *args, float *const *dst_parts,
                        unsigned long long *const *dst_counters, int world, int rank,
                        void *stream);
/* Wait until every counter holds `target` rows (k * rows after the k-th
 * exchange), at most timeout_ns, then merge the `world` parts of every row
 * (split_kv.py:198-228): out [rows][d_v] of dtype, lse f32 [rows].  On a
 * timeout nothing is written and *status (device int32) becomes
 * FA_DEVICE_TIMEOUT_EXCHANGE. */
#define FA_DEVICE_TIMEOUT_EXCHANGE 4
int fa_lse_merge_wait(const float *parts, int world, int64_t rows, int d_v,
                      const unsigned long long *counters, unsigned long long target, void *out,
                      int dtype, float *lse, int32_t *status, int64_t timeout_ns, void *stream);

/* fa_mla_combine_push and fa_lse_merge_wait in one cooperative launch (all
 * blocks resident): every block merges and pushes its share of the rows and
 * counts them, then waits (at most timeout_ns) for `target` rows from every
 * rank and merges its share of the gathered rows (this rank's gather buffer
 * and counters are dst_parts[rank] / dst_counters[rank]).  One launch after
 * the decode instead of two; on a timeout nothing is merged and *status is
 * FA_DEVICE_TIMEOUT_EXCHANGE. */
int fa_mla_combine_exchange(const fa_mla_args *args, float *const *dst_parts,
                            unsigned long long *const *dst_counters, int world, int rank,
                            unsigned long long target, void *out, int dtype, float *lse,
                            int32_t *status, int64_t timeout_ns, void *stream);

/* Write n latent rows (576 dims, bf16 / f16 as dtype; row r at
 * rows + r * rows_stride elements, unit inner stride) into the pool row
 * slots[r] = page * page_size + offset of kcache (layout as in fa_mla_args;
 * each pool row's 576 dims contiguous: unit inner stride).
 * A negative slot, or one at or past num_pages * page_size, skips its row.
 * Slots must be distinct (two rows aimed at one slot race).  rows / kcache
 * 16-byte aligned, slots (int64) 8-byte aligned, strides multiples of 8
 * elements.  Asynchronous on stream; n == 0 launches nothing. */
int fa_mla_append_rows(const void *rows, int64_t rows_stride, const int64_t *slots, int64_t n,
                       void *kcache, int64_t kv_stride_page, int64_t kv_stride_tok,
                       int32_t num_pages, int32_t page_size, int32_t dtype, void *stream);

/* No counterpart in the reference (the reference's Triton kernels have no
 * waits that can time out).  Self-test of the bounded wait inside every
 * kernel here: one warp waits on a barrier that nothing completes; after the
 * limit (about 2 s) the wait gives up and writes FA_DEVICE_TIMEOUT_SELFTEST
 * into *status (a device int32 the caller zeroed), and the kernel returns.
 * The CUDA context stays usable. */
#define FA_DEVICE_TIMEOUT_SELFTEST 7
int fa_selftest_wait_timeout(int32_t *status, void *stream);

/* No counterpart in the reference.  fa_mla_decode for callers that cannot
 * allocate device memory: serving engines that reserve nearly all of it for
 * their KV-cache pool up front, and plugin / FFI hosts that pass device
 * pointers but no allocator.  args->part_o / part_lse are ignored; the split
 * scratch comes from an array of FA_MLA_STATIC_WORKSPACE_BYTES that the
 * library defines in device memory (held by every GPU that loads it, until
 * exit).  Calls needing more ((batch + num_sm_parts) * s_q * h_q * (d_v + 1)
 * * 4 bytes, rounded) return FA_ERR_INVALID_ARGUMENT with the sizes in
 * fa_last_error().  All calls on a device share the array: calls that
 * overlap on the GPU race.  The first call in a CUDA context (once per
 * device, and again after cudaDeviceReset) resolves the array's address;
 * make it before capturing work into a stream. */
#define FA_MLA_STATIC_WORKSPACE_BYTES (48u << 20)
int fa_mla_decode_static_workspace(const fa_mla_args *args, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* FLAGATTN_B200_H_ */
