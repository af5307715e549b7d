// mla_tc.cu -- tensor-core (tcgen05 / TMEM / TMA) MLA decode for sm_100a,
// head-dim-split design.  Launched only for top-k decode over a latent pool
// whose pages are not back to back (page stride != page_size x token
// stride), where one TMA row map cannot address every row and key rows are
// copied row by row with cp.async instead.  Dense decode and top-k over
// ordinary pools run on the score / value kernel (mla_sv.cu).
//
// Problem: 128 query rows (query tokens x heads) share one latent key head of
// 576 dims; values are the first 512 dims of the same rows.  Per 64-token
// tile this is S = Q K^T (128 x 64 x 576) then O += P V (128 x 512 x 64): the
// reference computes it per page with tl.dot (paged.py:296-336).
//
// The f32 accumulator O[128 x 512] alone fills one SM's 512 TMEM columns, so
// a work unit runs on a 2-CTA cluster that splits the head dims:
//   rank 0: Q/K dims [0,256)   -> partial scores S0, output dims [0,256)
//   rank 1: Q/K dims [256,576) -> partial scores S1, output dims [256,512)
// Each CTA loads only its dims of every key row (so a row crosses HBM once),
// computes its partial scores on the tensor core, sends them to its peer with
// st.async (distributed shared memory) and adds the peer's partial: both CTAs
// then hold the same S = S0 + S1 (f32 addition commutes, so bit-identical),
// run the same online softmax and accumulate their half of O in TMEM.
// Precisely, rank r takes latent dims [256 r, 256 r + 256) and rope dims
// [512 + 32 r, 512 + 32 r + 32), so both ranks move 36 KB per 64-row tile.
//
// Resource plan (per CTA).  Shared memory is spent on key rows in flight:
//   TMEM   O [0,256) | Q latent half, bf16 pairs [256,384) | S [384,448)
//          | P0, P1 (bf16 pairs) [448,512)
//   smem   rope Q 8 KB | 4 KV stages x 36 KB | 2 score-exchange slots x 32 KB
// QK runs with A = Q from TMEM (16 MMAs) plus 2 MMAs with the rope part of Q
// from shared memory (64-byte swizzle); PV runs with A = P from TMEM.
//
// Warp roles (512 threads): warp 0 = TMA producer, warp 1 = TMEM owner and
// MMA issuer, warps 2-3 = key-row gatherers (sparse only), warps 4-11 =
// softmax / correction / epilogue (2 warps per 32 query rows, one per half of
// the tile's columns), warps 12-15 = query loaders (copy each piece's latent
// Q rows into TMEM).
// Every mbarrier wait is bounded (common.cuh); a timeout sets the device
// status word and the kernel unwinds instead of hanging.
#include "common.cuh"
#include "flagattn_b200.h"

namespace fa {

constexpr int kRows = 128;
constexpr int kBN = FA_MLA_BLOCK_N;                 // 64 key rows per tile
constexpr int kStages = 4;
constexpr int kThreads = 512;
constexpr int kSoftmaxThreads = 256;                // 8 warps: 2 column halves x 128 rows
constexpr int kChunkBytesRow = 128;                 // 64 dims x 2 bytes per swizzle row
constexpr int kLatentChunks = 4;                    // latent dims per CTA / 64
constexpr int kChunkBytes = kBN * kChunkBytesRow;   // 8 KB: 64 key rows x 64 dims
constexpr int kRopeDims = 32;                       // rope dims per CTA
constexpr int kRopeRowBytes = kRopeDims * 2;        // 64-byte swizzle rows
constexpr int kKvRopeBytes = kBN * kRopeRowBytes;   // 4 KB
constexpr int kStageBytes = kLatentChunks * kChunkBytes + kKvRopeBytes;  // 36 KB
constexpr int kQRopeBytes = kRows * kRopeRowBytes;  // 8 KB: 128 query rows x 32 rope dims
constexpr int kXBytes = kRows * kBN * 4;            // f32 partial scores of one tile
constexpr int kRedBytes = 2 * 2 * kRows * 4;        // row maxima of the column halves, 2 tiles
constexpr int kOffRope = 0;
constexpr int kOffKv = kOffRope + kQRopeBytes;
constexpr int kOffX = kOffKv + kStages * kStageBytes;
constexpr int kOffRed = kOffX + 2 * kXBytes;
constexpr int kOffBar = kOffRed + kRedBytes;
constexpr int kSmemUsed = kOffBar + 256;
constexpr int kSmemBytes = kSmemUsed + 1024;        // + base alignment slack
constexpr int kDvHalf = 256;                        // output dims per CTA
constexpr int kPvChunks = kDvHalf / 64;             // 4
constexpr int kLatentHalf = 256;                    // latent Q/K dims per CTA
constexpr uint32_t kColO = 0, kColQ = 256, kColS = 384, kColP = 448, kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;           // log2 units (factor 256)
static_assert(kSmemBytes <= 232448, "shared memory plan exceeds 227 KB");
static_assert(kOffKv % 1024 == 0 && kStageBytes % 1024 == 0 && kOffX % 1024 == 0,
              "swizzled operands need 1024-byte alignment");


#ifdef FA_TRACE
// Debug builds only: per-tile SM-clock timestamps of two parts (both ranks).
__device__ long long g_trace[2][2][64][16];
#define FA_TRACE_EV(slot, tile)                                                    \
  do {                                                                             \
    const int tp_ = (part == 0) ? 0 : (part == 37 ? 1 : -1);                       \
    if (tp_ >= 0 && (tile) < 64) g_trace[tp_][rank][(tile)][(slot)] = clock64();   \
  } while (0)
#else
#define FA_TRACE_EV(slot, tile) \
  do {                          \
  } while (0)
#endif

struct MlaBarriers {
  uint64_t q_full, q_empty;
  uint64_t kv_full[kStages], kv_empty[kStages];
  uint64_t s_full, s_empty;
  uint64_t p_full[2], pv_done[2];
  uint64_t x_full[2];
  uint64_t o_empty, drain;
  uint64_t pair[4];  // the two softmax warps that share 32 query rows
#ifdef FA_TRACE
  uint64_t dbg;
#endif
  uint32_t tmem_base;
  int abort_flag;
};

static_assert(sizeof(MlaBarriers) <= 256, "barrier block");

struct MlaParams {
  const uint16_t *q;       // query loaders read rows directly
  int64_t q_sb, q_ss, q_sh;
  const int32_t *block_table;
  int64_t bt_stride;
  const int32_t *seq_lens;
  int32_t n_ctx;
  const int32_t *indices;
  int64_t idx_sb, idx_ss;
  int32_t topk;
  const uint8_t *kcache;  // sparse gathers read rows directly
  int64_t kv_sp, kv_st;   // page / token strides in elements
  int32_t page_size;
  int64_t total_rows;     // num_pages * page_size (sparse index bound)
  const int32_t *tile_meta;
  const int32_t *num_splits;
  void *out;
  int64_t o_sb, o_ss, o_sh;
  float *lse;
  float *part_o;
  float *part_lse;
  int32_t batch, s_q, h_q, d_v;
  int32_t causal, paged, out_f32;
  float scale_log2;
  int32_t *status;
};

struct Piece {
  int b, tok0, tok_end, split_idx;
};

__device__ __forceinline__ Piece get_piece(const MlaParams &p, const int32_t *meta, int i,
                                           bool sparse) {
  Piece pc;
  pc.b = meta[0] + i;
  const int len = sparse ? p.topk : (p.seq_lens ? p.seq_lens[pc.b] : p.n_ctx);
  const int nblk = len > 0 ? (len + kBN - 1) / kBN : 0;
  const int lo = (i == 0) ? meta[1] : 0;
  const int hi = (pc.b == meta[2]) ? meta[3] : nblk;
  pc.tok0 = lo * kBN;
  pc.tok_end = min(hi * kBN, max(len, 0));
  pc.split_idx = (i == 0) ? meta[4] : 0;
  return pc;
}

// Walks the tiles of a part's pieces in order, skipping empty pieces.
// g counts tiles across pieces; qi counts the non-empty pieces started.
struct TileCursor {
  int piece, tok, tok0, tok_end, qi;
  uint32_t g;
  bool valid;

  __device__ __forceinline__ void seek(const MlaParams &p, const int32_t *meta, int n_pieces,
                                       bool sparse) {
    while (piece < n_pieces) {
      const Piece pc = get_piece(p, meta, piece, sparse);
      if (pc.tok_end > pc.tok0) {
        tok0 = tok = pc.tok0;
        tok_end = pc.tok_end;
        valid = true;
        return;
      }
      ++piece;
    }
    valid = false;
  }
  __device__ __forceinline__ void start(const MlaParams &p, const int32_t *meta, int n_pieces,
                                        bool sparse) {
    piece = 0;
    qi = 0;
    g = 0;
    seek(p, meta, n_pieces, sparse);
  }
  __device__ __forceinline__ void advance(const MlaParams &p, const int32_t *meta, int n_pieces,
                                          bool sparse) {
    tok += kBN;
    ++g;
    if (tok >= tok_end) {
      ++piece;
      ++qi;
      seek(p, meta, n_pieces, sparse);
    }
  }
};

template <typename T, bool kSparse>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    mla_decode_tc_kernel(const __grid_constant__ CUtensorMap q_rope_map,
                         const __grid_constant__ CUtensorMap kv_map,
                         const __grid_constant__ CUtensorMap kv_rope_map, const MlaParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  if (smem + kSmemUsed > smem_raw + kSmemBytes) {  // uniform over the cluster
    if (threadIdx.x == 0 && p.status) atomicExch(p.status, kDevBadSmemAlign);
    return;
  }
  MlaBarriers *bars = reinterpret_cast<MlaBarriers *>(smem + kOffBar);
  const uint32_t s_base = smem_u32(smem);
  const uint32_t rope_base = s_base + kOffRope;
  const uint32_t kv_base = s_base + kOffKv;
  const uint32_t x_base = s_base + kOffX;
  volatile int *abort_flag = &bars->abort_flag;

  const uint32_t rank = cluster_rank();
  const uint32_t peer = rank ^ 1u;
  const int part = blockIdx.x >> 1;
  const int mb = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int dim0 = static_cast<int>(rank) * kLatentHalf;        // latent dims of this CTA
  const int rope0 = 512 + static_cast<int>(rank) * kRopeDims;   // rope dims of this CTA
  const int32_t *meta = p.tile_meta + static_cast<int64_t>(part) * FA_MLA_META_INTS;
  const int n_pieces = meta[5];
  // query rows of this m-block: dense = 128 consecutive (s, h) rows; sparse =
  // the h_q heads of query token mb (index lists differ per query token).
  const int rows_total = p.s_q * p.h_q;
  const int row0 = kSparse ? mb * p.h_q : mb * kRows;
  const int n_rows = kSparse ? p.h_q : min(kRows, rows_total - row0);
  const int fmt = sizeof(T) == 2 && !std::is_same<T, __half>::value ? 1 : 0;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bars->q_full), 128 + 1);  // loaders + the rope TMA
    mbar_init(smem_u32(&bars->q_empty), 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&bars->kv_full[s]), kSparse ? 64 : 1);
      mbar_init(smem_u32(&bars->kv_empty[s]), 1);
    }
    mbar_init(smem_u32(&bars->s_full), 1);
    mbar_init(smem_u32(&bars->s_empty), kSoftmaxThreads);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&bars->p_full[i]), kSoftmaxThreads);
      mbar_init(smem_u32(&bars->pv_done[i]), 1);
      mbar_init(smem_u32(&bars->x_full[i]), 1);
    }
    mbar_init(smem_u32(&bars->o_empty), kSoftmaxThreads);
    mbar_init(smem_u32(&bars->drain), 1);
    for (int i = 0; i < 4; ++i) mbar_init(smem_u32(&bars->pair[i]), 64);
#ifdef FA_TRACE
    mbar_init(smem_u32(&bars->dbg), 1);
#endif
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&bars->tmem_base), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  cluster_sync();  // the peer's barriers exist before any remote access
  if (threadIdx.x == 0) FA_TRACE_EV(11, 0);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&q_rope_map);
      if (!kSparse) {
        tma_prefetch_desc(&kv_map);
        tma_prefetch_desc(&kv_rope_map);
      }
      uint32_t g = 0;
      int qi = 0;
      bool ok = true;
      for (int i = 0; i < n_pieces && ok; ++i) {
        const Piece pc = get_piece(p, meta, i, kSparse);
        if (pc.tok_end <= pc.tok0) continue;
        // rope part of Q -> shared memory
        ok = mbar_wait(smem_u32(&bars->q_empty), (qi & 1) ^ 1, abort_flag, p.status,
                       kDevTimeoutProducer);
        if (!ok) break;
        mbar_arrive_expect_tx(smem_u32(&bars->q_full), kQRopeBytes);
        tma_load_3d(rope_base, &q_rope_map, smem_u32(&bars->q_full), rope0, row0, pc.b);
        ++qi;
        if (kSparse) {
          g += (pc.tok_end - pc.tok0 + kBN - 1) / kBN;
          continue;
        }
        for (int tok = pc.tok0; tok < pc.tok_end; tok += kBN, ++g) {
          const int st = g % kStages;
          const uint32_t n = g / kStages;
          int c1, c2;
          if (p.paged) {
            c2 = p.block_table[static_cast<int64_t>(pc.b) * p.bt_stride + tok / p.page_size];
            c1 = tok % p.page_size;
          } else {
            c2 = pc.b;
            c1 = tok;
          }
          ok = mbar_wait(smem_u32(&bars->kv_empty[st]), (n & 1) ^ 1, abort_flag, p.status,
                         kDevTimeoutProducer);
          if (!ok) break;
          const uint32_t full = smem_u32(&bars->kv_full[st]);
          FA_TRACE_EV(0, g);
          mbar_arrive_expect_tx(full, kStageBytes);
          const uint32_t dst = kv_base + st * kStageBytes;
          for (int c = 0; c < kLatentChunks; ++c)
            tma_load_3d(dst + c * kChunkBytes, &kv_map, full, dim0 + 64 * c, c1, c2);
          tma_load_3d(dst + kLatentChunks * kChunkBytes, &kv_rope_map, full, rope0, c1, c2);
        }
      }
      // Drain: copies still in flight must land before the CTA may exit.
      if (*abort_flag) {
        volatile int never = 0;
        if (qi > 0) mbar_wait(smem_u32(&bars->q_full), (qi - 1) & 1, &never, nullptr, 0);
        for (uint32_t t = g > kStages ? g - kStages : 0; t < g; ++t)
          mbar_wait(smem_u32(&bars->kv_full[t % kStages]), (t / kStages) & 1, &never, nullptr, 0);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    // Two cursors walk the part's tiles: QK(g) may run ahead of PV; whichever
    // is ready is issued (PV first: it frees a KV stage for the producer).
    if (lane == 0) {
      const uint32_t idesc_qk = umma_idesc_f16(128, kBN, fmt, 0);
      const uint32_t idesc_pv = umma_idesc_f16(128, kDvHalf, fmt, 1);
      TileCursor cq, cp;
      cq.start(p, meta, n_pieces, kSparse);
      cp.start(p, meta, n_pieces, kSparse);
      long long t_last = 0;
      uint32_t idle = 0;
#ifdef FA_TRACE_MMA
      uint32_t dbg_n = 0;
#endif
      while (cp.valid) {
        bool did = false;
        if (cp.g < cq.g) {
          const uint32_t t = cp.g;
          const int st = t % kStages;
          const bool first = cp.tok == cp.tok0;
          const uint32_t ps = t & 1u;  // P slot in TMEM
          if (mbar_probe(smem_u32(&bars->p_full[ps]), (t >> 1) & 1) &&
              (!first || mbar_probe(smem_u32(&bars->o_empty), (cp.qi & 1) ^ 1))) {
            tc_fence_after();
            FA_TRACE_EV(2, t);
            const uint32_t vb = kv_base + st * kStageBytes;
#pragma unroll
            for (int kk = 0; kk < kBN / 16; ++kk) {
              const uint64_t bdesc = smem_desc_sw128(vb + kk * 16 * kChunkBytesRow, kChunkBytes, 1024);
              umma_ts(tmem + kColO, tmem + kColP + ps * (kBN / 2) + kk * 8, bdesc, idesc_pv,
                      (first && kk == 0) ? 0u : 1u);
            }
            tc_commit(smem_u32(&bars->kv_empty[st]));
            tc_commit(smem_u32(&bars->pv_done[ps]));
#ifdef FA_TRACE_MMA
            {  // debug: wait for this tile's PV to finish
              volatile int never = 0;
              tc_commit(smem_u32(&bars->dbg));
              mbar_wait(smem_u32(&bars->dbg), dbg_n & 1, &never, nullptr, 0);
              ++dbg_n;
              FA_TRACE_EV(13, t);
            }
#endif
            cp.advance(p, meta, n_pieces, kSparse);
            did = true;
          }
        }
        if (cq.valid) {
          const uint32_t g = cq.g;
          const int st = g % kStages;
          const bool first = cq.tok == cq.tok0;
          if ((!first || mbar_probe(smem_u32(&bars->q_full), cq.qi & 1)) &&
              mbar_probe(smem_u32(&bars->kv_full[st]), (g / kStages) & 1) &&
              mbar_probe(smem_u32(&bars->s_empty), (g & 1) ^ 1)) {
            if (kSparse) fence_proxy_async_smem();  // cp.async rows -> tensor-core reads
            tc_fence_after();
            FA_TRACE_EV(1, g);
            const uint32_t kb = kv_base + st * kStageBytes;
            const uint32_t sd = tmem + kColS;
#pragma unroll
            for (int c = 0; c < kLatentChunks; ++c) {
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                const uint64_t bdesc = smem_desc_sw128(kb + c * kChunkBytes + kk * 32, 16, 1024);
                umma_ts(sd, tmem + kColQ + (c * 4 + kk) * 8, bdesc, idesc_qk, (c | kk) ? 1u : 0u);
              }
            }
#pragma unroll
            for (int kk = 0; kk < kRopeDims / 16; ++kk) {
              const uint64_t adesc = smem_desc_sw64(rope_base + kk * 32, 16, 512);
              const uint64_t bdesc = smem_desc_sw64(kb + kLatentChunks * kChunkBytes + kk * 32, 16, 512);
              umma_ss(sd, adesc, bdesc, idesc_qk, 1u);
            }
            tc_commit(smem_u32(&bars->s_full));
            if (cq.tok + kBN >= cq.tok_end) tc_commit(smem_u32(&bars->q_empty));
#ifdef FA_TRACE_MMA
            {  // debug: wait for this tile's QK to finish
              volatile int never = 0;
              tc_commit(smem_u32(&bars->dbg));
              mbar_wait(smem_u32(&bars->dbg), dbg_n & 1, &never, nullptr, 0);
              ++dbg_n;
              FA_TRACE_EV(12, g);
            }
#endif
            cq.advance(p, meta, n_pieces, kSparse);
            did = true;
          }
        }
        if (did) {
          idle = 0;
          t_last = 0;
          continue;
        }
        // nothing ready: back off briefly so the polling does not take issue
        // slots from the softmax warps that share this SM sub-partition
        __nanosleep(32);
        if ((++idle & 63u) == 0) {
          if (*abort_flag) break;
          const long long now = clock64();
          if (t_last == 0) {
            t_last = now;
          } else if (now - t_last > kWaitLimitCycles) {
            *abort_flag = 1;
            if (p.status) atomicExch(p.status, kDevTimeoutMma);
            break;
          }
        }
      }
      // Make sure every issued MMA has finished before TMEM is released.
      tc_commit(smem_u32(&bars->drain));
      volatile int never = 0;
      mbar_wait(smem_u32(&bars->drain), 0, &never, p.status, kDevTimeoutDrain);
    }
    __syncwarp();
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------- sparse key-row gatherers
    if (kSparse) {
      const int gt = threadIdx.x - 64;  // 0..63
      uint32_t g = 0;
      bool ok = true;
      const int s_tok = mb;  // query token of this m-block
      for (int i = 0; i < n_pieces && ok; ++i) {
        const Piece pc = get_piece(p, meta, i, kSparse);
        if (pc.tok_end <= pc.tok0) continue;
        const int32_t *idx = p.indices + pc.b * p.idx_sb + s_tok * p.idx_ss;
        for (int tok = pc.tok0; tok < pc.tok_end; tok += kBN, ++g) {
          const int st = g % kStages;
          ok = mbar_wait(smem_u32(&bars->kv_empty[st]), ((g / kStages) & 1) ^ 1, abort_flag,
                         p.status, kDevTimeoutProducer);
          if (!ok) break;
          const uint32_t dst = kv_base + st * kStageBytes;
          // 16-byte units per key row: 4 latent chunks x 8 (128-byte swizzle
          // rows) then 4 rope units (64-byte swizzle rows)
          constexpr int units = kLatentChunks * 8 + kRopeRowBytes / 16;
          for (int k = gt; k < kBN * units; k += 64) {
            const int r = k / units;
            const int rem = k - r * units;
            const int pos = tok + r;
            int64_t row = -1;
            if (pos < pc.tok_end) row = idx[pos];
            const bool valid = row >= 0 && row < p.total_rows;
            int dim;
            uint32_t off_s;
            if (rem < kLatentChunks * 8) {
              const int c = rem >> 3, w = rem & 7;
              dim = dim0 + c * 64 + w * 8;
              off_s = c * kChunkBytes + r * kChunkBytesRow + ((w ^ (r & 7)) << 4);
            } else {
              const int w = rem - kLatentChunks * 8;
              dim = rope0 + w * 8;
              off_s = kLatentChunks * kChunkBytes + r * kRopeRowBytes + ((w ^ ((r >> 1) & 3)) << 4);
            }
            const uint8_t *src = p.kcache;
            if (valid) {
              const int64_t pg = row / p.page_size, off = row % p.page_size;
              src += (pg * p.kv_sp + off * p.kv_st + dim) * 2;
            }
            cp_async_16(dst + off_s, src, valid ? 16u : 0u);
          }
          cp_async_arrive(smem_u32(&bars->kv_full[st]));
        }
      }
      asm volatile("cp.async.wait_all;" ::: "memory");
    }
  } else if (warp >= 12) {
    // ------------------------------------------------------- query loaders
    // Thread t copies query row t's latent half (256 dims) into TMEM columns
    // [kColQ, kColQ + 128) as bf16/f16 pairs: the A operand of the QK MMAs.
    // The first half of the next piece's row is fetched into registers while
    // the current piece is in use.
    const int t = (warp & 3) * 32 + lane;
    const uint32_t trow = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const bool row_ok = t < n_rows;
    const int flat = row0 + t;
    const int s_tok = kSparse ? mb : (row_ok ? flat / p.h_q : 0);
    const int h = kSparse ? t : (row_ok ? flat % p.h_q : 0);
    uint32_t qr[kLatentHalf / 4];
    auto next_piece = [&](int from) {
      for (int j = from; j < n_pieces; ++j) {
        const Piece pc = get_piece(p, meta, j, kSparse);
        if (pc.tok_end > pc.tok0) return j;
      }
      return n_pieces;
    };
    auto fetch = [&](int j, int half) {  // dims [dim0 + 128 half, +128) -> qr
      const Piece pc = get_piece(p, meta, j, kSparse);
      const uint4 *src = reinterpret_cast<const uint4 *>(p.q + pc.b * p.q_sb + s_tok * p.q_ss +
                                                         h * p.q_sh + dim0 + half * 128);
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const uint4 v = row_ok ? __ldg(src + u) : make_uint4(0u, 0u, 0u, 0u);
        qr[4 * u] = v.x;
        qr[4 * u + 1] = v.y;
        qr[4 * u + 2] = v.z;
        qr[4 * u + 3] = v.w;
      }
    };
    auto store = [&](int half) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t w[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) w[j] = qr[c * 16 + j];
        tmem_st16(trow + kColQ + half * 64 + c * 16, w);
      }
    };
    int qi = 0;
    int i = next_piece(0);
    if (i < n_pieces) fetch(i, 0);
    while (i < n_pieces) {
      const bool ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars->q_empty), (qi & 1) ^ 1,
                                                        abort_flag, p.status, kDevTimeoutProducer));
      if (!ok) break;
      tc_fence_after();
      store(0);
      fetch(i, 1);
      store(1);
      tmem_wait_st();
      tc_fence_before();
      if (t == 0) FA_TRACE_EV(10, qi);
      mbar_arrive(smem_u32(&bars->q_full));
      ++qi;
      i = next_piece(i + 1);
      if (i < n_pieces) fetch(i, 0);
    }
  } else if (warp >= 4) {
    // ------------------------------------------ softmax / correction / out
    // 8 warps: warp w owns query rows 32 (w % 4) .. +31 (its TMEM lanes) and
    // score columns [32 ch, 32 ch + 32) of every tile, ch = (w - 4) / 4.  The
    // two warps of a row combine their row maxima through shared memory.
    // The score exchange runs one tile ahead of the softmax math: tile g+1's
    // partial scores travel to the peer while tile g's probabilities are
    // computed.
    const int ch = (warp - 4) >> 2;
    const int t = (warp & 3) * 32 + lane;  // query row within the m-block
    const int tt = ch * kRows + t;         // 0..255, splits shared work
    const int c0 = ch * (kBN / 2);         // first score column of this thread
    // bounded rendezvous of the two warps that share rows t (an mbarrier, so
    // an aborting partner cannot leave this warp waiting forever)
    const uint32_t pair_bar = smem_u32(&bars->pair[warp & 3]);
    uint32_t pair_uses = 0;
    auto pair_sync = [&]() -> bool {
      mbar_arrive(pair_bar);
      const bool r = __all_sync(0xffffffffu, mbar_wait(pair_bar, pair_uses & 1, abort_flag,
                                                       p.status, kDevTimeoutSoftmax));
      ++pair_uses;
      return r;
    };
    const uint32_t trow = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    float *red = reinterpret_cast<float *>(smem + kOffRed);  // [tile parity][ch][row]
    const int flat = row0 + t;
    const bool row_ok = t < n_rows;
    const int s_tok = kSparse ? mb : (row_ok ? flat / p.h_q : 0);
    const int h = kSparse ? t : (row_ok ? flat % p.h_q : 0);
    const int out_flat = s_tok * p.h_q + h;
    // Two exchange slots: tile gx travels through slot gx & 1.  A slot is
    // rewritten (tile gx + 2) only after the peer has received tile gx + 1
    // from this CTA, which this CTA sends after it has read tile gx from the
    // slot -- so the slots need no "free" handshake.
    const uint32_t x_remote = map_to_rank(x_base, peer);
    const uint32_t xf_local[2] = {smem_u32(&bars->x_full[0]), smem_u32(&bars->x_full[1])};
    const uint32_t xf_remote[2] = {map_to_rank(xf_local[0], peer), map_to_rank(xf_local[1], peer)};
    bool ok = true;

    // ---- score exchange, tile gx: own partial -> peer; peer's partial + own
    TileCursor cx;
    cx.start(p, meta, n_pieces, kSparse);
    float so[kBN / 2];  // own partial scores of tile cx.g (in flight)
    float sc[kBN / 2];  // full scores of the tile being processed
    auto x_begin = [&]() -> bool {
      const uint32_t gx = cx.g, xs = gx & 1u;
      if (t == 0 && ch == 0) FA_TRACE_EV(14, gx);
      if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&bars->s_full), gx & 1, abort_flag,
                                             p.status, kDevTimeoutSoftmax)))
        return false;
      if (t == 0 && ch == 0) FA_TRACE_EV(3, gx);
      tc_fence_after();
      {
        float v[16];
        tmem_ld16(trow + kColS + c0, v);
#pragma unroll
        for (int j = 0; j < 16; ++j) so[j] = v[j];
        tmem_ld16(trow + kColS + c0 + 16, v);
#pragma unroll
        for (int j = 0; j < 16; ++j) so[16 + j] = v[j];
      }
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(smem_u32(&bars->s_empty));
      if (t == 0 && ch == 0) {
        FA_TRACE_EV(4, gx);
        mbar_arrive_expect_tx(xf_local[xs], kXBytes);
      }
      const uint32_t dst = x_remote + xs * kXBytes;
#pragma unroll
      for (int c = 0; c < kBN / 8; ++c)
        st_async_v4(dst + ((ch * (kBN / 8) + c) * kRows + t) * 16, so[4 * c], so[4 * c + 1],
                    so[4 * c + 2], so[4 * c + 3], xf_remote[xs]);
      if (t == 0 && ch == 0) FA_TRACE_EV(5, gx);
      return true;
    };
    auto x_end = [&]() -> bool {
      const uint32_t gx = cx.g, xs = gx & 1u;
      if (!__all_sync(0xffffffffu, mbar_wait<true>(xf_local[xs], (gx >> 1) & 1, abort_flag,
                                                   p.status, kDevTimeoutExchange)))
        return false;
      if (t == 0 && ch == 0) FA_TRACE_EV(6, gx);
      const float4 *xr = reinterpret_cast<const float4 *>(smem + kOffX + xs * kXBytes);
#pragma unroll
      for (int c = 0; c < kBN / 8; ++c) {
        const float4 o = xr[(ch * (kBN / 8) + c) * kRows + t];
        sc[4 * c] = so[4 * c] + o.x;
        sc[4 * c + 1] = so[4 * c + 1] + o.y;
        sc[4 * c + 2] = so[4 * c + 2] + o.z;
        sc[4 * c + 3] = so[4 * c + 3] + o.w;
      }
      if (t == 0 && ch == 0) FA_TRACE_EV(15, gx);
      cx.advance(p, meta, n_pieces, kSparse);
      return true;
    };
    if (cx.valid) ok = x_begin() && x_end();

    uint32_t g = 0;
    int qi = 0;
    for (int i = 0; i < n_pieces && ok; ++i) {
      const Piece pc = get_piece(p, meta, i, kSparse);
      const int first_slot = p.num_splits[pc.b];
      const int n_split = p.num_splits[pc.b + 1] - first_slot;
      const int slot = first_slot + pc.split_idx;
      const int len = kSparse ? p.topk : (p.seq_lens ? p.seq_lens[pc.b] : p.n_ctx);
      const int row_len = (p.causal && !kSparse) ? len - (p.s_q - 1 - s_tok) : len;
      float m_run = -INFINITY, l_half = 0.f;
      const int32_t *idx = kSparse ? p.indices + pc.b * p.idx_sb + s_tok * p.idx_ss : nullptr;
      const bool has_tiles = pc.tok_end > pc.tok0;
      for (int tok = pc.tok0; tok < pc.tok_end && ok; tok += kBN, ++g) {
        const bool first = tok == pc.tok0;
        const bool more = cx.valid;  // tile g+1 exists
        if (more && !(ok = x_begin())) break;
        // mask: sparse rows by index, dense rows past the sequence / causal end
        if (kSparse) {
#pragma unroll
          for (int c = 0; c < kBN / 2; ++c) {
            const int pos = tok + c0 + c;
            const int64_t row = pos < pc.tok_end ? idx[pos] : -1;
            if (!(row >= 0 && row < p.total_rows)) sc[c] = -INFINITY;
          }
        } else if (tok + kBN > pc.tok_end || tok + kBN > row_len) {
          const int lim = min(pc.tok_end, row_len) - tok - c0;
#pragma unroll
          for (int c = 0; c < kBN / 2; ++c)
            if (c >= lim) sc[c] = -INFINITY;
        }
        float mx[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) mx[j] = sc[j];
#pragma unroll
        for (int c = 4; c < kBN / 2; c += 4) {
#pragma unroll
          for (int j = 0; j < 4; ++j) mx[j] = fmaxf(mx[j], sc[c + j]);
        }
        float mraw = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
        float *rslot = red + (g & 1u) * 2 * kRows;
        rslot[ch * kRows + t] = mraw;
        if (!(ok = pair_sync())) break;
        mraw = fmaxf(mraw, rslot[(ch ^ 1) * kRows + t]);
        // online softmax with a lazily updated running max (log2 units)
        const float mt = mraw * p.scale_log2;
        float alpha = 1.f;
        bool rescale = false;
        if (mt > -INFINITY && (m_run == -INFINITY || mt > m_run + kRescaleThreshold)) {
          alpha = (m_run == -INFINITY) ? 0.f : fast_exp2(m_run - mt);
          rescale = !first && m_run != -INFINITY;
          m_run = mt;
        }
        const float ms = (m_run == -INFINITY) ? 0.f : m_run;
        float ps[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t pk[kBN / 4];
#pragma unroll
        for (int c = 0; c < kBN / 2; c += 2) {
          const float p0 = fast_exp2(fmaf(sc[c], p.scale_log2, -ms));
          const float p1 = fast_exp2(fmaf(sc[c + 1], p.scale_log2, -ms));
          ps[(c >> 1) & 3] += p0 + p1;
          pk[c / 2] = Elem<T>::pack2(p0, p1);
        }
        l_half = l_half * alpha + ((ps[0] + ps[1]) + (ps[2] + ps[3]));
        if (t == 0 && ch == 0) FA_TRACE_EV(7, g);
        // P slot g & 1 is free once PV of tile g-2 has finished
        const uint32_t ps_slot = g & 1u;
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars->pv_done[ps_slot]),
                                               ((g >> 1) & 1) ^ 1, abort_flag, p.status,
                                               kDevTimeoutSoftmax));
        if (!ok) break;
        if (t == 0 && ch == 0) FA_TRACE_EV(8, g);
        if (__any_sync(0xffffffffu, rescale)) {
          // O may be rescaled once PV of tile g-1 (its last update) has finished
          const uint32_t pt = g - 1;
          ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars->pv_done[pt & 1u]),
                                                 (pt >> 1) & 1, abort_flag, p.status,
                                                 kDevTimeoutSoftmax));
          if (!ok) break;
          tc_fence_after();
          const float a = rescale ? alpha : 1.f;
#pragma unroll 1
          for (int c = 0; c < kDvHalf / 32; ++c) {
            const uint32_t col = kColO + ch * (kDvHalf / 2) + c * 16;
            float v[16];
            tmem_ld16(trow + col, v);
            tmem_wait_ld();
            uint32_t w[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) w[j] = __float_as_uint(v[j] * a);
            tmem_st16(trow + col, w);
          }
          tmem_wait_st();
        }
        // P row t, columns c0.. -> TMEM P slot as bf16/f16 pairs (PV's A operand)
        tmem_st16(trow + kColP + ps_slot * (kBN / 2) + ch * (kBN / 4), pk);
        const bool tail = !kSparse && pc.tok_end - tok < kBN;
        if (tail) {
          // rows past the sequence end may hold any bits (even NaN); P is 0
          // there but 0 * NaN is not, so clear them before the PV product.
          const int kv_valid = pc.tok_end - tok;
          const int units = (kBN - kv_valid) * kPvChunks * 8;
          uint8_t *stage = smem + kOffKv + (g % kStages) * kStageBytes;
          for (int u = tt; u < units; u += kSoftmaxThreads) {
            const int r = kv_valid + u / (kPvChunks * 8);
            const int rem = u % (kPvChunks * 8);
            *reinterpret_cast<uint4 *>(stage + (rem >> 3) * kChunkBytes + r * kChunkBytesRow +
                                       (rem & 7) * 16) = make_uint4(0u, 0u, 0u, 0u);
          }
          fence_proxy_async_smem();
        }
        tmem_wait_st();
        tc_fence_before();
        if (t == 0 && ch == 0) FA_TRACE_EV(9, g);
        mbar_arrive(smem_u32(&bars->p_full[ps_slot]));
        if (more && !(ok = x_end())) break;
      }
      if (!ok) break;
      // -------------------------------------------------------- epilogue
      // row sum = both column halves' sums (through the parity slot of the
      // last tile, once the partner has read that tile's maximum)
      float l_run = l_half;
      if (has_tiles) {
        float *rslot = red + ((g - 1) & 1u) * 2 * kRows;
        if (!(ok = pair_sync())) break;
        rslot[ch * kRows + t] = l_half;
        if (!(ok = pair_sync())) break;
        l_run = l_half + rslot[(ch ^ 1) * kRows + t];
      }
      const bool final_out = n_split == 1;
      const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
      const float ms = (m_run == -INFINITY) ? 0.f : m_run;
      const float lse = l_run > 0.f ? ms * 0.69314718055994531f + logf(l_run) : -INFINITY;
      if (has_tiles) {
        const uint32_t lt = g - 1;
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars->pv_done[lt & 1u]), (lt >> 1) & 1,
                                               abort_flag, p.status, kDevTimeoutSoftmax));
        if (!ok) break;
        tc_fence_after();
      }
#pragma unroll 1
      for (int c = 0; c < kDvHalf / 32; ++c) {
        const int col = ch * (kDvHalf / 2) + c * 16;
        float v[16];
        if (has_tiles) {
          tmem_ld16(trow + kColO + col, v);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = 0.f;
        }
        if (!row_ok) continue;
        const int d = static_cast<int>(rank) * kDvHalf + col;
        if (final_out && p.out_f32) {
          float4 *o = reinterpret_cast<float4 *>(static_cast<float *>(p.out) + pc.b * p.o_sb +
                                                 s_tok * p.o_ss + h * p.o_sh + d);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            o[j] = make_float4(v[4 * j] * inv_l, v[4 * j + 1] * inv_l, v[4 * j + 2] * inv_l,
                               v[4 * j + 3] * inv_l);
        } else if (final_out) {
          T *o = static_cast<T *>(p.out) + pc.b * p.o_sb + s_tok * p.o_ss + h * p.o_sh + d;
          uint4 w0, w1;
          w0.x = Elem<T>::pack2(v[0] * inv_l, v[1] * inv_l);
          w0.y = Elem<T>::pack2(v[2] * inv_l, v[3] * inv_l);
          w0.z = Elem<T>::pack2(v[4] * inv_l, v[5] * inv_l);
          w0.w = Elem<T>::pack2(v[6] * inv_l, v[7] * inv_l);
          w1.x = Elem<T>::pack2(v[8] * inv_l, v[9] * inv_l);
          w1.y = Elem<T>::pack2(v[10] * inv_l, v[11] * inv_l);
          w1.z = Elem<T>::pack2(v[12] * inv_l, v[13] * inv_l);
          w1.w = Elem<T>::pack2(v[14] * inv_l, v[15] * inv_l);
          reinterpret_cast<uint4 *>(o)[0] = w0;
          reinterpret_cast<uint4 *>(o)[1] = w1;
        } else {
          float4 *o = reinterpret_cast<float4 *>(
              p.part_o + (static_cast<int64_t>(slot) * rows_total + out_flat) * p.d_v + d);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            o[j] = make_float4(v[4 * j] * inv_l, v[4 * j + 1] * inv_l, v[4 * j + 2] * inv_l,
                               v[4 * j + 3] * inv_l);
        }
      }
      if (has_tiles) {
        tc_fence_before();
        mbar_arrive(smem_u32(&bars->o_empty));
        ++qi;
      }
      if (rank == 0 && ch == 0 && row_ok) {
        if (final_out)
          p.lse[(static_cast<int64_t>(pc.b) * p.h_q + h) * p.s_q + s_tok] = lse;
        else
          p.part_lse[static_cast<int64_t>(slot) * rows_total + out_flat] = lse;
      }
    }
  }

  // -------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) FA_TRACE_EV(11, 1);
  cluster_sync();  // the peer no longer touches this CTA's shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <typename T, bool kSparse>
static cudaError_t launch_mla_t(const CUtensorMap &qrm, const CUtensorMap &km, const CUtensorMap &krm,
                                const MlaParams &p, int num_parts, int m_blocks, cudaStream_t stream) {
  auto kern = mla_decode_tc_kernel<T, kSparse>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return e;
  dim3 grid(2 * num_parts, m_blocks);
  kern<<<grid, kThreads, kSmemBytes, stream>>>(qrm, km, krm, p);
  return cudaGetLastError();
}

// qrm: query rope map (box 32 dims x 128 rows, 64-byte swizzle); km / krm:
// key latent map (box 64 x 64, 128-byte swizzle) and key rope map (box 32 x
// 64, 64-byte swizzle) over the same cache.
cudaError_t launch_mla_tc(const CUtensorMap &qrm, const CUtensorMap &km, const CUtensorMap &krm,
                          const fa_mla_args *a, int m_blocks, int64_t total_rows,
                          cudaStream_t stream) {
  MlaParams p;
  p.q = static_cast<const uint16_t *>(a->q);
  p.q_sb = a->q_stride_b;
  p.q_ss = a->q_stride_s;
  p.q_sh = a->q_stride_h;
  p.block_table = a->block_table;
  p.bt_stride = a->bt_stride;
  p.seq_lens = a->seq_lens;
  p.n_ctx = a->n_ctx;
  p.indices = a->indices;
  p.idx_sb = a->idx_stride_b;
  p.idx_ss = a->idx_stride_s;
  p.topk = a->topk;
  p.kcache = static_cast<const uint8_t *>(a->kcache);
  p.kv_sp = a->kv_stride_page;
  p.kv_st = a->kv_stride_tok;
  p.page_size = a->page_size;
  p.total_rows = total_rows;
  p.tile_meta = a->tile_meta;
  p.num_splits = a->num_splits;
  p.out = a->out;
  p.o_sb = a->o_stride_b;
  p.o_ss = a->o_stride_s;
  p.o_sh = a->o_stride_h;
  p.lse = a->lse;
  p.part_o = a->part_o;
  p.part_lse = a->part_lse;
  p.batch = a->batch;
  p.s_q = a->s_q;
  p.h_q = a->h_q;
  p.d_v = a->d_v;
  p.causal = a->causal;
  p.paged = a->block_table != nullptr;
  p.out_f32 = a->out_dtype == FA_DTYPE_F32;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  p.status = a->status;
  // Only the top-k instance is launched (dense decode and top-k over
  // back-to-back pools run on the score / value kernel, mla_sv.cu).
  if (a->indices == nullptr) return cudaErrorInvalidValue;
  if (a->dtype == FA_DTYPE_F16)
    return launch_mla_t<__half, true>(qrm, km, krm, p, a->num_sm_parts, m_blocks, stream);
  return launch_mla_t<__nv_bfloat16, true>(qrm, km, krm, p, a->num_sm_parts, m_blocks, stream);
}

#ifdef FA_TRACE
extern "C" int fa_debug_trace_read(void *dst, size_t bytes) {
  return cudaMemcpyFromSymbol(dst, g_trace, bytes < sizeof(g_trace) ? bytes : sizeof(g_trace)) ==
                 cudaSuccess ? 0 : -1;
}
#endif

}  // namespace fa
