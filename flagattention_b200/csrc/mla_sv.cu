// mla_sv.cu -- MLA decode (dense paged and top-k) on tcgen05 with a score CTA
// and a value CTA.
//
// Problem: 128 query rows (query tokens x heads) share one latent key head of
// 576 dims; values are the first 512 dims of the same rows.  The reference
// computes it per page with tl.dot (paged.py:296-336): S = Q K^T, online
// softmax, O += P V.
//
// The f32 accumulator O[128 x 512] alone fills one SM's 512 TMEM columns, so
// a work unit runs on a 2-CTA cluster with a functional split:
//   rank 0, the score CTA: latent Q (512 dims) in TMEM as the A operand, two
//     128-column score buffers, S = Q K^T for 128-token tiles (N = 128), the
//     online softmax, and P sent as bf16/f16 into the value CTA's shared
//     memory as one bulk DSMEM copy per 64 tokens (one direction);
//   rank 1, the value CTA: O in all 512 TMEM columns, O += P V with P and V
//     from shared memory.
// Both CTAs read the key rows they need with their own TMA: the value CTA's
// 512 dims of a row are an L2 hit after the score CTA's 576, so HBM sees each
// row about once.  Nothing travels back from the value CTA except "slot free"
// arrivals (tcgen05.commit multicast).
//
// Score CTA (512 threads): warp 0 TMA producer (latent Q chunks and key
// chunks through one 9-slot ring of 16 KB = 128 rows x 64 dims, rope Q in two
// 16 KB buffers; it also gates each tile on its S buffer's release), warp 1
// MMA issuer (also copies the latent Q chunks from the ring into TMEM with
// tcgen05.cp), warps 4-11 softmax (two warps per 32 query rows, one per
// 64-token block of the tile).
// Value CTA (512 threads): warp 0 TMA producer (V in 32-token stages of
// 8 chunks x 4 KB, one TMA box per stage), warp 1 MMA issuer, warps 4-11 O rescaling, tail clearing and the
// epilogue (two warps per 32 rows, one per 256 output dims; stores staged
// through shared memory so that each store instruction writes whole rows).
// Top-k instance (kSparse): rows come from index lists with tile::gather4,
// issued by seven warps per CTA (0, 2, 3, 12-15); see the producer comments.
// Every mbarrier wait is bounded (common.cuh); a timeout sets the device
// status word and the kernel unwinds instead of hanging.
#include "common.cuh"
#include "flagattn_b200.h"

namespace fa {
namespace sv {

constexpr int kRows = 128;
constexpr int kGatherWarps = 7;                    // sparse: warps 0, 2, 3, 12-15 gather rows
constexpr int kBlk = FA_MLA_BLOCK_N;                 // 64 tokens: scheduler block, one page box
constexpr int kThreads = 512;
constexpr int kRowBytes = 128;                      // 64 dims x 2 bytes (one 128-byte swizzle row)
constexpr int kBoxBytes = kBlk * kRowBytes;         // 8 KB
constexpr int kChunkBytes = 2 * kBoxBytes;          // 16 KB: 128 rows x 64 dims
constexpr int kQChunks = 8;                         // latent Q, 512 dims
constexpr int kKChunks = 9;                         // key: 512 latent + 64 rope dims
constexpr int kRing = 9;
constexpr int kVRows = 32;                          // tokens per V stage
constexpr int kVChunkBytes = kVRows * kRowBytes;    // 4 KB: 32 rows x 64 dims
constexpr int kVStageBytes = 8 * kVChunkBytes;      // 32 KB: 512 dims
constexpr int kVStages = 3;
constexpr int kPBytes = kRows * kRowBytes;          // 16 KB: P of one 64-token block
constexpr int kMetaAlpha = kPBytes;                 // f32[128] O rescale factors
constexpr int kMetaFlags = kPBytes + 512;           // int[4] "rows of quadrant q rescale"
constexpr int kMetaInvL = kPBytes + 1024;           // f32[128] 1 / row sum (last block)
constexpr int kMetaLse = kPBytes + 1536;            // f32[128] LSE of the piece (last block)
constexpr int kPSlotBytes = kPBytes + 2048;         // 18 KB
constexpr int kPSlots = 4;
constexpr uint32_t kColQ = 0, kColS = 256, kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;           // log2 units (factor 256)
#ifdef FA_DEBUG_ABORT_TEST
constexpr uint32_t kAbortTestBlock = 6;             // P block whose m_read arrival is lost
#endif

constexpr int kOffBar = 0;
constexpr int kOffData = 1024;
// score CTA
constexpr int kOffQRope = kOffData;                         // 2 x 16 KB
constexpr int kOffRing = kOffQRope + 2 * kChunkBytes;       // 9 x 16 KB
constexpr int kOffRed = kOffRing + kRing * kChunkBytes;     // 2 KB row maxima / sums
constexpr int kOffStgP = kOffRed + 2048;                    // 2 x 18 KB P + metadata staging
constexpr int kSmemScore = kOffStgP + 2 * kPSlotBytes;
// value CTA
constexpr int kOffV = kOffData;                             // 3 x 32 KB
constexpr int kOffP = kOffV + kVStages * kVStageBytes;      // 4 x 18 KB
constexpr int kStageWarpBytes = 32 * 128;                   // epilogue staging per warp
constexpr int kOffStage = kOffP + kPSlots * kPSlotBytes;    // 8 x 4 KB
constexpr int kSmemValue = kOffStage + 8 * kStageWarpBytes;
constexpr int kSmemUsed = kSmemScore > kSmemValue ? kSmemScore : kSmemValue;
constexpr int kSmemBytes = kSmemUsed + 1024;                // + base alignment slack
static_assert(kSmemBytes <= 232448, "shared memory plan exceeds 227 KB");
static_assert(kOffRing % 1024 == 0 && kOffQRope % 1024 == 0 && kOffV % 1024 == 0 &&
                  kOffStgP % 1024 == 0 &&
                  kOffP % 1024 == 0 && kPSlotBytes % 1024 == 0,
              "swizzled operands need 1024-byte alignment");

// One block of barriers at the same offset in both CTAs, so a barrier of the
// peer is addressed by mapping the local offset (mapa / commit multicast).
struct Bars {
  // score CTA
  uint64_t rope_full[2], rope_empty[2];
  uint64_t ch_full[kRing], ch_empty[kRing];
  uint64_t s_full[2], s_empty[2];
  uint64_t pair[4];
  uint64_t stg_ready[2];     // the 128 rows of a P block are staged (one per block half)
  uint64_t p_free[kPSlots];  // arrived by the value CTA's PV commit
  // value CTA
  uint64_t v_full[kVStages], v_empty[kVStages];
  uint64_t p_full[kPSlots];  // the score CTA's st.async complete here
  uint64_t m_read[kPSlots];  // epilogue warps are done with the slot's metadata
  uint64_t pv_done[kPSlots];
  uint64_t o_empty;
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  // teardown accounting of the P transfers (see the teardown): score CTA, the
  // last block sent into each value slot (-1: none); value CTA, the same
  // numbers received from the score CTA, and the blocks its PV issuer armed /
  // saw land
  int sent_seq[kPSlots];
  int peer_sent[kPSlots];
  int armed_upto, done_upto;
  // sparse: per tile (g % 4), one byte per 4-row group with the invalid-index
  // bits of its key rows (row 4 group + j: bit j)
  alignas(16) uint8_t inval[4][32];
};
static_assert(sizeof(Bars) <= kOffData, "barrier block");

struct Params {
  const uint8_t *kcache;
  int64_t kv_sp, kv_st;   // page / token strides in elements
  const int32_t *block_table;
  int64_t bt_stride;
  const int32_t *seq_lens;
  int32_t n_ctx;
  int32_t page_size;
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
  // top-k sparse decode: indices[b][s][topk] are global pool rows
  // (page * page_size + offset); an index outside [0, total_rows) is masked
  const int32_t *indices;
  int64_t idx_sb, idx_ss;
  int32_t topk;  // 0: dense
  int64_t total_rows;
  int32_t uniform_rows;  // sparse: pool rows at one stride (2-D gather map)
};

struct Piece {
  int b, tok0, tok_end, split_idx;
};

// Length of sequence b's key list: its context (dense) or topk (sparse, the
// positions of its index list).
__device__ __forceinline__ int seq_len(const Params &p, int b) {
  return p.topk ? p.topk : (p.seq_lens ? p.seq_lens[b] : p.n_ctx);
}

// Piece i of a part (tile_meta row: begin batch, begin block, end batch, end
// block, split index of the first piece, number of pieces).  Out of line:
// every role walks the pieces, once per piece.
__device__ __noinline__ Piece get_piece_at(const int32_t *seq_lens, int n_ctx,
                                           const int32_t *meta, int i) {
  Piece pc;
  pc.b = meta[0] + i;
  const int len = seq_lens ? seq_lens[pc.b] : n_ctx;
  const int nblk = len > 0 ? (len + kBlk - 1) / kBlk : 0;
  const int lo = (i == 0) ? meta[1] : 0;
  const int hi = (pc.b == meta[2]) ? meta[3] : nblk;
  pc.tok0 = lo * kBlk;
  pc.tok_end = min(hi * kBlk, max(len, 0));
  pc.split_idx = (i == 0) ? meta[4] : 0;
  return pc;
}
__device__ __forceinline__ Piece get_piece(const Params &p, const int32_t *meta, int i) {
  return p.topk ? get_piece_at(nullptr, p.topk, meta, i) : get_piece_at(p.seq_lens, p.n_ctx, meta, i);
}

// Sparse: pool rows of index-list positions pos .. pos + 3 (-1 past `end`).
__device__ __forceinline__ void load_rows4(const int32_t *idx, int pos, int end, int (&r)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) r[j] = (pos + j < end) ? __ldg(idx + pos + j) : -1;
}

// Sparse: the first in-range pool row of a query token's index list (-1 when
// it has none), found by the whole warp 32 positions at a time.
__device__ __noinline__ int first_valid_row(const int32_t *idx, int topk, int64_t total_rows) {
  const int lane = threadIdx.x & 31;
  for (int base = 0; base < topk; base += 32) {
    const int r = base + lane < topk ? __ldg(idx + base + lane) : -1;
    const unsigned ok = __ballot_sync(0xffffffffu, r >= 0 && r < total_rows);
    if (ok) return __shfl_sync(0xffffffffu, r, __ffs(ok) - 1);
  }
  return -1;
}

// Sparse: this lane's invalid-row bits (row j invalid: bit j), with every
// invalid row replaced by `fallback`, a valid row of the same index list: the
// softmax masks the column and the value product adds 0 times a row the list
// attends anyway (finite unless the reference's own result is NaN).  A list
// with no valid row (fallback -1) reads pool row 0, whatever it holds: every
// weight is 0 there and the epilogue writes zeros for a row sum of 0.
__device__ __forceinline__ uint32_t fix_rows4(int (&r)[4], int64_t total_rows, int fallback) {
  uint32_t bad = 0;
  const int sub = fallback >= 0 ? fallback : 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (r[j] < 0 || r[j] >= total_rows) {
      bad |= 1u << j;
      r[j] = sub;
    }
  }
  return bad;
}

// Sparse: fetch 64 dims (from c0) of the four pool rows r[0..3] into four
// consecutive 128-byte rows at dst.  Pools whose rows all lie at one stride
// take one tile::gather4 over the 2-D row map; other pools (page stride !=
// page_size x token stride) take four one-row boxes of the 3-D page map.
__device__ __forceinline__ void gather_rows4(uint32_t dst, const CUtensorMap *map, uint32_t bar,
                                             int c0, const int (&r)[4], bool uniform,
                                             int page_size) {
  if (uniform) {
    tma_gather4(dst, map, bar, c0, r[0], r[1], r[2], r[3]);
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      tma_load_3d(dst + j * kRowBytes, map, bar, c0, r[j] % page_size, r[j] / page_size);
  }
}

// TMA coordinates (row in page, page) of token t of sequence b.
__device__ __forceinline__ void kv_coord(const Params &p, int b, int t, int &c1, int &c2) {
  if (p.paged) {
    c2 = __ldg(p.block_table + static_cast<int64_t>(b) * p.bt_stride + t / p.page_size);
    c1 = t % p.page_size;
  } else {
    c2 = b;
    c1 = t;
  }
}

// Position in a ring of kRing slots: slot index and the parity of its phase.
struct RingPos {
  uint32_t slot = 0, phase = 0;
  __device__ __forceinline__ void next() {
    if (++slot == kRing) {
      slot = 0;
      phase ^= 1u;
    }
  }
};


// ---------------------------------------------------------------------------
// Cold paths, kept out of line.  The kernel holds every role of both CTAs
// in one function; code that runs once per piece (or rarely) would otherwise
// share the instruction cache with the per-tile loops of the warps next to it.

// O[row, 256 ch + 0 .. 256) *= a for the calling warp's 32 rows (O rescale
// after the running max grew).
__device__ __noinline__ void rescale_o_half(uint32_t trow_col0, float a) {
#pragma unroll 1
  for (int c = 0; c < 8; ++c) {
    const uint32_t col = trow_col0 + c * 32;
    float v[32];
    tmem_ld32(col, v);
    tmem_wait_ld();
    uint32_t w0[16], w1[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      w0[j] = __float_as_uint(v[j] * a);
      w1[j] = __float_as_uint(v[16 + j] * a);
    }
    tmem_st16(col, w0);
    tmem_st16(col + 16, w1);
  }
  tmem_wait_st();
}

// Zero rows [lo, kVRows) of a V stage (all 8 chunks); 256 threads, index tt.
__device__ __noinline__ void clear_v_rows(uint8_t *stage, int lo, int tt) {
  const int units = (kVRows - lo) * 64;  // 8 chunks x 8 16-byte units per row
  for (int u = tt; u < units; u += 256) {
    const int r = lo + (u >> 6);
    const int rem = u & 63;
    *reinterpret_cast<uint4 *>(stage + (rem >> 3) * kVChunkBytes + r * kRowBytes + (rem & 7) * 16) =
        make_uint4(0u, 0u, 0u, 0u);
  }
}

// Epilogue of one piece for the calling warp: rows q4 * 32 .. +31 of the
// query block, output dims [256 ch, 256 ch + 256): O / l from TMEM (zeros when
// the piece had no keys) to `obase`.  Each warp stages 32 rows x 128 bytes in
// shared memory (16-byte units XOR-swizzled by row) and writes them back
// four whole rows per store instruction.  row_base(r) is the byte offset of
// flat query row r, or -1 when the row is absent.
struct OutRows {
  uint8_t *base;
  int64_t sb, ss, sh;  // final output strides (elements); split: row stride
  int b, h_q, row0, n_rows;
  int esz;             // bytes per element (output type; split rows use it too)
  bool split;          // split workspace row (slot * rows_total + flat) * d_v
  int64_t split_row0;  // slot * rows_total
  int d_v;
};

template <typename T>
__device__ __noinline__ void write_o_half(uint32_t trow, int ch, int q4, int lane, uint32_t stg_s,
                                          bool has_tiles, float inv_l, const OutRows o) {
  int64_t row_off[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int tr = q4 * 32 + 4 * k + (lane >> 3);
    const int fl = o.row0 + tr;
    if (tr >= o.n_rows) {
      row_off[k] = -1;
    } else if (!o.split) {
      const int st_ = fl / o.h_q, hh = fl % o.h_q;
      row_off[k] = (o.b * o.sb + st_ * o.ss + hh * o.sh) * o.esz;
    } else {
      row_off[k] = (o.split_row0 + fl) * o.d_v * o.esz;
    }
  }
  const int cols_it = 128 / o.esz;  // output dims per 128-byte row segment
  // A row whose sum is 0 attended no key (every column masked): its output
  // is 0, written as such rather than as O * 0 (the masked value rows of a
  // top-k list with no valid index are arbitrary pool bytes, possibly NaN).
  const bool zero_row = !has_tiles || inv_l == 0.f;
#pragma unroll 1
  for (int c0 = 0; c0 < 256; c0 += cols_it) {
    const int col = ch * 256 + c0;
    uint32_t w[32];
    if (o.esz == 4) {
      float v[32];
      if (has_tiles) {
        tmem_ld32(trow + col, v);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) w[j] = __float_as_uint(zero_row ? 0.f : v[j] * inv_l);
    } else {
      float v0[32], v1[32];
      if (has_tiles) {
        tmem_ld32(trow + col, v0);
        tmem_ld32(trow + col + 32, v1);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v0[j] = v1[j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        w[j] = zero_row ? 0u : Elem<T>::pack2(v0[2 * j] * inv_l, v0[2 * j + 1] * inv_l);
        w[16 + j] = zero_row ? 0u : Elem<T>::pack2(v1[2 * j] * inv_l, v1[2 * j + 1] * inv_l);
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u)
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(
                       stg_s + lane * 128 + ((u ^ (lane & 7)) << 4)),
                   "r"(w[4 * u]), "r"(w[4 * u + 1]), "r"(w[4 * u + 2]), "r"(w[4 * u + 3])
                   : "memory");
    __syncwarp();
    const int j = lane & 7;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int r = 4 * k + (lane >> 3);
      uint4 val;
      asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(val.x), "=r"(val.y), "=r"(val.z), "=r"(val.w)
                   : "r"(stg_s + r * 128 + ((j ^ (r & 7)) << 4))
                   : "memory");
      if (row_off[k] >= 0)
        *reinterpret_cast<uint4 *>(o.base + row_off[k] + static_cast<int64_t>(col) * o.esz + j * 16) = val;
    }
    __syncwarp();
  }
}

template <typename T, bool kSparse>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    mla_decode_sv_kernel(const __grid_constant__ CUtensorMap q_map,
                         const __grid_constant__ CUtensorMap kv_map,
                         const __grid_constant__ CUtensorMap v_map,
                         const __grid_constant__ CUtensorMap g_map, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  if (smem + kSmemUsed > smem_raw + kSmemBytes) {  // uniform over the cluster
    if (threadIdx.x == 0 && p.status) atomicExch(p.status, kDevBadSmemAlign);
    return;
  }
  Bars *bars = reinterpret_cast<Bars *>(smem + kOffBar);
  const uint32_t s_base = smem_u32(smem);
  volatile int *abort_flag = &bars->abort_flag;
  const uint32_t rank = cluster_rank();
  const int part = blockIdx.x >> 1;
  const int mb = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int32_t *meta = p.tile_meta + static_cast<int64_t>(part) * FA_MLA_META_INTS;
  const int n_pieces = meta[5];
  const int rows_total = p.s_q * p.h_q;
  // dense: 128 consecutive (s, h) rows; sparse: the h_q rows of query token
  // mb (each token has its own index list)
  const int row0 = kSparse ? mb * p.h_q : mb * kRows;
  const int n_rows = kSparse ? p.h_q : min(kRows, rows_total - row0);
  constexpr int fmt = std::is_same<T, __half>::value ? 0 : 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&bars->rope_full[i]), 1);
      mbar_init(smem_u32(&bars->rope_empty[i]), 1);
      mbar_init(smem_u32(&bars->s_full[i]), 1);
      mbar_init(smem_u32(&bars->s_empty[i]), 256);
    }
    for (int i = 0; i < kRing; ++i) {
      mbar_init(smem_u32(&bars->ch_full[i]), 1);
      mbar_init(smem_u32(&bars->ch_empty[i]), 1);
    }
    for (int i = 0; i < 4; ++i) mbar_init(smem_u32(&bars->pair[i]), 64);
    for (int i = 0; i < 2; ++i) mbar_init(smem_u32(&bars->stg_ready[i]), 128);
    for (int i = 0; i < kPSlots; ++i) {
      mbar_init(smem_u32(&bars->p_free[i]), 1);
      mbar_init(smem_u32(&bars->p_full[i]), 1);
      mbar_init(smem_u32(&bars->m_read[i]), 256);
      mbar_init(smem_u32(&bars->pv_done[i]), 1);
    }
    for (int i = 0; i < kVStages; ++i) {
      mbar_init(smem_u32(&bars->v_full[i]), 1);
      mbar_init(smem_u32(&bars->v_empty[i]), 1);
    }
    mbar_init(smem_u32(&bars->o_empty), 256);
    mbar_init(smem_u32(&bars->drain), 1);
    bars->abort_flag = 0;
    for (int i = 0; i < kPSlots; ++i) bars->sent_seq[i] = bars->peer_sent[i] = -1;
    bars->armed_upto = bars->done_upto = 0;
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
  // every CTA of the grid is resident: the combine kernel queued behind this
  // one may be launched (its blocks with nothing to merge finish meanwhile,
  // the others wait for this grid to complete)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (rank == 0) {
    // ================================================================ score CTA
    const uint32_t ring = s_base + kOffRing;
    const uint32_t qrope = s_base + kOffQRope;
    if (warp == 0 || (kSparse && (warp == 2 || warp == 3 || warp >= 12))) {
      // ---------------------------------------------------------- producer
      if constexpr (kSparse) {
        // Top-k rows: seven gather warps (0, 2, 3, 12-15), warp k owning row
        // groups k, k + 7, ... (rows 4 group .. + 3 of a tile, one
        // tile::gather4 per chunk: the TMA unit serialises the gathers of one
        // warp, so spreading them over warps multiplies the row rate).  Every
        // gather warp waits for each ring slot to be free; warp 0 also arms
        // the slots, loads the query and gates each tile on the release of
        // its S buffer.
        const int gw = warp == 0 ? 0 : (warp <= 3 ? warp - 1 : warp - 9);
        const int rg = gw + kGatherWarps * lane;  // this lane's row group (< 32)
        const bool has_rg = rg < 32;
        if (warp == 0 && lane == 0) {
          tma_prefetch_desc(&q_map);
          tma_prefetch_desc(&g_map);
        }
        RingPos rp;
        uint32_t issued = 0, tg = 0;
        int qi = 0;
        bool ok = true;
        auto take_slot = [&](uint32_t bytes) -> uint32_t {  // wait until free; warp 0 arms
          uint32_t full = 0xffffffffu;
          if (lane == 0 && mbar_wait(smem_u32(&bars->ch_empty[rp.slot]), rp.phase ^ 1, abort_flag,
                                     p.status, kDevTimeoutProducer)) {
            full = smem_u32(&bars->ch_full[rp.slot]);
            if (warp == 0) mbar_arrive_expect_tx(full, bytes);
          }
          full = __shfl_sync(0xffffffffu, full, 0);
          if (full != 0xffffffffu) ++issued;
          return full;
        };
        for (int i = 0; i < n_pieces && ok; ++i) {
          const Piece pc = get_piece(p, meta, i);
          if (pc.tok_end <= pc.tok0) continue;
          for (int c = 0; c < kQChunks; ++c) {  // latent Q: warp 0's slots
            if (warp == 0) {
              const uint32_t full = take_slot(kChunkBytes);
              if (!(ok = full != 0xffffffffu)) break;
              if (lane == 0)
                tma_load_3d(ring + rp.slot * kChunkBytes, &q_map, full, 64 * c, row0, pc.b);
            }
            rp.next();
          }
          if (!ok) break;
          if (warp == 0) {
            bool okr = true;
            if (lane == 0) {
              okr = mbar_wait(smem_u32(&bars->rope_empty[qi & 1]), ((qi >> 1) & 1) ^ 1, abort_flag,
                              p.status, kDevTimeoutProducer);
              if (okr) {
                mbar_arrive_expect_tx(smem_u32(&bars->rope_full[qi & 1]), kChunkBytes);
                tma_load_3d(qrope + (qi & 1) * kChunkBytes, &q_map,
                            smem_u32(&bars->rope_full[qi & 1]), 512, row0, pc.b);
              }
            }
            if (!(ok = __shfl_sync(0xffffffffu, okr ? 1 : 0, 0) != 0)) break;
          }
          ++qi;
          const int32_t *idx = p.indices + static_cast<int64_t>(pc.b) * p.idx_sb +
                               static_cast<int64_t>(mb) * p.idx_ss;
          const int fb = first_valid_row(idx, p.topk, p.total_rows);
          int nr[4] = {-1, -1, -1, -1};  // the next tile's rows, loaded one tile ahead
          if (has_rg) load_rows4(idx, pc.tok0 + 4 * rg, pc.tok_end, nr);
          for (int tok = pc.tok0; tok < pc.tok_end && ok; tok += 2 * kBlk, ++tg) {
            const int n_blk = (pc.tok_end - tok > kBlk) ? 2 : 1;
            int r[4] = {nr[0], nr[1], nr[2], nr[3]};
            if (has_rg && tok + 2 * kBlk < pc.tok_end)
              load_rows4(idx, tok + 2 * kBlk + 4 * rg, pc.tok_end, nr);
            const uint32_t bad = fix_rows4(r, p.total_rows, fb);
            if (has_rg) bars->inval[tg & 3u][rg] = static_cast<uint8_t>(bad);
            if (warp == 0) {  // S buffer release before the tile's first chunk is armed
              bool okw = true;
              if (lane == 0)
                okw = mbar_wait(smem_u32(&bars->s_empty[tg & 1u]), ((tg >> 1) & 1u) ^ 1u, abort_flag,
                                p.status, kDevTimeoutProducer);
              if (!(ok = __shfl_sync(0xffffffffu, okw ? 1 : 0, 0) != 0)) break;
            }
            __syncwarp();
            for (int c = 0; c < kKChunks; ++c) {
              const uint32_t full = take_slot(n_blk * kBoxBytes);
              if (!(ok = full != 0xffffffffu)) break;
              if (has_rg && rg < n_blk * 16)
                gather_rows4(ring + rp.slot * kChunkBytes + rg * 4 * kRowBytes, &g_map, full,
                             64 * c, r, p.uniform_rows, p.page_size);
              rp.next();
            }
          }
        }
        if (*abort_flag && warp == 0 && lane == 0) {  // copies in flight land before exit
          volatile int never = 0;
          for (uint32_t t = issued > kRing ? issued - kRing : 0; t < issued; ++t)
            mbar_wait(smem_u32(&bars->ch_full[t % kRing]), (t / kRing) & 1, &never, nullptr, 0);
          if (qi > 0)
            mbar_wait(smem_u32(&bars->rope_full[(qi - 1) & 1]), ((qi - 1) >> 1) & 1, &never,
                      nullptr, 0);
        }
      } else {
      if (lane == 0) {
        tma_prefetch_desc(&q_map);
        tma_prefetch_desc(&kv_map);
        RingPos rp;
        uint32_t issued = 0, tg = 0;
        int qi = 0;
        bool ok = true;
        auto next_slot = [&](uint32_t bytes) -> uint32_t {  // wait for a free slot, arm it
          if (!mbar_wait(smem_u32(&bars->ch_empty[rp.slot]), rp.phase ^ 1, abort_flag, p.status,
                         kDevTimeoutProducer))
            return 0xffffffffu;
          const uint32_t full = smem_u32(&bars->ch_full[rp.slot]);
          mbar_arrive_expect_tx(full, bytes);
          ++issued;
          return full;
        };
        for (int i = 0; i < n_pieces && ok; ++i) {
          const Piece pc = get_piece(p, meta, i);
          if (pc.tok_end <= pc.tok0) continue;
          // latent Q: 8 chunks of 64 dims x 128 rows through the ring
          for (int c = 0; c < kQChunks; ++c) {
            const uint32_t full = next_slot(kChunkBytes);
            if (!(ok = full != 0xffffffffu)) break;
            tma_load_3d(ring + rp.slot * kChunkBytes, &q_map, full, 64 * c, row0, pc.b);
            rp.next();
          }
          if (!ok) break;
          // rope Q (dims 512..575) -> buffer qi & 1
          ok = mbar_wait(smem_u32(&bars->rope_empty[qi & 1]), ((qi >> 1) & 1) ^ 1, abort_flag,
                         p.status, kDevTimeoutProducer);
          if (!ok) break;
          mbar_arrive_expect_tx(smem_u32(&bars->rope_full[qi & 1]), kChunkBytes);
          tma_load_3d(qrope + (qi & 1) * kChunkBytes, &q_map, smem_u32(&bars->rope_full[qi & 1]),
                      512, row0, pc.b);
          ++qi;
          // page coordinates of the next tile are looked up one tile ahead
          int nc1[2], nc2[2];
          for (int j = 0; j < 2; ++j)
            if (pc.tok0 + j * kBlk < pc.tok_end) kv_coord(p, pc.b, pc.tok0 + j * kBlk, nc1[j], nc2[j]);
          for (int tok = pc.tok0; tok < pc.tok_end && ok; tok += 2 * kBlk, ++tg) {
            const int n_blk = (pc.tok_end - tok > kBlk) ? 2 : 1;
            const int c1[2] = {nc1[0], nc1[1]}, c2[2] = {nc2[0], nc2[1]};
            for (int j = 0; j < 2; ++j)
              if (tok + (2 + j) * kBlk < pc.tok_end)
                kv_coord(p, pc.b, tok + (2 + j) * kBlk, nc1[j], nc2[j]);
            // The tile's S buffer (tg & 1) must have been released by the
            // softmax before the tile's first key chunk is published: the MMA
            // issuer orders its QK after that release through the chunk wait.
            if (!(ok = mbar_wait(smem_u32(&bars->s_empty[tg & 1u]), ((tg >> 1) & 1u) ^ 1u,
                                 abort_flag, p.status, kDevTimeoutProducer)))
              break;
            for (int c = 0; c < kKChunks; ++c) {
              const uint32_t full = next_slot(n_blk * kBoxBytes);
              if (!(ok = full != 0xffffffffu)) break;
              for (int j = 0; j < n_blk; ++j)
                tma_load_3d(ring + rp.slot * kChunkBytes + j * kBoxBytes, &kv_map, full, 64 * c,
                            c1[j], c2[j]);
              rp.next();
            }
          }
        }
        if (*abort_flag) {  // copies in flight must land before the CTA may exit
          volatile int never = 0;
          for (uint32_t t = issued > kRing ? issued - kRing : 0; t < issued; ++t)
            mbar_wait(smem_u32(&bars->ch_full[t % kRing]), (t / kRing) & 1, &never, nullptr, 0);
          if (qi > 0)
            mbar_wait(smem_u32(&bars->rope_full[(qi - 1) & 1]), ((qi - 1) >> 1) & 1, &never,
                      nullptr, 0);
        }
      }
      }
      __syncwarp();
    } else if (warp == 1) {
      // -------------------------------------------------------- MMA issuer
      // The whole warp runs the loop and an elected lane issues each MMA /
      // copy / commit.  The instruction descriptor must be a compile-time
      // constant: a runtime one costs about 40 extra cycles per MMA.
      {
      constexpr uint32_t kIdesc128 = umma_idesc_f16(128, 128, fmt, 0);
      const uint64_t ring_desc = smem_desc_sw128(ring, 16, 1024);
      const uint64_t rope_desc = smem_desc_sw128(qrope, 16, 1024);
      auto wait = [&](uint32_t bar, uint32_t parity) -> bool {
        // fast path: the phase is usually complete already (one test_wait,
        // uniform across the warp); otherwise the bounded wait
        if (mbar_probe(bar, parity)) return true;
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, p.status, kDevTimeoutMma)) != 0;
      };
      RingPos rp;
      uint32_t g = 0;
      int qi = 0;
      bool ok = true;
      // QK of one tile into S buffer sd: 8 latent chunks (A = Q from TMEM)
      // and the rope chunk (A = rope Q from shared memory).
      auto qk_tile = [&](auto idesc_tag, uint32_t sd, uint64_t rope_a) -> bool {
        constexpr uint32_t idesc = decltype(idesc_tag)::value;
#pragma unroll 1
        for (int c = 0; c < kKChunks; ++c) {
          if (!wait(smem_u32(&bars->ch_full[rp.slot]), rp.phase)) return false;
          if (c == 0) tc_fence_after();  // after the S buffer release (through the producer)
          // TMA data signalled by the mbarrier: no tcgen05 fence here (one
          // after every chunk drains the MMA queue and halves the rate)
          const uint64_t kdesc = ring_desc + static_cast<uint64_t>((rp.slot * kChunkBytes) >> 4);
          if (c < kQChunks) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_ts_warp(sd, tmem + kColQ + c * 32 + kk * 8, kdesc + 2 * kk, idesc,
                           (c | kk) ? 1u : 0u);
          } else {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) umma_ss_warp(sd, rope_a + 2 * kk, kdesc + 2 * kk, idesc, 1u);
          }
          tc_commit_warp(smem_u32(&bars->ch_empty[rp.slot]));
          rp.next();
        }
        return true;
      };
      for (int i = 0; i < n_pieces && ok; ++i) {
        const Piece pc = get_piece(p, meta, i);
        if (pc.tok_end <= pc.tok0) continue;
        // latent Q -> TMEM columns [0, 256): tcgen05.cp runs in order with
        // this warp's MMAs, so it starts after the previous piece's last QK
        for (int c = 0; c < kQChunks && ok; ++c) {
          ok = wait(smem_u32(&bars->ch_full[rp.slot]), rp.phase);
          if (!ok) break;
          const uint64_t qdesc = ring_desc + static_cast<uint64_t>((rp.slot * kChunkBytes) >> 4);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) tmem_cp_128x256b_warp(tmem + kColQ + c * 32 + kk * 8, qdesc + 2 * kk);
          tc_commit_warp(smem_u32(&bars->ch_empty[rp.slot]));
          rp.next();
        }
        ok = ok && wait(smem_u32(&bars->rope_full[qi & 1]), (qi >> 1) & 1);
        if (!ok) break;
        const uint64_t rope_a = rope_desc + static_cast<uint64_t>(((qi & 1) * kChunkBytes) >> 4);
        for (int tok = pc.tok0; tok < pc.tok_end && ok; tok += 2 * kBlk, ++g) {
          const uint32_t buf = g & 1u;
          const uint32_t sd = tmem + kColS + buf * 128;
          // S buffer reuse: the producer publishes this tile's first key
          // chunk only after the softmax released the buffer (s_empty), so
          // the chunk wait below (then a tcgen05 fence) orders the QK after
          // the softmax's reads.  Waiting on s_empty here instead costs about
          // 800 cycles of tensor-pipe time per tile (measured), even when the
          // phase is already complete.
          // A half tile at a piece end (only its first 64 key rows loaded)
          // runs the same N = 128 MMAs: the other 64 rows of the ring slot
          // hold stale but valid bytes, and their score columns are masked
          // (select) by the softmax.  One instantiation keeps the loop small.
          ok = qk_tile(std::integral_constant<uint32_t, kIdesc128>{}, sd, rope_a);
          if (!ok) break;
          tc_commit_warp(smem_u32(&bars->s_full[buf]));
        }
        if (!ok) break;
        tc_commit_warp(smem_u32(&bars->rope_empty[qi & 1]));
        ++qi;
      }
      // every issued MMA must finish before TMEM is released
      tc_commit_warp(smem_u32(&bars->drain));
      volatile int never = 0;
      mbar_wait(smem_u32(&bars->drain), 0, &never, p.status, kDevTimeoutDrain);
      }
      __syncwarp();
    } else if (warp >= 4 && warp < 12) {
      // --------------------------------------------------------- softmax
      // warp w: query rows 32 (w % 4) .. +31 (its TMEM lanes) and block
      // ch = (w - 4) / 4 of every tile (score columns 64 ch .. 64 ch + 63).
      const int ch = (warp - 4) >> 2;
      const int q4 = warp & 3;
      const int t = q4 * 32 + lane;
      const uint32_t trow = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
      const uint32_t pair_bar = smem_u32(&bars->pair[q4]);
      uint32_t pair_uses = 0;
      auto pair_sync = [&]() -> bool {
        mbar_arrive(pair_bar);
        const bool r = __all_sync(0xffffffffu, mbar_wait(pair_bar, pair_uses & 1, abort_flag,
                                                         p.status, kDevTimeoutSoftmax));
        ++pair_uses;
        return r;
      };
      float *red = reinterpret_cast<float *>(smem + kOffRed);  // [tile parity][ch][row]
      const int flat = row0 + t;
      const bool row_ok = t < n_rows;
      const int s_tok = row_ok ? flat / p.h_q : 0;
      const uint32_t p_remote = map_to_rank(s_base + kOffP, 1);
      const uint32_t pfull_remote = map_to_rank(smem_u32(&bars->p_full[0]), 1);
      bool ok = true;
      uint32_t g = 0, gb = 0;
      uint32_t stg_uses[2] = {0, 0};
      for (int i = 0; i < n_pieces && ok; ++i) {
        const Piece pc = get_piece(p, meta, i);
        const int len = seq_len(p, pc.b);
        const int row_len = p.causal ? len - (p.s_q - 1 - s_tok) : len;
        float m_run = -INFINITY, l_half = 0.f, l_run = 0.f;
        for (int tok = pc.tok0; tok < pc.tok_end && ok; tok += 2 * kBlk, ++g) {
          const bool first = tok == pc.tok0;
          const bool last = tok + 2 * kBlk >= pc.tok_end;
          const int n_blk = (pc.tok_end - tok > kBlk) ? 2 : 1;
          const uint32_t buf = g & 1u;
          ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars->s_full[buf]), (g >> 1) & 1,
                                                  abort_flag, p.status, kDevTimeoutSoftmax));
          if (!ok) break;
          tc_fence_after();
          float sc[64];
          {
            float v0[32], v1[32];
            tmem_ld32(trow + kColS + buf * 128 + ch * 64, v0);
            tmem_ld32(trow + kColS + buf * 128 + ch * 64 + 32, v1);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              sc[j] = v0[j];
              sc[32 + j] = v1[j];
            }
          }
          // sparse: this block's invalid-row bits (row groups 16 ch .. 16 ch +
          // 15), read before the S buffer is released (the tile whose rows
          // reuse the slot cannot start gathering before that release)
          uint4 bad4 = make_uint4(0u, 0u, 0u, 0u);
          if constexpr (kSparse) bad4 = *reinterpret_cast<const uint4 *>(&bars->inval[g & 3u][16 * ch]);
          tc_fence_before();
          mbar_arrive(smem_u32(&bars->s_empty[buf]));
          // mask columns past the sequence / causal end (select: NaN-safe)
          const int lim = min(pc.tok_end, row_len) - tok - ch * kBlk;
          if (lim < kBlk) {
#pragma unroll
            for (int c = 0; c < kBlk; ++c)
              if (c >= lim) sc[c] = -INFINITY;
          }
          if constexpr (kSparse) {
            // column c = block row 4 k + j: bit j of byte k (word k / 4)
            if (bad4.x | bad4.y | bad4.z | bad4.w) {
              const uint32_t bw[4] = {bad4.x, bad4.y, bad4.z, bad4.w};
#pragma unroll
              for (int c = 0; c < kBlk; ++c)
                if ((bw[c >> 4] >> (8 * ((c >> 2) & 3) + (c & 3))) & 1u) sc[c] = -INFINITY;
            }
          }
          // row maximum: three-input max in two chains (elements 0, 1 seed
          // them, 2..61 in steps of four, then 62, 63)
          static_assert(kBlk == 64, "max chain layout");
          float mx0 = sc[0], mx1 = sc[1];
#pragma unroll
          for (int c = 2; c < kBlk - 2; c += 4) {
            mx0 = fmax3(mx0, sc[c], sc[c + 1]);
            mx1 = fmax3(mx1, sc[c + 2], sc[c + 3]);
          }
          float mraw = fmaxf(fmax3(mx0, sc[kBlk - 2], sc[kBlk - 1]), mx1);
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
          // exponent argument and row sum in packed f32 pairs (one FFMA2 /
          // FADD2 per two scores), exp2 per score, bf16 pair pack
          const uint64_t sc2 = f32x2(p.scale_log2, p.scale_log2), nms2 = f32x2(-ms, -ms);
          uint64_t ps2[2] = {f32x2(0.f, 0.f), f32x2(0.f, 0.f)};
          uint32_t pk[kBlk / 2];
#pragma unroll
          for (int c = 0; c < kBlk; c += 2) {
            float x0, x1;
            f32x2_split(ffma2(f32x2(sc[c], sc[c + 1]), sc2, nms2), x0, x1);
            const float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
            const uint64_t pp = f32x2(p0, p1);
            ps2[(c >> 1) & 1] = fadd2(ps2[(c >> 1) & 1], pp);
            pk[c / 2] = Elem<T>::pack2(p0, p1);
          }
          float s0, s1, s2, s3;
          f32x2_split(ps2[0], s0, s1);
          f32x2_split(ps2[1], s2, s3);
          l_half = l_half * alpha + ((s0 + s1) + (s2 + s3));
          // A piece's last tile: the row sum of both blocks (through this
          // tile's parity slot, once the partner has read the tile maximum);
          // 1 / row sum and the piece's LSE (natural log of the scaled row sum)
          // travel with the piece's last block, so that the value CTA writes
          // the piece's output and LSE together.
          float inv_l = 0.f, lse_piece = -INFINITY;
          if (last) {
            if (!(ok = pair_sync())) break;
            rslot[ch * kRows + t] = l_half;
            if (!(ok = pair_sync())) break;
            l_run = l_half + rslot[(ch ^ 1) * kRows + t];
            const float msr = (m_run == -INFINITY) ? 0.f : m_run;
            lse_piece = l_run > 0.f ? msr * 0.69314718055994531f + logf(l_run) : -INFINITY;
            inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
          }
          // P of this warp's block -> the value CTA's slot (gb + ch) % kPSlots
          const uint32_t pb = gb + ch;
          const uint32_t pslot = pb % kPSlots;
          const uint32_t pdst = p_remote + pslot * kPSlotBytes;
          const uint32_t pbar = pfull_remote + pslot * 8;
          if (ch < n_blk) {
            // The block's P (16 KB) and its metadata (O rescale factors and
            // flags with a tile's first block, 1 / row sum and LSE with a
            // piece's last block) are staged in local shared memory (buffer
            // pb & 1, laid out like the value CTA's slot) and sent as ONE bulk
            // copy of the whole slot (kPSlotBytes): one transfer per block,
            // issued by one thread, which the teardown can account for
            // exactly.  Separate 16-byte remote stores per row crowd the
            // memory-instruction queues that the producer's and MMA warp's
            // instructions also use.  The staging buffer was last sent for
            // block pb - 2, whose PV has finished once p_free of its slot has
            // (its copy had landed).  (Relaying the copy's arrival back from
            // the value CTA instead measured no faster: this wait is not what
            // paces the pair.)
            ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars->p_free[pslot]),
                                                   ((pb / kPSlots) & 1) ^ 1, abort_flag, p.status,
                                                   kDevTimeoutSoftmax));
            if (ok && pb >= 2)
              ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars->p_free[(pb - 2) % kPSlots]),
                                                     ((pb - 2) / kPSlots) & 1, abort_flag,
                                                     p.status, kDevTimeoutSoftmax));
            if (!ok) break;
            const uint32_t stg = s_base + kOffStgP + (pb & 1) * kPSlotBytes;
#pragma unroll
            for (int u = 0; u < 8; ++u)
              asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(
                               stg + t * kRowBytes + ((u ^ (t & 7)) << 4)),
                           "r"(pk[4 * u]), "r"(pk[4 * u + 1]), "r"(pk[4 * u + 2]), "r"(pk[4 * u + 3])
                           : "memory");
            if (ch == 0) {
              const bool any = __any_sync(0xffffffffu, rescale);
              asm volatile("st.shared.f32 [%0], %1;" ::"r"(stg + kMetaAlpha + 4 * t),
                           "f"(rescale ? alpha : 1.f)
                           : "memory");
              if (lane == 0)
                asm volatile("st.shared.u32 [%0], %1;" ::"r"(stg + kMetaFlags + 4 * q4),
                             "r"(any ? 1u : 0u)
                             : "memory");
            }
            if (last && ch == n_blk - 1) {
              asm volatile("st.shared.f32 [%0], %1;" ::"r"(stg + kMetaInvL + 4 * t), "f"(inv_l)
                           : "memory");
              asm volatile("st.shared.f32 [%0], %1;" ::"r"(stg + kMetaLse + 4 * t), "f"(lse_piece)
                           : "memory");
            }
            fence_proxy_async_smem();  // generic-proxy writes -> the bulk copy's reads
            mbar_arrive(smem_u32(&bars->stg_ready[ch]));
            if (t == 0) {
              if (!mbar_wait(smem_u32(&bars->stg_ready[ch]), stg_uses[ch] & 1, abort_flag,
                             p.status, kDevTimeoutSoftmax)) {
                ok = false;
              } else {
                bulk_copy_to_peer(pdst, stg, kPSlotBytes, pbar);
                *reinterpret_cast<volatile int *>(&bars->sent_seq[pslot]) = static_cast<int>(pb);
              }
            }
            ++stg_uses[ch];
            if (!(ok = __all_sync(0xffffffffu, ok))) break;
          }
          gb += n_blk;
        }
      }
    }
  } else {
    // ================================================================ value CTA
    const uint32_t vbase = s_base + kOffV;
    const uint32_t pbase = s_base + kOffP;
    if (warp == 0 || (kSparse && (warp == 2 || warp == 3 || warp >= 12))) {
      // ------------------------------------------------------- V producer
      if constexpr (kSparse) {
        // Top-k rows: the seven gather warps (0, 2, 3, 12-15) split the 64
        // (value chunk, 4-row group) gathers of every 32-row stage, pair
        // q = warp index + 7 lane: chunk q / 8, rows 4 (q % 8) .. + 3.  Each
        // gather warp waits for the stage to be free; warp 0 arms it.
        const int gw = warp == 0 ? 0 : (warp <= 3 ? warp - 1 : warp - 9);
        const int q = gw + kGatherWarps * lane;
        const bool has_q = q < 64;
        const int d = q >> 3, rg = q & 7;
        if (warp == 0 && lane == 0) tma_prefetch_desc(&g_map);
        uint32_t vs = 0;
        bool ok = true;
        for (int i = 0; i < n_pieces && ok; ++i) {
          const Piece pc = get_piece(p, meta, i);
          const int32_t *idx = p.indices + static_cast<int64_t>(pc.b) * p.idx_sb +
                               static_cast<int64_t>(mb) * p.idx_ss;
          // stages start at tok0, tok0 + 32, ... (< tok_end); their rows are
          // loaded two stages ahead
          const int fb = first_valid_row(idx, p.topk, p.total_rows);
          int n1[4] = {-1, -1, -1, -1}, n2[4] = {-1, -1, -1, -1};
          if (has_q) {
            load_rows4(idx, pc.tok0 + 4 * rg, pc.tok_end, n1);
            load_rows4(idx, pc.tok0 + kVRows + 4 * rg, pc.tok_end, n2);
          }
          for (int bt = pc.tok0; bt < pc.tok_end && ok; bt += kBlk) {
            const int vb = min(kBlk, pc.tok_end - bt);
            const int n_sub = vb > kVRows ? 2 : 1;
            for (int j = 0; j < n_sub; ++j, ++vs) {
              int r[4] = {n1[0], n1[1], n1[2], n1[3]};
#pragma unroll
              for (int k = 0; k < 4; ++k) n1[k] = n2[k];
              const int ahead = bt + kVRows * (j + 2);
              if (has_q && ahead < pc.tok_end) load_rows4(idx, ahead + 4 * rg, pc.tok_end, n2);
              fix_rows4(r, p.total_rows, fb);
              const int st = vs % kVStages;
              const uint32_t full = smem_u32(&bars->v_full[st]);
              bool okw = true;
              if (lane == 0) {
                okw = mbar_wait(smem_u32(&bars->v_empty[st]), ((vs / kVStages) & 1) ^ 1, abort_flag,
                                p.status, kDevTimeoutProducer);
                if (okw && warp == 0) mbar_arrive_expect_tx(full, kVStageBytes);
              }
              if (!(ok = __shfl_sync(0xffffffffu, okw ? 1 : 0, 0) != 0)) break;
              if (has_q)
                gather_rows4(vbase + st * kVStageBytes + d * kVChunkBytes + rg * 4 * kRowBytes,
                             &g_map, full, 64 * d, r, p.uniform_rows, p.page_size);
            }
          }
        }
        if (*abort_flag && warp == 0 && lane == 0) {
          volatile int never = 0;
          for (uint32_t t = vs > kVStages ? vs - kVStages : 0; t < vs; ++t)
            mbar_wait(smem_u32(&bars->v_full[t % kVStages]), (t / kVStages) & 1, &never, nullptr,
                      0);
        }
      } else {
      if (lane == 0) {
        tma_prefetch_desc(&v_map);
        uint32_t vs = 0;
        bool ok = true;
        for (int i = 0; i < n_pieces && ok; ++i) {
          const Piece pc = get_piece(p, meta, i);
          for (int bt = pc.tok0; bt < pc.tok_end && ok; bt += kBlk) {
            const int vb = min(kBlk, pc.tok_end - bt);
            const int n_sub = vb > kVRows ? 2 : 1;
            int c1, c2;
            kv_coord(p, pc.b, bt, c1, c2);
            for (int j = 0; j < n_sub; ++j, ++vs) {
              const int st = vs % kVStages;
              ok = mbar_wait(smem_u32(&bars->v_empty[st]), ((vs / kVStages) & 1) ^ 1, abort_flag,
                             p.status, kDevTimeoutProducer);
              if (!ok) break;
              const uint32_t full = smem_u32(&bars->v_full[st]);
              mbar_arrive_expect_tx(full, kVStageBytes);
              // one box: 32 rows x the 8 value chunks, laid out chunk by chunk
              tma_load_4d(vbase + st * kVStageBytes, &v_map, full, 0, c1 + kVRows * j, 0, c2);
            }
          }
        }
        if (*abort_flag) {
          volatile int never = 0;
          for (uint32_t t = vs > kVStages ? vs - kVStages : 0; t < vs; ++t)
            mbar_wait(smem_u32(&bars->v_full[t % kVStages]), (t / kVStages) & 1, &never, nullptr,
                      0);
        }
      }
      }
      __syncwarp();
    } else if (warp == 1) {
      // ----------------------------------------------------- PV MMA issuer
      // Issued like the score CTA's MMAs (warp-wide, elected lane).
      {
      constexpr uint32_t idesc = umma_idesc_f16(128, 256, fmt, 1);
      const uint64_t p_desc = smem_desc_sw128(pbase, 16, 1024);
      const uint64_t v_desc = smem_desc_sw128(vbase, kVChunkBytes, 1024);
      auto wait = [&](uint32_t bar, uint32_t parity) -> bool {
        // fast path: the phase is usually complete already (one test_wait,
        // uniform across the warp); otherwise the bounded wait
        if (mbar_probe(bar, parity)) return true;
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, p.status, kDevTimeoutMma)) != 0;
      };
      uint32_t vs = 0, gb = 0;
      uint32_t armed = 0, landed = 0;  // P blocks armed / seen complete (teardown accounting)
      int pi = 0;
      bool ok = true;
      for (int i = 0; i < n_pieces && ok; ++i) {
        const Piece pc = get_piece(p, meta, i);
        if (pc.tok_end <= pc.tok0) continue;
        bool first_blk = true;
        for (int bt = pc.tok0; bt < pc.tok_end && ok; bt += kBlk, ++gb) {
          const int vb = min(kBlk, pc.tok_end - bt);
          const int n_sub = vb > kVRows ? 2 : 1;
          const uint32_t ps = gb % kPSlots;
          const uint32_t ph = (gb / kPSlots) & 1;
          // every block arrives as one copy of the whole slot (P + metadata)
          if (lane == 0) mbar_arrive_expect_tx(smem_u32(&bars->p_full[ps]), kPSlotBytes);
          armed = gb + 1;
          ok = wait(smem_u32(&bars->p_full[ps]), ph);
          if (ok) landed = gb + 1;
          ok = ok && wait(smem_u32(&bars->m_read[ps]), ph);
          if (ok && first_blk) ok = wait(smem_u32(&bars->o_empty), (pi & 1) ^ 1);
          if (!ok) break;
          fence_proxy_async_smem();  // cleared value rows -> tensor-core reads
          tc_fence_after();
          const uint64_t pa = p_desc + static_cast<uint64_t>((ps * kPSlotBytes) >> 4);
          for (int j = 0; j < n_sub; ++j, ++vs) {
            const uint32_t st = vs % kVStages;
            ok = wait(smem_u32(&bars->v_full[st]), (vs / kVStages) & 1);
            if (!ok) break;
            const uint64_t vd = v_desc + static_cast<uint64_t>((st * kVStageBytes) >> 4);
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
              const uint64_t adesc = pa + static_cast<uint64_t>(((2 * j + kk) * 32) >> 4);
#pragma unroll
              for (int hh = 0; hh < 2; ++hh)
                umma_ss_warp(tmem + 256 * hh, adesc,
                             vd + static_cast<uint64_t>((hh * 4 * kVChunkBytes + kk * 16 * kRowBytes) >> 4),
                             idesc, (first_blk && j == 0 && kk == 0) ? 0u : 1u);
            }
            tc_commit_warp(smem_u32(&bars->v_empty[st]));
          }
          if (!ok) break;
          tc_commit_warp(smem_u32(&bars->pv_done[ps]));
          tc_commit_mc_warp(smem_u32(&bars->p_free[ps]), 0x1);  // the score CTA may refill the slot
          first_blk = false;
        }
        ++pi;
      }
      if (lane == 0) {
        bars->armed_upto = static_cast<int>(armed);
        bars->done_upto = static_cast<int>(landed);
      }
      tc_commit_warp(smem_u32(&bars->drain));
      volatile int never = 0;
      mbar_wait(smem_u32(&bars->drain), 0, &never, p.status, kDevTimeoutDrain);
      }
      __syncwarp();
    } else if (warp >= 4 && warp < 12) {
      // ---------------------------------- O rescale, tail rows, epilogue
      // warp w: rows 32 (w % 4) .. +31, output dims [256 ch, 256 ch + 256)
      const int ch = (warp - 4) >> 2;
      const int q4 = warp & 3;
      const int t = q4 * 32 + lane;
      const int tt = ch * kRows + t;  // 0..255
      const uint32_t trow = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
      uint32_t vs = 0, gb = 0;
      bool ok = true;
      // A piece's bounds and split slots are fetched while the previous
      // piece's last PV runs (before its epilogue), so that after the
      // epilogue the next piece's first block is released at once: these
      // dependent global loads would otherwise sit between the two.
      Piece nxt{};
      int nxt_first = 0, nxt_n = 1;
      auto fetch = [&](int i) {
        nxt = get_piece(p, meta, i);
        nxt_first = p.num_splits[nxt.b];
        nxt_n = p.num_splits[nxt.b + 1] - nxt_first;
      };
      if (n_pieces > 0) fetch(0);
      for (int i = 0; i < n_pieces && ok; ++i) {
        const Piece pc = nxt;
        const int first_slot = nxt_first;
        const int n_split = nxt_n;
        const int slot_o = first_slot + pc.split_idx;
        const bool has_tiles = pc.tok_end > pc.tok0;
        float inv_l = 0.f, lse_row = -INFINITY;
        for (int bt = pc.tok0; bt < pc.tok_end && ok; bt += kBlk, ++gb) {
          const int vb = min(kBlk, pc.tok_end - bt);
          const int n_sub = vb > kVRows ? 2 : 1;
          const bool tile_first = ((bt - pc.tok0) & (2 * kBlk - 1)) == 0;
          const int ps = gb % kPSlots;
          const uint32_t ph = (gb / kPSlots) & 1;
          ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars->p_full[ps]), ph, abort_flag,
                                                  p.status, kDevTimeoutSoftmax));
          if (!ok) break;
          const uint8_t *slotp = smem + kOffP + ps * kPSlotBytes;
          if (tile_first && bt != pc.tok0) {
            const int *fl = reinterpret_cast<const int *>(slotp + kMetaFlags);
            if (fl[0] | fl[1] | fl[2] | fl[3]) {
              // O may be rescaled once the previous block's PV has finished
              const uint32_t pg = gb - 1;
              ok = __all_sync(0xffffffffu,
                              mbar_wait(smem_u32(&bars->pv_done[pg % kPSlots]), (pg / kPSlots) & 1,
                                        abort_flag, p.status, kDevTimeoutSoftmax));
              if (!ok) break;
              if (fl[q4]) {
                tc_fence_after();
                rescale_o_half(trow + ch * 256, reinterpret_cast<const float *>(slotp + kMetaAlpha)[t]);
              }
            }
          }
          if (bt + kBlk >= pc.tok_end) {
            inv_l = reinterpret_cast<const float *>(slotp + kMetaInvL)[t];
            lse_row = reinterpret_cast<const float *>(slotp + kMetaLse)[t];
          }
          if (vb < kBlk) {
            // rows past the sequence end may hold any bits (even NaN); P is 0
            // there but 0 * NaN is not, so clear them before the PV product.
            for (int j = 0; j < n_sub; ++j) {
              const int lo = max(vb - kVRows * j, 0);
              if (lo >= kVRows) continue;
              const uint32_t sv = vs + j;
              const int st = sv % kVStages;
              ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars->v_full[st]), (sv / kVStages) & 1,
                                                      abort_flag, p.status, kDevTimeoutSoftmax));
              if (!ok) break;
              clear_v_rows(smem + kOffV + st * kVStageBytes, lo, tt);
            }
            if (!ok) break;
            fence_proxy_async_smem();
          }
          tc_fence_before();
#ifdef FA_DEBUG_ABORT_TEST
          // the abort-path test build: block kAbortTestBlock's metadata-read
          // arrival is lost, so the PV issuer's wait for it runs out while
          // the score CTA still has later blocks in flight (teardown drain)
          if (gb != kAbortTestBlock)
#endif
          mbar_arrive(smem_u32(&bars->m_read[ps]));
          vs += n_sub;
        }
        if (!ok) break;
        if (i + 1 < n_pieces) fetch(i + 1);
        if (has_tiles) {
          const uint32_t lg = gb - 1;
          ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars->pv_done[lg % kPSlots]),
                                                 (lg / kPSlots) & 1, abort_flag, p.status,
                                                 kDevTimeoutSoftmax));
          if (!ok) break;
          tc_fence_after();
        }
        // O / l -> out (final) or the split workspace, in the output type:
        // half the bytes of f32 partials for a bf16 / f16 output, the same
        // rounding the reference applies to its partial O (out.dtype,
        // paged.py:103-113)
        const bool final_out = n_split == 1;
        OutRows o;
        o.base = final_out ? static_cast<uint8_t *>(p.out) : reinterpret_cast<uint8_t *>(p.part_o);
        o.sb = p.o_sb;
        o.ss = p.o_ss;
        o.sh = p.o_sh;
        o.b = pc.b;
        o.h_q = p.h_q;
        o.row0 = row0;
        o.n_rows = n_rows;
        o.esz = p.out_f32 ? 4 : 2;
        o.split = !final_out;
        o.split_row0 = static_cast<int64_t>(slot_o) * rows_total;
        o.d_v = p.d_v;
        write_o_half<T>(trow, ch, q4, lane, smem_u32(smem + kOffStage + (warp - 4) * kStageWarpBytes),
                        has_tiles, inv_l, o);
        if (has_tiles) {
          tc_fence_before();
          mbar_arrive(smem_u32(&bars->o_empty));
        }
        if (ch == 0 && t < n_rows) {
          const int flat = row0 + t;
          if (final_out)
            p.lse[(static_cast<int64_t>(pc.b) * p.h_q + flat % p.h_q) * p.s_q + flat / p.h_q] = lse_row;
          else
            p.part_lse[static_cast<int64_t>(slot_o) * rows_total + flat] = lse_row;
        }
      }
    }
  }

  // -------------------------------------------------------------- teardown
  // No P transfer may still be in flight when either CTA exits (after a
  // bounded wait gave up, the roles unwind at different points).  The score
  // CTA sends block b into slot b % kPSlots only after block b - kPSlots was
  // consumed, so per slot at most one sent block can be unconsumed: the last
  // one sent (sent_seq).  The score CTA hands those numbers over; the value
  // CTA arms (when its PV issuer had not) and waits for each of them, so every
  // copy issued has landed -- and has finished reading the score CTA's
  // staging buffer -- before the second cluster barrier lets the pair go.
  // Without a time-out every sent block was consumed and nothing is waited.
  tc_fence_before();
  __syncthreads();
  if (rank == 0 && threadIdx.x == 0) {
    for (int i = 0; i < kPSlots; ++i)
      asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(
                       map_to_rank(smem_u32(&bars->peer_sent[i]), 1)),
                   "r"(static_cast<uint32_t>(
                       *reinterpret_cast<volatile int *>(&bars->sent_seq[i])))
                   : "memory");
  }
  cluster_sync();
  if (rank == 1 && threadIdx.x == 0) {
    volatile int never = 0;
    const int done = bars->done_upto, armed = bars->armed_upto;
    for (int i = 0; i < kPSlots; ++i) {
      const int b = *reinterpret_cast<volatile int *>(&bars->peer_sent[i]);
      if (b < done) continue;  // consumed (or nothing sent into this slot)
      const uint32_t bar = smem_u32(&bars->p_full[i]);
      if (b >= armed) mbar_arrive_expect_tx(bar, kPSlotBytes);
      mbar_wait(bar, (static_cast<uint32_t>(b) / kPSlots) & 1u, &never, p.status, kDevTimeoutDrain);
    }
  }
  cluster_sync();  // the peer no longer touches this CTA's shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace sv


// q_map: query (box 64 dims x 128 rows), kv_map: key rows (box 64 x 64),
// v_map: value rows ({64 dims, rows, 64-dim chunks, pages} with a box of 32
// rows x 8 chunks); all 128-byte swizzle over the same layouts as the
// reference's caches ([pages, page, 1, 576]).
namespace {
template <typename T, bool kSparse>
cudaError_t launch_sv_t(const CUtensorMap &qm, const CUtensorMap &km, const CUtensorMap &vm,
                        const CUtensorMap &gm, const sv::Params &p, dim3 grid,
                        cudaStream_t stream) {
  auto kern = sv::mla_decode_sv_kernel<T, kSparse>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       sv::kSmemBytes);
  if (e != cudaSuccess) return e;
  kern<<<grid, sv::kThreads, sv::kSmemBytes, stream>>>(qm, km, vm, gm, p);
  return cudaGetLastError();
}
}  // namespace

// gm: 2-D gather map over every pool row ({576, num_pages * page_size},
// box {64, 1}); read only by the top-k instance (indices != nullptr).
cudaError_t launch_mla_sv(const CUtensorMap &qm, const CUtensorMap &km, const CUtensorMap &vm,
                          const CUtensorMap &gm, const fa_mla_args *a, int m_blocks,
                          cudaStream_t stream) {
  sv::Params p;
  p.kcache = static_cast<const uint8_t *>(a->kcache);
  p.kv_sp = a->kv_stride_page;
  p.kv_st = a->kv_stride_tok;
  p.block_table = a->block_table;
  p.bt_stride = a->bt_stride;
  p.seq_lens = a->seq_lens;
  p.n_ctx = a->n_ctx;
  p.page_size = a->page_size;
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
  const bool sparse = a->indices != nullptr;
  p.indices = a->indices;
  p.idx_sb = a->idx_stride_b;
  p.idx_ss = a->idx_stride_s;
  p.topk = sparse ? a->topk : 0;
  p.total_rows = static_cast<int64_t>(a->num_pages) * a->page_size;
  p.uniform_rows = a->kv_stride_page == static_cast<int64_t>(a->page_size) * a->kv_stride_tok;
  const dim3 grid(2 * a->num_sm_parts, m_blocks);
  if (a->dtype == FA_DTYPE_F16)
    return sparse ? launch_sv_t<__half, true>(qm, km, vm, gm, p, grid, stream)
                  : launch_sv_t<__half, false>(qm, km, vm, gm, p, grid, stream);
  return sparse ? launch_sv_t<__nv_bfloat16, true>(qm, km, vm, gm, p, grid, stream)
                : launch_sv_t<__nv_bfloat16, false>(qm, km, vm, gm, p, grid, stream);
}

}  // namespace fa
