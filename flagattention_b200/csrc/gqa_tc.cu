// gqa_tc.cu -- grouped-query decode on tcgen05, paged or contiguous caches.
//
// The reference's decode kernels (paged.py:208-363 for paged caches,
// split_kv.py:28-174 for contiguous keys) compute, for each (sequence, kv
// head), S = Q K^T over the query rows of the head's group (tl.dot at
// paged.py:314), an online softmax, and O += P V (paged.py:333).  Here that
// work runs on the fifth-generation tensor cores:
//
//   * one persistent CTA per SM walks "pieces": a token range of one entry
//     (entry = sequence * kv_heads + kv head); with the balanced schedule a
//     CTA cuts its own equal share of all entries' key blocks out of the
//     sequence lengths (compute_share), with an explicit split count it
//     takes the reference's fixed partitions round-robin;
//   * K and V tiles of 128 tokens arrive by TMA, one box per page (64 dims x
//     min(page, 128) rows, 128-byte swizzle), each into its own ring; boxes
//     outside the piece or past the sequence end are requested at an
//     out-of-range page coordinate, which the TMA unit fills with zeros
//     without touching HBM;
//   * Q and P live in TMEM and are the A operand of tcgen05.mma (M = 128):
//     only the group's rows carry data, so the padding costs tensor-pipe
//     time, of which a decode has plenty, and no shared memory;
//   * S (two 128-column buffers, P written over S in place) and O (D
//     columns) accumulate in TMEM.
//
// Row warps (0-3) own the query rows.  With R = group * m_q rows, each query
// row is held by kC = 4 / ceil(R / 32) warps ("copies", kC in {1, 2, 4}):
// copy c takes tile columns [c * 128 / kC, (c + 1) * 128 / kC) and keeps its
// own running maximum, row sum and O row (its P row is zero outside its
// columns), so four warps share the softmax of a small group and the
// exponentials run on all four SM sub-partitions.  The copies are merged
// once per piece in shared memory (the reference's split merge algebra,
// split_kv.py:198-228).  Warp 4 is the TMA producer, warp 5 issues the MMAs.
//
// Every mbarrier wait is bounded (common.cuh); a timeout sets the device
// status word and the kernel unwinds instead of hanging.
#include "common.cuh"
#include "flagattn_b200.h"

namespace fa {
namespace gqa {

constexpr int kThreads = 192;                // warps 0-3 rows, 4 producer, 5 MMA
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;    // log2 units (factor 256)
constexpr int kMaxStages = 12;

// Tokens per tile (QK N, PV K) for head size d and `rows` query rows per kv
// head: 128; 64 for head size 256, where O (256 TMEM columns), two S / P
// buffers and one Q buffer fill the 512 columns; 192 for head sizes up to 64
// with at most 64 rows (two or four row copies), whose tiles carry few bytes
// and are paced by per-tile latency (O, two 192-column S / P buffers and two
// Q buffers still fit; with one copy a 192-column row would spill).
__host__ __device__ constexpr int tile_tokens(int d, int rows) {
  return d == 256 ? 64 : (d <= 64 && rows <= 64 ? 192 : 128);
}
// the tile of a kernel instance with kC copies of each row
__host__ __device__ constexpr int tile_of(int d, int kC) { return tile_tokens(d, kC >= 2 ? 64 : 128); }
// Rows of one TMA box: a whole page up to the tile (pages divide it), or 64
// rows for 192-token tiles over pages of 64 tokens or more.
__host__ __device__ constexpr int box_rows_for(int tile, int page) {
  return tile == 192 ? (page < 64 ? page : 64) : (page < tile ? page : tile);
}

template <int kD, int kTileTokens>
struct Plan {
  static constexpr int kTile = kTileTokens;
  // a chunk: up to 64 dims of every tile row, one swizzle row of kRowBytes
  // (128; 64 / 32 for head sizes 32 / 16, with the matching swizzle)
  static constexpr int kChunkDims = kD < 64 ? kD : 64;
  static constexpr int kRowBytes = 2 * kChunkDims;
  static constexpr int kChunks = kD / kChunkDims;
  static constexpr int kChunkBytes = kTile * kRowBytes;
  static constexpr int kTileBytes = kChunks * kChunkBytes;       // 4 to 32 KB
  static constexpr uint32_t kSwizzle = smem_swizzle_code(kRowBytes);
  static constexpr uint32_t kAtomBytes = 8 * kRowBytes;          // 8-row swizzle atom
  // per ring: 3 for heads 128 / 256, else up to 12 stages of 96 KB in all
  static constexpr int kStages =
      kD >= 128 ? 3 : (98304 / kTileBytes < kMaxStages ? 98304 / kTileBytes : kMaxStages);
  static constexpr int kQBufs = kD == 256 ? 1 : 2;               // Q buffers in TMEM
  static constexpr int kOffK = 1024;
  static constexpr int kOffV = kOffK + kStages * kTileBytes;
  static constexpr int kOffStage = kOffV + kStages * kTileBytes;  // copy merge: [warp][lane][33] f32
  static constexpr int kStageBytes = 4 * 32 * 33 * 4;
  static constexpr int kOffStats = kOffStage + kStageBytes;      // [2][warp][lane] f32
  static constexpr int kSmemUsed = kOffStats + 2 * 4 * 32 * 4;
  static constexpr int kSmemBytes = kSmemUsed + 1024;            // base alignment slack
  // TMEM columns: O, two S / P buffers, Q buffers (bf16 / f16 pairs)
  static constexpr uint32_t kColO = 0;
  static constexpr uint32_t kColS = kD < 64 ? 64 : kD;
  static constexpr uint32_t kColQ = kColS + 2 * kTile;
  static_assert(kColQ + kQBufs * kD / 2 <= kTmemCols, "TMEM plan");
  static_assert(kStages <= kMaxStages, "ring");
  static_assert(kSmemBytes <= 232448, "shared memory plan exceeds 227 KB");
  static_assert(kOffK % 1024 == 0 && kOffV % 1024 == 0 && kTileBytes % 1024 == 0,
                "swizzled tiles need 1024-byte alignment");
};

// Balanced schedule: the cost line of all entries (entry e = sequence b *
// kv_heads + kv head; cost 1 + blocks(len_b) units, the unit before an
// entry's blocks standing for its per-piece overhead) is cut into `parts`
// equal shares; CTA p takes units [a0, a1) = [p T / parts, (p + 1) T / parts).
struct Share {
  long long a0, a1;     // this CTA's units
  long long x_lo;       // first unit of entry e_lo
  long long total;      // T
  int e_lo, e_hi;       // entries overlapping [a0, a1) (e_hi < e_lo: none)
  int parts;            // CTAs with work: min(gridDim.x, T)
};

struct Bars {
  uint64_t k_full[kMaxStages], k_empty[kMaxStages];
  uint64_t v_full[kMaxStages], v_empty[kMaxStages];
  uint64_t s_full[2];   // QK of a tile landed in S buffer (tile & 1)
  uint64_t p_full[2];   // the row warps wrote P over that buffer (and rescaled O)
  uint64_t q_full[2];   // the row warps wrote a piece's Q into TMEM buffer (piece & 1)
  uint64_t pv_done;     // one phase per tile, in tile order
  uint64_t merge;       // the row warps' meeting point when copies merge (4 arrivals)
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  long long warp_sum[kThreads / 32];
  Share share;
};
static_assert(sizeof(Bars) <= 1024, "barrier block");

struct Params {
  const void *q;
  int64_t q_sb, q_sh, q_sm;
  const int32_t *block_table;  // nullptr: contiguous [batch][n][kv heads] via strides
  int64_t bt_stride;
  int32_t page_size, num_pages, box_rows;
  const int32_t *seq_lens;     // nullptr: every sequence has n_ctx tokens
  int32_t n_ctx;
  int32_t batch, hq, hkv, group, m_q, rows, causal;
  int32_t tile_n;              // tokens per tile (tile_tokens): the schedule's block
  // pair != 0: an entry covers two adjacent kv heads (hkv and group above are
  // the halved / doubled counts; pair_group is one head's group), each TMA
  // box brings both heads' rows of a page, and a tile holds tile_n tokens of
  // each head (tile columns [box][head][row])
  int32_t pair, pair_group;
  float scale_log2;
  // num_splits == 0: the balanced schedule (Share); a split entry's pieces
  // go to slot parts + p (its first piece, in CTA p) and slots p (every
  // later piece, in CTA p), and the CTA holding an entry's first piece
  // writes merge[e] = {first slot or -1 when unsplit, first later slot,
  // number of later slots}.  num_splits >= 1: the reference's fixed
  // partitions, part = entry * num_splits + split (partition_size tokens),
  // taken round-robin; slot = part.
  int32_t num_splits, partition_size, num_parts;
  int4 *merge;
  void *o;
  int64_t o_sb, o_sh, o_sm;
  float *lse;       // nullable, [batch][hq][m_q]
  void *part_o;     // [slot][rows][d], element type T
  float *part_lse;  // [slot][rows]
  int *status;
};

struct Piece {
  int e, b, kvh, tok0, tok_end, len, slot;
  bool present;     // the walk's entry has a piece in this CTA
  bool final_out;   // written straight to the output
  bool entry_first; // holds the entry's first block (or the entry is empty)
  int p_lo, p_hi;   // CTAs holding the entry's first / last block (balanced)
  __device__ __forceinline__ int tiles(int tile) const {
    return tok_end > tok0 ? (tok_end - (tok0 - tok0 % tile) + tile - 1) / tile : 0;
  }
};

__device__ __forceinline__ int seq_len_of(const Params &p, int b) {
  return p.seq_lens ? __ldg(p.seq_lens + b) : p.n_ctx;
}
__device__ __forceinline__ int blocks_of(int len, int tile) {
  return len > 0 ? (len + tile - 1) / tile : 0;
}

// The CTA's share of the balanced schedule.  All threads take part: a block
// scan of the per-sequence costs into `scan` (shared memory not yet used by
// the TMA rings), then thread 0 locates the entries at both ends of the
// share by binary search.  Ends with __syncthreads.
__device__ __noinline__ void compute_share(const Params &p, long long *scan, Bars *bars) {
  const int B = p.batch, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (B + kThreads - 1) / kThreads;
  const int b0 = min(B, tid * per), b1 = min(B, b0 + per);
  long long local = 0;
  for (int b = b0; b < b1; ++b) local += 1 + blocks_of(seq_len_of(p, b), p.tile_n);
  long long incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) bars->warp_sum[warp] = incl;
  __syncthreads();
  long long run = incl - local;
  for (int w = 0; w < warp; ++w) run += bars->warp_sum[w];
  for (int b = b0; b < b1; ++b) {
    scan[b] = run;
    run += 1 + blocks_of(seq_len_of(p, b), p.tile_n);
  }
  if (b1 == B && b0 < b1) scan[B] = run;
  if (B == 0 && tid == 0) scan[0] = 0;
  __syncthreads();
  if (tid == 0) {
    Share sh;
    const long long hkv = p.hkv;
    sh.total = hkv * scan[B];
    sh.parts = static_cast<int>(min(static_cast<long long>(gridDim.x), sh.total));
    sh.e_lo = 0;
    sh.e_hi = -1;
    sh.x_lo = sh.a0 = sh.a1 = 0;
    if (static_cast<int>(blockIdx.x) < sh.parts) {
      sh.a0 = blockIdx.x * sh.total / sh.parts;
      sh.a1 = (blockIdx.x + 1) * sh.total / sh.parts;
      // entry holding unit u: sequence b = last with hkv * scan[b] <= u
      auto locate = [&](long long u, int &e, long long &x) {
        int lo = 0, hi = B - 1;
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (hkv * scan[mid] <= u) lo = mid; else hi = mid - 1;
        }
        const long long c = scan[lo + 1] - scan[lo];
        const long long h = (u - hkv * scan[lo]) / c;
        e = lo * p.hkv + static_cast<int>(h);
        x = hkv * scan[lo] + h * c;
      };
      long long x_hi;
      locate(sh.a0, sh.e_lo, sh.x_lo);
      locate(sh.a1 - 1, sh.e_hi, x_hi);
    }
    bars->share = sh;
  }
  __syncthreads();
}

// Position in the CTA's stream of pieces: balanced, entry e starting at unit
// x (entries e_lo .. e_hi); fixed partitions, part (blockIdx.x, + gridDim.x,
// ...).
struct Cursor {
  int e;
  long long x;
  int part;
};

__device__ __forceinline__ Cursor first_cursor(const Params &p, const Share *sh) {
  return p.num_splits == 0 ? Cursor{sh->e_lo, sh->x_lo, 0}
                           : Cursor{0, 0, static_cast<int>(blockIdx.x)};
}
__device__ __forceinline__ bool valid(const Params &p, const Share *sh, const Cursor &c) {
  return p.num_splits == 0 ? c.e <= sh->e_hi : c.part < p.num_parts;
}
__device__ __forceinline__ void advance(const Params &p, Cursor &c) {
  if (p.num_splits == 0) {
    c.x += 1 + blocks_of(seq_len_of(p, c.e / p.hkv), p.tile_n);
    ++c.e;
  } else {
    c.part += gridDim.x;
  }
}

__device__ __noinline__ Piece get_piece(const Params &p, const Share *sh, Cursor c) {
  Piece pc;
  if (p.num_splits == 0) {
    pc.e = c.e;
    pc.b = c.e / p.hkv;
    pc.len = max(seq_len_of(p, pc.b), 0);
    const int nb = blocks_of(pc.len, p.tile_n);
    // blocks of this entry inside [a0, a1): block j sits at unit x + 1 + j
    const long long j0 = min(max(sh->a0 - c.x - 1, 0ll), static_cast<long long>(nb));
    const long long j1 = min(max(sh->a1 - c.x - 1, 0ll), static_cast<long long>(nb));
    pc.present = nb > 0 ? j1 > j0 : c.x >= sh->a0;
    pc.tok0 = static_cast<int>(j0) * p.tile_n;
    pc.tok_end = min(static_cast<int>(j1) * p.tile_n, pc.len);
    auto part_of = [&](long long u) {
      return static_cast<int>(min(static_cast<long long>(sh->parts - 1),
                                  ((u + 1) * sh->parts + sh->total - 1) / sh->total - 1));
    };
    pc.p_lo = nb > 0 ? part_of(c.x + 1) : static_cast<int>(blockIdx.x);
    pc.p_hi = nb > 0 ? part_of(c.x + nb) : static_cast<int>(blockIdx.x);
    pc.entry_first = j0 == 0;
    pc.final_out = pc.p_lo == pc.p_hi;
    pc.slot = pc.entry_first ? sh->parts + static_cast<int>(blockIdx.x) : static_cast<int>(blockIdx.x);
  } else {
    pc.e = c.part / p.num_splits;
    pc.b = pc.e / p.hkv;
    const int split = c.part % p.num_splits;
    pc.len = max(seq_len_of(p, pc.b), 0);
    if (p.num_splits == 1) {
      pc.tok0 = 0;
      pc.tok_end = pc.len;
    } else {
      pc.tok0 = split * p.partition_size;
      pc.tok_end = min(pc.len, pc.tok0 + p.partition_size);
    }
    pc.present = true;
    pc.entry_first = split == 0;
    pc.final_out = p.num_splits == 1;
    pc.p_lo = pc.p_hi = 0;
    pc.slot = c.part;
  }
  pc.kvh = pc.e % p.hkv;
  return pc;
}

// Next piece with at least one tile (the Q buffers alternate over those).
__device__ __forceinline__ void next_with_tiles(const Params &p, const Share *sh, Cursor &c) {
  while (valid(p, sh, c)) {
    const Piece pc = get_piece(p, sh, c);
    if (pc.present && pc.tiles(p.tile_n) > 0) return;
    advance(p, c);
  }
}

// Warp-wide bounded wait: all lanes return the same verdict.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                          int *status, int code) {
  if (mbar_probe(bar, parity)) return true;
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, status, code)) != 0;
}

// ------------------------------------------------------------------ rows
// Query row r of an entry: head kvh * group + r / m_q, query token r % m_q.
template <typename T, int kD>
__device__ __forceinline__ void write_q(const Params &p, const Piece &pc, bool live, int g_idx,
                                        int m_idx, uint32_t t_q, uint32_t bar, int lane) {
  const int h = pc.kvh * p.group + g_idx;
  const uint4 *src = reinterpret_cast<const uint4 *>(
      static_cast<const T *>(p.q) + pc.b * p.q_sb + h * p.q_sh + m_idx * p.q_sm);
  // up to 64 dims (32 packed words) at a time: a 256-wide row would hold
  // 128 registers at once
  constexpr int kW = kD >= 64 ? 32 : kD / 2;
#pragma unroll
  for (int j = 0; j < kD / 2 / kW; ++j) {
    uint32_t w[kW];
#pragma unroll
    for (int i = 0; i < kW / 4; ++i) {
      const uint4 v = live ? __ldg(src + (kW / 4) * j + i) : make_uint4(0u, 0u, 0u, 0u);
      w[4 * i] = v.x;
      w[4 * i + 1] = v.y;
      w[4 * i + 2] = v.z;
      w[4 * i + 3] = v.w;
    }
    if constexpr (kW == 32)
      tmem_st32(t_q + kW * j, w);
    else if constexpr (kW == 16)
      tmem_st16p(t_q + kW * j, w);
    else
      tmem_st8p(t_q + kW * j, w);
  }
  tmem_wait_st();
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
}

// Barrier of the four row warps on an mbarrier (bounded, unlike bar.sync:
// a warp that unwound after a timeout cannot leave the others stuck).
struct RowSync {
  uint32_t bar, phase = 0;
  __device__ __forceinline__ bool sync(volatile int *abort_flag, int *status) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
    const bool ok = warp_wait(bar, phase & 1u, abort_flag, status, kDevTimeoutSoftmax);
    ++phase;
    return ok;
  }
};

// Normalised rows of one piece into the output (final) or a split slot.
// kC == 1: each lane writes its own row.  kC > 1: the copies of a row meet in
// shared memory, 32 columns at a time; thread (warp w, lane j) then writes
// column j of rows w, w + 4, ...
template <typename T, int kD, int kC>
__device__ __forceinline__ bool epilogue(const Params &p, const Piece &pc, bool has_tiles,
                                         bool live, int r, int g_idx, int m_idx, int warp,
                                         int lane, int quads, float m_use, float l,
                                         uint32_t t_o, float *stage, float *stat_m,
                                         float *stat_l, RowSync &rs, volatile int *abort_flag) {
  constexpr float kLn2 = 0.6931471805599453f;
  float f, lse;
  if (kC == 1) {
    f = l > 0.f ? 1.f / l : 0.f;
    lse = l > 0.f ? (m_use + __log2f(l)) * kLn2 : -INFINITY;
  } else {
    stat_m[warp * 32 + lane] = live ? m_use : -INFINITY;
    stat_l[warp * 32 + lane] = live ? l : 0.f;
    if (!rs.sync(abort_flag, p.status)) return false;
    const int q = warp % quads;
    float M = -INFINITY;
#pragma unroll
    for (int c = 0; c < kC; ++c) M = fmaxf(M, stat_m[(c * quads + q) * 32 + lane]);
    float L = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int c = 0; c < kC; ++c) {
        const float mc = stat_m[(c * quads + q) * 32 + lane];
        L += mc == -INFINITY ? 0.f : stat_l[(c * quads + q) * 32 + lane] * fast_exp2(mc - M);
      }
    }
    f = (L > 0.f && m_use != -INFINITY) ? fast_exp2(m_use - M) / L : 0.f;
    lse = L > 0.f ? (M + __log2f(L)) * kLn2 : -INFINITY;
  }
  const int h = pc.kvh * p.group + g_idx;
  // final rows go to the output, split rows to their slot; both in T
  T *orow = pc.final_out
                ? static_cast<T *>(p.o) + pc.b * p.o_sb + h * p.o_sh + m_idx * p.o_sm
                : static_cast<T *>(p.part_o) + (static_cast<int64_t>(pc.slot) * p.rows + r) * kD;
  constexpr int kOG = kD < 32 ? kD : 32;  // output columns per TMEM load
#pragma unroll 1
  for (int j = 0; j < kD / kOG; ++j) {
    float v[kOG];
    if (has_tiles) {
      if constexpr (kOG == 32)
        tmem_ld32(t_o + 32 * j, v);
      else
        tmem_ld16(t_o + kOG * j, v);
      tmem_wait_ld();
    } else {
#pragma unroll
      for (int i = 0; i < kOG; ++i) v[i] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < kOG; ++i) v[i] *= f;
    if (kC == 1) {
      if (live) {
        uint4 *dst = reinterpret_cast<uint4 *>(orow + kOG * j);
#pragma unroll
        for (int i = 0; i < kOG / 8; ++i) {
          uint4 u;
          u.x = Elem<T>::pack2(v[8 * i], v[8 * i + 1]);
          u.y = Elem<T>::pack2(v[8 * i + 2], v[8 * i + 3]);
          u.z = Elem<T>::pack2(v[8 * i + 4], v[8 * i + 5]);
          u.w = Elem<T>::pack2(v[8 * i + 6], v[8 * i + 7]);
          dst[i] = u;
        }
      }
    } else {
      float *mine = stage + (warp * 32 + lane) * 33;
#pragma unroll
      for (int i = 0; i < kOG; ++i) mine[i] = v[i];
      if (!rs.sync(abort_flag, p.status)) return false;
      for (int rr = warp; rr < p.rows && lane < kOG; rr += 4) {
        const int q = rr >> 5, i = rr & 31;
        float sum = 0.f;
#pragma unroll
        for (int c = 0; c < kC; ++c) sum += stage[((c * quads + q) * 32 + i) * 33 + lane];
        const int g2 = rr / p.m_q, m2 = rr % p.m_q;
        T *o2 = pc.final_out
                    ? static_cast<T *>(p.o) + pc.b * p.o_sb + (pc.kvh * p.group + g2) * p.o_sh +
                          m2 * p.o_sm
                    : static_cast<T *>(p.part_o) + (static_cast<int64_t>(pc.slot) * p.rows + rr) * kD;
        o2[kOG * j + lane] = Elem<T>::from_f(sum);
      }
      if (!rs.sync(abort_flag, p.status)) return false;
    }
  }
  const bool writer = live && (kC == 1 || warp < quads);
  if (writer) {
    if (pc.final_out) {
      if (p.lse) p.lse[(static_cast<int64_t>(pc.b) * p.hq + h) * p.m_q + m_idx] = lse;
    } else {
      p.part_lse[static_cast<int64_t>(pc.slot) * p.rows + r] = lse;
    }
  }
  tc_fence_before();  // the O reads above precede the next piece's first PV
  return true;
}

template <typename T, int kD, int kC>
__device__ __forceinline__ void row_role(const Params &p, Bars *bars, uint8_t *smem,
                                         uint32_t tmem, int warp, int lane) {
  using PL = Plan<kD, tile_of(kD, kC)>;
  constexpr int kCols = PL::kTile / kC;  // tile columns of one copy
  constexpr int kWords = kCols / 2;    // packed P words of one copy
  volatile int *abort_flag = &bars->abort_flag;
  const int quads = kC == 1 ? (p.rows + 31) / 32 : 4 / kC;
  if (warp >= quads * kC) return;      // kC == 1 with three quadrants: warp 3 idles
  const int copy = warp / quads;
  const int r = (warp % quads) * 32 + lane;
  const bool live = r < p.rows;
  const int g_idx = live ? r / p.m_q : 0;
  const int m_idx = live ? r % p.m_q : 0;
  // paired kv heads reach only heads 128 / 256 with two or more copies
  // (gqa_pairs_heads); other instances compile without that code
  constexpr bool kPairable = kC >= 2 && (kD == 128 || kD == 256);
  const int pair = kPairable ? p.pair : 0;
  const int hh_r = pair && live ? g_idx / p.pair_group : 0;  // head of the row within its pair
  // paired: bit j set where this copy's column j holds the row's own head
  // (column cj: box cj >> (lgR + 1), head (cj >> lgR) & 1, paired pages
  // hold 16 or 32 tokens); every bit for rows past the group
  const int lgR = pair ? __ffs(p.box_rows) - 1 : 0;
  uint64_t own = ~0ull;
  if (pair && live) {
    own = 0;
#pragma unroll
    for (int j = 0; j < (kCols < 64 ? kCols : 64); ++j)
      own |= static_cast<uint64_t>((((copy * kCols + j) >> lgR) & 1) == hh_r) << j;
  }
  const int tt = p.tile_n;                                    // tokens per tile
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t t_o = tmem + lane_off + PL::kColO;
  float *stage = reinterpret_cast<float *>(smem + PL::kOffStage);
  float *stat_m = reinterpret_cast<float *>(smem + PL::kOffStats);
  float *stat_l = stat_m + 128;
  const uint32_t vbase = smem_u32(smem + PL::kOffV);
  RowSync rs{smem_u32(&bars->merge)};

  const Share *sh = &bars->share;
  Cursor cur = first_cursor(p, sh);
  next_with_tiles(p, sh, cur);  // first piece that has tiles: its Q goes first
  uint32_t g = 0;               // tiles so far
  uint32_t k = 0;               // pieces with tiles so far
  if (valid(p, sh, cur))
    write_q<T, kD>(p, get_piece(p, sh, cur), live, g_idx, m_idx, tmem + lane_off + PL::kColQ,
                   smem_u32(&bars->q_full[0]), lane);
  bool ok = true;
  for (Cursor c = first_cursor(p, sh); valid(p, sh, c) && ok; advance(p, c)) {
    const Piece pc = get_piece(p, sh, c);
    if (!pc.present) continue;
    const int n_tiles = pc.tiles(p.tile_n);
    if (PL::kQBufs == 2 && n_tiles > 0) {
      // Q of the next piece with tiles, into the other buffer: its previous
      // user (two pieces back) finished all QKs before this piece started
      Cursor nq = c;
      advance(p, nq);
      next_with_tiles(p, sh, nq);
      if (valid(p, sh, nq))
        write_q<T, kD>(p, get_piece(p, sh, nq), live, g_idx, m_idx,
                       tmem + lane_off + PL::kColQ + ((k + 1) & 1) * (kD / 2),
                       smem_u32(&bars->q_full[(k + 1) & 1]), lane);
    }
    // valid tokens of this row: [tok0, hi_tok); causal rows stop at
    // m + len - m_q (bottom-right alignment, split_kv.py:88-92)
    const int row_end = p.causal ? min(pc.tok_end, m_idx + pc.len - p.m_q + 1) : pc.tok_end;
    float m_use = -INFINITY, l = 0.f;
    int n0 = pc.tok0 - pc.tok0 % tt;
    for (int t = 0; t < n_tiles; ++t, ++g, n0 += tt) {
      const uint32_t buf = g & 1u;
      if (!(ok = warp_wait(smem_u32(&bars->s_full[buf]), (g >> 1) & 1u, abort_flag, p.status,
                           kDevTimeoutSoftmax)))
        break;
      tc_fence_after();
      const uint32_t t_s = tmem + lane_off + PL::kColS + buf * PL::kTile;
      float s[kCols];
#pragma unroll
      for (int j = 0; j < kCols / 32; ++j) tmem_ld32(t_s + copy * kCols + 32 * j, s + 32 * j);
      if constexpr (kCols % 32 == 16)
        tmem_ld16(t_s + copy * kCols + kCols - 16,
                  *reinterpret_cast<float(*)[16]>(s + kCols - 16));
      tmem_wait_ld();
      // rows past the group (zero Q, so S = 0) count as fully valid: their
      // P and O rows are never read
      const int c0 = n0 + copy * kCols;
      const int lo = live ? pc.tok0 - c0 : 0;
      const int hi = live ? row_end - c0 : kCols;
      float mx = -INFINITY;
      if (pair) {
        if (__all_sync(0xffffffffu, !live || (n0 >= pc.tok0 && n0 + tt <= row_end))) {
#pragma unroll
          for (int j = 0; j < kCols; ++j) {
            s[j] = (j < 64 && ((own >> j) & 1)) ? s[j] : -INFINITY;  // select: NaN-safe
            mx = fmaxf(mx, s[j]);
          }
        } else {
          // token of column cj: n0 + box * R + (cj & (R - 1))
#pragma unroll
          for (int j = 0; j < kCols; ++j) {
            const int cj = copy * kCols + j;
            const int tok = n0 + ((cj >> (lgR + 1)) << lgR) + (cj & (p.box_rows - 1));
            const bool ok_j =
                !live || (j < 64 && ((own >> j) & 1) && tok >= pc.tok0 && tok < row_end);
            s[j] = ok_j ? s[j] : -INFINITY;  // select: NaN-safe
            mx = fmaxf(mx, s[j]);
          }
        }
      } else if (__all_sync(0xffffffffu, lo <= 0 && hi >= kCols)) {
#pragma unroll
        for (int j = 0; j < kCols; j += 2) mx = fmax3(mx, s[j], s[j + 1]);
      } else {
#pragma unroll
        for (int j = 0; j < kCols; ++j) {
          s[j] = (j >= lo && j < hi) ? s[j] : -INFINITY;  // select: NaN-safe
          mx = fmaxf(mx, s[j]);
        }
      }
      const float m_tile = mx * p.scale_log2;
      bool resc = false;
      float alpha = 1.f;
      if (t == 0) {
        m_use = m_tile;
      } else if (m_tile > m_use + kRescaleThreshold) {
        alpha = m_use == -INFINITY ? 0.f : fast_exp2(m_use - m_tile);
        resc = m_use != -INFINITY;  // O is all zeros while nothing was valid
        l *= alpha;
        m_use = m_tile;
      }
      const float msafe = m_use == -INFINITY ? 0.f : m_use;
      const uint64_t c2 = f32x2(p.scale_log2, p.scale_log2);
      const uint64_t nm2 = f32x2(-msafe, -msafe);
      uint32_t w[kWords];
      uint64_t acc2 = f32x2(0.f, 0.f);
#pragma unroll
      for (int j = 0; j < kWords; ++j) {
        float x0, x1;
        f32x2_split(ffma2(f32x2(s[2 * j], s[2 * j + 1]), c2, nm2), x0, x1);
        const float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
        acc2 = fadd2(acc2, f32x2(p0, p1));
        w[j] = Elem<T>::pack2(p0, p1);
      }
      float a0, a1;
      f32x2_split(acc2, a0, a1);
      l += a0 + a1;
      // P over the S buffer: this copy's words, zeros over the other copies'
      auto st_words = [&](uint32_t addr, const uint32_t *src) {  // kWords words
        constexpr int n32 = kWords / 32, rem = kWords % 32;
#pragma unroll
        for (int j = 0; j < n32; ++j) tmem_st32(addr + 32 * j, src + 32 * j);
        if constexpr (rem >= 16) tmem_st16p(addr + 32 * n32, src + 32 * n32);
        if constexpr (rem % 16 == 8) tmem_st8p(addr + kWords - 8, src + kWords - 8);
      };
      st_words(t_s + copy * kWords, w);
      if constexpr (kC > 1) {
        uint32_t z[kWords];
#pragma unroll
        for (int j = 0; j < kWords; ++j) z[j] = 0u;
#pragma unroll
        for (int cc = 1; cc < kC; ++cc) st_words(t_s + ((copy + cc) % kC) * kWords, z);
      }
      if (t > 0) {
        // PV of the previous tile must be complete before O is rescaled
        // (every row warp waits on every pv_done phase, in tile order)
        if (!(ok = warp_wait(smem_u32(&bars->pv_done), (g - 1) & 1u, abort_flag, p.status,
                             kDevTimeoutSoftmax)))
          break;
        if (__any_sync(0xffffffffu, resc)) {
          tc_fence_after();
          const float a = resc ? alpha : 1.f;
          constexpr int kOG = kD < 32 ? kD : 32;
#pragma unroll 1
          for (int j = 0; j < kD / kOG; ++j) {
            float v[kOG];
            uint32_t u[kOG];
            if constexpr (kOG == 32)
              tmem_ld32(t_o + 32 * j, v);
            else
              tmem_ld16(t_o + kOG * j, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < kOG; ++i) u[i] = __float_as_uint(v[i] * a);
            if constexpr (kOG == 32)
              tmem_st32(t_o + 32 * j, u);
            else
              tmem_st16(t_o + kOG * j, u);
          }
        }
      }
      // Value rows past the sequence end inside the last loaded page may
      // hold any bits (even NaN); P is 0 there but 0 * NaN is not, so clear
      // them before the PV product.
      if (warp == 0 && pc.len > n0 && pc.len < n0 + tt && pc.len <= pc.tok_end) {
        const int jb = (pc.len - 1 - n0) / p.box_rows;
        const int r0 = pc.len - n0, r1 = (jb + 1) * p.box_rows;
        const int btok = n0 + jb * p.box_rows;
        if (r1 > r0 && btok < pc.tok_end && btok + p.box_rows > pc.tok0) {
          const uint32_t st = g % PL::kStages;
          if (!(ok = warp_wait(smem_u32(&bars->v_full[st]), (g / PL::kStages) & 1u, abort_flag,
                               p.status, kDevTimeoutSoftmax)))
            break;
          const uint32_t tile = vbase + st * PL::kTileBytes;
          constexpr int kUnits = PL::kRowBytes / 16;  // 16-byte units per chunk row
          const int units = (r1 - r0) * kUnits;
          // paired heads: the box's rows are [head][row], cleared for both
          const int row0 = pair ? 2 * jb * p.box_rows + (r0 - jb * p.box_rows) : r0;
          for (int u = lane; u < units * PL::kChunks << pair; u += 32) {
            const int hh = u / (units * PL::kChunks), uu = u % (units * PL::kChunks);
            const int ch = uu / units, rem = uu % units;
            const uint32_t addr = tile + ch * PL::kChunkBytes +
                                  (row0 + hh * p.box_rows + rem / kUnits) * PL::kRowBytes +
                                  (rem % kUnits) * 16;
            asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0u)
                         : "memory");
          }
          fence_proxy_async_smem();
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars->p_full[buf]));
    }
    if (!ok) break;
    if (PL::kQBufs == 1 && n_tiles > 0) {
      // one Q buffer (head size 256): the next piece's Q goes in once every
      // score product of this piece has completed (each s_full was waited)
      Cursor nq = c;
      advance(p, nq);
      next_with_tiles(p, sh, nq);
      if (valid(p, sh, nq))
        write_q<T, kD>(p, get_piece(p, sh, nq), live, g_idx, m_idx, tmem + lane_off + PL::kColQ,
                       smem_u32(&bars->q_full[0]), lane);
    }
    if (n_tiles > 0) {
      if (!(ok = warp_wait(smem_u32(&bars->pv_done), (g - 1) & 1u, abort_flag, p.status,
                           kDevTimeoutSoftmax)))
        break;
      tc_fence_after();
      ++k;
    }
    if (!(ok = epilogue<T, kD, kC>(p, pc, n_tiles > 0, live, r, g_idx, m_idx, warp, lane, quads,
                                   m_use, l, t_o, stage, stat_m, stat_l, rs, abort_flag)))
      break;
  }
}

// ------------------------------------------------------------------ kernel
template <typename T, int kD, int kC>
__global__ void __launch_bounds__(kThreads, 1)
    gqa_decode_kernel(const __grid_constant__ CUtensorMap k_map,
                      const __grid_constant__ CUtensorMap v_map,
                      const __grid_constant__ Params p) {
  using PL = Plan<kD, tile_of(kD, kC)>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  if (smem + PL::kSmemUsed > smem_raw + PL::kSmemBytes) {
    if (threadIdx.x == 0 && p.status) atomicExch(p.status, kDevBadSmemAlign);
    return;
  }
  Bars *bars = reinterpret_cast<Bars *>(smem);
  volatile int *abort_flag = &bars->abort_flag;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr int fmt = std::is_same<T, __half>::value ? 0 : 1;
  const int quads = kC == 1 ? (p.rows + 31) / 32 : 4 / kC;
  const uint32_t row_warps = static_cast<uint32_t>(quads * kC);

  if (threadIdx.x == 0) {
    for (int i = 0; i < PL::kStages; ++i) {
      mbar_init(smem_u32(&bars->k_full[i]), 1);
      mbar_init(smem_u32(&bars->k_empty[i]), 1);
      mbar_init(smem_u32(&bars->v_full[i]), 1);
      mbar_init(smem_u32(&bars->v_empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&bars->s_full[i]), 1);
      mbar_init(smem_u32(&bars->p_full[i]), row_warps);
      mbar_init(smem_u32(&bars->q_full[i]), row_warps);
    }
    mbar_init(smem_u32(&bars->pv_done), 1);
    mbar_init(smem_u32(&bars->merge), 4);
    mbar_init(smem_u32(&bars->drain), 1);
    bars->abort_flag = 0;
    bars->share = Share{0, 0, 0, 0, 0, -1, 0};
    fence_barrier_init();
  }
  if (warp == kProducerWarp && lane == 0) {
    tma_prefetch_desc(&k_map);
    tma_prefetch_desc(&v_map);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(&bars->tmem_base), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  // The schedule comes from the kernel this one may overlap (programmatic
  // dependent launch); wait for it before the first metadata read, then let
  // the merge kernel queued behind this one launch.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (p.num_splits == 0) {
    // the rings are still empty: the schedule's scan uses their space, and
    // the TMA writes that follow are ordered after it
    compute_share(p, reinterpret_cast<long long *>(smem + PL::kOffK), bars);
    fence_proxy_async_smem();
  }

  if (warp < 4) {
    row_role<T, kD, kC>(p, bars, smem, tmem, warp, lane);
  } else if (warp == kProducerWarp) {
    // ------------------------------------------------------- TMA producer
    const uint32_t kbase = smem_u32(smem + PL::kOffK), vbase = smem_u32(smem + PL::kOffV);
    const int tt = p.tile_n;            // tokens per tile
    const int nbox = tt / p.box_rows;
    uint32_t g = 0, gk = 0, gv = 0;  // tiles begun, K tiles issued, V tiles issued
    bool ok = true;
    const Share *sh = &bars->share;
    for (Cursor c = first_cursor(p, sh); valid(p, sh, c) && ok; advance(p, c)) {
      const Piece pc = get_piece(p, sh, c);
      if (!pc.present) continue;
      if (p.num_splits == 0 && pc.entry_first && lane == 0)
        p.merge[pc.e] = make_int4(pc.final_out ? -1 : sh->parts + pc.p_lo, pc.p_lo + 1,
                                  pc.p_hi - pc.p_lo, 0);
      const int n_tiles = pc.tiles(p.tile_n);
      int n0 = pc.tok0 - pc.tok0 % tt;
      // box of lane j: tokens [n0 + j * box_rows, + box_rows); boxes that
      // miss the piece read an out-of-range page (zero fill, no traffic).
      // The page numbers of the next tile are read one tile ahead, so the
      // block-table load's latency overlaps this tile's waits and copies.
      auto box_coord = [&](int base, int &y_out, int &page_out) {
        y_out = 0;
        page_out = p.block_table ? p.num_pages : p.batch;
        if (lane < nbox) {
          const int tok = base + lane * p.box_rows;
          if (tok < pc.tok_end && tok + p.box_rows > pc.tok0) {
            if (p.block_table) {
              page_out = __ldg(p.block_table + pc.b * p.bt_stride + tok / p.page_size);
              y_out = tok % p.page_size;
            } else {
              page_out = pc.b;
              y_out = tok;
            }
          }
        }
      };
      int ny, npage;
      box_coord(n0, ny, npage);
      for (int t = 0; t < n_tiles; ++t, ++g, n0 += tt) {
        const int y = ny, page = npage;
        if (t + 1 < n_tiles) box_coord(n0 + tt, ny, npage);
        const uint32_t st = g % PL::kStages, ph = ((g / PL::kStages) & 1u) ^ 1u;
        if (!(ok = warp_wait(smem_u32(&bars->k_empty[st]), ph, abort_flag, p.status,
                             kDevTimeoutProducer)))
          break;
        const uint32_t kf = smem_u32(&bars->k_full[st]);
        if (lane == 0) mbar_arrive_expect_tx(kf, PL::kTileBytes);
        __syncwarp();
        if (lane < nbox) {
#pragma unroll
          for (int ch = 0; ch < PL::kChunks; ++ch)
            tma_load_4d(kbase + st * PL::kTileBytes + ch * PL::kChunkBytes +
                            lane * (p.box_rows << p.pair) * PL::kRowBytes,
                        &k_map, kf, ch * PL::kChunkDims, y, pc.kvh << p.pair, page);
        }
        ++gk;
        if (!(ok = warp_wait(smem_u32(&bars->v_empty[st]), ph, abort_flag, p.status,
                             kDevTimeoutProducer)))
          break;
        const uint32_t vf = smem_u32(&bars->v_full[st]);
        if (lane == 0) mbar_arrive_expect_tx(vf, PL::kTileBytes);
        __syncwarp();
        if (lane < nbox) {
#pragma unroll
          for (int ch = 0; ch < PL::kChunks; ++ch)
            tma_load_4d(vbase + st * PL::kTileBytes + ch * PL::kChunkBytes +
                            lane * (p.box_rows << p.pair) * PL::kRowBytes,
                        &v_map, vf, ch * PL::kChunkDims, y, pc.kvh << p.pair, page);
        }
        ++gv;
      }
    }
    if (*abort_flag) {
      // copies in flight must land before the CTA may exit: wait (bounded)
      // on the full barrier of every slot filled in the last ring's worth
      volatile int never = 0;
      for (uint32_t t = gk > PL::kStages ? gk - PL::kStages : 0; t < gk; ++t)
        mbar_wait(smem_u32(&bars->k_full[t % PL::kStages]), (t / PL::kStages) & 1u, &never,
                  nullptr, 0);
      for (uint32_t t = gv > PL::kStages ? gv - PL::kStages : 0; t < gv; ++t)
        mbar_wait(smem_u32(&bars->v_full[t % PL::kStages]), (t / PL::kStages) & 1u, &never,
                  nullptr, 0);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------- MMA issuer
    constexpr uint32_t kIdescQK = umma_idesc_f16(128, PL::kTile, fmt, 0);
    constexpr uint32_t kIdescPV = umma_idesc_f16(128, kD, fmt, 1);
    const uint32_t kbase = smem_u32(smem + PL::kOffK), vbase = smem_u32(smem + PL::kOffV);
    const uint64_t k_desc = smem_desc_swz(kbase, 16, PL::kAtomBytes, PL::kSwizzle);
    const uint64_t v_desc = smem_desc_swz(vbase, PL::kChunkBytes, PL::kAtomBytes, PL::kSwizzle);
    uint32_t g = 0, k = 0;
    bool ok = true;
    int pend = -1;             // tile whose PV is still to be issued
    bool pend_first = false;   // ... and whether it opens its piece
    auto issue_pv = [&](uint32_t gp, bool first) -> bool {
      const uint32_t buf = gp & 1u, st = gp % PL::kStages;
      if (!warp_wait(smem_u32(&bars->p_full[buf]), (gp >> 1) & 1u, abort_flag, p.status,
                     kDevTimeoutMma))
        return false;
      if (!warp_wait(smem_u32(&bars->v_full[st]), (gp / PL::kStages) & 1u, abort_flag, p.status,
                     kDevTimeoutMma))
        return false;
      tc_fence_after();
      const uint64_t vd = v_desc + static_cast<uint64_t>((st * PL::kTileBytes) >> 4);
#pragma unroll
      for (int kk = 0; kk < PL::kTile / 16; ++kk)
        umma_ts_warp(tmem + PL::kColO, tmem + PL::kColS + buf * PL::kTile + kk * 8,
                     vd + static_cast<uint64_t>((kk * 16 * PL::kRowBytes) >> 4), kIdescPV,
                     (first && kk == 0) ? 0u : 1u);
      tc_commit_warp(smem_u32(&bars->v_empty[st]));
      tc_commit_warp(smem_u32(&bars->pv_done));
      return true;
    };
    const Share *sh = &bars->share;
    for (Cursor c = first_cursor(p, sh); valid(p, sh, c) && ok; advance(p, c)) {
      const Piece pc = get_piece(p, sh, c);
      if (!pc.present) continue;
      const int n_tiles = pc.tiles(p.tile_n);
      if (n_tiles == 0) continue;
      const uint32_t qb = k % PL::kQBufs;
      if (!(ok = warp_wait(smem_u32(&bars->q_full[qb]), (k / PL::kQBufs) & 1u, abort_flag,
                           p.status, kDevTimeoutMma)))
        break;
      const uint32_t qcol = tmem + PL::kColQ + qb * (kD / 2);
      for (int t = 0; t < n_tiles && ok; ++t, ++g) {
        const uint32_t st = g % PL::kStages;
        if (!(ok = warp_wait(smem_u32(&bars->k_full[st]), (g / PL::kStages) & 1u, abort_flag,
                             p.status, kDevTimeoutMma)))
          break;
        tc_fence_after();
        const uint32_t sd = tmem + PL::kColS + (g & 1u) * PL::kTile;
        const uint64_t kd = k_desc + static_cast<uint64_t>((st * PL::kTileBytes) >> 4);
#pragma unroll
        for (int ch = 0; ch < PL::kChunks; ++ch)
#pragma unroll
          for (int kk = 0; kk < PL::kChunkDims / 16; ++kk)
            umma_ts_warp(sd, qcol + ch * 32 + kk * 8,
                         kd + static_cast<uint64_t>((ch * PL::kChunkBytes + kk * 32) >> 4), kIdescQK,
                         (ch | kk) ? 1u : 0u);
        tc_commit_warp(smem_u32(&bars->k_empty[st]));
        tc_commit_warp(smem_u32(&bars->s_full[g & 1u]));
        // the previous tile's PV goes after this QK, so the tensor pipe
        // computes S of tile g while the row warps still work on tile g - 1
        if (pend >= 0 && !(ok = issue_pv(static_cast<uint32_t>(pend), pend_first))) break;
        pend = static_cast<int>(g);
        pend_first = t == 0;
      }
      ++k;
    }
    if (ok && pend >= 0) ok = issue_pv(static_cast<uint32_t>(pend), pend_first);
    // every issued MMA must finish before TMEM is released
    tc_commit_warp(smem_u32(&bars->drain));
    volatile int never = 0;
    mbar_wait(smem_u32(&bars->drain), 0, &never, p.status, kDevTimeoutDrain);
    __syncwarp();
  }

  // -------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <typename T, int kD, int kC>
cudaError_t launch_t(const CUtensorMap &km, const CUtensorMap &vm, const Params &p, int grid,
                     bool pdl, cudaStream_t stream) {
  auto kern = gqa_decode_kernel<T, kD, kC>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       Plan<kD, tile_of(kD, kC)>::kSmemBytes);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = Plan<kD, tile_of(kD, kC)>::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, km, vm, p);
}

template <typename T, int kD>
cudaError_t launch_d(const CUtensorMap &km, const CUtensorMap &vm, const Params &p, int grid,
                     bool pdl, cudaStream_t stream) {
  if (p.rows <= 32) return launch_t<T, kD, 4>(km, vm, p, grid, pdl, stream);
  if (p.rows <= 64) return launch_t<T, kD, 2>(km, vm, p, grid, pdl, stream);
  if (p.pair) return cudaErrorInvalidValue;  // one-copy instances hold no paired code
  return launch_t<T, kD, 1>(km, vm, p, grid, pdl, stream);
}

}  // namespace gqa

namespace gqa {
int rows_of(const fa_decode_args *a) {
  return a->num_kv_heads > 0 ? (a->num_q_heads / a->num_kv_heads) * a->m_q : 0;
}
// Ring bytes of the instance the arguments select (the balanced schedule's
// scan lives there before the first copy).
template <int kD>
int ring_bytes(int rows) {
  return rows <= 64 ? Plan<kD, tile_tokens(kD, 64)>::kOffStage - Plan<kD, tile_tokens(kD, 64)>::kOffK
                    : Plan<kD, tile_tokens(kD, 128)>::kOffStage -
                          Plan<kD, tile_tokens(kD, 128)>::kOffK;
}
}  // namespace gqa

// Sequences the balanced schedule can scan at once: batch + 1 int64 in the
// (still empty) K and V rings.
int gqa_max_balanced_batch(const fa_decode_args *a) {
  const int rows = gqa::rows_of(a);
  int bytes;
  switch (a->d_qk) {
    case 16: bytes = gqa::ring_bytes<16>(rows); break;
    case 32: bytes = gqa::ring_bytes<32>(rows); break;
    case 64: bytes = gqa::ring_bytes<64>(rows); break;
    case 256: bytes = gqa::ring_bytes<256>(rows); break;
    default: bytes = gqa::ring_bytes<128>(rows); break;
  }
  return bytes / 8 - 1;
}

// Two adjacent kv heads per entry?  For paged head-128 / 256 caches with
// pages of 32 tokens or fewer, each TMA box (one page's rows of one 64-dim
// chunk) holds only 2-4 KB and the TMA unit's box rate, not HBM, paces the
// decode; a box over both heads' rows of a page halves the box count.  The
// tile keeps its rows (and so its bytes and MMA work): half of them per head.
// Needs an even number of kv heads and at most 64 query rows per pair (two
// or more row copies).  `a` describes the real heads.
bool gqa_pairs_heads(const fa_decode_args *a) {
  return a->block_table && (a->d_qk == 128 || a->d_qk == 256) &&
         (a->page_size == 16 || a->page_size == 32) &&
         a->num_kv_heads >= 2 &&
         a->num_kv_heads % 2 == 0 && 2 * gqa::rows_of(a) <= 64;
}

// Tokens per tile and rows per TMA box for the arguments as the kernel sees
// them (`pair`: kv heads already halved): a paired tile holds half its rows'
// worth of tokens of each of its two heads (64 at head 128, 32 at head 256).
int gqa_tile_tokens(const fa_decode_args *a, int pair) {
  return pair ? gqa::tile_tokens(a->d_qk, 128) / 2 : gqa::tile_tokens(a->d_qk, gqa::rows_of(a));
}
int gqa_box_rows(const fa_decode_args *a, int pair) {
  return gqa::box_rows_for(gqa_tile_tokens(a, pair), a->page_size);
}

// The tensor-core kernel serves bf16 / f16 with d_qk == d_v in {16, 32, 64,
// 128, 256}, at most 128 query rows per kv head, a positive scale, 16-byte
// aligned rows and pages of at least 16 tokens that divide the TMA box
// (box_rows_for, which must divide the tile) or are a multiple of it.
bool gqa_tc_eligible(const fa_decode_args *a) {
  auto al16 = [](const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  auto m8 = [](int64_t x) { return x % 8 == 0; };
  if (a->dtype != FA_DTYPE_BF16 && a->dtype != FA_DTYPE_F16) return false;
  const int d = a->d_qk;
  if (a->d_qk != a->d_v || (d != 16 && d != 32 && d != 64 && d != 128 && d != 256)) return false;
  if (a->num_kv_heads <= 0 || a->num_q_heads % a->num_kv_heads) return false;
  const int64_t rows = static_cast<int64_t>(a->num_q_heads / a->num_kv_heads) * a->m_q;
  if (rows < 1 || rows > 128) return false;
  if (!(a->scale > 0.f)) return false;
  if (!al16(a->q) || !al16(a->k) || !al16(a->v) || !al16(a->o)) return false;
  if (!m8(a->q_stride_b) || !m8(a->q_stride_h) || !m8(a->q_stride_m)) return false;
  if (!m8(a->o_stride_b) || !m8(a->o_stride_h) || !m8(a->o_stride_m)) return false;
  if (!m8(a->k_stride_seq) || !m8(a->k_stride_tok) || !m8(a->k_stride_head)) return false;
  if (a->block_table) {
    const int ps = a->page_size;
    if (ps < 16 || ps % 16) return false;
    // boxes tile the tile; pages divide the box or are multiples of it
    const int box = gqa_box_rows(a, 0);
    if (gqa_tile_tokens(a, 0) % box || (ps <= box ? (box % ps) : (ps % box))) return false;
    if (a->num_pages <= 0) return false;
  }
  return true;
}

// Launch the decode for eligible arguments, `a` as the kernel sees them
// (with `pair`, half the kv heads: gqa_pairs_heads).  Balanced schedule
// (a->num_splits == 0): one CTA per part (grid), merge records into `merge`
// (int4 per entry); fixed partitions: num_parts = entries * num_splits.
cudaError_t launch_gqa_tc(const CUtensorMap &km, const CUtensorMap &vm, const fa_decode_args *a,
                          int pair, int4 *merge, int num_parts, int grid, bool pdl,
                          cudaStream_t stream) {
  gqa::Params p;
  p.q = a->q;
  p.q_sb = a->q_stride_b;
  p.q_sh = a->q_stride_h;
  p.q_sm = a->q_stride_m;
  p.block_table = a->block_table;
  p.bt_stride = a->bt_stride;
  p.page_size = a->page_size;
  p.num_pages = a->num_pages;
  p.tile_n = gqa_tile_tokens(a, pair);
  p.box_rows = a->block_table ? gqa_box_rows(a, pair) : p.tile_n;
  p.pair = pair;
  p.pair_group = pair ? a->num_q_heads / a->num_kv_heads / 2 : 0;
  p.seq_lens = a->seq_lens;
  p.n_ctx = a->n_ctx;
  p.batch = a->batch;
  p.hq = a->num_q_heads;
  p.hkv = a->num_kv_heads;
  p.group = a->num_q_heads / a->num_kv_heads;
  p.m_q = a->m_q;
  p.rows = p.group * a->m_q;
  p.causal = a->causal;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  p.merge = merge;
  p.num_parts = num_parts;
  p.num_splits = a->num_splits;
  p.partition_size = a->partition_size;
  p.o = a->o;
  p.o_sb = a->o_stride_b;
  p.o_sh = a->o_stride_h;
  p.o_sm = a->o_stride_m;
  p.lse = a->lse;
  p.part_o = a->part_o;
  p.part_lse = a->part_lse;
  p.status = a->status;
  const bool f16 = a->dtype == FA_DTYPE_F16;
  if (a->d_qk == 64)
    return f16 ? gqa::launch_d<__half, 64>(km, vm, p, grid, pdl, stream)
               : gqa::launch_d<__nv_bfloat16, 64>(km, vm, p, grid, pdl, stream);
  if (a->d_qk == 256)
    return f16 ? gqa::launch_d<__half, 256>(km, vm, p, grid, pdl, stream)
               : gqa::launch_d<__nv_bfloat16, 256>(km, vm, p, grid, pdl, stream);
  if (a->d_qk == 32)
    return f16 ? gqa::launch_d<__half, 32>(km, vm, p, grid, pdl, stream)
               : gqa::launch_d<__nv_bfloat16, 32>(km, vm, p, grid, pdl, stream);
  if (a->d_qk == 16)
    return f16 ? gqa::launch_d<__half, 16>(km, vm, p, grid, pdl, stream)
               : gqa::launch_d<__nv_bfloat16, 16>(km, vm, p, grid, pdl, stream);
  return f16 ? gqa::launch_d<__half, 128>(km, vm, p, grid, pdl, stream)
             : gqa::launch_d<__nv_bfloat16, 128>(km, vm, p, grid, pdl, stream);
}

}  // namespace fa
