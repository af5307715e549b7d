// mla_tc.cu -- tensor-core (tcgen05 / TMEM / TMA) MLA decode for sm_100a.
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
//
// Warp roles (256 threads): warp 0 = TMA producer, warp 1 = TMEM owner and
// MMA issuer, warps 2-3 = key-row gatherers (sparse only), warps 4-7 =
// softmax / correction / epilogue (thread i owns query row i).
// Every mbarrier wait is bounded (common.cuh); a timeout sets the device
// status word and the kernel unwinds instead of hanging.
#include "common.cuh"
#include "flagattn_b200.h"

namespace fa {

constexpr int kRows = 128;
constexpr int kChunkBytesRow = 128;               // 64 dims x 2 bytes per swizzle row
constexpr int kMaxChunks = 5;                     // rank 1 holds dims 256..575
constexpr int kQChunkBytes = kRows * kChunkBytesRow;
constexpr int kQBytes = kMaxChunks * kQChunkBytes;  // 80 KB
constexpr int kDvHalf = 256;                      // output dims per CTA
constexpr int kPvChunks = kDvHalf / 64;           // 4
constexpr float kRescaleThreshold = 8.0f;         // log2 units (factor 256)

template <int BN>
struct TileCfg {
  static constexpr int kStages = BN == 64 ? 2 : 5;
  static constexpr int kKvChunkBytes = BN * kChunkBytesRow;
  static constexpr int kStageBytes = kMaxChunks * kKvChunkBytes;
  static constexpr int kXBytes = kRows * BN * 4;  // f32 partial scores
  static constexpr int kOffKv = kQBytes;
  static constexpr int kOffX = kOffKv + kStages * kStageBytes;
  static constexpr int kOffBar = kOffX + 2 * kXBytes;
  static constexpr int kSmemBytes = kOffBar + 512 + 1024;  // barriers + alignment slack
  // TMEM columns: O [0,256), S0, S1 (BN each), P0, P1 (BN/2 each)
  static constexpr uint32_t kColO = 0;
  static constexpr uint32_t kColS = 256;
  static constexpr uint32_t kColP = 256 + 2 * BN;
  static constexpr uint32_t kTmemCols = 512;
};

struct MlaBarriers {
  uint64_t q_full, q_empty;
  uint64_t kv_full[8], kv_empty[8];
  uint64_t s_full[2], s_empty[2];
  uint64_t p_full[2], pv_done[2];
  uint64_t x_full[2];
  uint64_t o_empty, drain;
  uint32_t tmem_base;
  int abort_flag;
};

struct MlaParams {
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
  const int nblk = len > 0 ? (len + FA_MLA_BLOCK_N - 1) / FA_MLA_BLOCK_N : 0;
  const int lo = (i == 0) ? meta[1] : 0;
  const int hi = (pc.b == meta[2]) ? meta[3] : nblk;
  pc.tok0 = lo * FA_MLA_BLOCK_N;
  pc.tok_end = min(hi * FA_MLA_BLOCK_N, max(len, 0));
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
                                          bool sparse, int bn) {
    tok += bn;
    ++g;
    if (tok >= tok_end) {
      ++piece;
      ++qi;
      seek(p, meta, n_pieces, sparse);
    }
  }
};

template <typename T, int BN, bool kSparse>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(256, 1)
    mla_decode_tc_kernel(const __grid_constant__ CUtensorMap q_map,
                         const __grid_constant__ CUtensorMap kv_map, const MlaParams p) {
  using Cfg = TileCfg<BN>;
  constexpr int kStages = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  MlaBarriers *bars = reinterpret_cast<MlaBarriers *>(smem + Cfg::kOffBar);
  const uint32_t s_base = smem_u32(smem);
  const uint32_t q_base = s_base;
  const uint32_t kv_base = s_base + Cfg::kOffKv;
  const uint32_t x_base = s_base + Cfg::kOffX;
  volatile int *abort_flag = &bars->abort_flag;

  const uint32_t rank = cluster_rank();
  const uint32_t peer = rank ^ 1u;
  const int part = blockIdx.x >> 1;
  const int mb = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_chunks = 4 + static_cast<int>(rank);
  const int dim0 = static_cast<int>(rank) * 256;
  const int32_t *meta = p.tile_meta + static_cast<int64_t>(part) * FA_MLA_META_INTS;
  const int n_pieces = meta[5];
  // query rows of this m-block: dense = 128 consecutive (s, h) rows; sparse =
  // the h_q heads of query token mb (index lists differ per query token).
  const int rows_total = p.s_q * p.h_q;
  const int row0 = kSparse ? mb * p.h_q : mb * kRows;
  const int n_rows = kSparse ? p.h_q : min(kRows, rows_total - row0);
  const int fmt = sizeof(T) == 2 && !std::is_same<T, __half>::value ? 1 : 0;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bars->q_full), 1);
    mbar_init(smem_u32(&bars->q_empty), 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&bars->kv_full[s]), kSparse ? 64 : 1);
      mbar_init(smem_u32(&bars->kv_empty[s]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&bars->s_full[i]), 1);
      mbar_init(smem_u32(&bars->s_empty[i]), 128);
      mbar_init(smem_u32(&bars->p_full[i]), 128);
      mbar_init(smem_u32(&bars->pv_done[i]), 1);
      mbar_init(smem_u32(&bars->x_full[i]), 1);
    }
    mbar_init(smem_u32(&bars->o_empty), 128);
    mbar_init(smem_u32(&bars->drain), 1);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&bars->tmem_base), Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  cluster_sync();  // the peer's barriers exist before any remote access

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&q_map);
      if (!kSparse) tma_prefetch_desc(&kv_map);
      uint32_t g = 0;
      int qi = 0;
      bool ok = true;
      for (int i = 0; i < n_pieces && ok; ++i) {
        const Piece pc = get_piece(p, meta, i, kSparse);
        if (pc.tok_end <= pc.tok0) continue;
        ok = mbar_wait(smem_u32(&bars->q_empty), (qi & 1) ^ 1, abort_flag, p.status,
                       kDevTimeoutProducer);
        if (!ok) break;
        mbar_arrive_expect_tx(smem_u32(&bars->q_full), n_chunks * kQChunkBytes);
        for (int c = 0; c < n_chunks; ++c)
          tma_load_3d(q_base + c * kQChunkBytes, &q_map, smem_u32(&bars->q_full), dim0 + 64 * c,
                      row0, pc.b);
        ++qi;
        if (kSparse) {
          g += (pc.tok_end - pc.tok0 + BN - 1) / BN;
          continue;
        }
        for (int tok = pc.tok0; tok < pc.tok_end; tok += BN, ++g) {
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
          mbar_arrive_expect_tx(full, n_chunks * Cfg::kKvChunkBytes);
          const uint32_t dst = kv_base + st * Cfg::kStageBytes;
          for (int c = 0; c < n_chunks; ++c)
            tma_load_3d(dst + c * Cfg::kKvChunkBytes, &kv_map, full, dim0 + 64 * c, c1, c2);
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
      const uint32_t idesc_qk = umma_idesc_f16(128, BN, fmt, 0);
      const uint32_t idesc_pv = umma_idesc_f16(128, kDvHalf, fmt, 1);
      TileCursor cq, cp;
      cq.start(p, meta, n_pieces, kSparse);
      cp.start(p, meta, n_pieces, kSparse);
      long long t_last = 0;
      uint32_t idle = 0;
      while (cp.valid) {
        bool did = false;
        if (cp.g < cq.g) {
          const uint32_t t = cp.g;
          const int st = t % kStages;
          const uint32_t pb = t & 1u;
          const bool first = cp.tok == cp.tok0;
          if (mbar_probe(smem_u32(&bars->p_full[pb]), (t >> 1) & 1) &&
              (!first || mbar_probe(smem_u32(&bars->o_empty), (cp.qi & 1) ^ 1))) {
            tc_fence_after();
            const uint32_t vb = kv_base + st * Cfg::kStageBytes;
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk) {
              const uint64_t bdesc = smem_desc_sw128(vb + kk * 16 * kChunkBytesRow,
                                                     Cfg::kKvChunkBytes, 1024);
              umma_ts(tmem + Cfg::kColO, tmem + Cfg::kColP + pb * (BN / 2) + kk * 8, bdesc,
                      idesc_pv, (first && kk == 0) ? 0u : 1u);
            }
            tc_commit(smem_u32(&bars->kv_empty[st]));
            tc_commit(smem_u32(&bars->pv_done[pb]));
            cp.advance(p, meta, n_pieces, kSparse, BN);
            did = true;
          }
        }
        if (cq.valid) {
          const uint32_t g = cq.g;
          const int st = g % kStages;
          const uint32_t sb = g & 1u;
          const bool first = cq.tok == cq.tok0;
          if ((!first || mbar_probe(smem_u32(&bars->q_full), cq.qi & 1)) &&
              mbar_probe(smem_u32(&bars->kv_full[st]), (g / kStages) & 1) &&
              mbar_probe(smem_u32(&bars->s_empty[sb]), ((g >> 1) & 1) ^ 1)) {
            if (kSparse) fence_proxy_async_smem();  // cp.async rows -> tensor-core reads
            tc_fence_after();
            const uint32_t kb = kv_base + st * Cfg::kStageBytes;
            for (int c = 0; c < n_chunks; ++c) {
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                const uint64_t adesc =
                    smem_desc_sw128(q_base + c * kQChunkBytes + kk * 32, 16, 1024);
                const uint64_t bdesc =
                    smem_desc_sw128(kb + c * Cfg::kKvChunkBytes + kk * 32, 16, 1024);
                umma_ss(tmem + Cfg::kColS + sb * BN, adesc, bdesc, idesc_qk, (c | kk) ? 1u : 0u);
              }
            }
            tc_commit(smem_u32(&bars->s_full[sb]));
            if (cq.tok + BN >= cq.tok_end) tc_commit(smem_u32(&bars->q_empty));
            cq.advance(p, meta, n_pieces, kSparse, BN);
            did = true;
          }
        }
        if (did) {
          idle = 0;
          t_last = 0;
        } else if ((++idle & 63u) == 0) {
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
        for (int tok = pc.tok0; tok < pc.tok_end; tok += BN, ++g) {
          const int st = g % kStages;
          ok = mbar_wait(smem_u32(&bars->kv_empty[st]), ((g / kStages) & 1) ^ 1, abort_flag,
                         p.status, kDevTimeoutProducer);
          if (!ok) break;
          const uint32_t dst = kv_base + st * Cfg::kStageBytes;
          const int units = n_chunks * 8;  // 16-byte units per row
          for (int k = gt; k < BN * units; k += 64) {
            const int r = k / units;
            const int rem = k - r * units;
            const int c = rem >> 3, w = rem & 7;
            const int pos = tok + r;
            int64_t row = -1;
            if (pos < pc.tok_end) row = idx[pos];
            const bool valid = row >= 0 && row < p.total_rows;
            const uint8_t *src = p.kcache;
            if (valid) {
              const int64_t pg = row / p.page_size, off = row % p.page_size;
              src += (pg * p.kv_sp + off * p.kv_st + dim0 + c * 64 + w * 8) * 2;
            }
            cp_async_16(dst + c * Cfg::kKvChunkBytes + r * kChunkBytesRow + ((w ^ (r & 7)) << 4),
                        src, valid ? 16u : 0u);
          }
          cp_async_arrive(smem_u32(&bars->kv_full[st]));
        }
      }
      asm volatile("cp.async.wait_all;" ::: "memory");
    }
  } else {
    // ------------------------------------------ softmax / correction / out
    const int t = threadIdx.x - 128;  // query row within the m-block
    const uint32_t lane_off = static_cast<uint32_t>((t >> 5) * 32) << 16;
    const uint32_t trow = tmem + lane_off;
    const int flat = row0 + t;
    const bool row_ok = t < n_rows;
    const int s_tok = kSparse ? mb : (row_ok ? flat / p.h_q : 0);
    const int h = kSparse ? t : (row_ok ? flat % p.h_q : 0);
    const int out_flat = s_tok * p.h_q + h;
    const uint32_t x_local[2] = {x_base, x_base + Cfg::kXBytes};
    const uint32_t x_remote[2] = {map_to_rank(x_base, peer), map_to_rank(x_base + Cfg::kXBytes, peer)};
    const uint32_t xf_local[2] = {smem_u32(&bars->x_full[0]), smem_u32(&bars->x_full[1])};
    const uint32_t xf_remote[2] = {map_to_rank(xf_local[0], peer), map_to_rank(xf_local[1], peer)};
    uint32_t g = 0;
    int qi = 0;
    bool ok = true;
    for (int i = 0; i < n_pieces && ok; ++i) {
      const Piece pc = get_piece(p, meta, i, kSparse);
      const int first_slot = p.num_splits[pc.b];
      const int n_split = p.num_splits[pc.b + 1] - first_slot;
      const int slot = first_slot + pc.split_idx;
      const int len = kSparse ? p.topk : (p.seq_lens ? p.seq_lens[pc.b] : p.n_ctx);
      const int row_len = (p.causal && !kSparse) ? len - (p.s_q - 1 - s_tok) : len;
      float m_run = -INFINITY, l_run = 0.f;
      const int32_t *idx = kSparse ? p.indices + pc.b * p.idx_sb + s_tok * p.idx_ss : nullptr;
      const bool has_tiles = pc.tok_end > pc.tok0;
      for (int tok = pc.tok0; tok < pc.tok_end && ok; tok += BN, ++g) {
        const uint32_t sb = g & 1u;
        const uint32_t n = g >> 1;
        const bool first = tok == pc.tok0;
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars->s_full[sb]), n & 1, abort_flag,
                                               p.status, kDevTimeoutSoftmax));
        if (!ok) break;
        tc_fence_after();
        float s[BN];
#pragma unroll
        for (int c = 0; c < BN / 16; ++c) {
          float v[16];
          tmem_ld16(trow + Cfg::kColS + sb * BN + c * 16, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) s[c * 16 + j] = v[j];
        }
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(smem_u32(&bars->s_empty[sb]));
        // exchange partial scores with the peer CTA
        if (t == 0) mbar_arrive_expect_tx(xf_local[sb], Cfg::kXBytes);
#pragma unroll
        for (int c = 0; c < BN / 4; ++c)
          st_async_v4(x_remote[sb] + (c * 128 + t) * 16, s[4 * c], s[4 * c + 1], s[4 * c + 2],
                      s[4 * c + 3], xf_remote[sb]);
        ok = __all_sync(0xffffffffu, mbar_wait<true>(xf_local[sb], n & 1, abort_flag, p.status,
                                                     kDevTimeoutExchange));
        if (!ok) break;
        const float4 *xr = reinterpret_cast<const float4 *>(smem + Cfg::kOffX + sb * Cfg::kXBytes);
#pragma unroll
        for (int c = 0; c < BN / 4; ++c) {
          const float4 o = xr[c * 128 + t];
          s[4 * c] += o.x;
          s[4 * c + 1] += o.y;
          s[4 * c + 2] += o.z;
          s[4 * c + 3] += o.w;
        }
        // mask and scale to log2 units
        float mt = -INFINITY;
        if (kSparse) {
#pragma unroll
          for (int c = 0; c < BN; ++c) {
            const int pos = tok + c;
            const int64_t row = pos < pc.tok_end ? idx[pos] : -1;
            const bool valid = row >= 0 && row < p.total_rows;
            s[c] = valid ? s[c] * p.scale_log2 : -INFINITY;
            mt = fmaxf(mt, s[c]);
          }
        } else {
#pragma unroll
          for (int c = 0; c < BN; ++c) {
            const bool valid = tok + c < row_len && tok + c < pc.tok_end;
            s[c] = valid ? s[c] * p.scale_log2 : -INFINITY;
            mt = fmaxf(mt, s[c]);
          }
        }
        // online softmax with a lazily updated running max
        float alpha = 1.f;
        bool rescale = false;
        if (mt > -INFINITY && (m_run == -INFINITY || mt > m_run + kRescaleThreshold)) {
          alpha = (m_run == -INFINITY) ? 0.f : fast_exp2(m_run - mt);
          rescale = !first && m_run != -INFINITY;
          m_run = mt;
        }
        const float ms = (m_run == -INFINITY) ? 0.f : m_run;
        float psum = 0.f;
        uint32_t pk[BN / 2];
#pragma unroll
        for (int c = 0; c < BN; c += 2) {
          const float p0 = fast_exp2(s[c] - ms);
          const float p1 = fast_exp2(s[c + 1] - ms);
          psum += p0 + p1;
          pk[c / 2] = Elem<T>::pack2(p0, p1);
        }
        l_run = l_run * alpha + psum;
        // P buffer sb is free once PV of tile g-2 has finished
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars->pv_done[sb]), (n & 1) ^ 1,
                                               abort_flag, p.status, kDevTimeoutSoftmax));
        if (!ok) break;
        if (__any_sync(0xffffffffu, rescale)) {
          const uint32_t pt = g - 1;
          ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&bars->pv_done[pt & 1u]), (pt >> 1) & 1,
                                                 abort_flag, p.status, kDevTimeoutSoftmax));
          if (!ok) break;
          tc_fence_after();
          const float a = rescale ? alpha : 1.f;
#pragma unroll 1
          for (int c = 0; c < kDvHalf / 16; ++c) {
            float v[16];
            tmem_ld16(trow + Cfg::kColO + c * 16, v);
            tmem_wait_ld();
            uint32_t w[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) w[j] = __float_as_uint(v[j] * a);
            tmem_st16(trow + Cfg::kColO + c * 16, w);
          }
        }
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t w[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) w[j] = pk[c * 16 + j];
          tmem_st16(trow + Cfg::kColP + sb * (BN / 2) + c * 16, w);
        }
        tmem_wait_st();
        if (!kSparse && pc.tok_end - tok < BN) {
          // rows past the sequence end may hold any bits (even NaN); P is 0
          // there but 0 * NaN is not, so clear them before the PV product.
          const int kv_valid = pc.tok_end - tok;
          const int units = (BN - kv_valid) * kPvChunks * 8;
          uint8_t *stage = smem + Cfg::kOffKv + (g % kStages) * Cfg::kStageBytes;
          for (int u = t; u < units; u += 128) {
            const int r = kv_valid + u / (kPvChunks * 8);
            const int rem = u % (kPvChunks * 8);
            *reinterpret_cast<uint4 *>(stage + (rem >> 3) * Cfg::kKvChunkBytes +
                                       r * kChunkBytesRow + (rem & 7) * 16) =
                make_uint4(0u, 0u, 0u, 0u);
          }
          fence_proxy_async_smem();
        }
        tc_fence_before();
        mbar_arrive(smem_u32(&bars->p_full[sb]));
      }
      if (!ok) break;
      // -------------------------------------------------------- epilogue
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
      for (int c = 0; c < kDvHalf / 16; ++c) {
        float v[16];
        if (has_tiles) {
          tmem_ld16(trow + Cfg::kColO + c * 16, v);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = 0.f;
        }
        if (!row_ok) continue;
        const int d = static_cast<int>(rank) * kDvHalf + c * 16;
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
      if (rank == 0 && row_ok) {
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
  cluster_sync();  // the peer no longer touches this CTA's shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

template <typename T, int BN, bool kSparse>
static cudaError_t launch_mla_t(const CUtensorMap &qm, const CUtensorMap &km, const MlaParams &p,
                                int num_parts, int m_blocks, cudaStream_t stream) {
  auto kern = mla_decode_tc_kernel<T, BN, kSparse>;
  const int smem = TileCfg<BN>::kSmemBytes;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dim3 grid(2 * num_parts, m_blocks);
  kern<<<grid, 256, smem, stream>>>(qm, km, p);
  return cudaGetLastError();
}

size_t mla_tc_smem_bytes(int block_n) {
  return block_n == 64 ? TileCfg<64>::kSmemBytes : TileCfg<32>::kSmemBytes;
}

cudaError_t launch_mla_tc(const CUtensorMap &qm, const CUtensorMap &km, const fa_mla_args *a,
                          int block_n, int m_blocks, int64_t total_rows, cudaStream_t stream) {
  MlaParams p;
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
  const bool sparse = a->indices != nullptr;
  const bool f16 = a->dtype == FA_DTYPE_F16;
#define FA_LAUNCH(T_, BN_, SP_) return launch_mla_t<T_, BN_, SP_>(qm, km, p, a->num_sm_parts, m_blocks, stream)
  if (block_n == 64) {
    if (f16) { if (sparse) FA_LAUNCH(__half, 64, true); FA_LAUNCH(__half, 64, false); }
    if (sparse) FA_LAUNCH(__nv_bfloat16, 64, true);
    FA_LAUNCH(__nv_bfloat16, 64, false);
  }
  if (f16) { if (sparse) FA_LAUNCH(__half, 32, true); FA_LAUNCH(__half, 32, false); }
  if (sparse) FA_LAUNCH(__nv_bfloat16, 32, true);
  FA_LAUNCH(__nv_bfloat16, 32, false);
#undef FA_LAUNCH
}

}  // namespace fa
