// merge.cuh -- log-sum-exp merge of one row's split partials, shared by the
// combine kernels (combine.cu) and the cross-GPU merges (exchange.cu).  Same
// algebra as the reference's _fwd_combine_kv_splits (split_kv.py:198-228):
//   lse = m + log(sum_s exp(lse_s - m)),  o = sum_s exp(lse_s - lse) * o_s
// with f32 LSEs, f32 accumulation and partial rows o_s stored as f32 or in the
// output's 16-bit type (the decode kernels keep split rows in the output
// type, as the reference keeps its partial O in out.dtype, paged.py:103-113,
// or fp16, split_kv.py:311).  One warp per row (d_v <= 512).  Lane l owns
// the columns 4 l + 128 k .. + 3 (k < 4) of f32 partials, and 8 l + 256 k ..
// + 7 (k < 2) of 16-bit partials, so that every load is 16 bytes.
#pragma once

#include "common.cuh"

namespace fa {

template <typename T>
__device__ __forceinline__ void store4(T *dst, float4 v) {
  if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float4 *>(dst) = v;
  } else {
    uint2 w;
    w.x = Elem<T>::pack2(v.x, v.y);
    w.y = Elem<T>::pack2(v.z, v.w);
    *reinterpret_cast<uint2 *>(dst) = w;
  }
}

// Loads of partials: through the read-only path when a separate kernel reads
// what an earlier one wrote (kCoherent false), at L2 (ld.global.cg) when
// other CTAs of the same kernel wrote them.
template <bool kCoherent>
__device__ __forceinline__ float load_part(const float *p) {
  return kCoherent ? __ldcg(p) : __ldg(p);
}
template <bool kCoherent>
__device__ __forceinline__ float4 load_part4(const float *p) {
  return kCoherent ? __ldcg(reinterpret_cast<const float4 *>(p))
                   : __ldg(reinterpret_cast<const float4 *>(p));
}
// Eight 16-bit partial values (16 bytes) widened to f32.
template <bool kCoherent, typename TP>
__device__ __forceinline__ void load_part8(const TP *p, float4 &lo, float4 &hi) {
  static_assert(sizeof(TP) == 2, "16-bit partials");
  const uint4 u = kCoherent ? __ldcg(reinterpret_cast<const uint4 *>(p))
                            : __ldg(reinterpret_cast<const uint4 *>(p));
  const TP *h = reinterpret_cast<const TP *>(&u);
  lo = make_float4(Elem<TP>::to_f(h[0]), Elem<TP>::to_f(h[1]), Elem<TP>::to_f(h[2]),
                   Elem<TP>::to_f(h[3]));
  hi = make_float4(Elem<TP>::to_f(h[4]), Elem<TP>::to_f(h[5]), Elem<TP>::to_f(h[6]),
                   Elem<TP>::to_f(h[7]));
}

// Column of the calling lane's accumulator k (0..3), for partials of type TP.
template <typename TP>
__device__ __forceinline__ int acc_col(int lane, int k) {
  return sizeof(TP) == 4 ? lane * 4 + k * 128 : lane * 8 + (k >> 1) * 256 + (k & 1) * 4;
}

// Running state of a row's merge: maximum m of the LSEs folded so far, sum z
// of exp(lse_s - m), and sum of exp(lse_s - m) * o_s (lane l's four float4
// columns).
struct MergeState {
  float m, z;
  float4 acc[4];
  __device__ __forceinline__ void init() {
    m = -INFINITY;
    z = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
};

// Fold partials s = s0, s0 + step, ... < n of one row into st, partial s at
// part_o[(first_slot + s) * o_slot_stride + o_row_off] and part_lse[(first_slot
// + s) * lse_slot_stride + lse_row].  Partials go in groups of kGroup: a
// group's LSEs and value rows are all loaded before any is used, and the
// groups are folded with a running maximum, so a warp waits for one memory
// round trip per group instead of one for the LSEs and then one per partial.
template <bool kCoherent, int kGroup = 2, typename TP = float>
__device__ __forceinline__ void fold_parts(MergeState &st, const TP *__restrict__ part_o,
                                           const float *__restrict__ part_lse, int first_slot,
                                           int s0, int step, int n, int64_t o_slot_stride,
                                           int64_t lse_slot_stride, int64_t o_row_off,
                                           int64_t lse_row, int d_v, int lane) {
  for (int s = s0; s < n; s += kGroup * step) {
    float ls[kGroup];
    float4 v[kGroup][4];
#pragma unroll
    for (int g = 0; g < kGroup; ++g) {
      const bool live = s + g * step < n;
      const int64_t slot = first_slot + s + g * step;
      ls[g] = live ? load_part<kCoherent>(part_lse + slot * lse_slot_stride + lse_row) : -INFINITY;
      const TP *src = part_o + slot * o_slot_stride + o_row_off;
      if constexpr (sizeof(TP) == 4) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int d = lane * 4 + k * 128;
          v[g][k] = (live && d < d_v) ? load_part4<kCoherent>(src + d)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      } else {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int d = lane * 8 + k * 256;
          v[g][2 * k] = v[g][2 * k + 1] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (live && d < d_v) load_part8<kCoherent>(src + d, v[g][2 * k], v[g][2 * k + 1]);
        }
      }
    }
    float mg = st.m;
#pragma unroll
    for (int g = 0; g < kGroup; ++g) mg = fmaxf(mg, ls[g]);
    if (mg == -INFINITY) continue;  // nothing but empty partials so far
    const float keep = (st.m == -INFINITY) ? 0.f : __expf(st.m - mg);
    st.z *= keep;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      st.acc[k].x *= keep;
      st.acc[k].y *= keep;
      st.acc[k].z *= keep;
      st.acc[k].w *= keep;
    }
#pragma unroll
    for (int g = 0; g < kGroup; ++g) {
      const float w = (ls[g] == -INFINITY) ? 0.f : __expf(ls[g] - mg);
      st.z += w;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        st.acc[k].x += w * v[g][k].x;
        st.acc[k].y += w * v[g][k].y;
        st.acc[k].z += w * v[g][k].z;
        st.acc[k].w += w * v[g][k].w;
      }
    }
    st.m = mg;
  }
}

// a <- a folded with b (two states of the same row).
__device__ __forceinline__ void fold_state(MergeState &a, const MergeState &b) {
  const float m = fmaxf(a.m, b.m);
  if (m == -INFINITY) return;
  const float ka = (a.m == -INFINITY) ? 0.f : __expf(a.m - m);
  const float kb = (b.m == -INFINITY) ? 0.f : __expf(b.m - m);
  a.z = a.z * ka + b.z * kb;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    a.acc[k].x = a.acc[k].x * ka + b.acc[k].x * kb;
    a.acc[k].y = a.acc[k].y * ka + b.acc[k].y * kb;
    a.acc[k].z = a.acc[k].z * ka + b.acc[k].z * kb;
    a.acc[k].w = a.acc[k].w * ka + b.acc[k].w * kb;
  }
  a.m = m;
}

// Merge state of query row `flat` of an MLA sequence whose n pieces sit in
// split slots first .. first + n - 1 (part_o [slot][rows][d_v]).
//   narrow (kWide false): the calling warp folds all n partials;
//   wide (kWide true): the four warps w0 .. w0 + 3 of the block (warp j =
//     w0 + j calls with j) fold partials j, j + 4, ... and the states meet in
//     `states` (shared, [warps][32]) folded in warp order; the result is valid
//     in warp w0.  Wide spreads one row's partials over four warps: for a few
//     sequences split over many parts (one long sequence over 37 parts) the
//     GPU has few rows but many partials per row.
template <bool kWide, typename TP = float>
__device__ __forceinline__ void mla_row_state(MergeState &st, const TP *__restrict__ part_o,
                                              const float *__restrict__ part_lse, int first, int n,
                                              int rows, int flat, int d_v, int lane, int j,
                                              int warp, MergeState (*states)[32]) {
  st.init();
  if (!kWide) {
    if (flat < rows)
      fold_parts<false, 2, TP>(st, part_o, part_lse, first, 0, 1, n,
                           static_cast<int64_t>(rows) * d_v, rows,
                           static_cast<int64_t>(flat) * d_v, flat, d_v, lane);
    return;
  }
  if (flat < rows && j < n)
    fold_parts<false, 4, TP>(st, part_o, part_lse, first, j, 4, n, static_cast<int64_t>(rows) * d_v,
                         rows, static_cast<int64_t>(flat) * d_v, flat, d_v, lane);
  states[warp][lane] = st;
  __syncthreads();
  if (j == 0) {
#pragma unroll
    for (int k = 1; k < 4; ++k) fold_state(st, states[warp + k][lane]);
  }
}

// Normalised output row and merged LSE of a state whose partials had type TP
// (which fixes the lane's columns, acc_col).
template <typename T, typename TP = float>
__device__ __forceinline__ float finish_row(const MergeState &st, int d_v, T *out, int lane) {
  const float lse = (st.z > 0.f) ? st.m + __logf(st.z) : -INFINITY;
  const float inv = (st.z > 0.f) ? 1.f / st.z : 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int d = acc_col<TP>(lane, k);
    const float4 o = make_float4(st.acc[k].x * inv, st.acc[k].y * inv, st.acc[k].z * inv,
                                 st.acc[k].w * inv);
    if (d < d_v) store4<T>(out + d, o);
  }
  return lse;
}

// Merge all `n` partials of one row (slot order) into out[0 .. d_v); returns
// the merged LSE.  The fold order is fixed, so the result does not depend on
// which CTA merges or when.
template <typename T, bool kCoherent = false>
__device__ __forceinline__ float merge_row(const float *__restrict__ part_o,
                                           const float *__restrict__ part_lse, int first_slot,
                                           int n, int64_t o_slot_stride, int64_t lse_slot_stride,
                                           int64_t o_row_off, int64_t lse_row, int d_v, T *out,
                                           int lane) {
  MergeState st;
  st.init();
  fold_parts<kCoherent>(st, part_o, part_lse, first_slot, 0, 1, n, o_slot_stride,
                        lse_slot_stride, o_row_off, lse_row, d_v, lane);
  return finish_row<T>(st, d_v, out, lane);
}

}  // namespace fa
