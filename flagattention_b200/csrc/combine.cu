// combine.cu -- log-sum-exp merge of split partial results.
//
// Same algebra as the reference's _fwd_combine_kv_splits (split_kv.py:198-228):
//   lse = m + log(sum_s exp(lse_s - m)),  o = sum_s exp(lse_s - lse) * o_s
// with f32 partials.  One warp per output row (d_v <= 512); lanes stride over
// the value dims with 16-byte loads.
#include "common.cuh"
#include "flagattn_b200.h"

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

// Merge `n` partial rows located at part_o[slot(s) * slot_stride + row_off]
// (and part_lse[slot(s) * lse_stride + row]).  Returns the merged lse.
// Partials go in groups of two: a group's LSEs and value rows are all loaded
// before any is used, and the groups are folded with a running maximum, so a
// warp waits for one memory round trip per group instead of one for the LSEs
// and then one per partial.  Two, not more: the merge is latency-bound on
// partials that come from DRAM, and a 64-register budget (eight 4-warp blocks
// per SM) hides more latency than more loads in flight per warp.
template <typename T>
__device__ __forceinline__ float merge_row(const float *__restrict__ part_o,
                                           const float *__restrict__ part_lse, int first_slot,
                                           int n, int64_t o_slot_stride, int64_t lse_slot_stride,
                                           int64_t o_row_off, int64_t lse_row, int d_v, T *out,
                                           int lane) {
  constexpr int kGroup = 2;
  float m = -INFINITY, z = 0.f;  // running maximum and sum of exp(lse_s - m)
  // Each lane owns up to 4 float4 columns (d = 4 lane + 128 k).
  float4 acc[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s0 = 0; s0 < n; s0 += kGroup) {
    float ls[kGroup];
    float4 v[kGroup][4];
#pragma unroll
    for (int g = 0; g < kGroup; ++g) {
      const bool live = s0 + g < n;
      ls[g] = live ? __ldg(part_lse + (first_slot + s0 + g) * lse_slot_stride + lse_row) : -INFINITY;
      const float *src = part_o + (first_slot + s0 + g) * o_slot_stride + o_row_off;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int d = lane * 4 + k * 128;
        v[g][k] = (live && d < d_v) ? __ldg(reinterpret_cast<const float4 *>(src + d))
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    float mg = m;
#pragma unroll
    for (int g = 0; g < kGroup; ++g) mg = fmaxf(mg, ls[g]);
    if (mg == -INFINITY) continue;  // nothing but empty partials so far
    const float keep = (m == -INFINITY) ? 0.f : __expf(m - mg);
    z *= keep;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      acc[k].x *= keep;
      acc[k].y *= keep;
      acc[k].z *= keep;
      acc[k].w *= keep;
    }
#pragma unroll
    for (int g = 0; g < kGroup; ++g) {
      const float w = (ls[g] == -INFINITY) ? 0.f : __expf(ls[g] - mg);
      z += w;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        acc[k].x += w * v[g][k].x;
        acc[k].y += w * v[g][k].y;
        acc[k].z += w * v[g][k].z;
        acc[k].w += w * v[g][k].w;
      }
    }
    m = mg;
  }
  const float lse = (z > 0.f) ? m + __logf(z) : -INFINITY;
  const float inv = (z > 0.f) ? 1.f / z : 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int d = lane * 4 + k * 128;
    const float4 o = make_float4(acc[k].x * inv, acc[k].y * inv, acc[k].z * inv, acc[k].w * inv);
    if (d < d_v) store4<T>(out + d, o);
  }
  return lse;
}

// Generic: rows decomposed as (b, h, m) with h < H, m < M; every row has
// num_parts partials laid out [part][rows][d_v]; lse out f32 [rows].
template <typename T>
__global__ void __launch_bounds__(128, 8) lse_combine_kernel(const float *__restrict__ part_o,
                                   const float *__restrict__ part_lse, int num_parts,
                                   int64_t o_part_stride, int64_t lse_part_stride, int64_t rows,
                                   int H, int M, int d_v, T *__restrict__ out, int64_t o_sb,
                                   int64_t o_sh, int64_t o_sm, float *__restrict__ lse) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  if (row >= rows) return;
  const int64_t b = row / (static_cast<int64_t>(H) * M);
  const int h = static_cast<int>((row / M) % H);
  const int m = static_cast<int>(row % M);
  T *o = out + b * o_sb + h * o_sh + m * o_sm;
  const float l = merge_row<T>(part_o, part_lse, 0, num_parts, o_part_stride, lse_part_stride,
                               row * d_v, row, d_v, o, lane);
  if (lse != nullptr && lane == 0) lse[row] = l;
}

// MLA: sequence b owns slots num_splits[b] .. num_splits[b+1]-1 of
// part_o [slot][s_q*h_q][d_v]; single-piece sequences were written directly.
template <typename T>
__global__ void __launch_bounds__(128, 8) mla_combine_kernel(const float *__restrict__ part_o,
                                   const float *__restrict__ part_lse,
                                   const int32_t *__restrict__ num_splits, int s_q, int h_q,
                                   int d_v, T *__restrict__ out, int64_t o_sb, int64_t o_ss,
                                   int64_t o_sh, float *__restrict__ lse) {
  const int lane = threadIdx.x & 31;
  const int b = blockIdx.y;
  const int rows = s_q * h_q;
  const int flat = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (flat >= rows) return;
  const int first = num_splits[b];
  const int n = num_splits[b + 1] - first;
  if (n <= 1) return;
  const int s = flat / h_q, h = flat % h_q;
  T *o = out + b * o_sb + s * o_ss + h * o_sh;
  const float l = merge_row<T>(part_o, part_lse, first, n, static_cast<int64_t>(rows) * d_v, rows,
                               static_cast<int64_t>(flat) * d_v, flat, d_v, o, lane);
  if (lane == 0) lse[(static_cast<int64_t>(b) * h_q + h) * s_q + s] = l;
}

template <typename T>
void launch_lse_combine_t(const float *part_o, const float *part_lse, int num_parts,
                          int64_t o_part_stride, int64_t lse_part_stride, int64_t rows, int H,
                          int M, int d_v, void *out, int64_t o_sb, int64_t o_sh, int64_t o_sm,
                          float *lse, cudaStream_t stream) {
  const int warps = 4;
  const int64_t grid = (rows + warps - 1) / warps;
  if (grid == 0) return;
  lse_combine_kernel<T><<<static_cast<unsigned>(grid), warps * 32, 0, stream>>>(
      part_o, part_lse, num_parts, o_part_stride, lse_part_stride, rows, H, M, d_v,
      static_cast<T *>(out), o_sb, o_sh, o_sm, lse);
}

// Partial p of row r: O at part_o + p * o_part_stride + r * d_v, LSE at
// part_lse + p * lse_part_stride + r.
void launch_lse_combine(const float *part_o, const float *part_lse, int num_parts,
                        int64_t o_part_stride, int64_t lse_part_stride, int64_t rows, int H, int M,
                        int d_v, void *out, int dtype, int64_t o_sb, int64_t o_sh, int64_t o_sm,
                        float *lse, cudaStream_t stream) {
  if (dtype == FA_DTYPE_BF16)
    launch_lse_combine_t<__nv_bfloat16>(part_o, part_lse, num_parts, o_part_stride,
                                        lse_part_stride, rows, H, M, d_v, out, o_sb, o_sh, o_sm,
                                        lse, stream);
  else if (dtype == FA_DTYPE_F16)
    launch_lse_combine_t<__half>(part_o, part_lse, num_parts, o_part_stride, lse_part_stride,
                                 rows, H, M, d_v, out, o_sb, o_sh, o_sm, lse, stream);
  else
    launch_lse_combine_t<float>(part_o, part_lse, num_parts, o_part_stride, lse_part_stride, rows,
                                H, M, d_v, out, o_sb, o_sh, o_sm, lse, stream);
}

void launch_mla_combine(const float *part_o, const float *part_lse, const int32_t *num_splits,
                        int batch, int s_q, int h_q, int d_v, void *out, int dtype, int64_t o_sb,
                        int64_t o_ss, int64_t o_sh, float *lse, cudaStream_t stream) {
  const int warps = 4;
  dim3 grid((s_q * h_q + warps - 1) / warps, batch);
  if (dtype == FA_DTYPE_BF16)
    mla_combine_kernel<__nv_bfloat16><<<grid, warps * 32, 0, stream>>>(
        part_o, part_lse, num_splits, s_q, h_q, d_v, static_cast<__nv_bfloat16 *>(out), o_sb,
        o_ss, o_sh, lse);
  else if (dtype == FA_DTYPE_F32)
    mla_combine_kernel<float><<<grid, warps * 32, 0, stream>>>(
        part_o, part_lse, num_splits, s_q, h_q, d_v, static_cast<float *>(out), o_sb, o_ss, o_sh,
        lse);
  else
    mla_combine_kernel<__half><<<grid, warps * 32, 0, stream>>>(
        part_o, part_lse, num_splits, s_q, h_q, d_v, static_cast<__half *>(out), o_sb, o_ss, o_sh,
        lse);
}

}  // namespace fa
