// combine.cu -- log-sum-exp merge of split partial results (merge.cuh: the
// reference's _fwd_combine_kv_splits algebra, split_kv.py:198-228), one warp
// per output row.
#include "common.cuh"
#include "flagattn_b200.h"
#include "merge.cuh"

namespace fa {

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
// part_o [slot][s_q*h_q][d_v] (partial rows in the output type T, as the decode
// writes them); a sequence of one piece was written straight to
// the output.  Narrow form: 128-thread blocks, one warp per row (four rows),
// partials loaded two at a time (one round trip per two partials; most rows
// have two, and the smaller register footprint keeps eight blocks per SM).  Wide
// form (few sequences each split over many parts): 256-thread blocks, two rows,
// four warps per row (mla_row_state).  Launched as a programmatic dependent of
// the decode kernel: its launch overlaps the decode, blocks of unsplit
// sequences exit while the decode still runs, and the others wait for the
// decode grid to complete (griddepcontrol.wait) before reading partials.
template <typename T, bool kWide>
__global__ void __launch_bounds__(kWide ? 256 : 128, kWide ? 2 : 8)
    mla_combine_kernel(const T *__restrict__ part_o, const float *__restrict__ part_lse,
                       const int32_t *__restrict__ num_splits, int s_q, int h_q, int d_v,
                       T *__restrict__ out, int64_t o_sb, int64_t o_ss, int64_t o_sh,
                       float *__restrict__ lse) {
  __shared__ MergeState states[kWide ? 8 : 1][32];
  const int b = blockIdx.y;
  const int first = num_splits[b];  // written by the metadata kernel, before the decode
  const int n = num_splits[b + 1] - first;
  if (n < 2) return;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows = s_q * h_q;
  const int flat = kWide ? blockIdx.x * 2 + (warp >> 2) : blockIdx.x * 4 + warp;
  const int j = kWide ? (warp & 3) : 0;
  MergeState st;
  mla_row_state<kWide, T>(st, part_o, part_lse, first, n, rows, flat, d_v, lane, j, warp, states);
  if (j != 0 || flat >= rows) return;
  const int s = flat / h_q, h = flat % h_q;
  const float l = finish_row<T, T>(st, d_v, out + b * o_sb + s * o_ss + h * o_sh, lane);
  if (lane == 0) lse[(static_cast<int64_t>(b) * h_q + h) * s_q + s] = l;
}

// Grouped-query entries (entry e = sequence * kv_heads + kv head, rows r =
// head-in-group * m_q + query token), partials part_o [slot][rows][d_v] in the
// output type T.
// Balanced schedule: merge[e] = {slot of the entry's first piece (-1: not
// split, written straight to the output), first slot of its later pieces,
// number of later pieces}, written by the decode.  Fixed partitions (merge
// == nullptr): slots e * splits .. + splits - 1.  Launched as a programmatic
// dependent of the decode; everything it reads comes from the decode.
template <typename T, bool kWide>
__global__ void __launch_bounds__(kWide ? 256 : 128, kWide ? 2 : 4)
    gqa_combine_kernel(const T *__restrict__ part_o, const float *__restrict__ part_lse,
                       const int4 *__restrict__ merge, int splits, int rows, int m_q, int group,
                       int hkv, int hq, int d_v, T *__restrict__ out, int64_t o_sb, int64_t o_sh,
                       int64_t o_sm, float *__restrict__ lse) {
  __shared__ MergeState states[kWide ? 8 : 1][32];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int row_blocks = kWide ? (rows + 1) / 2 : (rows + 3) / 4;
  const int e = blockIdx.x / row_blocks, rb = blockIdx.x % row_blocks;
  int head = -1, first = e * splits, n = splits;
  if (merge) {
    const int4 m = merge[e];
    if (m.x < 0) return;
    head = m.x;
    first = m.y;
    n = m.z;
  } else if (n < 2) {
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int flat = kWide ? rb * 2 + (warp >> 2) : rb * 4 + warp;
  const int j = kWide ? (warp & 3) : 0;
  const int64_t os = static_cast<int64_t>(rows) * d_v;
  MergeState st;
  st.init();
  if (flat < rows) {
    if (head >= 0 && j == 0)
      fold_parts<false, 1, T>(st, part_o, part_lse, head, 0, 1, 1, os, rows,
                           static_cast<int64_t>(flat) * d_v, flat, d_v, lane);
    fold_parts<false, 2, T>(st, part_o, part_lse, first, j, kWide ? 4 : 1, n, os, rows,
                         static_cast<int64_t>(flat) * d_v, flat, d_v, lane);
  }
  if (kWide) {
    states[warp][lane] = st;
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int k = 1; k < 4; ++k) fold_state(st, states[warp + k][lane]);
    }
  }
  if (j != 0 || flat >= rows) return;
  const int b = e / hkv, h = (e % hkv) * group + flat / m_q, m = flat % m_q;
  const float l = finish_row<T, T>(st, d_v, out + b * o_sb + h * o_sh + m * o_sm, lane);
  if (lse != nullptr && lane == 0) lse[(static_cast<int64_t>(b) * hq + h) * m_q + m] = l;
}

template <typename T>
cudaError_t launch_gqa_combine_t(const float *part_o, const float *part_lse,
                                 const int4 *merge, int splits, int entries, int rows,
                                 int m_q, int group, int hkv, int hq, int d_v, bool wide,
                                 void *out, int64_t o_sb, int64_t o_sh, int64_t o_sm, float *lse,
                                 cudaStream_t stream) {
  if (entries == 0) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  const int64_t blocks = static_cast<int64_t>(wide ? (rows + 1) / 2 : (rows + 3) / 4) * entries;
  if (blocks > INT32_MAX) return cudaErrorInvalidConfiguration;
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(wide ? 256 : 128);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  T *o = static_cast<T *>(out);
  const T *po = reinterpret_cast<const T *>(part_o);
  if (wide)
    return cudaLaunchKernelEx(&cfg, gqa_combine_kernel<T, true>, po, part_lse, merge, splits,
                              rows, m_q, group, hkv, hq, d_v, o, o_sb, o_sh, o_sm, lse);
  return cudaLaunchKernelEx(&cfg, gqa_combine_kernel<T, false>, po, part_lse, merge, splits,
                            rows, m_q, group, hkv, hq, d_v, o, o_sb, o_sh, o_sm, lse);
}

cudaError_t launch_gqa_combine(const float *part_o, const float *part_lse, const int4 *merge,
                               int splits, int entries, int rows, int m_q, int group, int hkv,
                               int hq, int d_v, bool wide, void *out, int dtype, int64_t o_sb,
                               int64_t o_sh, int64_t o_sm, float *lse, cudaStream_t stream) {
  if (dtype == FA_DTYPE_BF16)
    return launch_gqa_combine_t<__nv_bfloat16>(part_o, part_lse, merge, splits, entries, rows,
                                               m_q, group, hkv, hq, d_v, wide, out, o_sb, o_sh,
                                               o_sm, lse, stream);
  return launch_gqa_combine_t<__half>(part_o, part_lse, merge, splits, entries, rows, m_q, group,
                                      hkv, hq, d_v, wide, out, o_sb, o_sh, o_sm, lse, stream);
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

template <typename T>
cudaError_t launch_mla_combine_t(const float *part_o, const float *part_lse,
                                 const int32_t *num_splits, int batch, int s_q, int h_q, int d_v,
                                 bool wide, void *out, int64_t o_sb, int64_t o_ss, int64_t o_sh,
                                 float *lse, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  const int rows = s_q * h_q;
  cfg.gridDim = wide ? dim3((rows + 1) / 2, batch) : dim3((rows + 3) / 4, batch);
  cfg.blockDim = dim3(wide ? 256 : 128);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const T *po = reinterpret_cast<const T *>(part_o);
  if (wide)
    return cudaLaunchKernelEx(&cfg, mla_combine_kernel<T, true>, po, part_lse, num_splits, s_q,
                              h_q, d_v, static_cast<T *>(out), o_sb, o_ss, o_sh, lse);
  return cudaLaunchKernelEx(&cfg, mla_combine_kernel<T, false>, po, part_lse, num_splits, s_q,
                            h_q, d_v, static_cast<T *>(out), o_sb, o_ss, o_sh, lse);
}

cudaError_t launch_mla_combine(const float *part_o, const float *part_lse,
                               const int32_t *num_splits, int batch, int s_q, int h_q, int d_v,
                               bool wide, void *out, int dtype, int64_t o_sb, int64_t o_ss,
                               int64_t o_sh, float *lse, cudaStream_t stream) {
  if (dtype == FA_DTYPE_BF16)
    return launch_mla_combine_t<__nv_bfloat16>(part_o, part_lse, num_splits, batch, s_q, h_q, d_v,
                                               wide, out, o_sb, o_ss, o_sh, lse, stream);
  if (dtype == FA_DTYPE_F32)
    return launch_mla_combine_t<float>(part_o, part_lse, num_splits, batch, s_q, h_q, d_v, wide,
                                       out, o_sb, o_ss, o_sh, lse, stream);
  return launch_mla_combine_t<__half>(part_o, part_lse, num_splits, batch, s_q, h_q, d_v, wide,
                                      out, o_sb, o_ss, o_sh, lse, stream);
}

}  // namespace fa
