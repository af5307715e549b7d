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
// part_o [slot][s_q*h_q][d_v]; a sequence of one piece was written straight to
// the output.  One warp per row, partials loaded four at a time (a long split
// -- one 1M-token sequence spread over 37 parts -- waits for 10 memory round
// trips instead of 19).  Launched as a programmatic dependent of the decode
// kernel: its launch overlaps the decode, blocks of unsplit sequences exit
// while the decode still runs, and the others wait for the decode grid to
// complete (griddepcontrol.wait) before reading partials.
template <typename T>
__global__ void __launch_bounds__(128, 4) mla_combine_kernel(const float *__restrict__ part_o,
                                   const float *__restrict__ part_lse,
                                   const int32_t *__restrict__ num_splits, int s_q, int h_q,
                                   int d_v, T *__restrict__ out, int64_t o_sb, int64_t o_ss,
                                   int64_t o_sh, float *__restrict__ lse) {
  const int b = blockIdx.y;
  const int first = num_splits[b];  // written by the metadata kernel, before the decode
  const int n = num_splits[b + 1] - first;
  if (n < 2) return;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const int rows = s_q * h_q;
  const int flat = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (flat >= rows) return;
  MergeState st;
  st.init();
  fold_parts<false, 4>(st, part_o, part_lse, first, 0, 1, n, static_cast<int64_t>(rows) * d_v,
                       rows, static_cast<int64_t>(flat) * d_v, flat, d_v, lane);
  const int s = flat / h_q, h = flat % h_q;
  const float l = finish_row<T>(st, d_v, out + b * o_sb + s * o_ss + h * o_sh, lane);
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

template <typename T>
cudaError_t launch_mla_combine_t(const float *part_o, const float *part_lse,
                                 const int32_t *num_splits, int batch, int s_q, int h_q, int d_v,
                                 void *out, int64_t o_sb, int64_t o_ss, int64_t o_sh, float *lse,
                                 cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((s_q * h_q + 3) / 4, batch);
  cfg.blockDim = dim3(128);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, mla_combine_kernel<T>, part_o, part_lse, num_splits, s_q, h_q,
                            d_v, static_cast<T *>(out), o_sb, o_ss, o_sh, lse);
}

cudaError_t launch_mla_combine(const float *part_o, const float *part_lse,
                               const int32_t *num_splits, int batch, int s_q, int h_q, int d_v,
                               void *out, int dtype, int64_t o_sb, int64_t o_ss, int64_t o_sh,
                               float *lse, cudaStream_t stream) {
  if (dtype == FA_DTYPE_BF16)
    return launch_mla_combine_t<__nv_bfloat16>(part_o, part_lse, num_splits, batch, s_q, h_q, d_v,
                                               out, o_sb, o_ss, o_sh, lse, stream);
  if (dtype == FA_DTYPE_F32)
    return launch_mla_combine_t<float>(part_o, part_lse, num_splits, batch, s_q, h_q, d_v, out,
                                       o_sb, o_ss, o_sh, lse, stream);
  return launch_mla_combine_t<__half>(part_o, part_lse, num_splits, batch, s_q, h_q, d_v, out,
                                      o_sb, o_ss, o_sh, lse, stream);
}

}  // namespace fa
