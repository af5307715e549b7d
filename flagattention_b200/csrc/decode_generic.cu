// decode_generic.cu -- paged / contiguous decode for arbitrary head sizes.
//
// The general form of the reference decode kernels (paged.py:208-363 for
// paged caches, split_kv.py:28-174 for contiguous keys): grouped-query heads,
// any head size up to 576 (values up to 512), f16 / bf16 / f32, split over
// the key axis, bottom-right causal masking when several query rows share a
// sequence.  One CTA owns 16 query rows of one kv head (all rows read the same
// key/value rows, so each key tile is staged once in shared memory for the
// group) and one split of the keys; tiles of 16 keys go through an online
// softmax in f32.  The tensor-core MLA kernel (mla_sv.cu) serves the 576/512
// latent shape; this kernel serves every other shape.
#include "common.cuh"
#include "flagattn_b200.h"

namespace fa {

constexpr int kGenRows = 16;     // query rows per CTA
constexpr int kGenTile = 16;     // keys per tile
constexpr int kGenThreads = 256; // = kGenRows * kGenTile
constexpr int kGenMaxDvPerThread = 512 / 16;

struct GenericParams {
  const void *q;
  int64_t q_sb, q_sh, q_sm;
  const void *k;
  const void *v;
  int64_t k_sseq, k_stok, k_shead;
  const int32_t *block_table;
  int64_t bt_stride;
  int32_t page_size;
  const int32_t *seq_lens;
  int32_t n_ctx;
  int32_t batch, hq, hkv, m_q, d_qk, d_v, causal;
  float scale;
  int32_t num_splits, partition_size;
  void *o;
  int64_t o_sb, o_sh, o_sm;
  float *lse;
  float *part_o;
  float *part_lse;
};

template <typename T>
__device__ __forceinline__ const T *key_row(const GenericParams &p, const T *base, int b, int kvh,
                                            int n) {
  if (p.block_table != nullptr) {
    const int page = p.block_table[static_cast<int64_t>(b) * p.bt_stride + n / p.page_size];
    return base + static_cast<int64_t>(page) * p.k_sseq +
           static_cast<int64_t>(n % p.page_size) * p.k_stok + static_cast<int64_t>(kvh) * p.k_shead;
  }
  return base + static_cast<int64_t>(b) * p.k_sseq + static_cast<int64_t>(n) * p.k_stok +
         static_cast<int64_t>(kvh) * p.k_shead;
}

template <typename T>
__global__ void __launch_bounds__(kGenThreads)
    generic_decode_kernel(const GenericParams p) {
  extern __shared__ float gsmem[];
  const int dq = p.d_qk, dv = p.d_v;
  const int ldq = dq + 1;  // padded rows avoid bank conflicts in the dot products
  float *q_s = gsmem;                       // [kGenRows][ldq]
  float *k_s = q_s + kGenRows * ldq;        // [kGenTile][ldq]
  float *v_s = k_s + kGenTile * ldq;        // [kGenTile][dv]
  float *p_s = v_s + kGenTile * dv;         // [kGenRows][kGenTile]
  float *a_s = p_s + kGenRows * kGenTile;   // [kGenRows]

  const int split = blockIdx.x;
  const int group = p.hq / p.hkv;
  const int rows_per_kvh = group * p.m_q;
  const int row_blocks = (rows_per_kvh + kGenRows - 1) / kGenRows;
  const int kvh = blockIdx.y / row_blocks;
  const int rb = blockIdx.y % row_blocks;
  const int b = blockIdx.z;
  const int tid = threadIdx.x;
  const T *qb = static_cast<const T *>(p.q);
  const T *kb = static_cast<const T *>(p.k);
  const T *vb = static_cast<const T *>(p.v);

  const int n_len = p.seq_lens ? p.seq_lens[b] : p.n_ctx;
  const int part = p.partition_size > 0 ? p.partition_size : n_len;
  const int n_lo = split * part;
  const int n_hi = min(n_len, n_lo + part);

  // Query rows of this CTA: row r -> (head g within the group, query index m).
  for (int i = tid; i < kGenRows * dq; i += kGenThreads) {
    const int r = i / dq, d = i % dq;
    const int gr = rb * kGenRows + r;
    float val = 0.f;
    if (gr < rows_per_kvh) {
      const int h = kvh * group + gr / p.m_q, m = gr % p.m_q;
      val = Elem<T>::to_f(qb[b * p.q_sb + h * p.q_sh + m * p.q_sm + d]);
    }
    q_s[r * ldq + d] = val;
  }

  const int my_r = tid / kGenTile;      // score row of this thread
  const int my_t = tid % kGenTile;      // score column of this thread
  const int my_gr = rb * kGenRows + my_r;
  const int my_m = my_gr < rows_per_kvh ? my_gr % p.m_q : 0;
  // bottom-right causal limit: query m sees keys n <= m + (n_len - m_q)
  const int row_limit = p.causal ? my_m + n_len - p.m_q + 1 : n_len;
  float m_i = -INFINITY, l_i = 0.f;
  float acc[kGenMaxDvPerThread];
#pragma unroll
  for (int j = 0; j < kGenMaxDvPerThread; ++j) acc[j] = 0.f;
  const int o_r = tid / 16, o_c = tid % 16;  // output ownership: row o_r, dims o_c + 16 j

  for (int n0 = n_lo; n0 < n_hi; n0 += kGenTile) {
    __syncthreads();
    for (int i = tid; i < kGenTile * dq; i += kGenThreads) {
      const int t = i / dq, d = i % dq;
      const int n = n0 + t;
      k_s[t * ldq + d] = (n < n_hi) ? Elem<T>::to_f(key_row<T>(p, kb, b, kvh, n)[d]) : 0.f;
    }
    for (int i = tid; i < kGenTile * dv; i += kGenThreads) {
      const int t = i / dv, d = i % dv;
      const int n = n0 + t;
      v_s[t * dv + d] = (n < n_hi) ? Elem<T>::to_f(key_row<T>(p, vb, b, kvh, n)[d]) : 0.f;
    }
    __syncthreads();
    float s = 0.f;
    const float *qr = q_s + my_r * ldq;
    const float *kr = k_s + my_t * ldq;
    for (int d = 0; d < dq; ++d) s = fmaf(qr[d], kr[d], s);
    const int n = n0 + my_t;
    const bool valid = (n < n_hi) && (n < row_limit);
    s = valid ? s * p.scale : -INFINITY;
    float tmax = s;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
    const float m_new = fmaxf(m_i, tmax);
    const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
    const float alpha = (m_i == -INFINITY) ? 0.f : expf(m_i - m_use);
    const float pv = valid ? expf(s - m_use) : 0.f;
    float psum = pv;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
    l_i = l_i * alpha + psum;
    m_i = m_new;
    p_s[my_r * kGenTile + my_t] = pv;
    if (my_t == 0) a_s[my_r] = alpha;
    __syncthreads();
    const float al = a_s[o_r];
#pragma unroll
    for (int j = 0; j < kGenMaxDvPerThread; ++j) {
      const int d = o_c + 16 * j;
      if (d < dv) {
        float a = acc[j] * al;
#pragma unroll
        for (int t = 0; t < kGenTile; ++t) a = fmaf(p_s[o_r * kGenTile + t], v_s[t * dv + d], a);
        acc[j] = a;
      }
    }
  }

  // Row statistics live in every thread of the row's half warp; the output
  // owner of row o_r reads them through shared memory.
  __syncthreads();
  if (my_t == 0) {
    p_s[my_r * kGenTile + 0] = m_i;
    p_s[my_r * kGenTile + 1] = l_i;
  }
  __syncthreads();
  const float mr = p_s[o_r * kGenTile + 0];
  const float lr = p_s[o_r * kGenTile + 1];
  const int gr = rb * kGenRows + o_r;
  if (gr >= rows_per_kvh) return;
  const int h = kvh * group + gr / p.m_q, m = gr % p.m_q;
  const float inv = lr > 0.f ? 1.f / lr : 0.f;
  const float lse = lr > 0.f ? mr + logf(lr) : -INFINITY;
  const int64_t row = (static_cast<int64_t>(b) * p.hq + h) * p.m_q + m;
  if (p.num_splits == 1) {
    T *o = static_cast<T *>(p.o) + b * p.o_sb + h * p.o_sh + m * p.o_sm;
#pragma unroll
    for (int j = 0; j < kGenMaxDvPerThread; ++j) {
      const int d = o_c + 16 * j;
      if (d < dv) o[d] = Elem<T>::from_f(acc[j] * inv);
    }
    if (p.lse != nullptr && o_c == 0) p.lse[row] = lse;
  } else {
    const int64_t rows = static_cast<int64_t>(p.batch) * p.hq * p.m_q;
    float *po = p.part_o + (static_cast<int64_t>(split) * rows + row) * dv;
#pragma unroll
    for (int j = 0; j < kGenMaxDvPerThread; ++j) {
      const int d = o_c + 16 * j;
      if (d < dv) po[d] = acc[j] * inv;
    }
    if (o_c == 0) p.part_lse[static_cast<int64_t>(split) * rows + row] = lse;
  }
}

size_t generic_smem_bytes(int d_qk, int d_v) {
  return sizeof(float) * (static_cast<size_t>(kGenRows + kGenTile) * (d_qk + 1) +
                          static_cast<size_t>(kGenTile) * d_v + kGenRows * kGenTile + kGenRows);
}

template <typename T>
static cudaError_t launch_generic_t(const GenericParams &p, cudaStream_t stream) {
  const size_t smem = generic_smem_bytes(p.d_qk, p.d_v);
  cudaError_t e = cudaFuncSetAttribute(generic_decode_kernel<T>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const int group = p.hq / p.hkv;
  const int row_blocks = (group * p.m_q + kGenRows - 1) / kGenRows;
  dim3 grid(p.num_splits, p.hkv * row_blocks, p.batch);
  generic_decode_kernel<T><<<grid, kGenThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_generic_decode(const fa_decode_args *a, cudaStream_t stream) {
  GenericParams p;
  p.q = a->q;
  p.q_sb = a->q_stride_b;
  p.q_sh = a->q_stride_h;
  p.q_sm = a->q_stride_m;
  p.k = a->k;
  p.v = a->v;
  p.k_sseq = a->k_stride_seq;
  p.k_stok = a->k_stride_tok;
  p.k_shead = a->k_stride_head;
  p.block_table = a->block_table;
  p.bt_stride = a->bt_stride;
  p.page_size = a->page_size;
  p.seq_lens = a->seq_lens;
  p.n_ctx = a->n_ctx;
  p.batch = a->batch;
  p.hq = a->num_q_heads;
  p.hkv = a->num_kv_heads;
  p.m_q = a->m_q;
  p.d_qk = a->d_qk;
  p.d_v = a->d_v;
  p.causal = a->causal;
  p.scale = a->scale;
  p.num_splits = a->num_splits;
  p.partition_size = a->partition_size;
  p.o = a->o;
  p.o_sb = a->o_stride_b;
  p.o_sh = a->o_stride_h;
  p.o_sm = a->o_stride_m;
  p.lse = a->lse;
  p.part_o = a->part_o;
  p.part_lse = a->part_lse;
  switch (a->dtype) {
    case FA_DTYPE_BF16: return launch_generic_t<__nv_bfloat16>(p, stream);
    case FA_DTYPE_F16: return launch_generic_t<__half>(p, stream);
    default: return launch_generic_t<float>(p, stream);
  }
}

}  // namespace fa
