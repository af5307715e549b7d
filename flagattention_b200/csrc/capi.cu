// capi.cu -- the extern "C" boundary declared in include/flagattn_b200.h.
//
// Host-side argument validation (mirroring the reference's asserts, e.g.
// paged.py:45-46,124 and split_kv.py:281-289, as negative status codes),
// the reference's split heuristics, TMA tensor-map encoding and the launches.
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "flagattn_b200.h"

namespace fa {
void launch_mla_metadata(const int32_t *, int, int, int, int32_t *, int32_t *, cudaStream_t);
void launch_lse_combine(const float *, const float *, int, int64_t, int64_t, int64_t, int, int,
                        int, void *, int, int64_t, int64_t, int64_t, float *, cudaStream_t);
cudaError_t launch_mla_combine(const float *, const float *, const int32_t *, int, int, int, int,
                               bool, void *, int, int64_t, int64_t, int64_t, float *, cudaStream_t);
cudaError_t launch_generic_decode(const fa_decode_args *, cudaStream_t);
size_t generic_smem_bytes(int, int);
bool gqa_tc_eligible(const fa_decode_args *);
cudaError_t launch_gqa_tc(const CUtensorMap &, const CUtensorMap &, const fa_decode_args *, int,
                          int4 *, int, int, bool, cudaStream_t);
cudaError_t launch_gqa_combine(const float *, const float *, const int4 *, int, int, int, int,
                               int, int, int, int, bool, void *, int, int64_t, int64_t, int64_t,
                               float *, cudaStream_t);
int gqa_max_balanced_batch(const fa_decode_args *);
int gqa_tile_tokens(const fa_decode_args *, int pair);
int gqa_box_rows(const fa_decode_args *, int pair);
bool gqa_pairs_heads(const fa_decode_args *);
cudaError_t launch_mla_sv(const CUtensorMap &, const CUtensorMap &, const CUtensorMap &,
                          const CUtensorMap &, const fa_mla_args *, int, cudaStream_t);
}  // namespace fa

namespace {

thread_local char g_last_error[512] = "";

int fail(int status, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int status, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_fail(cudaError_t e, const char *what) {
  return fail(FA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int64_t cdiv64(int64_t a, int64_t b) { return (a + b - 1) / b; }

int next_pow2(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 3-D bf16/f16 map {d, rows, groups} with a {box_inner, box_rows, 1} box and
// the swizzle that matches the box width: 64 dims -> 128-byte swizzle, 32
// dims -> 64-byte swizzle (the UMMA SW128 / SW64 canonical layouts).
int encode_map(CUtensorMap *map, const void *base, int dtype, uint64_t d, uint64_t rows,
               uint64_t groups, uint64_t row_stride_elems, uint64_t group_stride_elems,
               uint32_t box_rows, uint32_t box_inner = 64) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(FA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {d, rows, groups};
  cuuint64_t strides[2] = {row_stride_elems * 2, group_stride_elems * 2};
  cuuint32_t box[3] = {box_inner, box_rows, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(map, dtype == FA_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                              : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                   3, const_cast<void *>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   box_inner == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(FA_ERR_INVALID_ARGUMENT,
                "tensor map rejected (code %d): dims {%llu,%llu,%llu} strides {%llu,%llu} B",
                static_cast<int>(r), (unsigned long long)d, (unsigned long long)rows,
                (unsigned long long)groups, (unsigned long long)strides[0],
                (unsigned long long)strides[1]);
  return FA_OK;
}

// 4-D map {d, rows, heads, groups} with a {64, box_rows, box_heads, 1} box
// and the 128-byte swizzle: a grouped-query cache, paged ([pages][kv heads]
// [page][d] or any strides) or contiguous ([batch][kv heads][n][d] or any
// strides); also the MLA value view, where "heads" are the 64-dim chunks of a
// latent row (stride 64 elements) so that one box brings rows x 512 dims laid
// out chunk by chunk.
int encode_map4(CUtensorMap *map, const void *base, int dtype, uint64_t d, uint64_t rows,
                uint64_t heads, uint64_t groups, int64_t row_stride, int64_t head_stride,
                int64_t group_stride, uint32_t box_rows, uint32_t box_heads = 1) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(FA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[4] = {d, rows, heads, groups};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(row_stride) * 2,
                           static_cast<cuuint64_t>(head_stride) * 2,
                           static_cast<cuuint64_t>(group_stride) * 2};
  // boxes of up to 64 dims: one swizzle row of 128 bytes, or of 64 / 32
  // bytes for head sizes 32 / 16 (the kernel's operand layout follows)
  const uint32_t inner = d < 64 ? static_cast<uint32_t>(d) : 64u;
  const CUtensorMapSwizzle swz = inner == 64   ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : inner == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                               : CU_TENSOR_MAP_SWIZZLE_32B;
  cuuint32_t box[4] = {inner, box_rows, box_heads, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = enc(map, dtype == FA_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                              : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                   4, const_cast<void *>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(FA_ERR_INVALID_ARGUMENT,
                "tensor map rejected (code %d): dims {%llu,%llu,%llu,%llu} strides "
                "{%llu,%llu,%llu} B",
                static_cast<int>(r), (unsigned long long)d, (unsigned long long)rows,
                (unsigned long long)heads, (unsigned long long)groups,
                (unsigned long long)strides[0], (unsigned long long)strides[1],
                (unsigned long long)strides[2]);
  return FA_OK;
}

// 2-D map over every row of a paged latent pool ({576, rows}, one row per
// box, 128-byte swizzle) for tile::gather4 loads of index-listed rows.
int encode_gather_map(CUtensorMap *map, const void *base, int dtype, uint64_t rows,
                      uint64_t row_stride_elems) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(FA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {576, rows};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {64, 1};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(map, dtype == FA_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                              : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                   2, const_cast<void *>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(FA_ERR_INVALID_ARGUMENT, "gather map rejected (code %d): rows %llu stride %llu B",
                static_cast<int>(r), (unsigned long long)rows,
                (unsigned long long)strides[0]);
  return FA_OK;
}

// K and V tensor maps of the grouped-query kernel: boxes of up to 64 dims x
// one page (at most one tile: 128 rows, 64 for head size 256, 64 of a
// 192-token tile for smaller heads) over {d, page rows, kv heads, pages}, or
// one tile of rows over {d, n, kv heads, batch} for contiguous caches.
// With `pair` (gqa_pairs_heads) a box spans two adjacent kv heads.  `a`
// describes the real heads.
int encode_kv_maps(const fa_decode_args *a, int pair, CUtensorMap *km, CUtensorMap *vm) {
  const bool paged = a->block_table != nullptr;
  const uint32_t box_rows = static_cast<uint32_t>(
      paged ? fa::gqa_box_rows(a, pair) : fa::gqa_tile_tokens(a, pair));
  const uint32_t box_heads = pair ? 2u : 1u;
  const uint64_t rows = paged ? a->page_size : static_cast<uint64_t>(a->n_ctx > 0 ? a->n_ctx : 1);
  const uint64_t groups = paged ? a->num_pages : a->batch;
  int st = encode_map4(km, a->k, a->dtype, a->d_qk, rows, a->num_kv_heads, groups,
                       a->k_stride_tok, a->k_stride_head, a->k_stride_seq, box_rows, box_heads);
  if (st != FA_OK) return st;
  return encode_map4(vm, a->v, a->dtype, a->d_v, rows, a->num_kv_heads, groups, a->k_stride_tok,
                     a->k_stride_head, a->k_stride_seq, box_rows, box_heads);
}

// The arguments as the tensor-core kernel sees them: with paired kv heads,
// half the kv heads (and so twice the group), everything else unchanged.
fa_decode_args kernel_view(const fa_decode_args *a, int pair) {
  fa_decode_args v = *a;
  if (pair) v.num_kv_heads /= 2;
  return v;
}

// Tensor-core kernel for these arguments?  Shapes, types and alignment
// (gqa_tc_eligible), a batch the maps can describe, and strides the TMA unit
// accepts (the encoder is asked; it runs on the host only).
bool tc_maps(const fa_decode_args *a, CUtensorMap *km, CUtensorMap *vm, int *pair) {
  *pair = 0;
  if (a->block_table == nullptr && a->seq_lens == nullptr && a->n_ctx < 1) return false;
  if (a->batch < 1 || !fa::gqa_tc_eligible(a)) return false;
  *pair = fa::gqa_pairs_heads(a) ? 1 : 0;
  return encode_kv_maps(a, *pair, km, vm) == FA_OK;
}
bool decode_on_tensor_cores(const fa_decode_args *a, int *pair = nullptr) {
  CUtensorMap km, vm;
  int pr = 0;
  const bool tc = tc_maps(a, &km, &vm, &pr);
  if (pair) *pair = pr;
  return tc;
}

int current_sm_count(int *sms) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  return fa_device_sm_count(dev, sms);
}

// `tc`: the arguments run on the tensor-core kernel (decode_on_tensor_cores).
int validate_decode(const fa_decode_args *a, bool tc) {
  if (!a) return fail(FA_ERR_INVALID_ARGUMENT, "null args");
  if (!a->q || !a->k || !a->v || !a->o) return fail(FA_ERR_INVALID_ARGUMENT, "null tensor");
  if (a->batch < 0 || a->num_q_heads <= 0 || a->num_kv_heads <= 0 || a->m_q <= 0)
    return fail(FA_ERR_INVALID_ARGUMENT, "bad batch/heads/m_q");
  if (a->num_q_heads % a->num_kv_heads != 0)
    return fail(FA_ERR_INVALID_ARGUMENT, "number of heads in q must be a multiple of that in k & v");
  if (a->d_qk <= 0 || a->d_qk > 576 || a->d_v <= 0 || a->d_v > 512 || a->d_v > a->d_qk)
    return fail(FA_ERR_UNSUPPORTED, "head size d_qk=%d d_v=%d outside [1,576]/[1,512]", a->d_qk,
                a->d_v);
  if (a->d_v % 4 != 0) return fail(FA_ERR_UNSUPPORTED, "d_v must be a multiple of 4");
  if (a->dtype != FA_DTYPE_BF16 && a->dtype != FA_DTYPE_F16 && a->dtype != FA_DTYPE_F32)
    return fail(FA_ERR_INVALID_ARGUMENT, "dtype %d", a->dtype);
  if (a->block_table) {
    if (a->page_size <= 0) return fail(FA_ERR_INVALID_ARGUMENT, "page_size %d", a->page_size);
    if (!a->seq_lens) return fail(FA_ERR_INVALID_ARGUMENT, "paged mode needs seq_lens");
    if (a->num_pages < 0) return fail(FA_ERR_INVALID_ARGUMENT, "num_pages %d", a->num_pages);
  } else if (!a->seq_lens && a->n_ctx < 0) {
    return fail(FA_ERR_INVALID_ARGUMENT, "n_ctx %d", a->n_ctx);
  }
  if (a->num_splits < 0 || (a->num_splits == 0 && !tc))
    return fail(FA_ERR_INVALID_ARGUMENT,
                "num_splits %d (0 selects the balanced schedule of the tensor-core kernel)",
                a->num_splits);
  if (a->num_splits == 0 && !a->sched)
    return fail(FA_ERR_INVALID_ARGUMENT, "the balanced schedule needs the sched scratch");
  if (a->num_splits == 0 && a->batch > fa::gqa_max_balanced_batch(a))
    return fail(FA_ERR_UNSUPPORTED, "balanced schedule: at most %d sequences per call",
                fa::gqa_max_balanced_batch(a));
  if (a->num_splits != 1 && (!a->part_o || !a->part_lse || !aligned16(a->part_o)))
    return fail(FA_ERR_INVALID_ARGUMENT, "split decode needs 16-byte aligned f32 workspace");
  if (a->num_splits > 1 && a->partition_size <= 0)
    return fail(FA_ERR_INVALID_ARGUMENT, "num_splits > 1 needs partition_size > 0");
  if (!tc && fa::generic_smem_bytes(a->d_qk, a->d_v) > 227 * 1024)
    return fail(FA_ERR_UNSUPPORTED, "head size too large for the generic kernel");
  return FA_OK;
}

// The tensor-core path: K / V tensor maps, then (balanced schedule) the
// scheduler kernel, the decode as its programmatic dependent and the merge
// of split entries as the decode's.
int run_decode_tc(const fa_decode_args *a, const CUtensorMap &km, const CUtensorMap &vm, int pair,
                  cudaStream_t s) {
  int sms = 0;
  int st = current_sm_count(&sms);
  if (st != FA_OK) return st;
  const int entries = a->batch * a->num_kv_heads;
  const int group = a->num_q_heads / a->num_kv_heads;
  const int qrows = group * a->m_q;
  cudaError_t e;
  if (a->num_splits == 0) {
    // every CTA cuts its share of the work out of the sequence lengths;
    // split entries leave merge records in the sched scratch
    int4 *merge = reinterpret_cast<int4 *>(a->sched);
    e = fa::launch_gqa_tc(km, vm, a, pair, merge, sms, sms, true, s);
    if (e != cudaSuccess) return cuda_fail(e, "tensor-core decode launch");
    e = fa::launch_gqa_combine(a->part_o, a->part_lse, merge, 0, entries, qrows, a->m_q, group,
                               a->num_kv_heads, a->num_q_heads, a->d_v,
                               static_cast<int64_t>(entries) * 4 <= sms, a->o, a->dtype,
                               a->o_stride_b, a->o_stride_h, a->o_stride_m, a->lse, s);
    if (e != cudaSuccess) return cuda_fail(e, "merge launch");
    return FA_OK;
  }
  const int ns = a->num_splits;
  const int64_t parts = static_cast<int64_t>(entries) * ns;
  if (parts > INT32_MAX) return fail(FA_ERR_UNSUPPORTED, "too many partitions");
  const int grid = static_cast<int>(parts < sms ? parts : sms);
  e = fa::launch_gqa_tc(km, vm, a, pair, nullptr, static_cast<int>(parts), grid, false, s);
  if (e != cudaSuccess) return cuda_fail(e, "tensor-core decode launch");
  if (ns > 1) {
    e = fa::launch_gqa_combine(a->part_o, a->part_lse, nullptr, ns, entries, qrows, a->m_q, group,
                               a->num_kv_heads, a->num_q_heads, a->d_v,
                               ns >= 8 && static_cast<int64_t>(entries) * 4 <= sms, a->o,
                               a->dtype, a->o_stride_b, a->o_stride_h, a->o_stride_m, a->lse, s);
    if (e != cudaSuccess) return cuda_fail(e, "merge launch");
  }
  return FA_OK;
}

int run_decode(const fa_decode_args *a, void *stream) {
  if (!a) return fail(FA_ERR_INVALID_ARGUMENT, "null args");
  // one eligibility test, one pair of tensor maps per call
  CUtensorMap km, vm;
  int pair = 0;
  const bool tc = tc_maps(a, &km, &vm, &pair);
  const fa_decode_args v = kernel_view(a, pair);  // the tensor-core kernel's view
  int st = validate_decode(tc ? &v : a, tc);
  if (st != FA_OK) return st;
  if (a->batch == 0) return FA_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (tc) return run_decode_tc(&v, km, vm, pair, s);
  cudaError_t e = fa::launch_generic_decode(a, s);
  if (e != cudaSuccess) return cuda_fail(e, "generic decode launch");
  if (a->num_splits > 1) {
    const int64_t rows = static_cast<int64_t>(a->batch) * a->num_q_heads * a->m_q;
    fa::launch_lse_combine(a->part_o, a->part_lse, a->num_splits, rows * a->d_v, rows, rows,
                           a->num_q_heads, a->m_q, a->d_v, a->o, a->dtype, a->o_stride_b,
                           a->o_stride_h, a->o_stride_m, a->lse, s);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "combine launch");
  }
  return FA_OK;
}

int mla_m_blocks(int s_q, int h_q, bool sparse) {
  return sparse ? s_q : static_cast<int>(cdiv64(static_cast<int64_t>(s_q) * h_q, 128));
}

int validate_mla(const fa_mla_args *a) {
  if (!a) return fail(FA_ERR_INVALID_ARGUMENT, "null args");
  const bool sparse = a->indices != nullptr;
  if (!a->q || !a->kcache || !a->out || !a->lse || !a->tile_meta || !a->num_splits)
    return fail(FA_ERR_INVALID_ARGUMENT, "null tensor");
  if (a->d_qk != 576 || a->d_v != 512)
    return fail(FA_ERR_UNSUPPORTED, "MLA path needs d_qk=576, d_v=512 (got %d/%d)", a->d_qk,
                a->d_v);
  if (a->dtype != FA_DTYPE_BF16 && a->dtype != FA_DTYPE_F16)
    return fail(FA_ERR_UNSUPPORTED, "MLA path computes in bf16 or f16");
  if (a->out_dtype != a->dtype && a->out_dtype != FA_DTYPE_F32)
    return fail(FA_ERR_INVALID_ARGUMENT, "out_dtype must equal dtype or be f32");
  if (a->batch < 0 || a->s_q <= 0 || a->h_q <= 0) return fail(FA_ERR_INVALID_ARGUMENT, "shape");
  if (sparse && a->h_q > 128) return fail(FA_ERR_UNSUPPORTED, "sparse path needs h_q <= 128");
  if (sparse && (a->topk <= 0 || a->causal))
    return fail(FA_ERR_INVALID_ARGUMENT, "sparse needs topk > 0 and causal == 0");
  if (a->num_sm_parts <= 0) return fail(FA_ERR_INVALID_ARGUMENT, "num_sm_parts");
  if (!aligned16(a->q) || !aligned16(a->kcache) || !aligned16(a->out))
    return fail(FA_ERR_INVALID_ARGUMENT, "q / kcache / out must be 16-byte aligned");
  if (a->q_stride_h % 8 || a->q_stride_b % 8 || a->q_stride_s % 8 || a->kv_stride_tok % 8 ||
      a->kv_stride_page % 8 || a->o_stride_b % 8 || a->o_stride_s % 8 || a->o_stride_h % 8)
    return fail(FA_ERR_INVALID_ARGUMENT, "strides must be multiples of 8 elements (16 bytes)");
  if (a->s_q > 1 && a->q_stride_s != static_cast<int64_t>(a->h_q) * a->q_stride_h)
    return fail(FA_ERR_UNSUPPORTED, "q rows (s_q, h_q) must be contiguous: q_stride_s == h_q*q_stride_h");
  if (a->page_size <= 0 || a->page_size % 64 != 0)
    return fail(FA_ERR_UNSUPPORTED, "page_size must be a multiple of 64 (got %d)", a->page_size);
  if (!sparse && a->block_table == nullptr && !a->seq_lens && a->n_ctx < 0)
    return fail(FA_ERR_INVALID_ARGUMENT, "n_ctx");
  if (!sparse && a->block_table != nullptr && !a->seq_lens)
    return fail(FA_ERR_INVALID_ARGUMENT, "paged dense decode needs seq_lens");
  if (!a->part_o || !a->part_lse || !aligned16(a->part_o))
    return fail(FA_ERR_INVALID_ARGUMENT, "workspace must be given and 16-byte aligned");
  return FA_OK;
}

}  // namespace

namespace fa {
// Record a message for fa_last_error() from another translation unit.
int record_error(int status, const char *msg) { return fail(status, "%s", msg); }
}  // namespace fa

extern "C" {

int fa_version(void) { return (0 << 16) | (3 << 8) | 0; }

const char *fa_status_string(int status) {
  switch (status) {
    case FA_OK: return "ok";
    case FA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case FA_ERR_UNSUPPORTED: return "unsupported";
    case FA_ERR_CUDA: return "cuda error";
    case FA_ERR_NO_DEVICE: return "no device";
    default: return "unknown status";
  }
}

const char *fa_last_error(void) { return g_last_error; }

int fa_device_sm_count(int device, int *sm_count) {
  if (!sm_count) return fail(FA_ERR_INVALID_ARGUMENT, "null out");
  cudaError_t e = cudaDeviceGetAttribute(sm_count, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return fail(FA_ERR_NO_DEVICE, "%s", cudaGetErrorString(e));
  return FA_OK;
}

int fa_paged_num_splits(int num_seqs, int num_kv_heads, int max_context_len, int kv_block_size,
                        int num_sms, int requested_splits, int *num_splits, int *partition_size) {
  if (!num_splits || !partition_size) return fail(FA_ERR_INVALID_ARGUMENT, "null out");
  int ns = requested_splits, ps = 0;
  if (ns == 0) {
    if (static_cast<int64_t>(num_seqs) * num_kv_heads > 2LL * num_sms) {
      ns = 1;
      if (max_context_len >= 4096) {
        ps = kv_block_size > 256 ? kv_block_size : 256;
        ns = static_cast<int>(cdiv64(max_context_len, ps));
      }
    } else {
      ps = kv_block_size > 256 ? kv_block_size : 256;
      ns = static_cast<int>(cdiv64(max_context_len, ps));
      if (max_context_len <= 1024 || kv_block_size >= 256) ns = 1;
    }
  } else if (ns > 1) {
    ps = next_pow2(static_cast<int>(cdiv64(max_context_len, ns)));
  }
  if (ns < 1) ns = 1;
  if (ns == 1) ps = 0;
  *num_splits = ns;
  *partition_size = ps;
  return FA_OK;
}

int fa_split_kv_num_splits(int batch, int heads, int m, int n, int block_m, int block_n,
                           int num_sms, int max_splits, int *num_splits) {
  if (!num_splits || block_m <= 0 || block_n <= 0 || num_sms <= 0)
    return fail(FA_ERR_INVALID_ARGUMENT, "bad heuristic arguments");
  const int64_t nb = static_cast<int64_t>(batch) * heads * cdiv64(m, block_m);
  *num_splits = 1;
  if (static_cast<double>(nb) >= 0.8 * num_sms) return FA_OK;
  const int64_t n_blocks = cdiv64(n, block_n);
  int64_t lim = num_sms;
  if (n_blocks < lim) lim = n_blocks;
  if (max_splits < lim) lim = max_splits;
  double best = 0.0;
  double eff[1024];
  bool avail[1024];
  if (lim > 1023) lim = 1023;
  for (int64_t s = 1; s <= lim; ++s) {
    const int64_t per = cdiv64(n_blocks, s);
    avail[s] = (s == 1) || (per * s - n_blocks < per);
    if (avail[s]) {
      const double waves = static_cast<double>(nb * s) / static_cast<double>(num_sms);
      eff[s] = waves / std::ceil(waves);
      if (eff[s] > best) best = eff[s];
    }
  }
  for (int64_t s = 1; s <= lim; ++s) {
    if (avail[s] && eff[s] >= 0.85 * best) {
      *num_splits = static_cast<int>(s);
      return FA_OK;
    }
  }
  return FA_OK;
}

int fa_decode_uses_tensor_cores(const fa_decode_args *a) {
  if (!a) return fail(FA_ERR_INVALID_ARGUMENT, "null args");
  return decode_on_tensor_cores(a) ? 1 : 0;
}

int fa_decode_workspace_size(const fa_decode_args *a, size_t *part_o_bytes,
                             size_t *part_lse_bytes, size_t *sched_bytes) {
  if (!a || !part_o_bytes || !part_lse_bytes || !sched_bytes)
    return fail(FA_ERR_INVALID_ARGUMENT, "null");
  if (a->batch < 0 || a->num_q_heads <= 0 || a->num_kv_heads <= 0 || a->m_q <= 0 ||
      a->d_v <= 0 || a->num_splits < 0)
    return fail(FA_ERR_INVALID_ARGUMENT, "bad arguments");
  size_t slots = 0, sched = 0;
  int pair = 0;
  const bool tc = decode_on_tensor_cores(a, &pair);
  const fa_decode_args v = kernel_view(a, pair);
  if (tc) a = &v;  // sizes of the tensor-core kernel's view (paired kv heads)
  if (a->num_splits == 0) {
    if (!tc)
      return fail(FA_ERR_INVALID_ARGUMENT, "num_splits 0 needs the tensor-core kernel");
    int sms = 0;
    int st = current_sm_count(&sms);
    if (st != FA_OK) return st;
    if (a->batch > fa::gqa_max_balanced_batch(a))
      return fail(FA_ERR_UNSUPPORTED, "balanced schedule: at most %d sequences per call",
                  fa::gqa_max_balanced_batch(a));
    // two split slots per CTA (its first and its last piece); one int4 merge
    // record per entry
    slots = 2 * static_cast<size_t>(sms);
    sched = static_cast<size_t>(a->batch) * a->num_kv_heads * 4 * sizeof(int32_t);
  } else if (a->num_splits > 1) {
    slots = static_cast<size_t>(a->batch) * a->num_kv_heads * a->num_splits;
  }
  // slot = the rows of one kv head's group (tensor-core layout) or, for the
  // CUDA-core layout [split][batch][heads][m_q], the same total
  const size_t rows = static_cast<size_t>(a->num_q_heads / a->num_kv_heads) * a->m_q;
  size_t cells = 0, o_bytes = 0, lse_bytes = 0;
  if (__builtin_mul_overflow(slots, rows, &cells) ||
      __builtin_mul_overflow(cells, static_cast<size_t>(a->d_v) * sizeof(float), &o_bytes) ||
      __builtin_mul_overflow(cells, sizeof(float), &lse_bytes))
    return fail(FA_ERR_INVALID_ARGUMENT, "workspace size overflows size_t");
  *part_o_bytes = o_bytes;
  *part_lse_bytes = lse_bytes;
  *sched_bytes = sched;
  return FA_OK;
}

int fa_paged_attention(const fa_decode_args *a, void *stream) {
  if (a && !a->block_table) return fail(FA_ERR_INVALID_ARGUMENT, "paged attention needs a block table");
  return run_decode(a, stream);
}

int fa_split_kv_attention(const fa_decode_args *a, void *stream) {
  if (a && a->block_table) return fail(FA_ERR_INVALID_ARGUMENT, "split-KV attention takes contiguous keys");
  return run_decode(a, stream);
}

int fa_lse_combine(const float *part_o, const float *part_lse, int num_parts, int64_t rows,
                   int d_v, void *o, int dtype, float *lse, void *stream) {
  return fa_lse_combine_strided(part_o, rows * d_v, part_lse, rows, num_parts, rows, d_v, o, dtype,
                                lse, stream);
}

int fa_lse_combine_strided(const float *part_o, int64_t o_part_stride, const float *part_lse,
                           int64_t lse_part_stride, int num_parts, int64_t rows, int d_v, void *o,
                           int dtype, float *lse, void *stream) {
  if (!part_o || !part_lse || !o || num_parts < 1 || rows < 0 || d_v <= 0 || d_v % 4)
    return fail(FA_ERR_INVALID_ARGUMENT, "bad combine arguments");
  if (d_v > 512) return fail(FA_ERR_UNSUPPORTED, "combine supports d_v <= 512 (got %d)", d_v);
  if (o_part_stride < rows * d_v || lse_part_stride < 0 || o_part_stride % 4)
    return fail(FA_ERR_INVALID_ARGUMENT, "combine part strides must cover a part (and keep "
                                         "16-byte alignment)");
  if (!aligned16(part_o)) return fail(FA_ERR_INVALID_ARGUMENT, "part_o must be 16-byte aligned");
  if (dtype != FA_DTYPE_BF16 && dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_F32)
    return fail(FA_ERR_INVALID_ARGUMENT, "dtype %d", dtype);
  fa::launch_lse_combine(part_o, part_lse, num_parts, o_part_stride, lse_part_stride, rows, 1, 1,
                         d_v, o, dtype, d_v, 0, 0, lse, static_cast<cudaStream_t>(stream));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? FA_OK : cuda_fail(e, "combine launch");
}

int fa_mla_num_sm_parts(int device, int s_q, int h_q, int sparse, int *num_sm_parts) {
  if (!num_sm_parts || s_q <= 0 || h_q <= 0) return fail(FA_ERR_INVALID_ARGUMENT, "bad arguments");
  int sms = 0;
  int st = fa_device_sm_count(device, &sms);
  if (st != FA_OK) return st;
  const int mb = mla_m_blocks(s_q, h_q, sparse != 0);
  int parts = sms / 2 / mb;
  *num_sm_parts = parts > 0 ? parts : 1;
  return FA_OK;
}

int fa_mla_workspace_size(int batch, int s_q, int h_q, int d_v, int num_sm_parts,
                          size_t *part_o_bytes, size_t *part_lse_bytes) {
  if (!part_o_bytes || !part_lse_bytes || batch < 0 || num_sm_parts < 1 || s_q <= 0 ||
      h_q <= 0 || d_v <= 0)
    return fail(FA_ERR_INVALID_ARGUMENT, "bad arguments");
  const size_t slots = static_cast<size_t>(batch) + num_sm_parts;
  size_t rows = 0, cells = 0, o_bytes = 0, lse_bytes = 0;
  if (__builtin_mul_overflow(static_cast<size_t>(s_q), static_cast<size_t>(h_q), &rows) ||
      __builtin_mul_overflow(slots, rows, &cells) ||
      __builtin_mul_overflow(cells, static_cast<size_t>(d_v) * sizeof(float), &o_bytes) ||
      __builtin_mul_overflow(cells, sizeof(float), &lse_bytes))
    return fail(FA_ERR_INVALID_ARGUMENT, "workspace size overflows size_t");
  *part_o_bytes = o_bytes;
  *part_lse_bytes = lse_bytes;
  return FA_OK;
}

int fa_mla_get_metadata(const int32_t *seq_lens, int batch, int topk, int num_sm_parts,
                        int32_t *tile_meta, int32_t *num_splits, void *stream) {
  if (batch < 0 || num_sm_parts < 1 || !tile_meta || !num_splits || (topk <= 0 && !seq_lens && batch))
    return fail(FA_ERR_INVALID_ARGUMENT, "bad metadata arguments");
  fa::launch_mla_metadata(seq_lens, batch, topk, num_sm_parts, tile_meta, num_splits,
                          static_cast<cudaStream_t>(stream));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? FA_OK : cuda_fail(e, "metadata launch");
}

int fa_mla_combine(const fa_mla_args *a, void *stream) {
  int st = validate_mla(a);
  if (st != FA_OK) return st;
  if (a->batch == 0) return FA_OK;
  // few sequences over many parts: each is split many ways, so the combine
  // spreads a row's partials over four warps
  const bool wide = static_cast<int64_t>(a->batch) * 4 <= a->num_sm_parts;
  cudaError_t e = fa::launch_mla_combine(a->part_o, a->part_lse, a->num_splits, a->batch, a->s_q,
                                         a->h_q, a->d_v, wide, a->out, a->out_dtype,
                                         a->o_stride_b, a->o_stride_s, a->o_stride_h, a->lse,
                                         static_cast<cudaStream_t>(stream));
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? FA_OK : cuda_fail(e, "MLA combine launch");
}

int fa_mla_decode_partial(const fa_mla_args *a, void *stream) {
  int st = validate_mla(a);
  if (st != FA_OK) return st;
  if (a->batch == 0) return FA_OK;
  const bool sparse = a->indices != nullptr;
  const int bn = FA_MLA_BLOCK_N;
  const int m_blocks = mla_m_blocks(a->s_q, a->h_q, sparse);
  const bool paged = a->block_table != nullptr;
  const uint64_t kv_rows = (sparse || paged) ? a->page_size : (a->n_ctx > 0 ? a->n_ctx : 1);
  const uint64_t kv_groups = (sparse || paged) ? a->num_pages : a->batch;
  // One score / value CTA kernel for dense and top-k decode: query box 64
  // dims x 128 rows, key rows in 64-row boxes, value rows in 32-row boxes.
  // Top-k rows come from a gather map: when every pool row lies at one stride
  // (pages back to back) a 2-D map over all rows read by tile::gather4,
  // otherwise the 3-D page map with one-row boxes.
  CUtensorMap qm, km, vm, gm;
  st = encode_map(&qm, a->q, a->dtype, 576, static_cast<uint64_t>(a->s_q) * a->h_q, a->batch,
                  a->q_stride_h, a->q_stride_b, 128, 64);
  if (st != FA_OK) return st;
  st = encode_map(&km, a->kcache, a->dtype, 576, kv_rows, kv_groups, a->kv_stride_tok,
                  a->kv_stride_page, bn, 64);
  if (st != FA_OK) return st;
  // values: {64 dims, rows, 9 chunks of 64 dims, pages}; one 32-row x 8-chunk
  // box (32 KB) fills a whole value stage, [chunk][row][64 dims]
  st = encode_map4(&vm, a->kcache, a->dtype, 64, kv_rows, 576 / 64, kv_groups, a->kv_stride_tok,
                   64, a->kv_stride_page, 32, 8);
  if (st != FA_OK) return st;
  if (sparse) {
    const bool uniform_rows =
        a->kv_stride_page == static_cast<int64_t>(a->page_size) * a->kv_stride_tok;
    st = uniform_rows
             ? encode_gather_map(&gm, a->kcache, a->dtype,
                                 static_cast<uint64_t>(a->num_pages) * a->page_size,
                                 a->kv_stride_tok)
             : encode_map(&gm, a->kcache, a->dtype, 576, a->page_size, a->num_pages,
                          a->kv_stride_tok, a->kv_stride_page, 1, 64);
    if (st != FA_OK) return st;
  } else {
    gm = qm;  // not read by the dense instance
  }
  cudaError_t e = fa::launch_mla_sv(qm, km, vm, gm, a, m_blocks, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? FA_OK : cuda_fail(e, "MLA decode launch");
}

int fa_mla_decode(const fa_mla_args *a, void *stream) {
  int st = fa_mla_decode_partial(a, stream);
  if (st != FA_OK || a->batch == 0) return st;
  return fa_mla_combine(a, stream);
}

}  // extern "C"
