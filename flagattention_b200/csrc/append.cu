// append.cu -- write new tokens' latent rows into their cache pages.
//
// The decode kernels read a token's 576-dim latent row (512 latent + 64 rope
// dims, bf16/f16) from page slot[token] / page_size, row slot % page_size of
// the pool.  This is the step before a decode: the tokens produced in the
// previous step get their rows.  The caller maps tokens to pool rows (a
// slot mapping, as paged serving engines keep one); a negative slot skips the
// token (padding), and a slot past the pool is skipped too, so no write can
// leave the pool.  Byte movement only: one warp per row, 72 coalesced 16-byte
// copies (1152 bytes), HBM-bound.
#include "common.cuh"
#include "flagattn_b200.h"

namespace fa {

constexpr int kRowChunks = 576 * 2 / 16;  // 16-byte pieces of a latent row
constexpr int kAppendRowsPerBlock = 8;   // one warp per row

__global__ void __launch_bounds__(32 * kAppendRowsPerBlock)
    append_rows_kernel(const uint8_t *__restrict__ rows, int64_t rows_stride_bytes,
                       const int64_t *__restrict__ slots, int64_t n, uint8_t *__restrict__ kcache,
                       int64_t page_stride_bytes, int64_t tok_stride_bytes, int page_size,
                       int64_t total_rows) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * kAppendRowsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= n) return;
  const int64_t slot = __ldg(slots + r);
  if (slot < 0 || slot >= total_rows) return;
  const uint4 *src = reinterpret_cast<const uint4 *>(rows + r * rows_stride_bytes);
  uint4 *dst = reinterpret_cast<uint4 *>(kcache + (slot / page_size) * page_stride_bytes +
                                         (slot % page_size) * tok_stride_bytes);
  for (int c = lane; c < kRowChunks; c += 32) dst[c] = __ldg(src + c);
}

int record_error(int status, const char *msg);  // capi.cu: message for fa_last_error()

}  // namespace fa

extern "C" int fa_mla_append_rows(const void *rows, int64_t rows_stride, const int64_t *slots,
                                  int64_t n, void *kcache, int64_t kv_stride_page,
                                  int64_t kv_stride_tok, int32_t num_pages, int32_t page_size,
                                  int32_t dtype, void *stream) {
  if (n < 0) return fa::record_error(FA_ERR_INVALID_ARGUMENT, "append: negative row count");
  if (dtype != FA_DTYPE_BF16 && dtype != FA_DTYPE_F16)
    return fa::record_error(FA_ERR_UNSUPPORTED, "append: latent rows are bf16 or f16");
  if (page_size <= 0 || num_pages < 0)
    return fa::record_error(FA_ERR_INVALID_ARGUMENT, "append: page_size / num_pages");
  if (n == 0) return FA_OK;
  if (!rows || !slots || !kcache) return fa::record_error(FA_ERR_INVALID_ARGUMENT, "append: null pointer");
  if ((reinterpret_cast<uintptr_t>(rows) & 15u) || (reinterpret_cast<uintptr_t>(kcache) & 15u) ||
      (reinterpret_cast<uintptr_t>(slots) & 7u))
    return fa::record_error(FA_ERR_INVALID_ARGUMENT,
                        "append: rows / kcache must be 16-byte aligned, slots 8-byte aligned");
  if (rows_stride < 576 || rows_stride % 8 || kv_stride_tok < 576 || kv_stride_tok % 8 ||
      kv_stride_page % 8 || kv_stride_page < static_cast<int64_t>(page_size) * kv_stride_tok)
    return fa::record_error(FA_ERR_INVALID_ARGUMENT,
                        "append: strides must be multiples of 8 elements covering a 576-dim row");
  const int64_t blocks = (n + fa::kAppendRowsPerBlock - 1) / fa::kAppendRowsPerBlock;
  if (blocks > 0x7fffffffLL) return fa::record_error(FA_ERR_INVALID_ARGUMENT, "append: too many rows");
  fa::append_rows_kernel<<<static_cast<unsigned>(blocks), 32 * fa::kAppendRowsPerBlock, 0,
                           static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t *>(rows), rows_stride * 2, slots, n,
      static_cast<uint8_t *>(kcache), kv_stride_page * 2, kv_stride_tok * 2, page_size,
      static_cast<int64_t>(num_pages) * page_size);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? FA_OK : fa::record_error(FA_ERR_CUDA, cudaGetErrorString(e));
}
