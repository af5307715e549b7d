// sched.cu -- device tile scheduler for the MLA decode kernels.
//
// Emits the metadata format declared in include/flagattn_b200.h: each of the
// num_sm_parts 2-SM parts receives an equal budget of 64-token blocks plus a
// fixed per-piece cost, and walks the sequences in order.  The loop is pure
// integer arithmetic so it equals the host specification bit-for-bit; the
// reference has no counterpart (its split count is one per call,
// split_kv.py:247-276 / paged.py:54-67).
#include "common.cuh"
#include "flagattn_b200.h"

namespace fa {

constexpr int kSchedThreads = 256;
constexpr int kSchedSmemSeqs = 10240;  // sequences staged in shared memory

__device__ __forceinline__ int blocks_of_len(int len) {
  return len > 0 ? (len + FA_MLA_BLOCK_N - 1) / FA_MLA_BLOCK_N : 0;
}

// The block stages the per-sequence block counts in shared memory (when the
// batch fits), then one thread walks the batch (O(batch + parts) work).
// A sequence's prefix entry is written when its last piece is placed.
__global__ void __launch_bounds__(kSchedThreads)
    mla_metadata_kernel(const int32_t *__restrict__ seq_lens, int batch, int topk, int num_parts,
                        int32_t *__restrict__ meta, int32_t *__restrict__ num_splits) {
  __shared__ int nb_s[kSchedSmemSeqs];
  __shared__ long long part_sum[kSchedThreads];
  const bool staged = batch <= kSchedSmemSeqs;
  long long local = 0;
  for (int b = threadIdx.x; b < batch; b += kSchedThreads) {
    const int nb = blocks_of_len(topk > 0 ? topk : seq_lens[b]);
    if (staged) nb_s[b] = nb;
    local += nb;
  }
  part_sum[threadIdx.x] = local;
  __syncthreads();
  if (threadIdx.x != 0) return;
  auto nblk = [&](int b) { return staged ? nb_s[b] : blocks_of_len(topk > 0 ? topk : seq_lens[b]); };
  const int fixed = FA_MLA_FIXED_COST;
  long long total = static_cast<long long>(fixed) * batch;
  for (int i = 0; i < kSchedThreads; ++i) total += part_sum[i];
  num_splits[0] = 0;
  const long long payload = (total + num_parts - 1) / num_parts + fixed;
  int b = 0, blk = 0;
  int nb = batch > 0 ? nblk(0) : 0;
  int cnt = 0;     // pieces of sequence b so far
  int prefix = 0;  // pieces of sequences 0 .. b-1
  for (int p = 0; p < num_parts; ++p) {
    const int begin_b = b, begin_blk = blk;
    const int begin_idx = b < batch ? cnt : 0;
    int pieces = 0, end_b = b, end_blk = blk;
    long long remain = payload;
    while (b < batch) {
      const int left = nb - blk;
      if (fixed + left <= remain) {
        remain -= fixed + left;
        prefix += cnt + 1;
        num_splits[b + 1] = prefix;
        ++pieces;
        end_b = b;
        end_blk = nb;
        ++b;
        blk = 0;
        cnt = 0;
        nb = b < batch ? nblk(b) : 0;
      } else {
        const long long take = remain - fixed;
        if (take > 0) {
          ++cnt;
          ++pieces;
          blk += static_cast<int>(take);
          end_b = b;
          end_blk = blk;
        }
        break;
      }
    }
    int32_t *m = meta + static_cast<int64_t>(p) * FA_MLA_META_INTS;
    m[0] = begin_b;
    m[1] = begin_blk;
    m[2] = end_b;
    m[3] = end_blk;
    m[4] = begin_idx;
    m[5] = pieces;
    m[6] = 0;
    m[7] = 0;
  }
}

void launch_mla_metadata(const int32_t *seq_lens, int batch, int topk, int num_parts,
                         int32_t *meta, int32_t *num_splits, cudaStream_t stream) {
  mla_metadata_kernel<<<1, kSchedThreads, 0, stream>>>(seq_lens, batch, topk, num_parts, meta, num_splits);
}

}  // namespace fa
