// exchange.cu -- KV-page-sharded decode across GPUs without a collective
// library call on the data path.
//
// Every rank decodes its range of the sequences' KV pages; its partial result
// (per query row: O normalised by its own row sum, f32, and the LSE) must
// reach every rank, which then merges the ranks' partials by log-sum-exp (the
// algebra of split_kv.py:198-228; the reference itself is single-GPU).
// Instead of a separate all-gather, the kernel that produces a rank's partial
// rows writes each finished row straight into the gather buffer of every
// rank (peer stores over NVLink through CUDA IPC mappings) and then adds the
// number of rows it delivered to a per-source counter on every rank.  The
// merge kernel on each rank waits -- with a time limit -- until every source's
// counter shows its rows, and merges from its local gather buffer.
//
// Gather buffer of a rank (f32): part r of rank r at parts + r * part_stride,
// part_stride = rows * (d_v + 1): O rows [rows][d_v] in (batch, token, head)
// order, then the rows' LSEs [rows].  Counters: uint64 [world], counter r =
// rows of rank r delivered so far.  Counters only grow: after the k-th
// exchange every counter holds k * rows, so nothing is reset between calls.
// No multicast object or multicast load is used: plain peer stores and local
// loads only.
#include <cstring>

#include "common.cuh"
#include "flagattn_b200.h"
#include "merge.cuh"

namespace fa {

struct PeerTargets {
  float *parts[FA_EXCHANGE_MAX_RANKS];
  unsigned long long *counters[FA_EXCHANGE_MAX_RANKS];
};

// A query row of the rank's decode per warp (narrow form, four rows per
// 128-thread block) or per four warps (wide form, two rows per 256-thread
// block: few sequences split over many parts, see mla_row_state).  A
// sequence split over several parts is merged from the split workspace; a
// sequence decoded by one part is read from the decode's f32 output.  The
// row then goes to slot `rank` of every rank's gather buffer.  Launched as a
// programmatic dependent of the decode kernel.
template <bool kWide>
__global__ void __launch_bounds__(kWide ? 256 : 128, kWide ? 2 : 4)
    mla_combine_push_kernel(const float *__restrict__ part_o, const float *__restrict__ part_lse,
                            const int32_t *__restrict__ num_splits, const float *__restrict__ out,
                            int64_t o_sb, int64_t o_ss, int64_t o_sh,
                            const float *__restrict__ lse_in, int batch, int s_q, int h_q, int d_v,
                            PeerTargets peers, int world, int rank) {
  __shared__ MergeState states[kWide ? 8 : 1][32];
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the decode's outputs are complete
  const int b = blockIdx.y;
  const int first = num_splits[b];
  const int n = num_splits[b + 1] - first;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows = s_q * h_q;
  const int64_t rows_all = static_cast<int64_t>(batch) * rows;
  const int64_t part_stride = rows_all * (d_v + 1);
  const int per_block = kWide ? 2 : 4;
  const int flat = blockIdx.x * per_block + (kWide ? (warp >> 2) : warp);
  const int j = kWide ? (warp & 3) : 0;
  float4 v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  float l = -INFINITY;
  if (n >= 2) {
    MergeState st;
    mla_row_state<kWide>(st, part_o, part_lse, first, n, rows, flat, d_v, lane, j, warp, states);
    l = (st.z > 0.f) ? st.m + __logf(st.z) : -INFINITY;
    const float inv = (st.z > 0.f) ? 1.f / st.z : 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k)
      v[k] = make_float4(st.acc[k].x * inv, st.acc[k].y * inv, st.acc[k].z * inv,
                         st.acc[k].w * inv);
  } else if (flat < rows && j == 0) {
    const int s = flat / h_q, h = flat % h_q;
    const float *src = out + b * o_sb + s * o_ss + h * o_sh;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int d = lane * 4 + k * 128;
      v[k] = d < d_v ? __ldg(reinterpret_cast<const float4 *>(src + d))
                     : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    l = __ldg(lse_in + (static_cast<int64_t>(b) * h_q + h) * s_q + s);
  }
  if (flat < rows && j == 0) {
    const int64_t grow = static_cast<int64_t>(b) * rows + flat;
#pragma unroll
    for (int r = 0; r < FA_EXCHANGE_MAX_RANKS; ++r) {  // unrolled: the pointers stay in registers
      if (r >= world) break;
      float *dst = peers.parts[r] + rank * part_stride;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int d = lane * 4 + k * 128;
        if (d < d_v) *reinterpret_cast<float4 *>(dst + grow * d_v + d) = v[k];
      }
      if (lane == 0) dst[rows_all * d_v + grow] = l;
    }
  }
  // every thread's peer stores are visible system-wide before the block's
  // rows are counted on the receivers
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int done = max(0, min(per_block, rows - static_cast<int>(blockIdx.x) * per_block));
    if (done > 0)
#pragma unroll
      for (int r = 0; r < FA_EXCHANGE_MAX_RANKS; ++r)
        if (r < world)
          atomicAdd_system(peers.counters[r] + rank, static_cast<unsigned long long>(done));
  }
}

__device__ __forceinline__ unsigned long long load_acquire_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Wait until every rank's counter holds `target` rows (the calling thread;
// at most timeout_ns of the global timer), then merge.  On a timeout the
// block writes nothing and the status word says so.
template <typename T>
__global__ void __launch_bounds__(128, 4)
    lse_merge_wait_kernel(const float *__restrict__ parts, int world, int64_t rows_all, int d_v,
                          const unsigned long long *__restrict__ counters,
                          unsigned long long target, T *__restrict__ out, float *__restrict__ lse,
                          int *status, long long timeout_ns) {
  __shared__ int arrived;
  if (threadIdx.x == 0) {
    const uint64_t t0 = global_ns();
    // another block already gave up: do not wait again
    int ok = (status == nullptr || *reinterpret_cast<volatile int *>(status) != kDevTimeoutExchange);
    for (int r = 0; r < world && ok; ++r) {
      while (load_acquire_sys(counters + r) < target) {
        if (static_cast<long long>(global_ns() - t0) > timeout_ns) {
          ok = 0;
          if (status) atomicExch(status, kDevTimeoutExchange);
          break;
        }
        __nanosleep(64);
      }
    }
    arrived = ok;
  }
  __syncthreads();
  if (!arrived) return;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 4 + (threadIdx.x >> 5);
  if (row >= rows_all) return;
  const int64_t part_stride = rows_all * (d_v + 1);
  MergeState st;
  st.init();
  fold_parts<true, 4>(st, parts, parts + rows_all * d_v, 0, 0, 1, world, part_stride, part_stride,
                      row * d_v, row, d_v, lane);
  const float l = finish_row<T>(st, d_v, out + row * d_v, lane);
  if (lane == 0) lse[row] = l;
}

int record_error(int status, const char *msg);

namespace {

using MemGetAddressRangeFn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);

MemGetAddressRangeFn address_range_fn() {
  static MemGetAddressRangeFn fn = [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      return static_cast<MemGetAddressRangeFn>(nullptr);
    }
    return reinterpret_cast<MemGetAddressRangeFn>(ptr);
  }();
  return fn;
}

}  // namespace
}  // namespace fa

extern "C" {

int fa_ipc_export(const void *ptr, void *handle, uint64_t *offset) {
  if (!ptr || !handle || !offset) return fa::record_error(FA_ERR_INVALID_ARGUMENT, "ipc export: null");
  auto range = fa::address_range_fn();
  if (!range) return fa::record_error(FA_ERR_CUDA, "ipc export: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fa::record_error(FA_ERR_INVALID_ARGUMENT, "ipc export: not a device allocation");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fa::record_error(FA_ERR_CUDA,
                            "ipc export: cudaIpcGetMemHandle failed (memory from cudaMalloc is "
                            "needed; a virtual-memory-managed pool cannot be exported this way)");
  }
  static_assert(sizeof(h) == FA_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *offset = reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base);
  return FA_OK;
}

int fa_ipc_open(const void *handle, void **base) {
  if (!handle || !base) return fa::record_error(FA_ERR_INVALID_ARGUMENT, "ipc open: null");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fa::record_error(FA_ERR_CUDA, "ipc open: cudaIpcOpenMemHandle failed");
  }
  return FA_OK;
}

int fa_ipc_close(void *base) {
  if (!base) return fa::record_error(FA_ERR_INVALID_ARGUMENT, "ipc close: null");
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fa::record_error(FA_ERR_CUDA, "ipc close: cudaIpcCloseMemHandle failed");
  }
  return FA_OK;
}

int fa_mla_combine_push(const fa_mla_args *a, float *const *dst_parts,
                        unsigned long long *const *dst_counters, int world, int rank,
                        void *stream) {
  if (!a || !dst_parts || !dst_counters)
    return fa::record_error(FA_ERR_INVALID_ARGUMENT, "combine push: null argument");
  if (world < 1 || world > FA_EXCHANGE_MAX_RANKS || rank < 0 || rank >= world)
    return fa::record_error(FA_ERR_INVALID_ARGUMENT, "combine push: world / rank");
  if (a->out_dtype != FA_DTYPE_F32 || !a->out || !a->lse || !a->part_o || !a->part_lse ||
      !a->num_splits || a->d_v != 512 || a->batch < 0 || a->s_q <= 0 || a->h_q <= 0)
    return fa::record_error(FA_ERR_INVALID_ARGUMENT,
                            "combine push: needs the decode's f32 output, LSE and workspace");
  if ((reinterpret_cast<uintptr_t>(a->out) & 15u) || (a->o_stride_b | a->o_stride_s | a->o_stride_h) & 3)
    return fa::record_error(FA_ERR_INVALID_ARGUMENT, "combine push: output not 16-byte aligned");
  fa::PeerTargets t = {};
  for (int r = 0; r < world; ++r) {
    if (!dst_parts[r] || !dst_counters[r] || (reinterpret_cast<uintptr_t>(dst_parts[r]) & 15u))
      return fa::record_error(FA_ERR_INVALID_ARGUMENT,
                              "combine push: every rank's gather buffer (16-byte aligned) and "
                              "counters are needed");
    t.parts[r] = dst_parts[r];
    t.counters[r] = dst_counters[r];
  }
  if (a->batch == 0) return FA_OK;
  const int rows = a->s_q * a->h_q;
  // few sequences over many parts: a row's partials spread over four warps
  const bool wide = static_cast<int64_t>(a->batch) * 4 <= a->num_sm_parts;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = wide ? dim3((rows + 1) / 2, a->batch) : dim3((rows + 3) / 4, a->batch);
  cfg.blockDim = dim3(wide ? 256 : 128);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto kern = wide ? fa::mla_combine_push_kernel<true> : fa::mla_combine_push_kernel<false>;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a->part_o, a->part_lse, a->num_splits,
                                     static_cast<const float *>(a->out), a->o_stride_b,
                                     a->o_stride_s, a->o_stride_h,
                                     static_cast<const float *>(a->lse), a->batch, a->s_q, a->h_q,
                                     a->d_v, t, world, rank);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fa::record_error(FA_ERR_CUDA, "combine push launch failed");
  }
  return FA_OK;
}

int fa_lse_merge_wait(const float *parts, int world, int64_t rows, int d_v,
                      const unsigned long long *counters, unsigned long long target, void *out,
                      int dtype, float *lse, int32_t *status, int64_t timeout_ns, void *stream) {
  if (!parts || !counters || !out || !lse || world < 1 || world > FA_EXCHANGE_MAX_RANKS ||
      rows < 0 || d_v != 512 || timeout_ns <= 0)
    return fa::record_error(FA_ERR_INVALID_ARGUMENT, "merge wait: bad arguments");
  if (reinterpret_cast<uintptr_t>(parts) & 15u)
    return fa::record_error(FA_ERR_INVALID_ARGUMENT, "merge wait: parts must be 16-byte aligned");
  if (dtype != FA_DTYPE_BF16 && dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_F32)
    return fa::record_error(FA_ERR_INVALID_ARGUMENT, "merge wait: dtype");
  if (rows == 0) return FA_OK;
  const dim3 grid(static_cast<unsigned>((rows + 3) / 4));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == FA_DTYPE_BF16)
    fa::lse_merge_wait_kernel<__nv_bfloat16><<<grid, 128, 0, s>>>(
        parts, world, rows, d_v, counters, target, static_cast<__nv_bfloat16 *>(out), lse, status,
        timeout_ns);
  else if (dtype == FA_DTYPE_F16)
    fa::lse_merge_wait_kernel<__half><<<grid, 128, 0, s>>>(
        parts, world, rows, d_v, counters, target, static_cast<__half *>(out), lse, status,
        timeout_ns);
  else
    fa::lse_merge_wait_kernel<float><<<grid, 128, 0, s>>>(
        parts, world, rows, d_v, counters, target, static_cast<float *>(out), lse, status,
        timeout_ns);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? FA_OK : fa::record_error(FA_ERR_CUDA, "merge wait launch failed");
}

}  // extern "C"
